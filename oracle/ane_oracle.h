/*
 * ane_oracle.h -- CPU restatement of the reference's quantized dense hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker for the CUDA
 * implementation in ane_b200/ and the timed CPU baseline of bench.py.  Nothing
 * in the product (ane_b200/, include/) links, loads or calls it.
 *
 * Every function restates one opcode handler of the reference interpreter
 * (joshmorgan1000/ane, src/bytecode_interpreter.s, AArch64 SME2 assembly that
 * cannot execute on x86) operation by operation, in the same IEEE fp32 order:
 *   quantize_fp32_i8              bytecode_interpreter.s:1876-1950
 *   dequantize_i8_fp32            bytecode_interpreter.s:1951-1977
 *   dense_i8                      bytecode_interpreter.s:1978-2446
 *   pack_b_i8                     bytecode_interpreter.s:2447-2582
 *   quantize_fp32_i8_channelwise  bytecode_interpreter.s:2583-2662
 *   q8_0_gemv                     bytecode_interpreter.s:7010-7063
 *   get_rows_q8_0                 bytecode_interpreter.s:12355-12408
 * dense_fused_i8 has no handler in the reference (README.md:87-97 only); it is
 * defined here as the composition quantize(A), quantize(B), dense_i8 with the
 * extra fp32 `scale` multiply of dense_fp32 (bytecode_interpreter.s:998-1019).
 *
 * Parity pinning: the reference's own known-answer tests
 * (tests/test_remaining_ops.cpp:131-184 exact int8 GEMM, :230-325 Q8_0 block
 * format and dequant, tests/test_dsl_coverage.cpp:334-368 quantize round trip)
 * are reproduced under tests/golden/ and checked against this library.  The
 * q8_0_gemv lane order and the FADDV tree have no reference test; they follow
 * the assembly text (partially pinned).
 */
#ifndef ANE_ORACLE_H
#define ANE_ORACLE_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- scalar helpers -------------------------------------------------------- */
float ane_ref_fp16_to_fp32(uint16_t h);          /* exact widening (ARM fcvt s,h) */
uint16_t ane_ref_fp32_to_fp16(float f);          /* IEEE round-to-nearest-even */
float ane_ref_relu_max(float y, float floor_v);  /* ARM FMAX: NaN propagates, max(-0,+0)=+0 */

/* ---- quantize_fp32_i8 (0x19) ------------------------------------------------
 * absmax = max |x_i| (NaN propagates).  absmax == 0 -> scale 1, inv 127; else
 * scale = absmax/127, inv = 127/absmax (both RN divisions).
 * q_i = (int8) trunc(rint_even(min(max(x_i*inv, -127), 127))), NaN -> 0.
 * Processes exactly `count` elements.  Returns the scale (also in *scale_out). */
float ane_ref_quantize_fp32_i8(const float* src, int8_t* dst, size_t count, float* scale_out);
/* absmax pass alone (first loop of the handler). */
float ane_ref_absmax(const float* src, size_t count);
/* second pass alone, given the absmax from the first. */
float ane_ref_scale_from_absmax(float absmax, float* inv_out);
int8_t ane_ref_quantize_one(float x, float inv);
/* second pass alone with a given absmax; returns the scale. */
float ane_ref_quantize_with_absmax(const float* src, int8_t* dst, size_t count, float absmax);

/* ---- quantize_fp32_i8_channelwise (0x1C) ------------------------------------ */
void ane_ref_quantize_fp32_i8_channelwise(uint32_t rows, uint32_t cols, const float* src,
                                          int8_t* dst, float* scales);

/* ---- dequantize_i8_fp32 (0x1A): out = float(q) * scale ------------------------ */
void ane_ref_dequantize_i8_fp32(size_t count, float scale, const int8_t* src, float* dst);

/* ---- pack_b_i8 (0x1B) -------------------------------------------------------- */
size_t ane_ref_packed_b_size(uint32_t K, uint32_t N);
void ane_ref_pack_b_i8(uint32_t K, uint32_t N, const int8_t* src, int8_t* dst);

/* ---- exact int8 GEMM helper: acc[m][n] = sum_k A[m*lda+k] * B[k*ldb+n] ------- */
void ane_ref_gemm_s8_s32(uint32_t M, uint32_t N, uint32_t K, const int8_t* A, size_t lda,
                         const int8_t* B, size_t ldb, int32_t* acc);

/* ---- dense_i8 (0x18) ----------------------------------------------------------
 * Reference memory contract: A row stride K64 (zero-padded), B in pack_b_i8
 * panel format packed with K64 rows, bias holds N32 floats, C rows 0..M16-1
 * written (stride N, columns < N).  C must therefore hold M16*N floats. */
void ane_ref_dense_i8(uint32_t M, uint32_t N, uint32_t K, float sa, float sb, uint8_t flags,
                      const int8_t* A, const int8_t* B_packed, const float* bias, float* C);

/* ---- dense_fused_i8 (0x80, defined by this build) ------------------------------
 * sa = quantize(A[M*K]), sb = quantize(B[K*N]); acc exact int32; comb = sa*sb;
 * y = float(acc)*comb; y = y*scale; relu ? fmax(y, 0) : y.  Only the M*N
 * outputs are written.  The optional outputs (NULL to skip) expose the int8
 * codes, the int32 accumulators and the two scales for bit-exact checks. */
void ane_ref_dense_fused_i8(uint32_t M, uint32_t N, uint32_t K, float scale, int relu,
                            const float* A, const float* B, float* C, int8_t* Aq_out,
                            int8_t* Bq_out, int32_t* acc_out, float* sa_out, float* sb_out);
/* Epilogue alone, from given int32 accumulators and scales. */
void ane_ref_dense_fused_epilogue(uint32_t M, uint32_t N, const int32_t* acc, float sa, float sb,
                                  float scale, int relu, float* C);

/* ---- q8_0_gemv (0x57), mode R (fp32 activation, the reference semantics) -------
 * Block = {fp16 d; int8 qs[32]} (34 B).  16 fp32 lanes; per block lane l does
 * acc[l] = fma(q[l]*d, x[32b+l], acc[l]) then fma(q[16+l]*d, x[32b+16+l], acc[l]).
 * out[m] = FADDV(acc) (pairwise halves tree).  K % 32 == 0. */
void ane_ref_q8_0_gemv(uint32_t M, uint32_t K, const float* x, const uint8_t* W, float* out);

/* ---- q4_0_gemv (0x58; :7064-7126): 18-byte blocks, element i = low nibble of
 * byte i, element 16+i = high nibble, value (nibble - 8) * d; q8_0_gemv's lane
 * order and FADDV tree. */
void ane_ref_q4_0_gemv(uint32_t M, uint32_t K, const float* x, const uint8_t* W, float* out);
/* K-quant matvecs (bytecode_interpreter.s:11024-11620), K % 256 == 0 */
void ane_ref_q4_k_gemv(uint32_t M, uint32_t K, const float* x, const uint8_t* W, float* out);
void ane_ref_q2_k_gemv(uint32_t M, uint32_t K, const float* x, const uint8_t* W, float* out);
void ane_ref_q3_k_gemv(uint32_t M, uint32_t K, const float* x, const uint8_t* W, float* out);
void ane_ref_q5_k_gemv(uint32_t M, uint32_t K, const float* x, const uint8_t* W, float* out);
void ane_ref_q6_k_gemv(uint32_t M, uint32_t K, const float* x, const uint8_t* W, float* out);

/* ---- Q8_0 helpers ---------------------------------------------------------------
 * Quantize fp32 rows into Q8_0 blocks with the ggml rule: d = absmax/127,
 * stored as fp16(d); q = round-half-away(x * (1/d)) (0 when d == 0). */
void ane_ref_quantize_q8_0(const float* x, uint8_t* blocks, size_t n_rows, size_t K);

/* ---- q8_0_gemv mode Q (Q8_0 activation, int32 block dots) ------------------------
 * sumi[m][b] = sum_j qw[j]*qx[j] (exact); out[m] = sum_b float(sumi)*(dw*dx) in
 * block order.  block_dots (NULL to skip) receives M*(K/32) int32 values. */
void ane_ref_q8_0_gemv_q8(uint32_t M, uint32_t K, const uint8_t* xq, const uint8_t* W,
                          float* out, int32_t* block_dots);

/* ---- MNIST-i8 training opcodes (tests/test_mnist_i8.cpp:304-346) ---------------------- */
void ane_ref_elementwise_scaled_add_fp32(uint32_t count, float scale, const float* a, const float* b, float* out);
void ane_ref_relu_backward_fp32(uint32_t count, const float* act, const float* grad, float* out);
void ane_ref_transpose_fp32(uint32_t M, uint32_t N, const float* src, float* dst);
void ane_ref_count_matches(uint32_t count, const int32_t* pred, const uint8_t* labels, int32_t* out);
void ane_ref_dense_fp32(uint32_t M, uint32_t N, uint32_t K, float scale, uint8_t flags, const float* A,
                        const float* B, const float* bias, float* C);
void ane_ref_softmax_argmax_fp32(uint32_t batch, uint32_t cols, const float* logits, float* probs,
                                 const uint8_t* labels, float* g_out, int32_t* argmax);

/* ---- dense_u8s8 (0x1E; :2841-3305): dense_i8 with unsigned A ----------------------- */
void ane_ref_dense_u8s8(uint32_t M, uint32_t N, uint32_t K, float sa, float sb, uint8_t flags,
                        const uint8_t* A, const int8_t* B_packed, const float* bias, float* C);

/* ---- integer CBLAS GEMMs (0x61-0x63; :8329-9139) ------------------------------------
 * kind 0 = igemm (s8 x s8), 1 = ugemm (u8 x u8), 2 = usgemm (u8 x s8);
 * C = RN(cvt(acc) * alpha), acc seeded with the bits of RN(beta*C) when beta != 0. */
void ane_ref_int_gemm(int kind, uint8_t flags, uint32_t M, uint32_t N, uint32_t K, uint32_t lda, uint32_t ldb,
                      uint32_t ldc, float alpha, float beta, const uint8_t* A, const uint8_t* B, float* C);

/* ---- Q8_0 MUL_MAT for NT activation rows (config 5 at batch 16) --------------------
 * No reference handler: the reference's ggml backend runs MUL_MAT Q8_0 as one
 * q8_0_gemv (src/ggml-backend/ggml-ane.cpp:137-143).  Per (activation row t,
 * weight row m) the batch-1 mode-Q terms, summed per segment of
 * ANE_Q8_SEG_BLOCKS blocks in block order, then over segments in order; every
 * sum starts from +0.  out[t * ldo + m]. */
#define ANE_Q8_SEG_BLOCKS 32
void ane_ref_mul_mat_q8_0_batch(uint32_t M, uint32_t K, uint32_t NT, const uint8_t* xq, const uint8_t* W,
                                float* out, size_t ldo);

/* ---- get_rows_q8_0 (0x7C) -------------------------------------------------------- */
void ane_ref_get_rows_q8_0(uint32_t n_rows, uint32_t dim, const uint8_t* table,
                           const uint32_t* indices, float* out);
void ane_ref_get_rows_q4_0(uint32_t n_rows, uint32_t dim, const uint8_t* table,
                           const uint32_t* indices, float* out);

/* ---- OpenMP variants (CPU baseline; identical results) ---------------------------- */
void ane_ref_dense_fused_i8_omp(uint32_t M, uint32_t N, uint32_t K, float scale, int relu,
                                const float* A, const float* B, float* C, int n_threads);
void ane_ref_q8_0_gemv_omp(uint32_t M, uint32_t K, const float* x, const uint8_t* W, float* out,
                           int n_threads);
int ane_ref_max_threads(void);

#ifdef __cplusplus
}
#endif
#endif
