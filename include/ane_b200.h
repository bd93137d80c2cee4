/*
 * ane_b200.h -- C ABI of the B200 (sm_100a) implementation of ane's quantized
 * dense hot path.  Plain pointers and sizes only.
 *
 * Two families of entry points:
 *   1. Reference-facing, synchronous, any pointer kind (pageable / pinned host,
 *      device, managed).  They keep the reference's calling contract: results
 *      are in caller memory on return, buffers are caller-owned.  Host buffers
 *      are copied to the device and back inside the call.
 *   2. `*_dev` entry points: device pointers, asynchronous on a caller stream
 *      (`stream` is a cudaStream_t passed as void*; NULL = legacy default).
 *
 * Every entry point returns an ane_status (0 = OK) and also records it in a
 * thread-local slot readable with ane_last_error(), because stream_exec keeps
 * the reference's `void` signature.
 */
#ifndef ANE_B200_H
#define ANE_B200_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum ane_status {
    ANE_OK = 0,
    ANE_ERR_INVALID_ARGUMENT = 1,   /* bad size, NULL pointer, misaligned K, ... */
    ANE_ERR_UNSUPPORTED_OPCODE = 2, /* stream_exec met an opcode outside the hot path */
    ANE_ERR_TRUNCATED_STREAM = 3,   /* stream_exec payload runs past the end */
    ANE_ERR_CUDA = 4,               /* a CUDA runtime/driver call failed */
    ANE_ERR_NO_DEVICE = 5,          /* no sm_100 device visible */
    ANE_ERR_OUT_OF_MEMORY = 6,
    ANE_ERR_DEVICE_TIMEOUT = 7      /* a bounded device-side wait gave up */
} ane_status;

/* ------------------------------------------------------------------ status */
int ane_last_error(void);                 /* status of this thread's last call */
const char* ane_last_error_string(void);  /* human-readable detail of it */
void ane_clear_error(void);
const char* ane_version(void);
/* Number of opcodes stream_exec executes, and whether `op` is one of them. */
int ane_opcode_supported(uint8_t op);
/* Payload bytes that follow opcode `op` in a stream (reference encoding), or -1. */
int ane_opcode_payload_size(uint8_t op);

/* ---------------------------------------------------------- drop-in boundary
 * Replaces `ane::interpreter::stream_exec` (reference include/ane/ane.hpp:37-39,
 * src/bytecode_interpreter.s:11-40,174-185).  Decodes the reference byte
 * stream `[u8 op][args packed by sizeof, little-endian]...` and executes the
 * hot-path opcodes on the GPU.  Stops at the first unsupported opcode or
 * truncated payload and records the status (ane_last_error). */
void stream_exec(const uint8_t* data, size_t size);

/* ------------------------------------------ reference-facing synchronous ops
 * Each mirrors one opcode; argument order = the reference's encoding order. */

/* quantize_fp32_i8 (0x19; bytecode_interpreter.s:1876-1950).  `count` elements
 * exactly (the reference rounds up to a multiple of 16 inside stream_exec). */
int ane_quantize_fp32_i8(uint32_t count, const float* src, int8_t* dst, float* scale_out);
/* dequantize_i8_fp32 (0x1A; :1951-1977). */
int ane_dequantize_i8_fp32(uint32_t count, float scale, const int8_t* src, float* dst);
/* pack_b_i8 (0x1B; :2447-2582).  dst holds ceil(N/16)*ceil(K/4)*64 bytes. */
int ane_pack_b_i8(uint32_t K, uint32_t N, const int8_t* src, int8_t* dst);
/* quantize_fp32_i8_channelwise (0x1C; :2583-2662). */
int ane_quantize_fp32_i8_channelwise(uint32_t rows, uint32_t cols, const float* src, int8_t* dst,
                                     float* scales);
/* dense_i8 (0x18; :1978-2446).  Reference memory contract: A is M16 x K64
 * (row stride K64), B_packed from pack_b_i8 with K64 rows, bias N32 floats,
 * C receives M16 rows of N floats (padded rows included). */
int ane_dense_i8(uint32_t M, uint32_t N, uint32_t K, float sa, float sb, uint8_t flags,
                 const int8_t* A, const int8_t* B_packed, const float* bias, float* C);
/* dense_u8s8 (0x1E; :2841-3305): dense_i8 with an unsigned A (u8 x s8 products),
 * same memory contract, scales, bias and ReLU. */
int ane_dense_u8s8(uint32_t M, uint32_t N, uint32_t K, float sa, float sb, uint8_t flags,
                   const uint8_t* A, const int8_t* B_packed, const float* bias, float* C);
/* Integer CBLAS GEMMs (0x61 cblas_igemm s8 x s8, 0x62 cblas_ugemm u8 x u8,
 * 0x63 cblas_usgemm u8 x s8; :8329-9139, docs/API.md:356-370):
 * C = alpha * cvt(op(A) @ op(B)), flags bit 0 = transpose A (A stored K x M),
 * bit 1 = transpose B (B stored N x K); lda / ldb in bytes, ldc in floats;
 * K % 64 == 0.  cvt = int32 -> fp32 (uint32 -> fp32 for ugemm), then one RN
 * multiply by alpha.  beta != 0 reproduces the reference: its int32
 * accumulator starts from the fp32 bit pattern of RN(beta * C) (the ZA tiles
 * are seeded with beta*C, :8411-8489) instead of adding beta*C in fp32. */
int ane_cblas_igemm(uint8_t flags, uint32_t M, uint32_t N, uint32_t K, uint32_t lda, uint32_t ldb, uint32_t ldc,
                    float alpha, float beta, const void* A, const void* B, float* C);
int ane_cblas_ugemm(uint8_t flags, uint32_t M, uint32_t N, uint32_t K, uint32_t lda, uint32_t ldb, uint32_t ldc,
                    float alpha, float beta, const void* A, const void* B, float* C);
int ane_cblas_usgemm(uint8_t flags, uint32_t M, uint32_t N, uint32_t K, uint32_t lda, uint32_t ldb, uint32_t ldc,
                     float alpha, float beta, const void* A, const void* B, float* C);
/* ---- the fp32 opcodes of the reference's MNIST-i8 training step
 * (tests/test_mnist_i8.cpp:304-346), each bit-identical with its handler: */
/* elementwise_scaled_add_fp32 (0x0D; :585-605): out = fma(b, scale, a). */
int ane_elementwise_scaled_add_fp32(uint32_t count, float scale, const float* a, const float* b, float* out);
/* relu_backward_fp32 (0x0F; :639-661): out = act > 0 ? grad : +0. */
int ane_relu_backward_fp32(uint32_t count, const float* act, const float* grad, float* out);
/* transpose_fp32 (0x11; :705-741): dst (N x M) = src (M x N)^T. */
int ane_transpose_fp32(uint32_t M, uint32_t N, const float* src, float* dst);
/* softmax_argmax_fp32 (0x12; :742-1007): per row of cols (a multiple of 16):
 * probs = the handler's polynomial softmax (exp via 2^n times a degree-4
 * polynomial, 16-lane sums, one RN division), g_out[0..15] = probs - one_hot
 * (only the first 16 columns of a g_out row are written), argmax = first
 * index of the maximum of the first 16 probs (15 if none compares equal). */
int ane_softmax_argmax_fp32(uint32_t batch, uint32_t cols, const float* logits, float* probs, const uint8_t* labels,
                            float* g_out, int32_t* argmax);
/* dense_fp32 (0x15; :1008-1826): C = fmax(RN((bias + A @ B) * scale), relu ? 0 :
 * -FLT_MAX), each element one fused multiply-add per k in order from bias;
 * A is M16 x K (rows written up to M16, like dense_i8).  As in the reference,
 * only k < (K & ~15) contribute (it runs K/16 whole blocks; row stride K). */
int ane_dense_fp32(uint32_t M, uint32_t N, uint32_t K, float scale, uint8_t flags, const float* A, const float* B,
                   const float* bias, float* C);
/* count_matches (0x16; :1827-1850): *out = #{i : pred[i] == labels[i]}. */
int ane_count_matches(uint32_t count, const int32_t* pred, const uint8_t* labels, int32_t* out);
/* q4_0_gemv (0x58; :7064-7126): W = M rows of K/32 Q4_0 blocks {fp16 d; 16
 * bytes} (18 B, unpadded); element i < 16 = low nibble of byte i, 16+i = its
 * high nibble, value (nibble - 8) * d; out[M].  Bit-exact with the reference's
 * 16-lane FMA order and FADDV tree (the q8_0_gemv scheme). */
int ane_q4_0_gemv(uint32_t M, uint32_t K, const float* in, const void* W, float* out);
/* get_rows_q8_0 (0x7C; :12355-12408): out[r][32b+j] = float(q) * float(d) of
 * block b of table row indices[r] (u32 indices; dim % 32 == 0).  With a host
 * table the rows up to the largest index are copied to the device. */
int ane_get_rows_q8_0(uint32_t n_rows, uint32_t dim, const void* table, const uint32_t* indices, float* out);
/* get_rows_q4_0 (0x7D; :12419-12466): out[r][32b+i] = (low nibble of byte i - 8)
 * * float(d), out[r][32b+16+i] = (high nibble - 8) * float(d), block b of table
 * row indices[r] (18-byte Q4_0 blocks; dim % 32 == 0). */
int ane_get_rows_q4_0(uint32_t n_rows, uint32_t dim, const void* table, const uint32_t* indices, float* out);
/* K-quant matvecs, out[M] = W x in for rows of floor(K/256) super-blocks:
 *   q4_k_gemv (0x75; :11024-11133) 144 B {fp16 d, fp16 dmin, scales[12], qs[128]}
 *   q2_k_gemv (0x76; :11146-11224)  84 B {scales[16], qs[64], fp16 d, fp16 dmin}
 *   q3_k_gemv (0x77; :11236-11360) 110 B {hmask[32], qs[64], scales[12], fp16 d}
 *   q5_k_gemv (0x78; :11372-11486) 176 B {fp16 d, fp16 dmin, scales[12], qh[32], qs[128]}
 *   q6_k_gemv (0x79; :11498-11606) 210 B {ql[128], qh[64], int8 scales[16], fp16 d}
 * Bit-exact with the handlers: their element layouts and value arithmetic
 * (including q3_k's shift of its second-half codes by the first half's x bits),
 * 16-lane FMA order and FADDV tree.  x 8-byte aligned; W 4-byte aligned (2-byte
 * for q3_k and q6_k). */
int ane_q4_k_gemv(uint32_t M, uint32_t K, const float* in, const void* W, float* out);
int ane_q2_k_gemv(uint32_t M, uint32_t K, const float* in, const void* W, float* out);
int ane_q3_k_gemv(uint32_t M, uint32_t K, const float* in, const void* W, float* out);
int ane_q5_k_gemv(uint32_t M, uint32_t K, const float* in, const void* W, float* out);
int ane_q6_k_gemv(uint32_t M, uint32_t K, const float* in, const void* W, float* out);
/* dense_fused_i8 (0x80, new; README.md:87-97 usage).  fp32 A (M x K, stride K)
 * and B (K x N, stride N) quantized per tensor to int8 (absmax/127), int8 x int8
 * -> exact int32, y = float(acc)*(sa*sb), y = y*scale, optional ReLU; C is
 * M x N fp32 (stride N).  Only the M*N outputs are written. */
int ane_dense_fused_i8(uint32_t M, uint32_t N, uint32_t K, float scale, uint8_t relu,
                       const float* A, const float* B, float* C);
/* q8_0_gemv (0x57; :7010-7063, docs/API.md:592-604).  W = M rows of K/32
 * Q8_0 blocks {fp16 d; int8 qs[32]} (34 B, unpadded); fp32 in[K]; out[M].
 * Bit-exact with the reference's 16-lane FMA order and FADDV tree. */
int ane_q8_0_gemv(uint32_t M, uint32_t K, const float* in, const void* W, float* out);

/* ------------------------------------------------------------ device ops
 * Device pointers; asynchronous on `stream`.  Workspace-taking ops accept a
 * caller buffer of at least the size reported by the matching *_workspace_size
 * (NULL -> the library uses a cached per-device allocation). */
size_t ane_dense_fused_i8_workspace_size(uint32_t M, uint32_t N, uint32_t K);
int ane_dense_fused_i8_dev(uint32_t M, uint32_t N, uint32_t K, float scale, uint8_t relu,
                           const float* A, const float* B, float* C, void* workspace,
                           size_t workspace_bytes, void* stream);
/* Quantize-only stages of dense_fused_i8 (for staged timing and tests):
 * Aq = M x K16 int8 (row stride K16 = ceil(K/16)*16, pad columns zero),
 * Bq = the codes of B in B's own layout, K rows of N16 = ceil(N/16)*16 bytes
 * (pad columns zero; allocate K16 rows: the GEMM reads rows up to K16, which
 * meet Aq's zero pad columns), scales[0]=sa, scales[1]=sb.  `partials` holds
 * ane_absmax_partials_count(M*K, K*N) floats. */
size_t ane_absmax_partials_count(size_t count_a, size_t count_b);
int ane_quantize_pair_dev(uint32_t M, uint32_t N, uint32_t K, const float* A, const float* B,
                          int8_t* Aq, int8_t* Bq, float* scales, float* partials, void* stream);
/* Multi-GPU building blocks (N-sharded dense_fused_i8): absmax of both tensors
 * into device absmax2[2] (reduce across ranks with MAX, then quantize with the
 * global values, so every shard uses the single-GPU scales). */
int ane_absmax_pair_dev(const float* A, size_t count_a, const float* B, size_t count_b, float* absmax2,
                        float* partials, void* stream);
int ane_quantize_pair_absmax_dev(uint32_t M, uint32_t N, uint32_t K, const float* A, const float* B, int8_t* Aq,
                                 int8_t* Bq, const float* absmax2, float* scales, void* stream);
/* int8 tensor-core GEMM with the dense_fused_i8 epilogue, operands resident:
 * Aq M x K16 (K-major), Bt N x K16 (K-major), scales device float[2].
 * out_mode 0: fp32 C = relu?(float(acc)*(s0*s1)*scale);  1: raw int32 acc. */
int ane_gemm_s8_dev(uint32_t M, uint32_t N, uint32_t K16, const int8_t* Aq, const int8_t* Bt,
                    const float* scales, float scale, uint8_t relu, int out_mode, void* C,
                    void* stream);
/* The same GEMM with B as dense_fused_i8's prologue leaves it: Bq = codes of B
 * stored K x N, row stride ldb bytes (a multiple of 16, >= N), K16 rows
 * readable (rows past the true K meet Aq's zero pad columns).  The tensor
 * cores read Bq as an MN-major operand, so B is never transposed.  No
 * counterpart in the reference (its B operand is the packed panel layout). */
int ane_gemm_s8_kn_dev(uint32_t M, uint32_t N, uint32_t K16, const int8_t* Aq, const int8_t* Bq, uint32_t ldb,
                       const float* scales, float scale, uint8_t relu, int out_mode, void* C, void* stream);
int ane_quantize_fp32_i8_dev(uint32_t count, const float* src, int8_t* dst, float* scale_out,
                             void* stream);
int ane_pack_b_i8_dev(uint32_t K, uint32_t N, const int8_t* src, int8_t* dst, void* stream);
int ane_dense_i8_dev(uint32_t M, uint32_t N, uint32_t K, float sa, float sb, uint8_t flags,
                     const int8_t* A, const int8_t* B_packed, const float* bias, float* C,
                     void* stream);
int ane_dense_u8s8_dev(uint32_t M, uint32_t N, uint32_t K, float sa, float sb, uint8_t flags,
                       const uint8_t* A, const int8_t* B_packed, const float* bias, float* C,
                       void* stream);
/* kind: 0 = igemm (s8 x s8), 1 = ugemm (u8 x u8), 2 = usgemm (u8 x s8). */
int ane_cblas_int_gemm_dev(int kind, uint8_t flags, uint32_t M, uint32_t N, uint32_t K, uint32_t lda,
                           uint32_t ldb, uint32_t ldc, float alpha, float beta, const void* A, const void* B,
                           float* C, void* stream);
int ane_q8_0_gemv_dev(uint32_t M, uint32_t K, const float* in, const void* W, float* out,
                      void* stream);
int ane_get_rows_q8_0_dev(uint32_t n_rows, uint32_t dim, const void* table, const uint32_t* indices, float* out,
                          void* stream);
int ane_q4_0_gemv_dev(uint32_t M, uint32_t K, const float* in, const void* W, float* out, void* stream);
int ane_get_rows_q4_0_dev(uint32_t n_rows, uint32_t dim, const void* table, const uint32_t* indices, float* out,
                          void* stream);
int ane_q4_k_gemv_dev(uint32_t M, uint32_t K, const float* in, const void* W, float* out, void* stream);
int ane_q2_k_gemv_dev(uint32_t M, uint32_t K, const float* in, const void* W, float* out, void* stream);
int ane_q3_k_gemv_dev(uint32_t M, uint32_t K, const float* in, const void* W, float* out, void* stream);
int ane_q5_k_gemv_dev(uint32_t M, uint32_t K, const float* in, const void* W, float* out, void* stream);
int ane_q6_k_gemv_dev(uint32_t M, uint32_t K, const float* in, const void* W, float* out, void* stream);
int ane_elementwise_scaled_add_fp32_dev(uint32_t count, float scale, const float* a, const float* b, float* out,
                                        void* stream);
int ane_relu_backward_fp32_dev(uint32_t count, const float* act, const float* grad, float* out, void* stream);
int ane_transpose_fp32_dev(uint32_t M, uint32_t N, const float* src, float* dst, void* stream);
int ane_count_matches_dev(uint32_t count, const int32_t* pred, const uint8_t* labels, int32_t* out, void* stream);
int ane_dense_fp32_dev(uint32_t M, uint32_t N, uint32_t K, float scale, uint8_t flags, const float* A, const float* B,
                       const float* bias, float* C, void* stream);
int ane_softmax_argmax_fp32_dev(uint32_t batch, uint32_t cols, const float* logits, float* probs,
                                const uint8_t* labels, float* g_out, int32_t* argmax, void* stream);
/* flags: ANE_Q8_WEIGHTS_STATIC (W not written by the preceding kernel). */
int ane_q4_0_gemv_ex_dev(uint32_t M, uint32_t K, const float* in, const void* W, float* out, uint32_t flags,
                         void* stream);
/* Q8_0 x Q8_0 matvec (the ggml / llama.cpp activation convention; the
 * reference's q8_0_gemv keeps x in fp32, see ane_q8_0_gemv).  x[K] is first
 * quantized to K/32 Q8_0 blocks (d = fp16(amax/127), q = roundf(x/d)); the
 * matvec computes exact int32 block dot products (dp4a) and
 * out[m] = sum_b float(sumi_b) * (dw_b * dx_b).  block_dots (NULL to skip)
 * receives the M x K/32 int32 block dots.  K % 256 == 0, W 16-byte aligned. */
int ane_quantize_q8_0_dev(uint32_t K, const float* x, void* xq_blocks, void* stream);
int ane_q8_0_gemv_q8_dev(uint32_t M, uint32_t K, const void* xq_blocks, const void* W, float* out,
                         int32_t* block_dots, void* stream);

/* The two matvecs above with a flags word.  The streamed kernels always start
 * early (programmatic dependent launch) and read x / write out only once the
 * previous kernel on the stream has finished.  ANE_Q8_WEIGHTS_STATIC promises
 * that W is not written by the kernel that precedes this call on the stream
 * (weights loaded once, then many matvecs), which lets the kernel start
 * streaming W into shared memory while that kernel is still running.  Without
 * the promise such a read could see W before the preceding kernel's writes.
 * No counterpart in the reference (its calls are synchronous). */
#define ANE_Q8_WEIGHTS_STATIC 1u
/* ggml MUL_MAT at batch 1 with Q8_0 weights and an fp32 activation
 * (src/ggml-backend/ggml-ane.cpp:142-177 hands the fp32 src1 to q8_0_gemv;
 * ggml's own CPU path first quantizes src1 to Q8_0): x[K] is quantized to
 * Q8_0 with the ggml rule inside the matvec, then the Q8_0 x Q8_0 matvec runs.
 * out (and block_dots, NULL to skip) equal ane_quantize_q8_0_dev followed by
 * ane_q8_0_gemv_q8_ex_dev bit for bit, in one launch.  K % 256 == 0, W and x
 * 16-byte aligned, flags as above. */
int ane_mul_mat_q8_0_dev(uint32_t M, uint32_t K, const float* x, const void* W, float* out, int32_t* block_dots,
                         uint32_t flags, void* stream);
int ane_q8_0_gemv_ex_dev(uint32_t M, uint32_t K, const float* in, const void* W, float* out,
                         uint32_t flags, void* stream);
int ane_q8_0_gemv_q8_ex_dev(uint32_t M, uint32_t K, const void* xq_blocks, const void* W, float* out,
                            int32_t* block_dots, uint32_t flags, void* stream);
/* The K-quant matvecs ane_q4_k_gemv_dev .. ane_q6_k_gemv_dev with a flags word
 * (ANE_Q8_WEIGHTS_STATIC, as above); op selects the format by its reference
 * opcode: 0x75 q4_k, 0x76 q2_k, 0x77 q3_k, 0x78 q5_k, 0x79 q6_k.  Results are
 * the same as without the flag.  No counterpart in the reference (its calls
 * are synchronous). */
int ane_kquant_gemv_ex_dev(uint8_t op, uint32_t M, uint32_t K, const float* in, const void* W, float* out,
                           uint32_t flags, void* stream);

/* ggml MUL_MAT with Q8_0 weights W[M rows x K] and NT (1..16) fp32 activation
 * rows x[t * ldx + k] (a decode step over NT tokens): y[t * ldy + m].  The
 * reference runs MUL_MAT Q8_0 as one q8_0_gemv (src/ggml-backend/ggml-ane.cpp:
 * 137-143); here the weights cross HBM once for all NT rows.  Each activation
 * row is quantized to Q8_0 with the ggml rule; per (t, m) the batch-1 terms
 * float(sumi) * (dw * dx) are summed in block order within segments of 32
 * blocks, then the segment sums in order (each sum from +0) -- an order fixed by
 * K alone.  K % 256 == 0; W and x 16-byte aligned, ldx % 4 == 0; `workspace`
 * holds ane_mul_mat_q8_0_batch_workspace_size(M, K) bytes (the quantized
 * activation), 256-byte aligned, any contents; calls sharing a workspace must
 * be ordered on one stream.  flags: ANE_Q8_WEIGHTS_STATIC.
 * No counterpart in the reference. */
size_t ane_mul_mat_q8_0_batch_workspace_size(uint32_t M, uint32_t K);
int ane_mul_mat_q8_0_batch_dev(uint32_t M, uint32_t K, uint32_t NT, const float* x, size_t ldx, const void* W,
                               float* y, size_t ldy, void* workspace, uint32_t flags, void* stream);

/* ------------------------------------------------ decode stack (config 5)
 * A row-sharded chain of Q8_0 MUL_MATs with the all-gather fused into each
 * matvec, one launch per projection (capturable in a CUDA graph).  Rank r of
 * `world` owns rows_local rows of every projection and computes them as
 * ane_mul_mat_q8_0_dev does (bit for bit).  Vectors are TAGGED: element i is
 * one 8-byte word {fp32 value, u32 tag} written by one store, so a reader that
 * sees the expected tag has the value -- no fence, flag or counter (a
 * system-scope fence per projection would cost several microseconds).
 * Projection j of token t (t = *tok, this GPU's count of finished tokens,
 * nproj projections per token) stores tag t*nproj + j + 1 into every rank's
 * vector (out_ranks[q] = rank q's vector at this rank's first row, 16-byte
 * aligned CUDA-IPC peer pointers; out_ranks[rank] local) and waits (bounded,
 * ~2 s) for tag t*nproj + j in `prev`, this GPU's copy of the previous
 * projection's vector: in the words it reads as x (x_from_prev: x = prev[0..K),
 * else x is the fp32 input) and in one guard word per (rank, CTA) of that
 * projection (prev_rows rows per rank, prev_ctas = ane_mul_mat_q8_0_ctas of
 * it), which that CTA stored after reading its own input -- so with two vectors
 * per rank alternating, no rank overwrites a vector another still reads.  For
 * j = 0, `prev` is the previous token's last vector (tag t*nproj; all zero
 * before the first token).  ane_q8_chain_token_end_dev waits until the `len`
 * words of the last vector carry tag t*nproj + nproj (the gathered output is
 * then complete on this GPU) and bumps *tok.  tok points at two uint32 words
 * (the count, then the token-end launch's arrival count); vectors and both
 * words start zeroed; every rank makes the same calls, with the same `len`
 * every token.  No counterpart in the reference (its ggml
 * backend issues one synchronous q8_0_gemv per MUL_MAT). */
uint32_t ane_mul_mat_q8_0_ctas(uint32_t rows_local, uint32_t K);
int ane_mul_mat_q8_0_gather_dev(uint32_t rows_local, uint32_t K, const float* x, const void* W, uint32_t world,
                                void* const* out_ranks, const void* prev, uint32_t x_from_prev, uint32_t prev_rows,
                                uint32_t prev_ctas, const uint32_t* tok, uint32_t nproj, uint32_t j, uint32_t flags,
                                void* stream);
int ane_q8_chain_token_end_dev(const void* last, uint32_t len, uint32_t nproj, uint32_t* tok, void* stream);
/* The same chain in mode R: each link is q8_0_gemv (bit for bit: the
 * reference's fp32-activation arithmetic) on x, or -- x_from_prev -- on the
 * previous projection's tagged vector prev (16-byte aligned), whose values a
 * first launch writes as fp32 into xbuf (K floats, 16-byte aligned) after
 * waiting (bounded) for their tags.  That launch also waits, before anything is
 * stored, for prev[q * prev_rows] (rank q's first row of the previous
 * projection) to carry the previous projection's tag for every rank q.  Rows
 * go to out_ranks[q] + r as tagged words, tags and tok as for
 * ane_mul_mat_q8_0_gather_dev; ane_q8_chain_token_end_dev ends a token.  K is
 * a positive multiple of 256, W 16-byte aligned.  No counterpart in the
 * reference. */
int ane_q8_0_gemv_gather_dev(uint32_t rows_local, uint32_t K, const float* x, float* xbuf, const void* W,
                             uint32_t world, void* const* out_ranks, const void* prev, uint32_t x_from_prev,
                             uint32_t prev_rows, const uint32_t* tok, uint32_t nproj, uint32_t j, uint32_t flags,
                             void* stream);

/* The same chain at batch NT <= 16 (decode of NT tokens per step), each link
 * being ane_mul_mat_q8_0_batch_dev's MUL_MAT (bit for bit): a vector holds NT
 * token rows of ldw tagged words (ldw even, >= every rank's rows and every K).
 * Output (token t, local row r) goes to out_ranks[q] + t*ldw + r on every rank
 * q (out_ranks[q] = rank q's vector at this rank's first row).  x_from_prev:
 * token t's activation is prev[t*ldw + 0..K) (prev = this GPU's vector of the
 * previous projection, 16-byte aligned), else the fp32 rows x (row stride
 * ldx).  Before any output is stored, the word prev[q * prev_rows] (rank q's
 * first row of the previous projection, token 0) must carry the previous
 * projection's tag for every rank q: a rank that has stored it has finished
 * reading the vector this call overwrites.  Tags: projection j of step s
 * (s = *tok) stores s*nproj + j + 1.  ane_q8_batch_step_end_dev waits until
 * the last projection's `rows` words of each of `ntok` token rows (`ld` words
 * apart) carry tag s*nproj + nproj, then bumps *tok (two zeroed uint32 words,
 * as for the batch-1 chain; the same rows and ntok every step).  workspace as for
 * ane_mul_mat_q8_0_batch_dev; flags: ANE_Q8_WEIGHTS_STATIC.  No counterpart
 * in the reference. */
int ane_mul_mat_q8_0_batch_gather_dev(uint32_t rows_local, uint32_t K, uint32_t NT, const float* x, size_t ldx,
                                      const void* W, void* workspace, uint32_t world, void* const* out_ranks,
                                      size_t ldw, const void* prev, uint32_t x_from_prev, uint32_t prev_rows,
                                      const uint32_t* tok, uint32_t nproj, uint32_t j, uint32_t flags, void* stream);
int ane_q8_batch_step_end_dev(const void* last, uint32_t rows, size_t ld, uint32_t ntok, uint32_t nproj,
                              uint32_t* tok, void* stream);

/* The same chain (batch 1, Q8_0 activation, as ane_mul_mat_q8_0_dev)
 * in ONE persistent cooperative launch, row-sharded over `world` GPUs.
 * Outputs are TAGGED vectors: element i is one 8-byte word {fp32 value, u32
 * tag}, written with a single store, so a reader that sees the expected tag
 * has the value (no fence or flag).  Projection j reads x -- a plain fp32
 * vector, or (x_tagged) the tagged output of projection j-1 -- and writes its
 * rows_local results to out[r] on every rank r < world (CUDA-IPC mapped peer
 * pointers; out[rank] is local); out_all is this rank's whole output vector
 * of projection j (word 0).  ctl = this rank's 2 uint32 control words, zero
 * before the first run and never reset; tagged vectors start zeroed.  Every
 * rank runs the same plan shape the same number of times.  No counterpart in
 * the reference (its ggml backend issues one synchronous q8_0_gemv per
 * MUL_MAT). */
typedef struct ane_q8_stack_proj {
    const void* W;        /* this rank's rows_local x K/32 Q8_0 blocks, 16-byte aligned */
    uint32_t rows_local;  /* rows of this rank */
    uint32_t K;           /* multiple of 256 */
    const void* x;        /* fp32[K] or K tagged words, this GPU's memory, 16-byte aligned */
    uint32_t x_tagged;    /* 1: x is projection j-1's tagged output */
    void* out[8];         /* per rank: where this rank's first output word goes on that rank */
    const void* out_all;  /* this rank's tagged output vector of this projection */
} ane_q8_stack_proj;
int ane_q8_stack_plan_create(const ane_q8_stack_proj* projs, uint32_t nproj, uint32_t world, uint32_t rank,
                             uint32_t* ctl, void** plan);
int ane_q8_stack_run(void* plan, void* stream);
void ane_q8_stack_plan_free(void* plan);
/* Quantize stage of the N-sharded dense_fused_i8 in one cooperative launch
 * (A and B read from HBM once, as in ane_dense_fused_i8_dev) with the tensor-
 * wide absmax of A and B taken over all `world` ranks: each rank stores its
 * two absmax words to every rank's exchange area (slot_peer[q] = this rank's
 * two 64-bit words on rank q, CUDA-IPC peer pointers; slots = this GPU's area
 * of 2*world words) and waits (bounded) for every rank's words of this call.
 * ctl = this GPU's 2 control words.  Exchange area and ctl start zeroed and
 * are never reset; every rank makes the same calls.  The exchange also acts as
 * the call's entry handshake (a rank leaves it only after all ranks entered).
 * Needs K % 16 == 0, N % 16 == 0, 16-byte aligned A, B, Aq, Bq, and
 * M*K + K*N >= 2^22 (else ANE_ERR_INVALID_ARGUMENT).  Aq is M x K, Bq K x N.
 * No counterpart in the reference. */
int ane_quantize_pair_xrank_dev(uint32_t M, uint32_t N, uint32_t K, const float* A, const float* B, int8_t* Aq,
                                int8_t* Bq, float* scales, float* partials, uint32_t world, uint32_t rank,
                                void* const* slot_peer, const void* slots, uint32_t* ctl, void* stream);
/* int8 GEMM (as ane_gemm_s8_kn_dev with ldb = N16, out_mode 0) fused with an all-gather of C over
 * `world` GPUs: every C tile is stored into each rank's gathered output from the
 * epilogue (C_ranks[q] = rank q's buffer at this rank's first element, row
 * stride ldc floats; CUDA-IPC peer pointers, C_ranks[rank] local), then every
 * CTA bumps every rank's counter (ctr_ranks[q]); a final one-thread kernel
 * waits (bounded) until this GPU has all ranks' tiles and bumps *epoch.
 * Counters and epoch start at zero and only grow; every rank makes the same
 * calls.  A stream-ordered collective before the call (the absmax all-reduce
 * of the sharded dense_fused_i8) must separate it from the previous call's
 * readers.  No counterpart in the reference. */
int ane_gemm_s8_gather_dev(uint32_t M, uint32_t N, uint32_t K16, const int8_t* Aq, const int8_t* Bq,
                           const float* scales, float scale, uint8_t relu, uint32_t world, uint32_t rank,
                           void* const* C_ranks, uint32_t ldc, uint32_t* const* ctr_ranks, uint32_t* epoch,
                           void* stream);
/* CUDA IPC for the peer pointers above: a 64-byte handle of the allocation that
 * holds dev_ptr plus dev_ptr's offset in it; open maps a peer's allocation
 * (NVLink peer access enabled lazily) and returns its base. */
int ane_ipc_get_handle(const void* dev_ptr, void* handle64, uint64_t* offset);
int ane_ipc_open_handle(const void* handle64, void** base);
int ane_ipc_close_handle(void* base);

/* dense_fused_i8 without any allocation.  No counterpart in the reference: it
 * exists for callers that cannot allocate device memory when they run the op
 * (a framework that already reserved nearly all GPU memory for its own pool, a
 * ggml-style backend inside graph_compute, latency-critical loops where
 * cudaMalloc/cudaFree would synchronise).  Same arguments and results as
 * ane_dense_fused_i8_dev, but the scratch is one fixed 40 MiB device array
 * inside the library (enough for M = N = K = 4096); a problem whose
 * ane_dense_fused_i8_workspace_size exceeds it returns ANE_ERR_INVALID_ARGUMENT.
 * Every GPU that loads this part of the library keeps the 40 MiB until exit.
 * All calls on a device share the array: calls whose kernels overlap on the
 * GPU race, so serialise them.  The first call on each device looks the array
 * up (cudaGetSymbolAddress); make it before any stream capture.  A timed-out
 * device wait inside the call is reported by ane_device_timeouts(). */
int ane_dense_fused_i8_noalloc_dev(uint32_t M, uint32_t N, uint32_t K, float scale, uint8_t relu,
                                   const float* A, const float* B, float* C, void* stream);

/* ------------------------------------------------------------ diagnostics */
/* Device-side bounded-wait failures on the current device since the last call
 * (and reset): every kernel wait is bounded (about 2 s) and, when it gives up,
 * counts here and unwinds instead of hanging.  Covers every entry point,
 * ane_dense_fused_i8_noalloc_dev included; the synchronous entry points also
 * return ANE_ERR_DEVICE_TIMEOUT themselves.  Call it after synchronising the
 * stream of an asynchronous (*_dev) call.  After a timeout, treat the device as
 * failed: copies that the kernel had in flight may still land. */
int ane_device_timeouts(void);
/* Kernel launches this library issued since process start (all threads). */
uint64_t ane_kernel_launch_count(void);

#ifdef __cplusplus
}
#endif
#endif
