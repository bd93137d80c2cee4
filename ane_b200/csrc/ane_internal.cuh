// ane_internal.cuh -- shared host/device helpers of libane_b200 (not installed).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <cstdlib>

#include <atomic>
#include <string>

#include "../../include/ane_b200.h"

namespace ane_b200 {

// ------------------------------------------------------------- status plumbing
// Thread-local last status + message (stream_exec returns void, like the reference).
void set_status(int code, const std::string& msg);
int ok();  // records ANE_OK and returns it

// Every kernel launch goes through this counter so tests and bench can prove
// that the CUDA path (not some fallback) ran.
extern std::atomic<uint64_t> g_launches;
inline void count_launch(uint64_t n = 1) { g_launches.fetch_add(n, std::memory_order_relaxed); }

#define ANE_CUDA_TRY(expr)                                                              \
    do {                                                                                \
        cudaError_t _e = (expr);                                                        \
        if (_e != cudaSuccess) {                                                        \
            ::ane_b200::set_status(ANE_ERR_CUDA, std::string(#expr) + ": " + cudaGetErrorString(_e)); \
            return ANE_ERR_CUDA;                                                        \
        }                                                                               \
    } while (0)

#define ANE_CHECK_LAUNCH()                                                              \
    do {                                                                                \
        cudaError_t _e = cudaGetLastError();                                            \
        ::ane_b200::count_launch();                                                     \
        if (_e != cudaSuccess) {                                                        \
            ::ane_b200::set_status(ANE_ERR_CUDA, std::string("kernel launch: ") + cudaGetErrorString(_e)); \
            return ANE_ERR_CUDA;                                                        \
        }                                                                               \
    } while (0)

#define ANE_ARG_CHECK(cond, msg)                                                        \
    do {                                                                                \
        if (!(cond)) {                                                                  \
            ::ane_b200::set_status(ANE_ERR_INVALID_ARGUMENT, msg);                      \
            return ANE_ERR_INVALID_ARGUMENT;                                            \
        }                                                                               \
    } while (0)

// Device properties of the current device (cached per device).
int num_sms();

// Raises `kernel`'s dynamic shared-memory limit to `bytes` on the current
// device.  The attribute belongs to one device context, so a process that
// drives several GPUs must set it on each: `done` is the caller's per-kernel
// bitmask of devices already set (devices >= 64 are set on every call).
int set_max_dynamic_smem_impl(const void* kernel, int bytes, std::atomic<uint64_t>& done);
template <typename F>
inline int set_max_dynamic_smem(F* kernel, int bytes, std::atomic<uint64_t>& done) {
    return set_max_dynamic_smem_impl(reinterpret_cast<const void*>(kernel), bytes, done);
}

// Integer tuning override from the environment (0 / unset = automatic choice).
inline int env_int(const char* name) {
    const char* v = getenv(name);
    return v ? atoi(v) : 0;
}

// Programmatic dependent launch (on unless ANE_PDL=0).
inline bool pdl_enabled() {
    static const bool on = [] {
        const char* v = getenv("ANE_PDL");
        return !(v && v[0] == '0');
    }();
    return on;
}

// Launches `kernel` with programmatic stream serialization: its CTAs may start
// (barrier setup, descriptor prefetch) while the previous kernel on the stream
// is still running.  Every kernel launched this way executes
// griddepcontrol.wait before it touches global memory that an earlier kernel
// may write, and griddepcontrol.launch_dependents to let the next one start.
template <typename... KArgs, typename... Args>
int launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    ANE_CUDA_TRY(cudaLaunchKernelEx(&cfg, kernel, args...));
    ANE_CHECK_LAUNCH();
    return ANE_OK;
}
// Bytes of the device allocation that holds p, counted from p (0 when p is not
// device memory or the driver cannot tell).
size_t device_bytes_from(const void* p);
// Verifies that the current device is sm_100 (the only target of this library).
int require_sm100();

// Device-side bounded-wait failure counter (incremented by kernels that give up).
int read_and_reset_device_timeouts(cudaStream_t s);
int* device_timeout_flag();  // device address of the counter
// Same for the allocation-free dense_fused_i8 path's own counter (noalloc.cu).
int noalloc_read_and_reset_timeouts(cudaStream_t s);

// While a ScopedLaunchOverride is alive on a thread, num_sms() and
// device_timeout_flag() return its values instead of touching the lazily
// initialised per-device state (which allocates on first use).
struct LaunchOverride {
    int sms;
    int* err;
};
class ScopedLaunchOverride {
public:
    explicit ScopedLaunchOverride(const LaunchOverride* o);
    ~ScopedLaunchOverride();

private:
    const LaunchOverride* prev_;
};

// dense_fused_i8 on a stream with a caller-provided workspace (layout below).
// Aq: codes of A, M x K16 (pad columns 0).  Bq: codes of B in B's own layout,
// K16 x N16 (row stride N16; rows past K are never written: they meet the zero
// pad columns of Aq).
struct FusedWs {
    int8_t* Aq;
    int8_t* Bq;
    float* scales;
    float* partials;
};
size_t fused_ws_layout(uint32_t M, uint32_t N, uint32_t K, FusedWs* w, void* base);
int dense_fused_on_stream(uint32_t M, uint32_t N, uint32_t K, float scale, uint8_t relu, const float* A,
                          const float* B, float* C, void* ws, cudaStream_t s);

// 2-D TMA tensor map: `outer` rows of `inner` elements, row stride in bytes
// (multiple of 16), box of box_inner x box_outer elements, zero OOB fill.
int encode_tensor_map_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, uint64_t inner,
                         uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
                         CUtensorMapSwizzle swizzle);

// 3-D TMA tensor map: dims[0] innermost (elements), strides of dims 1 and 2 in
// bytes (multiples of 16), box box[0] x box[1] x box[2] elements, zero OOB fill,
// no swizzle.
int encode_tensor_map_3d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, const uint64_t (&dims)[3],
                         const uint64_t (&stride_bytes)[2], const uint32_t (&box)[3]);

// ------------------------------------------------------- small math helpers
__host__ __device__ inline size_t ceil_div(size_t a, size_t b) { return (a + b - 1) / b; }
__host__ __device__ inline size_t round_up(size_t a, size_t b) { return ceil_div(a, b) * b; }

// ARM FMAX semantics (the reference's relu / -FLT_MAX floor): a NaN operand
// yields NaN, max(-0, +0) = +0.
__device__ __forceinline__ float arm_fmax(float y, float floor_v) {
    if (y != y) return y;
    if (y == floor_v) return (__float_as_uint(y) >> 31) ? floor_v : y;
    return y > floor_v ? y : floor_v;
}

// ------------------------------------------------------------ kernel launchers
// (definitions in the .cu files; all asynchronous on `s`)
int launch_absmax_partials(const float* a, size_t na, const float* b, size_t nb, float* partials,
                           int blocks_a, int blocks_b, cudaStream_t s);
int absmax_blocks_for(size_t n);
int launch_reduce_partials(const float* partials, int pblocks_a, int pblocks_b, float* absmax2, cudaStream_t s);
// dense_fused_i8 prologue as one cooperative kernel reading A and B from HBM
// once (prologue_coop.cu); partials must hold 2 x num_sms() floats.
bool prologue_coop_supported(uint32_t M, uint32_t N, uint32_t K, const float* A, const float* B, const int8_t* Aq,
                             const int8_t* Bq);
// Cross-GPU absmax exchange of the cooperative prologue (N-sharded dense_fused_i8).
struct CoopXRank {
    uint32_t world, rank;
    void* slot_peer[8];  // per rank q: this rank's two 64-bit words in q's exchange area
    const void* slots;   // this GPU's exchange area (2 words per rank)
    uint32_t* ctl;       // this GPU's 2 control words
};
// Writes Aq (M x K) and Bq (K x N), both in their tensor's own layout.
int launch_prologue_coop(uint32_t M, uint32_t N, uint32_t K, const float* A, const float* B, int8_t* Aq, int8_t* Bq,
                         float* scales, cudaStream_t s, const CoopXRank* x = nullptr);
// dense_fused_i8 prologue in three programmatic-dependent launches with each fp32
// tensor kept L2-resident between its absmax read and its quantize read;
// partials must hold 2 x 1024 floats.
// Aq: M x K16 (pad columns 0); Bq: K x N16 (B's layout, pad columns 0).
int launch_quantize_staged(uint32_t M, uint32_t N, uint32_t K, uint32_t K16, const float* A, const float* B,
                           int8_t* Aq, int8_t* Bq, float* scales, float* partials, cudaStream_t s);
int launch_quantize_pair(uint32_t M, uint32_t N, uint32_t K, uint32_t K16, const float* A,
                         const float* B, int8_t* Aq, int8_t* Bq, float* scales, const float* partials,
                         int blocks_a, int blocks_b, cudaStream_t s);
int launch_quantize_flat(size_t count, const float* src, int8_t* dst, float* scale_out,
                         float* partials, int blocks, cudaStream_t s);
int launch_quantize_channelwise(uint32_t rows, uint32_t cols, const float* src, int8_t* dst,
                                float* scales, cudaStream_t s);
int launch_dequantize(size_t count, float scale, const int8_t* src, float* dst, cudaStream_t s);
int launch_pack_b(uint32_t K, uint32_t N, const int8_t* src, int8_t* dst, cudaStream_t s);
int launch_unpack_b_to_kmajor(uint32_t K64, uint32_t N, const int8_t* Bp, int8_t* Bt,
                              cudaStream_t s);
// Strided (optionally transposed) int8 operand -> `rows` x K16 K-major, pad 0.
int launch_kmajor_i8(const void* src, size_t ld, bool trans, uint32_t rows, uint32_t K, uint32_t K16, void* dst,
                     cudaStream_t s);

// GEMM epilogue selector.
enum GemmOut : int {
    kOutFusedF32 = 0,  // y = float(acc)*(sa*sb); y = y*scale; relu ? fmax(y,0) : y
    kOutRawI32 = 1,    // int32 accumulators
    kOutDenseI8 = 2,   // y = float(acc)*(sa*sb); y = y + bias[n]; fmax(y, relu ? 0 : -FLT_MAX)
    kOutIntGemm = 3,   // integer CBLAS GEMM: y = cvt(acc [+ bits(beta*C) if beta != 0]) * alpha
};
struct GemmEpilogue {
    int mode;
    const float* scales;  // device float[2] (sa, sb) or NULL -> sa_imm, sb_imm
    float sa_imm, sb_imm;
    float scale;          // fused mode multiplier
    int relu;
    const float* bias;    // dense_i8 mode, device pointer (>= N floats)
    // operand signedness (tcgen05 kind::i8 takes each as s8 or u8)
    int a_unsigned = 0, b_unsigned = 0;
    // kOutIntGemm: alpha, beta, C read in place (row stride = ldc of the launch);
    // acc_unsigned: the accumulator converts as uint32 (ucvtf), else int32 (scvtf)
    float alpha = 1.0f, beta = 0.0f;
    int acc_unsigned = 0;
};
// C[M x ldc] += epilogue(Aq[M x K] * Bt[N x K]^T); K multiple of 16, both K-major
// with row stride K.
// Fused all-gather of the GEMM output (see Params in gemm_s8_sm100.cu).
struct GatherArgs {
    uint32_t world;
    void* C_rank[8];
    uint32_t* ctr_rank[8];
};
int launch_gemm_s8_tc(uint32_t M, uint32_t N, uint32_t K, const int8_t* Aq, const int8_t* Bt, void* C, size_t ldc,
                      const GemmEpilogue& ep, cudaStream_t s, const GatherArgs* gather = nullptr,
                      uint32_t* grid_out = nullptr);
// The same with B given as codes stored K x N (row stride ldb bytes, a multiple
// of 16; the buffer holds K rows, K a multiple of 16): B is read as an
// MN-major tcgen05 operand.
int launch_gemm_s8_tc_kn(uint32_t M, uint32_t N, uint32_t K, const int8_t* Aq, const int8_t* Bq, size_t ldb,
                         void* C, size_t ldc, const GemmEpilogue& ep, cudaStream_t s,
                         const GatherArgs* gather = nullptr, uint32_t* grid_out = nullptr);
int launch_gather_wait(const uint32_t* ctr, uint32_t* epoch, uint32_t per_call, cudaStream_t s);
int launch_fill_epilogue_zero_k(uint32_t M, uint32_t N, void* C, size_t ldc, const GemmEpilogue& ep,
                                cudaStream_t s);

// flags: ANE_Q8_WEIGHTS_STATIC lets the streamed kernels read W before the
// previous kernel on the stream has finished.
int launch_q8_0_gemv(uint32_t M, uint32_t K, const float* x, const uint8_t* W, float* out, uint32_t flags,
                     cudaStream_t s);
int launch_quantize_q8_0(uint32_t K, const float* x, uint8_t* out, cudaStream_t s);
int launch_q8_0_gemv_q8(uint32_t M, uint32_t K, const uint8_t* xq, const uint8_t* W, float* out, int32_t* block_dots,
                        uint32_t flags, cudaStream_t s);
// Persistent decode-stack kernel (decode_stack.cu).
int stack_plan_create(const ane_q8_stack_proj* projs, uint32_t nproj, uint32_t world, uint32_t rank, uint32_t* ctl,
                      void** plan_out);
int stack_plan_run(void* plan, cudaStream_t s);
void stack_plan_free(void* plan);
// ggml MUL_MAT at batch 1: fp32 x quantized to Q8_0 inside the matvec.
int launch_get_rows_q8_0(uint32_t n_rows, uint32_t dim, const uint8_t* table, const uint32_t* indices, float* out,
                         cudaStream_t s);
// K-quant matvecs (kquant_gemv.cu): fmt 0 = q4_k, 1 = q2_k, 2 = q3_k, 3 = q5_k,
// 4 = q6_k; floor(K / 256) super-blocks per row; flags: ANE_Q8_WEIGHTS_STATIC.
uint32_t kquant_block_bytes(uint32_t fmt);
int launch_kquant_gemv(uint32_t fmt, uint32_t M, uint32_t K, const float* x, const uint8_t* W, float* out,
                       uint32_t flags, cudaStream_t s);
int launch_get_rows_q4_0(uint32_t n_rows, uint32_t dim, const uint8_t* table, const uint32_t* idx, float* out,
                         cudaStream_t s);
int launch_q4_0_gemv(uint32_t M, uint32_t K, const float* x, const uint8_t* W, float* out, uint32_t flags,
                     cudaStream_t s);
// MNIST-i8 training opcodes (mnist_ops.cu)
int launch_scaled_add_f32(uint32_t n, float scale, const float* a, const float* b, float* out, cudaStream_t s);
int launch_relu_backward_f32(uint32_t n, const float* act, const float* grad, float* out, cudaStream_t s);
int launch_transpose_f32(uint32_t M, uint32_t N, const float* src, float* dst, cudaStream_t s);
int launch_count_matches(uint32_t n, const int32_t* pred, const uint8_t* labels, int32_t* out, cudaStream_t s);
int launch_dense_f32(uint32_t M, uint32_t N, uint32_t K, float scale, uint8_t flags, const float* A, const float* B,
                     const float* bias, float* C, cudaStream_t s);
int launch_softmax_argmax_f32(uint32_t batch, uint32_t cols, const float* logits, float* probs,
                              const uint8_t* labels, float* g_out, int32_t* argmax, cudaStream_t s);
int launch_mul_mat_q8_0(uint32_t M, uint32_t K, const float* x, const uint8_t* W, float* out, int32_t* block_dots,
                        uint32_t flags, cudaStream_t s);
// A row-sharded chain of MUL_MATs (the decode stack on `world` GPUs) with the
// all-gather fused into each matvec (q8_0_gemv_q8.cu).  Vectors are TAGGED:
// element i is one 8-byte word {fp32 value, u32 tag}, written by one store, so
// a reader that sees the expected tag has the value -- no fence, flag or
// counter.  Projection j of token t writes tag t*nproj + j + 1 into every
// rank's vector (out[q] = rank q's vector at this rank's first row; CUDA-IPC
// peer pointers) and reads tag t*nproj + j from this GPU's copy of the
// previous projection's vector `prev`: its input x (x_from_prev) and, always,
// one guard word per (rank, CTA) of that projection (the CTA's first row,
// stored after the CTA read its own input), so no rank overwrites a vector
// another rank still reads.
struct Q8ChainGather {
    uint32_t world;
    uint64_t* out[8];
    const uint64_t* prev;      // this GPU's vector of the previous projection (all ranks' rows)
    uint32_t x_from_prev;      // 1: x = prev[0..K); 0: x is the fp32 input
    uint32_t prev_rows, prev_groups, prev_ctas;  // the previous projection's per-rank split
    const uint32_t* tok;       // this GPU's count of finished tokens
    uint32_t nproj, j;         // projections per token, this projection
};
int launch_mul_mat_q8_0_gather(uint32_t M, uint32_t K, const float* x, const uint8_t* W, const Q8ChainGather& g,
                               uint32_t flags, cudaStream_t s);
uint32_t mul_mat_q8_0_ctas(uint32_t M, uint32_t K);
// The same chain link in mode R (q8_0_gemv on the fp32 activation): a kernel
// writes x as fp32 into xbuf from the previous projection's tagged vector (and
// waits for one guard word per rank), then the q8_0_gemv stream kernel stores
// its rows as tagged words into every rank's vector.  Uses world, out, prev,
// x_from_prev, prev_rows, tok, nproj, j of g.
int launch_q8_0_gemv_gather(uint32_t M, uint32_t K, const float* x, float* xbuf, const uint8_t* W,
                            const Q8ChainGather& g, uint32_t flags, cudaStream_t s);
// Ends a step of such a chain: waits (bounded) until every word of the last
// projection's output on this GPU (`ntok` token rows of `rows` words, row
// stride `ld` words) carries that projection's tag, then bumps *tok.
int launch_q8_chain_token_end(const uint64_t* last, uint32_t rows, size_t ld, uint32_t ntok, uint32_t nproj,
                              uint32_t* tok, cudaStream_t s);
// ggml MUL_MAT for NT <= 16 activation rows (q8_0_gemm_q8.cu); the workspace
// (mul_mat_q8_0_batch_workspace_size bytes, 256-byte aligned) receives the
// quantized activation.
size_t mul_mat_q8_0_batch_workspace_size(uint32_t M, uint32_t K);
int launch_mul_mat_q8_0_batch(uint32_t M, uint32_t K, uint32_t NT, const float* x, size_t ldx, const uint8_t* W,
                              float* y, size_t ldy, void* workspace, uint32_t flags, cudaStream_t s);
// The same MUL_MAT as one link of a row-sharded chain (decode at batch NT): the
// activation rows come from the previous projection's TAGGED output (or the
// plain fp32 x), and each output (token t, row r) leaves as one {value, tag}
// word stored into every rank's next vector at out[q] + t * ldw + r.
struct Q8BatchGather {
    uint32_t world;
    uint64_t* out[8];      // per rank: this rank's first row of that rank's vector
    size_t ldw;            // words per token row of every vector
    const uint64_t* prev;  // this GPU's vector of the previous projection
    uint32_t x_from_prev;  // 1: token t's x = prev[t * ldw + 0..K); 0: x is the fp32 input
    uint32_t prev_rows;    // the previous projection's rows per rank (guard words)
    const uint32_t* tok;   // this GPU's count of finished steps
    uint32_t nproj, j;     // projections per step, this projection
};
int launch_mul_mat_q8_0_batch_gather(uint32_t M, uint32_t K, uint32_t NT, const float* x, size_t ldx,
                                     const uint8_t* W, void* workspace, const Q8BatchGather& g, uint32_t flags,
                                     cudaStream_t s);

}  // namespace ane_b200
