// quantize.cu -- per-tensor absmax int8 quantization kernels (HBM-bound).
//
// Semantics follow the reference handler quantize_fp32_i8
// (src/bytecode_interpreter.s:1876-1950), bit for bit:
//   absmax = max|x| (NaN propagates); absmax == 0 -> scale 1, inv 127;
//   else scale = absmax/127, inv = 127/absmax (IEEE RN divisions);
//   q = rint_even(min(max(x*inv, -127), 127)), NaN -> 0.
// The reduction is a two-kernel scheme with no atomics and no zero-init:
// kernel 1 writes one partial max per block, kernel 2 re-reduces the partials
// (a few hundred floats, L2-resident) in every block before quantizing.
#include <float.h>

#include "ane_internal.cuh"
#include "sm100_ptx.cuh"

namespace ane_b200 {

static constexpr int kThreads = 256;

// ------------------------------------------------------------------ helpers
__device__ __forceinline__ uint32_t absbits(float v) { return __float_as_uint(v) & 0x7fffffffu; }

// Max of |x| as an unsigned compare of the magnitude bits: NaN > inf > finite,
// so a NaN anywhere wins, exactly like the reference's propagating fmax.
__device__ __forceinline__ uint32_t block_max_u32(uint32_t v) {
    __shared__ uint32_t red[kThreads / 32];
    for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
    int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) red[w] = v;
    __syncthreads();
    v = l < (int)(blockDim.x >> 5) ? red[l] : 0u;
    for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;  // valid in every warp
}

__device__ __forceinline__ void scale_from_absmax(float absmax, float* scale, float* inv) {
    if (absmax == 0.0f) {
        *scale = 1.0f;
        *inv = 127.0f;
    } else {  // NaN is unordered and takes this path, as fcmp/b.eq does
        *scale = __fdiv_rn(absmax, 127.0f);
        *inv = __fdiv_rn(127.0f, absmax);
    }
}

__device__ __forceinline__ int8_t quantize_one(float x, float inv) {
    float y = __fmul_rn(x, inv);
    if (y != y) return 0;  // fmax/fmin keep NaN, fcvtzs(NaN) = 0
    y = fminf(fmaxf(y, -127.0f), 127.0f);
    return (int8_t)__float2int_rn(y);  // frintn (ties to even) + fcvtzs
}

__device__ __forceinline__ uint32_t pack4(float a, float b, float c, float d, float inv) {
    uint32_t r = (uint32_t)(uint8_t)quantize_one(a, inv);
    r |= (uint32_t)(uint8_t)quantize_one(b, inv) << 8;
    r |= (uint32_t)(uint8_t)quantize_one(c, inv) << 16;
    r |= (uint32_t)(uint8_t)quantize_one(d, inv) << 24;
    return r;
}

// ------------------------------------------------------- L2 residency
// The staged prologue of dense_fused_i8 reads each fp32 tensor twice (absmax,
// then quantize).  One tensor (64 MB at 4096^2) fits in the 126 MB L2, both do
// not, so the first read marks lines evict_last and the second (last) read
// marks them evict_first.
__device__ __forceinline__ uint64_t l2_policy_evict_last() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ float4 ld_policy(const float4* ptr, uint64_t pol) {
    float4 v;
    asm volatile("ld.global.nc.L2::cache_hint.v4.f32 {%0, %1, %2, %3}, [%4], %5;"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "l"(ptr), "l"(pol));
    return v;
}

// ------------------------------------------------------- absmax partials
// max |x[i]| bits over the grid-stride share (bid of nblk) of x[0..n).  KEEP:
// loads marked evict_last (the tensor is read again by the next kernel).
template <bool KEEP>
__device__ __forceinline__ uint32_t absmax_range(const float* __restrict__ x, size_t n, int bid, int nblk) {
    uint32_t m = 0;
    const size_t tid = (size_t)bid * kThreads + threadIdx.x;
    const size_t stride = (size_t)nblk * kThreads;
    if ((reinterpret_cast<uintptr_t>(x) & 15) == 0) {
        const size_t n4 = n / 4;
        const float4* x4 = reinterpret_cast<const float4*>(x);
        const uint64_t pol = KEEP ? l2_policy_evict_last() : 0;
        auto load = [&](size_t i) { return KEEP ? ld_policy(x4 + i, pol) : __ldg(x4 + i); };
        size_t i = tid;
        // Two independent loads in flight per iteration.  Plain (L2-allocating)
        // loads otherwise: the quantize pass re-reads these tensors back to
        // front, so the tail of this pass is still L2-resident when it starts.
        for (; i + stride < n4; i += 2 * stride) {
            float4 v = load(i);
            float4 u = load(i + stride);
            m = max(m, max(max(absbits(v.x), absbits(v.y)), max(absbits(v.z), absbits(v.w))));
            m = max(m, max(max(absbits(u.x), absbits(u.y)), max(absbits(u.z), absbits(u.w))));
        }
        for (; i < n4; i += stride) {
            float4 v = load(i);
            m = max(m, max(max(absbits(v.x), absbits(v.y)), max(absbits(v.z), absbits(v.w))));
        }
        for (size_t j = n4 * 4 + tid; j < n; j += stride) m = max(m, absbits(x[j]));
    } else {
        for (size_t j = tid; j < n; j += stride) m = max(m, absbits(x[j]));
    }
    return m;
}

// Blocks [0, blocks_a) reduce a[0..na), blocks [blocks_a, +blocks_b) reduce b.
__global__ void __launch_bounds__(kThreads) absmax_partials_kernel(const float* __restrict__ a, size_t na,
                                                                   const float* __restrict__ b, size_t nb,
                                                                   float* __restrict__ partials,
                                                                   int blocks_a) {
    const bool seg_b = (int)blockIdx.x >= blocks_a;
    const int nblk = seg_b ? (int)gridDim.x - blocks_a : blocks_a;
    const int bid = seg_b ? (int)blockIdx.x - blocks_a : (int)blockIdx.x;
    const uint32_t m = block_max_u32(absmax_range<false>(seg_b ? b : a, seg_b ? nb : na, bid, nblk));
    if (threadIdx.x == 0) partials[blockIdx.x] = __uint_as_float(m);
}

__device__ __forceinline__ float reduce_partials(const float* __restrict__ p, int n) {
    uint32_t m = 0;
    for (int i = threadIdx.x; i < n; i += blockDim.x) m = max(m, __float_as_uint(p[i]));
    return __uint_as_float(block_max_u32(m));
}

// ---------------------------------------------------- row-major quantize
// dst[r*ld + k] = q(src[r*K + k]) for k < K, 0 for K <= k < ld.
__device__ void quantize_rows(const float* __restrict__ src, int8_t* __restrict__ dst, uint32_t rows,
                              uint32_t K, uint32_t ld, float inv, int bid, int nblk) {
    const size_t tid = (size_t)bid * blockDim.x + threadIdx.x;
    const size_t stride = (size_t)nblk * blockDim.x;
    const bool vec = (K % 16 == 0) && (ld == K) && ((reinterpret_cast<uintptr_t>(src) & 15) == 0) &&
                     ((reinterpret_cast<uintptr_t>(dst) & 15) == 0);
    if (vec) {
        // 16 elements -> one 16-byte store per chunk; walked from the end so the
        // first chunks read are the ones the absmax pass left in L2; two chunks
        // (eight 16-byte loads) in flight per thread.
        const size_t chunks = (size_t)rows * K / 16;
        const float4* s4 = reinterpret_cast<const float4*>(src);
        uint4* d16 = reinterpret_cast<uint4*>(dst);
        auto quant16 = [&](size_t c, const float4& v0, const float4& v1, const float4& v2, const float4& v3) {
            uint4 o;
            o.x = pack4(v0.x, v0.y, v0.z, v0.w, inv);
            o.y = pack4(v1.x, v1.y, v1.z, v1.w, inv);
            o.z = pack4(v2.x, v2.y, v2.z, v2.w, inv);
            o.w = pack4(v3.x, v3.y, v3.z, v3.w, inv);
            d16[c] = o;
        };
        // last read of src: lines leave L2 first (evict_first)
        const uint64_t pol = l2_policy_evict_first();
        size_t j = tid;
        for (; j + stride < chunks; j += 2 * stride) {
            const size_t c0 = chunks - 1 - j, c1 = chunks - 1 - (j + stride);
            float4 a0 = ld_policy(s4 + 4 * c0 + 0, pol), a1 = ld_policy(s4 + 4 * c0 + 1, pol);
            float4 a2 = ld_policy(s4 + 4 * c0 + 2, pol), a3 = ld_policy(s4 + 4 * c0 + 3, pol);
            float4 b0 = ld_policy(s4 + 4 * c1 + 0, pol), b1 = ld_policy(s4 + 4 * c1 + 1, pol);
            float4 b2 = ld_policy(s4 + 4 * c1 + 2, pol), b3 = ld_policy(s4 + 4 * c1 + 3, pol);
            quant16(c0, a0, a1, a2, a3);
            quant16(c1, b0, b1, b2, b3);
        }
        for (; j < chunks; j += stride) {
            const size_t c0 = chunks - 1 - j;
            float4 a0 = ld_policy(s4 + 4 * c0 + 0, pol), a1 = ld_policy(s4 + 4 * c0 + 1, pol);
            float4 a2 = ld_policy(s4 + 4 * c0 + 2, pol), a3 = ld_policy(s4 + 4 * c0 + 3, pol);
            quant16(c0, a0, a1, a2, a3);
        }
    } else {
        const size_t total = (size_t)rows * ld;
        for (size_t i = tid; i < total; i += stride) {
            size_t r = i / ld, k = i % ld;
            dst[i] = k < K ? quantize_one(src[r * K + k], inv) : (int8_t)0;
        }
    }
}

// Quantize A (row-major -> Aq, row stride lda) and B (row-major -> Bq, row
// stride ldb: B's own layout) in one launch: blocks [0, blocks_a) take A, the
// rest take B.
__global__ void __launch_bounds__(kThreads) quantize_pair_kernel(
    const float* __restrict__ A, const float* __restrict__ B, int8_t* __restrict__ Aq,
    int8_t* __restrict__ Bq, float* __restrict__ scales, const float* __restrict__ partials,
    uint32_t M, uint32_t N, uint32_t K, uint32_t lda, uint32_t ldb, int pblocks_a, int pblocks_b, int blocks_a) {
    const bool seg_b = (int)blockIdx.x >= blocks_a;
    const float absmax = seg_b ? reduce_partials(partials + pblocks_a, pblocks_b)
                               : reduce_partials(partials, pblocks_a);
    float scale, inv;
    scale_from_absmax(absmax, &scale, &inv);
    const int bid = seg_b ? (int)blockIdx.x - blocks_a : (int)blockIdx.x;
    const int nblk = seg_b ? (int)gridDim.x - blocks_a : blocks_a;
    if (bid == 0 && threadIdx.x == 0) scales[seg_b ? 1 : 0] = scale;
    if (!seg_b)
        quantize_rows(A, Aq, M, K, lda, inv, bid, nblk);
    else
        quantize_rows(B, Bq, K, N, ldb, inv, bid, nblk);
}

// ------------------------------------------ staged dense_fused_i8 prologue
// Three launches that keep each fp32 tensor L2-resident between its two reads:
//   absmax_keep_kernel          absmax partials of A (A marked evict_last)
//   quantize_a_absmax_b_kernel  quantize A (its last read)  +  absmax partials of
//                               B (B marked evict_last), in one grid
//   quantize_b_kernel           quantize of B into its own layout (its last read)
// All three are launched with programmatic dependent launch: they signal the
// next launch at entry and wait for the previous one before touching memory.
__global__ void __launch_bounds__(kThreads) absmax_keep_kernel(const float* __restrict__ x, size_t n,
                                                               float* __restrict__ partials) {
    ptx::griddep_launch_dependents();
    ptx::griddep_wait();
    const uint32_t m = block_max_u32(absmax_range<true>(x, n, blockIdx.x, gridDim.x));
    if (threadIdx.x == 0) partials[blockIdx.x] = __uint_as_float(m);
}

__global__ void __launch_bounds__(kThreads) quantize_a_absmax_b_kernel(
    const float* __restrict__ A, int8_t* __restrict__ Aq, uint32_t M, uint32_t K, uint32_t ld,
    const float* __restrict__ B, size_t nb_elems, float* __restrict__ scales, float* __restrict__ partials, int pa,
    int qa) {
    ptx::griddep_launch_dependents();
    ptx::griddep_wait();
    if ((int)blockIdx.x < qa) {
        float scale, inv;
        scale_from_absmax(reduce_partials(partials, pa), &scale, &inv);
        if (blockIdx.x == 0 && threadIdx.x == 0) scales[0] = scale;
        quantize_rows(A, Aq, M, K, ld, inv, blockIdx.x, qa);
    } else {
        const int bid = (int)blockIdx.x - qa, nblk = (int)gridDim.x - qa;
        const uint32_t m = block_max_u32(absmax_range<true>(B, nb_elems, bid, nblk));
        if (threadIdx.x == 0) partials[pa + bid] = __uint_as_float(m);
    }
}

__global__ void __launch_bounds__(kThreads) quantize_b_kernel(const float* __restrict__ B, int8_t* __restrict__ Bq,
                                                              uint32_t K, uint32_t N, uint32_t ldb,
                                                              float* __restrict__ scales,
                                                              const float* __restrict__ partials_b, int pb) {
    ptx::griddep_launch_dependents();
    ptx::griddep_wait();
    float scale, inv;
    scale_from_absmax(reduce_partials(partials_b, pb), &scale, &inv);
    if (blockIdx.x == 0 && threadIdx.x == 0) scales[1] = scale;
    quantize_rows(B, Bq, K, N, ldb, inv, blockIdx.x, gridDim.x);
}

// Flat quantize of one tensor (opcode 0x19).
__global__ void __launch_bounds__(kThreads) quantize_flat_kernel(const float* __restrict__ src,
                                                                 int8_t* __restrict__ dst, size_t count,
                                                                 float* __restrict__ scale_out,
                                                                 const float* __restrict__ partials,
                                                                 int pblocks) {
    const float absmax = reduce_partials(partials, pblocks);
    float scale, inv;
    scale_from_absmax(absmax, &scale, &inv);
    if (blockIdx.x == 0 && threadIdx.x == 0) *scale_out = scale;
    // treat as rows of 16 when possible so the vector path applies
    if (count % 16 == 0)
        quantize_rows(src, dst, (uint32_t)(count / 16), 16, 16, inv, blockIdx.x, gridDim.x);
    else {
        const size_t stride = (size_t)gridDim.x * blockDim.x;
        for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < count; i += stride)
            dst[i] = quantize_one(src[i], inv);
    }
}

// Per-row quantize (opcode 0x1C): one block per row.
__global__ void __launch_bounds__(kThreads) quantize_channelwise_kernel(const float* __restrict__ src,
                                                                        int8_t* __restrict__ dst,
                                                                        float* __restrict__ scales,
                                                                        uint32_t rows, uint32_t cols) {
    for (uint32_t r = blockIdx.x; r < rows; r += gridDim.x) {
        const float* x = src + (size_t)r * cols;
        uint32_t m = 0;
        for (uint32_t i = threadIdx.x; i < cols; i += blockDim.x) m = max(m, absbits(x[i]));
        float scale, inv;
        scale_from_absmax(__uint_as_float(block_max_u32(m)), &scale, &inv);
        if (threadIdx.x == 0) scales[r] = scale;
        for (uint32_t i = threadIdx.x; i < cols; i += blockDim.x) dst[(size_t)r * cols + i] = quantize_one(x[i], inv);
    }
}

// Opcode 0x1A: out = float(q) * scale (scvtf then fmul).
__global__ void dequantize_kernel(const int8_t* __restrict__ src, float* __restrict__ dst, size_t count,
                                  float scale) {
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < count; i += stride)
        dst[i] = __fmul_rn(__int2float_rn(src[i]), scale);
}

// Final reduction of the partials of two tensors into absmax2[0..1] (one block each).
__global__ void __launch_bounds__(kThreads) reduce_partials_kernel(const float* __restrict__ partials,
                                                                   int pblocks_a, int pblocks_b,
                                                                   float* __restrict__ absmax2) {
    const float m = blockIdx.x == 0 ? reduce_partials(partials, pblocks_a)
                                    : reduce_partials(partials + pblocks_a, pblocks_b);
    if (threadIdx.x == 0) absmax2[blockIdx.x] = m;
}

// ------------------------------------------------------------------ launchers
int launch_reduce_partials(const float* partials, int pblocks_a, int pblocks_b, float* absmax2, cudaStream_t s) {
    reduce_partials_kernel<<<2, kThreads, 0, s>>>(partials, pblocks_a, pblocks_b, absmax2);
    ANE_CHECK_LAUNCH();
    return ANE_OK;
}

int absmax_blocks_for(size_t n) {
    size_t want = ceil_div(n, (size_t)kThreads * 32);  // >= 32 elements per thread
    size_t cap = (size_t)num_sms() * 4;
    if (cap > 1024) cap = 1024;  // ane_absmax_partials_count() reserves 2 x 1024 slots
    if (want < 1) want = 1;
    return (int)(want < cap ? want : cap);
}

int launch_absmax_partials(const float* a, size_t na, const float* b, size_t nb, float* partials,
                           int blocks_a, int blocks_b, cudaStream_t s) {
    absmax_partials_kernel<<<blocks_a + blocks_b, kThreads, 0, s>>>(a, na, b, nb, partials, blocks_a);
    ANE_CHECK_LAUNCH();
    return ANE_OK;
}

int launch_quantize_pair(uint32_t M, uint32_t N, uint32_t K, uint32_t K16, const float* A,
                         const float* B, int8_t* Aq, int8_t* Bq, float* scales, const float* partials,
                         int pblocks_a, int pblocks_b, cudaStream_t s) {
    const uint32_t N16 = (uint32_t)round_up(N, 16);
    const size_t work_a = (size_t)M * K16, work_b = (size_t)K * N16;
    const int sms = num_sms();
    // split ~4 waves of blocks between the two tensors in proportion to their size
    int total = sms * 8;  // 8 resident 256-thread blocks per SM
    int ba = (int)((double)total * (double)work_a / (double)(work_a + work_b + 1));
    if (ba < 1) ba = 1;
    int bb = total - ba;
    if (bb < 1) bb = 1;
    quantize_pair_kernel<<<ba + bb, kThreads, 0, s>>>(A, B, Aq, Bq, scales, partials, M, N, K, K16, N16,
                                                      pblocks_a, pblocks_b, ba);
    ANE_CHECK_LAUNCH();
    return ANE_OK;
}

int launch_quantize_staged(uint32_t M, uint32_t N, uint32_t K, uint32_t K16, const float* A, const float* B,
                           int8_t* Aq, int8_t* Bq, float* scales, float* partials, cudaStream_t s) {
    const size_t na = (size_t)M * K, nb = (size_t)K * N;
    const int pa = absmax_blocks_for(na), pb = absmax_blocks_for(nb);
    const int sms = num_sms();
    int rc = launch_pdl(absmax_keep_kernel, dim3(pa), dim3(kThreads), 0, s, A, na, partials);
    if (rc) return rc;
    int qa = sms * 4;  // quantize-A blocks beside the pb absmax-B blocks
    const size_t chunks_a = (size_t)M * K16 / 16;
    if ((size_t)qa * kThreads > chunks_a) qa = (int)ceil_div(chunks_a, (size_t)kThreads);
    if (qa < 1) qa = 1;
    rc = launch_pdl(quantize_a_absmax_b_kernel, dim3(qa + pb), dim3(kThreads), 0, s, A, Aq, M, K, K16, B, nb,
                    scales, partials, pa, qa);
    if (rc) return rc;
    const uint32_t N16 = (uint32_t)round_up(N, 16);
    int qb = sms * 8;
    const size_t chunks_b = (size_t)K * N16 / 16;
    if ((size_t)qb * kThreads > chunks_b) qb = (int)ceil_div(chunks_b, (size_t)kThreads);
    if (qb < 1) qb = 1;
    return launch_pdl(quantize_b_kernel, dim3(qb), dim3(kThreads), 0, s, B, Bq, K, N, N16, scales,
                      (const float*)partials + pa, pb);
}

int launch_quantize_flat(size_t count, const float* src, int8_t* dst, float* scale_out, float* partials,
                         int blocks, cudaStream_t s) {
    int rc = launch_absmax_partials(src, count, nullptr, 0, partials, blocks, 0, s);
    if (rc) return rc;
    int qb = (int)ceil_div(count, (size_t)kThreads * 16);
    if (qb > num_sms() * 4) qb = num_sms() * 4;
    if (qb < 1) qb = 1;
    quantize_flat_kernel<<<qb, kThreads, 0, s>>>(src, dst, count, scale_out, partials, blocks);
    ANE_CHECK_LAUNCH();
    return ANE_OK;
}

int launch_quantize_channelwise(uint32_t rows, uint32_t cols, const float* src, int8_t* dst,
                                float* scales, cudaStream_t s) {
    int g = (int)(rows < 65535u ? rows : 65535u);
    if (g < 1) return ANE_OK;
    quantize_channelwise_kernel<<<g, kThreads, 0, s>>>(src, dst, scales, rows, cols);
    ANE_CHECK_LAUNCH();
    return ANE_OK;
}

int launch_dequantize(size_t count, float scale, const int8_t* src, float* dst, cudaStream_t s) {
    if (count == 0) return ANE_OK;
    int g = (int)ceil_div(count, (size_t)kThreads * 8);
    if (g > num_sms() * 8) g = num_sms() * 8;
    dequantize_kernel<<<g, kThreads, 0, s>>>(src, dst, count, scale);
    ANE_CHECK_LAUNCH();
    return ANE_OK;
}

}  // namespace ane_b200
