// q8_0_gemv.cu -- Q8_0 matrix-vector product, bit-exact with the reference.
//
// Reference handler q8_0_gemv (src/bytecode_interpreter.s:7010-7063): per
// output row, 16 fp32 lanes; for each 34-byte block {fp16 d; int8 qs[32]}
// lane l does
//     acc[l] = fma(float(qs[l])*d,    x[32b+l],    acc[l])
//     acc[l] = fma(float(qs[16+l])*d, x[32b+16+l], acc[l])
// and the row result is FADDV(acc): a pairwise tree over contiguous halves.
// The product float(q)*d is exact in fp32 (8-bit x 11-bit significands), so the
// only roundings are the FMAs and the tree -- reproduced here in the same order.
//
// The kernel is HBM-bound (1.0625 B per weight).  One thread owns 4 of the 16
// lanes of a row (lanes 4g..4g+3), so 4 threads per row and 8 rows per warp;
// the 4-lane pairs of the FADDV tree reduce in-thread, the last two levels by
// xor-shuffles 1 and 2 (addition is commutative, so each lane's partner order
// matches the tree's lo+hi).
//
// int8 -> fp32 without the (quarter-rate) I2F unit: byte u = q ^ 0x80 placed by
// PRMT into 0x4700_uu00 is the float 32768 + u = 32896 + q exactly; then
// fma(f, d, -32896*d) = q*d exactly (32896 = 2^7 * 257, so 32896*d has <= 20
// significant bits).  Non-finite d takes the direct product instead.
#include <cuda_fp16.h>

#include "ane_internal.cuh"

namespace ane_b200 {

static constexpr int kQThreads = 256;
static constexpr int kRowsPerBlock = kQThreads / 4;

__device__ __forceinline__ float dq_fast(uint32_t xored_word, uint32_t sel, float d, float negcd) {
    const float f = __uint_as_float(__byte_perm(xored_word, 0x47000000u, sel));
    return __fmaf_rn(f, d, negcd);
}

// Four lanes' worth of one half-block: 4 bytes q[j..j+3] (j = 4g or 16+4g).
__device__ __forceinline__ void fma4(float (&acc)[4], uint32_t qword, float d, float negcd, bool finite,
                                     const float4 xv) {
    float dq0, dq1, dq2, dq3;
    if (finite) {
        const uint32_t u = qword ^ 0x80808080u;
        dq0 = dq_fast(u, 0x7404u, d, negcd);  // bytes {0x00, u0, 0x00, 0x47}
        dq1 = dq_fast(u, 0x7414u, d, negcd);
        dq2 = dq_fast(u, 0x7424u, d, negcd);
        dq3 = dq_fast(u, 0x7434u, d, negcd);
    } else {
        dq0 = __fmul_rn((float)(int8_t)(qword & 0xff), d);
        dq1 = __fmul_rn((float)(int8_t)((qword >> 8) & 0xff), d);
        dq2 = __fmul_rn((float)(int8_t)((qword >> 16) & 0xff), d);
        dq3 = __fmul_rn((float)(int8_t)(qword >> 24), d);
    }
    acc[0] = __fmaf_rn(dq0, xv.x, acc[0]);
    acc[1] = __fmaf_rn(dq1, xv.y, acc[1]);
    acc[2] = __fmaf_rn(dq2, xv.z, acc[2]);
    acc[3] = __fmaf_rn(dq3, xv.w, acc[3]);
}

__device__ __forceinline__ uint32_t ld_u16(const uint8_t* p) {
    return (uint32_t)__ldg(reinterpret_cast<const unsigned short*>(p));
}

// 4 bytes at a 2-byte-aligned address.
__device__ __forceinline__ uint32_t ld_4b_a2(const uint8_t* p) {
    return ld_u16(p) | (ld_u16(p + 2) << 16);
}

// x is staged in shared memory (K floats) by every block.
__global__ void __launch_bounds__(kQThreads) q8_0_gemv_kernel(const float* __restrict__ x,
                                                             const uint8_t* __restrict__ W,
                                                             float* __restrict__ out, uint32_t M, uint32_t K) {
    extern __shared__ __align__(16) float xs[];
    for (uint32_t i = threadIdx.x; i < K; i += blockDim.x) xs[i] = x[i];
    __syncthreads();
    const uint32_t nb = K / 32;
    const size_t row_bytes = (size_t)nb * 34;
    const uint32_t g = threadIdx.x & 3;
    for (uint32_t row0 = blockIdx.x * kRowsPerBlock; row0 < M; row0 += gridDim.x * kRowsPerBlock) {
        const uint32_t m = row0 + (threadIdx.x >> 2);
        const bool valid = m < M;
        const uint8_t* rp = W + (size_t)(valid ? m : 0) * row_bytes;
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        if (valid) {
#pragma unroll 2
            for (uint32_t b = 0; b < nb; b++) {
                const uint8_t* blk = rp + (size_t)b * 34;
                const float d = __half2float(__ushort_as_half((unsigned short)ld_u16(blk)));
                const float negcd = __fmul_rn(-32896.0f, d);
                const bool finite = isfinite(d);
                const uint32_t q_lo = ld_4b_a2(blk + 2 + 4 * g);
                const uint32_t q_hi = ld_4b_a2(blk + 18 + 4 * g);
                const float4 x_lo = *reinterpret_cast<const float4*>(xs + 32 * b + 4 * g);
                const float4 x_hi = *reinterpret_cast<const float4*>(xs + 32 * b + 16 + 4 * g);
                fma4(acc, q_lo, d, negcd, finite, x_lo);
                fma4(acc, q_hi, d, negcd, finite, x_hi);
            }
        }
        // FADDV tree: level 1-2 in-thread, levels 3-4 across the 4 threads of the row
        float s = __fadd_rn(__fadd_rn(acc[0], acc[1]), __fadd_rn(acc[2], acc[3]));
        s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, 1));
        s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, 2));
        if (valid && g == 0) out[m] = s;
    }
}

int launch_q8_0_gemv(uint32_t M, uint32_t K, const float* x, const uint8_t* W, float* out, cudaStream_t s) {
    if (M == 0) return ANE_OK;
    ANE_ARG_CHECK(K % 32 == 0, "q8_0_gemv: K must be a multiple of 32");
    ANE_ARG_CHECK(((uintptr_t)W & 1) == 0, "q8_0_gemv: W must be 2-byte aligned");
    const size_t smem = (size_t)K * sizeof(float);
    ANE_ARG_CHECK(smem <= 200 * 1024, "q8_0_gemv: K too large for the shared activation buffer");
    if (smem > 48 * 1024) {
        ANE_CUDA_TRY(cudaFuncSetAttribute(q8_0_gemv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    }
    uint32_t blocks = (M + kRowsPerBlock - 1) / kRowsPerBlock;
    q8_0_gemv_kernel<<<blocks, kQThreads, smem, s>>>(x, W, out, M, K);
    ANE_CHECK_LAUNCH();
    return ANE_OK;
}

}  // namespace ane_b200
