// mnist_ops.cu -- the fp32 opcodes of the reference's MNIST-i8 training step
// (tests/test_mnist_i8.cpp:304-346), so that step runs on the GPU opcode for
// opcode: elementwise_scaled_add_fp32 (0x0D), relu_backward_fp32 (0x0F),
// transpose_fp32 (0x11), softmax_argmax_fp32 (0x12), dense_fp32 (0x15) and
// count_matches (0x16).  Each follows its handler in
// src/bytecode_interpreter.s operation for operation (same roundings, same
// order), so the results are bit-identical with the reference's.
#include <float.h>

#include "ane_internal.cuh"
#include "sm100_ptx.cuh"

namespace ane_b200 {
namespace {

// out = fma(b, scale, a)  (fmla z0, p0/m, z1, z16; :585-605)
__global__ void scaled_add_kernel(uint32_t n, float scale, const float* __restrict__ a, const float* __restrict__ b,
                                  float* __restrict__ out) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        out[i] = __fmaf_rn(b[i], scale, a[i]);
}

// out = act > 0 ? grad : +0  (fcmgt + sel; NaN act -> 0; :639-661)
__global__ void relu_backward_kernel(uint32_t n, const float* __restrict__ act, const float* __restrict__ grad,
                                     float* __restrict__ out) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        out[i] = act[i] > 0.0f ? grad[i] : 0.0f;
}

// dst[N x M] = src[M x N]^T through 32 x 32 shared-memory tiles (:705-741).
__global__ void transpose_f32_kernel(uint32_t M, uint32_t N, const float* __restrict__ src, float* __restrict__ dst) {
    __shared__ float tile[32][33];
    const uint32_t i0 = blockIdx.y * 32, j0 = blockIdx.x * 32, tx = threadIdx.x, ty = threadIdx.y;
#pragma unroll
    for (uint32_t k = 0; k < 32; k += 8) {
        const uint32_t i = i0 + ty + k, j = j0 + tx;
        if (i < M && j < N) tile[ty + k][tx] = src[(size_t)i * N + j];
    }
    __syncthreads();
#pragma unroll
    for (uint32_t k = 0; k < 32; k += 8) {
        const uint32_t j = j0 + ty + k, i = i0 + tx;
        if (i < M && j < N) dst[(size_t)j * M + i] = tile[tx][ty + k];
    }
}

// count of pred[i] == (int32)labels[i]  (cmpeq + cntp; :1827-1850)
__global__ void count_matches_kernel(uint32_t n, const int32_t* __restrict__ pred, const uint8_t* __restrict__ labels,
                                     int32_t* __restrict__ out) {
    __shared__ int32_t part[32];
    int32_t c = 0;
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) c += pred[i] == (int32_t)labels[i];
    for (int o = 16; o > 0; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = c;
    __syncthreads();
    if (threadIdx.x < 32) {
        c = threadIdx.x < blockDim.x / 32 ? part[threadIdx.x] : 0;
        for (int o = 16; o > 0; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
        if (threadIdx.x == 0) *out = c;
    }
}

// ARM FMAX: NaN wins, max(-0, +0) = +0.
__device__ __forceinline__ float fmax_arm(float a, float b) {
    if (a != a) return a;
    if (b != b) return b;
    if (a == b) return signbit(a) ? b : a;
    return a > b ? a : b;
}

// dense_fp32 (:1008-1826): acc = bias[c], then one fused multiply-add per k in
// order (FMOPA), y = RN(acc * scale), fmax(y, relu ? 0 : -FLT_MAX); rows < M16
// (not predicated), columns < N.  The handler runs K/16 whole k-blocks over a
// row stride of K, so only k < (K & ~15) contribute (MNIST calls it with K = 50).
// 16 x 16 output tile per CTA, k in 16-wide shared-memory slices (the FMA order
// per element stays k = 0, 1, 2, ...).
__global__ void dense_fp32_kernel(uint32_t M16, uint32_t N, uint32_t K, float scale, float floor_v,
                                  const float* __restrict__ A, const float* __restrict__ B,
                                  const float* __restrict__ bias, float* __restrict__ C) {
    __shared__ float As[16][17], Bs[16][17];
    const uint32_t tx = threadIdx.x, ty = threadIdx.y;
    const uint32_t r = blockIdx.y * 16 + ty, c = blockIdx.x * 16 + tx;
    float acc = c < N ? bias[c] : 0.0f;
    const uint32_t Kb = K & ~15u;  // whole k-blocks only
    for (uint32_t k0 = 0; k0 < Kb; k0 += 16) {
        As[ty][tx] = r < M16 ? A[(size_t)r * K + k0 + tx] : 0.0f;
        Bs[ty][tx] = c < N ? B[(size_t)(k0 + ty) * N + c] : 0.0f;
        __syncthreads();
#pragma unroll
        for (uint32_t k = 0; k < 16; k++) acc = __fmaf_rn(As[ty][k], Bs[k][tx], acc);
        __syncthreads();
    }
    if (r < M16 && c < N) C[(size_t)r * N + c] = fmax_arm(__fmul_rn(acc, scale), floor_v);
}

// softmax_argmax_fp32 (:742-1007): one warp per row, lanes 0..15 as the 16 SVE
// lanes (lane l owns columns l, l+16, ...).
__device__ __forceinline__ float smx_exp(float x, float m) {
    const float log2e = __uint_as_float(0x3FB8AA3Bu), c4 = __uint_as_float(0x3C1D955Au),
                c3 = __uint_as_float(0x3D635847u), c2 = __uint_as_float(0x3E75FDF0u),
                c1 = __uint_as_float(0x3F317218u);
    const float t = __fmul_rn(__fsub_rn(x, m), log2e);
    const float n = floorf(t);                       // frintm
    const float f = __fsub_rn(t, n);
    float p = __fmul_rn(c4, f);
    p = __fadd_rn(p, c3);
    p = __fmul_rn(p, f);
    p = __fadd_rn(p, c2);
    p = __fmul_rn(p, f);
    p = __fadd_rn(p, c1);
    p = __fmul_rn(p, f);
    p = __fadd_rn(p, 1.0f);
    int e = __float2int_rz(n);                       // fcvtzs (saturating, NaN -> 0)
    e = e < -127 ? -127 : e;                          // smax
    return __fmul_rn(p, __uint_as_float((uint32_t)(e + 127) << 23));
}

__global__ void softmax_argmax_kernel(uint32_t batch, uint32_t cols, const float* __restrict__ logits,
                                      float* __restrict__ probs, const uint8_t* __restrict__ labels,
                                      float* __restrict__ g_out, int32_t* __restrict__ argmax) {
    const uint32_t row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const uint32_t l = threadIdx.x & 31;
    if (row >= batch) return;  // warp-uniform
    const float* x = logits + (size_t)row * cols;
    float* pr = probs + (size_t)row * cols;
    // pass 1: max (fmax per lane, then across the 16 lanes; NaN wins)
    float m = -INFINITY;
    if (l < 16)
        for (uint32_t i = l; i < cols; i += 16) m = fmax_arm(m, x[i]);
    for (int o = 1; o < 16; o <<= 1) m = fmax_arm(m, __shfl_xor_sync(0xffffffffu, m, o));
    // pass 2: exponentials, per-lane sums in column order, FADDV tree
    float s = 0.0f;
    if (l < 16)
        for (uint32_t i = l; i < cols; i += 16) {
            const float e = smx_exp(x[i], m);
            pr[i] = e;
            s = __fadd_rn(s, e);
        }
    for (int o = 1; o < 16; o <<= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, o));
    // pass 3: normalize by RN(1 / S)
    const float inv = __fdiv_rn(1.0f, s);
    float p0 = 0.0f;
    if (l < 16)
        for (uint32_t i = l; i < cols; i += 16) {
            const float p = __fmul_rn(pr[i], inv);
            pr[i] = p;
            if (i == l) p0 = p;
        }
    // pass 4: g_out = probs - one_hot(label) over the first 16 columns
    const uint32_t lab = labels[row];
    if (l < 16) g_out[(size_t)row * cols + l] = (l == lab) ? __fsub_rn(p0, 1.0f) : p0;
    // pass 5: argmax over the first 16 columns: first lane equal to the max, else 15
    float mx = l < 16 ? p0 : -INFINITY;
    for (int o = 1; o < 16; o <<= 1) mx = fmax_arm(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    const uint32_t hit = __ballot_sync(0xffffffffu, l < 16 && p0 == mx) & 0xffffu;
    if (l == 0) argmax[row] = hit ? (int32_t)(__ffs(hit) - 1) : 15;
}

int grid_for(size_t n) {
    size_t g = (n + 255) / 256;
    const size_t cap = (size_t)num_sms() * 8;
    return (int)(g < 1 ? 1 : (g > cap ? cap : g));
}

}  // namespace

int launch_scaled_add_f32(uint32_t n, float scale, const float* a, const float* b, float* out, cudaStream_t s) {
    if (n == 0) return ANE_OK;
    scaled_add_kernel<<<grid_for(n), 256, 0, s>>>(n, scale, a, b, out);
    ANE_CHECK_LAUNCH();
    return ANE_OK;
}

int launch_relu_backward_f32(uint32_t n, const float* act, const float* grad, float* out, cudaStream_t s) {
    if (n == 0) return ANE_OK;
    relu_backward_kernel<<<grid_for(n), 256, 0, s>>>(n, act, grad, out);
    ANE_CHECK_LAUNCH();
    return ANE_OK;
}

int launch_transpose_f32(uint32_t M, uint32_t N, const float* src, float* dst, cudaStream_t s) {
    if (M == 0 || N == 0) return ANE_OK;
    transpose_f32_kernel<<<dim3((N + 31) / 32, (M + 31) / 32), dim3(32, 8), 0, s>>>(M, N, src, dst);
    ANE_CHECK_LAUNCH();
    return ANE_OK;
}

int launch_count_matches(uint32_t n, const int32_t* pred, const uint8_t* labels, int32_t* out, cudaStream_t s) {
    count_matches_kernel<<<1, 1024, 0, s>>>(n, pred, labels, out);
    ANE_CHECK_LAUNCH();
    return ANE_OK;
}

int launch_dense_f32(uint32_t M, uint32_t N, uint32_t K, float scale, uint8_t flags, const float* A, const float* B,
                     const float* bias, float* C, cudaStream_t s) {
    const uint32_t M16 = (M + 15) & ~15u;
    if (M16 == 0 || N == 0) return ANE_OK;
    dense_fp32_kernel<<<dim3((N + 15) / 16, M16 / 16), dim3(16, 16), 0, s>>>(M16, N, K, scale,
                                                                           (flags & 1) ? 0.0f : -FLT_MAX, A, B,
                                                                           bias, C);
    ANE_CHECK_LAUNCH();
    return ANE_OK;
}

int launch_softmax_argmax_f32(uint32_t batch, uint32_t cols, const float* logits, float* probs,
                              const uint8_t* labels, float* g_out, int32_t* argmax, cudaStream_t s) {
    if (batch == 0) return ANE_OK;
    ANE_ARG_CHECK(cols >= 16 && cols % 16 == 0, "softmax_argmax_fp32: cols must be a positive multiple of 16");
    softmax_argmax_kernel<<<(batch + 7) / 8, 256, 0, s>>>(batch, cols, logits, probs, labels, g_out, argmax);
    ANE_CHECK_LAUNCH();
    return ANE_OK;
}

}  // namespace ane_b200
