// pack.cu -- the reference's pack_b_i8 panel format, to and from the GPU's layout.
//
// Panel format (src/bytecode_interpreter.s:2447-2582, pack_b_i8):
//   G = ceil(K/4), P = ceil(N/16);
//   packed[(p*G + g)*64 + c*4 + d] = B[(4g+d)*N + 16p + c]  (0 outside K x N).
// The tensor-core GEMM wants B K-major (Bt[n][k], row stride K), so dense_i8
// converts the caller's packed B with unpack_b_to_kmajor before the GEMM.
#include "ane_internal.cuh"

namespace ane_b200 {

// One thread per 4-byte (c, g, p) word of the packed output: gathers B[4g..4g+3][n].
__global__ void pack_b_kernel(const int8_t* __restrict__ src, int8_t* __restrict__ dst, uint32_t K,
                              uint32_t N, uint32_t G, uint32_t P) {
    const size_t words = (size_t)P * G * 16;
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    for (size_t w = (size_t)blockIdx.x * blockDim.x + threadIdx.x; w < words; w += stride) {
        const uint32_t c = (uint32_t)(w % 16);
        const size_t pg = w / 16;  // p*G + g
        const uint32_t g = (uint32_t)(pg % G), p = (uint32_t)(pg / G);
        const uint32_t n = 16 * p + c;
        uint32_t v = 0;
        if (n < N) {
#pragma unroll
            for (int d = 0; d < 4; d++) {
                const uint32_t k = 4 * g + d;
                if (k < K) v |= (uint32_t)(uint8_t)src[(size_t)k * N + n] << (8 * d);
            }
        }
        reinterpret_cast<uint32_t*>(dst)[w] = v;
    }
}

// Bt[n][k] (row stride K64) from a packed B that was packed with K64 rows.
// Thread (n, j) assembles Bt[n][16j .. 16j+15] from four 4-byte packed words.
__global__ void unpack_b_kernel(const int8_t* __restrict__ Bp, int8_t* __restrict__ Bt, uint32_t K64,
                                uint32_t N) {
    const uint32_t G = K64 / 4, J = K64 / 16;
    const size_t items = ceil_div(N, 16) * 16 * J;  // whole panels; columns >= N are skipped below
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    const uint32_t* Bw = reinterpret_cast<const uint32_t*>(Bp);
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < items; i += stride) {
        // consecutive threads take consecutive columns of a panel -> coalesced words
        const uint32_t c = (uint32_t)(i % 16);
        const size_t rest = i / 16;
        const uint32_t j = (uint32_t)(rest % J);
        const uint32_t p = (uint32_t)(rest / J);
        const uint32_t n = 16 * p + c;
        if (n >= N) continue;
        uint4 o;
        const size_t base = ((size_t)p * G + 4 * j) * 16 + c;
        o.x = Bw[base + 0 * 16];
        o.y = Bw[base + 1 * 16];
        o.z = Bw[base + 2 * 16];
        o.w = Bw[base + 3 * 16];
        *reinterpret_cast<uint4*>(Bt + (size_t)n * K64 + 16 * j) = o;
    }
}

int launch_pack_b(uint32_t K, uint32_t N, const int8_t* src, int8_t* dst, cudaStream_t s) {
    const uint32_t G = (K + 3) / 4, P = (N + 15) / 16;
    const size_t words = (size_t)P * G * 16;
    if (words == 0) return ANE_OK;
    int g = (int)ceil_div(words, 256 * 4);
    if (g > num_sms() * 8) g = num_sms() * 8;
    pack_b_kernel<<<g, 256, 0, s>>>(src, dst, K, N, G, P);
    ANE_CHECK_LAUNCH();
    return ANE_OK;
}

int launch_unpack_b_to_kmajor(uint32_t K64, uint32_t N, const int8_t* Bp, int8_t* Bt, cudaStream_t s) {
    const size_t items = (size_t)ceil_div(N, 16) * 16 * (K64 / 16);
    if (items == 0) return ANE_OK;
    int g = (int)ceil_div(items, 256 * 2);
    if (g > num_sms() * 8) g = num_sms() * 8;
    unpack_b_kernel<<<g, 256, 0, s>>>(Bp, Bt, K64, N);
    ANE_CHECK_LAUNCH();
    return ANE_OK;
}

// Strided int8 operand -> K-major rows for the tensor-core GEMM (integer CBLAS
// GEMMs, cblas_igemm / ugemm / usgemm, src/bytecode_interpreter.s:8329-9139):
//   dst[r][k] = k < K ? (trans ? src[k * ld + r] : src[r * ld + k]) : 0,
// r < rows, k < K16 (row stride K16).  32 x 32 byte tiles through shared memory
// so both the reads and the writes run along contiguous bytes.
__global__ void kmajor_i8_kernel(const uint8_t* __restrict__ src, size_t ld, int trans, uint32_t rows, uint32_t K,
                                 uint32_t K16, uint8_t* __restrict__ dst) {
    __shared__ uint8_t tile[32][33];
    const uint32_t k0 = blockIdx.x * 32, r0 = blockIdx.y * 32, tx = threadIdx.x, ty = threadIdx.y;
    if (trans) {  // src is K x rows: read along r, write along k
#pragma unroll
        for (uint32_t i = 0; i < 32; i += 8) {
            const uint32_t k = k0 + ty + i, r = r0 + tx;
            tile[ty + i][tx] = (k < K && r < rows) ? src[(size_t)k * ld + r] : (uint8_t)0;
        }
        __syncthreads();
#pragma unroll
        for (uint32_t i = 0; i < 32; i += 8) {
            const uint32_t r = r0 + ty + i, k = k0 + tx;
            if (r < rows && k < K16) dst[(size_t)r * K16 + k] = tile[tx][ty + i];
        }
    } else {  // src is rows x K
#pragma unroll
        for (uint32_t i = 0; i < 32; i += 8) {
            const uint32_t r = r0 + ty + i, k = k0 + tx;
            if (r < rows && k < K16) dst[(size_t)r * K16 + k] = k < K ? src[(size_t)r * ld + k] : (uint8_t)0;
        }
    }
}

int launch_kmajor_i8(const void* src, size_t ld, bool trans, uint32_t rows, uint32_t K, uint32_t K16, void* dst,
                     cudaStream_t s) {
    if (rows == 0 || K16 == 0) return ANE_OK;
    const dim3 grid((K16 + 31) / 32, (rows + 31) / 32), block(32, 8);
    kmajor_i8_kernel<<<grid, block, 0, s>>>(static_cast<const uint8_t*>(src), ld, trans ? 1 : 0, rows, K, K16,
                                            static_cast<uint8_t*>(dst));
    ANE_CHECK_LAUNCH();
    return ANE_OK;
}

}  // namespace ane_b200
