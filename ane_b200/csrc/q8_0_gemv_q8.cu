// q8_0_gemv_q8.cu -- Q8_0 matvec with a Q8_0-quantized activation ("mode Q").
//
// The reference's q8_0_gemv keeps the activation in fp32
// (src/bytecode_interpreter.s:7016-7063, reproduced bit-exactly in
// q8_0_gemv.cu).  The ggml/llama.cpp convention for Q8_0 x Q8_0 instead
// quantizes the activation per 32-block to Q8_0 as well and reduces each block
// with integer dot products.  This file implements that variant:
//   quantize:  per block amax = max|x| (sequential compare, ggml's MAX), d = amax/127
//              stored as fp16(d), q = roundf(x * (d ? 1/d : 0))  (x * id is one RN multiply)
//   dot:       sumi_b = sum_j qw[j]*qx[j] (exact int32 via dp4a),
//              out[m] = sum_b float(sumi_b) * (dw_b * dx_b)
// The int32 block dots are exact; the fp32 sum over blocks runs per lane in
// block order and then across 16 lanes by xor shuffles (an order of its own,
// checked against the sequential CPU restatement within a tolerance).
//
// Memory: the weights stream through the same TMA ring as the fp32-activation
// kernel (one producer warp, 16-block chunks per row); the activation blocks are
// re-laid-out once per CTA into shared memory as an aligned int8 array + fp32
// scales so each dp4a operand is one aligned 32-bit load.
#include <cuda_fp16.h>

#include "ane_internal.cuh"
#include "sm100_ptx.cuh"

namespace ane_b200 {
namespace {

constexpr int kCB = 16;             // blocks per chunk
constexpr int kCBytes = kCB * 34;   // 544
constexpr int kMaxSlotsQ = 8;  // full[8] + empty[8] fill the 128-byte barrier area
static_assert((4 * kCBytes) % 128 == 0, "TMA destinations stay 128-byte aligned");

// One warp per 32 blocks of x: thread j quantizes block (warp*32 + j)... one
// thread per block keeps ggml's sequential amax (NaN behaviour included).
__global__ void quantize_q8_0_kernel(const float* __restrict__ x, uint8_t* __restrict__ out, uint32_t nblocks) {
    const uint32_t b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= nblocks) return;
    const float* xb = x + (size_t)b * 32;
    float v[32];
#pragma unroll
    for (int j = 0; j < 32; j += 4) {
        const float4 t = *reinterpret_cast<const float4*>(xb + j);
        v[j] = t.x;
        v[j + 1] = t.y;
        v[j + 2] = t.z;
        v[j + 3] = t.w;
    }
    float amax = 0.0f;
#pragma unroll
    for (int j = 0; j < 32; j++) {
        const float a = fabsf(v[j]);
        amax = amax > a ? amax : a;
    }
    const float d = __fdiv_rn(amax, 127.0f);
    const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
    // a block starts at an even byte offset: write it as 17 little-endian 16-bit words
    unsigned short* blk = reinterpret_cast<unsigned short*>(out + (size_t)b * 34);
    blk[0] = __half_as_ushort(__float2half_rn(d));
#pragma unroll
    for (int j = 0; j < 32; j += 2) {
        const uint32_t lo = (uint8_t)(int8_t)(int)roundf(__fmul_rn(v[j], id));
        const uint32_t hi = (uint8_t)(int8_t)(int)roundf(__fmul_rn(v[j + 1], id));
        blk[1 + j / 2] = (unsigned short)(lo | (hi << 8));
    }
}

__global__ void q8_0_gemv_q8_kernel(const __grid_constant__ CUtensorMap wmap, const uint8_t* __restrict__ xq,
                                    float* __restrict__ out, int32_t* __restrict__ block_dots, uint32_t M, uint32_t K,
                                    uint32_t nslots, int* err) {
    extern __shared__ __align__(128) uint8_t smem[];
    const uint32_t nw = blockDim.x / 32 - 1;
    const uint32_t rows_per_cta = 4 * nw;
    const uint32_t nb = K / 32, nchunks = (nb + kCB - 1) / kCB;
    const uint32_t slot_bytes = rows_per_cta * kCBytes;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    uint64_t* empty = full + nslots;
    float* xd = reinterpret_cast<float*>(smem + 128);                       // nb scales
    int8_t* xs = reinterpret_cast<int8_t*>(smem + 128 + round_up(nb * 4, 128));  // K codes
    uint8_t* ring = smem + 128 + round_up(nb * 4, 128) + round_up(K, 128);
    const uint32_t r0 = blockIdx.x * rows_per_cta;
    const uint32_t nrows = min(rows_per_cta, M - r0);
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < nslots; s++) {
            ptx::mbar_init(&full[s], 1);
            ptx::mbar_init(&empty[s], nw);
        }
        ptx::fence_mbarrier_init();
    }
    // activation blocks -> aligned codes + scales (all threads)
    for (uint32_t b = threadIdx.x; b < nb; b += blockDim.x) {
        const uint8_t* blk = xq + (size_t)b * 34;
        xd[b] = __half2float(__ushort_as_half((unsigned short)(blk[0] | (blk[1] << 8))));
    }
    for (uint32_t i = threadIdx.x; i < nb * 8; i += blockDim.x) {
        const uint8_t* src = xq + (size_t)(i >> 3) * 34 + 2 + (i & 7) * 4;
        const uint32_t w = (uint32_t)src[0] | ((uint32_t)src[1] << 8) | ((uint32_t)src[2] << 16) |
                           ((uint32_t)src[3] << 24);
        reinterpret_cast<uint32_t*>(xs)[i] = w;
    }
    __syncthreads();

    if (warp == 0) {
        if (lane == 0) {
            ptx::prefetch_tmap(&wmap);
            for (uint32_t c = 0; c < nchunks; c++) {
                const uint32_t slot = c % nslots;
                if (!ptx::mbar_wait(&empty[slot], ((c / nslots) & 1) ^ 1, err)) break;
                ptx::mbar_arrive_expect_tx(&full[slot], slot_bytes);
                ptx::tma_load_2d(ring + (size_t)slot * slot_bytes, &wmap, &full[slot], (int)(c * (kCBytes / 4)),
                                 (int)r0);
            }
        }
        return;
    }
    // compute warp: 4 rows; per chunk, (row, block) pairs p = lane and lane + 32,
    // row = p / 16, block = p % 16 -> each lane feeds two rows
    const uint32_t wrow0 = (warp - 1) * 4;
    const uint32_t ra = wrow0 + (lane >> 4), rb = wrow0 + 2 + (lane >> 4), bl = lane & 15;
    float suma = 0.f, sumb = 0.f;
    bool alive = true;
    for (uint32_t c = 0; c < nchunks && alive; c++) {
        const uint32_t slot = c % nslots;
        if (!ptx::mbar_wait(&full[slot], (c / nslots) & 1, err)) { alive = false; break; }
        const uint32_t b = c * kCB + bl;
        if (b < nb) {
            const int32_t* xw = reinterpret_cast<const int32_t*>(xs + (size_t)b * 32);
            int4 x0 = *reinterpret_cast<const int4*>(xw), x1 = *reinterpret_cast<const int4*>(xw + 4);
            const int32_t xv[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
            const float dx = xd[b];
#pragma unroll
            for (int h = 0; h < 2; h++) {
                const uint32_t r = h ? rb : ra;
                if (r >= nrows) continue;
                const uint8_t* blk = ring + (size_t)slot * slot_bytes + r * kCBytes + bl * 34;
                // qs starts 2 bytes into the block: 9 halfword-pair loads, byte-aligned words by permute
                const unsigned short* hw = reinterpret_cast<const unsigned short*>(blk);
                const float dw = __half2float(__ushort_as_half(hw[0]));
                int32_t sumi = 0;
#pragma unroll
                for (int k = 0; k < 8; k++) {
                    const int32_t w = (int32_t)((uint32_t)hw[1 + 2 * k] | ((uint32_t)hw[2 + 2 * k] << 16));
                    sumi = __dp4a(w, xv[k], sumi);
                }
                if (block_dots) block_dots[(size_t)(r0 + r) * nb + b] = sumi;
                const float t = __fmul_rn(__int2float_rn(sumi), __fmul_rn(dw, dx));
                if (h) sumb = __fadd_rn(sumb, t); else suma = __fadd_rn(suma, t);
            }
        }
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(&empty[slot]);
    }
#pragma unroll
    for (int o = 1; o < 16; o <<= 1) {
        suma = __fadd_rn(suma, __shfl_xor_sync(0xffffffffu, suma, o));
        sumb = __fadd_rn(sumb, __shfl_xor_sync(0xffffffffu, sumb, o));
    }
    if (alive && bl == 0) {
        if (ra < nrows) out[r0 + ra] = suma;
        if (rb < nrows) out[r0 + rb] = sumb;
    }
}

}  // namespace

int launch_quantize_q8_0(uint32_t K, const float* x, uint8_t* out, cudaStream_t s) {
    ANE_ARG_CHECK(K % 32 == 0, "quantize_q8_0: K must be a multiple of 32");
    ANE_ARG_CHECK(((uintptr_t)x & 15) == 0, "quantize_q8_0: x must be 16-byte aligned");
    const uint32_t nb = K / 32;
    if (nb == 0) return ANE_OK;
    quantize_q8_0_kernel<<<(nb + 127) / 128, 128, 0, s>>>(x, out, nb);
    ANE_CHECK_LAUNCH();
    return ANE_OK;
}

int launch_q8_0_gemv_q8(uint32_t M, uint32_t K, const uint8_t* xq, const uint8_t* W, float* out, int32_t* block_dots,
                        cudaStream_t s) {
    if (M == 0) return ANE_OK;
    ANE_ARG_CHECK(K % 256 == 0, "q8_0_gemv_q8: K must be a multiple of 256");
    ANE_ARG_CHECK(((uintptr_t)W & 15) == 0, "q8_0_gemv_q8: W must be 16-byte aligned");
    const uint32_t sms = (uint32_t)num_sms();
    static const int force_warps = env_int("ANE_Q8_WARPS"), force_slots = env_int("ANE_Q8_SLOTS");
    uint32_t nw = force_warps > 0 ? (uint32_t)force_warps : (M + 4 * 6 * sms - 1) / (4 * 6 * sms);
    nw = nw < 1 ? 1 : (nw > 8 ? 8 : nw);
    const uint32_t rows = 4 * nw, nb = K / 32;
    const size_t fixed = 128 + round_up((size_t)nb * 4, 128) + round_up(K, 128);
    const uint32_t blocks = (M + rows - 1) / rows, blocks_per_sm = (blocks + sms - 1) / sms;
    const uint32_t nchunks = (nb + kCB - 1) / kCB;
    const size_t slot = (size_t)rows * kCBytes;
    const size_t share = 227 * 1024 / (blocks_per_sm ? blocks_per_sm : 1) - 1024;  // 1 KB reserved per CTA
    uint32_t nslots = share > fixed ? (uint32_t)((share - fixed) / slot) : 2;
    nslots = nslots < 2 ? 2 : (nslots > (uint32_t)kMaxSlotsQ ? (uint32_t)kMaxSlotsQ : nslots);
    if (nslots > nchunks) nslots = nchunks < 2 ? 2 : nchunks;
    if (force_slots > 0) nslots = force_slots < 2 ? 2 : (force_slots > kMaxSlotsQ ? kMaxSlotsQ : force_slots);
    const size_t smem = fixed + (size_t)nslots * slot;
    ANE_ARG_CHECK(smem <= 200 * 1024, "q8_0_gemv_q8: K too large");
    static const cudaError_t attr_err =
        cudaFuncSetAttribute(q8_0_gemv_q8_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    ANE_CUDA_TRY(attr_err);
    const uint64_t row_bytes = (uint64_t)nb * 34;
    CUtensorMap wmap;
    int rc = encode_tensor_map_2d(&wmap, CU_TENSOR_MAP_DATA_TYPE_UINT32, W, row_bytes / 4, M, row_bytes, kCBytes / 4,
                                  rows, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
    q8_0_gemv_q8_kernel<<<blocks, 32 * (nw + 1), smem, s>>>(wmap, xq, out, block_dots, M, K, nslots,
                                                           device_timeout_flag());
    ANE_CHECK_LAUNCH();
    return ANE_OK;
}

}  // namespace ane_b200
