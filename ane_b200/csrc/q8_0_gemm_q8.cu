// q8_0_gemm_q8.cu -- ggml MUL_MAT of Q8_0 weights against NT <= 16 fp32
// activation rows (a decode step over a batch of tokens) on the tensor cores.
//
// The reference's ggml backend maps MUL_MAT Q8_0 onto one q8_0_gemv
// (src/ggml-backend/ggml-ane.cpp:137-143); with NT tokens the weights should
// cross HBM once per step, not NT times, so the NT matvecs run as one
// weight-streaming GEMM.  Arithmetic per (token t, weight row m): the batch-1
// Q8_0 x Q8_0 terms float(sumi) * (dw * dx), each sumi an exact int32 block dot,
// summed from +0 in block order within segments of kSegBlocks blocks; the
// segment sums are added from +0 in segment order.  The grouping depends on K
// only, so results do not change with M, the row shard or the GPU count.
//
// Launch 1 (quantize_x_slices_kernel): the activation rows, quantized with the
// ggml Q8_0 rule, into one slice per K segment:
//     codes  [kSegBlocks][NT16][8 words]   words of a block stored as 0,4,1,5,2,6,3,7
//     scales [kSegBlocks][NT16] fp32
// (NT16 = 16 tokens, zero past NT) -- the layout the MMA fragments load with
// one 64-bit shared-memory load per token and block.
// Launch 2 (q8_0_gemm_q8_kernel): work units u = s * ngroups + g (K segment s,
// 16-row group g) are split evenly over one CTA per SM.  A producer warp streams
// each compute warp's unit through a TMA ring (chunks of 8 blocks: 16 rows x
// 272 B) and bulk-copies the CTA's activation slices once.  A compute warp
// runs one mma.sync m16n8k32 (s8 x s8 -> s32) per block and token octet --
// weight rows as M, tokens as N -- and applies the block scales in fp32.  Its
// 16 x 16 segment sums go to a workspace; the warp that completes a row group
// (an atomic count per group) adds the group's segments in order and writes y.
// No warp waits for another CTA.
#include <cuda.h>

#include "ane_internal.cuh"
#include "q8_mmq.cuh"
#include "sm100_ptx.cuh"

namespace ane_b200 {
namespace {

constexpr uint32_t kRows = 16;                            // weight rows per unit (MMA M)
constexpr uint32_t kSegBlocks = 32;                       // blocks per K segment
constexpr uint32_t kChunk = 8;                            // blocks per ring chunk
constexpr uint32_t kChunkBytes = kChunk * 34;             // 272 B of a row
constexpr uint32_t kTileBytes = kRows * kChunkBytes;      // 4352 = 34 x 128
constexpr uint32_t kChunksPerSeg = kSegBlocks / kChunk;   // 4
constexpr uint32_t kTok = 16;                             // activation rows per slice
constexpr uint32_t kSliceCodes = kSegBlocks * kTok * 32;  // 16 KB
constexpr uint32_t kSliceBytes = kSliceCodes + kSegBlocks * kTok * 4;  // + scales = 18 KB
constexpr uint32_t kMaxWarps = 8;
constexpr uint32_t kMaxXSegs = 4;
constexpr uint32_t kMaxSlots = 8;
static_assert(kTileBytes % 128 == 0 && kSliceBytes % 128 == 0, "TMA / bulk destinations stay 128-byte aligned");

__host__ __device__ constexpr size_t round_up256(size_t v) { return (v + 255) / 256 * 256; }

// ------------------------------------------------------- activation slices
// Thread i = (block b, token t): ggml Q8_0 quantization of x[t][32b..32b+31]
// (q8_quantize_words, the arithmetic of every other Q8_0 activation path here).
__global__ void quantize_x_slices_kernel(const float* __restrict__ x, size_t ldx, uint32_t NT, uint32_t nb,
                                         uint8_t* __restrict__ slices) {
    ptx::griddep_launch_dependents();
    ptx::griddep_wait();  // x may come from the previous kernel; the slices may still be read by it
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= nb * kTok) return;
    const uint32_t b = i / kTok, t = i % kTok;
    const uint32_t s = b / kSegBlocks, j = b % kSegBlocks;
    uint8_t* sl = slices + (size_t)s * kSliceBytes;
    uint4* codes = reinterpret_cast<uint4*>(sl + ((size_t)j * kTok + t) * 32);
    float* scale = reinterpret_cast<float*>(sl + kSliceCodes) + j * kTok + t;
    if (t >= NT) {
        codes[0] = make_uint4(0, 0, 0, 0);
        codes[1] = make_uint4(0, 0, 0, 0);
        *scale = 0.0f;
        return;
    }
    float v[32];
    const float4* xb = reinterpret_cast<const float4*>(x + (size_t)t * ldx + (size_t)b * 32);
#pragma unroll
    for (int k = 0; k < 8; k++) {
        const float4 f = xb[k];
        v[4 * k] = f.x;
        v[4 * k + 1] = f.y;
        v[4 * k + 2] = f.z;
        v[4 * k + 3] = f.w;
    }
    uint32_t w[8];
    *scale = q8_quantize_words(v, w);
    // lane q of an MMA fragment reads words (q, q+4) = codes 4q..4q+3 and 16+4q..16+4q+3
    codes[0] = make_uint4(w[0], w[4], w[1], w[5]);
    codes[1] = make_uint4(w[2], w[6], w[3], w[7]);
}

__device__ __forceinline__ void mma_s8_16832(const uint32_t (&a)[4], uint32_t b0, uint32_t b1, int32_t (&d)[4]) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%10, %10, %10, %10};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(0));
}

// term = float(sumi) * (dw * dx), added to acc: three RN operations, never fused
__device__ __forceinline__ float q8_term_add(float acc, int32_t sumi, float dw, float dx) {
    return __fadd_rn(acc, __fmul_rn(__int2float_rn(sumi), __fmul_rn(dw, dx)));
}

// Codes 4q..4q+3 and 16+4q..16+4q+3 of the 34-byte Q8_0 block at `blk` in the
// ring, as two words.  ALIGNED: blk is 2 mod 4, so the codes (blk + 2) are
// word aligned; otherwise blk is word aligned and the codes straddle words.
template <bool ALIGNED>
__device__ __forceinline__ void block_words(const uint8_t* blk, uint32_t q, uint32_t& lo, uint32_t& hi) {
    if (ALIGNED) {  // codes start at blk + 2, a multiple of 4
        const uint32_t* c = reinterpret_cast<const uint32_t*>(blk + 2);
        lo = c[q];
        hi = c[q + 4];
    } else {  // blk is 4-byte aligned; codes straddle word boundaries by 2 bytes
        const uint32_t* c = reinterpret_cast<const uint32_t*>(blk);
        lo = __funnelshift_r(c[q], c[q + 1], 16);
        hi = __funnelshift_r(c[q + 4], c[q + 5], 16);
    }
}

// ------------------------------------------------------------- the product
struct GemmQ8Args {
    float* y;
    size_t ldy;
    float* partials;     // [ngroups][nseg][16 rows][kTok]
    uint32_t* counters;  // [ngroups], zero between calls
    uint32_t M, nb, NT, ngroups, nseg, units, nw, nslots, flags;
};

template <uint32_t G>  // token octets (NT <= 8G)
__global__ void __launch_bounds__(32 * (kMaxWarps + 1), 1)
    q8_0_gemm_q8_kernel(const __grid_constant__ CUtensorMap wmap, const uint8_t* __restrict__ slices,
                        const GemmQ8Args a, int* err) {
    extern __shared__ __align__(128) uint8_t smem[];
    const uint32_t nw = a.nw, nslots = a.nslots;
    const uint32_t slot_bytes = nw * kTileBytes;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);  // nslots
    uint64_t* empty = full + kMaxSlots;                  // nslots
    uint64_t* xbar = empty + kMaxSlots;
    const uint32_t u0 = (uint32_t)((uint64_t)a.units * blockIdx.x / gridDim.x);
    const uint32_t u1 = (uint32_t)((uint64_t)a.units * (blockIdx.x + 1) / gridDim.x);
    const uint32_t s_lo = u0 / a.ngroups, nxs = u1 > u0 ? (u1 - 1) / a.ngroups - s_lo + 1 : 0;
    uint8_t* xsm = smem + 256;                                    // nxs activation slices
    uint8_t* ring = xsm + (size_t)nxs * kSliceBytes;
    const uint32_t npass = (u1 - u0 + nw - 1) / nw, ntiles = npass * kChunksPerSeg;
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < nslots; s++) {
            ptx::mbar_init(&full[s], 1);
            ptx::mbar_init(&empty[s], nw);
        }
        ptx::mbar_init(xbar, 1);
        ptx::fence_mbarrier_init();
    }
    __syncthreads();
    ptx::griddep_launch_dependents();

    if (warp == 0) {
        if (lane == 0 && u1 > u0) {
            ptx::prefetch_tmap(&wmap);
            // stage t = chunk t % 4 of pass t / 4, for every compute warp's unit
            auto issue = [&](uint32_t t, uint32_t slot) {
                const uint32_t pass = t / kChunksPerSeg, c = t % kChunksPerSeg;
                uint32_t bytes = 0;
                for (uint32_t w = 0; w < nw; w++) {
                    const uint32_t u = u0 + pass * nw + w;
                    if (u >= u1) break;
                    if ((u / a.ngroups) * kSegBlocks + c * kChunk < a.nb) bytes += kTileBytes;
                }
                ptx::mbar_arrive_expect_tx(&full[slot], bytes);
                uint8_t* dst = ring + (size_t)slot * slot_bytes;
                for (uint32_t w = 0; w < nw; w++) {
                    const uint32_t u = u0 + pass * nw + w;
                    if (u >= u1) break;
                    const uint32_t s = u / a.ngroups, g = u - s * a.ngroups;
                    const uint32_t blk0 = s * kSegBlocks + c * kChunk;
                    if (blk0 >= a.nb) continue;  // the last segment's missing chunks
                    // x in 32-bit words: blk0 * 34 / 4 = 68 * (blk0 / 8), a multiple of 4 words
                    ptx::tma_load_2d(dst + (size_t)w * kTileBytes, &wmap, &full[slot], (int)(blk0 / kChunk * 68),
                                     (int)(g * kRows));
                }
            };
            // static weights: the first stages are requested before the previous kernel ends
            const uint32_t pre = (a.flags & ANE_Q8_WEIGHTS_STATIC) ? min(nslots, ntiles) : 0;
            for (uint32_t t = 0; t < pre; t++) issue(t, t);
            ptx::griddep_wait();  // the slices come from the quantize kernel
            ptx::mbar_arrive_expect_tx(xbar, nxs * kSliceBytes);
            ptx::bulk_load(xsm, slices + (size_t)s_lo * kSliceBytes, nxs * kSliceBytes, xbar);
            for (uint32_t t = pre; t < ntiles; t++) {
                const uint32_t slot = t % nslots;
                if (!ptx::mbar_wait(&empty[slot], ((t / nslots) & 1) ^ 1, err)) break;
                issue(t, slot);
            }
        }
        return;
    }
    // ------------------------------------------------------------ compute
    ptx::griddep_wait();  // y, partials and counters may belong to the previous kernel
    const uint32_t cw = warp - 1;
    if (u1 <= u0) return;
    bool alive = ptx::mbar_wait(xbar, 0, err);
    const uint32_t g = lane >> 2, q = lane & 3;
    for (uint32_t pass = 0; pass < npass; pass++) {
        const uint32_t u = u0 + pass * nw + cw;
        const bool active = u < u1;
        const uint32_t s = active ? u / a.ngroups : 0, grp = active ? u - s * a.ngroups : 0;
        const uint8_t* xs = xsm + (size_t)(s - s_lo) * kSliceBytes;
        const float* xd = reinterpret_cast<const float*>(xs + kSliceCodes);
        float acc[G][4];
#pragma unroll
        for (uint32_t n = 0; n < G; n++) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.0f;
        for (uint32_t c = 0; c < kChunksPerSeg; c++) {
            const uint32_t t = pass * kChunksPerSeg + c, slot = t % nslots;
            if (!alive || !ptx::mbar_wait(&full[slot], (t / nslots) & 1, err)) {
                alive = false;
                break;
            }
            if (active && s * kSegBlocks + c * kChunk < a.nb) {
                const uint8_t* tile = ring + (size_t)slot * slot_bytes + (size_t)cw * kTileBytes;
                const uint8_t* r0 = tile + g * kChunkBytes;
                const uint8_t* r1 = tile + (g + 8) * kChunkBytes;
#pragma unroll
                for (uint32_t j = 0; j < kChunk; j++) {
                    uint32_t fa[4];
                    if (j & 1) {
                        block_words<true>(r0 + j * 34, q, fa[0], fa[2]);
                        block_words<true>(r1 + j * 34, q, fa[1], fa[3]);
                    } else {
                        block_words<false>(r0 + j * 34, q, fa[0], fa[2]);
                        block_words<false>(r1 + j * 34, q, fa[1], fa[3]);
                    }
                    const float dw0 = __half2float(*reinterpret_cast<const __half*>(r0 + j * 34));
                    const float dw1 = __half2float(*reinterpret_cast<const __half*>(r1 + j * 34));
                    const uint32_t jj = c * kChunk + j;  // block within the segment
#pragma unroll
                    for (uint32_t n = 0; n < G; n++) {
                        const uint2 b = *reinterpret_cast<const uint2*>(xs + ((size_t)jj * kTok + 8 * n + g) * 32 + 8 * q);
                        int32_t d[4];
                        mma_s8_16832(fa, b.x, b.y, d);
                        const float2 dx = *reinterpret_cast<const float2*>(xd + jj * kTok + 8 * n + 2 * q);
                        acc[n][0] = q8_term_add(acc[n][0], d[0], dw0, dx.x);
                        acc[n][1] = q8_term_add(acc[n][1], d[1], dw0, dx.y);
                        acc[n][2] = q8_term_add(acc[n][2], d[2], dw1, dx.x);
                        acc[n][3] = q8_term_add(acc[n][3], d[3], dw1, dx.y);
                    }
                }
            }
            __syncwarp();
            if (lane == 0) ptx::mbar_arrive(&empty[slot]);
        }
        if (!alive) break;
        if (!active) continue;
        // this unit's 16 x kTok segment sums; the warp completing the row group sums its segments
        float* P = a.partials + ((size_t)grp * a.nseg + s) * kRows * kTok;
#pragma unroll
        for (uint32_t n = 0; n < G; n++) {
            *reinterpret_cast<float2*>(P + g * kTok + 8 * n + 2 * q) = make_float2(acc[n][0], acc[n][1]);
            *reinterpret_cast<float2*>(P + (g + 8) * kTok + 8 * n + 2 * q) = make_float2(acc[n][2], acc[n][3]);
        }
        __threadfence();
        __syncwarp();
        uint32_t last = 0;
        if (lane == 0) last = atomicAdd(a.counters + grp, 1u) == a.nseg - 1;
        last = __shfl_sync(0xffffffffu, last, 0);
        if (!last) continue;
        __threadfence();
        const float* PG = a.partials + (size_t)grp * a.nseg * kRows * kTok;
        // lane -> (row r = lane % 16, tokens lane / 16, +2, ...): 16 consecutive rows per store
        for (uint32_t tt = lane >> 4; tt < a.NT; tt += 2) {
            const uint32_t r = lane & 15, row = grp * kRows + r;
            float v = 0.0f;
            for (uint32_t s2 = 0; s2 < a.nseg; s2++) v = __fadd_rn(v, __ldcg(PG + ((size_t)s2 * kRows + r) * kTok + tt));
            if (row < a.M) a.y[(size_t)tt * a.ldy + row] = v;
        }
        if (lane == 0) a.counters[grp] = 0;  // for the next call (ordered by the kernel boundary)
    }
}

}  // namespace

// Workspace: activation slices | segment sums | per-group counters.
struct GemmQ8Layout {
    uint32_t nb, nseg, ngroups;
    size_t slices, partials, counters, total;
};
static GemmQ8Layout gemm_q8_layout(uint32_t M, uint32_t K) {
    GemmQ8Layout L;
    L.nb = K / 32;
    L.nseg = (L.nb + kSegBlocks - 1) / kSegBlocks;
    L.ngroups = (M + kRows - 1) / kRows;
    L.slices = 0;
    L.partials = round_up256((size_t)L.nseg * kSliceBytes);
    L.counters = L.partials + round_up256((size_t)L.ngroups * L.nseg * kRows * kTok * 4);
    L.total = L.counters + round_up256((size_t)L.ngroups * 4);
    return L;
}

size_t mul_mat_q8_0_batch_workspace_size(uint32_t M, uint32_t K) { return gemm_q8_layout(M, K).total; }

int launch_mul_mat_q8_0_batch(uint32_t M, uint32_t K, uint32_t NT, const float* x, size_t ldx, const uint8_t* W,
                              float* y, size_t ldy, void* workspace, uint32_t flags, cudaStream_t s) {
    if (M == 0 || NT == 0) return ANE_OK;
    ANE_ARG_CHECK(NT <= kTok, "mul_mat_q8_0_batch: at most 16 activation rows");
    ANE_ARG_CHECK(K % 256 == 0 && K > 0, "mul_mat_q8_0_batch: K must be a positive multiple of 256");
    ANE_ARG_CHECK(((uintptr_t)W & 15) == 0, "mul_mat_q8_0_batch: W must be 16-byte aligned");
    ANE_ARG_CHECK(((uintptr_t)x & 15) == 0 && (NT == 1 || ldx % 4 == 0) && ldx >= K,
                  "mul_mat_q8_0_batch: x rows must be 16-byte aligned (ldx % 4 == 0, ldx >= K)");
    ANE_ARG_CHECK(ldy >= M || NT == 1, "mul_mat_q8_0_batch: ldy < M");
    ANE_ARG_CHECK(workspace && ((uintptr_t)workspace & 255) == 0, "mul_mat_q8_0_batch: workspace must be 256-byte aligned");
    const GemmQ8Layout L = gemm_q8_layout(M, K);
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    const uint32_t sms = (uint32_t)num_sms();
    GemmQ8Args a;
    a.y = y;
    a.ldy = ldy;
    a.partials = reinterpret_cast<float*>(ws + L.partials);
    a.counters = reinterpret_cast<uint32_t*>(ws + L.counters);
    a.M = M;
    a.nb = L.nb;
    a.NT = NT;
    a.ngroups = L.ngroups;
    a.nseg = L.nseg;
    a.units = L.ngroups * L.nseg;
    a.flags = flags;
    const uint32_t ctas = a.units < sms ? a.units : sms;
    const uint32_t per = (a.units + ctas - 1) / ctas;
    a.nw = per < kMaxWarps ? per : kMaxWarps;
    // activation slices the widest CTA range touches
    uint32_t max_xs = 0;
    for (uint32_t c = 0; c < ctas; c++) {
        const uint32_t u0 = (uint32_t)((uint64_t)a.units * c / ctas), u1 = (uint32_t)((uint64_t)a.units * (c + 1) / ctas);
        const uint32_t n = (u1 - 1) / a.ngroups - u0 / a.ngroups + 1;
        max_xs = n > max_xs ? n : max_xs;
    }
    ANE_ARG_CHECK(max_xs <= kMaxXSegs, "mul_mat_q8_0_batch: too few weight rows for this K");
    const size_t fixed = 256 + (size_t)max_xs * kSliceBytes, slot_bytes = (size_t)a.nw * kTileBytes;
    // half an SM per CTA when possible, so the next kernel's CTAs fit beside it
    const size_t budget = 227 * 1024 / 2 - 1024;
    uint32_t slots = budget > fixed + 2 * slot_bytes ? (uint32_t)((budget - fixed) / slot_bytes) : 2;
    static const int force_slots = env_int("ANE_Q8B_SLOTS");
    if (force_slots > 0) slots = (uint32_t)force_slots;
    a.nslots = slots < 2 ? 2 : (slots > kMaxSlots ? kMaxSlots : slots);
    const size_t smem = fixed + a.nslots * slot_bytes;
    ANE_ARG_CHECK(smem <= 227 * 1024, "mul_mat_q8_0_batch: shared memory plan too large");

    const uint64_t row_bytes = (uint64_t)L.nb * 34;
    CUtensorMap wmap;
    int rc = encode_tensor_map_2d(&wmap, CU_TENSOR_MAP_DATA_TYPE_UINT32, W, row_bytes / 4, M, row_bytes,
                                  kChunkBytes / 4, kRows, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
    uint8_t* slices = ws + L.slices;
    const uint32_t nthreads = L.nb * kTok;
    rc = launch_pdl(quantize_x_slices_kernel, dim3((nthreads + 255) / 256), dim3(256), 0, s, x, ldx, NT, L.nb, slices);
    if (rc) return rc;
    const dim3 grid(ctas), block(32 * (a.nw + 1));
    if (NT <= 8) {
        static const cudaError_t e1 = cudaFuncSetAttribute(q8_0_gemm_q8_kernel<1>,
                                                           cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
        ANE_CUDA_TRY(e1);
        return launch_pdl(q8_0_gemm_q8_kernel<1>, grid, block, smem, s, wmap, (const uint8_t*)slices, a,
                          device_timeout_flag());
    }
    static const cudaError_t e2 = cudaFuncSetAttribute(q8_0_gemm_q8_kernel<2>,
                                                       cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    ANE_CUDA_TRY(e2);
    return launch_pdl(q8_0_gemm_q8_kernel<2>, grid, block, smem, s, wmap, (const uint8_t*)slices, a,
                      device_timeout_flag());
}

}  // namespace ane_b200
