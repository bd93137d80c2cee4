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
// Launch 1 (quantize_x_chunks_kernel): the activation rows, quantized with the
// ggml Q8_0 rule, into one record per chunk of kChunk blocks:
//     codes  [kChunk][16 tokens][8 words]   words of a block stored as 0,4,1,5,2,6,3,7
//     scales [kChunk][8][2] fp32            token t at (t % 8) * 2 + t / 8
// (zero past NT) -- the layout the MMA fragments load with one 64-bit
// shared-memory load per token and block.
// Launch 2 (q8_0_gemm_q8_kernel): the structure of the batch-1 streaming matvec.
// Rows are dealt to the CTAs in balanced runs of 4; a compute warp owns 8 rows
// (or the run's last 4) over the whole of K.  One producer warp per CTA feeds a
// ring whose stage t holds chunk t of K: the activation record (one bulk copy)
// and every compute warp's 8 x 272 B weight tile (2-D TMA).  Per block a warp
// runs one mma.sync m16n8k32 (s8 x s8 -> s32) -- the 16 tokens as M, its 8
// weight rows as N -- issuing a chunk's eight products before their fp32 scale
// math; the int32 dots become floats by an exact magic-number add.  Segment
// sums stay in registers; nothing crosses warps or CTAs.
#include <cuda.h>

#include "ane_internal.cuh"
#include "q8_mmq.cuh"
#include "sm100_ptx.cuh"

namespace ane_b200 {
namespace {

constexpr uint32_t kRows = 8;                             // weight rows per compute warp (MMA N)
constexpr uint32_t kSegBlocks = 32;                       // blocks per K segment (the sum grouping)
constexpr uint32_t kChunk = 8;                            // blocks per ring stage
constexpr uint32_t kChunkBytes = kChunk * 34;             // 272 B of a row
constexpr uint32_t kTileBytes = kRows * kChunkBytes;      // 2176 = 17 x 128
constexpr uint32_t kChunksPerSeg = kSegBlocks / kChunk;   // 4
constexpr uint32_t kTok = 16;                             // activation rows per record (MMA M)
constexpr uint32_t kXCodes = kChunk * kTok * 32;          // 4096
constexpr uint32_t kXChunkBytes = kXCodes + kChunk * kTok * 4;  // + scales = 4608 = 36 x 128
constexpr uint32_t kMaxWarps = 16;
constexpr uint32_t kMaxSlots = 8;
static_assert(kTileBytes % 128 == 0 && kXChunkBytes % 128 == 0, "TMA / bulk destinations stay 128-byte aligned");
static_assert(kSegBlocks % kChunk == 0, "a stage never straddles two segments");

__host__ __device__ constexpr size_t round_up256(size_t v) { return (v + 255) / 256 * 256; }

// ------------------------------------------------------- activation records
// Thread i = (block b, token t): ggml Q8_0 quantization of x[t][32b..32b+31]
// (q8_quantize_words, the arithmetic of every other Q8_0 activation path here).
__global__ void quantize_x_chunks_kernel(const float* __restrict__ x, size_t ldx, uint32_t NT, uint32_t nb,
                                         uint8_t* __restrict__ chunks) {
    ptx::griddep_launch_dependents();
    ptx::griddep_wait();  // x may come from the previous kernel; the records may still be read by it
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= nb * kTok) return;
    const uint32_t b = i / kTok, t = i % kTok;
    const uint32_t c = b / kChunk, j = b % kChunk;
    uint8_t* rec = chunks + (size_t)c * kXChunkBytes;
    uint4* codes = reinterpret_cast<uint4*>(rec + ((size_t)j * kTok + t) * 32);
    float* scale = reinterpret_cast<float*>(rec + kXCodes) + j * kTok + (t % 8) * 2 + t / 8;
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

// Two IEEE fp32 products (round to nearest even) in one packed instruction.
// Only ever followed by another multiply, so nothing can fuse it into an FMA.
__device__ __forceinline__ float2 fmul2_rn(float2 a, float2 b) {
    float2 d;
    asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
        "mov.b64 ra, {%2, %3};\n\t"
        "mov.b64 rb, {%4, %5};\n\t"
        "mul.rn.f32x2 rd, ra, rb;\n\t"
        "mov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return d;
}

// float(s) for |s| < 2^22, exactly: the bits of 1.5 * 2^23 + s, minus 1.5 * 2^23
// (|sumi| <= 32 * 128 * 127 < 2^19).  Integer add + fp32 add, both full rate.
__device__ __forceinline__ float i2f_exact(int32_t s) {
    return __fsub_rn(__int_as_float(0x4B400000 + s), 12582912.0f);
}

// acc + float(sumi) * p with p = RN(dw * dx): separate RN operations, never fused
__device__ __forceinline__ float q8_term_add(float acc, int32_t sumi, float p) {
    return __fadd_rn(acc, __fmul_rn(i2f_exact(sumi), p));
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
    uint32_t M, nb, NT, quads, nw, nslots, flags;
};

__global__ void __launch_bounds__(32 * (kMaxWarps + 1), 1)
    q8_0_gemm_q8_kernel(const __grid_constant__ CUtensorMap wmap8, const __grid_constant__ CUtensorMap wmap4,
                        const uint8_t* __restrict__ xchunks, const GemmQ8Args a, int* err) {
    extern __shared__ __align__(128) uint8_t smem[];
    const uint32_t nw = a.nw, nslots = a.nslots, nchunks = a.nb / kChunk;
    const uint32_t slot_bytes = kXChunkBytes + nw * kTileBytes;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);  // nslots
    uint64_t* empty = full + kMaxSlots;                  // nslots
    uint8_t* ring = smem + 256;
    // this CTA's rows: quads [q0, q1) (balanced); warp unit i = quads q0+2i, q0+2i+1
    const uint32_t q0 = (uint32_t)((uint64_t)a.quads * blockIdx.x / gridDim.x);
    const uint32_t q1 = (uint32_t)((uint64_t)a.quads * (blockIdx.x + 1) / gridDim.x);
    const uint32_t units = (q1 - q0 + 1) / 2, npass = (units + nw - 1) / nw, ntiles = npass * nchunks;
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < nslots; s++) {
            ptx::mbar_init(&full[s], 1);
            ptx::mbar_init(&empty[s], nw);
        }
        ptx::fence_mbarrier_init();
    }
    __syncthreads();
    ptx::griddep_launch_dependents();

    if (warp == 0) {
        if (lane == 0 && units > 0) {
            ptx::prefetch_tmap(&wmap8);
            ptx::prefetch_tmap(&wmap4);
            // stage t = chunk t % nchunks of pass t / nchunks: the activation record, then the weight tiles
            auto stage_bytes = [&](uint32_t t) {
                const uint32_t pass = t / nchunks;
                uint32_t bytes = kXChunkBytes;
                for (uint32_t w = 0; w < nw; w++) {
                    const uint32_t qa = q0 + 2 * (pass * nw + w);
                    if (qa >= q1) break;
                    bytes += (qa + 1 < q1 ? 2u : 1u) * (kTileBytes / 2);
                }
                return bytes;
            };
            auto issue_weights = [&](uint32_t t, uint32_t slot) {
                const uint32_t pass = t / nchunks, c = t - pass * nchunks;
                uint8_t* dst = ring + (size_t)slot * slot_bytes + kXChunkBytes;
                for (uint32_t w = 0; w < nw; w++) {
                    const uint32_t qa = q0 + 2 * (pass * nw + w);
                    if (qa >= q1) break;
                    // x in 32-bit words: c * 272 / 4 = 68 c (a multiple of 4 words)
                    ptx::tma_load_2d(dst + (size_t)w * kTileBytes, qa + 1 < q1 ? &wmap8 : &wmap4, &full[slot],
                                     (int)(c * (kChunkBytes / 4)), (int)(qa * 4));
                }
            };
            auto issue_x = [&](uint32_t t, uint32_t slot) {
                const uint32_t c = t % nchunks;
                ptx::bulk_load(ring + (size_t)slot * slot_bytes, xchunks + (size_t)c * kXChunkBytes, kXChunkBytes,
                               &full[slot]);
            };
            // static weights: the first stages' weight tiles are requested before the
            // previous kernel ends; their activation records only after it
            const uint32_t pre = (a.flags & ANE_Q8_WEIGHTS_STATIC) ? min(nslots, ntiles) : 0;
            for (uint32_t t = 0; t < pre; t++) {
                ptx::mbar_arrive_expect_tx(&full[t], stage_bytes(t));
                issue_weights(t, t);
            }
            ptx::griddep_wait();  // the activation records come from the quantize kernel
            for (uint32_t t = 0; t < pre; t++) issue_x(t, t);
            for (uint32_t t = pre; t < ntiles; t++) {
                const uint32_t slot = t % nslots;
                if (!ptx::mbar_wait(&empty[slot], ((t / nslots) & 1) ^ 1, err)) break;
                ptx::mbar_arrive_expect_tx(&full[slot], stage_bytes(t));
                issue_x(t, slot);
                issue_weights(t, slot);
            }
        }
        return;
    }
    // ------------------------------------------------------------ compute
    ptx::griddep_wait();  // y may still be read by the kernel before this one
    const uint32_t cw = warp - 1;
    if (units == 0) return;
    const uint32_t g = lane >> 2, q = lane & 3;
    bool alive = true;
    for (uint32_t pass = 0; pass < npass && alive; pass++) {
        const uint32_t qa = q0 + 2 * (pass * nw + cw);
        const bool active = qa < q1;
        const uint32_t rows = active ? (qa + 1 < q1 ? 8u : 4u) : 0u;  // real rows of this warp's tile
        // thread (g, q): tokens g, g+8 x weight rows 2q, 2q+1 of the tile
        float seg[4] = {0.0f, 0.0f, 0.0f, 0.0f}, total[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        for (uint32_t c = 0; c < nchunks; c++) {
            const uint32_t t = pass * nchunks + c, slot = t % nslots;
            if (!ptx::mbar_wait(&full[slot], (t / nslots) & 1, err)) {
                alive = false;
                break;
            }
            if (active) {
                const uint8_t* xs = ring + (size_t)slot * slot_bytes;
                const float* xd = reinterpret_cast<const float*>(xs + kXCodes);
                const uint8_t* tile = xs + kXChunkBytes + (size_t)cw * kTileBytes;
                const uint8_t* rb = tile + g * kChunkBytes;         // B fragment: weight row g
                const uint8_t* rd0 = tile + (2 * q) * kChunkBytes;  // scales of rows 2q, 2q+1
                const uint8_t* rd1 = rd0 + kChunkBytes;
                int32_t d[kChunk][4];
#pragma unroll
                for (uint32_t j = 0; j < kChunk; j++) {  // the chunk's eight products first
                    uint32_t b0 = 0, b1 = 0;
                    if (g < rows) {
                        if (j & 1)
                            block_words<true>(rb + j * 34, q, b0, b1);
                        else
                            block_words<false>(rb + j * 34, q, b0, b1);
                    }
                    const uint2 x0 = *reinterpret_cast<const uint2*>(xs + ((size_t)j * kTok + g) * 32 + 8 * q);
                    const uint2 x1 = *reinterpret_cast<const uint2*>(xs + ((size_t)j * kTok + g + 8) * 32 + 8 * q);
                    const uint32_t fa[4] = {x0.x, x1.x, x0.y, x1.y};
                    mma_s8_16832(fa, b0, b1, d[j]);
                }
#pragma unroll
                for (uint32_t j = 0; j < kChunk; j++) {  // then their terms, in block order
                    const float2 dw = make_float2(__half2float(*reinterpret_cast<const __half*>(rd0 + j * 34)),
                                                  __half2float(*reinterpret_cast<const __half*>(rd1 + j * 34)));
                    const float2 dx = *reinterpret_cast<const float2*>(xd + j * kTok + 2 * g);  // tokens g, g+8
                    const float2 p0 = fmul2_rn(make_float2(dx.x, dx.x), dw);  // token g   x rows 2q, 2q+1
                    const float2 p1 = fmul2_rn(make_float2(dx.y, dx.y), dw);  // token g+8 x rows 2q, 2q+1
                    seg[0] = q8_term_add(seg[0], d[j][0], p0.x);
                    seg[1] = q8_term_add(seg[1], d[j][1], p0.y);
                    seg[2] = q8_term_add(seg[2], d[j][2], p1.x);
                    seg[3] = q8_term_add(seg[3], d[j][3], p1.y);
                }
                if ((c + 1) % kChunksPerSeg == 0 || c + 1 == nchunks) {  // segment complete
#pragma unroll
                    for (int k = 0; k < 4; k++) {
                        total[k] = __fadd_rn(total[k], seg[k]);
                        seg[k] = 0.0f;
                    }
                }
            }
            __syncwarp();
            if (lane == 0) ptx::mbar_arrive(&empty[slot]);
        }
        if (!alive || !active) continue;
        const uint32_t row0 = qa * 4 + 2 * q;  // rows 2q, 2q+1 of the tile
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const uint32_t row = row0 + (k & 1), tok = g + 8 * (k >> 1);
            if (2 * q + (k & 1) < rows && row < a.M && tok < a.NT) a.y[(size_t)tok * a.ldy + row] = total[k];
        }
    }
}

}  // namespace

// Workspace: the activation records, nb / kChunk of kXChunkBytes.
size_t mul_mat_q8_0_batch_workspace_size(uint32_t M, uint32_t K) {
    (void)M;
    return round_up256((size_t)(K / 32 / kChunk) * kXChunkBytes);
}

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
    const uint32_t sms = (uint32_t)num_sms(), nb = K / 32;
    GemmQ8Args a;
    a.y = y;
    a.ldy = ldy;
    a.M = M;
    a.nb = nb;
    a.NT = NT;
    a.quads = (M + 3) / 4;
    a.flags = flags;
    // balanced runs of quads per CTA; one or more CTAs per SM so that a CTA
    // needs at most kMaxWarps compute warps (8 rows each)
    const uint32_t units_per_sm = (a.quads + 2 * sms - 1) / (2 * sms);
    uint32_t cps = (units_per_sm + kMaxWarps - 1) / kMaxWarps;
    if (cps == 0) cps = 1;
    uint32_t ctas = sms * cps;
    if (ctas > a.quads) ctas = a.quads;
    const uint32_t max_quads = (a.quads + ctas - 1) / ctas;
    a.nw = (max_quads + 1) / 2;
    if (a.nw > kMaxWarps) a.nw = kMaxWarps;
    const size_t slot_bytes = kXChunkBytes + (size_t)a.nw * kTileBytes;
    // with one CTA per SM, room for the next kernel's CTA beside it
    const size_t budget = (cps == 1 ? 227 * 1024 / 2 : 227 * 1024 / cps) - 1024;
    uint32_t slots = budget > 256 + 2 * slot_bytes ? (uint32_t)((budget - 256) / slot_bytes) : 2;
    static const int force_slots = env_int("ANE_Q8B_SLOTS");
    if (force_slots > 0) slots = (uint32_t)force_slots;
    a.nslots = slots < 2 ? 2 : (slots > kMaxSlots ? kMaxSlots : slots);
    const size_t smem = 256 + a.nslots * slot_bytes;
    ANE_ARG_CHECK(smem <= 227 * 1024, "mul_mat_q8_0_batch: shared memory plan too large");

    const uint64_t row_bytes = (uint64_t)nb * 34;
    CUtensorMap wmap8, wmap4;
    int rc = encode_tensor_map_2d(&wmap8, CU_TENSOR_MAP_DATA_TYPE_UINT32, W, row_bytes / 4, M, row_bytes,
                                  kChunkBytes / 4, kRows, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
    rc = encode_tensor_map_2d(&wmap4, CU_TENSOR_MAP_DATA_TYPE_UINT32, W, row_bytes / 4, M, row_bytes,
                              kChunkBytes / 4, kRows / 2, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
    uint8_t* chunks = static_cast<uint8_t*>(workspace);
    const uint32_t nthreads = nb * kTok;
    rc = launch_pdl(quantize_x_chunks_kernel, dim3((nthreads + 255) / 256), dim3(256), 0, s, x, ldx, NT, nb, chunks);
    if (rc) return rc;
    static const cudaError_t attr_err =
        cudaFuncSetAttribute(q8_0_gemm_q8_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    ANE_CUDA_TRY(attr_err);
    return launch_pdl(q8_0_gemm_q8_kernel, dim3(ctas), dim3(32 * (a.nw + 1)), smem, s, wmap8, wmap4,
                      (const uint8_t*)chunks, a, device_timeout_flag());
}

}  // namespace ane_b200
