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
// Launch 1 (quantize_x_segments_kernel): the activation rows, quantized with the
// ggml Q8_0 rule, into one record per K segment of 32 blocks:
//     codes  [32 blocks][8 g][4 q][4 words]   lane (g, q) of an MMA A fragment: words q of
//                                              tokens g, g+8, then words q+4 of tokens g, g+8
//     scales [32 blocks][8][2] fp32            token t at (t % 8) * 2 + t / 8
// (zero past NT) -- the layout the MMA A fragments load with one 128-bit
// shared-memory load per lane and block.
// Launch 2 (q8_0_gemm_q8_kernel): rows are dealt to one CTA per SM in balanced
// runs of 4; the CTA's rows form tiles of 8 (the run's last tile may hold 4).
// One producer warp feeds a ring whose stage holds one K segment: the
// activation record (one bulk copy) and each tile's 8 rows as one 2-D TMA box
// of 138 x 8 int64 elements from the segment start (long box rows keep the TMA
// engine at HBM rate -- 272-byte rows held it near 2 TB/s -- and the 1104-byte
// row pitch keeps the fragment loads free of bank conflicts).  Two groups of
// compute warps take alternate segments, one warp per tile in each group.  Per
// block a warp runs one mma.sync m16n8k32 (s8 x s8 -> s32) -- the 16 tokens as
// M, the tile's 8 rows as N -- the next eight products ahead of the current
// eight blocks' fp32 scale math; the int32 dots become floats exactly through
// a magic number the MMA adds as its C operand.  A warp's segment sum joins the
// row total in segment order through a per-tile shared-memory baton (one
// mbarrier phase per segment), so the fp32 order is the contract's whatever
// the group timing.
#include <cuda.h>

#include "ane_internal.cuh"
#include "q8_mmq.cuh"
#include "sm100_ptx.cuh"

namespace ane_b200 {
namespace {

constexpr uint32_t kRows = 8;                             // weight rows per tile (MMA N)
constexpr uint32_t kSegBlocks = 32;                       // blocks per K segment (the sum grouping)
constexpr uint32_t kSegBytes = kSegBlocks * 34;           // 1088 B of a row per segment
constexpr uint32_t kRowPitch = kSegBytes + 16;            // 276 words: rows g = 0..7 start in distinct 4-bank groups
constexpr uint32_t kTileBytes = kRows * kRowPitch;        // 8832 = 69 x 128
constexpr uint32_t kTok = 16;                             // activation rows per record (MMA M)
constexpr uint32_t kXCodes = kSegBlocks * kTok * 32;      // 16384
constexpr uint32_t kXSegBytes = kXCodes + kSegBlocks * kTok * 4;  // + scales = 18432 = 144 x 128
constexpr uint32_t kMaxTiles = 6;                         // tiles per pass (compute warps per group)
constexpr uint32_t kMaxGroups = 2;
constexpr uint32_t kMaxSlots = 8;
constexpr uint32_t kTotBytes = 32 * 4 * 4;                // one tile's running totals: 32 lanes x 4 floats
constexpr uint32_t kRingOffset = 256 + kMaxTiles * kTotBytes;  // 3328 = 26 x 128
static_assert(kTileBytes % 128 == 0 && kXSegBytes % 128 == 0 && kRingOffset % 128 == 0,
              "TMA / bulk destinations stay 128-byte aligned");
static_assert(kSegBytes % 16 == 0 && kRowPitch / 8 <= 256 && (kRowPitch / 4) % 8 == 4,
              "a segment start is a 16-byte aligned TMA x; one box row of int64 elements; a row pitch of 4 mod 8 "
              "words keeps the fragment loads free of bank conflicts");

__host__ __device__ constexpr size_t round_up256(size_t v) { return (v + 255) / 256 * 256; }

// ------------------------------------------------------- activation records
// Thread i = (block b, token t): ggml Q8_0 quantization of x[t][32b..32b+31]
// (q8_quantize_words, the arithmetic of every other Q8_0 activation path here).
// Blocks past nb in the last segment's record are never written nor read.
//
// GATHER (one link of a row-sharded chain, decode at batch NT): x is either the
// plain fp32 input or, with x_from_prev, the previous projection's TAGGED output
// on this GPU (token t's words at prev + t * ldw): all 16 two-word loads of a
// block in flight, then the pairs without the previous projection's tag read
// again together each round (bounded).  Block 0 also waits for one word per
// rank of the previous projection's output: a rank's word proves that rank
// has finished reading the vector the GEMM after this kernel overwrites.
__device__ __forceinline__ uint4 ld_word2(const uint64_t* p) {
    uint64_t a, b;
    asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
    return make_uint4((uint32_t)a, (uint32_t)(a >> 32), (uint32_t)b, (uint32_t)(b >> 32));
}
__device__ __forceinline__ bool wait_word(const uint64_t* p, uint32_t tag, int* err) {
    const long long t0 = clock64();
    while (true) {
        uint64_t w;
        asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
        if ((uint32_t)(w >> 32) == tag) return true;
        if (clock64() - t0 > ptx::kWaitTimeoutCycles) {
            atomicAdd(err, 1);
            return false;
        }
        __nanosleep(64);
    }
}

template <bool GATHER>
__global__ void quantize_x_segments_kernel(const float* __restrict__ x, size_t ldx, uint32_t NT, uint32_t nb,
                                           uint8_t* __restrict__ records, const __grid_constant__ Q8BatchGather bg,
                                           int* err) {
    ptx::griddep_launch_dependents();
    ptx::griddep_wait();  // x may come from the previous kernel; the records may still be read by it
    uint32_t tag_in = 0;  // the previous projection's tag
    if constexpr (GATHER) {
        tag_in = *reinterpret_cast<const volatile uint32_t*>(bg.tok) * bg.nproj + bg.j;
        if (blockIdx.x == 0 && threadIdx.x < bg.world) wait_word(bg.prev + (size_t)threadIdx.x * bg.prev_rows, tag_in, err);
    }
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= nb * kTok) return;
    const uint32_t b = i / kTok, t = i % kTok;
    const uint32_t s = b / kSegBlocks, j = b % kSegBlocks;
    uint8_t* rec = records + (size_t)s * kXSegBytes;
    // token t = g + 8h: word q at lane (g, q) word h, word q+4 at lane (g, q) word 2+h
    uint32_t* codes = reinterpret_cast<uint32_t*>(rec + (size_t)j * kTok * 32 + (t % 8) * 64) + t / 8;
    float* scale = reinterpret_cast<float*>(rec + kXCodes) + j * kTok + (t % 8) * 2 + t / 8;
    if (t >= NT) {
#pragma unroll
        for (int q = 0; q < 4; q++) codes[4 * q] = codes[4 * q + 2] = 0u;
        *scale = 0.0f;
        return;
    }
    float v[32];
    if (GATHER && bg.x_from_prev) {
        const uint64_t* blk = bg.prev + (size_t)t * bg.ldw + (size_t)b * 32;
        uint32_t miss = 0;
#pragma unroll
        for (int k = 0; k < 16; k++) {
            const uint4 w = ld_word2(blk + 2 * k);
            v[2 * k] = __uint_as_float(w.x);
            v[2 * k + 1] = __uint_as_float(w.z);
            miss |= (w.y != tag_in || w.w != tag_in) ? 1u << k : 0u;
        }
        const long long t0 = miss ? clock64() : 0;
        while (miss) {
            if (clock64() - t0 > ptx::kWaitTimeoutCycles) {
                atomicAdd(err, 1);
                break;  // counted; the values are whatever was there
            }
            __nanosleep(64);
#pragma unroll
            for (int k = 0; k < 16; k++) {
                if (!((miss >> k) & 1u)) continue;
                const uint4 w = ld_word2(blk + 2 * k);
                if (w.y == tag_in && w.w == tag_in) {
                    v[2 * k] = __uint_as_float(w.x);
                    v[2 * k + 1] = __uint_as_float(w.z);
                    miss &= ~(1u << k);
                }
            }
        }
    } else {
        const float4* xb = reinterpret_cast<const float4*>(x + (size_t)t * ldx + (size_t)b * 32);
#pragma unroll
        for (int k = 0; k < 8; k++) {
            const float4 f = xb[k];
            v[4 * k] = f.x;
            v[4 * k + 1] = f.y;
            v[4 * k + 2] = f.z;
            v[4 * k + 3] = f.w;
        }
    }
    uint32_t w[8];
    *scale = q8_quantize_words(v, w);
#pragma unroll
    for (int q = 0; q < 4; q++) {
        codes[4 * q] = w[q];
        codes[4 * q + 2] = w[q + 4];
    }
}

// d = a x b + c (s8 x s8 -> s32, exact; the int32 add wraps)
__device__ __forceinline__ void mma_s8_16832(const uint32_t (&a)[4], uint32_t b0, uint32_t b1, int32_t c,
                                             int32_t (&d)[4]) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%10, %10, %10, %10};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(c));
}

// Packed IEEE fp32 operations, round to nearest even, subnormals kept: two
// lanes per instruction, each lane exactly the scalar operation.  Used only
// where no product feeds a sum (products of products, sums of exact values),
// since the assembler may contract a packed multiply and add into an FMA.
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
__device__ __forceinline__ float2 fadd2_rn(float2 a, float2 b) {
    float2 d;
    asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
        "mov.b64 ra, {%2, %3};\n\t"
        "mov.b64 rb, {%4, %5};\n\t"
        "add.rn.f32x2 rd, ra, rb;\n\t"
        "mov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return d;
}

// The products carry the magic number 1.5 * 2^23 (0x4B400000) added by the
// tensor core (the MMA's C operand): for |sumi| < 2^22 the bits 0x4B400000 +
// sumi are the float 1.5 * 2^23 + sumi, so one packed fp32 add of -1.5 * 2^23
// gives float(sumi) exactly (|sumi| <= 32 * 128 * 127 < 2^19).
constexpr int32_t kMagic = 0x4B400000;
__device__ __forceinline__ float2 magic2_to_float(int32_t m0, int32_t m1) {
    return fadd2_rn(make_float2(__int_as_float(m0), __int_as_float(m1)), make_float2(-12582912.0f, -12582912.0f));
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

// The products of blocks j0..j0+7 of one tile: d[u] = kMagic + the int32 dots
// of block j0+u for (token g | g+8) x (tile row 2q | 2q+1).
__device__ __forceinline__ void block_products(const uint8_t* xs, const uint8_t* rb, uint32_t j0, uint32_t rows,
                                               uint32_t g, uint32_t q, int32_t (&d)[8][4]) {
#pragma unroll
    for (uint32_t u = 0; u < 8; u++) {
        const uint32_t j = j0 + u;
        uint32_t b0 = 0, b1 = 0;
        if (g < rows) {
            if (u & 1)
                block_words<true>(rb + j * 34, q, b0, b1);
            else
                block_words<false>(rb + j * 34, q, b0, b1);
        }
        const uint4 xa = *reinterpret_cast<const uint4*>(xs + (size_t)j * kTok * 32 + (g * 4 + q) * 16);
        const uint32_t fa[4] = {xa.x, xa.y, xa.z, xa.w};
        mma_s8_16832(fa, b0, b1, kMagic, d[u]);
    }
}

// The terms of blocks j0..j0+7, added in block order.
__device__ __forceinline__ void block_terms(const float* xd, const uint8_t* rd0, const uint8_t* rd1, uint32_t j0,
                                            uint32_t g, const int32_t (&d)[8][4], float2& seg01, float2& seg23) {
#pragma unroll
    for (uint32_t u = 0; u < 8; u++) {
        const uint32_t j = j0 + u;
        const float2 dw = make_float2(__half2float(*reinterpret_cast<const __half*>(rd0 + j * 34)),
                                      __half2float(*reinterpret_cast<const __half*>(rd1 + j * 34)));
        const float2 dx = *reinterpret_cast<const float2*>(xd + j * kTok + 2 * g);  // tokens g, g+8
        const float2 p0 = fmul2_rn(make_float2(dx.x, dx.x), dw);  // token g   x rows 2q, 2q+1
        const float2 p1 = fmul2_rn(make_float2(dx.y, dx.y), dw);  // token g+8 x rows 2q, 2q+1
        // the term products and the sums stay scalar: a packed product feeding a
        // packed sum is contracted into an FMA by the assembler
        const float2 f01 = magic2_to_float(d[u][0], d[u][1]), f23 = magic2_to_float(d[u][2], d[u][3]);
        seg01.x = __fadd_rn(seg01.x, __fmul_rn(f01.x, p0.x));
        seg01.y = __fadd_rn(seg01.y, __fmul_rn(f01.y, p0.y));
        seg23.x = __fadd_rn(seg23.x, __fmul_rn(f23.x, p1.x));
        seg23.y = __fadd_rn(seg23.y, __fmul_rn(f23.y, p1.y));
    }
}

// One K segment of one tile: the sum from +0, in block order, of the terms of
// blocks [0, nblk) (nblk a multiple of 8).  Thread (g, q) holds tokens g, g+8 x
// tile rows 2q, 2q+1: seg01 = (tok g, row 2q | 2q+1), seg23 = (tok g+8, ...).
// Software-pipelined: the next eight products are issued before the current
// eight blocks' terms, so the tensor-core latency hides behind the fp32 work.
__device__ __forceinline__ void segment_sums(const uint8_t* xs, const uint8_t* tile, uint32_t nblk, uint32_t rows,
                                             uint32_t g, uint32_t q, float2& seg01, float2& seg23) {
    const float* xd = reinterpret_cast<const float*>(xs + kXCodes);
    const uint8_t* rb = tile + g * kRowPitch;         // B fragment: tile row g
    const uint8_t* rd0 = tile + (2 * q) * kRowPitch;  // scales of rows 2q, 2q+1
    const uint8_t* rd1 = rd0 + kRowPitch;
    seg01 = make_float2(0.0f, 0.0f);
    seg23 = make_float2(0.0f, 0.0f);
    int32_t da[8][4], db[8][4];
    block_products(xs, rb, 0, rows, g, q, da);
    for (uint32_t j0 = 0; j0 < nblk; j0 += 16) {
        const bool more = j0 + 8 < nblk;
        if (more) block_products(xs, rb, j0 + 8, rows, g, q, db);
        block_terms(xd, rd0, rd1, j0, g, da, seg01, seg23);
        if (!more) break;
        if (j0 + 16 < nblk) block_products(xs, rb, j0 + 16, rows, g, q, da);
        block_terms(xd, rd0, rd1, j0 + 8, g, db, seg01, seg23);
    }
}

// ------------------------------------------------------------- the product
struct GemmQ8Args {
    float* y;
    size_t ldy;
    uint32_t M, nb, NT, quads;
    uint32_t ntiles;  // tiles per pass (compute warps per group)
    uint32_t ngroups, nslots, flags;
};

template <bool GATHER>
__global__ void __launch_bounds__(32 * (kMaxTiles * kMaxGroups + 1), 1)
    q8_0_gemm_q8_kernel(const __grid_constant__ CUtensorMap wmap8, const __grid_constant__ CUtensorMap wmap4,
                        const uint8_t* __restrict__ records, const GemmQ8Args a,
                        const __grid_constant__ Q8BatchGather bg, int* err) {
    extern __shared__ __align__(128) uint8_t smem[];
    const uint32_t T = a.ntiles, nslots = a.nslots, nseg = (a.nb + kSegBlocks - 1) / kSegBlocks;
    const uint32_t slot_bytes = kXSegBytes + T * kTileBytes;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);  // nslots
    uint64_t* empty = full + kMaxSlots;                  // nslots: T arrivals (the stage's group)
    uint64_t* baton = empty + kMaxSlots;                 // T: one phase per segment of the tile
    float* totals = reinterpret_cast<float*>(smem + 256);
    uint8_t* ring = smem + kRingOffset;
    // this CTA's rows: quads [q0, q1) (balanced); tile i of pass p = quads q0+2(pT+i), +1
    const uint32_t q0 = (uint32_t)((uint64_t)a.quads * blockIdx.x / gridDim.x);
    const uint32_t q1 = (uint32_t)((uint64_t)a.quads * (blockIdx.x + 1) / gridDim.x);
    const uint32_t tiles = (q1 - q0 + 1) / 2, npass = (tiles + T - 1) / T, nstages = npass * nseg;
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < nslots; s++) {
            ptx::mbar_init(&full[s], 1);
            ptx::mbar_init(&empty[s], T);
        }
        for (uint32_t i = 0; i < T; i++) ptx::mbar_init(&baton[i], 1);
        ptx::fence_mbarrier_init();
    }
    __syncthreads();
    ptx::griddep_launch_dependents();

    if (warp == 0) {
        if (lane == 0 && tiles > 0) {
            ptx::prefetch_tmap(&wmap8);
            ptx::prefetch_tmap(&wmap4);
            // stage t = segment t % nseg of pass t / nseg: the activation record, then
            // one TMA box per tile (full boxes: rows past M and bytes past the row end
            // arrive as zero fill and are never stored)
            auto weight_bytes = [&](uint32_t t) {
                const uint32_t pass = t / nseg;
                uint32_t bytes = 0;
                for (uint32_t i = 0; i < T; i++) {
                    const uint32_t qa = q0 + 2 * (pass * T + i);
                    if (qa >= q1) break;
                    bytes += (qa + 1 < q1 ? 2u : 1u) * (kTileBytes / 2);
                }
                return bytes;
            };
            auto issue_weights = [&](uint32_t t, uint32_t slot) {
                const uint32_t pass = t / nseg, s = t - pass * nseg;
                uint8_t* dst = ring + (size_t)slot * slot_bytes + kXSegBytes;
                for (uint32_t i = 0; i < T; i++) {
                    const uint32_t qa = q0 + 2 * (pass * T + i);
                    if (qa >= q1) break;
                    // x in int64 elements: s * 1088 / 8 = 136 s (16-byte aligned)
                    ptx::tma_load_2d(dst + (size_t)i * kTileBytes, qa + 1 < q1 ? &wmap8 : &wmap4, &full[slot],
                                     (int)(s * (kSegBytes / 8)), (int)(qa * 4));
                }
            };
            auto issue_x = [&](uint32_t t, uint32_t slot) {
                const uint32_t s = t % nseg;
                ptx::bulk_load(ring + (size_t)slot * slot_bytes, records + (size_t)s * kXSegBytes, kXSegBytes,
                               &full[slot]);
            };
            // static weights: the first stages' weight tiles are requested before the
            // previous kernel ends; their activation records only after it
            const uint32_t pre = (a.flags & ANE_Q8_WEIGHTS_STATIC) ? min(nslots, nstages) : 0;
            for (uint32_t t = 0; t < pre; t++) {
                ptx::mbar_arrive_expect_tx(&full[t], kXSegBytes + weight_bytes(t));
                issue_weights(t, t);
            }
            ptx::griddep_wait();  // the activation records come from the quantize kernel
            for (uint32_t t = 0; t < pre; t++) issue_x(t, t);
            for (uint32_t t = pre; t < nstages; t++) {
                const uint32_t slot = t % nslots;
                if (!ptx::mbar_wait(&empty[slot], ((t / nslots) & 1) ^ 1, err)) break;
                ptx::mbar_arrive_expect_tx(&full[slot], kXSegBytes + weight_bytes(t));
                issue_x(t, slot);
                issue_weights(t, slot);
            }
        }
        return;
    }
    // ------------------------------------------------------------ compute
    ptx::griddep_wait();  // y may still be read by the kernel before this one
    // GATHER: this projection's tag (the step count is final once the kernels
    // before this one have ended)
    const uint32_t tag_out = GATHER ? *reinterpret_cast<const volatile uint32_t*>(bg.tok) * bg.nproj + bg.j + 1u : 0u;
    const uint32_t cw = warp - 1, grp = cw / T, ti = cw % T;
    if (tiles == 0 || grp >= a.ngroups) return;
    const uint32_t g = lane >> 2, q = lane & 3;
    float* tot = totals + ti * (kTotBytes / 4) + lane * 4;
    // stage t goes to group t % ngroups, so with two groups stage t - 2 is always
    // this warp's own: when it waits on phase t - 1 of the baton, phase t - 2 is
    // complete and the parity test is exact.  A full-barrier parity wait is exact
    // too: by the baton, every stage before t - 2 of this tile has been consumed,
    // so slot t % nslots is at most one phase behind.  That argument needs the
    // baton, so a warp whose tile has no rows in a pass leaves (a tile without
    // rows has none in every later pass): out of step with the other group, an
    // odd ring could show it a slot two phases behind, its parity wait would pass
    // at once, and its early arrival would free a slot still being read.  Tile
    // 0's warp, which has rows in every pass, arrives for the ones that left.
    for (uint32_t t = grp; t < nstages; t += a.ngroups) {
        const uint32_t pass = t / nseg, s = t - pass * nseg, slot = t % nslots;
        const uint32_t qa = q0 + 2 * (pass * T + ti);
        if (qa >= q1) break;
        const uint32_t absent = T - min(T, tiles - pass * T);  // warps of this group that have left
        // one verdict per warp: no lane may reach the warp-wide MMAs or shuffles
        // without the others after a timed-out wait
        if (!__all_sync(0xffffffffu, ptx::mbar_wait(&full[slot], (t / nslots) & 1, err))) break;
        const uint32_t rows = qa + 1 < q1 ? 8u : 4u;  // real rows of this tile
        const uint8_t* xs = ring + (size_t)slot * slot_bytes;
        const uint32_t nblk = min(kSegBlocks, a.nb - s * kSegBlocks);
        float2 seg01, seg23;
        segment_sums(xs, xs + kXSegBytes + (size_t)ti * kTileBytes, nblk, rows, g, q, seg01, seg23);
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive_cnt(&empty[slot], ti == 0 ? 1u + absent : 1u);
        // the row totals, in segment order: wait for stage t - 1's phase of this
        // tile's baton, add this segment, pass the baton on
        if (t > 0 && !__all_sync(0xffffffffu, ptx::mbar_wait(&baton[ti], (t - 1) & 1, err))) break;
        float4 acc = s == 0 ? make_float4(0.0f, 0.0f, 0.0f, 0.0f) : *reinterpret_cast<const float4*>(tot);
        const float2 lo = fadd2_rn(make_float2(acc.x, acc.y), seg01);
        const float2 hi = fadd2_rn(make_float2(acc.z, acc.w), seg23);
        if (s + 1 < nseg) {
            *reinterpret_cast<float4*>(tot) = make_float4(lo.x, lo.y, hi.x, hi.y);
        } else {
            const uint32_t row0 = qa * 4 + 2 * q;  // rows 2q, 2q+1 of the tile
            const float v[4] = {lo.x, lo.y, hi.x, hi.y};
#pragma unroll
            for (int k = 0; k < 4; k++) {
                const uint32_t row = row0 + (k & 1), tok = g + 8 * (k >> 1);
                if (2 * q + (k & 1) < rows && row < a.M && tok < a.NT) {
                    if constexpr (GATHER) {
                        // one 8-byte {value, tag} word per rank: seen whole or not at all
                        const uint64_t w = (uint64_t)__float_as_uint(v[k]) | ((uint64_t)tag_out << 32);
                        for (uint32_t q8 = 0; q8 < bg.world; q8++)
                            asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(bg.out[q8] + (size_t)tok * bg.ldw + row),
                                         "l"(w)
                                         : "memory");
                    } else {
                        a.y[(size_t)tok * a.ldy + row] = v[k];
                    }
                }
            }
        }
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(&baton[ti]);
    }
}

}  // namespace
// Workspace: the activation records, one of kXSegBytes per K segment.
size_t mul_mat_q8_0_batch_workspace_size(uint32_t M, uint32_t K) {
    (void)M;
    return round_up256((size_t)((K / 32 + kSegBlocks - 1) / kSegBlocks) * kXSegBytes);
}

namespace {

// bg == nullptr: the plain MUL_MAT (x fp32, y fp32); else one chain link.
int launch_batch_impl(uint32_t M, uint32_t K, uint32_t NT, const float* x, size_t ldx, const uint8_t* W, float* y,
                      size_t ldy, void* workspace, uint32_t flags, cudaStream_t s, const Q8BatchGather* bg) {
    if (M == 0 || NT == 0) return ANE_OK;
    ANE_ARG_CHECK(NT <= kTok, "mul_mat_q8_0_batch: at most 16 activation rows");
    ANE_ARG_CHECK(K % 256 == 0 && K > 0, "mul_mat_q8_0_batch: K must be a positive multiple of 256");
    ANE_ARG_CHECK(((uintptr_t)W & 15) == 0, "mul_mat_q8_0_batch: W must be 16-byte aligned");
    if (!bg || !bg->x_from_prev)
        ANE_ARG_CHECK(x && ((uintptr_t)x & 15) == 0 && (NT == 1 || ldx % 4 == 0) && ldx >= K,
                      "mul_mat_q8_0_batch: x rows must be 16-byte aligned (ldx % 4 == 0, ldx >= K)");
    if (!bg) ANE_ARG_CHECK(ldy >= M || NT == 1, "mul_mat_q8_0_batch: ldy < M");
    ANE_ARG_CHECK(workspace && ((uintptr_t)workspace & 255) == 0, "mul_mat_q8_0_batch: workspace must be 256-byte aligned");
    const uint32_t sms = (uint32_t)num_sms(), nb = K / 32, nseg = (nb + kSegBlocks - 1) / kSegBlocks;
    GemmQ8Args a;
    a.y = y;
    a.ldy = ldy;
    a.M = M;
    a.nb = nb;
    a.NT = NT;
    a.quads = (M + 3) / 4;
    a.flags = flags;
    // balanced runs of quads, one CTA per SM; a CTA's tiles in as few balanced
    // passes as the tile cap allows; two warp groups unless K is one segment
    static const int force_tiles = env_int("ANE_Q8B_TILES"), force_slots = env_int("ANE_Q8B_SLOTS"),
                     force_groups = env_int("ANE_Q8B_GROUPS"), force_budget_kb = env_int("ANE_Q8B_SMEM_KB");
    const uint32_t ctas = a.quads < sms ? a.quads : sms;
    const uint32_t max_quads = (a.quads + ctas - 1) / ctas, max_tiles = (max_quads + 1) / 2;
    uint32_t tcap = force_tiles > 0 ? (uint32_t)force_tiles : 5u;
    if (tcap > kMaxTiles) tcap = kMaxTiles;
    const uint32_t npass = (max_tiles + tcap - 1) / tcap;
    a.ntiles = (max_tiles + npass - 1) / npass;
    a.ngroups = nseg >= 2 ? kMaxGroups : 1u;
    if (force_groups == 1) a.ngroups = 1;
    const size_t slot_bytes = kXSegBytes + (size_t)a.ntiles * kTileBytes;
    // three stages (measured on B200: 2 starve one group, 4 were slower than 3)
    const size_t budget = force_budget_kb > 0 ? (size_t)force_budget_kb * 1024 : 227 * 1024;
    uint32_t slots = budget > kRingOffset + 2 * slot_bytes ? (uint32_t)((budget - kRingOffset) / slot_bytes) : 2;
    if (slots > 3 && force_budget_kb <= 0) slots = 3;
    if (force_slots > 0) slots = (uint32_t)force_slots;
    a.nslots = slots < 2 ? 2 : (slots > kMaxSlots ? kMaxSlots : slots);
    const size_t smem = kRingOffset + a.nslots * slot_bytes;
    ANE_ARG_CHECK(smem <= 227 * 1024, "mul_mat_q8_0_batch: shared memory plan too large");

    // box rows of kRowPitch bytes from each segment start: the pitch the box lands
    // in shared memory with; the 16 bytes past the segment are the next one's (or
    // zero fill past the row end) and are never read
    const uint64_t row_bytes = (uint64_t)nb * 34;  // a multiple of 272, so of 8 and 16
    CUtensorMap wmap8, wmap4;
    int rc = encode_tensor_map_2d(&wmap8, CU_TENSOR_MAP_DATA_TYPE_INT64, W, row_bytes / 8, M, row_bytes,
                                  kRowPitch / 8, kRows, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
    rc = encode_tensor_map_2d(&wmap4, CU_TENSOR_MAP_DATA_TYPE_INT64, W, row_bytes / 8, M, row_bytes, kRowPitch / 8,
                              kRows / 2, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
    uint8_t* records = static_cast<uint8_t*>(workspace);
    const uint32_t nthreads = nb * kTok;  // blocks of 64: the activation spreads over more SMs
    const Q8BatchGather none{};
    if (!bg) {
        rc = launch_pdl(quantize_x_segments_kernel<false>, dim3((nthreads + 63) / 64), dim3(64), 0, s, x, ldx, NT,
                        nb, records, none, device_timeout_flag());
        if (rc) return rc;
        static std::atomic<uint64_t> smem_set{0};  // devices whose limit is raised
        if (int arc = set_max_dynamic_smem(q8_0_gemm_q8_kernel<false>, 227 * 1024, smem_set)) return arc;
        return launch_pdl(q8_0_gemm_q8_kernel<false>, dim3(ctas), dim3(32 * (1 + a.ntiles * a.ngroups)), smem, s,
                          wmap8, wmap4, (const uint8_t*)records, a, none, device_timeout_flag());
    }
    rc = launch_pdl(quantize_x_segments_kernel<true>, dim3((nthreads + 63) / 64), dim3(64), 0, s, x, ldx, NT, nb,
                    records, *bg, device_timeout_flag());
    if (rc) return rc;
    static std::atomic<uint64_t> smem_set_g{0};
    if (int arc = set_max_dynamic_smem(q8_0_gemm_q8_kernel<true>, 227 * 1024, smem_set_g)) return arc;
    return launch_pdl(q8_0_gemm_q8_kernel<true>, dim3(ctas), dim3(32 * (1 + a.ntiles * a.ngroups)), smem, s, wmap8,
                      wmap4, (const uint8_t*)records, a, *bg, device_timeout_flag());
}

}  // namespace

int launch_mul_mat_q8_0_batch(uint32_t M, uint32_t K, uint32_t NT, const float* x, size_t ldx, const uint8_t* W,
                              float* y, size_t ldy, void* workspace, uint32_t flags, cudaStream_t s) {
    return launch_batch_impl(M, K, NT, x, ldx, W, y, ldy, workspace, flags, s, nullptr);
}

int launch_mul_mat_q8_0_batch_gather(uint32_t M, uint32_t K, uint32_t NT, const float* x, size_t ldx,
                                     const uint8_t* W, void* workspace, const Q8BatchGather& g, uint32_t flags,
                                     cudaStream_t s) {
    return launch_batch_impl(M, K, NT, x, ldx, W, nullptr, 0, workspace, flags, s, &g);
}

}  // namespace ane_b200
