// gemm_s8_sm100.cu -- int8 x int8 -> int32 tensor-core GEMM for B200 (sm_100a)
// with the fused fp32 epilogue of dense_fused_i8 / dense_i8.
//
// Replaces the SME2 `smopa` loop nest of the reference handler dense_i8
// (src/bytecode_interpreter.s:1978-2446).  The arithmetic contract is the
// reference's: exact int32 accumulation over K, then per element
//   y = float_rn(acc); y = y * (sa*sb); [y = y*scale | y = y + bias[n]]; fmax(...)
// with every fp32 op a separate IEEE RN operation (no FMA contraction).
//
// Two kernels, both persistent and warp-specialised (192 threads per CTA):
//   warp 0      TMA producer into a shared-memory ring (SWIZZLE_128B, K-major).
//   warp 1      TMEM allocator + MMA issuer (one thread issues tcgen05.mma).
//   warps 2..5  epilogue: tcgen05.ld from the TMEM lane quarter the warp may
//               access, fp32 epilogue, then a 32x32 shared-memory transpose
//               (XOR-swizzled 16-byte chunks) so every global store instruction
//               writes four full 128-byte rows.
// * gemm_s8_pair_kernel: CTA pairs (cluster of 2, tcgen05 cta_group::2), tile
//   256 x 256.  Each CTA loads 128 rows of A and 128 rows of B^T per stage;
//   the even CTA issues M=256,N=256,K=32 MMAs that read both CTAs' shared
//   memory and write 128 accumulator rows into each CTA's TMEM.  Half the
//   operand bytes per SM of a 1-CTA 128x256 tile.
// * gemm_s8_single_kernel: one CTA, tile 128 x 256 (used when M <= 128).
// Two TMEM accumulators (2 x 256 int32 columns) per CTA let the epilogue of
// tile i overlap the MMAs of tile i+1.  No TMA multicast anywhere.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <float.h>

#include <stdlib.h>
#include <string.h>

#include <mutex>

#include "ane_internal.cuh"
#include "sm100_ptx.cuh"

namespace ane_b200 {
namespace {

constexpr int BK = 128;  // bytes = int8 elements = one 128-B swizzle row
constexpr int UMMA_K = 32;
constexpr int ACC_COLS = 256;
constexpr int TMEM_COLS = 2 * ACC_COLS;
constexpr int NUM_THREADS = 192;
constexpr int EPI_STAGE_WORDS = 32 * 32;  // per epilogue warp
constexpr int EPI_BYTES = 4 * EPI_STAGE_WORDS * 4;

// single-CTA configuration
constexpr int S_BM = 128, S_BN = 256, S_STAGES = 4;
constexpr int S_A = S_BM * BK, S_B = S_BN * BK, S_STAGE = S_A + S_B;
// CTA-pair configuration (per-CTA halves)
constexpr int P_BM = 256, P_BN = 256, P_HM = 128, P_HN = 128, P_STAGES = 6;
constexpr int P_A = P_HM * BK, P_B = P_HN * BK, P_STAGE = P_A + P_B;

template <int STAGES>
struct Barriers {
    uint64_t full[STAGES];
    uint64_t empty[STAGES];
    uint64_t tmem_full[2];
    uint64_t tmem_empty[2];
    uint32_t tmem_base;
};
// The 1-CTA kernel's operand region holds S_STAGES full stages; with a small M
// its stages are smaller (A tiles of round_up(M, 8) rows) and more of them fit.
constexpr int S_OPS = S_STAGES * S_STAGE, S_MAX_STAGES = 16;
constexpr size_t S_SMEM = (size_t)S_OPS + EPI_BYTES + sizeof(Barriers<S_MAX_STAGES>) + 1024;
constexpr size_t P_SMEM = (size_t)P_STAGES * P_STAGE + EPI_BYTES + sizeof(Barriers<P_STAGES>) + 1024;
static_assert(S_SMEM <= 232448 && P_SMEM <= 232448, "shared memory budget");

constexpr uint32_t kGatherMaxRanks = 8;
// MN-major B: bytes between two 128-column SWIZZLE_128B atoms of one stage
// (the single-CTA kernel's 256-column tile is two such boxes)
constexpr uint32_t kMnAtomBytes = 128 * BK;
constexpr uint32_t P_BN_COLS = 256;  // pair tile width (= P_BN)

struct Params {
    uint32_t M, N, K;
    uint32_t tiles_m, tiles_n, num_kb;
    uint32_t s_bn;  // 1-CTA kernel: columns per tile (256; 128 or 64 for an MN-major B when few tiles)
    // 1-CTA kernel ring: A tile rows loaded per stage (128, or round_up(M, 8) for
    // M < 128), stages, bytes of an A and a B tile, offset of the B tiles
    uint32_t s_am, s_stages, s_a_bytes, s_b_bytes, s_b_base;
    void* C;
    size_t ldc;
    int vec_ok;  // C rows allow 16-byte stores
    GemmEpilogue ep;
    int* err;
    // fused all-gather (world > 1): every tile is also stored into each rank's
    // gathered C (C_rank[q] = that rank's buffer at this rank's first row), and
    // each CTA adds 1 to every rank's counter once its stores are issued
    uint32_t world;
    void* C_rank[kGatherMaxRanks];
    uint32_t* ctr_rank[kGatherMaxRanks];
    // pair kernel, last partial wave: tiles tail_start.. are cut along N into
    // `split` parts (1, 2 or 4) of 256/split columns, each over the full K, so
    // the leftover tiles spread over all CTA pairs instead of a few
    uint32_t tail_start, split, num_units;
};

// One work unit of the pair kernel: a 256-row tile, columns n0 .. n0+ncols-1.
struct PairUnit {
    uint32_t m0, n0, ncols;
};
__device__ __forceinline__ PairUnit pair_unit(const Params& p, uint32_t u) {
    uint32_t t = u, j = 0, ncols = P_BN_COLS;
    if (u >= p.tail_start) {
        const uint32_t v = u - p.tail_start;
        t = p.tail_start + v / p.split;
        j = v % p.split;
        ncols = P_BN_COLS / p.split;
    }
    return {(t / p.tiles_n) * 256u, (t % p.tiles_n) * P_BN_COLS + j * ncols, ncols};
}

// max that propagates NaN (ARM FMAX, not IEEE maxNum); one instruction.
__device__ __forceinline__ float max_nan(float a, float b) {
    float r;
    asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
    return r;
}
// ReLU with the reference's FMAX semantics: NaN stays NaN, and the "+ 0.0f"
// turns a -0 result into +0 (FMAX(-0, +0) = +0) without changing anything else.
__device__ __forceinline__ float relu_arm(float y) { return __fadd_rn(max_nan(y, 0.0f), 0.0f); }

// Fused all-gather: after the CTA's last epilogue store, publish to every rank
// (release at system scope: the peers read these rows over NVLink).
__device__ __forceinline__ void gather_signal(const Params& p) {
    if (p.world > 1 && threadIdx.x == 0) {
        __threadfence_system();
        for (uint32_t q = 0; q < p.world; q++)
            asm volatile("red.release.sys.global.add.u32 [%0], 1;" ::"l"(p.ctr_rank[q]) : "memory");
    }
}

__device__ __forceinline__ float tile_comb(const Params& p) {
    if (p.ep.mode == kOutRawI32) return 0.0f;
    const float s0 = p.ep.scales ? p.ep.scales[0] : p.ep.sa_imm;
    const float s1 = p.ep.scales ? p.ep.scales[1] : p.ep.sb_imm;
    return __fmul_rn(s0, s1);
}

// One warp stores a 32 x 32 block: lane i holds row (row0 + i), columns nc..nc+31
// as raw accumulators in r[].  Rows are transposed through this warp's
// shared-memory stage so global stores are row-contiguous.
__device__ __forceinline__ void store_block(const Params& p, float comb, const uint32_t (&r)[32], uint32_t* stage,
                                            uint32_t row0, uint32_t nc, int lane) {
    if (row0 >= p.M || nc >= p.N) return;  // warp-uniform
    uint32_t v[32];
    // The mode / relu branches are warp-uniform and hoisted out of the element
    // loops; each loop is straight-line RN arithmetic.
    if (p.ep.mode == kOutRawI32) {
#pragma unroll
        for (int j = 0; j < 32; j++) v[j] = r[j];
    } else if (p.ep.mode == kOutFusedF32) {
        const float scale = p.ep.scale;
        if (p.ep.relu) {
#pragma unroll
            for (int j = 0; j < 32; j++)
                v[j] = __float_as_uint(relu_arm(__fmul_rn(__fmul_rn(__int2float_rn((int32_t)r[j]), comb), scale)));
        } else {
#pragma unroll
            for (int j = 0; j < 32; j++)
                v[j] = __float_as_uint(__fmul_rn(__fmul_rn(__int2float_rn((int32_t)r[j]), comb), scale));
        }
    } else if (p.ep.mode == kOutIntGemm) {
        // the reference seeds its int32 accumulator with the fp32 bits of beta*C
        // when beta != 0 (cblas integer GEMM macro, bytecode_interpreter.s:8411-8489)
        const float alpha = p.ep.alpha, beta = p.ep.beta;
        const bool fold = __float_as_uint(beta) != 0u;
        const uint32_t m = row0 + lane;
        const float* crow = reinterpret_cast<const float*>(p.C) + (size_t)m * p.ldc + nc;
#pragma unroll
        for (int j = 0; j < 32; j++) {
            uint32_t a = r[j];
            if (fold && m < p.M && nc + j < p.N) a += __float_as_uint(__fmul_rn(crow[j], beta));
            const float f = p.ep.acc_unsigned ? __uint2float_rn(a) : __int2float_rn((int32_t)a);
            v[j] = __float_as_uint(__fmul_rn(f, alpha));
        }
    } else {
        const float floor_v = p.ep.relu ? 0.0f : -FLT_MAX;
        const float* bias = p.ep.bias + nc;
#pragma unroll
        for (int j = 0; j < 32; j++) {
            const float y = __fadd_rn(__fmul_rn(__int2float_rn((int32_t)r[j]), comb), nc + j < p.N ? bias[j] : 0.0f);
            v[j] = __float_as_uint(p.ep.relu ? relu_arm(y) : max_nan(y, floor_v));
        }
    }
    uint32_t* my_row = stage + lane * 32;
#pragma unroll
    for (int c = 0; c < 8; c++)
        *reinterpret_cast<uint4*>(my_row + ((c ^ (lane & 7)) * 4)) =
            make_uint4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
    __syncwarp();
    const uint32_t cc = lane & 7;
    const uint32_t n = nc + 4 * cc;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const uint32_t rr = 4 * i + (lane >> 3);
        const uint4 val = *reinterpret_cast<const uint4*>(stage + rr * 32 + ((cc ^ (rr & 7)) * 4));
        const uint32_t m = row0 + rr;
        if (m < p.M && n < p.N) {
            for (uint32_t q = 0; q < (p.world > 1 ? p.world : 1u); q++) {
                uint32_t* out = reinterpret_cast<uint32_t*>(p.world > 1 ? p.C_rank[q] : p.C) + (size_t)m * p.ldc + n;
                if (p.vec_ok && n + 4 <= p.N) {
                    *reinterpret_cast<uint4*>(out) = val;
                } else {
                    out[0] = val.x;
                    if (n + 1 < p.N) out[1] = val.y;
                    if (n + 2 < p.N) out[2] = val.z;
                    if (n + 3 < p.N) out[3] = val.w;
                }
            }
        }
    }
    __syncwarp();
}

// Drains one 128-row x `ncols`-column TMEM accumulator of this CTA (warp = one lane
// quarter) and stores it.  Calls `release()` right after the last TMEM read.
template <class Release>
__device__ __forceinline__ void drain_accumulator(const Params& p, uint32_t taddr, uint32_t row0, uint32_t n0,
                                                  uint32_t ncols, uint32_t* stage, int lane, Release release) {
    const float comb = tile_comb(p);
    const int chunks = (int)(ncols / 32);
#pragma unroll 1
    for (int c = 0; c < chunks; c++) {
        uint32_t r[32];
        ptx::tmem_ld_32x32b_x32(taddr + c * 32, r);
        ptx::tmem_ld_wait();
        if (c == chunks - 1) {
            ptx::tc_fence_before();
            __syncwarp();
            release();
        }
        store_block(p, comb, r, stage, row0, n0 + c * 32, lane);
    }
}

// ------------------------------------------------------------ 1-CTA kernel
// BKN: B is given as the codes stored K x N (MN-major operand) instead of N x K.
// With an MN-major B a tile may be 128 or 64 columns wide (p.s_bn): for small
// M the 256-column tiles would leave most SMs idle, each busy one streaming the
// whole K alone.  128 columns: one SWIZZLE_128B box; 64: one SWIZZLE_64B box
// (tmap_b64).
template <bool BKN>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    gemm_s8_single_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                          const __grid_constant__ CUtensorMap tmap_b64, const Params p) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    // All A tiles first (stage i at i * s_a_bytes), then the B tiles.  The MMA
    // reads 128 A rows from each A tile; with fewer rows loaded the rest are
    // other stages' (or not yet written) bytes that only reach accumulator
    // rows >= M, which are never stored.  s_b_base leaves 16 KB after the last A
    // tile, so those reads stay inside the operand region.
    uint8_t* sa = smem;
    uint8_t* sb = smem + p.s_b_base;
    uint32_t* epi = reinterpret_cast<uint32_t*>(smem + (size_t)S_OPS);
    auto* bars = reinterpret_cast<Barriers<S_MAX_STAGES>*>(smem + (size_t)S_OPS + EPI_BYTES);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t num_tiles = p.tiles_m * p.tiles_n;
    const uint32_t nstages = p.s_stages;

    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < nstages; s++) {
            ptx::mbar_init(&bars->full[s], 1);
            ptx::mbar_init(&bars->empty[s], 1);
        }
        for (int a = 0; a < 2; a++) {
            ptx::mbar_init(&bars->tmem_full[a], 1);
            ptx::mbar_init(&bars->tmem_empty[a], 4);
        }
        ptx::fence_mbarrier_init();
        ptx::prefetch_tmap(&tmap_a);
        ptx::prefetch_tmap(BKN && p.s_bn == 64 ? &tmap_b64 : &tmap_b);
    }
    if (warp == 1) {
        ptx::tmem_alloc(&bars->tmem_base, TMEM_COLS);
        ptx::tmem_relinquish();
    }
    ptx::tc_fence_before();
    __syncthreads();
    ptx::tc_fence_after();
    const uint32_t tmem_base = bars->tmem_base;
    // programmatic dependent launch: the prologue above may overlap the previous
    // kernel on the stream; operands, scales and C are touched only after it ends
    ptx::griddep_launch_dependents();
    ptx::griddep_wait();

    if (warp == 0) {
        if (lane == 0) {
            uint32_t stage = 0, phase = 0;
            bool alive = true;
            const uint32_t bn = BKN ? p.s_bn : (uint32_t)S_BN;
            for (uint32_t t = blockIdx.x; t < num_tiles && alive; t += gridDim.x) {
                const int m0 = (int)((t / p.tiles_n) * S_BM), n0 = (int)((t % p.tiles_n) * bn);
                for (uint32_t kb = 0; kb < p.num_kb; kb++) {
                    if (!ptx::mbar_wait(&bars->empty[stage], phase ^ 1, p.err)) { alive = false; break; }
                    ptx::mbar_arrive_expect_tx(&bars->full[stage], p.s_a_bytes + p.s_b_bytes);
                    ptx::tma_load_2d(sa + (size_t)stage * p.s_a_bytes, &tmap_a, &bars->full[stage], (int)(kb * BK), m0);
                    if constexpr (BKN) {
                        if (bn == 64) {
                            ptx::tma_load_2d(sb + (size_t)stage * p.s_b_bytes, &tmap_b64, &bars->full[stage], n0,
                                             (int)(kb * BK));
                        } else {
                            // 128-column SWIZZLE_128B boxes, one N atom each (16 KB apart)
                            ptx::tma_load_2d(sb + (size_t)stage * p.s_b_bytes, &tmap_b, &bars->full[stage], n0,
                                             (int)(kb * BK));
                            if (bn == 256)
                                ptx::tma_load_2d(sb + (size_t)stage * p.s_b_bytes + kMnAtomBytes, &tmap_b, &bars->full[stage],
                                                 n0 + 128, (int)(kb * BK));
                        }
                    } else {
                        ptx::tma_load_2d(sb + (size_t)stage * p.s_b_bytes, &tmap_b, &bars->full[stage], (int)(kb * BK), n0);
                    }
                    if (++stage == nstages) { stage = 0; phase ^= 1; }
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            const uint32_t bn = BKN ? p.s_bn : (uint32_t)S_BN;
            const uint32_t brow = bn < 128 ? bn : 128u;  // bytes per K row of a B atom
            const uint32_t idesc = ptx::idesc_i8(S_BM, (int)bn, !p.ep.a_unsigned, !p.ep.b_unsigned) |
                                   (BKN ? ptx::kIdescBMnMajor : 0u);
            uint32_t stage = 0, phase = 0, acc = 0, acc_phase = 0;
            bool alive = true;
            for (uint32_t t = blockIdx.x; t < num_tiles && alive; t += gridDim.x) {
                if (!ptx::mbar_wait(&bars->tmem_empty[acc], acc_phase ^ 1, p.err)) break;
                ptx::tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * ACC_COLS;
                for (uint32_t kb = 0; kb < p.num_kb; kb++) {
                    if (!ptx::mbar_wait(&bars->full[stage], phase, p.err)) { alive = false; break; }
                    ptx::tc_fence_after();
                    const uint32_t a_addr = ptx::smem_u32(sa + (size_t)stage * p.s_a_bytes);
                    const uint32_t b_addr = ptx::smem_u32(sb + (size_t)stage * p.s_b_bytes);
#pragma unroll
                    for (int k = 0; k < BK / UMMA_K; k++) {
                        const uint64_t bdesc = BKN ? ptx::sdesc_mn(b_addr + k * UMMA_K * brow, brow, kMnAtomBytes)
                                                   : ptx::sdesc_kmajor_sw128(b_addr + k * UMMA_K);
                        ptx::umma_i8(d_tmem, ptx::sdesc_kmajor_sw128(a_addr + k * UMMA_K), bdesc, idesc,
                                     (kb | k) != 0);
                    }
                    ptx::umma_commit(&bars->empty[stage]);
                    if (++stage == nstages) { stage = 0; phase ^= 1; }
                }
                if (!alive) break;
                ptx::umma_commit(&bars->tmem_full[acc]);
                acc ^= 1;
                if (acc == 0) acc_phase ^= 1;
            }
        }
    } else {
        const uint32_t quarter = (uint32_t)(warp & 3);
        uint32_t* stage = epi + (warp - 2) * EPI_STAGE_WORDS;
        uint32_t acc = 0, acc_phase = 0;
        const uint32_t bn = BKN ? p.s_bn : (uint32_t)S_BN;
        for (uint32_t t = blockIdx.x; t < num_tiles; t += gridDim.x) {
            const uint32_t m0 = (t / p.tiles_n) * S_BM, n0 = (t % p.tiles_n) * bn;
            // one verdict per warp: no lane reaches the warp-wide tcgen05.ld alone
            if (!__all_sync(0xffffffffu, ptx::mbar_wait(&bars->tmem_full[acc], acc_phase, p.err))) break;
            ptx::tc_fence_after();
            const uint32_t taddr = tmem_base + ((quarter * 32) << 16) + acc * ACC_COLS;
            uint64_t* empty_bar = &bars->tmem_empty[acc];
            drain_accumulator(p, taddr, m0 + quarter * 32, n0, bn, stage, lane, [&] {
                if (lane == 0) ptx::mbar_arrive(empty_bar);
            });
            acc ^= 1;
            if (acc == 0) acc_phase ^= 1;
        }
    }

    ptx::tc_fence_before();
    __syncthreads();
    gather_signal(p);
    if (warp == 1) {
        ptx::tc_fence_after();
        ptx::tmem_dealloc(tmem_base, TMEM_COLS);
    }
}

// --------------------------------------------------------- CTA-pair kernel
// BKN: B is given as the codes stored K x N (MN-major operand).  Then each CTA's
// B half of a unit (`half` = 128, 64 or 32 columns) is one TMA box of `half`
// columns x BK rows with the swizzle of that width: tmap_b, tmap_b64, tmap_b32.
// Without BKN, tmap_b holds 128-row K-major boxes and tmap_b32 32-row ones.
template <bool BKN>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    gemm_s8_pair_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                        const __grid_constant__ CUtensorMap tmap_b64, const __grid_constant__ CUtensorMap tmap_b32,
                        const Params p) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sa = smem;
    uint8_t* sb = smem + (size_t)P_STAGES * P_A;
    uint32_t* epi = reinterpret_cast<uint32_t*>(smem + (size_t)P_STAGES * P_STAGE);
    auto* bars = reinterpret_cast<Barriers<P_STAGES>*>(smem + (size_t)P_STAGES * P_STAGE + EPI_BYTES);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = ptx::cluster_ctarank();  // 0 = leader (issues the MMAs)
    const uint32_t pair = blockIdx.x >> 1, num_pairs = gridDim.x >> 1;
    const uint32_t num_units = p.num_units;

    if (threadIdx.x == 0) {
        for (int s = 0; s < P_STAGES; s++) {
            ptx::mbar_init(&bars->full[s], 1);   // leader's producer arrive (+ tx of both CTAs)
            ptx::mbar_init(&bars->empty[s], 1);  // one multicast commit per CTA
        }
        for (int a = 0; a < 2; a++) {
            ptx::mbar_init(&bars->tmem_full[a], 1);
            ptx::mbar_init(&bars->tmem_empty[a], 8);  // 4 epilogue warps x 2 CTAs (leader's copy is used)
        }
        ptx::fence_mbarrier_init();
        ptx::prefetch_tmap(&tmap_a);
        ptx::prefetch_tmap(&tmap_b);
        if (p.split > 1) ptx::prefetch_tmap(&tmap_b32);
        if (BKN && p.split > 1) ptx::prefetch_tmap(&tmap_b64);
    }
    if (warp == 1) {
        ptx::tmem_alloc_cg2(&bars->tmem_base, TMEM_COLS);
        ptx::tmem_relinquish_cg2();
    }
    ptx::tc_fence_before();
    ptx::cluster_sync();
    ptx::tc_fence_after();
    const uint32_t tmem_base = bars->tmem_base;
    // programmatic dependent launch: the prologue above may overlap the previous
    // kernel on the stream; operands, scales and C are touched only after it ends
    ptx::griddep_launch_dependents();
    ptx::griddep_wait();

    if (warp == 0) {
        if (lane == 0) {
            uint32_t stage = 0, phase = 0;
            bool alive = true;
            for (uint32_t u = pair; u < num_units && alive; u += num_pairs) {
                const PairUnit un = pair_unit(p, u);
                if (un.n0 >= p.N) continue;  // a split part entirely right of N (all roles skip it)
                const uint32_t half = un.ncols / 2;  // B rows this CTA supplies
                const int m0 = (int)(un.m0 + rank * P_HM);
                const int n0 = (int)(un.n0 + rank * half);
                const uint32_t tx = 2 * (P_A + half * BK);
                for (uint32_t kb = 0; kb < p.num_kb; kb++) {
                    if (!ptx::mbar_wait(&bars->empty[stage], phase ^ 1, p.err)) { alive = false; break; }
                    if (rank == 0) ptx::mbar_arrive_expect_tx(&bars->full[stage], tx);
                    const uint32_t full_leader = ptx::mapa_shared(ptx::smem_u32(&bars->full[stage]), 0);
                    ptx::tma_load_2d_cg2(sa + (size_t)stage * P_A, &tmap_a, full_leader, (int)(kb * BK), m0);
                    if constexpr (BKN) {
                        const CUtensorMap* bm = half == P_HN ? &tmap_b : half == 64 ? &tmap_b64 : &tmap_b32;
                        ptx::tma_load_2d_cg2(sb + (size_t)stage * P_B, bm, full_leader, n0, (int)(kb * BK));
                    } else if (half == P_HN) {
                        ptx::tma_load_2d_cg2(sb + (size_t)stage * P_B, &tmap_b, full_leader, (int)(kb * BK), n0);
                    } else {
                        // 32-row boxes, each 4 KB apart: the same SWIZZLE_128B image as one taller box
                        for (uint32_t r = 0; r < half; r += 32)
                            ptx::tma_load_2d_cg2(sb + (size_t)stage * P_B + r * BK, &tmap_b32, full_leader,
                                                 (int)(kb * BK), n0 + (int)r);
                    }
                    if (++stage == P_STAGES) { stage = 0; phase ^= 1; }
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && rank == 0) {
            uint32_t stage = 0, phase = 0, acc = 0, acc_phase = 0;
            bool alive = true;
            for (uint32_t u = pair; u < num_units && alive; u += num_pairs) {
                const PairUnit un = pair_unit(p, u);
                if (un.n0 >= p.N) continue;
                const uint32_t idesc = ptx::idesc_i8(P_BM, (int)un.ncols, !p.ep.a_unsigned, !p.ep.b_unsigned) |
                                       (BKN ? ptx::kIdescBMnMajor : 0u);
                const uint32_t half = un.ncols / 2;  // B columns (MN-major row bytes) per CTA
                if (!ptx::mbar_wait(&bars->tmem_empty[acc], acc_phase ^ 1, p.err)) break;
                ptx::tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * ACC_COLS;
                for (uint32_t kb = 0; kb < p.num_kb; kb++) {
                    if (!ptx::mbar_wait(&bars->full[stage], phase, p.err)) { alive = false; break; }
                    ptx::tc_fence_after();
                    const uint32_t a_addr = ptx::smem_u32(sa + (size_t)stage * P_A);
                    const uint32_t b_addr = ptx::smem_u32(sb + (size_t)stage * P_B);
#pragma unroll
                    for (int k = 0; k < BK / UMMA_K; k++) {
                        const uint64_t bdesc = BKN ? ptx::sdesc_mn(b_addr + k * UMMA_K * half, half, kMnAtomBytes)
                                                   : ptx::sdesc_kmajor_sw128(b_addr + k * UMMA_K);
                        ptx::umma_i8_cg2(d_tmem, ptx::sdesc_kmajor_sw128(a_addr + k * UMMA_K), bdesc, idesc,
                                         (kb | k) != 0);
                    }
                    ptx::umma_commit_cg2_mc(&bars->empty[stage], 0x3);  // frees the stage in both CTAs
                    if (++stage == P_STAGES) { stage = 0; phase ^= 1; }
                }
                if (!alive) break;
                ptx::umma_commit_cg2_mc(&bars->tmem_full[acc], 0x3);
                acc ^= 1;
                if (acc == 0) acc_phase ^= 1;
            }
        }
    } else {
        const uint32_t quarter = (uint32_t)(warp & 3);
        uint32_t* stage = epi + (warp - 2) * EPI_STAGE_WORDS;
        uint32_t acc = 0, acc_phase = 0;
        for (uint32_t u = pair; u < num_units; u += num_pairs) {
            const PairUnit un = pair_unit(p, u);
            if (un.n0 >= p.N) continue;
            const uint32_t m0 = un.m0 + rank * P_HM;
            // one verdict per warp: no lane reaches the warp-wide tcgen05.ld alone
            if (!__all_sync(0xffffffffu, ptx::mbar_wait(&bars->tmem_full[acc], acc_phase, p.err))) break;
            ptx::tc_fence_after();
            const uint32_t taddr = tmem_base + ((quarter * 32) << 16) + acc * ACC_COLS;
            const uint32_t empty_leader = ptx::mapa_shared(ptx::smem_u32(&bars->tmem_empty[acc]), 0);
            drain_accumulator(p, taddr, m0 + quarter * 32, un.n0, un.ncols, stage, lane, [&] {
                if (lane == 0) ptx::mbar_arrive_cluster(empty_leader);
            });
            acc ^= 1;
            if (acc == 0) acc_phase ^= 1;
        }
    }

    // Both CTAs are done with TMEM and with each other's shared memory only when
    // every role of both has finished.
    ptx::tc_fence_before();
    ptx::cluster_sync();
    gather_signal(p);
    if (warp == 1) {
        ptx::tc_fence_after();
        ptx::tmem_dealloc_cg2(tmem_base, TMEM_COLS);
    }
}

// Fills C with the epilogue of an all-zero accumulator (K == 0).
__global__ void fill_zero_k_kernel(uint32_t M, uint32_t N, void* C, size_t ldc, GemmEpilogue ep) {
    const size_t total = (size_t)M * N;
    float comb = 0.0f;
    if (ep.mode != kOutRawI32) {
        const float s0 = ep.scales ? ep.scales[0] : ep.sa_imm;
        const float s1 = ep.scales ? ep.scales[1] : ep.sb_imm;
        comb = __fmul_rn(s0, s1);
    }
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const uint32_t m = (uint32_t)(i / N), n = (uint32_t)(i % N);
        if (ep.mode == kOutRawI32) {
            reinterpret_cast<int32_t*>(C)[(size_t)m * ldc + n] = 0;
            continue;
        }
        if (ep.mode == kOutIntGemm) {
            float* c = reinterpret_cast<float*>(C) + (size_t)m * ldc + n;
            const uint32_t a = __float_as_uint(ep.beta) != 0u ? __float_as_uint(__fmul_rn(*c, ep.beta)) : 0u;
            const float f = ep.acc_unsigned ? __uint2float_rn(a) : __int2float_rn((int32_t)a);
            *c = __fmul_rn(f, ep.alpha);
            continue;
        }
        float y = __fmul_rn(0.0f, comb);
        if (ep.mode == kOutDenseI8) {
            y = arm_fmax(__fadd_rn(y, ep.bias[n]), ep.relu ? 0.0f : -FLT_MAX);
        } else {
            y = __fmul_rn(y, ep.scale);
            if (ep.relu) y = arm_fmax(y, 0.0f);
        }
        reinterpret_cast<float*>(C)[(size_t)m * ldc + n] = y;
    }
}

// K-major int8 operand: `rows` x K (row stride K bytes), box = box_rows x BK.
int make_kmajor_map(CUtensorMap* map, const int8_t* base, uint32_t rows, uint32_t K, uint32_t box_rows) {
    return encode_tensor_map_2d(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, base, K, rows, K, BK, box_rows,
                                CU_TENSOR_MAP_SWIZZLE_128B);
}
// MN-major int8 operand (B codes K x N, row stride ldb bytes), box = `cols`
// (128, 64 or 32) x BK rows with the swizzle of that width.  Rows past `rows`
// and columns past N read as zero.
int make_mn_map(CUtensorMap* map, const int8_t* base, uint32_t N, uint32_t rows, size_t ldb, uint32_t cols) {
    const CUtensorMapSwizzle sw = cols == 128  ? CU_TENSOR_MAP_SWIZZLE_128B
                                  : cols == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                               : CU_TENSOR_MAP_SWIZZLE_32B;
    return encode_tensor_map_2d(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, base, N, rows, ldb, cols, BK, sw);
}

// B operand of one launch: Bt (N x K, K-major) or Bq (K x N, row stride ldb).
struct BOperand {
    const int8_t* ptr;
    size_t ldb;      // Bq: row stride in bytes (multiple of 16)
};

template <bool BKN>
int launch_gemm_impl(uint32_t M, uint32_t N, uint32_t K, const int8_t* Aq, const BOperand& bop, void* C, size_t ldc,
                     const GemmEpilogue& ep, cudaStream_t s, const GatherArgs* gather, uint32_t* grid_out) {
    const int8_t* Bt = bop.ptr;
    if (M == 0 || N == 0) return ANE_OK;
    if (K == 0) return launch_fill_epilogue_zero_k(M, N, C, ldc, ep, s);
    ANE_ARG_CHECK(K % 16 == 0, "gemm: K must be a multiple of 16 (TMA row stride)");
    ANE_ARG_CHECK((reinterpret_cast<uintptr_t>(Aq) & 15) == 0 && (reinterpret_cast<uintptr_t>(Bt) & 15) == 0,
                  "gemm: int8 operands must be 16-byte aligned");
    ANE_ARG_CHECK(!BKN || (bop.ldb % 16 == 0 && bop.ldb >= N),
                  "gemm: B stored K x N needs a row stride that is a multiple of 16 and >= N");
    Params p;
    p.M = M;
    p.N = N;
    p.K = K;
    p.num_kb = (K + BK - 1) / BK;
    p.C = C;
    p.ldc = ldc;
    p.vec_ok = (ldc % 4 == 0) && ((reinterpret_cast<uintptr_t>(C) & 15) == 0);
    p.ep = ep;
    p.err = device_timeout_flag();
    p.world = 1;
    p.tail_start = p.split = p.num_units = 0;
    if (gather && gather->world > 1) {
        ANE_ARG_CHECK(gather->world <= kGatherMaxRanks, "gemm gather: at most 8 ranks");
        p.world = gather->world;
        bool aligned = (ldc % 4 == 0);
        for (uint32_t q = 0; q < p.world; q++) {
            ANE_ARG_CHECK(gather->C_rank[q] && gather->ctr_rank[q], "gemm gather: NULL peer pointer");
            p.C_rank[q] = gather->C_rank[q];
            p.ctr_rank[q] = gather->ctr_rank[q];
            aligned = aligned && ((reinterpret_cast<uintptr_t>(gather->C_rank[q]) & 15) == 0);
        }
        p.vec_ok = aligned;
    }
    const int sms = num_sms();
    // ANE_GEMM_KERNEL=single|pair overrides the shape-based choice (tuning aid).
    static const char* force = getenv("ANE_GEMM_KERNEL");
    bool pair = M > (uint32_t)S_BM;
    if (force && !strcmp(force, "single")) pair = false;
    if (force && !strcmp(force, "pair")) pair = true;
    CUtensorMap ta, tb;
    const uint32_t s_am = M >= (uint32_t)S_BM ? (uint32_t)S_BM : (M + 7) / 8 * 8;  // 1-CTA kernel: A rows per stage
    int rc = make_kmajor_map(&ta, Aq, M, K, pair ? P_HM : s_am);
    if (rc) return rc;
    rc = BKN ? make_mn_map(&tb, Bt, N, K, bop.ldb, 128) : make_kmajor_map(&tb, Bt, N, K, pair ? P_HN : S_BN);
    if (rc) return rc;
    if (!pair) {
        static std::atomic<uint64_t> smem_set{0};  // devices whose limit is raised
        rc = set_max_dynamic_smem(gemm_s8_single_kernel<BKN>, (int)S_SMEM, smem_set);
        if (rc) return rc;
        p.tiles_m = (M + S_BM - 1) / S_BM;
        // MN-major B: the tile width (256, 128 or 64 columns) with the fewest
        // waves x width, ties to the wider tile (fewer tiles)
        p.s_bn = S_BN;
        if (BKN) {
            uint64_t best = ~0ull;
            for (uint32_t bn : {256u, 128u, 64u}) {
                const uint64_t tiles = (uint64_t)p.tiles_m * ((N + bn - 1) / bn);
                const uint64_t cost = (tiles + sms - 1) / sms * bn;
                if (cost < best) {
                    best = cost;
                    p.s_bn = bn;
                }
            }
        }
        p.tiles_n = (N + p.s_bn - 1) / p.s_bn;
        // the ring: as many stages (<= S_MAX_STAGES) as the operand region holds
        // with the A tiles first and 16 KB of room after the last one
        p.s_am = s_am;
        p.s_a_bytes = s_am * BK;
        p.s_b_bytes = p.s_bn * BK;
        p.s_stages = S_STAGES;  // the full-size plan, which always fits
        p.s_b_base = S_STAGES * S_A;
        for (uint32_t st = S_MAX_STAGES; st >= 2; st--) {
            const uint32_t a_end = (st - 1) * p.s_a_bytes + (uint32_t)S_A;
            const uint32_t base = ((a_end > st * p.s_a_bytes ? a_end : st * p.s_a_bytes) + 1023) / 1024 * 1024;
            if (base + st * p.s_b_bytes <= (uint32_t)S_OPS) {
                p.s_stages = st;
                p.s_b_base = base;
                break;
            }
        }
        CUtensorMap tb64 = tb;
        if (BKN && p.s_bn == 64) {
            rc = make_mn_map(&tb64, Bt, N, K, bop.ldb, 64);
            if (rc) return rc;
        }
        const uint32_t tiles = p.tiles_m * p.tiles_n;
        const uint32_t grid = tiles < (uint32_t)sms ? tiles : (uint32_t)sms;
        if (grid_out) *grid_out = grid;
        return launch_pdl(gemm_s8_single_kernel<BKN>, dim3(grid), dim3(NUM_THREADS), S_SMEM, s, ta, tb, tb64, p);
    }
    static std::atomic<uint64_t> smem_set2{0};
    rc = set_max_dynamic_smem(gemm_s8_pair_kernel<BKN>, (int)P_SMEM, smem_set2);
    if (rc) return rc;
    p.tiles_m = (M + P_BM - 1) / P_BM;
    p.tiles_n = (N + P_BN - 1) / P_BN;
    const uint32_t tiles = p.tiles_m * p.tiles_n;
    uint32_t pairs = (uint32_t)sms / 2;
    // Last partial wave: r leftover tiles would keep r pairs busy for a whole
    // tile while the rest idle.  Cutting each into s = 2 or 4 column parts
    // (s*r <= pairs) ends that wave after 1/s of a tile.  Every part runs the
    // full K, so no partial sums are combined.  ANE_GEMM_TAIL_SPLIT=0 turns it off.
    p.tail_start = tiles;
    p.split = 1;
    static const bool tail_split = [] {
        const char* v = getenv("ANE_GEMM_TAIL_SPLIT");
        return !(v && v[0] == '0');
    }();
    const uint32_t r = tiles % pairs;
    if (tail_split && r != 0) {
        const uint32_t sp = pairs / r >= 4 ? 4u : pairs / r >= 2 ? 2u : 1u;
        if (sp > 1) {
            p.tail_start = tiles - r;
            p.split = sp;
        }
    }
    p.num_units = p.tail_start + p.split * (tiles - p.tail_start);
    if (pairs > p.num_units) pairs = p.num_units;
    if (grid_out) *grid_out = 2 * pairs;
    CUtensorMap tb64 = tb, tb32 = tb;  // unused unless the tail is split
    if (p.split > 1) {
        if (BKN) {
            rc = make_mn_map(&tb64, Bt, N, K, bop.ldb, 64);
            if (rc) return rc;
            rc = make_mn_map(&tb32, Bt, N, K, bop.ldb, 32);
        } else {
            rc = make_kmajor_map(&tb32, Bt, N, K, 32);
        }
        if (rc) return rc;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * pairs, 1, 1);
    cfg.blockDim = dim3(NUM_THREADS, 1, 1);
    cfg.dynamicSmemBytes = P_SMEM;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 2 : 1;
    ANE_CUDA_TRY(cudaLaunchKernelEx(&cfg, gemm_s8_pair_kernel<BKN>, ta, tb, tb64, tb32, p));
    ANE_CHECK_LAUNCH();
    return ANE_OK;
}

}  // namespace

int launch_gemm_s8_tc(uint32_t M, uint32_t N, uint32_t K, const int8_t* Aq, const int8_t* Bt, void* C, size_t ldc,
                      const GemmEpilogue& ep, cudaStream_t s, const GatherArgs* gather, uint32_t* grid_out) {
    const BOperand b{Bt, 0};
    return launch_gemm_impl<false>(M, N, K, Aq, b, C, ldc, ep, s, gather, grid_out);
}

int launch_gemm_s8_tc_kn(uint32_t M, uint32_t N, uint32_t K, const int8_t* Aq, const int8_t* Bq, size_t ldb,
                         void* C, size_t ldc, const GemmEpilogue& ep, cudaStream_t s, const GatherArgs* gather,
                         uint32_t* grid_out) {
    const BOperand b{Bq, ldb};
    return launch_gemm_impl<true>(M, N, K, Aq, b, C, ldc, ep, s, gather, grid_out);
}

// Fused all-gather, receiving side: one thread waits (bounded) until every CTA
// of every rank has published this call's rows to this GPU, then bumps the
// call count.  Counters only grow: call e needs (e + 1) x per_call arrivals.
__global__ void gather_wait_kernel(const uint32_t* ctr, uint32_t* epoch, uint32_t per_call, int* err) {
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    const uint32_t target = (*reinterpret_cast<volatile uint32_t*>(epoch) + 1u) * per_call;
    const long long t0 = clock64();
    while (true) {
        uint32_t v;
        asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(ctr) : "memory");
        if ((int32_t)(v - target) >= 0) break;
        if (clock64() - t0 > ptx::kWaitTimeoutCycles) {
            atomicAdd(err, 1);
            break;
        }
        __nanosleep(100);
    }
    *epoch += 1u;
}

int launch_gather_wait(const uint32_t* ctr, uint32_t* epoch, uint32_t per_call, cudaStream_t s) {
    gather_wait_kernel<<<1, 32, 0, s>>>(ctr, epoch, per_call, device_timeout_flag());
    ANE_CHECK_LAUNCH();
    return ANE_OK;
}

int launch_fill_epilogue_zero_k(uint32_t M, uint32_t N, void* C, size_t ldc, const GemmEpilogue& ep, cudaStream_t s) {
    const size_t total = (size_t)M * N;
    if (total == 0) return ANE_OK;
    int g = (int)ceil_div(total, 256 * 4);
    if (g > num_sms() * 4) g = num_sms() * 4;
    fill_zero_k_kernel<<<g, 256, 0, s>>>(M, N, C, ldc, ep);
    ANE_CHECK_LAUNCH();
    return ANE_OK;
}

}  // namespace ane_b200
