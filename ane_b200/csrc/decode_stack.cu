// decode_stack.cu -- a whole Q8_0 decode step (a chain of Q8_0 x Q8_0
// projections, ggml MUL_MAT at batch 1) in ONE persistent cooperative launch,
// row-sharded over up to 8 GPUs with the all-gather fused into the epilogue.
//
// Per CTA (one per SM): warp 0 streams the weight rows of every projection, in
// order, through the shared-memory TMA ring (the same 4-row x 544-byte boxes as
// the one-projection kernel, q8_stream.cuh); it never waits for activations, so
// HBM keeps streaming across projection boundaries.  Compute warps, per
// projection j:
//   1. read x and quantize it to Q8_0 in shared memory (q8_mmq.cuh, the ggml
//      rule).  x is either a plain fp32 vector (a layer input) or the previous
//      projection's output in TAGGED form (below): the reader spins (bounded)
//      on each element until its tag is projection j-1's.  CTAs without rows
//      in projection j skip it;
//   2. compute this CTA's rows (q8_mmq.cuh: exact int32 block dots, the same
//      fp32 order as the one-projection kernel);
//   3. store each row result into EVERY rank's output vector as one 8-byte
//      {value, tag} word -- over NVLink to CUDA-IPC mapped peer memory for the
//      other ranks (plain stores; no multicast, no TMA on peer memory).
// Tagged words (the low-latency protocol NCCL calls LL): an aligned 8-byte
// store is seen whole or not at all, so a reader that sees the expected tag
// has the value, with no fence, flag or counter round trip.  tag = e*nproj +
// j + 1, e = this GPU's count of finished launches (bumped by its last CTA), so
// stale words from earlier projections or launches never match.  Overwrite
// hazards: projection j writes the vector projection j-1 read.  Only CTAs with
// rows in a projection read its input, and each of them does so before it
// publishes its first row, so before its first store of projection j a CTA
// checks one word per (rank, CTA) row range of projection j-1 (at most 8 x 148
// words, loaded at the start of the projection).  All spins are bounded (~2 s)
// and record a device timeout; a timed-out CTA stops at the next common point.
// A launch returns only after every word of the gathered last output carries
// its tag on this GPU.
#include <cstring>
#include <string>
#include <vector>

#include "ane_internal.cuh"
#include "q8_mmq.cuh"
#include "q8_stream.cuh"
#include "sm100_ptx.cuh"

namespace ane_b200 {

constexpr uint32_t kStackMaxRanks = 8;
constexpr uint32_t kStackWarps = 15;  // compute warps per CTA: 16 warps in all, so 128 registers each

struct alignas(64) StackProj {
    CUtensorMap wmap;               // this rank's rows of W as a 2-D uint32 tensor
    const void* x;                  // fp32[K], or K tagged words (x_tagged)
    uint2* out[kStackMaxRanks];     // per rank: this rank's first row in that rank's tagged output vector
    const uint2* out_all;           // this rank's tagged output vector (all ranks' rows), word 0
    uint32_t rows, K, groups, x_tagged;
};

namespace {

// A tagged word is ONE 64-bit scalar access (value in the low half, tag in the
// high half): a 32-bit vector pair may reach a peer GPU as two writes, which a
// reader could see half updated.
__device__ __forceinline__ uint2 split(uint64_t w) { return make_uint2((uint32_t)w, (uint32_t)(w >> 32)); }
// Two tagged words (16 bytes) as two 64-bit elements.
__device__ __forceinline__ uint4 ld_word2(const uint2* p) {
    uint64_t a, b;
    asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
    const uint2 x = split(a), y = split(b);
    return make_uint4(x.x, x.y, y.x, y.y);
}
__device__ __forceinline__ uint2 ld_word(const uint2* p) {
    uint64_t a;
    asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(a) : "l"(p) : "memory");
    return split(a);
}
__device__ __forceinline__ void st_word(uint2* p, float value, uint32_t tag) {
    const uint64_t w = (uint64_t)__float_as_uint(value) | ((uint64_t)tag << 32);
    asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
// Spins until *p carries `tag`; returns the value (0 and *dead = true on timeout).
__device__ __forceinline__ float wait_word(const uint2* p, uint32_t tag, bool* dead, int* err) {
    uint2 v = ld_word(p);
    if (v.y == tag) return __uint_as_float(v.x);
    const long long t0 = clock64();
    while (true) {
        __nanosleep(32);
        v = ld_word(p);
        if (v.y == tag) return __uint_as_float(v.x);
        if (clock64() - t0 > ptx::kWaitTimeoutCycles) {
            atomicAdd(err, 1);
            *dead = true;
            return 0.0f;
        }
    }
}

__global__ void __launch_bounds__(32 * (kStackWarps + 1), 1)
    decode_stack_kernel(const StackProj* __restrict__ projs, uint32_t nproj, uint32_t world, uint32_t* ctl,
                        uint32_t nslots, uint32_t kmax, int* err) {
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr uint32_t nw = kStackWarps;
    __shared__ uint32_t epoch_s;
    __shared__ int dead_s;
    const uint32_t G = gridDim.x, c = blockIdx.x;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    uint64_t* empty = full + nslots;
    int8_t* xs = reinterpret_cast<int8_t*>(smem + 128);
    float* xd = reinterpret_cast<float*>(smem + 128 + round_up(kmax, 128));
    uint8_t* ring = smem + 128 + round_up(kmax, 128) + round_up(kmax / 32 * 4, 128);
    const uint32_t slot_bytes = nw * kQ8WarpTileBytes;
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < nslots; s++) {
            ptx::mbar_init(&full[s], 1);
            ptx::mbar_init(&empty[s], nw);
        }
        ptx::fence_mbarrier_init();
        epoch_s = *reinterpret_cast<volatile uint32_t*>(ctl);
        dead_s = 0;
    }
    __syncthreads();
    const uint32_t epoch = epoch_s;
    auto tag_of = [&](uint32_t e, uint32_t j) { return e * nproj + j + 1u; };

    if (warp == 0) {
        // ------------------------------------------------------ weight stream
        if (lane == 0) {
            uint32_t t = 0;
            bool alive = true;
            for (uint32_t j = 0; j < nproj && alive; j++) {
                const StackProj* P = projs + j;
                ptx::prefetch_tmap(&P->wmap);
                const uint32_t groups = P->groups;
                const uint32_t g0 = (uint32_t)((uint64_t)groups * c / G), g1 = (uint32_t)((uint64_t)groups * (c + 1) / G);
                const uint32_t npass = (g1 - g0 + nw - 1) / nw;
                const uint32_t nchunks = (P->K / 32 + kQ8ChunkBlocks - 1) / kQ8ChunkBlocks;
                for (uint32_t pass = 0; pass < npass && alive; pass++) {
                    // the pass's (chunk, group) tiles in chunk-major order, nw tiles
                    // per stage: every stage is full whatever the pass's group count
                    const uint32_t gp = g0 + pass * nw, nwp = min(nw, g1 - gp);
                    const uint32_t ntiles = nwp * nchunks, nst = (ntiles + nw - 1) / nw;
                    for (uint32_t st = 0; st < nst; st++, t++) {
                        const uint32_t slot = t % nslots;
                        if (!ptx::mbar_wait(&empty[slot], ((t / nslots) & 1) ^ 1, err)) {
                            alive = false;
                            break;
                        }
                        const uint32_t i0 = st * nw, n = min(nw, ntiles - i0);
                        uint8_t* dst = ring + (size_t)slot * slot_bytes;
                        ptx::mbar_arrive_expect_tx(&full[slot], n * kQ8WarpTileBytes);
                        for (uint32_t k = 0; k < n; k++) {
                            const uint32_t ch = (i0 + k) / nwp, w = i0 + k - ch * nwp;
                            ptx::tma_load_2d(dst + k * kQ8WarpTileBytes, &P->wmap, &full[slot],
                                             (int)(ch * (kQ8ChunkBytes / 4)), (int)((gp + w) * kQ8RowsPerWarp));
                        }
                        // a stage is freed by one arrival per tile: those it does not hold
                        if (n < nw) ptx::mbar_arrive_cnt(&empty[slot], nw - n);
                    }
                }
            }
        }
        return;
    }

    // ------------------------------------------------------------ compute
    const uint32_t cw = warp - 1, r = lane & 3, pp = lane >> 2;
    const uint32_t ct = threadIdx.x - 32;  // compute thread 0 .. nw*32-1
    uint32_t t = 0;
    bool dead = false;  // this warp met a timeout: it skips work but keeps the barrier schedule
    constexpr uint32_t kGuards = (kStackMaxRanks * 256 + nw * 32 - 1) / (nw * 32);  // guard words per thread
    for (uint32_t j = 0; j < nproj; j++) {
        const StackProj* P = projs + j;
        const uint32_t K = P->K, nb = K / 32, nchunks = (nb + kQ8ChunkBlocks - 1) / kQ8ChunkBlocks;
        const uint32_t tag = tag_of(epoch, j);
        const uint32_t groups = P->groups, rows = P->rows;
        const uint32_t g0 = (uint32_t)((uint64_t)groups * c / G), g1 = (uint32_t)((uint64_t)groups * (c + 1) / G);
        const uint32_t npass = (g1 - g0 + nw - 1) / nw;
        // 0. guard: projection j overwrites the vector that projection j-1 (of this
        //    launch, or the last one of the previous launch) read.  Every (rank, CTA)
        //    with rows in j-1 read its input before publishing its first row, so
        //    one word per such row range with j-1's tag proves the vector is free.
        //    Loads are issued now; words not there yet are read again in the same
        //    rounds as the activation's (one round trip per round for both).
        const bool guard = npass > 0 && (j > 0 || epoch > 0);
        const StackProj* Q = projs + (j ? j - 1 : nproj - 1);
        const uint32_t qtag = j ? tag_of(epoch, j - 1) : tag_of(epoch - 1, nproj - 1);
        const uint2* gptr[kGuards];
        uint2 gval[kGuards];
#pragma unroll
        for (uint32_t k = 0; k < kGuards; k++) {
            gptr[k] = nullptr;
            const uint32_t idx = ct + k * nw * 32;
            if (guard && idx < world * G) {
                const uint32_t rq = idx / G, cq = idx - rq * G;
                const uint32_t q0 = (uint32_t)((uint64_t)Q->groups * cq / G);
                const uint32_t q1 = (uint32_t)((uint64_t)Q->groups * (cq + 1) / G);
                if (q1 > q0) {
                    gptr[k] = Q->out_all + (size_t)rq * Q->rows + q0 * kQ8RowsPerWarp;
                    gval[k] = ld_word(gptr[k]);
                }
            }
        }
        bool gchecked = false;
        uint32_t gmiss = 0;  // guard words still without j-1's tag
        auto guard_miss = [&]() {
            uint32_t m = 0;
#pragma unroll
            for (uint32_t k = 0; k < kGuards; k++)
                if (gptr[k] && gval[k].y != qtag) m |= 1u << k;
            return m;
        };
        auto guard_round = [&](uint32_t m) {
#pragma unroll
            for (uint32_t k = 0; k < kGuards; k++)
                if ((m >> k) & 1u)
                    if (ld_word(gptr[k]).y == qtag) m &= ~(1u << k);
            return m;
        };
        // 1. activation -> Q8_0 codes + scales in shared memory (one thread per
        //    block); a CTA without rows in this projection does not read it
        if (!dead && npass > 0) {
            if (P->x_tagged) {
                const uint2* xw = reinterpret_cast<const uint2*>(P->x);
                const uint32_t want = tag_of(epoch, j - 1);
                for (uint32_t b = ct; b < nb && !dead; b += nw * 32) {
                    // all 16 loads of the block in flight at once; the pairs not yet
                    // published are read again together, one round trip per round
                    // (a CTA that finished the last projection early reads words
                    // other CTAs are still computing), bounded
                    const uint2* blk = xw + (size_t)b * 32;
                    float v[32];
                    uint32_t miss = 0;
#pragma unroll
                    for (int k = 0; k < 16; k++) {
                        const uint4 w = ld_word2(blk + 2 * k);
                        v[2 * k] = __uint_as_float(w.x);
                        v[2 * k + 1] = __uint_as_float(w.z);
                        miss |= (w.y != want || w.w != want) ? 1u << k : 0u;
                    }
                    if (!gchecked) {
                        gmiss = guard_miss();
                        gchecked = true;
                    }
                    const long long t0 = (miss | gmiss) ? clock64() : 0;
                    while (miss | gmiss) {
                        if (clock64() - t0 > ptx::kWaitTimeoutCycles) {
                            atomicAdd(err, 1);
                            dead = true;
                            break;
                        }
                        __nanosleep(64);
#pragma unroll
                        for (int k = 0; k < 16; k++) {
                            if (!((miss >> k) & 1u)) continue;
                            const uint4 w = ld_word2(blk + 2 * k);
                            if (w.y == want && w.w == want) {
                                v[2 * k] = __uint_as_float(w.x);
                                v[2 * k + 1] = __uint_as_float(w.z);
                                miss &= ~(1u << k);
                            }
                        }
                        gmiss = guard_round(gmiss);
                    }
                    if (!dead) q8_quantize_regs(v, xs, xd, b);
                }
            } else {
                for (uint32_t b = ct; b < nb; b += nw * 32)
                    q8_quantize_block<true>(reinterpret_cast<const float*>(P->x) + (size_t)b * 32, xs, xd, b);
            }
        }
        // threads without an activation block: their guard words alone
        if (!gchecked) gmiss = guard_miss();
        if (!dead && gmiss) {
            const long long t0 = clock64();
            while (gmiss) {
                if (clock64() - t0 > ptx::kWaitTimeoutCycles) {
                    atomicAdd(err, 1);
                    dead = true;
                    break;
                }
                __nanosleep(64);
                gmiss = guard_round(gmiss);
            }
        }
        if (dead) dead_s = 1;
        __syncwarp();
        ptx::named_barrier_sync(1, nw * 32);
        if (dead_s) dead = true;
        // 2. this CTA's rows: ring stages in the producer's order
        for (uint32_t pass = 0; pass < npass; pass++) {
            const uint32_t gp = g0 + pass * nw, nwp = min(nw, g1 - gp);
            const uint32_t nst = (nwp * nchunks + nw - 1) / nw;  // the producer's stages
            const uint32_t row = (gp + cw) * kQ8RowsPerWarp + r;
            float sum = 0.f;
            if (cw < nwp && !dead) {
                // this warp's tiles are cw, cw + nwp, cw + 2 nwp, ... (its chunks in
                // order); two per step, so the second's loads and block dots run
                // alongside the first's (each lane still adds its terms in block order)
                uint32_t wslot = t % nslots, wphase = (t / nslots) & 1u;  // next stage to wait for
                uint32_t waited = 0, aslot = wslot, astage = 0;           // aslot: slot of stage astage
                const uint32_t lane_off = r * kQ8ChunkBytes + pp * 68;
                for (uint32_t ch = 0; ch < nchunks; ch += 2) {
                    const bool two = ch + 1 < nchunks;
                    const uint32_t i0 = ch * nwp + cw, i1 = i0 + nwp;
                    const uint32_t s0 = i0 / nw, s1 = two ? i1 / nw : s0;
                    while (waited <= s1 && !dead) {
                        if (!ptx::mbar_wait(&full[wslot], wphase, err)) dead = true;
                        waited++;
                        if (++wslot == nslots) {
                            wslot = 0;
                            wphase ^= 1u;
                        }
                    }
                    if (dead) break;
                    while (astage < s0) {
                        astage++;
                        aslot = aslot + 1 == nslots ? 0u : aslot + 1;
                    }
                    const uint32_t bslot = s1 == s0 ? aslot : (aslot + 1 == nslots ? 0u : aslot + 1);
                    const uint32_t b = ch * kQ8ChunkBlocks + 2 * pp;
                    if (row < rows) {
                        int32_t d0, d1;
                        if (b < nb)
                            q8_pair(reinterpret_cast<const uint32_t*>(ring + (size_t)aslot * slot_bytes +
                                                                      (i0 % nw) * kQ8WarpTileBytes + lane_off),
                                    xs, xd, b, d0, d1, sum);
                        if (two && b + kQ8ChunkBlocks < nb)
                            q8_pair(reinterpret_cast<const uint32_t*>(ring + (size_t)bslot * slot_bytes +
                                                                      (i1 % nw) * kQ8WarpTileBytes + lane_off),
                                    xs, xd, b + kQ8ChunkBlocks, d0, d1, sum);
                    }
                    // the vote consumes every lane's sum, so all of this step's ring reads
                    // have returned: the tiles can be freed without release semantics
                    __all_sync(0xffffffffu, sum == sum);
                    if (lane == 0) {
                        ptx::mbar_arrive_relaxed(&empty[aslot]);
                        if (two) ptx::mbar_arrive_relaxed(&empty[bslot]);
                    }
                }
                // A warp's last tile may sit in the stage before the last.  It still
                // waits for every stage of the pass: a parity wait is exact only while
                // the slot is at most one phase away, and a warp that skipped a stage
                // could otherwise meet that slot two phases on in a later pass.
                while (waited < nst && !dead) {
                    if (!ptx::mbar_wait(&full[wslot], wphase, err)) dead = true;
                    waited++;
                    if (++wslot == nslots) {
                        wslot = 0;
                        wphase ^= 1u;
                    }
                }
            }
            t += nst;
            sum = q8_row_total(sum);
            // 3. publish: one tagged word per row and rank
            if (!dead && cw < nwp && row < rows && pp == 0)
                for (uint32_t q = 0; q < world; q++) st_word(P->out[q] + row, sum, tag);
        }
        // every compute warp is done with xs / xd before the next projection rewrites them
        if (dead) dead_s = 1;
        __syncwarp();
        ptx::named_barrier_sync(1, nw * 32);
        if (dead_s) return;
    }
    // The launch ends only when the gathered last output is complete on this GPU:
    // peers may still be storing their rows into it (CTAs split the words).
    {
        const StackProj* L = projs + nproj - 1;
        const uint32_t total = world * L->rows, last = tag_of(epoch, nproj - 1);
        for (uint32_t i = c * nw * 32 + ct; i < total && !dead; i += G * nw * 32)
            wait_word(L->out_all + i, last, &dead, err);
        if (dead) dead_s = 1;
        __syncwarp();
        ptx::named_barrier_sync(1, nw * 32);
        if (dead_s) return;
    }
    // this launch is finished on this CTA; the last CTA of this GPU bumps the epoch
    if (cw == 0 && lane == 0) {
        const uint32_t prev = atomicAdd(ctl + 1, 1u);
        if (prev == G - 1) {
            ctl[1] = 0;
            __threadfence();
            atomicAdd(ctl, 1u);
        }
    }
}

}  // namespace

// ------------------------------------------------------------------ host
struct StackPlan {
    StackProj* dev_projs = nullptr;
    uint32_t nproj = 0, world = 1, nslots = 2, kmax = 0;
    uint32_t* ctl = nullptr;
    size_t smem = 0;
};

int stack_plan_create(const ane_q8_stack_proj* projs, uint32_t nproj, uint32_t world, uint32_t rank, uint32_t* ctl,
                      void** plan_out) {
    ANE_ARG_CHECK(plan_out && projs && ctl, "q8_stack: NULL argument");
    ANE_ARG_CHECK(nproj > 0, "q8_stack: no projections");
    ANE_ARG_CHECK(world >= 1 && world <= kStackMaxRanks && rank < world, "q8_stack: world must be 1..8, rank < world");
    uint32_t kmax = 0;
    std::vector<StackProj> host(nproj);
    for (uint32_t j = 0; j < nproj; j++) {
        const ane_q8_stack_proj& p = projs[j];
        ANE_ARG_CHECK(p.K % 256 == 0 && p.K > 0, "q8_stack: K must be a positive multiple of 256");
        ANE_ARG_CHECK(p.rows_local > 0, "q8_stack: every rank needs at least one row");
        ANE_ARG_CHECK(((uintptr_t)p.W & 15) == 0 && ((uintptr_t)p.x & 15) == 0,
                      "q8_stack: W and x must be 16-byte aligned");
        ANE_ARG_CHECK(!p.x_tagged || j > 0, "q8_stack: the first projection's input must be a plain vector");
        ANE_ARG_CHECK(p.out_all && ((uintptr_t)p.out_all & 7) == 0, "q8_stack: out_all must be 8-byte aligned");
        StackProj& h = host[j];
        memset(&h, 0, sizeof(h));
        const uint64_t row_bytes = (uint64_t)p.K / 32 * 34;
        int rc = encode_tensor_map_2d(&h.wmap, CU_TENSOR_MAP_DATA_TYPE_UINT32, p.W, row_bytes / 4, p.rows_local,
                                      row_bytes, kQ8ChunkBytes / 4, kQ8RowsPerWarp, CU_TENSOR_MAP_SWIZZLE_NONE);
        if (rc) return rc;
        h.x = p.x;
        h.x_tagged = p.x_tagged ? 1u : 0u;
        for (uint32_t q = 0; q < world; q++) {
            ANE_ARG_CHECK(p.out[q] != nullptr && ((uintptr_t)p.out[q] & 7) == 0,
                          "q8_stack: an 8-byte-aligned output pointer per rank is required");
            h.out[q] = static_cast<uint2*>(p.out[q]);
        }
        h.out_all = static_cast<const uint2*>(p.out_all);
        h.rows = p.rows_local;
        h.K = p.K;
        h.groups = (p.rows_local + kQ8RowsPerWarp - 1) / kQ8RowsPerWarp;
        kmax = p.K > kmax ? p.K : kmax;
    }
    const size_t fixed = 128 + round_up((size_t)kmax, 128) + round_up((size_t)kmax / 32 * 4, 128);
    const size_t slot = (size_t)kStackWarps * kQ8WarpTileBytes;
    const size_t budget = 226 * 1024;
    ANE_ARG_CHECK(fixed + 2 * slot <= budget, "q8_stack: K too large for the shared activation buffer");
    uint32_t nslots = (uint32_t)((budget - fixed) / slot);
    nslots = nslots > kQ8MaxSlots ? kQ8MaxSlots : nslots;
    auto* plan = new StackPlan();
    plan->nproj = nproj;
    plan->world = world;
    plan->nslots = nslots;
    plan->kmax = kmax;
    plan->ctl = ctl;
    plan->smem = fixed + nslots * slot;
    cudaError_t e = cudaMalloc(&plan->dev_projs, sizeof(StackProj) * nproj);
    if (e == cudaSuccess)
        e = cudaMemcpy(plan->dev_projs, host.data(), sizeof(StackProj) * nproj, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        cudaFree(plan->dev_projs);
        delete plan;
        ANE_CUDA_TRY(e);
    }
    *plan_out = plan;
    return ANE_OK;
}

int stack_plan_run(void* plan_ptr, cudaStream_t s) {
    ANE_ARG_CHECK(plan_ptr, "q8_stack: NULL plan");
    auto* plan = static_cast<StackPlan*>(plan_ptr);
    static std::atomic<uint64_t> smem_set{0};  // devices whose limit is raised
    if (int arc = set_max_dynamic_smem(decode_stack_kernel, 226 * 1024, smem_set)) return arc;
    ANE_ARG_CHECK(num_sms() <= 256, "q8_stack: the guard words assume at most 256 SMs");
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)num_sms(), 1, 1);
    cfg.blockDim = dim3(32 * (kStackWarps + 1), 1, 1);
    cfg.dynamicSmemBytes = plan->smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;  // every CTA resident: no wait can be on an unscheduled CTA
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    ANE_CUDA_TRY(cudaLaunchKernelEx(&cfg, decode_stack_kernel, (const StackProj*)plan->dev_projs, plan->nproj,
                                    plan->world, plan->ctl, plan->nslots, plan->kmax, device_timeout_flag()));
    ANE_CHECK_LAUNCH();
    return ANE_OK;
}

void stack_plan_free(void* plan_ptr) {
    auto* plan = static_cast<StackPlan*>(plan_ptr);
    if (!plan) return;
    cudaFree(plan->dev_projs);
    delete plan;
}

}  // namespace ane_b200
