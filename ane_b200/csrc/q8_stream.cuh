// q8_stream.cuh -- work plan and launch of the streamed Q8_0 matvec kernels
// (q8_0_gemv.cu: fp32 activation, q8_0_gemv_q8.cu: Q8_0 activation).
//
// Both kernels stream the weight rows HBM -> shared memory with 2-D TMA copies
// and compute from shared memory.  Rows are handed out in groups of four (one
// compute warp each).  CTA i of n owns the contiguous row groups
// [G*i/n, G*(i+1)/n), so every SM gets the same number of rows to within one
// group; a CTA with more groups than compute warps streams them in passes.
// One producer warp per CTA feeds a ring of `slots` stages; stage t holds chunk
// t % nchunks (16 blocks = 544 bytes per row) of pass t / nchunks for every
// compute warp (4 rows x 544 bytes = 2176 bytes per warp, a multiple of 128 so
// every TMA destination stays 128-byte aligned).
#pragma once
#include "ane_internal.cuh"

namespace ane_b200 {

constexpr uint32_t kQ8RowsPerWarp = 4;
constexpr uint32_t kQ8ChunkBlocks = 16;
constexpr uint32_t kQ8ChunkBytes = kQ8ChunkBlocks * 34;                // 544
constexpr uint32_t kQ8WarpTileBytes = kQ8RowsPerWarp * kQ8ChunkBytes;  // 2176 = 17 x 128
constexpr uint32_t kQ8MaxWarps = 24;
constexpr uint32_t kQ8MaxSlots = 8;
static_assert(kQ8WarpTileBytes % 128 == 0, "TMA destinations stay 128-byte aligned");

struct Q8Plan {
    uint32_t groups;  // row groups of 4 rows
    uint32_t ctas;
    uint32_t warps;   // compute warps per CTA (plus one producer warp)
    uint32_t slots;   // ring stages
    size_t slot_bytes;
    size_t smem;
};

// extra_slot_bytes: per-stage bytes besides the weights (the x slice of the fp32
// kernel); fixed_bytes: shared memory outside the ring (barriers, staged x).
// With programmatic dependent launch the next matvec's CTAs start their
// prologue while this grid drains (see the budget below).  ANE_Q8_WARPS /
// ANE_Q8_SLOTS / ANE_Q8_CPS (CTAs per SM) override the choice (tuning aids).
// block_bytes / warp_tile_bytes: 34 / 2176 for Q8_0; 18 / 1152 for Q4_0 (same
// 4 rows x 16 blocks per warp tile).  max_warps: the most 4-row groups one CTA
// takes per pass.
inline Q8Plan plan_q8_stream(uint32_t M, uint32_t K, size_t extra_slot_bytes, size_t fixed_bytes,
                             uint32_t block_bytes = 34, uint32_t warp_tile_bytes = kQ8WarpTileBytes,
                             uint32_t max_warps = kQ8MaxWarps) {
    static const int force_warps = env_int("ANE_Q8_WARPS"), force_slots = env_int("ANE_Q8_SLOTS"),
                     force_cps = env_int("ANE_Q8_CPS");
    const uint32_t sms = (uint32_t)num_sms();
    Q8Plan p{};
    p.groups = (M + kQ8RowsPerWarp - 1) / kQ8RowsPerWarp;
    const uint32_t per_sm = (p.groups + sms - 1) / sms;
    // Small matrices (<= 160 KB of weights per SM): one CTA per SM, and room for
    // the next grid's CTA beside it.  Larger ones: at least two CTAs per SM
    // (finer-grained hand-over between grids) and the whole shared memory for
    // the rings (more bytes in flight per SM).
    const double sm_bytes = (double)M * (K / 32) * block_bytes / sms;
    uint32_t cps = (per_sm + max_warps - 1) / max_warps;
    if (sm_bytes > 160.0 * 1024 && cps < 2 && per_sm >= 2) cps = 2;
    if (force_cps > 0) cps = (uint32_t)force_cps;
    if (force_warps > 0) {
        const uint32_t w = force_warps > (int)max_warps ? max_warps : (uint32_t)force_warps;
        p.ctas = (p.groups + w - 1) / w;
    } else {
        p.ctas = sms * cps;
    }
    if (p.ctas > p.groups) p.ctas = p.groups;
    if (p.ctas == 0) p.ctas = 1;
    p.warps = (p.groups + p.ctas - 1) / p.ctas;
    if (p.warps > max_warps) p.warps = max_warps;  // the CTA then streams several passes
    p.slot_bytes = (size_t)p.warps * warp_tile_bytes + extra_slot_bytes;
    // With one CTA per SM, the next grid's CTAs fit beside this grid's, one per
    // SM, so they are placed evenly; with more, a reserved spare would be filled
    // unevenly as CTAs finish, so the rings take the whole share instead.
    const uint32_t resident = (p.ctas + sms - 1) / sms;
    const size_t budget = 227 * 1024 / (resident == 1 ? 2 : resident) - 1024;
    uint32_t slots = budget > fixed_bytes ? (uint32_t)((budget - fixed_bytes) / p.slot_bytes) : 0;
    if (force_slots > 0) slots = (uint32_t)force_slots;
    p.slots = slots < 2 ? 2 : (slots > kQ8MaxSlots ? kQ8MaxSlots : slots);
    p.smem = fixed_bytes + (size_t)p.slots * p.slot_bytes;
    return p;
}

// Launches a streamed Q8_0 kernel with programmatic stream serialization; the
// kernels read x and write out only after griddepcontrol.wait, and W too unless
// the caller passed ANE_Q8_WEIGHTS_STATIC.
template <typename... KArgs, typename... Args>
int launch_q8_stream(void (*kernel)(KArgs...), const Q8Plan& p, cudaStream_t s, Args... args) {
    return launch_pdl(kernel, dim3(p.ctas, 1, 1), dim3(32 * (p.warps + 1), 1, 1), p.smem, s, args...);
}

}  // namespace ane_b200
