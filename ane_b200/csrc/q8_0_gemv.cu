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
#include "sm100_ptx.cuh"

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

// ----------------------------------------------------------- streamed kernel
// For K % 256 == 0 and 16-byte-aligned W (every row starts 16-byte aligned):
// each CTA owns `rows` consecutive output rows; 8 threads per row, thread j
// owning lanes 2j and 2j+1 (bytes q[2j..2j+1] and q[16+2j..16+2j+1] of every
// block).  Weight rows stream through a ring of kSlots shared-memory slots in
// chunks of kChunkBlocks blocks (272 B per row) with cp.async.bulk, so HBM
// reads run up to kSlots-1 chunks ahead of the FMA chains; x sits in shared
// memory for the whole kernel.  FADDV: level 1 in-thread, levels 2-4 by xor
// shuffles 1, 2, 4 across the 8 threads of the row.
static constexpr int kChunkBlocks = 16;
static constexpr int kChunkBytes = kChunkBlocks * 34;  // 544 = 34 x 16
static constexpr int kChunkXBytes = kChunkBlocks * 32 * 4;
static constexpr int kMaxSlots = 8;  // full[8] + empty[8] fill the 128-byte barrier area
// TMA shared-memory destinations must be 128-byte aligned: every slot is
// rows*544 + 2048 bytes with rows a multiple of 4 (4*544 = 17*128).
static_assert((4 * kChunkBytes) % 128 == 0 && kChunkXBytes % 128 == 0, "slot alignment");

// q as fp32 from the biased byte: 0x4700_uu00 = 32768 + u = 32896 + q, minus
// 32896 (exact).  Then q*d is one RN multiply, exact for finite d and the same
// IEEE special cases as the reference's scvtf+fmul for inf/NaN d.
__device__ __forceinline__ float q_to_f32(uint32_t biased_word, uint32_t sel) {
    return __fadd_rn(__uint_as_float(__byte_perm(biased_word, 0x47000000u, sel)), -32896.0f);
}
__device__ __forceinline__ void q8_fma2_exact(float& acc0, float& acc1, uint32_t w, float d, float2 xlo,
                                              float2 xhi) {
    // w bytes: {q[2j], q[2j+1], q[16+2j], q[16+2j+1]}
    const uint32_t u = w ^ 0x80808080u;
    acc0 = __fmaf_rn(__fmul_rn(q_to_f32(u, 0x7404u), d), xlo.x, acc0);  // lane 2j,   first half
    acc1 = __fmaf_rn(__fmul_rn(q_to_f32(u, 0x7414u), d), xlo.y, acc1);  // lane 2j+1, first half
    acc0 = __fmaf_rn(__fmul_rn(q_to_f32(u, 0x7424u), d), xhi.x, acc0);  // lane 2j,   second half
    acc1 = __fmaf_rn(__fmul_rn(q_to_f32(u, 0x7434u), d), xhi.y, acc1);  // lane 2j+1, second half
}

__device__ __forceinline__ void q8_fma2(float& acc0, float& acc1, uint32_t w, float d, float negcd, bool finite,
                                        float2 xlo, float2 xhi) {
    // w bytes: {q[2j], q[2j+1], q[16+2j], q[16+2j+1]}
    float dq0, dq1, dq2, dq3;
    if (finite) {
        const uint32_t u = w ^ 0x80808080u;
        dq0 = dq_fast(u, 0x7404u, d, negcd);
        dq1 = dq_fast(u, 0x7414u, d, negcd);
        dq2 = dq_fast(u, 0x7424u, d, negcd);
        dq3 = dq_fast(u, 0x7434u, d, negcd);
    } else {
        dq0 = __fmul_rn((float)(int8_t)(w & 0xff), d);
        dq1 = __fmul_rn((float)(int8_t)((w >> 8) & 0xff), d);
        dq2 = __fmul_rn((float)(int8_t)((w >> 16) & 0xff), d);
        dq3 = __fmul_rn((float)(int8_t)(w >> 24), d);
    }
    acc0 = __fmaf_rn(dq0, xlo.x, acc0);  // lane 2j,   first half
    acc1 = __fmaf_rn(dq1, xlo.y, acc1);  // lane 2j+1, first half
    acc0 = __fmaf_rn(dq2, xhi.x, acc0);  // lane 2j,   second half
    acc1 = __fmaf_rn(dq3, xhi.y, acc1);  // lane 2j+1, second half
}

// Warp 0 of every CTA is the producer: it refills a slot as soon as all compute
// warps have released it (per-slot `empty` mbarrier), so compute warps never
// wait on each other.  Compute warps w = 1..NW each own 4 rows.
__global__ void q8_0_gemv_stream_kernel(const __grid_constant__ CUtensorMap wmap, const uint8_t* __restrict__ W,
                                        const float* __restrict__ x,
                                        float* __restrict__ out, uint32_t M, uint32_t K, uint32_t nslots,
                                        int* err) {
    extern __shared__ __align__(128) uint8_t smem[];
    const uint32_t nw = blockDim.x / 32 - 1;  // compute warps
    const uint32_t rows_per_cta = 4 * nw;
    // the last chunk may hold fewer than kChunkBlocks blocks (the TMA zero-fills the rest)
    const uint32_t nb = K / 32, nchunks = (nb + kChunkBlocks - 1) / kChunkBlocks;
    const uint32_t w_bytes = rows_per_cta * kChunkBytes;  // weight part of a slot
    const uint32_t slot_bytes = w_bytes + kChunkXBytes;   // + the chunk's slice of x
    auto chunk_blocks = [&](uint32_t c) { return min((uint32_t)kChunkBlocks, nb - c * kChunkBlocks); };
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);  // nslots
    uint64_t* empty = full + nslots;                     // nslots
    uint8_t* ring = smem + 128;                          // nslots x slot_bytes
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
    __syncthreads();

    if (warp == 0) {
        // ---------------------------------------------------------- producer
        // Per chunk: one 2-D TMA for rows r0.. of the CTA x 544 bytes (136 uint32;
        // rows past M and bytes past the row end of a half last chunk read as
        // zero, the transaction counts the full box) and one 1-D bulk copy of
        // the chunk's x slice (512 or 256 floats).
        if (lane == 0) {
            ptx::prefetch_tmap(&wmap);
            for (uint32_t c = 0; c < nchunks; c++) {
                const uint32_t slot = c % nslots;
                if (!ptx::mbar_wait(&empty[slot], ((c / nslots) & 1) ^ 1, err)) break;
                const uint32_t xbytes = chunk_blocks(c) * 32 * 4;
                uint8_t* dst = ring + (size_t)slot * slot_bytes;
                ptx::mbar_arrive_expect_tx(&full[slot], w_bytes + xbytes);
                ptx::tma_load_2d(dst, &wmap, &full[slot], (int)(c * (kChunkBytes / 4)), (int)r0);
                ptx::bulk_load(dst + w_bytes, x + (size_t)c * kChunkBlocks * 32, xbytes, &full[slot]);
            }
        }
        return;
    }
    // ------------------------------------------------------------ compute
    const uint32_t row = (warp - 1) * 4 + (lane >> 3), j = lane & 7;
    const bool active = row < nrows;
    float acc0 = 0.f, acc1 = 0.f;
    bool alive = true;
    for (uint32_t c = 0; c < nchunks && alive; c++) {
        const uint32_t slot = c % nslots;
        if (!ptx::mbar_wait(&full[slot], (c / nslots) & 1, err)) { alive = false; break; }
        if (active) {
            const uint8_t* rp = ring + (size_t)slot * slot_bytes + row * kChunkBytes;
            const float* xc = reinterpret_cast<const float*>(ring + (size_t)slot * slot_bytes + w_bytes) + 2 * j;
            const int cb = (int)chunk_blocks(c);  // 16, or 8 for the half last chunk
            for (int b0 = 0; b0 < cb; b0 += 8) {
                // load phase: all shared-memory reads of 8 blocks issue back to back
                uint32_t dbits[8], w[8];
                float2 xl[8], xh[8];
#pragma unroll
                for (int i = 0; i < 8; i++) {
                    const uint8_t* blk = rp + (b0 + i) * 34;
                    dbits[i] = *reinterpret_cast<const unsigned short*>(blk);
                    w[i] = *reinterpret_cast<const unsigned short*>(blk + 2 + 2 * j) |
                           ((uint32_t)*reinterpret_cast<const unsigned short*>(blk + 18 + 2 * j) << 16);
                    xl[i] = *reinterpret_cast<const float2*>(xc + (b0 + i) * 32);
                    xh[i] = *reinterpret_cast<const float2*>(xc + (b0 + i) * 32 + 16);
                }
                // compute phase: blocks in order, two FMA chains.  fma(f, d, -32896*d)
                // equals q*d exactly for every finite d; an inf/NaN d makes the row
                // result non-finite, and such rows are recomputed below.
#pragma unroll
                for (int i = 0; i < 8; i++) {
                    const float d = __half2float(__ushort_as_half((unsigned short)dbits[i]));
                    q8_fma2(acc0, acc1, w[i], d, __fmul_rn(-32896.0f, d), true, xl[i], xh[i]);
                }
            }
        }
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(&empty[slot]);  // this warp is done with the slot
    }
    auto faddv = [](float a0, float a1) {  // level 1 in-thread, levels 2-4 across the row's 8 threads
        float t = __fadd_rn(a0, a1);
        t = __fadd_rn(t, __shfl_xor_sync(0xffffffffu, t, 1));
        t = __fadd_rn(t, __shfl_xor_sync(0xffffffffu, t, 2));
        return __fadd_rn(t, __shfl_xor_sync(0xffffffffu, t, 4));
    };
    float s = faddv(acc0, acc1);
    // Rare path: a non-finite row result may come from an inf/NaN block scale, for
    // which the fma shortcut differs from the reference's scvtf + fmul; replay
    // such rows (row-uniform decision) from global memory with the direct product.
    const bool redo = active && alive && !isfinite(s);
    if (__any_sync(0xffffffffu, redo)) {
        float a0 = 0.f, a1 = 0.f;
        if (redo) {
            const uint8_t* rp = W + (size_t)(r0 + row) * ((size_t)nb * 34);
            for (uint32_t b = 0; b < nb; b++) {
                const uint8_t* blk = rp + (size_t)b * 34;
                const uint32_t w = (uint32_t)*reinterpret_cast<const unsigned short*>(blk + 2 + 2 * j) |
                                   ((uint32_t)*reinterpret_cast<const unsigned short*>(blk + 18 + 2 * j) << 16);
                const float d = __half2float(__ushort_as_half(*reinterpret_cast<const unsigned short*>(blk)));
                q8_fma2_exact(a0, a1, w, d, *reinterpret_cast<const float2*>(x + 32 * b + 2 * j),
                              *reinterpret_cast<const float2*>(x + 32 * b + 16 + 2 * j));
            }
        }
        const float t = faddv(a0, a1);
        if (redo) s = t;
    }
    if (active && j == 0 && alive) out[r0 + row] = s;
}

int launch_q8_0_gemv(uint32_t M, uint32_t K, const float* x, const uint8_t* W, float* out, cudaStream_t s) {
    if (M == 0) return ANE_OK;
    ANE_ARG_CHECK(K % 32 == 0, "q8_0_gemv: K must be a multiple of 32");
    ANE_ARG_CHECK(((uintptr_t)W & 1) == 0, "q8_0_gemv: W must be 2-byte aligned");
    if (K % 256 == 0 && ((uintptr_t)W & 15) == 0 && ((uintptr_t)x & 15) == 0) {
        // ~6 resident CTAs per SM, each 1 producer warp + nw compute warps (4 rows each)
        const uint32_t sms = (uint32_t)num_sms();
        // ANE_Q8_WARPS (1..8 compute warps) and ANE_Q8_SLOTS (2..8) override the
        // shape-based choice (tuning aids)
        static const int force_warps = env_int("ANE_Q8_WARPS"), force_slots = env_int("ANE_Q8_SLOTS");
        uint32_t nw = force_warps > 0 ? (uint32_t)force_warps : (M + 4 * 6 * sms - 1) / (4 * 6 * sms);
        nw = nw < 1 ? 1 : (nw > 8 ? 8 : nw);
        const uint32_t rows = 4 * nw;
        // as many ring slots as fit a fair share of the SM's shared memory (up to
        // every chunk of the CTA): more bytes in flight per CTA from the start
        const uint32_t blocks_per_sm = (((M + rows - 1) / rows) + sms - 1) / sms;
        const size_t slot = (size_t)rows * kChunkBytes + kChunkXBytes;
        const uint32_t nchunks = (K / 32 + kChunkBlocks - 1) / kChunkBlocks;
        // (228 KB per SM, 1 KB of it reserved per resident CTA)
        const size_t share = 227 * 1024 / (blocks_per_sm ? blocks_per_sm : 1) - 1024;
        uint32_t nslots = share > 128 ? (uint32_t)((share - 128) / slot) : 2;
        nslots = nslots < 2 ? 2 : (nslots > (uint32_t)kMaxSlots ? (uint32_t)kMaxSlots : nslots);
        if (nslots > nchunks) nslots = nchunks < 2 ? 2 : nchunks;
        if (force_slots > 0) nslots = force_slots < 2 ? 2 : (force_slots > kMaxSlots ? kMaxSlots : force_slots);
        const size_t smem = 128 + (size_t)nslots * slot;
        static const cudaError_t attr_err = cudaFuncSetAttribute(
            q8_0_gemv_stream_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        ANE_CUDA_TRY(attr_err);
        const uint32_t blocks = (M + rows - 1) / rows;
        const uint64_t row_bytes = (uint64_t)(K / 32) * 34;
        CUtensorMap wmap;
        int rc = encode_tensor_map_2d(&wmap, CU_TENSOR_MAP_DATA_TYPE_UINT32, W, row_bytes / 4, M, row_bytes,
                                      kChunkBytes / 4, rows, CU_TENSOR_MAP_SWIZZLE_NONE);
        if (rc) return rc;
        q8_0_gemv_stream_kernel<<<blocks, 32 * (nw + 1), smem, s>>>(wmap, W, x, out, M, K, nslots,
                                                                    device_timeout_flag());
        ANE_CHECK_LAUNCH();
        return ANE_OK;
    }
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
