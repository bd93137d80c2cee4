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
#include "q8_stream.cuh"
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
// For K % 256 == 0 and 16-byte-aligned W and x (every row starts 16-byte
// aligned).  Work split, ring and launch: q8_stream.cuh.  A compute warp owns 4
// rows, 8 threads per row, thread j owning lanes 2j and 2j+1 (bytes
// q[2j..2j+1] and q[16+2j..16+2j+1] of every block).  Each ring stage carries,
// next to the 4-row weight tiles of every compute warp, the chunk's 512-float
// slice of x.  FADDV: level 1 in-thread, levels 2-4 by xor shuffles 1, 2, 4
// across the 8 threads of the row.
static constexpr int kChunkXBytes = kQ8ChunkBlocks * 32 * 4;
static_assert(kChunkXBytes % 128 == 0, "slot alignment");

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

// One block for lanes {2j, 2j+1}, finite d: the four products q*d come from two
// packed FMAs fma(f, d, -32896*d) (exact), the two accumulate steps are packed
// FMAs on {acc[2j], acc[2j+1]} -- per lane the same roundings, in the same
// order, as the reference's fmul + fmla.
__device__ __forceinline__ float2 q8_block_fast(float2 acc, uint32_t w, float d, float2 xlo, float2 xhi) {
    const uint32_t u = w ^ 0x80808080u;
    const float2 dd = make_float2(d, d);
    const float ncd = __fmul_rn(-32896.0f, d);
    const float2 nc = make_float2(ncd, ncd);
    const float2 f01 = make_float2(__uint_as_float(__byte_perm(u, 0x47000000u, 0x7404u)),
                                   __uint_as_float(__byte_perm(u, 0x47000000u, 0x7414u)));
    const float2 f23 = make_float2(__uint_as_float(__byte_perm(u, 0x47000000u, 0x7424u)),
                                   __uint_as_float(__byte_perm(u, 0x47000000u, 0x7434u)));
    const float2 dq01 = ptx::ffma2(f01, dd, nc);
    const float2 dq23 = ptx::ffma2(f23, dd, nc);
    acc = ptx::ffma2(dq01, xlo, acc);
    return ptx::ffma2(dq23, xhi, acc);
}

// Warp 0 of every CTA is the producer (one elected lane): per stage it issues
// one 4-row x 544-byte TMA box per compute warp with rows in the pass and one
// bulk copy of the x slice, after the consumers have released the stage.
// (The launch bound lets ptxas keep a whole 8-block load phase in registers.)
// GATHER (one link of a row-sharded decode chain): each row result leaves as
// one 8-byte {value, tag} word stored into every rank's next vector instead of
// out[row]; x is then the fp32 vector q8_unpack_tagged_kernel wrote.
template <bool GATHER>
__global__ void __launch_bounds__(32 * (kQ8MaxWarps + 1), 1)
    q8_0_gemv_stream_kernel(const __grid_constant__ CUtensorMap wmap, const uint8_t* __restrict__ W,
                            const float* __restrict__ x, float* __restrict__ out, uint32_t M, uint32_t K,
                            uint32_t groups, uint32_t nw, uint32_t nslots, uint32_t flags, int* err,
                            const __grid_constant__ Q8ChainGather pg) {
    extern __shared__ __align__(128) uint8_t smem[];
    // the last chunk may hold 8 blocks (K % 512 == 256): the TMA box then runs
    // past the row end and zero-fills, and the transaction counts the full box
    const uint32_t nb = K / 32, nchunks = (nb + kQ8ChunkBlocks - 1) / kQ8ChunkBlocks;
    const uint32_t w_bytes = nw * kQ8WarpTileBytes;  // weight part of a stage
    const uint32_t slot_bytes = w_bytes + kChunkXBytes;
    auto chunk_blocks = [&](uint32_t c) { return min((uint32_t)kQ8ChunkBlocks, nb - c * kQ8ChunkBlocks); };
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);  // nslots
    uint64_t* empty = full + nslots;                     // nslots
    uint8_t* ring = smem + 128;                          // nslots x slot_bytes
    const uint32_t g0 = (uint32_t)((uint64_t)groups * blockIdx.x / gridDim.x);
    const uint32_t g1 = (uint32_t)((uint64_t)groups * (blockIdx.x + 1) / gridDim.x);
    const uint32_t npass = (g1 - g0 + nw - 1) / nw, ntiles = npass * nchunks;
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
        if (lane == 0) {
            ptx::prefetch_tmap(&wmap);
            auto issue_weights = [&](uint32_t t, uint32_t slot) {
                const uint32_t pass = t / nchunks, c = t - pass * nchunks;
                const uint32_t gp = g0 + pass * nw, nwp = min(nw, g1 - gp);
                uint8_t* dst = ring + (size_t)slot * slot_bytes;
                ptx::mbar_arrive_expect_tx(&full[slot], nwp * kQ8WarpTileBytes + chunk_blocks(c) * 32 * 4);
                for (uint32_t w = 0; w < nwp; w++)
                    ptx::tma_load_2d(dst + w * kQ8WarpTileBytes, &wmap, &full[slot], (int)(c * (kQ8ChunkBytes / 4)),
                                     (int)((gp + w) * kQ8RowsPerWarp));
            };
            auto issue_x = [&](uint32_t t, uint32_t slot) {
                const uint32_t c = t % nchunks;
                ptx::bulk_load(ring + (size_t)slot * slot_bytes + w_bytes, x + (size_t)c * kQ8ChunkBlocks * 32,
                               chunk_blocks(c) * 32 * 4, &full[slot]);
            };
            // static weights: the first stages' weight tiles are requested before
            // the previous kernel on the stream has finished
            const uint32_t pre = (flags & ANE_Q8_WEIGHTS_STATIC) ? min(nslots, ntiles) : 0;
            for (uint32_t t = 0; t < pre; t++) issue_weights(t, t);
            ptx::griddep_wait();  // x may be written by the previous kernel
            for (uint32_t t = 0; t < pre; t++) issue_x(t, t);
            for (uint32_t t = pre; t < ntiles; t++) {
                const uint32_t slot = t % nslots;
                if (!ptx::mbar_wait(&empty[slot], ((t / nslots) & 1) ^ 1, err)) break;
                issue_weights(t, slot);
                issue_x(t, slot);
            }
        }
        return;
    }
    // ------------------------------------------------------------ compute
    ptx::griddep_wait();  // out (and x, on the replay path) may belong to the previous kernel
    // GATHER: this projection's tag (the count is final once the kernels before
    // this one have ended)
    const uint32_t tag_out = GATHER ? *reinterpret_cast<const volatile uint32_t*>(pg.tok) * pg.nproj + pg.j + 1u : 0u;
    const uint32_t cw = warp - 1, rr = lane >> 3, j = lane & 7;
    bool alive = true;
    for (uint32_t pass = 0; pass < npass && alive; pass++) {
        const uint32_t gp = g0 + pass * nw;
        const uint32_t row = (gp + cw) * kQ8RowsPerWarp + rr;
        const bool active = gp + cw < g1 && row < M;
        float2 acc = make_float2(0.f, 0.f);
        for (uint32_t c = 0; c < nchunks; c++) {
            const uint32_t t = pass * nchunks + c, slot = t % nslots;
            // one verdict per warp: after a timed-out wait every lane leaves together
            if (!__all_sync(0xffffffffu, ptx::mbar_wait(&full[slot], (t / nslots) & 1, err))) { alive = false; break; }
            if (active) {
                const uint8_t* st = ring + (size_t)slot * slot_bytes;
                const uint8_t* rp = st + cw * kQ8WarpTileBytes + rr * kQ8ChunkBytes;
                const float* xc = reinterpret_cast<const float*>(st + w_bytes) + 2 * j;
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
                    // compute phase: blocks in order.  The fast dequant equals q*d
                    // exactly for every finite d; an inf/NaN d makes the row result
                    // non-finite, and such rows are recomputed below.
#pragma unroll
                    for (int i = 0; i < 8; i++) {
                        const float d = __half2float(__ushort_as_half((unsigned short)dbits[i]));
                        acc = q8_block_fast(acc, w[i], d, xl[i], xh[i]);
                    }
                }
            }
            __syncwarp();
            if (lane == 0) ptx::mbar_arrive(&empty[slot]);  // this warp is done with the stage
        }
        auto faddv = [](float a0, float a1) {  // level 1 in-thread, levels 2-4 across the row's 8 threads
            float t = __fadd_rn(a0, a1);
            t = __fadd_rn(t, __shfl_xor_sync(0xffffffffu, t, 1));
            t = __fadd_rn(t, __shfl_xor_sync(0xffffffffu, t, 2));
            return __fadd_rn(t, __shfl_xor_sync(0xffffffffu, t, 4));
        };
        float s = faddv(acc.x, acc.y);
        // Rare path: a non-finite row result may come from an inf/NaN block scale,
        // for which the fma shortcut differs from the reference's scvtf + fmul;
        // replay such rows (row-uniform decision) from global memory with the
        // direct product.
        const bool redo = active && alive && !isfinite(s);
        if (__any_sync(0xffffffffu, redo)) {
            float a0 = 0.f, a1 = 0.f;
            if (redo) {
                const uint8_t* rp = W + (size_t)row * ((size_t)nb * 34);
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
        if (active && j == 0 && alive) {
            if constexpr (GATHER) {
                const uint64_t w = (uint64_t)__float_as_uint(s) | ((uint64_t)tag_out << 32);
                for (uint32_t q = 0; q < pg.world; q++)
                    asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(pg.out[q] + row), "l"(w) : "memory");
            } else {
                out[row] = s;
            }
        }
    }
}

// The fp32 input of a mode-R chain link: waits (bounded) until each of the K
// words of the previous projection's tagged vector on this GPU carries that
// projection's tag and writes its value to x (16-byte loads, eight per thread
// in flight, the missing ones read again together each round).  Block 0 also
// waits for one word per rank of the previous projection (that rank's first
// row): a rank that stored it has finished reading the vector the matvec after
// this kernel overwrites.  K = 0: the guard alone (a layer's first projection,
// whose x is the fp32 layer input).
constexpr uint32_t kUnpackThreads = 256, kUnpackPairs = 8;
__global__ void __launch_bounds__(kUnpackThreads) q8_unpack_tagged_kernel(const uint64_t* __restrict__ prev,
                                                                          uint32_t K, float* __restrict__ x,
                                                                          uint32_t world, uint32_t prev_rows,
                                                                          const uint32_t* tok, uint32_t nproj,
                                                                          uint32_t jproj, int* err) {
    ptx::griddep_launch_dependents();
    ptx::griddep_wait();  // x may still be read by the kernel before this one
    const uint32_t tag = *reinterpret_cast<const volatile uint32_t*>(tok) * nproj + jproj;
    auto ld_word = [](const uint64_t* p) {
        uint64_t w;
        asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
        return w;
    };
    if (blockIdx.x == 0 && threadIdx.x < world) {
        const uint64_t* g = prev + (size_t)threadIdx.x * prev_rows;
        const long long t0 = clock64();
        while ((uint32_t)(ld_word(g) >> 32) != tag) {
            if (clock64() - t0 > ptx::kWaitTimeoutCycles) {
                atomicAdd(err, 1);
                break;
            }
            __nanosleep(64);
        }
    }
    const uint32_t npairs = K / 2, stride = gridDim.x * kUnpackThreads;
    for (uint32_t base = blockIdx.x * kUnpackThreads + threadIdx.x; base < npairs; base += stride * kUnpackPairs) {
        uint2 v[kUnpackPairs];
        uint32_t miss = 0;
#pragma unroll
        for (uint32_t u = 0; u < kUnpackPairs; u++) {
            const uint32_t i = base + u * stride;
            if (i < npairs) {
                uint64_t a, b;
                asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(prev + 2 * i) : "memory");
                v[u] = make_uint2((uint32_t)a, (uint32_t)b);
                if ((uint32_t)(a >> 32) != tag || (uint32_t)(b >> 32) != tag) miss |= 1u << u;
            }
        }
        const long long t0 = miss ? clock64() : 0;
        while (miss) {
            if (clock64() - t0 > ptx::kWaitTimeoutCycles) {
                atomicAdd(err, 1);
                break;
            }
            __nanosleep(64);
#pragma unroll
            for (uint32_t u = 0; u < kUnpackPairs; u++) {
                if (!((miss >> u) & 1u)) continue;
                const uint32_t i = base + u * stride;
                uint64_t a, b;
                asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(prev + 2 * i) : "memory");
                if ((uint32_t)(a >> 32) == tag && (uint32_t)(b >> 32) == tag) {
                    v[u] = make_uint2((uint32_t)a, (uint32_t)b);
                    miss &= ~(1u << u);
                }
            }
        }
#pragma unroll
        for (uint32_t u = 0; u < kUnpackPairs; u++) {
            const uint32_t i = base + u * stride;
            if (i < npairs) reinterpret_cast<float2*>(x)[i] = make_float2(__uint_as_float(v[u].x), __uint_as_float(v[u].y));
        }
    }
}

int launch_q8_0_gemv(uint32_t M, uint32_t K, const float* x, const uint8_t* W, float* out, uint32_t flags,
                     cudaStream_t s) {
    if (M == 0) return ANE_OK;
    ANE_ARG_CHECK(K % 32 == 0, "q8_0_gemv: K must be a multiple of 32");
    ANE_ARG_CHECK(((uintptr_t)W & 1) == 0, "q8_0_gemv: W must be 2-byte aligned");
    if (K % 256 == 0 && ((uintptr_t)W & 15) == 0 && ((uintptr_t)x & 15) == 0) {
        const Q8Plan p = plan_q8_stream(M, K, kChunkXBytes, 128);
        static std::atomic<uint64_t> smem_set{0};  // devices whose limit is raised
        if (int arc = set_max_dynamic_smem(q8_0_gemv_stream_kernel<false>, 200 * 1024, smem_set)) return arc;
        ANE_ARG_CHECK(p.smem <= 200 * 1024, "q8_0_gemv: shared-memory plan too large");
        const uint64_t row_bytes = (uint64_t)(K / 32) * 34;
        CUtensorMap wmap;
        int rc = encode_tensor_map_2d(&wmap, CU_TENSOR_MAP_DATA_TYPE_UINT32, W, row_bytes / 4, M, row_bytes,
                                      kQ8ChunkBytes / 4, kQ8RowsPerWarp, CU_TENSOR_MAP_SWIZZLE_NONE);
        if (rc) return rc;
        const Q8ChainGather none{};
        return launch_q8_stream(q8_0_gemv_stream_kernel<false>, p, s, wmap, W, x, out, M, K, p.groups, p.warps,
                                p.slots, flags, device_timeout_flag(), none);
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

int launch_q8_0_gemv_gather(uint32_t M, uint32_t K, const float* x, float* xbuf, const uint8_t* W,
                            const Q8ChainGather& g, uint32_t flags, cudaStream_t s) {
    ANE_ARG_CHECK(M > 0 && K % 256 == 0 && K > 0, "q8_0_gemv gather: K must be a positive multiple of 256");
    ANE_ARG_CHECK(g.world >= 1 && g.world <= 8 && g.prev && g.tok && g.nproj > 0 && g.j < g.nproj && g.prev_rows > 0,
                  "q8_0_gemv gather: bad chain arguments");
    ANE_ARG_CHECK(((uintptr_t)W & 15) == 0 && ((uintptr_t)g.prev & 15) == 0, "q8_0_gemv gather: W and prev must be 16-byte aligned");
    const float* xin = g.x_from_prev ? xbuf : x;
    ANE_ARG_CHECK(xin && ((uintptr_t)xin & 15) == 0, "q8_0_gemv gather: x must be 16-byte aligned");
    // the input (or the guard alone): one kernel, then the matvec
    const uint32_t kx = g.x_from_prev ? K : 0u;
    const uint32_t per = kUnpackThreads * kUnpackPairs * 2;
    const uint32_t blocks = kx ? (kx + per - 1) / per : 1u;
    int rc = launch_pdl(q8_unpack_tagged_kernel, dim3(blocks), dim3(kUnpackThreads), 0, s, g.prev, kx, xbuf, g.world,
                        g.prev_rows, g.tok, g.nproj, g.j, device_timeout_flag());
    if (rc) return rc;
    const Q8Plan p = plan_q8_stream(M, K, kChunkXBytes, 128);
    static std::atomic<uint64_t> smem_set{0};
    if (int arc = set_max_dynamic_smem(q8_0_gemv_stream_kernel<true>, 200 * 1024, smem_set)) return arc;
    ANE_ARG_CHECK(p.smem <= 200 * 1024, "q8_0_gemv gather: shared-memory plan too large");
    const uint64_t row_bytes = (uint64_t)(K / 32) * 34;
    CUtensorMap wmap;
    rc = encode_tensor_map_2d(&wmap, CU_TENSOR_MAP_DATA_TYPE_UINT32, W, row_bytes / 4, M, row_bytes,
                              kQ8ChunkBytes / 4, kQ8RowsPerWarp, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
    return launch_q8_stream(q8_0_gemv_stream_kernel<true>, p, s, wmap, W, xin, (float*)nullptr, M, K, p.groups,
                            p.warps, p.slots, flags, device_timeout_flag(), g);
}

}  // namespace ane_b200
