// q4_0_gemv.cu -- Q4_0 matrix-vector product, bit-exact with the reference.
//
// Reference handler q4_0_gemv (src/bytecode_interpreter.s:7064-7126), the one
// ggml MUL_MAT dispatches for Q4_0 weights (src/ggml-backend/ggml-ane.cpp:
// 144-149): 18-byte blocks {fp16 d; 16 bytes}, element i < 16 = low nibble of
// byte i, element 16+i = its high nibble, value (nibble - 8) * d.  Per output
// row 16 fp32 lanes; lane l does
//     acc[l] = fma((lo(q[l]) - 8) * d, x[32b+l],    acc[l])
//     acc[l] = fma((hi(q[l]) - 8) * d, x[32b+16+l], acc[l])
// and the row is FADDV(acc) -- q8_0_gemv's scheme with another block decoder,
// so this kernel keeps the Q8_0 mode-R streaming kernel's structure: 4 rows per
// compute warp, 8 threads per row owning lanes {2j, 2j+1}, a TMA ring of 4-row x
// 288-byte tiles plus the chunk's x slice, FADDV by xor shuffles 1, 2, 4.
//
// Nibble -> fp32 without the conversion unit: f = 16 + nibble is the float with
// the nibble in mantissa bits 19..22; fma(f, d, -24*d) = (nibble - 8) * d
// exactly (24 * d has <= 13 significant bits), the reference's scvtf + fmul
// result.  A non-finite d breaks that identity, so rows whose result is not
// finite are recomputed with the direct product.
#include <cuda_fp16.h>

#include "ane_internal.cuh"
#include "q8_stream.cuh"
#include "sm100_ptx.cuh"

namespace ane_b200 {
namespace {

constexpr uint32_t kQ4BlockBytes = 18;
constexpr uint32_t kQ4ChunkBytes = kQ8ChunkBlocks * kQ4BlockBytes;          // 288
constexpr uint32_t kQ4WarpTileBytes = kQ8RowsPerWarp * kQ4ChunkBytes;       // 1152 = 9 x 128
constexpr uint32_t kQ4ChunkXBytes = kQ8ChunkBlocks * 32 * 4;                // 2048
static_assert(kQ4WarpTileBytes % 128 == 0 && kQ4ChunkBytes % 16 == 0, "TMA boxes and slots stay aligned");

// 16 + nibble as fp32 (nibble in mantissa bits 19..22 of 16.0f = 0x41800000).
__device__ __forceinline__ float nib_f(uint32_t nib_at_19) { return __uint_as_float(0x41800000u | nib_at_19); }

// One block for lanes {2j, 2j+1}: w = bytes q[2j] | q[2j+1] << 8.
__device__ __forceinline__ float2 q4_block_fast(float2 acc, uint32_t w, float d, float2 xlo, float2 xhi) {
    const float2 dd = make_float2(d, d);
    const float ncd = __fmul_rn(-24.0f, d);
    const float2 nc = make_float2(ncd, ncd);
    const uint32_t m = 0xFu << 19;
    const float2 f_lo = make_float2(nib_f((w << 19) & m), nib_f((w << 11) & m));  // lo(q[2j]), lo(q[2j+1])
    const float2 f_hi = make_float2(nib_f((w << 15) & m), nib_f((w << 7) & m));   // hi(q[2j]), hi(q[2j+1])
    const float2 dq_lo = ptx::ffma2(f_lo, dd, nc);
    const float2 dq_hi = ptx::ffma2(f_hi, dd, nc);
    acc = ptx::ffma2(dq_lo, xlo, acc);
    return ptx::ffma2(dq_hi, xhi, acc);
}

// The reference's arithmetic literally (int -> float, RN multiply, FMA): the replay path.
__device__ __forceinline__ void q4_block_exact(float& a0, float& a1, uint32_t w, float d, float2 xlo, float2 xhi) {
    a0 = __fmaf_rn(__fmul_rn((float)((int)(w & 0xF) - 8), d), xlo.x, a0);
    a1 = __fmaf_rn(__fmul_rn((float)((int)((w >> 8) & 0xF) - 8), d), xlo.y, a1);
    a0 = __fmaf_rn(__fmul_rn((float)((int)((w >> 4) & 0xF) - 8), d), xhi.x, a0);
    a1 = __fmaf_rn(__fmul_rn((float)((int)((w >> 12) & 0xF) - 8), d), xhi.y, a1);
}

__global__ void __launch_bounds__(32 * (kQ8MaxWarps + 1), 1)
    q4_0_gemv_stream_kernel(const __grid_constant__ CUtensorMap wmap, const uint8_t* __restrict__ W,
                            const float* __restrict__ x, float* __restrict__ out, uint32_t M, uint32_t K,
                            uint32_t groups, uint32_t nw, uint32_t nslots, uint32_t flags, int* err) {
    extern __shared__ __align__(128) uint8_t smem[];
    // the last chunk may hold 8 blocks (K % 512 == 256): the TMA box then runs
    // past the row end and zero-fills, and the transaction counts the full box
    const uint32_t nb = K / 32, nchunks = (nb + kQ8ChunkBlocks - 1) / kQ8ChunkBlocks;
    const uint32_t w_bytes = nw * kQ4WarpTileBytes;
    const uint32_t slot_bytes = w_bytes + kQ4ChunkXBytes;
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
                ptx::mbar_arrive_expect_tx(&full[slot], nwp * kQ4WarpTileBytes + chunk_blocks(c) * 32 * 4);
                for (uint32_t w = 0; w < nwp; w++)
                    ptx::tma_load_2d(dst + w * kQ4WarpTileBytes, &wmap, &full[slot], (int)(c * (kQ4ChunkBytes / 4)),
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
    ptx::griddep_wait();  // out may belong to the previous kernel
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
                const uint8_t* rp = st + cw * kQ4WarpTileBytes + rr * kQ4ChunkBytes;
                const float* xc = reinterpret_cast<const float*>(st + w_bytes) + 2 * j;
                const int cb = (int)chunk_blocks(c);  // 16, or 8 for the half last chunk
                for (int b0 = 0; b0 < cb; b0 += 8) {
                    // load phase: all shared-memory reads of 8 blocks issue back to back
                    uint32_t dbits[8], w[8];
                    float2 xl[8], xh[8];
#pragma unroll
                    for (int i = 0; i < 8; i++) {
                        const uint8_t* blk = rp + (b0 + i) * kQ4BlockBytes;
                        dbits[i] = *reinterpret_cast<const unsigned short*>(blk);
                        w[i] = *reinterpret_cast<const unsigned short*>(blk + 2 + 2 * j);
                        xl[i] = *reinterpret_cast<const float2*>(xc + (b0 + i) * 32);
                        xh[i] = *reinterpret_cast<const float2*>(xc + (b0 + i) * 32 + 16);
                    }
#pragma unroll
                    for (int i = 0; i < 8; i++) {
                        const float d = __half2float(__ushort_as_half((unsigned short)dbits[i]));
                        acc = q4_block_fast(acc, w[i], d, xl[i], xh[i]);
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
        // a non-finite result may come from an inf/NaN block scale, where the fma
        // shortcut differs from scvtf + fmul: replay such rows from global memory
        const bool redo = active && alive && !isfinite(s);
        if (__any_sync(0xffffffffu, redo)) {
            float a0 = 0.f, a1 = 0.f;
            if (redo) {
                const uint8_t* rp = W + (size_t)row * ((size_t)nb * kQ4BlockBytes);
                for (uint32_t b = 0; b < nb; b++) {
                    const uint8_t* blk = rp + (size_t)b * kQ4BlockBytes;
                    const uint32_t w = *reinterpret_cast<const unsigned short*>(blk + 2 + 2 * j);
                    const float d = __half2float(__ushort_as_half(*reinterpret_cast<const unsigned short*>(blk)));
                    q4_block_exact(a0, a1, w, d, *reinterpret_cast<const float2*>(x + 32 * b + 2 * j),
                                   *reinterpret_cast<const float2*>(x + 32 * b + 16 + 2 * j));
                }
            }
            const float t = faddv(a0, a1);
            if (redo) s = t;
        }
        if (active && j == 0 && alive) out[row] = s;
    }
}

// Generic path (K % 256 != 0 or misaligned W / x): one thread per row, the
// reference's per-lane loop literally.
__global__ void q4_0_gemv_simple_kernel(const float* __restrict__ x, const uint8_t* __restrict__ W,
                                        float* __restrict__ out, uint32_t M, uint32_t K) {
    const uint32_t m = blockIdx.x * blockDim.x + threadIdx.x;
    if (m >= M) return;
    const uint32_t nb = K / 32;
    const uint8_t* row = W + (size_t)m * nb * kQ4BlockBytes;
    float acc[16];
#pragma unroll
    for (int l = 0; l < 16; l++) acc[l] = 0.f;
    for (uint32_t b = 0; b < nb; b++) {
        const uint8_t* blk = row + (size_t)b * kQ4BlockBytes;
        const float d = __half2float(__ushort_as_half((unsigned short)(blk[0] | (blk[1] << 8))));
#pragma unroll
        for (int l = 0; l < 16; l++)
            acc[l] = __fmaf_rn(__fmul_rn((float)((int)(blk[2 + l] & 0xF) - 8), d), x[32 * b + l], acc[l]);
#pragma unroll
        for (int l = 0; l < 16; l++)
            acc[l] = __fmaf_rn(__fmul_rn((float)((int)(blk[2 + l] >> 4) - 8), d), x[32 * b + 16 + l], acc[l]);
    }
    float s8[8], s4[4];
#pragma unroll
    for (int i = 0; i < 8; i++) s8[i] = __fadd_rn(acc[2 * i], acc[2 * i + 1]);
#pragma unroll
    for (int i = 0; i < 4; i++) s4[i] = __fadd_rn(s8[2 * i], s8[2 * i + 1]);
    out[m] = __fadd_rn(__fadd_rn(s4[0], s4[1]), __fadd_rn(s4[2], s4[3]));
}

}  // namespace

int launch_q4_0_gemv(uint32_t M, uint32_t K, const float* x, const uint8_t* W, float* out, uint32_t flags,
                     cudaStream_t s) {
    if (M == 0) return ANE_OK;
    ANE_ARG_CHECK(K % 32 == 0, "q4_0_gemv: K must be a multiple of 32");
    if (K % 256 == 0 && ((uintptr_t)W & 15) == 0 && ((uintptr_t)x & 15) == 0) {
        const Q8Plan p = plan_q8_stream(M, K, kQ4ChunkXBytes, 128, kQ4BlockBytes, kQ4WarpTileBytes);
        static std::atomic<uint64_t> smem_set{0};  // devices whose limit is raised
        if (int arc = set_max_dynamic_smem(q4_0_gemv_stream_kernel, 200 * 1024, smem_set)) return arc;
        ANE_ARG_CHECK(p.smem <= 200 * 1024, "q4_0_gemv: shared-memory plan too large");
        const uint64_t row_bytes = (uint64_t)(K / 32) * kQ4BlockBytes;
        CUtensorMap wmap;
        int rc = encode_tensor_map_2d(&wmap, CU_TENSOR_MAP_DATA_TYPE_UINT32, W, row_bytes / 4, M, row_bytes,
                                      kQ4ChunkBytes / 4, kQ8RowsPerWarp, CU_TENSOR_MAP_SWIZZLE_NONE);
        if (rc) return rc;
        return launch_q8_stream(q4_0_gemv_stream_kernel, p, s, wmap, W, x, out, M, K, p.groups, p.warps, p.slots,
                                flags, device_timeout_flag());
    }
    q4_0_gemv_simple_kernel<<<(M + 127) / 128, 128, 0, s>>>(x, W, out, M, K);
    ANE_CHECK_LAUNCH();
    return ANE_OK;
}

}  // namespace ane_b200
