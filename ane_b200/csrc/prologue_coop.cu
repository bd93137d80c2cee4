// prologue_coop.cu -- the dense_fused_i8 quantize prologue as ONE cooperative,
// persistent kernel that reads each fp32 tensor from HBM exactly once.
//
// Per tensor the prologue needs two passes: the per-tensor absmax
// (quantize_fp32_i8, src/bytecode_interpreter.s:1876-1950) must be complete
// before the first code can be produced.  At M=N=K=4096 each fp32 tensor is
// 64 MB, more than the part of the 126 MB L2 that keeps a re-read tensor, so a
// second pass streams it from HBM again.  Here every CTA (one per SM) owns a
// contiguous slice of the tensor; during the absmax pass it keeps the first
// 192 KB of its slice in shared memory (~28 MB over 148 SMs) and marks the rest
// evict_last in L2 (~36 MB); after a grid-wide barrier it quantizes from shared
// memory and L2.  HBM traffic per call: A and B once (fp32) plus Aq and Bt
// (int8) -- 160 MB at 4096^3 instead of 288 MB.
//
//   phase A1  absmax of the CTA's A slice (cache it), partials[c]      | barrier
//   phase A2  global absmax of A -> scales[0]; codes of the slice -> Aq
//   phase B1  absmax of the CTA's B units (32 rows x 512 columns; cache the
//             first three), partials[G+c]                            | barrier
//   phase B2  global absmax of B -> scales[1]; per unit, codes transposed
//             through shared memory -> one aligned 32-byte run per Bt row
//
// The grid barrier is a self-resetting sense-reversal barrier on two words of a
// per-device __device__ array (zero at module load); its waits are bounded and
// record a device timeout instead of hanging.  Two launches of this kernel can
// never be resident at once (each CTA takes more than half of an SM's shared
// memory), so one barrier per device suffices.
#include <cuda.h>
#include <string.h>

#include "ane_internal.cuh"
#include "sm100_ptx.cuh"

namespace ane_b200 {
namespace {

constexpr int kCoopThreads = 512;
// B is handled in units of 32 rows x 512 columns (64 KB of fp32); a unit's codes
// form one aligned 32-byte run in each of 512 rows of Bt.
constexpr uint32_t kUnitRows = 32, kUnitCols = 512, kUnitF4 = kUnitRows * kUnitCols / 4;
constexpr uint32_t kCacheSlots = 3;                      // units of B kept in shared memory
constexpr uint32_t kCacheF4 = kCacheSlots * kUnitF4;    // 192 KB, also the A cache
constexpr size_t kCoopSmem = (size_t)kCacheF4 * 16;     // dynamic; + 18 KB static staging
constexpr uint32_t kStageRow = kUnitCols + 4;           // staged words per 4-row group (16-byte rows)
static_assert(kCoopSmem > 114 * 1024, "more than half of an SM: one resident launch per SM");
static_assert(kUnitCols == kCoopThreads, "one column of a unit per thread");

__device__ unsigned int g_coop_barrier[2];  // {arrivals, generation}

// m is a running magnitude (>= 0 or NaN); every element enters through its |.|
__device__ __forceinline__ float absmax4(float m, float4 v) {
    const float xy = ptx::absmax_nan(fabsf(v.x), v.y), zw = ptx::absmax_nan(fabsf(v.z), v.w);
    return ptx::absmax_nan(ptx::absmax_nan(m, xy), zw);
}
__device__ __forceinline__ uint64_t policy_evict_last() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ uint64_t policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ float4 ld4(const float4* ptr, uint64_t pol) {
    float4 v;
    asm volatile("ld.global.nc.L2::cache_hint.v4.f32 {%0, %1, %2, %3}, [%4], %5;"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "l"(ptr), "l"(pol));
    return v;
}

__device__ uint32_t block_max(uint32_t v) {
    __shared__ uint32_t red[kCoopThreads / 32];
    for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) red[w] = v;
    __syncthreads();
    v = l < kCoopThreads / 32 ? red[l] : 0u;
    for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Sense-reversal grid barrier.  Returns false (and bumps *err) if the wait
// gave up after ~2 s.
__device__ bool grid_barrier(unsigned int nblocks, int* err) {
    __shared__ int ok_s;
    unsigned int* bar = g_coop_barrier;
    __syncthreads();
    if (threadIdx.x == 0) {
        int ok = 1;
        unsigned int gen, prev;
        asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(gen) : "l"(bar + 1) : "memory");
        asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], 1;" : "=r"(prev) : "l"(bar) : "memory");
        if (prev == nblocks - 1) {
            asm volatile("st.relaxed.gpu.global.u32 [%0], 0;" ::"l"(bar) : "memory");
            asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(bar + 1) : "memory");
        } else {
            const long long t0 = clock64();
            while (true) {
                unsigned int g;
                asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(g) : "l"(bar + 1) : "memory");
                if (g != gen) break;
                if (clock64() - t0 > ptx::kWaitTimeoutCycles) {
                    atomicAdd(err, 1);
                    ok = 0;
                    break;
                }
                __nanosleep(32);
            }
        }
        ok_s = ok;
    }
    __syncwarp();  // warp 0 reconverges after lane 0's spin
    __syncthreads();
    return ok_s != 0;
}

__device__ __forceinline__ void scale_from_absmax(float absmax, float* scale, float* inv) {
    if (absmax == 0.0f) {
        *scale = 1.0f;
        *inv = 127.0f;
    } else {  // NaN is unordered and takes this path, as the reference's fcmp/b.eq does
        *scale = __fdiv_rn(absmax, 127.0f);
        *inv = __fdiv_rn(127.0f, absmax);
    }
}

// ------------------------------------------------------------ int8 codes
// General rule, per element: q = rint_even(min(max(RN(x*inv), -127), 127)), NaN -> 0.
__device__ __forceinline__ uint32_t q8(float x, float inv) {
    float y = __fmul_rn(x, inv);
    if (y != y) return 0u;
    y = fminf(fmaxf(y, -127.0f), 127.0f);
    return (uint32_t)(uint8_t)(int8_t)__float2int_rn(y);
}
// Fast rule, valid when 0 < inv < inf: then no x is inf/NaN (absmax would be)
// and |RN(x*inv)| <= 127*(1 + 2^-23) < 127.5 for |x| <= absmax, so the clamp
// never acts; RN(y + 1.5*2^23) has rint_even(y) in the low mantissa bits, whose
// low byte is the int8 code (two's complement).  One multiply and one add per
// code, no conversion unit.  The two roundings must stay separate (a fused
// multiply-add rounds ties of RN(x*inv) differently): __fmul_rn / __fadd_rn are
// never contracted.
__device__ __forceinline__ uint32_t code_bits(float x, float inv) {
    return __float_as_uint(__fadd_rn(__fmul_rn(x, inv), 12582912.0f));
}
__device__ __forceinline__ uint32_t pack4_fast(float4 v, float inv) {
    return __byte_perm(__byte_perm(code_bits(v.x, inv), code_bits(v.y, inv), 0x0040),
                       __byte_perm(code_bits(v.z, inv), code_bits(v.w, inv), 0x0040), 0x5410);
}
template <bool FAST>
__device__ __forceinline__ uint32_t pack4(float4 v, float inv) {
    if (FAST) return pack4_fast(v, inv);
    return q8(v.x, inv) | (q8(v.y, inv) << 8) | (q8(v.z, inv) << 16) | (q8(v.w, inv) << 24);
}
__device__ __forceinline__ bool fast_inv(float inv) { return inv > 0.0f && inv < __int_as_float(0x7f800000); }

// ----------------------------------------------------------------- phases
// Batches of 8 float4 per thread (64 KB per CTA); the streaming loops
// are ping-pong pipelined: batch k+1 is requested before batch k is consumed.
constexpr size_t kBatch = (size_t)kCoopThreads * 8;

__device__ __forceinline__ void load_batch(float4 (&v)[8], const float4* __restrict__ x4, size_t base, size_t n,
                                           uint64_t pol_lo, uint64_t pol_hi, size_t split) {
#pragma unroll
    for (int j = 0; j < 8; j++) {
        const size_t i = base + threadIdx.x + (size_t)j * kCoopThreads;
        v[j] = i < n ? ld4(x4 + i, i < split ? pol_lo : pol_hi) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
}

// Absmax (as a float magnitude) of x4[0..n); the first min(n, kCacheF4) float4
// are copied to `cache` (read once: evict_first), the rest stay in L2 (evict_last).
__device__ float absmax_and_cache(const float4* __restrict__ x4, size_t n, float4* cache) {
    const uint64_t keep = policy_evict_last(), once = policy_evict_first();
    float m = 0.0f;
    auto consume = [&](const float4 (&v)[8], size_t base) {
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const size_t i = base + threadIdx.x + (size_t)j * kCoopThreads;
            m = absmax4(m, v[j]);
            if (i < kCacheF4 && i < n) cache[i] = v[j];
        }
    };
    float4 a[8], b[8];
    load_batch(a, x4, 0, n, once, keep, kCacheF4);
    for (size_t base = 0; base < n; base += 2 * kBatch) {
        if (base + kBatch < n) load_batch(b, x4, base + kBatch, n, once, keep, kCacheF4);
        consume(a, base);
        if (base + kBatch >= n) break;
        if (base + 2 * kBatch < n) load_batch(a, x4, base + 2 * kBatch, n, once, keep, kCacheF4);
        consume(b, base + kBatch);
    }
    return m;
}

// Codes of the CTA's A slice: shared-memory part, then the L2 part (pipelined).
template <bool FAST>
__device__ void quantize_slice(const float4* __restrict__ A4, size_t n, const float4* cache, uint32_t* out,
                               float inv) {
    const uint64_t once = policy_evict_first();
    const size_t nc = n < kCacheF4 ? n : kCacheF4;
    float4 a[8], b[8];
    if (nc < n) load_batch(a, A4, nc, n, once, once, 0);  // first L2 batch in flight during the smem part
    for (size_t i = threadIdx.x; i < nc; i += kCoopThreads) out[i] = pack4<FAST>(cache[i], inv);
    auto consume = [&](const float4 (&v)[8], size_t base) {
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const size_t i = base + threadIdx.x + (size_t)j * kCoopThreads;
            if (i < n) out[i] = pack4<FAST>(v[j], inv);
        }
    };
    for (size_t base = nc; base < n; base += 2 * kBatch) {
        if (base + kBatch < n) load_batch(b, A4, base + kBatch, n, once, once, 0);
        consume(a, base);
        if (base + kBatch >= n) break;
        if (base + 2 * kBatch < n) load_batch(a, A4, base + 2 * kBatch, n, once, once, 0);
        consume(b, base + kBatch);
    }
}

// Geometry of B unit u: rows [r0, r0+rows), columns [c0, c0+4*cols4).
struct BUnit {
    uint32_t r0, rows, c0, cols4;
};
__device__ __forceinline__ BUnit b_unit(uint32_t u, uint32_t nch, uint32_t K, uint32_t N) {
    BUnit g;
    const uint32_t ks = u / nch, nc = u - ks * nch;
    g.r0 = ks * kUnitRows;
    g.rows = min(kUnitRows, K - g.r0);
    g.c0 = nc * kUnitCols;
    g.cols4 = min(kUnitCols, N - g.c0) / 4;
    return g;
}

// Pack, transpose and write one unit of B codes from the thread's eight float4
// (two 4-row groups of column quad c4): a 4x4 block of codes is transposed in
// registers (8 byte permutes) and staged as Bt rows; then every Bt row of the
// unit receives one aligned 32-byte run.
template <bool FAST>
__device__ __forceinline__ void unit_codes_out(const float4 (&cur)[2][4], const BUnit& g, uint32_t c4, uint32_t rg,
                                               uint32_t* stage, int8_t* __restrict__ Bt, uint32_t K, float inv) {
    const uint32_t groups = g.rows / 4;
    if (c4 < g.cols4) {
#pragma unroll
        for (uint32_t h = 0; h < 2; h++) {
            const uint32_t gi = rg + 4 * h;
            if (gi >= groups) break;
            uint32_t P[4];
#pragma unroll
            for (int i = 0; i < 4; i++) P[i] = pack4<FAST>(cur[h][i], inv);  // row 4gi+i, columns 4c4..+3
            const uint32_t t0 = __byte_perm(P[0], P[1], 0x5140), t1 = __byte_perm(P[0], P[1], 0x7362);
            const uint32_t t2 = __byte_perm(P[2], P[3], 0x5140), t3 = __byte_perm(P[2], P[3], 0x7362);
            uint4 cols;  // word j: rows 4gi..4gi+3 of column 4c4+j
            cols.x = __byte_perm(t0, t2, 0x5410);
            cols.y = __byte_perm(t0, t2, 0x7632);
            cols.z = __byte_perm(t1, t3, 0x5410);
            cols.w = __byte_perm(t1, t3, 0x7632);
            *reinterpret_cast<uint4*>(stage + gi * kStageRow + 4 * c4) = cols;
        }
    }
    __syncthreads();
    // Bt row c0 + n receives `groups` (8 or 4) consecutive words at column r0,
    // written as 16-byte pieces: piece q = (n, half), words 4*half..4*half+3
    const uint32_t cols = 4 * g.cols4, hshift = groups == 8 ? 1 : 0;
    for (uint32_t q = threadIdx.x; q < (cols << hshift); q += kCoopThreads) {
        const uint32_t n = q >> hshift, half = q & hshift;
        const uint32_t* sp = stage + 4 * half * kStageRow + n;
        const uint4 o = make_uint4(sp[0], sp[kStageRow], sp[2 * kStageRow], sp[3 * kStageRow]);
        *reinterpret_cast<uint4*>(Bt + (size_t)(g.c0 + n) * K + g.r0 + 16 * half) = o;
    }
    __syncthreads();  // stage is rewritten by the next unit
}

// The thread's eight float4 of unit g from a shared-memory copy of the unit
// (32 rows x 512 columns, row pitch 128 float4); zero outside the unit.
__device__ __forceinline__ void unit_from_smem(float4 (&v)[2][4], const float4* cu, const BUnit& g, uint32_t c4,
                                               uint32_t rg) {
    const uint32_t groups = g.rows / 4;
#pragma unroll
    for (uint32_t h = 0; h < 2; h++) {
        const uint32_t gi = rg + 4 * h;
#pragma unroll
        for (int i = 0; i < 4; i++)
            v[h][i] = (c4 >= g.cols4 || gi >= groups) ? make_float4(0.f, 0.f, 0.f, 0.f)
                                                       : cu[(4 * gi + i) * (kUnitCols / 4) + c4];
    }
}

// Codes of B units [ub0, ub1), transposed: thread (c4 = t % 128, rg = t / 128)
// takes 4-row groups g = rg, rg + 4 of column quad c4.
// With a tensor map (bmap): unit k of the CTA is read from shared-memory slot
// k % kCacheSlots -- units 0..2 are still there from the absmax phase; unit
// k + 3 is brought into slot k % 3 by one 3-D TMA box (from L2, where the
// absmax phase left it) as soon as unit k's values are in registers, so the
// copies run two units ahead of the arithmetic.  Returns false if a copy did
// not arrive in time (device timeout recorded).
// Without: the next unit's eight float4 are requested (shared memory or L2)
// before the current unit is processed.
template <bool FAST>
__device__ bool quantize_units_transposed(const float4* __restrict__ B4, uint32_t N4, uint32_t K, uint32_t N,
                                          uint32_t nch, uint32_t ub0, uint32_t ub1, float4* cache,
                                          uint32_t* stage, int8_t* __restrict__ Bt, float inv,
                                          const CUtensorMap* bmap, uint64_t* tbar, int* err) {
    const uint64_t once = policy_evict_first();
    const uint32_t c4 = threadIdx.x % (kUnitCols / 4), rg = threadIdx.x / (kUnitCols / 4);
    if (bmap) {
        const uint32_t n = ub1 - ub0;
        for (uint32_t k = 0; k < n; k++) {
            const uint32_t slot = k % kCacheSlots;
            if (k >= kCacheSlots) {
                const bool ok = ptx::mbar_wait(&tbar[slot], (k / kCacheSlots - 1) & 1, err);
                if (__syncthreads_or(!ok)) return false;
            }
            const BUnit g = b_unit(ub0 + k, nch, K, N);
            float4 cur[2][4];
            unit_from_smem(cur, cache + slot * kUnitF4, g, c4, rg);
            __syncthreads();  // every thread holds its values: the slot may be refilled
            if (threadIdx.x == 0 && k + kCacheSlots < n) {
                const BUnit gn = b_unit(ub0 + k + kCacheSlots, nch, K, N);
                ptx::fence_proxy_async_smem();  // the slot's generic accesses before the async-proxy write
                ptx::mbar_arrive_expect_tx(&tbar[slot], kUnitF4 * 16);
                ptx::tma_load_3d(cache + slot * kUnitF4, bmap, &tbar[slot], 0, (int)(gn.c0 / 256), (int)gn.r0);
            }
            unit_codes_out<FAST>(cur, g, c4, rg, stage, Bt, K, inv);
        }
        return true;
    }
    auto load_unit = [&](float4 (&v)[2][4], uint32_t u) {
        const BUnit g = b_unit(u, nch, K, N);
        const uint32_t slot = u - ub0, groups = g.rows / 4;
        if (slot < kCacheSlots) {
            unit_from_smem(v, cache + slot * kUnitF4, g, c4, rg);
            return;
        }
#pragma unroll
        for (uint32_t h = 0; h < 2; h++) {
            const uint32_t gi = rg + 4 * h;
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const uint32_t r = 4 * gi + i;
                v[h][i] = (c4 >= g.cols4 || gi >= groups)
                              ? make_float4(0.f, 0.f, 0.f, 0.f)
                              : ld4(B4 + (size_t)(g.r0 + r) * N4 + g.c0 / 4 + c4, once);
            }
        }
    };
    float4 cur[2][4], nxt[2][4];
    if (ub0 < ub1) load_unit(cur, ub0);
    for (uint32_t u = ub0; u < ub1; u++) {
        if (u + 1 < ub1) load_unit(nxt, u + 1);
        unit_codes_out<FAST>(cur, b_unit(u, nch, K, N), c4, rg, stage, Bt, K, inv);
#pragma unroll
        for (int h = 0; h < 2; h++)
#pragma unroll
            for (int i = 0; i < 4; i++) cur[h][i] = nxt[h][i];
    }
    return true;
}

__device__ float global_absmax(const float* __restrict__ partials, unsigned int n) {
    uint32_t m = 0;
    // __ldcg: written by other CTAs before the barrier; read at L2, never a stale L1 line
    for (unsigned int i = threadIdx.x; i < n; i += kCoopThreads) m = max(m, __float_as_uint(__ldcg(partials + i)));
    return __uint_as_float(block_max(m));
}

// Cross-GPU absmax (N-sharded dense_fused_i8): every rank publishes its
// tensor-wide absmax of A and of B to every rank as 64-bit {bits, tag} words
// (one store each, through CUDA-IPC peer pointers) and takes the max of all
// ranks' words carrying this call's tag, so each shard is quantized with the
// scales one GPU would compute.  tag = this GPU's call count + 1, bumped by its
// last CTA.  The exchange is also the entry handshake of a call: a rank leaves
// it only after every rank has entered the same call.
struct CoopRanks {
    uint32_t world, rank;
    uint64_t* slot_peer[8];  // on rank q: this rank's words {A, B} in q's exchange area
    const uint64_t* slots;   // this GPU's exchange area: words {A, B} of every rank
    uint32_t* ctl;           // this GPU's {calls, CTAs done}
};

__device__ __forceinline__ uint32_t exchange_absmax(const CoopRanks& xr, uint32_t which, uint32_t local_bits,
                                                    uint32_t tag, int* err, bool* ok) {
    __shared__ uint32_t m_s;
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        const uint64_t w = (uint64_t)local_bits | ((uint64_t)tag << 32);
        for (uint32_t q = 0; q < xr.world; q++)
            asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(xr.slot_peer[q] + which), "l"(w) : "memory");
    }
    if (threadIdx.x == 0) m_s = local_bits;
    __syncthreads();
    if (threadIdx.x < xr.world) {
        const uint64_t* p = xr.slots + 2 * threadIdx.x + which;
        const long long t0 = clock64();
        while (true) {
            uint64_t v;
            asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
            if ((uint32_t)(v >> 32) == tag) {
                atomicMax(&m_s, (uint32_t)v);  // magnitude bits: NaN > inf > finite, like the reference's max
                break;
            }
            if (clock64() - t0 > ptx::kWaitTimeoutCycles) {
                atomicAdd(err, 1);
                *ok = false;
                break;
            }
            __nanosleep(64);
        }
    }
    __syncwarp();
    __syncthreads();
    return m_s;
}

__global__ void __launch_bounds__(kCoopThreads, 1)
    prologue_coop_kernel(const float* __restrict__ A, const float* __restrict__ B, int8_t* __restrict__ Aq,
                         int8_t* __restrict__ Bt, uint32_t M, uint32_t N, uint32_t K, float* __restrict__ scales,
                         float* __restrict__ partials, CoopRanks xr, const __grid_constant__ CUtensorMap bmap,
                         uint32_t use_tma, int* err) {
    extern __shared__ __align__(128) float4 cache[];  // 128-byte aligned: TMA destination
    __shared__ __align__(16) uint32_t stage[kUnitRows / 4 * kStageRow];
    __shared__ uint64_t tbar[kCacheSlots];  // B units refilled into the cache slots
    __shared__ uint32_t tag_s;
    __shared__ int fail_s;
    const unsigned int G = gridDim.x, c = blockIdx.x;
    if (threadIdx.x == 0) {
        tag_s = xr.world > 1 ? *reinterpret_cast<volatile uint32_t*>(xr.ctl) + 1u : 0u;
        fail_s = 0;
        for (uint32_t i = 0; i < kCacheSlots; i++) ptx::mbar_init(&tbar[i], 1);
        ptx::fence_mbarrier_init();
    }
    __syncthreads();
    const uint32_t tag = tag_s;
    auto rank_absmax = [&](uint32_t which, float local) -> float {
        if (xr.world <= 1) return local;
        bool ok = true;
        const uint32_t m = exchange_absmax(xr, which, __float_as_uint(local), tag, err, &ok);
        if (!ok) fail_s = 1;
        return __uint_as_float(m);
    };

    // ------------------------------------------------------------------ A
    const size_t na4 = (size_t)M * K / 4;
    const size_t a0 = na4 * c / G, a1 = na4 * (c + 1) / G;
    const float4* A4 = reinterpret_cast<const float4*>(A) + a0;
    // magnitudes are non-negative or NaN: their bit patterns order like the values
    uint32_t m = block_max(__float_as_uint(absmax_and_cache(A4, a1 - a0, cache)));
    if (threadIdx.x == 0) partials[c] = __uint_as_float(m);
    if (!grid_barrier(G, err)) return;
    float scale, inv;
    scale_from_absmax(rank_absmax(0, global_absmax(partials, G)), &scale, &inv);
    __syncthreads();
    if (fail_s) return;
    if (c == 0 && threadIdx.x == 0) scales[0] = scale;
    uint32_t* outA = reinterpret_cast<uint32_t*>(Aq) + a0;  // K % 16 == 0: Aq row stride is K
    if (fast_inv(inv))
        quantize_slice<true>(A4, a1 - a0, cache, outA, inv);
    else
        quantize_slice<false>(A4, a1 - a0, cache, outA, inv);
    __syncthreads();  // the cache is reused for B

    // ------------------------------------------------------------------ B
    // Units u = ks * nch + nc (rows 32ks.., columns 512nc..); CTA c owns units
    // [U*c/G, U*(c+1)/G); the first kCacheSlots of them stay in shared memory.
    const uint32_t nks = (K + kUnitRows - 1) / kUnitRows, nch = (N + kUnitCols - 1) / kUnitCols;
    const uint32_t U = nks * nch;
    const uint32_t ub0 = (uint32_t)((uint64_t)U * c / G), ub1 = (uint32_t)((uint64_t)U * (c + 1) / G);
    const float4* B4 = reinterpret_cast<const float4*>(B);
    const uint32_t N4 = N / 4;
    {
        const uint64_t keep = policy_evict_last(), once = policy_evict_first();
        const uint32_t c4 = threadIdx.x % (kUnitCols / 4), r = threadIdx.x / (kUnitCols / 4);
        float mf = 0.0f;
        // unit u: rows r + 4j (j < 8) of column quad c4; the first kCacheSlots
        // units are read once (evict_first) into shared memory, the rest stay in
        // L2 (evict_last).  Unit u+1 is requested before unit u is consumed.
        auto load_unit = [&](float4 (&v)[kUnitRows / 4], uint32_t u) {
            const BUnit g = b_unit(u, nch, K, N);
            const uint64_t pol = u - ub0 < kCacheSlots ? once : keep;
#pragma unroll
            for (uint32_t j = 0; j < kUnitRows / 4; j++) {
                const uint32_t rr = r + 4 * j;
                v[j] = (c4 < g.cols4 && rr < g.rows) ? ld4(B4 + (size_t)(g.r0 + rr) * N4 + g.c0 / 4 + c4, pol)
                                                     : make_float4(0.f, 0.f, 0.f, 0.f);
            }
        };
        float4 cur[kUnitRows / 4], nxt[kUnitRows / 4];
        if (ub0 < ub1) load_unit(cur, ub0);
        for (uint32_t u = ub0; u < ub1; u++) {
            if (u + 1 < ub1) load_unit(nxt, u + 1);
            const BUnit g = b_unit(u, nch, K, N);
            const uint32_t slot = u - ub0;
            float4* dst = slot < kCacheSlots ? cache + slot * kUnitF4 : nullptr;
#pragma unroll
            for (uint32_t j = 0; j < kUnitRows / 4; j++) {
                const uint32_t rr = r + 4 * j;
                mf = absmax4(mf, cur[j]);  // zero-filled outside the unit
                if (dst && c4 < g.cols4 && rr < g.rows) dst[rr * (kUnitCols / 4) + c4] = cur[j];  // pitch 128 float4
            }
#pragma unroll
            for (uint32_t j = 0; j < kUnitRows / 4; j++) cur[j] = nxt[j];
        }
        m = block_max(__float_as_uint(mf));
    }
    if (threadIdx.x == 0) partials[G + c] = __uint_as_float(m);
    if (!grid_barrier(G, err)) return;
    scale_from_absmax(rank_absmax(1, global_absmax(partials + G, G)), &scale, &inv);
    __syncthreads();
    if (fail_s) return;
    if (c == 0 && threadIdx.x == 0) scales[1] = scale;
    const CUtensorMap* bm = use_tma ? &bmap : nullptr;
    const bool done = fast_inv(inv)
                          ? quantize_units_transposed<true>(B4, N4, K, N, nch, ub0, ub1, cache, stage, Bt, inv, bm, tbar, err)
                          : quantize_units_transposed<false>(B4, N4, K, N, nch, ub0, ub1, cache, stage, Bt, inv, bm, tbar, err);
    if (!done) return;
    // this call is finished on this CTA; the last CTA of this GPU bumps the call count
    if (xr.world > 1 && threadIdx.x == 0) {
        const uint32_t prev = atomicAdd(xr.ctl + 1, 1u);
        if (prev == G - 1) {
            xr.ctl[1] = 0;
            __threadfence();
            atomicAdd(xr.ctl, 1u);
        }
    }
}

}  // namespace

bool prologue_coop_supported(uint32_t M, uint32_t N, uint32_t K, const float* A, const float* B, const int8_t* Aq,
                             const int8_t* Bt) {
    // large enough that two HBM passes would cost more than the barriers;
    // 16-byte vector loads of A and B and 16-byte stores into Bt
    const uintptr_t align = (uintptr_t)A | (uintptr_t)B | (uintptr_t)Aq | (uintptr_t)Bt;
    return K % 16 == 0 && N % 4 == 0 && (align & 15) == 0 && (size_t)M * K >= ((size_t)1 << 22) &&
           (size_t)K * N >= ((size_t)1 << 22);
}

int launch_prologue_coop(uint32_t M, uint32_t N, uint32_t K, const float* A, const float* B, int8_t* Aq, int8_t* Bt,
                         float* scales, float* partials, cudaStream_t s, const CoopXRank* x) {
    CoopRanks xr{};
    xr.world = 1;
    if (x && x->world > 1) {
        ANE_ARG_CHECK(x->world <= 8 && x->rank < x->world && x->slots && x->ctl, "prologue: bad rank exchange");
        xr.world = x->world;
        xr.rank = x->rank;
        for (uint32_t q = 0; q < x->world; q++) {
            ANE_ARG_CHECK(x->slot_peer[q] && ((uintptr_t)x->slot_peer[q] & 7) == 0, "prologue: bad peer slot");
            xr.slot_peer[q] = static_cast<uint64_t*>(x->slot_peer[q]);
        }
        xr.slots = static_cast<const uint64_t*>(x->slots);
        xr.ctl = x->ctl;
    }
    static std::atomic<uint64_t> smem_set{0};  // devices whose limit is raised
    if (int arc = set_max_dynamic_smem(prologue_coop_kernel, (int)kCoopSmem, smem_set)) return arc;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)num_sms(), 1, 1);
    cfg.blockDim = dim3(kCoopThreads, 1, 1);
    cfg.dynamicSmemBytes = kCoopSmem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;  // all CTAs resident: the grid barrier cannot wait on an unscheduled CTA
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    // B as (256 columns, N / 256 column halves, K rows): one 256 x 2 x 32 box is a
    // whole B unit (32 rows x 512 columns) in the shared-memory layout of the cache
    CUtensorMap bmap;
    memset(&bmap, 0, sizeof(bmap));
    uint32_t use_tma = 0;
    if (N % 256 == 0) {
        const uint64_t dims[3] = {256, N / 256, K}, strides[2] = {1024, (uint64_t)N * 4};
        const uint32_t box[3] = {256, 2, kUnitRows};
        int rc = encode_tensor_map_3d(&bmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, B, dims, strides, box);
        if (rc) return rc;
        use_tma = 1;
    }
    ANE_CUDA_TRY(cudaLaunchKernelEx(&cfg, prologue_coop_kernel, A, B, Aq, Bt, M, N, K, scales, partials, xr, bmap,
                                    use_tma, device_timeout_flag()));
    ANE_CHECK_LAUNCH();
    return ANE_OK;
}

}  // namespace ane_b200
