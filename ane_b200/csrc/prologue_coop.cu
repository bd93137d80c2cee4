// prologue_coop.cu -- the dense_fused_i8 quantize prologue as ONE cooperative,
// persistent kernel that reads each fp32 tensor from HBM exactly once.
//
// Per tensor the prologue needs two passes: the per-tensor absmax
// (quantize_fp32_i8, src/bytecode_interpreter.s:1876-1950) must be complete
// before the first code can be produced.  At M=N=K=4096 each fp32 tensor is
// 64 MB, more than the part of the 126 MB L2 that keeps a re-read tensor, so a
// second pass would stream it from HBM again.  Here each tensor is split into
//   * a RESIDENT part: CTA c (one per SM) owns a fixed 192 KB slice that
//     bulk copies bring into its shared memory during the absmax pass
//     (~28 MB over 148 SMs); the quantize pass reads it from there;
//   * a REMAINDER, handed out in 64 KB chunks (A) or 64 KB units (B) through
//     per-phase work counters, so CTAs that stream faster take more and all
//     finish together; the absmax pass marks it evict_last in L2 and the
//     quantize pass reads it back from L2.
// HBM traffic per call: A and B once (fp32) plus Aq and Bt (int8).
//
//   A1  resident A slice -> smem (bulk copies); remainder chunks: absmax;
//       absmax of the smem slice; atomicMax into the launch's abs_a  | barrier
//   A2  codes of the smem slice -> Aq; then B's resident units are requested
//       into the freed shared memory (TMA) while the A remainder is quantized
//       from L2 -> Aq
//   B1  remainder units of B: absmax; then the resident units in smem;
//       atomicMax into abs_b                                          | barrier
//   B2  per unit (32 rows x 512 columns), codes transposed through shared
//       memory -> one aligned 32-byte run per Bt row; resident units first,
//       then remainder units refilled into the freed slots by TMA from L2,
//       two units ahead of the arithmetic
//
// Each launch takes one of kSlots per-device control blocks (round robin on
// the host), so launches that overlap on the GPU from different streams never
// share counters.  Every word of a block is zero between launches: after each
// grid barrier CTA 0 zeroes the counters of the phases that just ended, the
// last CTA to finish zeroes the rest.  Every wait is bounded and records a
// device timeout instead of hanging; after a timeout the block may be left
// mid-count and the device must be treated as failed.
#include <cuda.h>
#include <string.h>

#include <atomic>

#include "ane_internal.cuh"
#include "sm100_ptx.cuh"

namespace ane_b200 {
namespace {

constexpr int kCoopThreads = 512;
// B is handled in units of 32 rows x 512 columns (64 KB of fp32); a unit's codes
// form one aligned 32-byte run in each of 512 rows of Bt.
constexpr uint32_t kUnitRows = 32, kUnitCols = 512, kUnitF4 = kUnitRows * kUnitCols / 4;
constexpr uint32_t kCacheSlots = 3;                    // resident B units per CTA
constexpr uint32_t kCacheF4 = kCacheSlots * kUnitF4;  // 192 KB: also A's resident slice
constexpr size_t kCoopSmem = (size_t)kCacheF4 * 16;   // dynamic; + ~17 KB static staging
constexpr uint32_t kStageRow = kUnitCols + 4;         // staged words per 4-row group (16-byte rows)
constexpr uint32_t kChunkF4 = kCoopThreads * 8;       // remainder chunk of A: 8 float4 per thread (64 KB)
constexpr uint32_t kBulkPieceF4 = kCacheF4 / 4;       // resident A slice in 4 bulk copies of 48 KB
constexpr uint32_t kNone = 0xffffffffu;
constexpr uint32_t kSlots = 16;  // control blocks per device
static_assert(kCoopSmem > 114 * 1024, "more than half of an SM: one resident CTA per SM");
static_assert(kUnitCols == kCoopThreads, "one column of a unit per thread");

constexpr uint32_t kOwnMax = 64;  // remainder chunks / units a CTA records in phase 1

// Control block of one launch (all zero between launches).  Every word has a
// 128-byte line of its own: the barrier's arrival count, the absmax words and
// the work counters each see a different stream of atomics.
struct alignas(128) CtlWord {
    unsigned int v;
    unsigned int pad[31];
};
struct CoopCtl {
    CtlWord bar_count;                  // grid barrier arrivals (barrier k completes at k x CTAs)
    CtlWord ctr_a1, ctr_a2, ctr_b1, ctr_b2;  // remainder work counters, one per phase
    CtlWord abs_a, abs_b;               // tensor-wide |max| as magnitude bits
    CtlWord ovf_a, ovf_b;               // some CTA took more than kOwnMax chunks / units in phase 1
    CtlWord done;                       // CTAs that finished the launch
};
__device__ CoopCtl g_coop_ctl[kSlots];

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
__device__ __forceinline__ unsigned int ld_gpu(const unsigned int* p) {
    unsigned int v;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_gpu(unsigned int* p, unsigned int v) {
    asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
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

// Grid barrier number `which` (1, 2) of the launch: every CTA adds one to the
// arrival count with a release reduction (no reply to wait for) and polls the
// count with acquire loads until it reaches which * nblocks -- one trip to L2
// per arrival and no second hop through a releasing CTA.  The count is zeroed
// by the last CTA to finish the launch.  Afterwards CTA 0 zeroes the work
// counters of the phases every CTA has now left (barrier 1: A1's; barrier 2:
// A2's, B1's, abs_a and ovf_a, which every CTA read after barrier 1).
// Returns false (and bumps *err) if the wait gave up.
__device__ bool grid_barrier(CoopCtl* ctl, unsigned int nblocks, int which, int* err) {
    __shared__ int ok_s;
    __syncthreads();
    if (threadIdx.x == 0) {
        int ok = 1;
        const unsigned int target = (unsigned int)which * nblocks;
        asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(&ctl->bar_count.v) : "memory");
        const long long t0 = clock64();
        while (true) {
            unsigned int n;
            asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(n) : "l"(&ctl->bar_count.v) : "memory");
            if (n >= target) break;
            if (clock64() - t0 > ptx::kWaitTimeoutCycles) {
                atomicAdd(err, 1);
                ok = 0;
                break;
            }
        }
        if (ok && blockIdx.x == 0) {
            if (which == 1) {
                st_gpu(&ctl->ctr_a1.v, 0u);
            } else {
                st_gpu(&ctl->ctr_a2.v, 0u);
                st_gpu(&ctl->ctr_b1.v, 0u);
                st_gpu(&ctl->abs_a.v, 0u);
                st_gpu(&ctl->ovf_a.v, 0u);
            }
        }
        ok_s = ok;
    }
    __syncwarp();  // warp 0 reconverges after lane 0's spin
    __syncthreads();
    return ok_s != 0;
}

// Next index of a work counter, the same value in every thread of the CTA.
// Consecutive grabs alternate between two broadcast words, so one
// __syncthreads per grab suffices (a word is rewritten two grabs later, after
// every thread passed the barrier of the grab in between).
__device__ __forceinline__ uint32_t grab(unsigned int* ctr, uint32_t* bcast, uint32_t& k) {
    uint32_t* w = bcast + (k++ & 1u);
    if (threadIdx.x == 0) *w = atomicAdd(ctr, 1u);
    __syncthreads();
    return *w;
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

// ------------------------------------------------------------ A (flat)
// Geometry of A's split (float4 indices): CTA c's resident slice [res0,
// res0 + nres), remainder [rem0, n) in chunks of kChunkF4.
struct ASplit {
    size_t n, res0, nres, rem0;
    uint32_t nchunks;
};
__device__ __forceinline__ ASplit a_split(size_t n, unsigned int c, unsigned int G) {
    ASplit s;
    s.n = n;
    s.res0 = min(n, (size_t)c * kCacheF4);
    s.nres = min(n, (size_t)(c + 1) * kCacheF4) - s.res0;
    s.rem0 = min(n, (size_t)G * kCacheF4);
    s.nchunks = (uint32_t)ceil_div(n - s.rem0, kChunkF4);
    return s;
}

// The thread's eight float4 of remainder chunk ch (zero past the end).
__device__ __forceinline__ void load_chunk(float4 (&v)[8], const float4* __restrict__ x4, const ASplit& s,
                                           uint32_t ch, uint64_t pol) {
    const size_t base = s.rem0 + (size_t)ch * kChunkF4 + threadIdx.x;
#pragma unroll
    for (int j = 0; j < 8; j++) {
        const size_t i = base + (size_t)j * kCoopThreads;
        v[j] = i < s.n ? ld4(x4 + i, pol) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
}

// Notes remainder item `idx` as taken by this CTA in phase 1 (the leader
// thread writes the list; every calling thread counts).  Past kOwnMax items
// the list is incomplete and the launch-wide overflow flag sends phase 2 back
// to a work counter.
__device__ __forceinline__ void record_own(uint32_t idx, uint32_t* own, uint32_t& nown, unsigned int* ovf,
                                           bool leader = threadIdx.x == 0) {
    if (leader) {
        if (nown < kOwnMax)
            own[nown] = idx;
        else if (nown == kOwnMax)
            atomicExch(ovf, 1u);
    }
    nown++;
}

// Runs body(v, ch) over the remainder chunks this CTA takes from `ctr`; chunk
// k+1 is requested before chunk k is consumed.  With `own`, the chunks taken
// are recorded (record_own) so that phase 2 can revisit the same chunks on the
// same SM, next to the L2 slice that cached them.
template <class Body>
__device__ __forceinline__ void for_each_chunk(const float4* __restrict__ x4, const ASplit& s, unsigned int* ctr,
                                               uint32_t* bcast, uint32_t& gk, uint64_t pol, uint32_t* own,
                                               uint32_t& nown, unsigned int* ovf, Body body) {
    float4 a[8], b[8];
    uint32_t cur = grab(ctr, bcast, gk);
    if (cur < s.nchunks) load_chunk(a, x4, s, cur, pol);
    while (cur < s.nchunks) {
        if (own) record_own(cur, own, nown, ovf);
        const uint32_t nxt = grab(ctr, bcast, gk);
        if (nxt < s.nchunks) load_chunk(b, x4, s, nxt, pol);
        body(a, cur);
        if (nxt >= s.nchunks) break;
        if (own) record_own(nxt, own, nown, ovf);
        cur = grab(ctr, bcast, gk);
        if (cur < s.nchunks) load_chunk(a, x4, s, cur, pol);
        body(b, nxt);
    }
}

// Phase 2 over the chunks recorded in phase 1 (no counter, no barrier).
template <class Body>
__device__ __forceinline__ void for_own_chunks(const float4* __restrict__ x4, const ASplit& s, const uint32_t* own,
                                               uint32_t nown, uint64_t pol, Body body) {
    float4 a[8], b[8];
    if (nown) load_chunk(a, x4, s, own[0], pol);
    for (uint32_t k = 0; k < nown; k += 2) {
        if (k + 1 < nown) load_chunk(b, x4, s, own[k + 1], pol);
        body(a, own[k]);
        if (k + 1 >= nown) break;
        if (k + 2 < nown) load_chunk(a, x4, s, own[k + 2], pol);
        body(b, own[k + 1]);
    }
}

template <bool FAST>
__device__ __forceinline__ void codes_of_chunk(const float4 (&v)[8], uint32_t ch, const ASplit& s, uint32_t* out,
                                               float inv) {
    const size_t base = s.rem0 + (size_t)ch * kChunkF4 + threadIdx.x;
#pragma unroll
    for (int j = 0; j < 8; j++) {
        const size_t i = base + (size_t)j * kCoopThreads;
        if (i < s.n) out[i] = pack4<FAST>(v[j], inv);
    }
}

// ------------------------------------------------------------ B (units)
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

// Units of B: CTA c's resident units [first, first + nres), remainder [rem0, U).
struct BSplit {
    uint32_t U, nch, first, nres, rem0;
};
__device__ __forceinline__ BSplit b_split(uint32_t K, uint32_t N, unsigned int c, unsigned int G) {
    BSplit s;
    s.nch = (N + kUnitCols - 1) / kUnitCols;
    s.U = ((K + kUnitRows - 1) / kUnitRows) * s.nch;
    s.first = kCacheSlots * c;
    s.nres = s.U > s.first ? min(kCacheSlots, s.U - s.first) : 0u;
    s.rem0 = min(s.U, kCacheSlots * G);
    return s;
}

// Absmax layout: thread (c4 = t % 128, r = t / 128) reads rows r + 4j (j < 8)
// of column quad c4; zero outside the unit.
__device__ __forceinline__ void load_unit_rows(float4 (&v)[kUnitRows / 4], const float4* __restrict__ B4, uint32_t N4,
                                               const BUnit& g, uint64_t pol) {
    const uint32_t c4 = threadIdx.x % (kUnitCols / 4), r = threadIdx.x / (kUnitCols / 4);
#pragma unroll
    for (uint32_t j = 0; j < kUnitRows / 4; j++) {
        const uint32_t rr = r + 4 * j;
        v[j] = (c4 < g.cols4 && rr < g.rows) ? ld4(B4 + (size_t)(g.r0 + rr) * N4 + g.c0 / 4 + c4, pol)
                                             : make_float4(0.f, 0.f, 0.f, 0.f);
    }
}

// ------------------------------------------------ A2 and B1 side by side
// While A's remainder is quantized from L2 (warps 0-7), B's remainder streams
// from HBM for its absmax (warps 8-15): the two halves of the CTA keep L2 and
// HBM busy at the same time.  Each half has kHalf threads; `lt` is the
// thread's index within its half.
constexpr uint32_t kHalf = kCoopThreads / 2;
constexpr uint32_t kBarB = 1;  // named barrier of the B half (barrier 0 is __syncthreads)

// Pass p (0, 1) of A chunk ch for a half: eight float4 per thread.
__device__ __forceinline__ void load_chunk_half(float4 (&v)[8], const float4* __restrict__ x4, const ASplit& s,
                                                uint32_t ch, uint32_t p, uint32_t lt, uint64_t pol) {
    const size_t base = s.rem0 + (size_t)ch * kChunkF4 + p * (kChunkF4 / 2) + lt;
#pragma unroll
    for (int j = 0; j < 8; j++) {
        const size_t i = base + (size_t)j * kHalf;
        v[j] = i < s.n ? ld4(x4 + i, pol) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
}
template <bool FAST>
__device__ __forceinline__ void codes_of_chunk_half(const float4 (&v)[8], uint32_t ch, uint32_t p, uint32_t lt,
                                                    const ASplit& s, uint32_t* out, float inv) {
    const size_t base = s.rem0 + (size_t)ch * kChunkF4 + p * (kChunkF4 / 2) + lt;
#pragma unroll
    for (int j = 0; j < 8; j++) {
        const size_t i = base + (size_t)j * kHalf;
        if (i < s.n) out[i] = pack4<FAST>(v[j], inv);
    }
}
// Codes of the A chunks recorded in A1, by one half: steps (chunk, pass) with
// step t+1 requested before step t is consumed; no barrier.
template <bool FAST>
__device__ void quantize_own_chunks_half(const float4* __restrict__ x4, const ASplit& s, const uint32_t* own,
                                         uint32_t nown, uint32_t lt, uint32_t* out, float inv, uint64_t pol) {
    const uint32_t steps = 2 * nown;
    float4 a[8], b[8];
    if (steps) load_chunk_half(a, x4, s, own[0], 0, lt, pol);
    for (uint32_t t = 0; t < steps; t += 2) {
        load_chunk_half(b, x4, s, own[t / 2], 1, lt, pol);
        codes_of_chunk_half<FAST>(a, own[t / 2], 0, lt, s, out, inv);
        if (t + 2 < steps) load_chunk_half(a, x4, s, own[t / 2 + 1], 0, lt, pol);
        codes_of_chunk_half<FAST>(b, own[t / 2], 1, lt, s, out, inv);
    }
}

// Half h (rows 16h .. 16h+15) of B unit g for a half of the CTA: thread
// (c4 = lt % 128, r = lt / 128) reads rows 16h + r + 2j (j < 8) of column quad
// c4; zero outside the unit.
__device__ __forceinline__ void load_unit_half(float4 (&v)[8], const float4* __restrict__ B4, uint32_t N4,
                                               const BUnit& g, uint32_t h, uint32_t lt, uint64_t pol) {
    const uint32_t c4 = lt % (kUnitCols / 4), r = lt / (kUnitCols / 4);
#pragma unroll
    for (uint32_t j = 0; j < 8; j++) {
        const uint32_t rr = 16 * h + r + 2 * j;
        v[j] = (c4 < g.cols4 && rr < g.rows) ? ld4(B4 + (size_t)(g.r0 + rr) * N4 + g.c0 / 4 + c4, pol)
                                             : make_float4(0.f, 0.f, 0.f, 0.f);
    }
}
// Next index of a work counter for the B half (its own named barrier and
// broadcast words; the same one-barrier-per-grab argument as grab()).
__device__ __forceinline__ uint32_t grab_half(unsigned int* ctr, uint32_t* bcast, uint32_t& k, uint32_t lt) {
    uint32_t* w = bcast + (k++ & 1u);
    if (lt == 0) *w = atomicAdd(ctr, 1u);
    ptx::named_barrier_sync(kBarB, kHalf);
    return *w;
}

// Codes layout: thread (c4 = t % 128, rg = t / 128) takes 4-row groups rg and
// rg + 4 of column quad c4, from a shared-memory copy of the unit (32 rows x
// 512 columns, row pitch 128 float4; zero outside the unit) ...
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
// ... or straight from global memory (L2).
__device__ __forceinline__ void unit_from_global(float4 (&v)[2][4], const float4* __restrict__ B4, uint32_t N4,
                                                 const BUnit& g, uint32_t c4, uint32_t rg, uint64_t pol) {
    const uint32_t groups = g.rows / 4;
#pragma unroll
    for (uint32_t h = 0; h < 2; h++) {
        const uint32_t gi = rg + 4 * h;
#pragma unroll
        for (int i = 0; i < 4; i++)
            v[h][i] = (c4 >= g.cols4 || gi >= groups)
                          ? make_float4(0.f, 0.f, 0.f, 0.f)
                          : ld4(B4 + (size_t)(g.r0 + 4 * gi + i) * N4 + g.c0 / 4 + c4, pol);
    }
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

// Phase B2: codes of this CTA's resident units and of its remainder units,
// transposed into Bt.  The remainder units are the ones this CTA streamed in
// B1 (own[0..nown), so they come from the L2 slice next to this SM), or, if
// some CTA's list overflowed (use_own false), units taken from ctr_b2.  With
// the tensor map, the slots form a ring: after slot s's values are in
// registers, the next remainder unit is requested into slot s (one 3-D TMA
// box, from L2 where B1 left it), so copies run two units ahead of the
// arithmetic.  Without it (N % 256 != 0), remainder units are read from L2
// directly.  Returns false if a copy did not arrive in time (device timeout
// recorded).
template <bool FAST>
__device__ bool quantize_b_units(const float4* __restrict__ B4, uint32_t N4, uint32_t K, uint32_t N, const BSplit& s,
                                 float4* cache, uint32_t* stage, int8_t* __restrict__ Bt, float inv,
                                 const CUtensorMap* bmap, uint64_t* tbar, CoopCtl* ctl, uint32_t* bcast,
                                 uint32_t& gk, const uint32_t* own, uint32_t nown, bool use_own, int* err) {
    __shared__ uint32_t slot_unit[kCacheSlots];
    const uint64_t once = policy_evict_first();
    const uint32_t c4 = threadIdx.x % (kUnitCols / 4), rg = threadIdx.x / (kUnitCols / 4);
    if (!bmap) {
        for (uint32_t k = 0; k < s.nres; k++) {
            const BUnit g = b_unit(s.first + k, s.nch, K, N);
            float4 cur[2][4];
            unit_from_smem(cur, cache + k * kUnitF4, g, c4, rg);
            unit_codes_out<FAST>(cur, g, c4, rg, stage, Bt, K, inv);
        }
        for (uint32_t k = 0;; k++) {
            const uint32_t u = use_own ? (k < nown ? own[k] : kNone) : s.rem0 + grab(&ctl->ctr_b2.v, bcast, gk);
            if (u >= s.U) break;
            const BUnit g = b_unit(u, s.nch, K, N);
            float4 cur[2][4];
            unit_from_global(cur, B4, N4, g, c4, rg, once);
            unit_codes_out<FAST>(cur, g, c4, rg, stage, Bt, K, inv);
        }
        return true;
    }
    // the resident units fill the slots first; when this CTA has fewer than
    // kCacheSlots of them (a small B), it has no remainder units either
    if (threadIdx.x == 0)
        for (uint32_t k = 0; k < kCacheSlots; k++) slot_unit[k] = k < s.nres ? s.first + k : kNone;
    __syncthreads();
    uint32_t next_own = 0;  // thread 0: next entry of own[] to request
    for (uint32_t k = 0;; k++) {
        const uint32_t slot = k % kCacheSlots;
        const uint32_t u = slot_unit[slot];  // written three iterations ago, barriers in between
        if (u == kNone) break;               // CTA-uniform; the work counter only grows, so no later slot is full
        if (k >= kCacheSlots) {
            const bool ok = ptx::mbar_wait(&tbar[slot], (k / kCacheSlots - 1) & 1, err);
            if (__syncthreads_or(!ok)) return false;
        }
        const BUnit g = b_unit(u, s.nch, K, N);
        float4 cur[2][4];
        unit_from_smem(cur, cache + slot * kUnitF4, g, c4, rg);
        __syncthreads();  // every thread holds its values: the slot may be refilled
        if (threadIdx.x == 0) {
            uint32_t nu = kNone;
            if (use_own)
                nu = next_own < nown ? own[next_own++] : kNone;
            else if (s.rem0 < s.U)
                nu = s.rem0 + atomicAdd(&ctl->ctr_b2.v, 1u);
            if (nu < s.U) {
                const BUnit gn = b_unit(nu, s.nch, K, N);
                ptx::fence_proxy_async_smem();  // the slot's generic reads before the async-proxy write
                ptx::mbar_arrive_expect_tx(&tbar[slot], kUnitF4 * 16);
                ptx::tma_load_3d_hint(cache + slot * kUnitF4, bmap, &tbar[slot], 0, (int)(gn.c0 / 256), (int)gn.r0,
                                      once);
                slot_unit[slot] = nu;
            } else {
                slot_unit[slot] = kNone;
            }
        }
        unit_codes_out<FAST>(cur, g, c4, rg, stage, Bt, K, inv);  // its barriers publish slot_unit
    }
    return true;
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
                         CoopRanks xr, const __grid_constant__ CUtensorMap bmap, uint32_t use_tma, uint32_t slot,
                         int* err) {
    extern __shared__ __align__(128) float4 cache[];  // 128-byte aligned: bulk-copy / TMA destination
    __shared__ __align__(16) uint32_t stage[kUnitRows / 4 * kStageRow];
    __shared__ uint64_t rbar[2];            // resident slice of A / resident units of B arrived
    __shared__ uint64_t tbar[kCacheSlots];  // remainder units of B refilled into the slots
    __shared__ uint32_t bcast[2], bcast_b[2];
    __shared__ uint32_t own_a[kOwnMax], own_b[kOwnMax];  // remainder items this CTA streamed in phase 1
    __shared__ uint32_t tag_s, abs_s, ovf_s, nown_b_s;
    __shared__ int fail_s;
    const unsigned int G = gridDim.x, c = blockIdx.x;
    CoopCtl* ctl = &g_coop_ctl[slot];
    const uint64_t keep = policy_evict_last(), once = policy_evict_first();
    uint32_t gk = 0;                 // grabs so far (the same in every thread)
    uint32_t nown_a = 0, nown_b = 0;  // items taken in phase 1 (the same in every thread)
    if (threadIdx.x == 0) {
        tag_s = xr.world > 1 ? *reinterpret_cast<volatile uint32_t*>(xr.ctl) + 1u : 0u;
        fail_s = 0;
        ptx::mbar_init(&rbar[0], 1);
        ptx::mbar_init(&rbar[1], 1);
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

    // ------------------------------------------------------------------ A1
    const float4* A4 = reinterpret_cast<const float4*>(A);
    const ASplit sa = a_split((size_t)M * K / 4, c, G);
    if (threadIdx.x == 0 && sa.nres) {
        ptx::mbar_arrive_expect_tx(&rbar[0], (uint32_t)(sa.nres * 16));
        for (size_t off = 0; off < sa.nres; off += kBulkPieceF4) {
            const size_t n = min((size_t)kBulkPieceF4, sa.nres - off);
            ptx::bulk_load_hint(cache + off, A4 + sa.res0 + off, (uint32_t)(n * 16), &rbar[0], once);
        }
    }
    float m = 0.0f;
    for_each_chunk(A4, sa, &ctl->ctr_a1.v, bcast, gk, keep, own_a, nown_a, &ctl->ovf_a.v,
                   [&](const float4(&v)[8], uint32_t) {
#pragma unroll
                       for (int j = 0; j < 8; j++) m = absmax4(m, v[j]);  // zero-filled past the end
                   });
    if (sa.nres) {
        const bool ok = ptx::mbar_wait(&rbar[0], 0, err);
        if (__syncthreads_or(!ok)) return;
        for (size_t i = threadIdx.x; i < sa.nres; i += kCoopThreads) m = absmax4(m, cache[i]);
    }
    // magnitudes are non-negative or NaN: their bit patterns order like the values
    uint32_t mb = block_max(__float_as_uint(m));
    if (threadIdx.x == 0) atomicMax(&ctl->abs_a.v, mb);
    if (!grid_barrier(ctl, G, 1, err)) return;

    // ------------------------------------------------------------------ A2
    if (threadIdx.x == 0) {
        abs_s = ld_gpu(&ctl->abs_a.v);
        ovf_s = ld_gpu(&ctl->ovf_a.v);
    }
    __syncthreads();
    const bool own_ok_a = ovf_s == 0;  // every CTA's chunk list is complete: revisit them
    float scale, inv;
    scale_from_absmax(rank_absmax(0, __uint_as_float(abs_s)), &scale, &inv);
    __syncthreads();
    if (fail_s) return;
    if (c == 0 && threadIdx.x == 0) scales[0] = scale;
    uint32_t* outA = reinterpret_cast<uint32_t*>(Aq);  // K % 16 == 0: Aq row stride is K, codes flat like A
    const bool fa = fast_inv(inv);
    for (size_t i = threadIdx.x; i < sa.nres; i += kCoopThreads)
        outA[sa.res0 + i] = fa ? pack4<true>(cache[i], inv) : pack4<false>(cache[i], inv);
    __syncthreads();  // the slice is read: B's resident units may land in shared memory
    const uint32_t N4 = N / 4;
    const float4* B4 = reinterpret_cast<const float4*>(B);
    const BSplit sb = b_split(K, N, c, G);
    if (use_tma && threadIdx.x == 0 && sb.nres) {
        ptx::fence_proxy_async_smem();  // the generic reads above before the async-proxy writes
        ptx::mbar_arrive_expect_tx(&rbar[1], sb.nres * kUnitF4 * 16);
        for (uint32_t k = 0; k < sb.nres; k++) {
            const BUnit g = b_unit(sb.first + k, sb.nch, K, N);
            ptx::tma_load_3d_hint(cache + k * kUnitF4, &bmap, &rbar[1], 0, (int)(g.c0 / 256), (int)g.r0, once);
        }
    }
    // ------------------------------------------------- A2 remainder | B1
    float mf = 0.0f;  // this thread's running |max| of B
    if (own_ok_a) {
        // the two halves of the CTA side by side: A's recorded chunks from L2
        // (warps 0-7) while B's remainder units stream from HBM (warps 8-15)
        if (threadIdx.x < kHalf) {
            if (fa)
                quantize_own_chunks_half<true>(A4, sa, own_a, nown_a, threadIdx.x, outA, inv, once);
            else
                quantize_own_chunks_half<false>(A4, sa, own_a, nown_a, threadIdx.x, outA, inv, once);
        } else {
            // remainder units (evict_last: B2 reads them back from L2); half 1
            // of a unit and half 0 of the next are requested before the
            // current half is consumed
            const uint32_t lt = threadIdx.x - kHalf;
            uint32_t k2 = 0, nb = 0;
            float4 h0[8], h1[8];
            uint32_t u = sb.rem0 + grab_half(&ctl->ctr_b1.v, bcast_b, k2, lt);
            if (u < sb.U) load_unit_half(h0, B4, N4, b_unit(u, sb.nch, K, N), 0, lt, keep);
            while (u < sb.U) {
                record_own(u, own_b, nb, &ctl->ovf_b.v, lt == 0);
                const BUnit g = b_unit(u, sb.nch, K, N);
                load_unit_half(h1, B4, N4, g, 1, lt, keep);
#pragma unroll
                for (int j = 0; j < 8; j++) mf = absmax4(mf, h0[j]);  // zero-filled outside the unit
                u = sb.rem0 + grab_half(&ctl->ctr_b1.v, bcast_b, k2, lt);
                if (u < sb.U) load_unit_half(h0, B4, N4, b_unit(u, sb.nch, K, N), 0, lt, keep);
#pragma unroll
                for (int j = 0; j < 8; j++) mf = absmax4(mf, h1[j]);
            }
            if (lt == 0) nown_b_s = nb;
        }
        __syncthreads();
        nown_b = nown_b_s;
    } else {
        // some CTA's chunk list overflowed: the whole CTA quantizes chunks
        // from a work counter, then streams B's remainder units
        auto codes_a = [&](const float4(&v)[8], uint32_t ch) {
            if (fa)
                codes_of_chunk<true>(v, ch, sa, outA, inv);
            else
                codes_of_chunk<false>(v, ch, sa, outA, inv);
        };
        uint32_t unused = 0;
        for_each_chunk(A4, sa, &ctl->ctr_a2.v, bcast, gk, once, nullptr, unused, nullptr, codes_a);
        float4 cur[kUnitRows / 4], nxt[kUnitRows / 4];
        auto absmax_unit = [&](const float4(&v)[kUnitRows / 4]) {
#pragma unroll
            for (uint32_t j = 0; j < kUnitRows / 4; j++) mf = absmax4(mf, v[j]);
        };
        uint32_t u = sb.rem0 + grab(&ctl->ctr_b1.v, bcast, gk);
        if (u < sb.U) load_unit_rows(cur, B4, N4, b_unit(u, sb.nch, K, N), keep);
        while (u < sb.U) {
            record_own(u, own_b, nown_b, &ctl->ovf_b.v);
            const uint32_t un = sb.rem0 + grab(&ctl->ctr_b1.v, bcast, gk);
            if (un < sb.U) load_unit_rows(nxt, B4, N4, b_unit(un, sb.nch, K, N), keep);
            absmax_unit(cur);
            if (un >= sb.U) break;
            record_own(un, own_b, nown_b, &ctl->ovf_b.v);
            u = sb.rem0 + grab(&ctl->ctr_b1.v, bcast, gk);
            if (u < sb.U) load_unit_rows(cur, B4, N4, b_unit(u, sb.nch, K, N), keep);
            absmax_unit(nxt);
        }
    }

    // ------------------------------------------------------------------ B1
    {
        float4 cur[kUnitRows / 4];
        auto absmax_unit = [&](const float4(&v)[kUnitRows / 4]) {
#pragma unroll
            for (uint32_t j = 0; j < kUnitRows / 4; j++) mf = absmax4(mf, v[j]);  // zero-filled outside the unit
        };
        // resident units: landed by TMA during A2, or read here into the slots
        if (use_tma) {
            if (sb.nres) {
                const bool ok = ptx::mbar_wait(&rbar[1], 0, err);
                if (__syncthreads_or(!ok)) return;
                for (uint32_t i = threadIdx.x; i < sb.nres * kUnitF4; i += kCoopThreads) mf = absmax4(mf, cache[i]);
            }
        } else {
            const uint32_t c4 = threadIdx.x % (kUnitCols / 4), r = threadIdx.x / (kUnitCols / 4);
            for (uint32_t k = 0; k < sb.nres; k++) {
                const BUnit g = b_unit(sb.first + k, sb.nch, K, N);
                load_unit_rows(cur, B4, N4, g, once);
                absmax_unit(cur);
                float4* dst = cache + k * kUnitF4;
#pragma unroll
                for (uint32_t j = 0; j < kUnitRows / 4; j++)
                    dst[(r + 4 * j) * (kUnitCols / 4) + c4] = cur[j];  // pitch 128 float4; zeros outside
            }
        }
        mb = block_max(__float_as_uint(mf));
    }
    if (threadIdx.x == 0) atomicMax(&ctl->abs_b.v, mb);
    if (!grid_barrier(ctl, G, 2, err)) return;

    // ------------------------------------------------------------------ B2
    if (threadIdx.x == 0) {
        abs_s = ld_gpu(&ctl->abs_b.v);
        ovf_s = ld_gpu(&ctl->ovf_b.v);
    }
    __syncthreads();
    const bool own_ok_b = ovf_s == 0;
    scale_from_absmax(rank_absmax(1, __uint_as_float(abs_s)), &scale, &inv);
    __syncthreads();
    if (fail_s) return;
    if (c == 0 && threadIdx.x == 0) scales[1] = scale;
    const CUtensorMap* bm = use_tma ? &bmap : nullptr;
    const bool done = fast_inv(inv) ? quantize_b_units<true>(B4, N4, K, N, sb, cache, stage, Bt, inv, bm, tbar, ctl,
                                                             bcast, gk, own_b, nown_b, own_ok_b, err)
                                    : quantize_b_units<false>(B4, N4, K, N, sb, cache, stage, Bt, inv, bm, tbar, ctl,
                                                              bcast, gk, own_b, nown_b, own_ok_b, err);
    if (!done) return;
    if (threadIdx.x == 0) {
        // the last CTA to finish zeroes what was used after barrier 2
        unsigned int prev;
        asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], 1;" : "=r"(prev) : "l"(&ctl->done.v) : "memory");
        if (prev == G - 1) {
            st_gpu(&ctl->bar_count.v, 0u);
            st_gpu(&ctl->ctr_b2.v, 0u);
            st_gpu(&ctl->abs_b.v, 0u);
            st_gpu(&ctl->ovf_b.v, 0u);
            st_gpu(&ctl->done.v, 0u);
        }
        // N-sharded calls: the last CTA of this GPU bumps the call count (the exchange tag)
        if (xr.world > 1) {
            const uint32_t p2 = atomicAdd(xr.ctl + 1, 1u);
            if (p2 == G - 1) {
                xr.ctl[1] = 0;
                __threadfence();
                atomicAdd(xr.ctl, 1u);
            }
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
                         float* scales, cudaStream_t s, const CoopXRank* x) {
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
    // a control block per launch, round robin: launches that overlap on the GPU
    // (other streams) use different blocks
    static std::atomic<uint32_t> next_slot{0};
    const uint32_t slot = next_slot.fetch_add(1, std::memory_order_relaxed) % kSlots;
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
    // whole B unit (32 rows x 512 columns) in the shared-memory layout of the slots
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
    ANE_CUDA_TRY(cudaLaunchKernelEx(&cfg, prologue_coop_kernel, A, B, Aq, Bt, M, N, K, scales, xr, bmap, use_tma, slot,
                                    device_timeout_flag()));
    ANE_CHECK_LAUNCH();
    return ANE_OK;
}

}  // namespace ane_b200
