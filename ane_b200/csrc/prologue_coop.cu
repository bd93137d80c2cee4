// prologue_coop.cu -- the dense_fused_i8 quantize prologue as ONE cooperative,
// persistent kernel that reads each fp32 tensor from HBM exactly once.
//
// Per tensor the prologue needs two passes: the per-tensor absmax
// (quantize_fp32_i8, src/bytecode_interpreter.s:1876-1950) must be complete
// before the first code can be produced.  At M=N=K=4096 each fp32 tensor is
// 64 MB, more than the part of the 126 MB L2 that keeps a re-read tensor, so a
// plain second pass would stream it from HBM again.  Both outputs keep their
// input's layout (Aq = codes of A, M x K; Bq = codes of B, K x N: the GEMM
// reads B as an MN-major operand), so A and B are handled alike, as flat
// arrays cut into 32 KB chunks:
//   * RESIDENT chunks: chunks 6c .. 6c+5 belong to CTA c (one CTA per SM).
//     They are the last chunks the CTA loads for a tensor and stay in its
//     shared memory until their codes are made (28 MB per tensor over 148 SMs);
//   * REMAINDER chunks: handed out by a work counter per phase, so SMs that
//     stream faster take more.  The absmax pass marks them evict_last in L2
//     and the codes pass reads them back from there.
// HBM traffic per call: A and B once (fp32) plus Aq and Bq (int8).
//
// Roles: warp 16 (one lane) is the producer: it grabs chunk indices and
// issues 1-D bulk copies into a ring of kStages 32 KB stages, each tagged with
// what the consumers must do with it.  Warps 0-15 consume the stages in the
// order they were filled.  Phases (| = grid barrier):
//   1  remainder chunks of A (absmax), resident chunks of A (absmax, kept) |
//   2  codes of A's resident chunks; remainder chunks of A from L2 (codes)
//      interleaved with remainder chunks of B (absmax); resident chunks of B
//      (absmax, kept) |
//   3  codes of B's resident chunks; remainder chunks of B from L2 (codes)
// The producer never waits at a grid barrier: while the consumers wait for the
// tensor-wide absmax it already streams the next phase's chunks into the free
// stage.  One stage is always free at a phase boundary (6 resident chunks,
// 7 stages).
//
// Each launch takes one of kSlots per-device control blocks (round robin on
// the host), so launches that overlap on the GPU from different streams never
// share counters.  Every word of a block is zero between launches: after each
// grid barrier CTA 0 zeroes what every CTA is done with, the last CTA to
// finish zeroes the rest.  Every wait is bounded and records a device timeout
// instead of hanging; after a timeout the block may be left mid-count (and
// bulk copies may still be landing in a CTA that left), so the device must be
// treated as failed.
#include <string.h>

#include <atomic>

#include "ane_internal.cuh"
#include "sm100_ptx.cuh"

namespace ane_b200 {
namespace {

constexpr uint32_t kConsumers = 512;                  // warps 0-15
constexpr uint32_t kThreads = kConsumers + 32;        // + producer warp 16
constexpr uint32_t kChunkF4 = 2048;                   // 32 KB of fp32 per chunk / stage
constexpr uint32_t kStages = 7;
constexpr uint32_t kResident = 6;                     // resident chunks per CTA and tensor
constexpr size_t kCoopSmem = (size_t)kStages * kChunkF4 * 16;  // 224 KB dynamic
constexpr uint32_t kSlots = 16;                       // control blocks per device
constexpr uint32_t kBarConsumers = 1;                 // named barrier of the consumer warps
static_assert(kResident < kStages, "a free stage at every phase boundary");
static_assert(kChunkF4 % kConsumers == 0, "whole float4s per consumer thread");
static_assert(kCoopSmem > 114 * 1024, "more than half of an SM: one resident CTA per SM");

// Stage tags (what the consumers do with a filled stage).
constexpr uint32_t kTagAbsmax = 0;     // absmax, release the stage
constexpr uint32_t kTagAbsmaxRes = 1;  // absmax, keep (a resident chunk)
constexpr uint32_t kTagCodes = 2;      // codes, release
constexpr uint32_t kTagEnd = 3;        // no data: the phase (or the CTA's stream) ends here
constexpr uint32_t kTagB = 1u << 8;    // the stage holds a chunk of B (else of A)
constexpr uint32_t kTagLast = 0x80000000u;  // flag: last load of the phase
struct StageMeta {
    uint32_t tag;    // kTag* | kTagB | kTagLast
    uint32_t chunk;  // chunk index within its tensor
};

// Control block of one launch (all zero between launches).  Every word has a
// 128-byte line of its own: each sees a different stream of atomics.
struct alignas(128) CtlWord {
    unsigned int v;
    unsigned int pad[31];
};
// A grid barrier's arrival count and the tensor-wide absmax it publishes share
// one 8-byte word, so the poll that sees the last arrival also reads the max.
struct alignas(128) BarWord {
    unsigned int count;  // CTAs arrived
    unsigned int abs;    // |max| so far as magnitude bits (NaN > inf > finite)
    unsigned int pad[30];
};
struct CoopCtl {
    BarWord bar_a, bar_b;                    // barrier 1 (absmax of A), barrier 2 (absmax of B)
    CtlWord ctr_a1, ctr_a2, ctr_b1, ctr_b2;  // remainder counters: A absmax, A codes, B absmax, B codes
    CtlWord done;                            // CTAs that finished the launch
};
__device__ CoopCtl g_coop_ctl[kSlots];

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
__device__ __forceinline__ void st_gpu(unsigned int* p, unsigned int v) {
    asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void st_gpu64(void* p, unsigned long long v) {
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ void consumers_sync() { ptx::named_barrier_sync(kBarConsumers, kConsumers); }
// AND of `v` over the consumer threads (and a barrier among them).
__device__ __forceinline__ bool consumers_and(bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "barrier.red.and.pred q, %2, %3, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)v), "r"(kBarConsumers), "r"(kConsumers)
        : "memory");
    return r != 0;
}

// Max over the consumer threads (magnitude bits order like the values).
__device__ uint32_t consumers_max(uint32_t v, uint32_t* red) {
    for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    consumers_sync();
    if (l == 0) red[w] = v;
    consumers_sync();
    v = l < (int)(kConsumers / 32) ? red[l] : 0u;
    for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
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
__device__ __forceinline__ uint32_t pack4_general(float4 v, float inv) {
    return q8(v.x, inv) | (q8(v.y, inv) << 8) | (q8(v.z, inv) << 16) | (q8(v.w, inv) << 24);
}
__device__ __forceinline__ bool fast_inv(float inv) { return inv > 0.0f && inv < __int_as_float(0x7f800000); }

// One flat fp32 tensor of n float4 (n % 4 == 0: whole 16-byte code words).
struct Flat {
    const float4* x;
    uint32_t* codes;      // 4 codes per float4, the tensor's own layout
    size_t n;             // float4s
    uint32_t nchunks;     // ceil(n / kChunkF4)
    uint32_t rem0;        // first remainder chunk (kResident x CTAs)
    uint32_t res0, nres;  // this CTA's resident chunks
};
__device__ __forceinline__ Flat make_flat(const float* x, int8_t* q, size_t count, unsigned int c, unsigned int G) {
    Flat f;
    f.x = reinterpret_cast<const float4*>(x);
    f.codes = reinterpret_cast<uint32_t*>(q);
    f.n = count / 4;
    f.nchunks = (uint32_t)ceil_div(f.n, kChunkF4);
    f.rem0 = min(f.nchunks, kResident * G);
    f.res0 = min(f.nchunks, kResident * c);
    f.nres = min(f.nchunks, kResident * (c + 1)) - f.res0;
    return f;
}
__device__ __forceinline__ uint32_t chunk_bytes(const Flat& f, uint32_t ch) {
    return (uint32_t)(min((size_t)kChunkF4, f.n - (size_t)ch * kChunkF4) * 16);
}

// Absmax of one stage holding chunk ch of a tensor of n float4: thread t
// reads float4 t, t+512, ... (conflict-free).  Tensor fields are passed by
// value: a reference chosen at run time would put both tensors' descriptions
// in local memory, which misses the small L1 left beside 224 KB of shared memory.
__device__ __forceinline__ float stage_absmax(float m, const float4* st, size_t n, uint32_t ch) {
    const size_t base = (size_t)ch * kChunkF4;
    float4 v[kChunkF4 / kConsumers];
#pragma unroll
    for (uint32_t j = 0; j < kChunkF4 / kConsumers; j++) {
        const uint32_t i = threadIdx.x + j * kConsumers;
        v[j] = base + i < n ? st[i] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (uint32_t j = 0; j < kChunkF4 / kConsumers; j++) m = absmax4(m, v[j]);
    return m;
}
// Codes of one stage, one 32-bit word of 4 codes per float4 (coalesced stores).
__device__ __forceinline__ void stage_codes(const float4* st, uint32_t* codes, size_t n, uint32_t ch, float inv,
                                            bool fast) {
    const size_t base = (size_t)ch * kChunkF4;
    float4 v[kChunkF4 / kConsumers];
#pragma unroll
    for (uint32_t j = 0; j < kChunkF4 / kConsumers; j++) v[j] = st[threadIdx.x + j * kConsumers];
    if (fast) {
#pragma unroll
        for (uint32_t j = 0; j < kChunkF4 / kConsumers; j++) {
            const size_t i = base + threadIdx.x + j * kConsumers;
            if (i < n) codes[i] = pack4_fast(v[j], inv);
        }
    } else {
#pragma unroll
        for (uint32_t j = 0; j < kChunkF4 / kConsumers; j++) {
            const size_t i = base + threadIdx.x + j * kConsumers;
            if (i < n) codes[i] = pack4_general(v[j], inv);
        }
    }
}

// Grid barrier `which` (1: A, 2: B) of the launch, run by consumer thread 0
// with its CTA's |max| (magnitude bits): an atomic max into the barrier word
// whose reply is waited for, so the max is performed at the word's L2 slice
// before the arrival that follows it to the same 8-byte word; then acquire
// polls of the whole word until every CTA arrived.  The poll that sees the
// last arrival carries the tensor-wide max, returned in *abs.  Afterwards CTA 0
// zeroes what every CTA is done with (barrier 1: A's absmax counter; barrier 2:
// A's codes counter, B's absmax counter and barrier 1's word, which every CTA
// left before arriving here); the last CTA of the launch zeroes the rest.
// Returns false (and bumps *err) if the wait gave up.
__device__ bool grid_barrier_leader(CoopCtl* ctl, unsigned int nblocks, int which, uint32_t local_abs,
                                    uint32_t* abs, int* err) {
    BarWord* w = which == 1 ? &ctl->bar_a : &ctl->bar_b;
    const unsigned int prev = atomicMax(&w->abs, local_abs);
    // the arrival is issued once the max's reply is back: its increment depends
    // on the reply (magnitude bits never have bit 31 set, so it is always 1)
    asm volatile("red.relaxed.gpu.global.add.u32 [%0], %1;" ::"l"(&w->count), "r"(1u + (prev >> 31)) : "memory");
    const long long t0 = clock64();
    unsigned long long v;
    while (true) {
        asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(&w->count) : "memory");
        if ((unsigned int)v >= nblocks) break;
        if (clock64() - t0 > ptx::kWaitTimeoutCycles) {
            atomicAdd(err, 1);
            return false;
        }
    }
    *abs = (uint32_t)(v >> 32);
    if (blockIdx.x == 0) {
        if (which == 1) {
            st_gpu(&ctl->ctr_a1.v, 0u);
        } else {
            st_gpu(&ctl->ctr_a2.v, 0u);
            st_gpu(&ctl->ctr_b1.v, 0u);
            st_gpu64(&ctl->bar_a.count, 0ull);
        }
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

// Run by all consumer threads; returns the max over ranks (bits).
__device__ uint32_t exchange_absmax(const CoopRanks& xr, uint32_t which, uint32_t local_bits, uint32_t tag,
                                    uint32_t* m_s, int* err, int* fail_s) {
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        const uint64_t w = (uint64_t)local_bits | ((uint64_t)tag << 32);
        for (uint32_t q = 0; q < xr.world; q++)
            asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(xr.slot_peer[q] + which), "l"(w) : "memory");
    }
    if (threadIdx.x == 0) *m_s = local_bits;
    consumers_sync();
    if (threadIdx.x < xr.world) {
        const uint64_t* p = xr.slots + 2 * threadIdx.x + which;
        const long long t0 = clock64();
        while (true) {
            uint64_t v;
            asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
            if ((uint32_t)(v >> 32) == tag) {
                atomicMax(m_s, (uint32_t)v);  // magnitude bits: NaN > inf > finite, like the reference's max
                break;
            }
            if (clock64() - t0 > ptx::kWaitTimeoutCycles) {
                atomicAdd(err, 1);
                *fail_s = 1;
                break;
            }
            __nanosleep(64);
        }
    }
    __syncwarp();
    consumers_sync();
    return *m_s;
}

// ------------------------------------------------------------ producer
struct Producer {
    float4* stages;
    uint64_t* full;
    uint64_t* empty;
    StageMeta* meta;
    uint32_t k;  // loads issued so far
    int* err;
    bool alive;

    // Waits until stage k % kStages is free (its previous load, k - kStages,
    // consumed), tags it and requests `bytes` from `src` into it (a tag-only
    // stage when bytes == 0).
    __device__ __forceinline__ void issue(const float4* src, uint32_t bytes, uint32_t tag, uint32_t chunk,
                                          uint64_t pol) {
        if (!alive) return;
        const uint32_t s = k % kStages;
        if (k >= kStages && !ptx::mbar_wait(&empty[s], (k / kStages - 1) & 1, err)) {
            alive = false;
            return;
        }
        meta[s].tag = tag;
        meta[s].chunk = chunk;
        if (bytes) {
            ptx::mbar_arrive_expect_tx(&full[s], bytes);
            ptx::bulk_load_hint(stages + (size_t)s * kChunkF4, src, bytes, &full[s], pol);
        } else {
            ptx::mbar_arrive(&full[s]);
        }
        k++;
    }
    __device__ __forceinline__ void chunk(const Flat& f, uint32_t ch, uint32_t tag, uint64_t pol) {
        issue(f.x + (size_t)ch * kChunkF4, chunk_bytes(f, ch), tag, ch, pol);
    }
    // Remainder chunks of f taken from work counter `ctr` until none is left;
    // each index is requested one step before it is used, so the atomic's round
    // trip overlaps the wait for a free stage.
    __device__ __forceinline__ void remainder(const Flat& f, unsigned int* ctr, uint32_t tag, uint64_t pol) {
        uint32_t i = atomicAdd(ctr, 1u);
        while (f.rem0 + i < f.nchunks && alive) {
            const uint32_t nxt = atomicAdd(ctr, 1u);
            chunk(f, f.rem0 + i, tag, pol);
            i = nxt;
        }
    }
    // The CTA's resident chunks of f, the last one flagged as the phase's last load.
    __device__ __forceinline__ void resident(const Flat& f, uint32_t tensor_bit, uint64_t pol) {
        for (uint32_t i = 0; i < f.nres; i++)
            chunk(f, f.res0 + i, kTagAbsmaxRes | tensor_bit | (i + 1 == f.nres ? kTagLast : 0u), pol);
    }
};

__global__ void __launch_bounds__(kThreads, 1)
    prologue_coop_kernel(const float* __restrict__ A, const float* __restrict__ B, int8_t* __restrict__ Aq,
                         int8_t* __restrict__ Bq, uint32_t M, uint32_t N, uint32_t K, float* __restrict__ scales,
                         const __grid_constant__ CoopRanks xr, uint32_t slot, int* err) {
    extern __shared__ __align__(128) float4 stages[];  // kStages x 32 KB; bulk-copy destinations
    __shared__ uint64_t full[kStages], empty[kStages];
    __shared__ StageMeta meta[kStages];
    __shared__ uint32_t red[kConsumers / 32];
    __shared__ uint32_t tag_s, abs_s, m_s;
    __shared__ int fail_s;
    const unsigned int G = gridDim.x, c = blockIdx.x;
    CoopCtl* ctl = &g_coop_ctl[slot];
    const Flat fa = make_flat(A, Aq, (size_t)M * K, c, G);
    const Flat fb = make_flat(B, Bq, (size_t)K * N, c, G);
    if (threadIdx.x == 0) {
        fail_s = 0;
        for (uint32_t i = 0; i < kStages; i++) {
            ptx::mbar_init(&full[i], 1);                  // the producer's arrive (+ the copy's bytes)
            ptx::mbar_init(&empty[i], kConsumers / 32);  // one arrive per consumer warp
        }
        ptx::fence_mbarrier_init();
    }
    // Programmatic dependent launch: the next kernel (the GEMM) may be scheduled
    // now -- its CTAs take an SM only when a CTA of this grid leaves it -- and
    // this grid's set-up above overlapped the previous kernel; nothing in global
    // memory is touched before that kernel has finished.
    ptx::griddep_launch_dependents();
    ptx::griddep_wait();
    if (threadIdx.x == 0) tag_s = xr.world > 1 ? *reinterpret_cast<volatile uint32_t*>(xr.ctl) + 1u : 0u;
    __syncthreads();

    if (threadIdx.x >= kConsumers) {
        // ------------------------------------------------------ producer
        if (threadIdx.x != kConsumers) return;
        Producer p{stages, full, empty, meta, 0u, err, true};
        const uint64_t keep = policy_evict_last(), once = policy_evict_first();
        // phase 1: A's remainder (kept in L2 for its codes), then A's resident chunks
        if (fa.nres) {
            p.remainder(fa, &ctl->ctr_a1.v, kTagAbsmax, keep);
            p.resident(fa, 0, once);
        }
        // phase 2: A's remainder again (codes, last read) beside B's remainder
        // (absmax, kept in L2), then B's resident chunks
        if (fb.nres || fa.nres) {
            bool more_a = fa.nres != 0, more_b = fb.nres != 0;
            uint32_t ia = more_a ? atomicAdd(&ctl->ctr_a2.v, 1u) : 0u;
            uint32_t ib = more_b ? atomicAdd(&ctl->ctr_b1.v, 1u) : 0u;
            while ((more_a || more_b) && p.alive) {
                if (more_a) {
                    if (fa.rem0 + ia < fa.nchunks) {
                        const uint32_t nxt = atomicAdd(&ctl->ctr_a2.v, 1u);
                        p.chunk(fa, fa.rem0 + ia, kTagCodes, once);
                        ia = nxt;
                    } else {
                        more_a = false;
                    }
                }
                if (more_b) {
                    if (fb.rem0 + ib < fb.nchunks) {
                        const uint32_t nxt = atomicAdd(&ctl->ctr_b1.v, 1u);
                        p.chunk(fb, fb.rem0 + ib, kTagAbsmax | kTagB, keep);
                        ib = nxt;
                    } else {
                        more_b = false;
                    }
                }
            }
            if (fb.nres)
                p.resident(fb, kTagB, once);
            else
                p.issue(nullptr, 0, kTagEnd | kTagLast, 0, 0);  // no B chunks here: end of phase 2
        }
        // phase 3: B's remainder from L2 (codes), then the end of the stream
        if (fb.nres) {
            p.remainder(fb, &ctl->ctr_b2.v, kTagCodes | kTagB, once);
            p.issue(nullptr, 0, kTagEnd | kTagLast, 0, 0);
        }
        return;
    }

    // ---------------------------------------------------------- consumers
    const int lane = threadIdx.x & 31;
    uint32_t kc = 0;  // loads consumed (waited for) so far, the same in every consumer thread
    // Resident chunks are the last loads of their phase, consumed in order:
    // resident chunk i sits in stage (res_first + i) % kStages.  (A register,
    // not an array: with 224 KB of shared memory there is almost no L1 left for
    // a local-memory array, and each read would be a trip to L2.)
    uint32_t res_first = 0, nres_held = 0;
    float inv_a = 0.0f, inv_b = 0.0f;
    bool fast_a = false, fast_b = false;
    bool ok = true;
    // Frees stage s for the producer.  Every lane's reads of the stage have
    // returned (their values fed the absmax or the code stores), so the arrive
    // need not order anything: a relaxed arrive does not wait for the code
    // stores still in flight, which a release arrive would.
    auto release = [&](uint32_t s) {
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive_relaxed(&empty[s]);
    };
    // Waits for load kc; returns its stage or kStages after a timeout (one
    // verdict per warp, so no lane continues alone).
    auto next = [&]() -> uint32_t {
        const uint32_t s = kc % kStages;
        const bool got = __all_sync(0xffffffffu, ptx::mbar_wait(&full[s], (kc / kStages) & 1, err));
        kc++;
        return got ? s : kStages;
    };
    // Consumes loads until the one flagged last: absmax (running max m), or
    // codes with the tensor's inverse scale.  Resident chunks stay in place.
    auto run_phase = [&](float& m) -> bool {
        while (true) {
            const uint32_t s = next();
            if (s == kStages) return false;
            const StageMeta md = meta[s];
            const uint32_t kind = md.tag & 0xffu;
            const bool isb = (md.tag & kTagB) != 0;
            const size_t n = isb ? fb.n : fa.n;
            const float4* st = stages + (size_t)s * kChunkF4;
            if (kind == kTagAbsmax || kind == kTagAbsmaxRes) {
                m = stage_absmax(m, st, n, md.chunk);
            } else if (kind == kTagCodes) {
                stage_codes(st, isb ? fb.codes : fa.codes, n, md.chunk, isb ? inv_b : inv_a, isb ? fast_b : fast_a);
            }
            if (kind == kTagAbsmaxRes) {
                if (nres_held++ == 0) res_first = kc - 1;  // codes in the next phase
            } else {
                release(s);
            }
            if (md.tag & kTagLast) return true;
        }
    };
    // Codes of the resident chunks held from the previous phase, in load order.
    auto codes_resident = [&](const Flat& f, float inv, bool fast) {
        for (uint32_t i = 0; i < nres_held; i++) {
            const uint32_t s = (res_first + i) % kStages;
            stage_codes(stages + (size_t)s * kChunkF4, f.codes, f.n, f.res0 + i, inv, fast);
            release(s);
        }
        nres_held = 0;
    };
    // Tensor-wide absmax: CTA max -> grid barrier (carrying the max) -> (ranks) -> scale.
    auto global_scale = [&](float m, int which, float* inv, bool* fast) -> bool {
        const uint32_t mb = consumers_max(__float_as_uint(m), red);
        if (threadIdx.x == 0) {
            uint32_t bits = 0;
            if (grid_barrier_leader(ctl, G, which, mb, &bits, err))
                abs_s = bits;
            else
                fail_s = 1;
        }
        consumers_sync();
        if (fail_s) return false;
        uint32_t bits = abs_s;
        if (xr.world > 1) bits = exchange_absmax(xr, (uint32_t)(which - 1), bits, tag_s, &m_s, err, &fail_s);
        if (fail_s) return false;
        float scale;
        scale_from_absmax(__uint_as_float(bits), &scale, inv);
        *fast = fast_inv(*inv);
        if (c == 0 && threadIdx.x == 0) scales[which - 1] = scale;
        return true;
    };

    // phase 1
    float ma = 0.0f, mbv = 0.0f;
    if (fa.nres) ok = run_phase(ma);
    ok = consumers_and(ok);
    if (!ok || !global_scale(ma, 1, &inv_a, &fast_a)) return;
    // phase 2
    codes_resident(fa, inv_a, fast_a);
    if (fb.nres || fa.nres) ok = run_phase(mbv);
    ok = consumers_and(ok);
    if (!ok || !global_scale(mbv, 2, &inv_b, &fast_b)) return;
    // phase 3
    codes_resident(fb, inv_b, fast_b);
    if (fb.nres) {
        float unused = 0.0f;
        if (!run_phase(unused)) return;
    }
    consumers_sync();
    if (threadIdx.x == 0) {
        // the last CTA to finish zeroes what was used after barrier 2
        unsigned int prev;
        asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], 1;" : "=r"(prev) : "l"(&ctl->done.v) : "memory");
        if (prev == G - 1) {
            st_gpu64(&ctl->bar_b.count, 0ull);
            st_gpu(&ctl->ctr_b2.v, 0u);
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
                             const int8_t* Bq) {
    // large enough that a second HBM pass would cost more than the grid
    // barriers (one small tensor is fine: its chunks simply sit with the first
    // CTAs); both tensors flat with 16-byte rows (K and N multiples of 16: the
    // code arrays are the operands' own layouts) and 16-byte aligned
    const uintptr_t align = (uintptr_t)A | (uintptr_t)B | (uintptr_t)Aq | (uintptr_t)Bq;
    return K % 16 == 0 && N % 16 == 0 && (align & 15) == 0 && M > 0 && K > 0 && N > 0 &&
           (size_t)M * K + (size_t)K * N >= ((size_t)1 << 22);
}

int launch_prologue_coop(uint32_t M, uint32_t N, uint32_t K, const float* A, const float* B, int8_t* Aq, int8_t* Bq,
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
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = kCoopSmem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeCooperative;  // all CTAs resident: the grid barrier cannot wait on an unscheduled CTA
    attr[0].val.cooperative = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 2 : 1;
    ANE_CUDA_TRY(cudaLaunchKernelEx(&cfg, prologue_coop_kernel, A, B, Aq, Bq, M, N, K, scales, xr, slot,
                                    device_timeout_flag()));
    ANE_CHECK_LAUNCH();
    return ANE_OK;
}

}  // namespace ane_b200
