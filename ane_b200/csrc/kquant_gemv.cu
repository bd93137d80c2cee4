// kquant_gemv.cu -- the K-quant matvecs q4_k_gemv (0x75), q2_k_gemv (0x76),
// q3_k_gemv (0x77), q5_k_gemv (0x78), q6_k_gemv (0x79)
// (src/bytecode_interpreter.s:11024-11620) and get_rows_q4_0 (0x7D, :12419-12466).
//
// Arithmetic of every matvec handler: rows of K/256 super-blocks; 16
// accumulator lanes, lane l taking element l of every 16-element chunk of the
// row in order with one fused multiply-add; the row result is the FADDV tree
// ((a0+a1)+(a2+a3))+... over the 16 lanes.  Element values are the handler's
// separately rounded operations (integer -> float exact, one multiply by the
// sub-block scale, one add of the sub-block min where the format has one),
// computed without the conversion unit and two lanes per packed instruction
// (the identities are stated at the decoders).  The byte layouts are the handlers' own, including q3_k's stale shift
// vector: its second 16 elements of every 32-element sub-block shift the packed
// 2-bit codes right first by the bit pattern of the x values the first half
// loaded (shifts >= 32 give 0, as SVE LSR does), then by 2l.
//
// Threads: 8 per row, thread t holding lanes 2t and 2t+1 (the first FADDV level
// in-thread, the other three by xor shuffles 1, 2, 4) -- the q4_0 / q8_0 mode-R
// lane mapping, 4 rows per compute warp.  Streamed kernel (rows whose byte
// length is a multiple of 16): the mode-R ring -- one producer warp per CTA,
// each stage = C super-blocks of every compute warp's 4 rows (one 2-D TMA box
// per warp; C = 4 for q4_k / q5_k, 8 for q2_k / q3_k / q6_k, so a box row is a
// multiple of 16 bytes) plus the matching slice of x (bulk copy); the decoders
// read shared memory.  Otherwise a direct-load kernel with the same decoders
// and lane mapping.  Loads follow each layout's alignment (144- and 176-byte
// super-blocks keep 16-byte alignment, 84-byte ones 4-byte, 110- and 210-byte
// ones only 2-byte).
#include <cuda_fp16.h>

#include <cuda.h>
#include <string.h>

#include "ane_internal.cuh"
#include "q8_stream.cuh"
#include "sm100_ptx.cuh"

namespace ane_b200 {
namespace {

enum KFormat { kQ4K = 0, kQ2K = 1, kQ3K = 2, kQ5K = 3, kQ6K = 4 };

template <int F>
struct KBlock;
template <>
struct KBlock<kQ4K> {
    static constexpr uint32_t bytes = 144, chunk = 4, elem = 4;  // super-blocks per stage, TMA element bytes
};
template <>
struct KBlock<kQ2K> {
    static constexpr uint32_t bytes = 84, chunk = 8, elem = 4;  // super-blocks per stage, TMA element bytes
};
template <>
struct KBlock<kQ3K> {
    static constexpr uint32_t bytes = 110, chunk = 8, elem = 4;  // super-blocks per stage, TMA element bytes
};
template <>
struct KBlock<kQ5K> {
    static constexpr uint32_t bytes = 176, chunk = 4, elem = 4;  // super-blocks per stage, TMA element bytes
};
template <>
struct KBlock<kQ6K> {
    static constexpr uint32_t bytes = 210, chunk = 8, elem = 8;  // super-blocks per stage, TMA element bytes
};

__device__ __forceinline__ float h2f(uint32_t bits) { return __half2float(__ushort_as_half((unsigned short)bits)); }
__device__ __forceinline__ uint32_t ld_u16(const uint8_t* p) { return *reinterpret_cast<const unsigned short*>(p); }
__device__ __forceinline__ uint32_t ld_u32_a2(const uint8_t* p) { return ld_u16(p) | (ld_u16(p + 2) << 16); }

// 6-bit scale and min of sub-block j from the 12 packed bytes s (q4_k / q5_k)
__device__ __forceinline__ void k_scale_min(const uint8_t* s, uint32_t j, uint32_t& sc, uint32_t& m) {
    if (j < 4) {
        sc = s[j] & 0x3Fu;
        m = s[j + 4] & 0x3Fu;
    } else {
        sc = (s[j + 4] & 0x0Fu) | ((uint32_t)(s[j - 4] >> 6) << 4);
        m = (uint32_t)(s[j + 4] >> 4) | ((uint32_t)(s[j] >> 6) << 4);
    }
}

// Element values without the conversion unit.  For an integer v < 2^23 the
// float with bit pattern 0x4B000000 | v is 2^23 + v exactly, so subtracting
// 2^23 (plus the format's code offset) gives the code as a float exactly -- the
// handlers' int -> float conversion.  A code left at bit position p (v = q·2^p)
// is paired with the scale times 2^-p, which is exact (a nonzero scale is at
// least 2^-24 in magnitude; 0, inf and NaN stay what they are), so every
// product is the handler's.
//
// Formats with a min compute RN(RN(q·dsc) + dmm).  dsc is an fp16 d times a
// code of at most 6 bits (<= 17 significant bits) and q has at most 5 bits, so
// q·dsc is exact and RN(RN(q·dsc) + dmm) = fma(q, dsc, dmm) for every input,
// inf and NaN included.  Formats without one compute RN((q - off)·dsc), one
// multiply.  A thread's two lanes (2t, 2t+1) share each packed operation.
constexpr uint32_t kMag = 0x4B000000u;  // 2^23
constexpr float kMagF = 8388608.0f;
__device__ __forceinline__ float mag(uint32_t v) { return __uint_as_float(kMag | v); }
// 2^23 + byte k of v
__device__ __forceinline__ float mag_byte(uint32_t v, uint32_t k) {
    return __uint_as_float(__byte_perm(v, kMag, 0x7440u + k));
}
// {fma(q0, s.x, m.x), fma(q1, s.y, m.y)} from f = {2^23 + q0, 2^23 + q1}
__device__ __forceinline__ float2 kq_min_pair(float2 f, float2 s, float2 m) {
    return ptx::ffma2(ptx::fadd2(f, make_float2(-kMagF, -kMagF)), s, m);
}
// {RN((f.x - o.x)·s.x), RN((f.y - o.y)·s.y)}, no = -o (o = 2^23 + the code offset)
__device__ __forceinline__ float2 kq_off_pair(float2 f, float2 no, float2 s) {
    return ptx::fmul2(ptx::fadd2(f, no), s);
}

// One super-block of a row for thread t's lanes 2t (acc.x) and 2t+1 (acc.y).
// sh (a constant at every call site): the row's 8 threads are converged (all
// 32 lanes of the warp call together); thread t decodes sub-block t's scale (and
// t + 8's in the 16-sub-block formats) and the others take it by a width-8
// shuffle -- the same values, decoded once per row instead of in every thread.
template <int F>
__device__ __forceinline__ void kq_superblock(const uint8_t* __restrict__ blk, const float* __restrict__ xb,
                                              uint32_t t, float2& acc, bool sh);

__device__ __forceinline__ float row_bcast(float v, uint32_t j) { return __shfl_sync(0xffffffffu, v, (int)j, 8); }

template <>
__device__ __forceinline__ void kq_superblock<kQ4K>(const uint8_t* __restrict__ blk, const float* __restrict__ xb,
                                                    uint32_t t, float2& acc, bool sh) {
    const float d = h2f(ld_u16(blk)), nd = -h2f(ld_u16(blk + 2));
    const uint8_t* qs = blk + 16;
    float tdsc = 0.0f, tdmm = 0.0f;  // sub-block t's, when shared
    if (sh) {
        uint32_t sc, mn;
        k_scale_min(blk + 4, t, sc, mn);
        tdsc = __fmul_rn(d, (float)sc);
        tdmm = __fmul_rn(nd, (float)mn);
    }
#pragma unroll
    for (uint32_t j = 0; j < 8; j++) {
        float dsc, dmm;
        if (sh) {
            dsc = row_bcast(tdsc, j);
            dmm = row_bcast(tdmm, j);
        } else {
            uint32_t sc, mn;
            k_scale_min(blk + 4, j, sc, mn);
            dsc = __fmul_rn(d, (float)sc);
            dmm = __fmul_rn(nd, (float)mn);
        }
        const uint32_t b = ld_u16(qs + 16 * j + 2 * t);  // bytes of lanes 2t, 2t+1
        const float2 xl = *reinterpret_cast<const float2*>(xb + 32 * j + 2 * t);
        const float2 xh = *reinterpret_cast<const float2*>(xb + 32 * j + 16 + 2 * t);
        const float2 m = make_float2(dmm, dmm);
        // low nibbles at bits 0 and 8 (codes x 1, x 256), high ones at 4 and 12 (x 16, x 4096)
        const float2 slo = make_float2(dsc, __fmul_rn(dsc, 0.00390625f));
        const float2 shi = make_float2(__fmul_rn(dsc, 0.0625f), __fmul_rn(dsc, 0.000244140625f));
        acc = ptx::ffma2(kq_min_pair(make_float2(mag(b & 0x000Fu), mag(b & 0x0F00u)), slo, m), xl, acc);
        acc = ptx::ffma2(kq_min_pair(make_float2(mag(b & 0x00F0u), mag(b & 0xF000u)), shi, m), xh, acc);
    }
}

template <>
__device__ __forceinline__ void kq_superblock<kQ2K>(const uint8_t* __restrict__ blk, const float* __restrict__ xb,
                                                    uint32_t t, float2& acc, bool sh) {
    const uint32_t dd = *reinterpret_cast<const uint32_t*>(blk + 80);
    const float d = h2f(dd & 0xFFFFu), nd = -h2f(dd >> 16);
    float tdsc0 = 0.0f, tdmm0 = 0.0f, tdsc1 = 0.0f, tdmm1 = 0.0f;  // sub-blocks t and t + 8, when shared
    if (sh) {
        tdsc0 = __fmul_rn(d, (float)(blk[t] & 0x0Fu));
        tdmm0 = __fmul_rn(nd, (float)(blk[t] >> 4));
        tdsc1 = __fmul_rn(d, (float)(blk[t + 8] & 0x0Fu));
        tdmm1 = __fmul_rn(nd, (float)(blk[t + 8] >> 4));
    }
#pragma unroll
    for (uint32_t j = 0; j < 16; j++) {
        float dsc, dmm;
        if (sh) {
            dsc = row_bcast(j < 8 ? tdsc0 : tdsc1, j & 7);
            dmm = row_bcast(j < 8 ? tdmm0 : tdmm1, j & 7);
        } else {
            const uint32_t s = blk[j];
            dsc = __fmul_rn(d, (float)(s & 0x0Fu));
            dmm = __fmul_rn(nd, (float)(s >> 4));
        }
        // lane 2t's code at bits 0-1 (x 1), lane 2t+1's at bits 2-3 (x 4)
        const uint32_t ws = *reinterpret_cast<const uint32_t*>(blk + 16 + 4 * j) >> (4 * t);
        const float2 xv = *reinterpret_cast<const float2*>(xb + 16 * j + 2 * t);
        const float2 sp = make_float2(dsc, __fmul_rn(dsc, 0.25f));
        acc = ptx::ffma2(kq_min_pair(make_float2(mag(ws & 3u), mag(ws & 0xCu)), sp, make_float2(dmm, dmm)), xv,
                         acc);
    }
}

template <>
__device__ __forceinline__ void kq_superblock<kQ3K>(const uint8_t* __restrict__ blk, const float* __restrict__ xb,
                                                    uint32_t t, float2& acc, bool sh) {
    const uint8_t *hm = blk, *qs = blk + 32, *sc = blk + 96;
    const float d = h2f(ld_u16(blk + 108));
    const uint32_t l0 = 2 * t, l1 = 2 * t + 1;
    auto scale_of = [&](uint32_t j) {
        const uint32_t s6 = j < 4 ? (sc[j] & 0x3Fu) : ((sc[j + 4] & 0x0Fu) | ((uint32_t)(sc[j - 4] >> 6) << 4));
        return __fmul_rn(d, (float)((int32_t)s6 - 32));
    };
    const float tdsc = sh ? scale_of(t) : 0.0f;
    // lane 2t's 3-bit code at bits 0-2 (x 1), lane 2t+1's at bits 2-4 (x 4); offset 4
    const float2 no = make_float2(-(kMagF + 4.0f), -(kMagF + 16.0f));
#pragma unroll
    for (uint32_t j = 0; j < 8; j++) {
        const float dsc = sh ? row_bcast(tdsc, j) : scale_of(j);
        const float2 sp = make_float2(dsc, __fmul_rn(dsc, 0.25f));
        const uint32_t w0 = ld_u32_a2(qs + 8 * j), h0 = ld_u16(hm + 4 * j);
        const float2 xl = *reinterpret_cast<const float2*>(xb + 32 * j + 2 * t);
        const float2 xh = *reinterpret_cast<const float2*>(xb + 32 * j + 16 + 2 * t);
        const uint32_t ws = w0 >> (4 * t);
        const uint32_t e00 = (ws & 3u) | (((h0 >> l0) & 1u) << 2);
        const uint32_t e01 = (ws & 0xCu) | (((h0 >> l1) & 1u) << 4);
        acc = ptx::ffma2(kq_off_pair(make_float2(mag(e00), mag(e01)), no, sp), xl, acc);
        // second half: the stale shift by the first half's x bits, then by 2l
        const uint32_t w1 = ld_u32_a2(qs + 8 * j + 4), h1 = ld_u16(hm + 4 * j + 2);
        const uint32_t t0 = ptx::shr_clamp(w1, __float_as_uint(xl.x)) >> (4 * t);
        const uint32_t t1 = ptx::shr_clamp(w1, __float_as_uint(xl.y)) >> (4 * t);
        const uint32_t e10 = (t0 & 3u) | (((h1 >> l0) & 1u) << 2);
        const uint32_t e11 = (t1 & 0xCu) | (((h1 >> l1) & 1u) << 4);
        acc = ptx::ffma2(kq_off_pair(make_float2(mag(e10), mag(e11)), no, sp), xh, acc);
    }
}

template <>
__device__ __forceinline__ void kq_superblock<kQ5K>(const uint8_t* __restrict__ blk, const float* __restrict__ xb,
                                                    uint32_t t, float2& acc, bool sh) {
    const float d = h2f(ld_u16(blk)), nd = -h2f(ld_u16(blk + 2));
    const uint8_t *qh = blk + 16, *qs = blk + 48;
    float tdsc = 0.0f, tdmm = 0.0f;
    if (sh) {
        uint32_t sc, mn;
        k_scale_min(blk + 4, t, sc, mn);
        tdsc = __fmul_rn(d, (float)sc);
        tdmm = __fmul_rn(nd, (float)mn);
    }
#pragma unroll
    for (uint32_t j = 0; j < 8; j++) {
        float dsc, dmm;
        if (sh) {
            dsc = row_bcast(tdsc, j);
            dmm = row_bcast(tdmm, j);
        } else {
            uint32_t sc, mn;
            k_scale_min(blk + 4, j, sc, mn);
            dsc = __fmul_rn(d, (float)sc);
            dmm = __fmul_rn(nd, (float)mn);
        }
        const uint32_t h = *reinterpret_cast<const uint32_t*>(qh + 4 * j);
        const uint32_t b = ld_u16(qs + 16 * j + 2 * t);
        const float2 xl = *reinterpret_cast<const float2*>(xb + 32 * j + 2 * t);
        const float2 xh = *reinterpret_cast<const float2*>(xb + 32 * j + 16 + 2 * t);
        // the four 5-bit codes as bytes: nibble | high bit << 4, high bits h[2t], h[2t+1],
        // h[16+2t], h[16+2t+1] moved to bits 4, 12, 20, 28 by one multiply (no carries)
        const uint32_t hb = (h >> (2 * t)) & 0x00030003u;
        const uint32_t v = ((b | (b << 12)) & 0x0F0F0F0Fu) | ((hb * 0x810u) & 0x10101010u);
        const float2 sp = make_float2(dsc, dsc), m = make_float2(dmm, dmm);
        acc = ptx::ffma2(kq_min_pair(make_float2(mag_byte(v, 0), mag_byte(v, 1)), sp, m), xl, acc);
        acc = ptx::ffma2(kq_min_pair(make_float2(mag_byte(v, 2), mag_byte(v, 3)), sp, m), xh, acc);
    }
}

template <>
__device__ __forceinline__ void kq_superblock<kQ6K>(const uint8_t* __restrict__ blk, const float* __restrict__ xb,
                                                    uint32_t t, float2& acc, bool sh) {
    const uint8_t *ql = blk, *qh = blk + 128;
    const int8_t* sc = reinterpret_cast<const int8_t*>(blk + 192);
    const float d = h2f(ld_u16(blk + 208));
    const float tdsc0 = sh ? __fmul_rn(d, (float)sc[t]) : 0.0f, tdsc1 = sh ? __fmul_rn(d, (float)sc[t + 8]) : 0.0f;
    // lane 2t's 6-bit code at bits 0-5 (x 1), lane 2t+1's at bits 4-9 (x 16); offset 32
    const float2 no = make_float2(-(kMagF + 32.0f), -(kMagF + 512.0f));
#pragma unroll
    for (uint32_t j = 0; j < 16; j++) {
        const float dsc = sh ? row_bcast(j < 8 ? tdsc0 : tdsc1, j & 7) : __fmul_rn(d, (float)sc[j]);
        const uint32_t hs = ld_u32_a2(qh + 4 * j) >> (4 * t);  // bits 0-1: lane 2t's high bits, 2-3: lane 2t+1's
        const uint32_t b = ql[8 * j + t];                      // element 2t: low nibble, 2t+1: high nibble
        const float2 xv = *reinterpret_cast<const float2*>(xb + 16 * j + 2 * t);
        const uint32_t e0 = (b & 0x0Fu) | ((hs << 4) & 0x30u);
        const uint32_t e1 = (b & 0xF0u) | ((hs << 6) & 0x300u);
        acc = ptx::ffma2(kq_off_pair(make_float2(mag(e0), mag(e1)), no, make_float2(dsc, __fmul_rn(dsc, 0.0625f))),
                         xv, acc);
    }
}

template <int F>
__global__ void __launch_bounds__(256) kquant_gemv_kernel(const float* __restrict__ x, const uint8_t* __restrict__ W,
                                                          float* __restrict__ out, uint32_t M, uint32_t nsb) {
    const uint32_t row = blockIdx.x * (blockDim.x / 8) + threadIdx.x / 8, t = threadIdx.x % 8;
    float2 acc = make_float2(0.0f, 0.0f);
    if (row < M) {
        const uint8_t* rp = W + (size_t)row * nsb * KBlock<F>::bytes;
        for (uint32_t b = 0; b < nsb; b++)
            kq_superblock<F>(rp + (size_t)b * KBlock<F>::bytes, x + 256 * b, t, acc, false);
    }
    // FADDV: level 1 in-thread (lanes 2t, 2t+1), levels 2-4 across the row's 8 threads
    float s = __fadd_rn(acc.x, acc.y);
    s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, 1));
    s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, 2));
    s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, 4));
    if (row < M && t == 0) out[row] = s;
}

// Row segments of the bulk-copy variant: a row's chunk (up to CB bytes from a
// 2-byte-aligned address) is copied as the 16-byte-aligned span around it, so a
// segment slot holds CB + 30 bytes rounded up to 16.
template <int F>
struct KSeg {
    static constexpr uint32_t CB = KBlock<F>::chunk * KBlock<F>::bytes;
    static constexpr uint32_t seg = (CB + 30 + 15) / 16 * 16;
    static constexpr uint32_t tile = kQ8RowsPerWarp * seg;
};

// The streamed matvec: stage t = chunk t % nchunks of pass t / nchunks.
// BULK = false: one 2-D TMA box per warp (rows a whole number of 16-byte units).
// BULK = true (any row length): every row's chunk arrives by one 1-D bulk copy
// of the 16-byte-aligned span around it; the producer warp's 32 lanes share the
// copies, and readers start at the chunk's offset in its span (its address mod
// 16), so every load keeps the alignment it has in global memory.
template <int F, bool BULK>
__global__ void __launch_bounds__(32 * (kQ8MaxWarps + 1), 1)
    kquant_stream_kernel(const __grid_constant__ CUtensorMap wmap, const uint8_t* __restrict__ W,
                         const float* __restrict__ x, float* __restrict__ out, uint32_t M, uint32_t nsb,
                         uint32_t groups, uint32_t nw, uint32_t nslots, uint32_t flags, int* err) {
    constexpr uint32_t BB = KBlock<F>::bytes, C = KBlock<F>::chunk, CB = C * BB;
    // one warp's 4 rows: a 128-byte-pitch TMA box, or 4 bulk-copy segments
    constexpr uint32_t TILE = BULK ? KSeg<F>::tile : (kQ8RowsPerWarp * CB + 127) / 128 * 128;
    constexpr uint32_t RPITCH = BULK ? KSeg<F>::seg : CB;
    const size_t row_bytes = (size_t)nsb * BB;
    extern __shared__ __align__(128) uint8_t smem[];
    const uint32_t nchunks = (nsb + C - 1) / C;
    const uint32_t w_bytes = nw * TILE, slot_bytes = w_bytes + C * 1024;
    auto chunk_sbs = [&](uint32_t c) { return min(C, nsb - c * C); };
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);  // nslots
    uint64_t* empty = full + nslots;                     // nslots
    uint8_t* ring = smem + 128;
    const uint32_t g0 = (uint32_t)((uint64_t)groups * blockIdx.x / gridDim.x);
    const uint32_t g1 = (uint32_t)((uint64_t)groups * (blockIdx.x + 1) / gridDim.x);
    const uint32_t npass = (g1 - g0 + nw - 1) / nw, ntiles = npass * nchunks;
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (uint32_t i = 0; i < nslots; i++) {
            ptx::mbar_init(&full[i], 1);
            ptx::mbar_init(&empty[i], nw);
        }
        ptx::fence_mbarrier_init();
    }
    __syncthreads();
    ptx::griddep_launch_dependents();

    // ANE_Q8_WEIGHTS_STATIC: the first stages' weights are requested before the
    // previous kernel on the stream has finished (it does not write W); x is
    // always requested after it has
    const uint32_t pre = (flags & ANE_Q8_WEIGHTS_STATIC) ? min(nslots, ntiles) : 0;
    auto issue_x = [&](uint32_t t, uint32_t slot) {
        const uint32_t c = t % nchunks;
        ptx::bulk_load(ring + (size_t)slot * slot_bytes + w_bytes, x + (size_t)c * C * 256, chunk_sbs(c) * 1024,
                       &full[slot]);
    };
    if (warp == 0 && BULK) {
        // stage t's weights: the warp's 32 lanes share the row copies; lane 0
        // arms the stage with the bytes of the copies and of the x slice
        auto issue_weights = [&](uint32_t t, uint32_t slot) {
            const uint32_t pass = t / nchunks, c = t - pass * nchunks;
            const uint32_t gp = g0 + pass * nw, nwp = min(nw, g1 - gp);
            const uint32_t nbytes = chunk_sbs(c) * BB;
            uint8_t* dst = ring + (size_t)slot * slot_bytes;
            // copy i = (warp w, row rr); rows past M are not copied (never stored)
            auto span = [&](uint32_t i, uintptr_t& a0) -> uint32_t {
                const uint32_t row = (gp + i / kQ8RowsPerWarp) * kQ8RowsPerWarp + i % kQ8RowsPerWarp;
                if (row >= M) return 0u;
                const uintptr_t a = reinterpret_cast<uintptr_t>(W) + (size_t)row * row_bytes + (size_t)c * CB;
                a0 = a & ~(uintptr_t)15;
                return (uint32_t)(((a + nbytes + 15) & ~(uintptr_t)15) - a0);
            };
            uint32_t mine = 0;
            for (uint32_t i = lane; i < nwp * kQ8RowsPerWarp; i += 32) {
                uintptr_t a0;
                mine += span(i, a0);
            }
            for (int o = 16; o > 0; o >>= 1) mine += __shfl_xor_sync(0xffffffffu, mine, o);
            if (lane == 0) ptx::mbar_arrive_expect_tx(&full[slot], mine + chunk_sbs(c) * 1024);
            __syncwarp();
            for (uint32_t i = lane; i < nwp * kQ8RowsPerWarp; i += 32) {
                uintptr_t a0 = 0;
                const uint32_t len = span(i, a0);
                if (len)
                    ptx::bulk_load(dst + (i / kQ8RowsPerWarp) * TILE + (i % kQ8RowsPerWarp) * RPITCH,
                                   reinterpret_cast<const void*>(a0), len, &full[slot]);
            }
        };
        for (uint32_t t = 0; t < pre; t++) issue_weights(t, t);  // fresh slots: no wait
        ptx::griddep_wait();  // x (and W, without the flag) may be written by the previous kernel
        for (uint32_t t = 0; t < pre && lane == 0; t++) issue_x(t, t);
        for (uint32_t t = pre; t < ntiles; t++) {
            const uint32_t slot = t % nslots;
            bool ok = true;
            if (lane == 0) ok = ptx::mbar_wait(&empty[slot], ((t / nslots) & 1) ^ 1, err);
            if (!__shfl_sync(0xffffffffu, ok, 0)) break;
            issue_weights(t, slot);
            if (lane == 0) issue_x(t, slot);
        }
        return;
    }
    if (warp == 0) {
        if (lane == 0) {
            // full boxes: the part past the row end (a short last chunk) is zero fill
            auto issue_weights = [&](uint32_t t, uint32_t slot) {
                const uint32_t pass = t / nchunks, c = t - pass * nchunks;
                const uint32_t gp = g0 + pass * nw, nwp = min(nw, g1 - gp);
                uint8_t* dst = ring + (size_t)slot * slot_bytes;
                ptx::mbar_arrive_expect_tx(&full[slot], nwp * kQ8RowsPerWarp * CB + chunk_sbs(c) * 1024);
                for (uint32_t w = 0; w < nwp; w++)
                    ptx::tma_load_2d(dst + w * TILE, &wmap, &full[slot], (int)(c * (CB / KBlock<F>::elem)),
                                     (int)((gp + w) * kQ8RowsPerWarp));
            };
            ptx::prefetch_tmap(&wmap);
            for (uint32_t t = 0; t < pre; t++) issue_weights(t, t);  // fresh slots: no wait
            ptx::griddep_wait();  // x (and W, without the flag) may be written by the previous kernel
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
    const uint32_t cw = warp - 1, rr = lane >> 3, t8 = lane & 7;
    bool alive = true;
    for (uint32_t pass = 0; pass < npass && alive; pass++) {
        const uint32_t gp = g0 + pass * nw;
        const uint32_t row = (gp + cw) * kQ8RowsPerWarp + rr;
        // the whole warp computes (rows past M read the box's zero fill), so the
        // decoders' width-8 shuffles see all 32 lanes; only the store is per row
        const bool warp_on = gp + cw < g1, active = warp_on && row < M;
        float2 acc = make_float2(0.0f, 0.0f);
        for (uint32_t c = 0; c < nchunks; c++) {
            const uint32_t t = pass * nchunks + c, slot = t % nslots;
            // one verdict per warp, so no lane is left behind at a shuffle
            if (!__all_sync(0xffffffffu, ptx::mbar_wait(&full[slot], (t / nslots) & 1, err))) {
                alive = false;
                break;
            }
            if (warp_on) {
                const uint8_t* st = ring + (size_t)slot * slot_bytes;
                const uint8_t* rp = st + cw * TILE + rr * RPITCH;
                if (BULK)  // the chunk's offset within its copied span
                    rp += (reinterpret_cast<uintptr_t>(W) + (size_t)row * row_bytes + (size_t)c * CB) & 15;
                const float* xc = reinterpret_cast<const float*>(st + w_bytes);
                const uint32_t n = chunk_sbs(c);
                for (uint32_t k = 0; k < n; k++) kq_superblock<F>(rp + k * BB, xc + 256 * k, t8, acc, true);
            }
            __syncwarp();
            if (lane == 0) ptx::mbar_arrive(&empty[slot]);
        }
        float sum = __fadd_rn(acc.x, acc.y);
        sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, 1));
        sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, 2));
        sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, 4));
        if (active && alive && t8 == 0) out[row] = sum;
    }
}

template <int F, bool BULK>
int launch_kquant_stream(uint32_t M, uint32_t nsb, const float* x, const uint8_t* W, float* out, uint32_t flags,
                         cudaStream_t s) {
    constexpr uint32_t BB = KBlock<F>::bytes, C = KBlock<F>::chunk, CB = C * BB;
    constexpr uint32_t TILE = BULK ? KSeg<F>::tile : (kQ8RowsPerWarp * CB + 127) / 128 * 128;
    // many rows of short K can ask for more groups per CTA than two ring slots
    // of 200 KB hold: halve the groups per CTA (more CTAs) until they fit
    Q8Plan p;
    for (uint32_t mw = kQ8MaxWarps; mw >= 1; mw /= 2) {
        p = plan_q8_stream(M, nsb * 256, C * 1024, 128, (BB + 7) / 8, TILE, mw);
        if (p.smem <= 200 * 1024) break;
    }
    static std::atomic<uint64_t> smem_set{0};  // devices whose limit is raised
    if (int arc = set_max_dynamic_smem(kquant_stream_kernel<F, BULK>, 200 * 1024, smem_set)) return arc;
    ANE_ARG_CHECK(p.smem <= 200 * 1024, "kquant_gemv: shared-memory plan too large");
    const uint64_t row_bytes = (uint64_t)nsb * BB;
    CUtensorMap wmap;
    memset(&wmap, 0, sizeof(wmap));
    if (!BULK) {
        const uint32_t E = KBlock<F>::elem;
        int rc = encode_tensor_map_2d(&wmap, E == 8 ? CU_TENSOR_MAP_DATA_TYPE_INT64 : CU_TENSOR_MAP_DATA_TYPE_UINT32,
                                      W, row_bytes / E, M, row_bytes, CB / E, kQ8RowsPerWarp,
                                      CU_TENSOR_MAP_SWIZZLE_NONE);
        if (rc) return rc;
    }
    return launch_q8_stream(kquant_stream_kernel<F, BULK>, p, s, wmap, W, x, out, M, nsb, p.groups, p.warps,
                            p.slots, flags, device_timeout_flag());
}

template <int F>
int launch_kquant(uint32_t M, uint32_t nsb, const float* x, const uint8_t* W, float* out, uint32_t flags,
                  cudaStream_t s) {
    // streamed when a row is a whole number of 16-byte units (the TMA row stride)
    // and W, x are 16-byte aligned (TMA base, bulk copies of x)
    const uint64_t row_bytes = (uint64_t)nsb * KBlock<F>::bytes;
    if (row_bytes % 16 == 0 && ((uintptr_t)W & 15) == 0 && ((uintptr_t)x & 15) == 0)
        return launch_kquant_stream<F, false>(M, nsb, x, W, out, flags, s);
    // any row length: bulk copies of 16-byte-aligned spans, as long as the last
    // span (up to 15 bytes past the matrix) stays inside W's allocation
    const uint64_t total = (uint64_t)M * row_bytes;
    const uint64_t tail = ((reinterpret_cast<uintptr_t>(W) + total + 15) & ~(uint64_t)15) -
                          reinterpret_cast<uintptr_t>(W);
    if (((uintptr_t)x & 15) == 0 && device_bytes_from(W) >= tail)
        return launch_kquant_stream<F, true>(M, nsb, x, W, out, flags, s);
    kquant_gemv_kernel<F><<<(M + 31) / 32, 256, 0, s>>>(x, W, out, M, nsb);
    ANE_CHECK_LAUNCH();
    return ANE_OK;
}

// get_rows_q4_0: one thread per (row, block, i < 16): elements i and 16 + i.
__global__ void get_rows_q4_0_kernel(uint32_t n_rows, uint32_t nb, const uint8_t* __restrict__ table,
                                     const uint32_t* __restrict__ idx, float* __restrict__ out) {
    const size_t n = (size_t)n_rows * nb * 16;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const uint32_t e = (uint32_t)(i % 16);
        const size_t rb = i / 16;
        const uint32_t r = (uint32_t)(rb / nb), b = (uint32_t)(rb % nb);
        const uint8_t* blk = table + ((size_t)idx[r] * nb + b) * 18;
        const float d = h2f(ld_u16(blk));
        const uint32_t q = blk[2 + e];
        float* o = out + (size_t)r * nb * 32 + (size_t)b * 32;
        o[e] = __fmul_rn((float)((int32_t)(q & 0x0Fu) - 8), d);
        o[16 + e] = __fmul_rn((float)((int32_t)(q >> 4) - 8), d);
    }
}

}  // namespace

uint32_t kquant_block_bytes(uint32_t fmt) {
    switch (fmt) {
        case kQ4K: return KBlock<kQ4K>::bytes;
        case kQ2K: return KBlock<kQ2K>::bytes;
        case kQ3K: return KBlock<kQ3K>::bytes;
        case kQ5K: return KBlock<kQ5K>::bytes;
        case kQ6K: return KBlock<kQ6K>::bytes;
        default: return 0;
    }
}

int launch_kquant_gemv(uint32_t fmt, uint32_t M, uint32_t K, const float* x, const uint8_t* W, float* out,
                       uint32_t flags, cudaStream_t s) {
    ANE_ARG_CHECK(fmt <= kQ6K, "kquant_gemv: unknown format");
    if (M == 0) return ANE_OK;
    // float2 loads of x; the widest aligned weight load per format (16-byte
    // super-blocks: 4-byte words; 84-byte: 4-byte; 110 / 210-byte: 2-byte)
    const uint32_t wal = (fmt == kQ3K || fmt == kQ6K) ? 2u : 4u;
    ANE_ARG_CHECK(((uintptr_t)x & 7) == 0 && ((uintptr_t)W & (wal - 1)) == 0,
                  "kquant_gemv: x must be 8-byte aligned, W 4-byte (2-byte for q3_k / q6_k)");
    const uint32_t nsb = K / 256;  // the handlers run floor(K / 256) super-blocks (lsr #8)
    if (nsb == 0) {
        ANE_CUDA_TRY(cudaMemsetAsync(out, 0, (size_t)M * 4, s));
        return ANE_OK;
    }
    switch (fmt) {
        case kQ4K: return launch_kquant<kQ4K>(M, nsb, x, W, out, flags, s);
        case kQ2K: return launch_kquant<kQ2K>(M, nsb, x, W, out, flags, s);
        case kQ3K: return launch_kquant<kQ3K>(M, nsb, x, W, out, flags, s);
        case kQ5K: return launch_kquant<kQ5K>(M, nsb, x, W, out, flags, s);
        default: return launch_kquant<kQ6K>(M, nsb, x, W, out, flags, s);
    }
}

int launch_get_rows_q4_0(uint32_t n_rows, uint32_t dim, const uint8_t* table, const uint32_t* idx, float* out,
                         cudaStream_t s) {
    const uint32_t nb = dim / 32;
    if (n_rows == 0 || nb == 0) return ANE_OK;
    const size_t n = (size_t)n_rows * nb * 16;
    size_t g = (n + 255) / 256;
    const size_t cap = (size_t)num_sms() * 16;
    if (g > cap) g = cap;
    get_rows_q4_0_kernel<<<(unsigned)g, 256, 0, s>>>(n_rows, nb, table, idx, out);
    ANE_CHECK_LAUNCH();
    return ANE_OK;
}

}  // namespace ane_b200
