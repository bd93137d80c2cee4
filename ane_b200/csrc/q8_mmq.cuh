// q8_mmq.cuh -- device pieces of the Q8_0 x Q8_0 matvec shared by the
// one-projection kernel (q8_0_gemv_q8.cu) and the persistent decode-stack
// kernel (decode_stack.cu), so both compute every output with the same
// operations in the same order.
//
//   activation:  per 32-block  amax = max|x| (sequential compare, ggml's MAX),
//                d = RN(amax/127), id = d ? RN(1/d) : 0, q = roundf(RN(x*id)),
//                stored as aligned int8 codes xs[K] and fp32 scales xd[b] = fp16(d)
//   matvec:      lane (row r, block pair pp) of a warp: per chunk two exact int32
//                block dots (dp4a) and two fp32 terms float(sumi) * (dw * dx)
#pragma once
#include <cuda_fp16.h>
#include <stdint.h>

namespace ane_b200 {

// One 32-element block in registers -> its 32 codes as 8 little-endian words;
// returns the block scale as stored (fp16(d), widened).
__device__ __forceinline__ float q8_quantize_words(const float (&v)[32], uint32_t (&w)[8]) {
    float amax = 0.0f;
#pragma unroll
    for (int j = 0; j < 32; j++) {
        const float a = fabsf(v[j]);
        amax = amax > a ? amax : a;
    }
    const float d = __fdiv_rn(amax, 127.0f);
    const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
#pragma unroll
    for (int j = 0; j < 32; j += 4) {
        uint32_t x = 0;
#pragma unroll
        for (int i = 0; i < 4; i++) x |= (uint32_t)(uint8_t)(int8_t)(int)roundf(__fmul_rn(v[j + i], id)) << (8 * i);
        w[j / 4] = x;
    }
    return __half2float(__float2half_rn(d));
}

// Quantizes one 32-element block held in registers into xs[32b..32b+31], xd[b].
__device__ __forceinline__ void q8_quantize_regs(const float (&v)[32], int8_t* xs, float* xd, uint32_t b) {
    uint32_t w[8];
    xd[b] = q8_quantize_words(v, w);
    uint32_t* dst = reinterpret_cast<uint32_t*>(xs + (size_t)b * 32);
#pragma unroll
    for (int j = 0; j < 8; j++) dst[j] = w[j];
}

// Quantizes block b of x (32 floats at xb) into xs[32b..32b+31] and xd[b].
// GLOBAL: x lives in global memory written by another CTA or GPU -> L2 loads.
template <bool GLOBAL>
__device__ __forceinline__ void q8_quantize_block(const float* xb, int8_t* xs, float* xd, uint32_t b) {
    float v[32];
#pragma unroll
    for (int j = 0; j < 8; j++) {
        const float4* p = reinterpret_cast<const float4*>(xb) + j;
        const float4 t = GLOBAL ? __ldcg(p) : *p;
        v[4 * j] = t.x;
        v[4 * j + 1] = t.y;
        v[4 * j + 2] = t.z;
        v[4 * j + 3] = t.w;
    }
    q8_quantize_regs(v, xs, xd, b);
}

// One block quantized by 4 lanes (lanes 4k .. 4k+3 of a warp, quarter i = lane
// & 3 holding elements 8i .. 8i+7): the same operations as q8_quantize_words,
// with the absmax fold split into 4 in-order segments.  The fold
// acc = acc > a ? acc : a (a = |x|) restarts at a NaN (NaN > a and a > NaN are
// false), so a segment holding a NaN yields its own fold from 0 whatever came
// before, and any other segment yields the fold step applied to (acc, its own
// maximum); combining the 4 segment results in order that way gives the
// sequential 32-element fold bit for bit.  All 32 lanes of the warp call
// together (width-4 shuffles); store = false lanes compute but write nothing.
__device__ __forceinline__ void q8_quantize_quarter(const float* xq8, int8_t* xs, float* xd, uint32_t b,
                                                    uint32_t i, bool store) {
    const float4 t0 = reinterpret_cast<const float4*>(xq8)[0], t1 = reinterpret_cast<const float4*>(xq8)[1];
    const float v[8] = {t0.x, t0.y, t0.z, t0.w, t1.x, t1.y, t1.z, t1.w};
    float r = 0.0f;
    bool nan = false;
#pragma unroll
    for (int j = 0; j < 8; j++) {
        const float a = fabsf(v[j]);
        nan |= a != a;
        r = r > a ? r : a;
    }
    float amax = 0.0f;
#pragma unroll
    for (int k = 0; k < 4; k++) {
        const float rk = __shfl_sync(0xffffffffu, r, k, 4);
        const bool nk = __shfl_sync(0xffffffffu, (int)nan, k, 4) != 0;
        amax = nk ? rk : (amax > rk ? amax : rk);
    }
    const float d = __fdiv_rn(amax, 127.0f);
    const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
    uint32_t w[2];
#pragma unroll
    for (int j = 0; j < 8; j += 4) {
        uint32_t x = 0;
#pragma unroll
        for (int q = 0; q < 4; q++) x |= (uint32_t)(uint8_t)(int8_t)(int)roundf(__fmul_rn(v[j + q], id)) << (8 * q);
        w[j / 4] = x;
    }
    if (store) {
        reinterpret_cast<uint2*>(xs + (size_t)b * 32)[i] = make_uint2(w[0], w[1]);
        if (i == 0) xd[b] = __half2float(__float2half_rn(d));
    }
}

// Block pair (b, b+1) of one weight row against the activation: pw = the 68
// bytes of the pair (4-byte aligned: the even block's codes straddle words 0..8,
// the odd block's codes are words 9..16).  Adds the two terms to `sum` in block
// order; returns the exact block dots in s0, s1.
__device__ __forceinline__ void q8_pair(const uint32_t* pw, const int8_t* xs, const float* xd, uint32_t b,
                                        int32_t& s0, int32_t& s1, float& sum) {
    uint32_t w[17];
#pragma unroll
    for (int k = 0; k < 17; k++) w[k] = pw[k];
    const int4* x0 = reinterpret_cast<const int4*>(xs + (size_t)b * 32);
    const int4 xa0 = x0[0], xa1 = x0[1], xb0 = x0[2], xb1 = x0[3];
    const float dx0 = xd[b], dx1 = xd[b + 1];
    s0 = 0;
    s1 = 0;
    s0 = __dp4a((int)__funnelshift_r(w[0], w[1], 16), xa0.x, s0);
    s0 = __dp4a((int)__funnelshift_r(w[1], w[2], 16), xa0.y, s0);
    s0 = __dp4a((int)__funnelshift_r(w[2], w[3], 16), xa0.z, s0);
    s0 = __dp4a((int)__funnelshift_r(w[3], w[4], 16), xa0.w, s0);
    s0 = __dp4a((int)__funnelshift_r(w[4], w[5], 16), xa1.x, s0);
    s0 = __dp4a((int)__funnelshift_r(w[5], w[6], 16), xa1.y, s0);
    s0 = __dp4a((int)__funnelshift_r(w[6], w[7], 16), xa1.z, s0);
    s0 = __dp4a((int)__funnelshift_r(w[7], w[8], 16), xa1.w, s0);
    s1 = __dp4a((int)w[9], xb0.x, s1);
    s1 = __dp4a((int)w[10], xb0.y, s1);
    s1 = __dp4a((int)w[11], xb0.z, s1);
    s1 = __dp4a((int)w[12], xb0.w, s1);
    s1 = __dp4a((int)w[13], xb1.x, s1);
    s1 = __dp4a((int)w[14], xb1.y, s1);
    s1 = __dp4a((int)w[15], xb1.z, s1);
    s1 = __dp4a((int)w[16], xb1.w, s1);
    const float dw0 = __half2float(__ushort_as_half((unsigned short)(w[0] & 0xffffu)));
    const float dw1 = __half2float(__ushort_as_half((unsigned short)(w[8] >> 16)));
    sum = __fadd_rn(sum, __fmul_rn(__int2float_rn(s0), __fmul_rn(dw0, dx0)));
    sum = __fadd_rn(sum, __fmul_rn(__int2float_rn(s1), __fmul_rn(dw1, dx1)));
}

// Row total across the 8 block-pair lanes of a row (lane = 4*pp + r).
__device__ __forceinline__ float q8_row_total(float sum) {
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, o));
    return sum;
}

}  // namespace ane_b200
