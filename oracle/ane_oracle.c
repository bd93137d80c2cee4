/*
 * ane_oracle.c -- CPU restatement of the reference's quantized dense hot path.
 *
 * TEST INFRASTRUCTURE ONLY (parity checker and timed CPU baseline); never part
 * of the product.  See ane_oracle.h for the reference file:line each function
 * follows.  Build with -ffp-contract=off and without -ffast-math: every fp32
 * operation here is one IEEE round-to-nearest-even operation, as in the asm.
 */
#include "ane_oracle.h"

#include <float.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------ scalars */

float ane_ref_fp16_to_fp32(uint16_t h) {
    /* fcvt s,h (bytecode_interpreter.s:7034): exact widening. */
    uint32_t sign = (uint32_t)(h >> 15) << 31;
    uint32_t e = (h >> 10) & 0x1f;
    uint32_t m = h & 0x3ff;
    uint32_t bits;
    if (e == 0) {
        if (m == 0) {
            bits = sign;
        } else { /* subnormal half -> normal float */
            int shift = 0;
            while ((m & 0x400) == 0) { m <<= 1; shift++; }
            m &= 0x3ff;
            bits = sign | ((uint32_t)(127 - 15 + 1 - shift) << 23) | (m << 13);
        }
    } else if (e == 31) {
        bits = sign | 0x7f800000u | (m << 13);
    } else {
        bits = sign | ((e - 15 + 127) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

uint16_t ane_ref_fp32_to_fp16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t absx = x & 0x7fffffffu;
    if (absx >= 0x7f800000u) { /* inf / nan */
        return (uint16_t)(sign | 0x7c00u | (absx > 0x7f800000u ? (0x200u | ((absx >> 13) & 0x3ffu)) : 0));
    }
    if (absx >= 0x477ff000u) /* rounds to >= 65520 -> inf */
        return (uint16_t)(sign | 0x7c00u);
    int e = (int)(absx >> 23) - 127;
    uint32_t mant = (absx & 0x7fffffu) | 0x800000u;
    if (e < -25) return (uint16_t)sign; /* below half of the smallest subnormal */
    if (e < -14) {                      /* subnormal half */
        int shift = -14 - e + 13;       /* bits dropped from the 24-bit mantissa */
        uint32_t q = mant >> shift;
        uint32_t rem = mant & ((1u << shift) - 1);
        uint32_t halfway = 1u << (shift - 1);
        if (rem > halfway || (rem == halfway && (q & 1))) q++;
        return (uint16_t)(sign | q);
    }
    uint32_t q = mant >> 13;
    uint32_t rem = mant & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1))) q++;
    uint32_t he = (uint32_t)(e + 15);
    if (q == 0x800u) { q = 0x400u; he++; }
    return (uint16_t)(sign | (he << 10) | (q & 0x3ffu));
}

float ane_ref_relu_max(float y, float floor_v) {
    /* ARM FMAX (not FMAXNM): a NaN operand yields NaN; max(-0, +0) = +0. */
    if (isnan(y)) return y;
    if (isnan(floor_v)) return floor_v;
    if (y == floor_v) return signbit(y) ? floor_v : y;
    return y > floor_v ? y : floor_v;
}

static inline float arm_fmin(float a, float b) {
    if (isnan(a)) return a;
    if (isnan(b)) return b;
    if (a == b) return signbit(a) ? a : b;
    return a < b ? a : b;
}

/* --------------------------------------------------------- quantize_fp32_i8 */

float ane_ref_absmax(const float* src, size_t count) {
    /* bytecode_interpreter.s:1893-1900: fabs + fmax into 16 lanes, then fmaxv.
     * max is order-independent except for NaN, which propagates either way. */
    float m = 0.0f;
    for (size_t i = 0; i < count; i++) m = ane_ref_relu_max(m, fabsf(src[i]));
    return m;
}

float ane_ref_scale_from_absmax(float absmax, float* inv_out) {
    /* bytecode_interpreter.s:1902-1914.  fcmp #0.0 / b.eq: NaN is unordered,
     * so a NaN absmax takes the division path. */
    float scale, inv;
    if (absmax == 0.0f) {
        scale = 1.0f;
        inv = 127.0f;
    } else {
        scale = absmax / 127.0f;
        inv = 127.0f / absmax;
    }
    if (inv_out) *inv_out = inv;
    return scale;
}

int8_t ane_ref_quantize_one(float x, float inv) {
    /* bytecode_interpreter.s:1929-1941: fmul, fmax -127, fmin 127, frintn,
     * fcvtzs (NaN -> 0), st1b truncating narrow. */
    float y = x * inv;
    y = ane_ref_relu_max(y, -127.0f);
    y = arm_fmin(y, 127.0f);
    if (isnan(y)) return 0;
    y = rintf(y); /* default rounding mode: nearest, ties to even */
    return (int8_t)(int32_t)y;
}

float ane_ref_quantize_fp32_i8(const float* src, int8_t* dst, size_t count, float* scale_out) {
    float inv;
    float scale = ane_ref_scale_from_absmax(ane_ref_absmax(src, count), &inv);
    if (scale_out) *scale_out = scale;
    for (size_t i = 0; i < count; i++) dst[i] = ane_ref_quantize_one(src[i], inv);
    return scale;
}

float ane_ref_quantize_with_absmax(const float* src, int8_t* dst, size_t count, float absmax) {
    /* second pass of the handler alone, given an absmax reduced elsewhere
     * (the N-sharded op reduces it across ranks). */
    float inv;
    float scale = ane_ref_scale_from_absmax(absmax, &inv);
    for (size_t i = 0; i < count; i++) dst[i] = ane_ref_quantize_one(src[i], inv);
    return scale;
}

void ane_ref_quantize_fp32_i8_channelwise(uint32_t rows, uint32_t cols, const float* src,
                                          int8_t* dst, float* scales) {
    /* bytecode_interpreter.s:2583-2662: the per-tensor rule applied per row. */
    for (uint32_t r = 0; r < rows; r++)
        ane_ref_quantize_fp32_i8(src + (size_t)r * cols, dst + (size_t)r * cols, cols, &scales[r]);
}

void ane_ref_dequantize_i8_fp32(size_t count, float scale, const int8_t* src, float* dst) {
    /* bytecode_interpreter.s:1966-1975: scvtf then fmul. */
    for (size_t i = 0; i < count; i++) dst[i] = (float)src[i] * scale;
}

/* ---------------------------------------------------------------- pack_b_i8 */

size_t ane_ref_packed_b_size(uint32_t K, uint32_t N) {
    size_t groups = ((size_t)K + 3) / 4;
    size_t panels = ((size_t)N + 15) / 16;
    return panels * groups * 64;
}

void ane_ref_pack_b_i8(uint32_t K, uint32_t N, const int8_t* src, int8_t* dst) {
    /* bytecode_interpreter.s:2466-2580:
     * dst[(p*G + g)*64 + c*4 + d] = B[(4g+d)*N + 16p+c], zero outside K x N. */
    size_t G = ((size_t)K + 3) / 4;
    size_t P = ((size_t)N + 15) / 16;
    for (size_t p = 0; p < P; p++)
        for (size_t g = 0; g < G; g++)
            for (size_t c = 0; c < 16; c++)
                for (size_t d = 0; d < 4; d++) {
                    size_t k = 4 * g + d, n = 16 * p + c;
                    dst[(p * G + g) * 64 + c * 4 + d] = (k < K && n < N) ? src[k * N + n] : 0;
                }
}

/* --------------------------------------------------------------- int8 GEMM */

void ane_ref_gemm_s8_s32(uint32_t M, uint32_t N, uint32_t K, const int8_t* A, size_t lda,
                         const int8_t* B, size_t ldb, int32_t* acc) {
    for (uint32_t m = 0; m < M; m++) {
        int32_t* row = acc + (size_t)m * N;
        for (uint32_t n = 0; n < N; n++) row[n] = 0;
        for (uint32_t k = 0; k < K; k++) {
            int32_t a = A[(size_t)m * lda + k];
            const int8_t* b = B + (size_t)k * ldb;
            for (uint32_t n = 0; n < N; n++) row[n] += a * (int32_t)b[n];
        }
    }
}

void ane_ref_dense_i8(uint32_t M, uint32_t N, uint32_t K, float sa, float sb, uint8_t flags,
                      const int8_t* A, const int8_t* B_packed, const float* bias, float* C) {
    /* bytecode_interpreter.s:1995-2446.  M16 x N32 tiles, K padded to K64,
     * A row stride K64, B panel stride K64/4*64 bytes, C rows not predicated. */
    uint32_t M16 = (M + 15) & ~15u;
    uint32_t N32 = (N + 31) & ~31u;
    uint32_t K64 = (K + 63) & ~63u;
    size_t G = K64 / 4;
    float comb = sa * sb;                           /* :2017 fmul s20,s20,s22 */
    float floor_v = (flags & 1) ? 0.0f : -FLT_MAX;  /* :2022-2029 */
    for (uint32_t r = 0; r < M16; r++) {
        for (uint32_t n = 0; n < N32 && n < N; n++) {
            size_t p = n / 16, c = n % 16;
            int32_t acc = 0;
            for (uint32_t k = 0; k < K64; k++) {
                size_t g = k / 4, d = k % 4;
                acc += (int32_t)A[(size_t)r * K64 + k] *
                       (int32_t)B_packed[(p * G + g) * 64 + c * 4 + d];
            }
            float y = (float)acc;                 /* scvtf */
            y = y * comb;                         /* fmul */
            y = y + bias[n];                      /* fadd */
            C[(size_t)r * N + n] = ane_ref_relu_max(y, floor_v); /* fmax */
        }
    }
}

/* dense_u8s8 (bytecode_interpreter.s:2841-3305): dense_i8 with an unsigned A
 * (usmopa), the same padding, epilogue and ReLU floor. */
void ane_ref_dense_u8s8(uint32_t M, uint32_t N, uint32_t K, float sa, float sb, uint8_t flags,
                        const uint8_t* A, const int8_t* B_packed, const float* bias, float* C) {
    uint32_t M16 = (M + 15) & ~15u;
    uint32_t N32 = (N + 31) & ~31u;
    uint32_t K64 = (K + 63) & ~63u;
    size_t G = K64 / 4;
    float comb = sa * sb;
    float floor_v = (flags & 1) ? 0.0f : -FLT_MAX;
    for (uint32_t r = 0; r < M16; r++) {
        for (uint32_t n = 0; n < N32 && n < N; n++) {
            size_t p = n / 16, c = n % 16;
            int32_t acc = 0;
            for (uint32_t k = 0; k < K64; k++) {
                size_t g = k / 4, d = k % 4;
                acc += (int32_t)A[(size_t)r * K64 + k] * (int32_t)B_packed[(p * G + g) * 64 + c * 4 + d];
            }
            float y = (float)acc;
            y = y * comb;
            y = y + bias[n];
            C[(size_t)r * N + n] = ane_ref_relu_max(y, floor_v);
        }
    }
}

/* Integer CBLAS GEMMs (bytecode_interpreter.s:8329-9139, macro CBLAS_INTEGER_GEMM):
 * kind 0 igemm (s8 x s8, scvtf), 1 ugemm (u8 x u8, ucvtf), 2 usgemm (u8 x s8, scvtf).
 * op(A)[m][k] = flags&1 ? A[k*lda+m] : A[m*lda+k]; op(B)[k][n] = flags&2 ? B[n*ldb+k]
 * : B[k*ldb+n].  The 32-bit accumulator starts at 0, or -- when beta's bits are
 * not zero -- at the bit pattern of RN(beta * C[m][n]) (the ZA tile is loaded
 * with fmul(C, beta), :8411-8489); products are added modulo 2^32; then
 * C = RN(cvt(acc) * alpha). */
void ane_ref_int_gemm(int kind, uint8_t flags, uint32_t M, uint32_t N, uint32_t K, uint32_t lda, uint32_t ldb,
                      uint32_t ldc, float alpha, float beta, const uint8_t* A, const uint8_t* B, float* C) {
    uint32_t beta_bits;
    memcpy(&beta_bits, &beta, 4);
    for (uint32_t m = 0; m < M; m++)
        for (uint32_t n = 0; n < N; n++) {
            float* c = C + (size_t)m * ldc + n;
            uint32_t acc = 0;
            if (beta_bits != 0) {
                float bc = *c * beta;
                memcpy(&acc, &bc, 4);
            }
            for (uint32_t k = 0; k < K; k++) {
                uint8_t a = (flags & 1) ? A[(size_t)k * lda + m] : A[(size_t)m * lda + k];
                uint8_t b = (flags & 2) ? B[(size_t)n * ldb + k] : B[(size_t)k * ldb + n];
                int32_t av = kind == 0 ? (int32_t)(int8_t)a : (int32_t)a;
                int32_t bv = kind == 1 ? (int32_t)b : (int32_t)(int8_t)b;
                acc += (uint32_t)(av * bv);
            }
            float f = kind == 1 ? (float)acc : (float)(int32_t)acc;
            *c = f * alpha;
        }
}

/* ------------------------------------------- MNIST-i8 training opcodes */

static inline float faddv16(const float* a);
static inline float f32_bits(uint32_t u) {
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* elementwise_scaled_add_fp32 (0x0D; :585-605): out = fma(b, scale, a) (fmla). */
void ane_ref_elementwise_scaled_add_fp32(uint32_t count, float scale, const float* a, const float* b, float* out) {
    for (uint32_t i = 0; i < count; i++) out[i] = fmaf(b[i], scale, a[i]);
}

/* relu_backward_fp32 (0x0F; :639-661): out = act > 0 ? grad : +0 (fcmgt; NaN -> 0). */
void ane_ref_relu_backward_fp32(uint32_t count, const float* act, const float* grad, float* out) {
    for (uint32_t i = 0; i < count; i++) out[i] = act[i] > 0.0f ? grad[i] : 0.0f;
}

/* transpose_fp32 (0x11; :705-741): dst[N x M] = src[M x N]^T. */
void ane_ref_transpose_fp32(uint32_t M, uint32_t N, const float* src, float* dst) {
    for (uint32_t i = 0; i < M; i++)
        for (uint32_t j = 0; j < N; j++) dst[(size_t)j * M + i] = src[(size_t)i * N + j];
}

/* count_matches (0x16; :1827-1850): number of i with pred[i] == (int32)labels[i]. */
void ane_ref_count_matches(uint32_t count, const int32_t* pred, const uint8_t* labels, int32_t* out) {
    int32_t n = 0;
    for (uint32_t i = 0; i < count; i++) n += pred[i] == (int32_t)labels[i];
    *out = n;
}

/* dense_fp32 (0x15; :1008-1826): C[r][c] = fmax(RN((bias[c] + sum_k A[r][k]*B[k][c]) * scale),
 * relu ? 0 : -FLT_MAX), the accumulator starting at bias[c] and taking one fused
 * multiply-add per k in order (FMOPA); rows r < M16 written (not predicated),
 * columns c < N; A row stride K, B and C row stride N.  The handler runs K/16
 * whole k-blocks (lsr w15, w2, #4): only k < (K & ~15) contribute. */
void ane_ref_dense_fp32(uint32_t M, uint32_t N, uint32_t K, float scale, uint8_t flags, const float* A,
                        const float* B, const float* bias, float* C) {
    uint32_t M16 = (M + 15) & ~15u;
    float floor_v = (flags & 1) ? 0.0f : -FLT_MAX;
    for (uint32_t r = 0; r < M16; r++)
        for (uint32_t c = 0; c < N; c++) {
            float acc = bias[c];
            for (uint32_t k = 0; k < (K & ~15u); k++) acc = fmaf(A[(size_t)r * K + k], B[(size_t)k * N + c], acc);
            C[(size_t)r * N + c] = ane_ref_relu_max(acc * scale, floor_v);
        }
}

/* softmax_argmax_fp32 (0x12; :742-1007), per row of `cols` (a multiple of 16):
 *   m = max over the row (fmax, NaN wins)
 *   e_i = 2^n * p(f): t = RN((x_i - m) * log2e), n = floor(t), f = RN(t - n),
 *         p = ((((c4*f + c3)*f + c2)*f + ln2)*f + 1) with every * and + rounded,
 *         2^n built from the exponent bits of max(trunc(n), -127) (+127 << 23)
 *   probs_i = RN(e_i * RN(1 / S)), S = FADDV over 16 lanes of the lane sums
 *             (lane l adds e_l, e_{l+16}, ... in order)
 *   g_out[0..15] = probs[0..15], g_out[label] -= 1 (first 16 columns only)
 *   argmax = first index of max(probs[0..15]) among the first 16 (15 if none). */
static float smx_exp(float x, float m) {
    const float log2e = f32_bits(0x3FB8AA3Bu);  /* the handler's movz/movk constants */
    const float c4 = f32_bits(0x3C1D955Au);
    const float c3 = f32_bits(0x3D635847u);
    const float c2 = f32_bits(0x3E75FDF0u);
    const float c1 = f32_bits(0x3F317218u);
    float xm = x - m;
    float t = xm * log2e;
    float n = floorf(t);
    float f = t - n;
    float p = c4 * f;
    p = p + c3;
    p = p * f;
    p = p + c2;
    p = p * f;
    p = p + c1;
    p = p * f;
    p = p + 1.0f;
    int32_t e;
    if (n != n) e = 0;                                  /* fcvtzs: NaN -> 0 */
    else if (n >= 2147483648.0f) e = INT32_MAX;         /* saturating */
    else if (n < -2147483648.0f) e = INT32_MIN;
    else e = (int32_t)n;
    if (e < -127) e = -127;
    uint32_t bits = (uint32_t)(e + 127) << 23;
    float two_n;
    memcpy(&two_n, &bits, 4);
    return p * two_n;
}

void ane_ref_softmax_argmax_fp32(uint32_t batch, uint32_t cols, const float* logits, float* probs,
                                 const uint8_t* labels, float* g_out, int32_t* argmax) {
    for (uint32_t r = 0; r < batch; r++) {
        const float* x = logits + (size_t)r * cols;
        float* pr = probs + (size_t)r * cols;
        float m = -INFINITY;
        for (uint32_t i = 0; i < cols; i++) m = ane_ref_relu_max(m, x[i]) ;  /* fmax (NaN wins) */
        float lane[16] = {0};
        for (uint32_t i = 0; i < cols; i++) {
            float e = smx_exp(x[i], m);
            pr[i] = e;
            lane[i % 16] = lane[i % 16] + e;
        }
        float S = faddv16(lane);
        float inv = 1.0f / S;
        for (uint32_t i = 0; i < cols; i++) pr[i] = pr[i] * inv;
        float* g = g_out + (size_t)r * cols;
        for (uint32_t i = 0; i < 16; i++) g[i] = (i == labels[r]) ? pr[i] - 1.0f : pr[i];
        float mx = -INFINITY;
        for (uint32_t i = 0; i < 16; i++) mx = ane_ref_relu_max(mx, i < cols ? pr[i] : -INFINITY);
        int32_t idx = 15;
        for (int32_t i = 15; i >= 0; i--)
            if ((i < (int32_t)cols ? pr[i] : -INFINITY) == mx) idx = i;
        argmax[r] = idx;
    }
}

/* ---------------------------------------------------------- dense_fused_i8 */

void ane_ref_dense_fused_epilogue(uint32_t M, uint32_t N, const int32_t* acc, float sa, float sb,
                                  float scale, int relu, float* C) {
    float comb = sa * sb;
    for (size_t i = 0; i < (size_t)M * N; i++) {
        float y = (float)acc[i];
        y = y * comb;
        y = y * scale;
        C[i] = relu ? ane_ref_relu_max(y, 0.0f) : y;
    }
}

void ane_ref_dense_fused_i8(uint32_t M, uint32_t N, uint32_t K, float scale, int relu,
                            const float* A, const float* B, float* C, int8_t* Aq_out,
                            int8_t* Bq_out, int32_t* acc_out, float* sa_out, float* sb_out) {
    size_t MK = (size_t)M * K, KN = (size_t)K * N, MN = (size_t)M * N;
    int8_t* Aq = Aq_out ? Aq_out : (int8_t*)malloc(MK ? MK : 1);
    int8_t* Bq = Bq_out ? Bq_out : (int8_t*)malloc(KN ? KN : 1);
    int32_t* acc = acc_out ? acc_out : (int32_t*)malloc((MN ? MN : 1) * sizeof(int32_t));
    float sa = ane_ref_quantize_fp32_i8(A, Aq, MK, NULL);
    float sb = ane_ref_quantize_fp32_i8(B, Bq, KN, NULL);
    ane_ref_gemm_s8_s32(M, N, K, Aq, K, Bq, N, acc);
    ane_ref_dense_fused_epilogue(M, N, acc, sa, sb, scale, relu, C);
    if (sa_out) *sa_out = sa;
    if (sb_out) *sb_out = sb;
    if (!Aq_out) free(Aq);
    if (!Bq_out) free(Bq);
    if (!acc_out) free(acc);
}

/* --------------------------------------------------------------- q8_0_gemv */

static inline float faddv16(const float* a) {
    /* SVE FADDV over 16 fp32 lanes: Reduce() splits into low/high halves
     * recursively, so the tree is ((a0+a1)+(a2+a3))+((a4+a5)+(a6+a7)) ... */
    float s8[8], s4[4], s2[2];
    for (int i = 0; i < 8; i++) s8[i] = a[2 * i] + a[2 * i + 1];
    for (int i = 0; i < 4; i++) s4[i] = s8[2 * i] + s8[2 * i + 1];
    for (int i = 0; i < 2; i++) s2[i] = s4[2 * i] + s4[2 * i + 1];
    return s2[0] + s2[1];
}

static void q8_0_gemv_rows(uint32_t m0, uint32_t m1, uint32_t K, const float* x,
                           const uint8_t* W, float* out) {
    uint32_t nb = K / 32;
    for (uint32_t m = m0; m < m1; m++) {
        const uint8_t* row = W + (size_t)m * nb * 34;
        float acc[16] = {0};
        for (uint32_t b = 0; b < nb; b++) {
            const uint8_t* blk = row + (size_t)b * 34;
            uint16_t hb = (uint16_t)(blk[0] | (blk[1] << 8));
            float d = ane_ref_fp16_to_fp32(hb);      /* ldr h0 ; fcvt */
            const int8_t* qs = (const int8_t*)(blk + 2);
            const float* xb = x + (size_t)b * 32;
            for (int l = 0; l < 16; l++) {             /* first half, :7042-7047 */
                float dq = (float)qs[l] * d;           /* scvtf ; fmul */
                acc[l] = fmaf(dq, xb[l], acc[l]);      /* fmla */
            }
            for (int l = 0; l < 16; l++) {             /* second half, :7049-7055 */
                float dq = (float)qs[16 + l] * d;
                acc[l] = fmaf(dq, xb[16 + l], acc[l]);
            }
        }
        out[m] = faddv16(acc);                         /* faddv ; str */
    }
}

void ane_ref_q8_0_gemv(uint32_t M, uint32_t K, const float* x, const uint8_t* W, float* out) {
    q8_0_gemv_rows(0, M, K, x, W, out);
}

/* q4_0_gemv (bytecode_interpreter.s:7064-7126): 18-byte blocks {fp16 d; 16 bytes},
 * element i < 16 = low nibble of byte i, element 16+i = its high nibble, value
 * (nibble - 8) * d; lane l accumulates element l then 16+l of every block, then
 * the FADDV tree -- the q8_0_gemv scheme with another block decoder. */
void ane_ref_q4_0_gemv(uint32_t M, uint32_t K, const float* x, const uint8_t* W, float* out) {
    uint32_t nb = K / 32;
    for (uint32_t m = 0; m < M; m++) {
        const uint8_t* row = W + (size_t)m * nb * 18;
        float acc[16] = {0};
        for (uint32_t b = 0; b < nb; b++) {
            const uint8_t* blk = row + (size_t)b * 18;
            float d = ane_ref_fp16_to_fp32((uint16_t)(blk[0] | (blk[1] << 8)));  /* ldr h0 ; fcvt */
            const uint8_t* qs = blk + 2;
            const float* xb = x + (size_t)b * 32;
            for (int l = 0; l < 16; l++) {  /* low nibbles: and #0x0F ; sub 8 ; scvtf ; fmul ; fmla */
                float dq = (float)((int32_t)(qs[l] & 0x0F) - 8) * d;
                acc[l] = fmaf(dq, xb[l], acc[l]);
            }
            for (int l = 0; l < 16; l++) {  /* high nibbles: lsr #4 ; ... */
                float dq = (float)((int32_t)(qs[l] >> 4) - 8) * d;
                acc[l] = fmaf(dq, xb[16 + l], acc[l]);
            }
        }
        out[m] = faddv16(acc);
    }
}

/* ------------------------------------------------------ K-quant matvecs
 * q4_k / q2_k / q3_k / q5_k / q6_k _gemv (bytecode_interpreter.s:11024-11620):
 * rows of K/256 super-blocks; 16 accumulator lanes, lane l taking every
 * 16-element chunk's element l in row order with one fused multiply-add
 * (fmla), the row = the FADDV tree.  Each element's value is computed with
 * separately rounded operations exactly as the handlers do (ucvtf/scvtf exact,
 * then fmul, then fadd where the format has a min term).  The layouts are the
 * handlers' own (their comments name the ggml formats; the byte layouts below
 * are what the code reads), including two of their quirks: q3_k's second half
 * of every 32-element sub-block shifts its packed 2-bit codes right first by
 * the bit pattern of the x values the first half loaded (a clobbered shift
 * vector; SVE clamps shifts >= 32 to a zero result), and q6_k's value lanes
 * 8..15 carry garbage that zip1 discards. */

static inline uint32_t le16(const uint8_t* p) { return (uint32_t)p[0] | ((uint32_t)p[1] << 8); }
static inline uint32_t bits_of(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    return u;
}
static inline uint32_t le32(const uint8_t* p) { return le16(p) | (le16(p + 2) << 16); }

/* 6-bit scale and min of sub-block j from the 12 packed bytes (q4_k :11052-11085,
 * q5_k :11402-11423) */
static inline void k_scale_min(const uint8_t* s, int j, uint32_t* sc, uint32_t* m) {
    if (j < 4) {
        *sc = s[j] & 0x3Fu;
        *m = s[j + 4] & 0x3Fu;
    } else {
        *sc = (s[j + 4] & 0x0Fu) | ((uint32_t)(s[j - 4] >> 6) << 4);
        *m = (uint32_t)(s[j + 4] >> 4) | ((uint32_t)(s[j] >> 6) << 4);
    }
}

/* q4_k (:11024-11133): 144-byte super-blocks {fp16 d, fp16 dmin, scales[12], qs[128]};
 * 8 sub-blocks of 32: element i < 16 = low nibble of qs[16j+i], 16+i = its high
 * nibble; value RN(RN(q * RN(d*sc)) + RN(-dmin*m)). */
void ane_ref_q4_k_gemv(uint32_t M, uint32_t K, const float* x, const uint8_t* W, float* out) {
    uint32_t nsb = K / 256;
    for (uint32_t r = 0; r < M; r++) {
        float acc[16] = {0};
        for (uint32_t b = 0; b < nsb; b++) {
            const uint8_t* blk = W + ((size_t)r * nsb + b) * 144;
            float d = ane_ref_fp16_to_fp32((uint16_t)le16(blk));
            float nd = -ane_ref_fp16_to_fp32((uint16_t)le16(blk + 2));  /* fneg */
            const uint8_t* qs = blk + 16;
            const float* xb = x + (size_t)b * 256;
            for (int j = 0; j < 8; j++) {
                uint32_t sc, mn;
                k_scale_min(blk + 4, j, &sc, &mn);
                float dsc = d * (float)sc, dmm = nd * (float)mn;
                for (int l = 0; l < 16; l++) {
                    float t = (float)(qs[16 * j + l] & 0x0F) * dsc;
                    float v = t + dmm;
                    acc[l] = fmaf(v, xb[32 * j + l], acc[l]);
                }
                for (int l = 0; l < 16; l++) {
                    float t = (float)(qs[16 * j + l] >> 4) * dsc;
                    float v = t + dmm;
                    acc[l] = fmaf(v, xb[32 * j + 16 + l], acc[l]);
                }
            }
        }
        out[r] = faddv16(acc);
    }
}

/* q2_k (:11146-11224): 84-byte super-blocks {scales[16], qs[64], fp16 d, fp16 dmin};
 * 16 sub-blocks of 16: sc = scales[j] & 15, m = scales[j] >> 4, element l = bits
 * 2l..2l+1 of the little-endian word qs[4j..4j+3]. */
void ane_ref_q2_k_gemv(uint32_t M, uint32_t K, const float* x, const uint8_t* W, float* out) {
    uint32_t nsb = K / 256;
    for (uint32_t r = 0; r < M; r++) {
        float acc[16] = {0};
        for (uint32_t b = 0; b < nsb; b++) {
            const uint8_t* blk = W + ((size_t)r * nsb + b) * 84;
            float d = ane_ref_fp16_to_fp32((uint16_t)le16(blk + 80));
            float nd = -ane_ref_fp16_to_fp32((uint16_t)le16(blk + 82));
            const float* xb = x + (size_t)b * 256;
            for (int j = 0; j < 16; j++) {
                float dsc = d * (float)(blk[j] & 0x0F), dmm = nd * (float)(blk[j] >> 4);
                uint32_t w = le32(blk + 16 + 4 * j);
                for (int l = 0; l < 16; l++) {
                    float t = (float)((w >> (2 * l)) & 3u) * dsc;
                    float v = t + dmm;
                    acc[l] = fmaf(v, xb[16 * j + l], acc[l]);
                }
            }
        }
        out[r] = faddv16(acc);
    }
}

/* q3_k (:11236-11360): 110-byte super-blocks {hmask[32], qs[64], scales[12], fp16 d};
 * 8 sub-blocks of 32; scale s6 (the q4_k 6-bit scale rule) - 32, signed; code
 * q = 2 low bits | hmask bit << 2, value RN((q - 4) * RN(d * (s6 - 32))). */
void ane_ref_q3_k_gemv(uint32_t M, uint32_t K, const float* x, const uint8_t* W, float* out) {
    uint32_t nsb = K / 256;
    for (uint32_t r = 0; r < M; r++) {
        float acc[16] = {0};
        for (uint32_t b = 0; b < nsb; b++) {
            const uint8_t* blk = W + ((size_t)r * nsb + b) * 110;
            const uint8_t *hm = blk, *qs = blk + 32, *sc = blk + 96;
            float d = ane_ref_fp16_to_fp32((uint16_t)le16(blk + 108));
            const float* xb = x + (size_t)b * 256;
            for (int j = 0; j < 8; j++) {
                uint32_t s6 = j < 4 ? (sc[j] & 0x3Fu) : ((sc[j + 4] & 0x0Fu) | ((uint32_t)(sc[j - 4] >> 6) << 4));
                float dsc = d * (float)((int32_t)s6 - 32);
                uint32_t w0 = le32(qs + 8 * j), h0 = le16(hm + 4 * j);
                for (int l = 0; l < 16; l++) {
                    uint32_t q = ((w0 >> (2 * l)) & 3u) | (((h0 >> l) & 1u) << 2);
                    float v = (float)((int32_t)q - 4) * dsc;
                    acc[l] = fmaf(v, xb[32 * j + l], acc[l]);
                }
                uint32_t w1 = le32(qs + 8 * j + 4), h1 = le16(hm + 4 * j + 2);
                for (int l = 0; l < 16; l++) {
                    /* lsr by the first half's x bits (the stale z1), then by 2l */
                    uint32_t xs = bits_of(xb[32 * j + l]);
                    uint32_t t = xs >= 32u ? 0u : (w1 >> xs);
                    uint32_t q = ((t >> (2 * l)) & 3u) | (((h1 >> l) & 1u) << 2);
                    float v = (float)((int32_t)q - 4) * dsc;
                    acc[l] = fmaf(v, xb[32 * j + 16 + l], acc[l]);
                }
            }
        }
        out[r] = faddv16(acc);
    }
}

/* q5_k (:11372-11486): 176-byte super-blocks {fp16 d, fp16 dmin, scales[12], qh[32],
 * qs[128]}; q4_k's scales and nibbles, plus bit l (first half) or 16+l (second
 * half) of the little-endian word qh[4j..4j+3] as bit 4. */
void ane_ref_q5_k_gemv(uint32_t M, uint32_t K, const float* x, const uint8_t* W, float* out) {
    uint32_t nsb = K / 256;
    for (uint32_t r = 0; r < M; r++) {
        float acc[16] = {0};
        for (uint32_t b = 0; b < nsb; b++) {
            const uint8_t* blk = W + ((size_t)r * nsb + b) * 176;
            float d = ane_ref_fp16_to_fp32((uint16_t)le16(blk));
            float nd = -ane_ref_fp16_to_fp32((uint16_t)le16(blk + 2));
            const uint8_t *qh = blk + 16, *qs = blk + 48;
            const float* xb = x + (size_t)b * 256;
            for (int j = 0; j < 8; j++) {
                uint32_t sc, mn;
                k_scale_min(blk + 4, j, &sc, &mn);
                float dsc = d * (float)sc, dmm = nd * (float)mn;
                uint32_t h = le32(qh + 4 * j);
                for (int l = 0; l < 16; l++) {
                    uint32_t q = (qs[16 * j + l] & 0x0Fu) | (((h >> l) & 1u) << 4);
                    float t = (float)q * dsc;
                    float v = t + dmm;
                    acc[l] = fmaf(v, xb[32 * j + l], acc[l]);
                }
                for (int l = 0; l < 16; l++) {
                    uint32_t q = (uint32_t)(qs[16 * j + l] >> 4) | (((h >> (16 + l)) & 1u) << 4);
                    float t = (float)q * dsc;
                    float v = t + dmm;
                    acc[l] = fmaf(v, xb[32 * j + 16 + l], acc[l]);
                }
            }
        }
        out[r] = faddv16(acc);
    }
}

/* q6_k (:11498-11606): 210-byte super-blocks {ql[128], qh[64], int8 scales[16],
 * fp16 d}; 16 sub-blocks of 16: element n = nibble (low for even n, high for
 * odd) of ql[8j + n/2] | bits 2n..2n+1 of the little-endian word qh[4j..4j+3]
 * << 4; value RN((q - 32) * RN(d * scale)). */
void ane_ref_q6_k_gemv(uint32_t M, uint32_t K, const float* x, const uint8_t* W, float* out) {
    uint32_t nsb = K / 256;
    for (uint32_t r = 0; r < M; r++) {
        float acc[16] = {0};
        for (uint32_t b = 0; b < nsb; b++) {
            const uint8_t* blk = W + ((size_t)r * nsb + b) * 210;
            const uint8_t *ql = blk, *qh = blk + 128;
            const int8_t* sc = (const int8_t*)(blk + 192);
            float d = ane_ref_fp16_to_fp32((uint16_t)le16(blk + 208));
            const float* xb = x + (size_t)b * 256;
            for (int j = 0; j < 16; j++) {
                float dsc = d * (float)sc[j];
                uint32_t h = le32(qh + 4 * j);
                for (int n = 0; n < 16; n++) {
                    uint32_t byte = ql[8 * j + n / 2];
                    uint32_t nib = (n & 1) ? (byte >> 4) : (byte & 0x0Fu);
                    uint32_t q = nib | (((h >> (2 * n)) & 3u) << 4);
                    float v = (float)((int32_t)q - 32) * dsc;
                    acc[n] = fmaf(v, xb[16 * j + n], acc[n]);
                }
            }
        }
        out[r] = faddv16(acc);
    }
}

void ane_ref_quantize_q8_0(const float* x, uint8_t* blocks, size_t n_rows, size_t K) {
    size_t nb = K / 32;
    for (size_t r = 0; r < n_rows; r++)
        for (size_t b = 0; b < nb; b++) {
            const float* xb = x + r * K + b * 32;
            uint8_t* blk = blocks + (r * nb + b) * 34;
            float amax = 0.0f;
            for (int j = 0; j < 32; j++) {
                float v = fabsf(xb[j]);
                amax = amax > v ? amax : v;
            }
            float d = amax / 127.0f;
            float id = d != 0.0f ? 1.0f / d : 0.0f;
            uint16_t hd = ane_ref_fp32_to_fp16(d);
            blk[0] = (uint8_t)(hd & 0xff);
            blk[1] = (uint8_t)(hd >> 8);
            for (int j = 0; j < 32; j++) blk[2 + j] = (uint8_t)(int8_t)roundf(xb[j] * id);
        }
}

void ane_ref_q8_0_gemv_q8(uint32_t M, uint32_t K, const uint8_t* xq, const uint8_t* W,
                          float* out, int32_t* block_dots) {
    uint32_t nb = K / 32;
    for (uint32_t m = 0; m < M; m++) {
        float sumf = 0.0f;
        for (uint32_t b = 0; b < nb; b++) {
            const uint8_t* wb = W + ((size_t)m * nb + b) * 34;
            const uint8_t* xb = xq + (size_t)b * 34;
            int32_t sumi = 0;
            for (int j = 0; j < 32; j++) sumi += (int32_t)(int8_t)wb[2 + j] * (int32_t)(int8_t)xb[2 + j];
            if (block_dots) block_dots[(size_t)m * nb + b] = sumi;
            float dw = ane_ref_fp16_to_fp32((uint16_t)(wb[0] | (wb[1] << 8)));
            float dx = ane_ref_fp16_to_fp32((uint16_t)(xb[0] | (xb[1] << 8)));
            sumf += (float)sumi * (dw * dx);
        }
        out[m] = sumf;
    }
}

/* Q8_0 x Q8_0 product for NT activation rows (ggml MUL_MAT with ne1 = NT):
 * the batch-1 formula above per (weight row, activation row), with the fp32
 * terms grouped into segments of ANE_Q8_SEG_BLOCKS blocks: each segment is
 * summed from +0 in block order, then the segment sums are added from +0 in
 * segment order.  out[t * ldo + m]; xq holds NT rows of K/32 blocks. */
void ane_ref_mul_mat_q8_0_batch(uint32_t M, uint32_t K, uint32_t NT, const uint8_t* xq, const uint8_t* W,
                                float* out, size_t ldo) {
    uint32_t nb = K / 32;
    for (uint32_t t = 0; t < NT; t++)
        for (uint32_t m = 0; m < M; m++) {
            float total = 0.0f;
            for (uint32_t s0 = 0; s0 < nb; s0 += ANE_Q8_SEG_BLOCKS) {
                float part = 0.0f;
                uint32_t s1 = s0 + ANE_Q8_SEG_BLOCKS < nb ? s0 + ANE_Q8_SEG_BLOCKS : nb;
                for (uint32_t b = s0; b < s1; b++) {
                    const uint8_t* wb = W + ((size_t)m * nb + b) * 34;
                    const uint8_t* xb = xq + ((size_t)t * nb + b) * 34;
                    int32_t sumi = 0;
                    for (int j = 0; j < 32; j++) sumi += (int32_t)(int8_t)wb[2 + j] * (int32_t)(int8_t)xb[2 + j];
                    float dw = ane_ref_fp16_to_fp32((uint16_t)(wb[0] | (wb[1] << 8)));
                    float dx = ane_ref_fp16_to_fp32((uint16_t)(xb[0] | (xb[1] << 8)));
                    part += (float)sumi * (dw * dx);
                }
                total += part;
            }
            out[(size_t)t * ldo + m] = total;
        }
}

void ane_ref_get_rows_q8_0(uint32_t n_rows, uint32_t dim, const uint8_t* table,
                           const uint32_t* indices, float* out) {
    /* bytecode_interpreter.s:12365-12405. */
    uint32_t nb = dim / 32;
    for (uint32_t r = 0; r < n_rows; r++) {
        const uint8_t* row = table + (size_t)indices[r] * nb * 34;
        for (uint32_t b = 0; b < nb; b++) {
            const uint8_t* blk = row + (size_t)b * 34;
            float d = ane_ref_fp16_to_fp32((uint16_t)(blk[0] | (blk[1] << 8)));
            for (int j = 0; j < 32; j++)
                out[(size_t)r * dim + b * 32 + j] = (float)(int8_t)blk[2 + j] * d;
        }
    }
}

void ane_ref_get_rows_q4_0(uint32_t n_rows, uint32_t dim, const uint8_t* table,
                           const uint32_t* indices, float* out) {
    /* bytecode_interpreter.s:12419-12466: 18-byte Q4_0 blocks; element i < 16 =
     * (low nibble of byte i) - 8, element 16+i = (high nibble) - 8, times d
     * (scvtf exact, one RN multiply). */
    uint32_t nb = dim / 32;
    for (uint32_t r = 0; r < n_rows; r++) {
        const uint8_t* row = table + (size_t)indices[r] * nb * 18;
        for (uint32_t b = 0; b < nb; b++) {
            const uint8_t* blk = row + (size_t)b * 18;
            float d = ane_ref_fp16_to_fp32((uint16_t)(blk[0] | (blk[1] << 8)));
            for (int i = 0; i < 16; i++) {
                out[(size_t)r * dim + b * 32 + i] = (float)((int32_t)(blk[2 + i] & 0x0F) - 8) * d;
                out[(size_t)r * dim + b * 32 + 16 + i] = (float)((int32_t)(blk[2 + i] >> 4) - 8) * d;
            }
        }
    }
}

/* ------------------------------------------------------- OpenMP baselines */

int ane_ref_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

static float absmax_omp(const float* src, size_t n, int nt) {
    float m = 0.0f;
    int saw_nan = 0;
#ifdef _OPENMP
#pragma omp parallel for num_threads(nt) reduction(max : m) reduction(| : saw_nan)
#endif
    for (size_t i = 0; i < n; i++) {
        float v = fabsf(src[i]);
        if (isnan(v)) saw_nan = 1;
        m = v > m ? v : m;
    }
    (void)nt;
    return saw_nan ? NAN : m;
}

void ane_ref_dense_fused_i8_omp(uint32_t M, uint32_t N, uint32_t K, float scale, int relu,
                                const float* A, const float* B, float* C, int n_threads) {
    size_t MK = (size_t)M * K, KN = (size_t)K * N;
    int nt = n_threads > 0 ? n_threads : ane_ref_max_threads();
    int8_t* Aq = (int8_t*)malloc(MK ? MK : 1);
    int8_t* Bt = (int8_t*)malloc(KN ? KN : 1); /* quantized B, transposed N x K */
    float inv_a, inv_b;
    float sa = ane_ref_scale_from_absmax(absmax_omp(A, MK, nt), &inv_a);
    float sb = ane_ref_scale_from_absmax(absmax_omp(B, KN, nt), &inv_b);
#ifdef _OPENMP
#pragma omp parallel for num_threads(nt)
#endif
    for (size_t i = 0; i < MK; i++) Aq[i] = ane_ref_quantize_one(A[i], inv_a);
#ifdef _OPENMP
#pragma omp parallel for num_threads(nt)
#endif
    for (uint32_t k = 0; k < K; k++)
        for (uint32_t n = 0; n < N; n++) Bt[(size_t)n * K + k] = ane_ref_quantize_one(B[(size_t)k * N + n], inv_b);
    float comb = sa * sb;
#ifdef _OPENMP
#pragma omp parallel for num_threads(nt) schedule(dynamic, 1)
#endif
    for (uint32_t m = 0; m < M; m++) {
        const int8_t* a = Aq + (size_t)m * K;
        for (uint32_t n = 0; n < N; n++) {
            const int8_t* b = Bt + (size_t)n * K;
            int32_t s = 0;
            for (uint32_t k = 0; k < K; k++) s += (int32_t)a[k] * (int32_t)b[k];
            float y = (float)s;
            y = y * comb;
            y = y * scale;
            C[(size_t)m * N + n] = relu ? ane_ref_relu_max(y, 0.0f) : y;
        }
    }
    free(Aq);
    free(Bt);
}

void ane_ref_q8_0_gemv_omp(uint32_t M, uint32_t K, const float* x, const uint8_t* W, float* out,
                           int n_threads) {
    int nt = n_threads > 0 ? n_threads : ane_ref_max_threads();
#ifdef _OPENMP
#pragma omp parallel num_threads(nt)
    {
        int t = omp_get_thread_num(), T = omp_get_num_threads();
        uint32_t per = (M + T - 1) / T;
        uint32_t m0 = per * t, m1 = m0 + per > M ? M : m0 + per;
        if (m0 < m1) q8_0_gemv_rows(m0, m1, K, x, W, out);
    }
#else
    (void)nt;
    q8_0_gemv_rows(0, M, K, x, W, out);
#endif
}
