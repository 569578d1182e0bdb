/*
 * vvq2_oracle.c -- CPU restatement of the vibevoice.cpp Qwen2 hot path.
 *
 * TEST INFRASTRUCTURE ONLY (see vvq2_oracle.h).  Compiled with
 * -ffp-contract=off so every float operation rounds the way the written
 * expression says; no -ffast-math.
 */
#include "vvq2_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

#define QK8_0 32
#define QK_K 256

/* block layouts (ggml's public GGUF formats) */
typedef struct { uint16_t d; int8_t qs[QK8_0]; } blk_q8_0;                   /* 34 B  */
typedef struct { uint16_t d, dmin; uint8_t scales[12]; uint8_t qh[QK_K / 8];
                 uint8_t qs[QK_K / 2]; } blk_q5_K;                            /* 176 B */
typedef struct { uint8_t ql[QK_K / 2]; uint8_t qh[QK_K / 4]; int8_t scales[QK_K / 16];
                 uint16_t d; } blk_q6_K;                                      /* 210 B */
typedef struct { float d; int8_t qs[QK_K]; int16_t bsums[QK_K / 16]; } blk_q8_K; /* 292 B */

_Static_assert(sizeof(blk_q8_0) == 34, "q8_0 size");
_Static_assert(sizeof(blk_q5_K) == 176, "q5_K size");
_Static_assert(sizeof(blk_q6_K) == 210, "q6_K size");
_Static_assert(sizeof(blk_q8_K) == 292, "q8_K size");

/* ------------------------------------------------------------------ fp16 */

/* IEEE binary16 conversions, round to nearest even.  Where the build targets
 * F16C (x86-64-v3 and up) the hardware instructions do them; the software
 * routines below give the identical result for every non-NaN input (checked
 * over all 2^32 floats and all 2^16 halves) and serve other hosts. */
static uint16_t fp32_to_fp16_sw(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t mant = x & 0x7FFFFFu;
    const int32_t exp = (int32_t)((x >> 23) & 0xFFu);
    if (exp == 0xFF) return (uint16_t)(sign | 0x7C00u | (mant ? (0x200u | (mant >> 13)) : 0u));
    const int32_t e = exp - 127 + 15;
    if (e >= 0x1F) return (uint16_t)(sign | 0x7C00u);
    if (e <= 0) {                       /* f16 subnormal or zero, round to nearest even */
        if (e < -10) return (uint16_t)sign;
        mant |= 0x800000u;
        const int shift = 14 - e;
        uint32_t hm = mant >> shift;
        const uint32_t rem = mant & ((1u << shift) - 1u);
        const uint32_t half = 1u << (shift - 1);
        if (rem > half || (rem == half && (hm & 1u))) hm++;
        return (uint16_t)(sign | hm);
    }
    uint32_t h = sign | ((uint32_t)e << 10) | (mant >> 13);
    const uint32_t rem = mant & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;   /* carry may bump exponent: correct */
    return (uint16_t)h;
}

static float fp16_to_fp32_sw(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    const uint32_t exp = (h >> 10) & 0x1Fu;
    const uint32_t mant = h & 0x3FFu;
    uint32_t x;
    if (exp == 0) {
        if (mant == 0) {
            x = sign;
        } else {
            float v = ldexpf((float)mant, -24);
            memcpy(&x, &v, 4);
            x |= sign;
        }
    } else if (exp == 0x1F) {
        x = sign | 0x7F800000u | (mant << 13);
    } else {
        x = sign | ((exp - 15u + 127u) << 23) | (mant << 13);
    }
    float f;
    memcpy(&f, &x, 4);
    return f;
}

#if defined(__F16C__)
#include <immintrin.h>
uint16_t vvo_fp32_to_fp16(float f) { return (uint16_t)_cvtss_sh(f, _MM_FROUND_TO_NEAREST_INT); }
float vvo_fp16_to_fp32(uint16_t h) { return _cvtsh_ss(h); }
#else
uint16_t vvo_fp32_to_fp16(float f) { return fp32_to_fp16_sw(f); }
float vvo_fp16_to_fp32(uint16_t h) { return fp16_to_fp32_sw(h); }
#endif

static float f16r(float x) { return vvo_fp16_to_fp32(vvo_fp32_to_fp16(x)); }

int vvo_block_elems(int type) {
    switch (type) {
        case VVO_F32: case VVO_F16: return 1;
        case VVO_Q8_0: return QK8_0;
        case VVO_Q5_K: case VVO_Q6_K: return QK_K;
        default: return 0;
    }
}

static size_t block_bytes(int type) {
    switch (type) {
        case VVO_F32: return 4;
        case VVO_F16: return 2;
        case VVO_Q8_0: return sizeof(blk_q8_0);
        case VVO_Q5_K: return sizeof(blk_q5_K);
        case VVO_Q6_K: return sizeof(blk_q6_K);
        default: return 0;
    }
}

size_t vvo_row_bytes(int type, int64_t n) {
    const int be = vvo_block_elems(type);
    if (be == 0 || n % be) return 0;
    return (size_t)(n / be) * block_bytes(type);
}

/* ------------------------------------------------------------ dequantize */

/* ggml dequantize_row_q8_0: y = d * q */
static void deq_q8_0(const blk_q8_0* b, int64_t nb, float* y) {
    for (int64_t i = 0; i < nb; i++) {
        const float d = vvo_fp16_to_fp32(b[i].d);
        for (int j = 0; j < QK8_0; j++) y[i * QK8_0 + j] = (float)b[i].qs[j] * d;
    }
}

/* ggml get_scale_min_k4: 6-bit scale/min pairs packed in 12 bytes */
static void scale_min_k4(int j, const uint8_t* q, uint8_t* d, uint8_t* m) {
    if (j < 4) {
        *d = q[j] & 63;
        *m = q[j + 4] & 63;
    } else {
        *d = (uint8_t)((q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4));
        *m = (uint8_t)((q[j + 4] >> 4) | ((q[j] >> 6) << 4));
    }
}

/* ggml dequantize_row_q5_K: y = (d*sc)*q - (dmin*m), q = 4 low bits | high bit */
static void deq_q5_K(const blk_q5_K* b, int64_t nb, float* y) {
    for (int64_t i = 0; i < nb; i++) {
        const uint8_t* ql = b[i].qs;
        const uint8_t* qh = b[i].qh;
        const float d = vvo_fp16_to_fp32(b[i].d);
        const float mn = vvo_fp16_to_fp32(b[i].dmin);
        int is = 0;
        uint8_t u1 = 1, u2 = 2;
        for (int j = 0; j < QK_K; j += 64) {
            uint8_t sc, m;
            scale_min_k4(is + 0, b[i].scales, &sc, &m);
            const float d1 = d * sc, m1 = mn * m;
            scale_min_k4(is + 1, b[i].scales, &sc, &m);
            const float d2 = d * sc, m2 = mn * m;
            for (int l = 0; l < 32; ++l) *y++ = d1 * (float)((ql[l] & 0xF) + (qh[l] & u1 ? 16 : 0)) - m1;
            for (int l = 0; l < 32; ++l) *y++ = d2 * (float)((ql[l] >> 4) + (qh[l] & u2 ? 16 : 0)) - m2;
            ql += 32;
            is += 2;
            u1 = (uint8_t)(u1 << 2);
            u2 = (uint8_t)(u2 << 2);
        }
    }
}

/* ggml dequantize_row_q6_K: y = (d*sc)*(q-32) */
static void deq_q6_K(const blk_q6_K* b, int64_t nb, float* y) {
    for (int64_t i = 0; i < nb; i++) {
        const float d = vvo_fp16_to_fp32(b[i].d);
        const uint8_t* ql = b[i].ql;
        const uint8_t* qh = b[i].qh;
        const int8_t* sc = b[i].scales;
        for (int n = 0; n < QK_K; n += 128) {
            for (int l = 0; l < 32; ++l) {
                const int is = l / 16;
                const int q1 = (int)((ql[l + 0] & 0xF) | (((qh[l] >> 0) & 3) << 4)) - 32;
                const int q2 = (int)((ql[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4)) - 32;
                const int q3 = (int)((ql[l + 0] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
                const int q4 = (int)((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
                y[l + 0] = d * (float)sc[is + 0] * (float)q1;
                y[l + 32] = d * (float)sc[is + 2] * (float)q2;
                y[l + 64] = d * (float)sc[is + 4] * (float)q3;
                y[l + 96] = d * (float)sc[is + 6] * (float)q4;
            }
            y += 128;
            ql += 64;
            qh += 32;
            sc += 8;
        }
    }
}

int vvo_dequantize(int type, const void* src, int64_t n, float* dst) {
    const int be = vvo_block_elems(type);
    if (!be || n % be) return -2;
    switch (type) {
        case VVO_F32: memcpy(dst, src, (size_t)n * 4); return 0;
        case VVO_F16: {
            const uint16_t* h = (const uint16_t*)src;
            for (int64_t i = 0; i < n; i++) dst[i] = vvo_fp16_to_fp32(h[i]);
            return 0;
        }
        case VVO_Q8_0: deq_q8_0((const blk_q8_0*)src, n / QK8_0, dst); return 0;
        case VVO_Q5_K: deq_q5_K((const blk_q5_K*)src, n / QK_K, dst); return 0;
        case VVO_Q6_K: deq_q6_K((const blk_q6_K*)src, n / QK_K, dst); return 0;
        default: return -6;
    }
}

/* -------------------------------------------------------------- quantize */

/* ggml quantize_row_q8_0_ref: d = amax/127, id = 1/d, q = roundf(x*id) */
int vvo_quantize_q8_0(const float* x, int64_t n, void* dst) {
    if (n % QK8_0) return -2;
    blk_q8_0* y = (blk_q8_0*)dst;
    for (int64_t i = 0; i < n / QK8_0; i++) {
        float amax = 0.0f;
        for (int j = 0; j < QK8_0; j++) {
            const float v = fabsf(x[i * QK8_0 + j]);
            if (v > amax) amax = v;
        }
        const float d = amax / 127.0f;
        const float id = d != 0.0f ? 1.0f / d : 0.0f;
        y[i].d = vvo_fp32_to_fp16(d);
        for (int j = 0; j < QK8_0; j++) y[i].qs[j] = (int8_t)roundf(x[i * QK8_0 + j] * id);
    }
    return 0;
}

/* ggml nearest_int: round half to even (magic-number add in RNE mode) */
static int nearest_int(float f) { return (int)rintf(f); }

/* ggml quantize_row_q8_K_ref: iscale = -127/max (max = signed value of
 * largest magnitude), q = min(127, nearest_int(iscale*x)), d = 1/iscale */
int vvo_quantize_q8_K(const float* x, int64_t n, void* dst) {
    if (n % QK_K) return -2;
    blk_q8_K* y = (blk_q8_K*)dst;
    for (int64_t i = 0; i < n / QK_K; i++, x += QK_K) {
        float max = 0.0f, amax = 0.0f;
        for (int j = 0; j < QK_K; ++j) {
            const float ax = fabsf(x[j]);
            if (ax > amax) { amax = ax; max = x[j]; }
        }
        if (amax == 0.0f) {
            memset(&y[i], 0, sizeof(y[i]));
            continue;
        }
        const float iscale = -127.0f / max;
        for (int j = 0; j < QK_K; ++j) {
            const int v = nearest_int(iscale * x[j]);
            y[i].qs[j] = (int8_t)(v < 127 ? v : 127);
        }
        for (int j = 0; j < QK_K / 16; ++j) {
            int s = 0;
            for (int l = 0; l < 16; ++l) s += y[i].qs[j * 16 + l];
            y[i].bsums[j] = (int16_t)s;
        }
        y[i].d = 1.0f / iscale;
    }
    return 0;
}

static int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

/* Test-weight generator for Q6_K: per 16-wide sub-block scale = amax/31,
 * super-block d = max|scale|/127, int8 sub-scales, 6-bit q offset by 32. */
int vvo_quantize_q6_K(const float* x, int64_t n, void* dst) {
    if (n % QK_K) return -2;
    blk_q6_K* y = (blk_q6_K*)dst;
    for (int64_t i = 0; i < n / QK_K; i++, x += QK_K) {
        float sub[16], smax = 0.0f;
        for (int j = 0; j < 16; j++) {
            float a = 0.0f;
            for (int l = 0; l < 16; l++) { const float v = fabsf(x[j * 16 + l]); if (v > a) a = v; }
            sub[j] = a / 31.0f;
            if (sub[j] > smax) smax = sub[j];
        }
        memset(&y[i], 0, sizeof(y[i]));
        const float d = smax / 127.0f;
        y[i].d = vvo_fp32_to_fp16(d);
        const float dr = vvo_fp16_to_fp32(y[i].d);
        int8_t sc[16];
        uint8_t q[QK_K];
        for (int j = 0; j < 16; j++) {
            sc[j] = (int8_t)(dr > 0 ? clampi((int)lrintf(sub[j] / dr), -127, 127) : 0);
            y[i].scales[j] = sc[j];
            const float s = dr * (float)sc[j];
            for (int l = 0; l < 16; l++) {
                const int v = s != 0.0f ? (int)lrintf(x[j * 16 + l] / s) : 0;
                q[j * 16 + l] = (uint8_t)(clampi(v, -32, 31) + 32);
            }
        }
        /* pack: element e in half n (128), position l (32), quarter k (4) */
        for (int h = 0; h < 2; h++) {
            uint8_t* ql = y[i].ql + 64 * h;
            uint8_t* qh = y[i].qh + 32 * h;
            const uint8_t* qq = q + 128 * h;
            for (int l = 0; l < 32; l++) {
                const uint8_t q1 = qq[l], q2 = qq[l + 32], q3 = qq[l + 64], q4 = qq[l + 96];
                ql[l] = (uint8_t)((q1 & 0xF) | ((q3 & 0xF) << 4));
                ql[l + 32] = (uint8_t)((q2 & 0xF) | ((q4 & 0xF) << 4));
                qh[l] = (uint8_t)((q1 >> 4) | ((q2 >> 4) << 2) | ((q3 >> 4) << 4) | ((q4 >> 4) << 6));
            }
        }
    }
    return 0;
}

/* Test-weight generator for Q5_K: per 32-wide sub-block affine
 * x ~ (d*sc)*q - (dmin*m), 6-bit sc/m, 5-bit q. */
int vvo_quantize_q5_K(const float* x, int64_t n, void* dst) {
    if (n % QK_K) return -2;
    blk_q5_K* y = (blk_q5_K*)dst;
    for (int64_t i = 0; i < n / QK_K; i++, x += QK_K) {
        float scl[8], mns[8], smax = 0.0f, mmax = 0.0f;
        for (int j = 0; j < 8; j++) {
            float lo = x[j * 32], hi = x[j * 32];
            for (int l = 1; l < 32; l++) {
                const float v = x[j * 32 + l];
                if (v < lo) lo = v;
                if (v > hi) hi = v;
            }
            if (lo > 0) lo = 0;
            scl[j] = (hi - lo) / 31.0f;
            mns[j] = -lo;
            if (scl[j] > smax) smax = scl[j];
            if (mns[j] > mmax) mmax = mns[j];
        }
        memset(&y[i], 0, sizeof(y[i]));
        y[i].d = vvo_fp32_to_fp16(smax / 63.0f);
        y[i].dmin = vvo_fp32_to_fp16(mmax / 63.0f);
        const float dr = vvo_fp16_to_fp32(y[i].d), mr = vvo_fp16_to_fp32(y[i].dmin);
        uint8_t sc[8], mq[8], q[QK_K];
        for (int j = 0; j < 8; j++) {
            sc[j] = (uint8_t)(dr > 0 ? clampi((int)lrintf(scl[j] / dr), 0, 63) : 0);
            mq[j] = (uint8_t)(mr > 0 ? clampi((int)lrintf(mns[j] / mr), 0, 63) : 0);
            const float s = dr * sc[j], m = mr * mq[j];
            for (int l = 0; l < 32; l++) {
                const int v = s != 0.0f ? (int)lrintf((x[j * 32 + l] + m) / s) : 0;
                q[j * 32 + l] = (uint8_t)clampi(v, 0, 31);
            }
        }
        /* 6-bit scale/min packing, inverse of scale_min_k4 */
        for (int j = 0; j < 4; j++) {
            y[i].scales[j] = (uint8_t)((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
            y[i].scales[j + 4] = (uint8_t)((mq[j] & 63) | ((mq[j + 4] >> 4) << 6));
            y[i].scales[j + 8] = (uint8_t)((sc[j + 4] & 0xF) | ((mq[j + 4] & 0xF) << 4));
        }
        /* 64-element chunk c: low nibble (first 32) / high nibble (second 32),
         * high bit at qh bit 2c / 2c+1 */
        for (int c = 0; c < 4; c++) {
            for (int l = 0; l < 32; l++) {
                const uint8_t a = q[64 * c + l], b = q[64 * c + 32 + l];
                y[i].qs[32 * c + l] = (uint8_t)((a & 0xF) | ((b & 0xF) << 4));
                y[i].qh[l] |= (uint8_t)(((a >> 4) & 1) << (2 * c));
                y[i].qh[l] |= (uint8_t)(((b >> 4) & 1) << (2 * c + 1));
            }
        }
    }
    return 0;
}

/* ------------------------------------------------------------- vec dots */

/* ggml_vec_dot_q8_0_q8_0 (generic): sumf += sumi * (dx*dy), block order */
static float dot_q8_0(const blk_q8_0* w, const blk_q8_0* x, int nb) {
    float sumf = 0.0f;
    for (int ib = 0; ib < nb; ib++) {
        int sumi = 0;
        for (int j = 0; j < QK8_0; j++) sumi += (int)w[ib].qs[j] * (int)x[ib].qs[j];
        sumf += (float)sumi * (vvo_fp16_to_fp32(w[ib].d) * vvo_fp16_to_fp32(x[ib].d));
    }
    return sumf;
}

/* SIMD Q8_0 x Q8_0 dots (VVO_SIMD): the same per-block integer sums as
 * dot_q8_0, accumulated in vector lanes (the lane-wise float order of a SIMD
 * backend).  The signed x signed byte product uses the unsigned x signed
 * multiply-add: |w| * (x with the sign of w), exact since ggml's quantizer
 * never emits -128.  Only the timed CPU baseline uses these. */
#if defined(__x86_64__)
#include <immintrin.h>

__attribute__((target("avx2,fma,f16c"))) static float dot_q8_0_avx2(const blk_q8_0* w, const blk_q8_0* x, int nb) {
    __m256 acc = _mm256_setzero_ps();
    const __m256i ones = _mm256_set1_epi16(1);
    for (int ib = 0; ib < nb; ib++) {
        const __m256i a = _mm256_loadu_si256((const __m256i*)w[ib].qs);
        const __m256i b = _mm256_loadu_si256((const __m256i*)x[ib].qs);
        const __m256i p16 = _mm256_maddubs_epi16(_mm256_sign_epi8(a, a), _mm256_sign_epi8(b, a));
        const __m256 s = _mm256_cvtepi32_ps(_mm256_madd_epi16(p16, ones));
        const float d = _cvtsh_ss(w[ib].d) * _cvtsh_ss(x[ib].d);
        acc = _mm256_fmadd_ps(_mm256_set1_ps(d), s, acc);
    }
    __m128 h = _mm_add_ps(_mm256_castps256_ps128(acc), _mm256_extractf128_ps(acc, 1));
    h = _mm_add_ps(h, _mm_movehl_ps(h, h));
    h = _mm_add_ss(h, _mm_movehdup_ps(h));
    return _mm_cvtss_f32(h);
}

__attribute__((target("avx512f,avx512bw,avx512vnni,avx2,fma,f16c")))
static float dot_q8_0_vnni(const blk_q8_0* w, const blk_q8_0* x, int nb) {
    __m512 acc = _mm512_setzero_ps();
    int ib = 0;
    for (; ib + 1 < nb; ib += 2) {   /* two blocks per 512-bit register, one scale per half */
        const __m512i a = _mm512_inserti64x4(_mm512_castsi256_si512(_mm256_loadu_si256((const __m256i*)w[ib].qs)),
                                             _mm256_loadu_si256((const __m256i*)w[ib + 1].qs), 1);
        const __m512i b = _mm512_inserti64x4(_mm512_castsi256_si512(_mm256_loadu_si256((const __m256i*)x[ib].qs)),
                                             _mm256_loadu_si256((const __m256i*)x[ib + 1].qs), 1);
        const __mmask64 neg = _mm512_movepi8_mask(a);
        const __m512i sb = _mm512_mask_sub_epi8(b, neg, _mm512_setzero_si512(), b);
        const __m512 s = _mm512_cvtepi32_ps(_mm512_dpbusd_epi32(_mm512_setzero_si512(), _mm512_abs_epi8(a), sb));
        const float d0 = _cvtsh_ss(w[ib].d) * _cvtsh_ss(x[ib].d);
        const float d1 = _cvtsh_ss(w[ib + 1].d) * _cvtsh_ss(x[ib + 1].d);
        const __m512 dv = _mm512_mask_mov_ps(_mm512_set1_ps(d0), (__mmask16)0xFF00, _mm512_set1_ps(d1));
        acc = _mm512_fmadd_ps(dv, s, acc);
    }
    float sum = _mm512_reduce_add_ps(acc);
    if (ib < nb) sum += dot_q8_0_avx2(w + ib, x + ib, 1);
    return sum;
}

typedef float (*dot_q8_0_fn)(const blk_q8_0*, const blk_q8_0*, int);

static dot_q8_0_fn simd_dot(void) {
    __builtin_cpu_init();
    if (__builtin_cpu_supports("avx512vnni") && __builtin_cpu_supports("avx512bw")) return dot_q8_0_vnni;
    if (__builtin_cpu_supports("avx2") && __builtin_cpu_supports("fma")) return dot_q8_0_avx2;
    return NULL;
}

const char* vvo_simd_isa(void) {
    const dot_q8_0_fn f = simd_dot();
    return f == dot_q8_0_vnni ? "avx512vnni" : f == dot_q8_0_avx2 ? "avx2" : "generic";
}
#else
typedef float (*dot_q8_0_fn)(const blk_q8_0*, const blk_q8_0*, int);
static dot_q8_0_fn simd_dot(void) { return NULL; }
const char* vvo_simd_isa(void) { return "generic"; }
#endif

/* ggml_vec_dot_q6_K_q8_K (generic): per super-block isum = sum_j sc_j * dot_j,
 * sumf += (d_w * d_x) * isum */
static float dot_q6_K(const blk_q6_K* w, const blk_q8_K* x, int nb) {
    float sumf = 0.0f;
    for (int i = 0; i < nb; i++) {
        int8_t a[QK_K];
        const uint8_t* ql = w[i].ql;
        const uint8_t* qh = w[i].qh;
        for (int h = 0; h < 2; h++) {
            for (int l = 0; l < 32; l++) {
                a[128 * h + l + 0] = (int8_t)(((ql[l + 0] & 0xF) | (((qh[l] >> 0) & 3) << 4)) - 32);
                a[128 * h + l + 32] = (int8_t)(((ql[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4)) - 32);
                a[128 * h + l + 64] = (int8_t)(((ql[l + 0] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32);
                a[128 * h + l + 96] = (int8_t)(((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32);
            }
            ql += 64;
            qh += 32;
        }
        int isum = 0;
        for (int j = 0; j < 16; j++) {
            int s = 0;
            for (int l = 0; l < 16; l++) s += (int)a[j * 16 + l] * (int)x[i].qs[j * 16 + l];
            isum += (int)w[i].scales[j] * s;
        }
        const float d = vvo_fp16_to_fp32(w[i].d) * x[i].d;
        sumf += d * (float)isum;
    }
    return sumf;
}

/* ggml_vec_dot_q5_K_q8_K (generic): d*sum_j sc_j*dot_j - dmin*sum_j m_j*bsum_j */
static float dot_q5_K(const blk_q5_K* w, const blk_q8_K* x, int nb) {
    float sumf = 0.0f;
    for (int i = 0; i < nb; i++) {
        uint8_t a[QK_K];
        const uint8_t* ql = w[i].qs;
        const uint8_t* qh = w[i].qh;
        for (int c = 0; c < 4; c++) {
            for (int l = 0; l < 32; l++) {
                a[64 * c + l] = (uint8_t)((ql[l] & 0xF) + ((qh[l] >> (2 * c)) & 1 ? 16 : 0));
                a[64 * c + 32 + l] = (uint8_t)((ql[l] >> 4) + ((qh[l] >> (2 * c + 1)) & 1 ? 16 : 0));
            }
            ql += 32;
        }
        int isum = 0, msum = 0;
        for (int j = 0; j < 8; j++) {
            uint8_t sc, m;
            scale_min_k4(j, w[i].scales, &sc, &m);
            int s = 0;
            for (int l = 0; l < 32; l++) s += (int)a[j * 32 + l] * (int)x[i].qs[j * 32 + l];
            isum += (int)sc * s;
            msum += (int)m * ((int)x[i].bsums[2 * j] + (int)x[i].bsums[2 * j + 1]);
        }
        const float d = vvo_fp16_to_fp32(w[i].d) * x[i].d;
        const float dmin = vvo_fp16_to_fp32(w[i].dmin) * x[i].d;
        sumf += d * (float)isum;
        sumf -= dmin * (float)msum;
    }
    return sumf;
}

int vvo_matvec(const vvo_tensor* w, const float* x, float* y, int flags) {
    const int64_t K = w->ne0, R = w->ne1;
    const size_t rb = vvo_row_bytes(w->type, K);
    if (!rb) return -2;
    const uint8_t* base = (const uint8_t*)w->data;
    if (!(flags & VVO_ACT_GGML)) {
        /* exact: dequantized f32 weights x f32 activations, double sum */
#pragma omp parallel
        {
            float* row = (float*)malloc((size_t)K * sizeof(float));
#pragma omp for schedule(static)
            for (int64_t r = 0; r < R; r++) {
                vvo_dequantize(w->type, base + (size_t)r * rb, K, row);
                double s = 0.0;
                for (int64_t k = 0; k < K; k++) s += (double)row[k] * (double)x[k];
                y[r] = (float)s;
            }
            free(row);
        }
        return 0;
    }
    switch (w->type) {
        case VVO_F32: {
            const float* W = (const float*)base;
#pragma omp parallel for schedule(static)
            for (int64_t r = 0; r < R; r++) {
                double s = 0.0;   /* ggml_vec_dot_f32 generic: ggml_float accumulator */
                for (int64_t k = 0; k < K; k++) s += (double)(W[r * K + k] * x[k]);
                y[r] = (float)s;
            }
            return 0;
        }
        case VVO_F16: {
            const uint16_t* W = (const uint16_t*)base;
            float* xh = (float*)malloc((size_t)K * sizeof(float));
            for (int64_t k = 0; k < K; k++) xh[k] = f16r(x[k]);   /* vec_dot_type F16 */
#pragma omp parallel for schedule(static)
            for (int64_t r = 0; r < R; r++) {
                double s = 0.0;
                for (int64_t k = 0; k < K; k++) s += (double)(vvo_fp16_to_fp32(W[r * K + k]) * xh[k]);
                y[r] = (float)s;
            }
            free(xh);
            return 0;
        }
        case VVO_Q8_0: {
            blk_q8_0* xq = (blk_q8_0*)malloc((size_t)(K / QK8_0) * sizeof(blk_q8_0));
            vvo_quantize_q8_0(x, K, xq);
            dot_q8_0_fn dot = (flags & VVO_SIMD) ? simd_dot() : NULL;
            if (!dot) dot = dot_q8_0;
#pragma omp parallel for schedule(static)
            for (int64_t r = 0; r < R; r++)
                y[r] = dot((const blk_q8_0*)(base + (size_t)r * rb), xq, (int)(K / QK8_0));
            free(xq);
            return 0;
        }
        case VVO_Q5_K:
        case VVO_Q6_K: {
            blk_q8_K* xq = (blk_q8_K*)malloc((size_t)(K / QK_K) * sizeof(blk_q8_K));
            vvo_quantize_q8_K(x, K, xq);
#pragma omp parallel for schedule(static)
            for (int64_t r = 0; r < R; r++) {
                const void* wr = base + (size_t)r * rb;
                y[r] = w->type == VVO_Q5_K ? dot_q5_K((const blk_q5_K*)wr, xq, (int)(K / QK_K))
                                           : dot_q6_K((const blk_q6_K*)wr, xq, (int)(K / QK_K));
            }
            free(xq);
            return 0;
        }
        default: return -6;
    }
}

/* ---------------------------------------------------------- elementwise */

/* ggml_compute_forward_rms_norm_f32 followed by ggml_mul(w) */
void vvo_rms_norm(const float* x, const float* w, int n, float eps, float* y) {
    double sum = 0.0;
    for (int i = 0; i < n; i++) sum += (double)(x[i] * x[i]);
    const float mean = (float)(sum / n);
    const float scale = 1.0f / sqrtf(mean + eps);
    for (int i = 0; i < n; i++) y[i] = (x[i] * scale) * w[i];
}

/* NEOX rotate-half RoPE on [n_heads][hd] at one absolute position.
 * VVO_ROPE_GGML: ggml_rope_cache_init (theta_0 = pos, theta_{i+1} = theta_i *
 * powf(base, -2/hd), cosf/sinf) and the f32 rotation x0*c - x1*s, x0*s + x1*c.
 * Otherwise the fp64 formula of tests/dump_rope_reference.py:22-37. */
void vvo_rope_neox(const float* x, int n_heads, int hd, int pos, float base,
                   int flags, float* y) {
    const int half = hd / 2;
    float cs[512], sn[512];
    double cd[512], sd[512];
    if (flags & VVO_ROPE_GGML) {
        const float ts = powf(base, -2.0f / (float)hd);
        float th = (float)pos;
        for (int i = 0; i < half; i++) {
            cs[i] = cosf(th);
            sn[i] = sinf(th);
            th *= ts;
        }
    } else {
        for (int i = 0; i < half; i++) {
            const double inv = 1.0 / pow((double)base, (double)(2 * i) / (double)hd);
            const double a = (double)pos * inv;
            cd[i] = cos(a);
            sd[i] = sin(a);
        }
    }
    for (int h = 0; h < n_heads; h++) {
        const float* xi = x + (size_t)h * hd;
        float* yo = y + (size_t)h * hd;
        for (int i = 0; i < half; i++) {
            const float x0 = xi[i], x1 = xi[i + half];
            if (flags & VVO_ROPE_GGML) {
                yo[i] = x0 * cs[i] - x1 * sn[i];
                yo[i + half] = x0 * sn[i] + x1 * cs[i];
            } else {
                yo[i] = (float)((double)x0 * cd[i] - (double)x1 * sd[i]);
                yo[i + half] = (float)((double)x0 * sd[i] + (double)x1 * cd[i]);
            }
        }
    }
}

/* ---------------------------------------------------------------- model */

struct vvo_model {
    vvo_hparams hp;
    int n_rows, max_seq, flags;
    vvo_layer* layers;
    int* have_layer;
    vvo_tensor out_norm, lm_head, tok_embd;
    float* kc;   /* [n_layers][n_rows][max_seq][n_kv*hd] */
    float* vc;
    int* past;   /* [n_rows] */
};

static size_t kv_off(const vvo_model* m, int layer, int row, int pos) {
    const size_t kvw = (size_t)m->hp.n_kv_heads * m->hp.head_dim;
    return (((size_t)layer * m->n_rows + row) * m->max_seq + pos) * kvw;
}

vvo_model* vvo_model_new(const vvo_hparams* hp, int n_rows, int max_seq, int flags) {
    if (!hp || n_rows <= 0 || max_seq <= 0 || hp->head_dim > 1024 || hp->head_dim % 2) return NULL;
    vvo_model* m = (vvo_model*)calloc(1, sizeof(vvo_model));
    m->hp = *hp;
    m->n_rows = n_rows;
    m->max_seq = max_seq;
    m->flags = flags;
    m->layers = (vvo_layer*)calloc((size_t)hp->n_layers, sizeof(vvo_layer));
    m->have_layer = (int*)calloc((size_t)hp->n_layers, sizeof(int));
    const size_t n = (size_t)hp->n_layers * n_rows * max_seq * hp->n_kv_heads * hp->head_dim;
    m->kc = (float*)calloc(n, sizeof(float));
    m->vc = (float*)calloc(n, sizeof(float));
    m->past = (int*)calloc((size_t)n_rows, sizeof(int));
    if (!m->layers || !m->kc || !m->vc || !m->past) { vvo_model_free(m); return NULL; }
    return m;
}

void vvo_model_free(vvo_model* m) {
    if (!m) return;
    free(m->layers); free(m->have_layer); free(m->kc); free(m->vc); free(m->past);
    free(m);
}

int vvo_model_set_layer(vvo_model* m, int layer, const vvo_layer* w) {
    if (!m || !w || layer < 0 || layer >= m->hp.n_layers) return -2;
    m->layers[layer] = *w;
    m->have_layer[layer] = 1;
    return 0;
}

int vvo_model_set_output(vvo_model* m, const vvo_tensor* on, const vvo_tensor* lm,
                         const vvo_tensor* te) {
    if (!m) return -2;
    if (on) m->out_norm = *on;
    if (lm) m->lm_head = *lm;
    if (te) m->tok_embd = *te;
    return 0;
}

static float kv_store(const vvo_model* m, float v) { return (m->flags & VVO_KV_F16) ? f16r(v) : v; }

int vvo_kv_load(vvo_model* m, int row, int layer, const float* k, const float* v, int n_pos) {
    if (!m || row < 0 || row >= m->n_rows || layer < 0 || layer >= m->hp.n_layers ||
        n_pos < 0 || n_pos > m->max_seq) return -2;
    const size_t kvw = (size_t)m->hp.n_kv_heads * m->hp.head_dim;
    for (size_t i = 0; i < (size_t)n_pos * kvw; i++) {
        m->kc[kv_off(m, layer, row, 0) + i] = kv_store(m, k[i]);
        m->vc[kv_off(m, layer, row, 0) + i] = kv_store(m, v[i]);
    }
    return 0;
}

int vvo_kv_read(const vvo_model* m, int row, int layer, float* k, float* v, int n_pos) {
    if (!m || row < 0 || row >= m->n_rows || layer < 0 || layer >= m->hp.n_layers ||
        n_pos < 0 || n_pos > m->max_seq) return -2;
    const size_t kvw = (size_t)m->hp.n_kv_heads * m->hp.head_dim;
    memcpy(k, m->kc + kv_off(m, layer, row, 0), (size_t)n_pos * kvw * sizeof(float));
    memcpy(v, m->vc + kv_off(m, layer, row, 0), (size_t)n_pos * kvw * sizeof(float));
    return 0;
}

int vvo_set_past_len(vvo_model* m, int row, int past_len) {
    if (!m || row < 0 || row >= m->n_rows || past_len < 0 || past_len > m->max_seq) return -2;
    m->past[row] = past_len;
    return 0;
}

int vvo_past_len(const vvo_model* m, int row) {
    if (!m || row < 0 || row >= m->n_rows) return -2;
    return m->past[row];
}

static void add_bias(const vvo_tensor* b, float* y, int n) {
    if (!b->data) return;
    float tmp[8192];
    const float* bb = (const float*)b->data;
    if (b->type != VVO_F32) {
        vvo_dequantize(b->type, b->data, n, tmp);
        bb = tmp;
    }
    for (int i = 0; i < n; i++) y[i] += bb[i];
}

static const float* as_f32(const vvo_tensor* t, float* scratch, int n) {
    if (t->type == VVO_F32) return (const float*)t->data;
    vvo_dequantize(t->type, t->data, n, scratch);
    return scratch;
}

#if defined(__x86_64__)
/* attend() in the VVO_FA_F16ACC mode with 8-lane AVX2 / F16C arithmetic (the
 * VVO_SIMD timed baseline): the same per-key updates -- online max, the f16
 * VKQ accumulator rounded after every scale and every add -- with the Q.K
 * product summed in 8 float lanes instead of one double chain.  hd % 8 == 0. */
__attribute__((target("avx2,fma,f16c"))) static void attend_f16acc_simd(const float* qv, const float* K,
                                                                         const float* V, size_t stride,
                                                                         int hd, int lim, float scale,
                                                                         float* out) {
    float M = -INFINITY, S = 0.0f;
    __m256 acc[128];
    __m256 q8[128];
    const int nv = hd / 8;
    for (int c = 0; c < nv; c++) {
        acc[c] = _mm256_setzero_ps();
        q8[c] = _mm256_cvtph_ps(_mm256_cvtps_ph(_mm256_loadu_ps(qv + 8 * c), _MM_FROUND_TO_NEAREST_INT));
    }
    for (int j = 0; j < lim; j++) {
        const float* kj = K + (size_t)j * stride;
        __m256 d8 = _mm256_setzero_ps();
        for (int c = 0; c < nv; c++) d8 = _mm256_fmadd_ps(q8[c], _mm256_loadu_ps(kj + 8 * c), d8);
        __m128 h = _mm_add_ps(_mm256_castps256_ps128(d8), _mm256_extractf128_ps(d8, 1));
        h = _mm_add_ps(h, _mm_movehl_ps(h, h));
        h = _mm_add_ss(h, _mm_movehdup_ps(h));
        const float s = _mm_cvtss_f32(h) * scale;
        const float Mold = M;
        float ms = 1.0f, vs = 1.0f;
        if (s > M) {
            M = s;
            ms = expf(Mold - M);
            const __m256 m8 = _mm256_set1_ps(ms);
            for (int c = 0; c < nv; c++)
                acc[c] = _mm256_cvtph_ps(_mm256_cvtps_ph(_mm256_mul_ps(acc[c], m8), _MM_FROUND_TO_NEAREST_INT));
        } else {
            vs = expf(s - M);
        }
        const float* vj = V + (size_t)j * stride;
        const __m256 v8s = _mm256_set1_ps(vs);
        for (int c = 0; c < nv; c++)
            acc[c] = _mm256_cvtph_ps(_mm256_cvtps_ph(_mm256_fmadd_ps(_mm256_loadu_ps(vj + 8 * c), v8s, acc[c]),
                                                     _MM_FROUND_TO_NEAREST_INT));
        S = S * ms + vs;
    }
    const __m256 inv = _mm256_set1_ps(1.0f / S);
    for (int c = 0; c < nv; c++) _mm256_storeu_ps(out + 8 * c, _mm256_mul_ps(acc[c], inv));
}

static int have_avx2_f16c(void) {
    __builtin_cpu_init();
    return __builtin_cpu_supports("avx2") && __builtin_cpu_supports("fma") && __builtin_cpu_supports("f16c");
}
#endif

/* one query head against keys [0, L) with key j visible iff j <= qpos */
static void attend(const vvo_model* m, const float* q, int layer, int row, int kvh, int L,
                   int qpos, float* out) {
    const int hd = m->hp.head_dim, nkv = m->hp.n_kv_heads;
    const float scale = 1.0f / sqrtf((float)hd);
    const int lim = qpos + 1 < L ? qpos + 1 : L;
    float qv[1024];
    for (int d = 0; d < hd; d++) qv[d] = (m->flags & VVO_Q_F16) ? f16r(q[d]) : q[d];
    const float* K = m->kc + kv_off(m, layer, row, 0) + (size_t)kvh * hd;
    const float* V = m->vc + kv_off(m, layer, row, 0) + (size_t)kvh * hd;
    const size_t stride = (size_t)nkv * hd;
#if defined(__x86_64__)
    if ((m->flags & VVO_FA_F16ACC) && (m->flags & VVO_SIMD) && hd % 8 == 0 && hd <= 1024 && have_avx2_f16c()) {
        attend_f16acc_simd(qv, K, V, stride, hd, lim, scale, out);
        return;
    }
#endif
    if (m->flags & VVO_FA_F16ACC) {
        /* ggml_compute_forward_flash_attn_ext_f16_one_chunk with F16 V:
         * online softmax, VKQ16 accumulator rounded to f16 every update */
        float M = -INFINITY, S = 0.0f;
        float acc[1024];
        for (int d = 0; d < hd; d++) acc[d] = 0.0f;
        for (int j = 0; j < lim; j++) {
            double sd = 0.0;   /* ggml_vec_dot_f16: f16 x f16 products, ggml_float sum */
            for (int d = 0; d < hd; d++) sd += (double)(f16r(qv[d]) * K[j * stride + d]);
            const float s = (float)sd * scale;
            const float Mold = M;
            float ms = 1.0f, vs = 1.0f;
            if (s > M) {
                M = s;
                ms = expf(Mold - M);
                for (int d = 0; d < hd; d++) acc[d] = f16r(acc[d] * ms);
            } else {
                vs = expf(s - M);
            }
            for (int d = 0; d < hd; d++) acc[d] = f16r(acc[d] + V[j * stride + d] * vs);
            S = S * ms + vs;
        }
        const float Sinv = 1.0f / S;
        for (int d = 0; d < hd; d++) out[d] = acc[d] * Sinv;
        return;
    }
    /* exact two-pass softmax in double */
    double* sc = (double*)malloc((size_t)lim * sizeof(double));
    double mx = -INFINITY;
    for (int j = 0; j < lim; j++) {
        double s = 0.0;
        for (int d = 0; d < hd; d++) s += (double)qv[d] * (double)K[j * stride + d];
        sc[j] = s * (double)scale;
        if (sc[j] > mx) mx = sc[j];
    }
    double l = 0.0, o[1024];
    for (int d = 0; d < hd; d++) o[d] = 0.0;
    for (int j = 0; j < lim; j++) {
        const double p = exp(sc[j] - mx);
        l += p;
        for (int d = 0; d < hd; d++) o[d] += p * (double)V[j * stride + d];
    }
    for (int d = 0; d < hd; d++) out[d] = (float)(o[d] / l);
    free(sc);
}

/* ggml_vec_swiglu_f32: silu(g) * u with silu(x) = x / (1 + expf(-x)) */
static float silu(float x) { return x / (1.0f + expf(-x)); }

int vvo_forward(vvo_model* m, int n_sel, const int* rows, int n_tok, const float* x,
                const int* pos_start, int first_layer, int n_layers, int apply_output_norm,
                int advance, float* y) {
    if (!m || n_sel <= 0 || n_tok <= 0 || first_layer < 0 ||
        first_layer + n_layers > m->hp.n_layers) return -2;
    const vvo_hparams* hp = &m->hp;
    const int H = hp->hidden, nq = hp->n_heads, nkv = hp->n_kv_heads, hd = hp->head_dim;
    const int qw = nq * hd, kvw = nkv * hd, F = hp->ffn, grp = nq / nkv;
    for (int s = 0; s < n_sel; s++) {
        if (rows[s] < 0 || rows[s] >= m->n_rows) return -2;
        if (m->past[rows[s]] + n_tok > m->max_seq) return -2;   /* never abort on overflow */
    }
    for (int li = first_layer; li < first_layer + n_layers; li++)
        if (!m->have_layer[li]) return -2;
    const int fl = m->flags;
    const size_t nrow = (size_t)n_sel * n_tok;
    float* h = (float*)malloc(nrow * H * sizeof(float));
    memcpy(h, x, nrow * H * sizeof(float));
    float* xn = (float*)malloc((size_t)H * sizeof(float));
    float* q = (float*)malloc(nrow * qw * sizeof(float));
    float* tmp = (float*)malloc((size_t)(qw > F ? qw : F) * sizeof(float));
    float* att = (float*)malloc(nrow * qw * sizeof(float));
    float* g = (float*)malloc((size_t)F * sizeof(float));
    float* u = (float*)malloc((size_t)F * sizeof(float));
    float* o = (float*)malloc((size_t)H * sizeof(float));
    float* nw = (float*)malloc((size_t)H * sizeof(float));
    float* k = (float*)malloc((size_t)kvw * sizeof(float));
    float* v = (float*)malloc((size_t)kvw * sizeof(float));
    for (int li = first_layer; li < first_layer + n_layers; li++) {
        const vvo_layer* w = &m->layers[li];
        /* 1. norm, Q/K/V, bias, RoPE, K/V append for every new token */
        for (int s = 0; s < n_sel; s++) {
            const int r = rows[s];
            for (int t = 0; t < n_tok; t++) {
                const float* hx = h + ((size_t)s * n_tok + t) * H;
                vvo_rms_norm(hx, as_f32(&w->attn_norm, nw, H), H, hp->rms_eps, xn);
                vvo_matvec(&w->attn_q, xn, tmp, fl);
                add_bias(&w->attn_q_bias, tmp, qw);
                vvo_rope_neox(tmp, nq, hd, pos_start[s] + t, hp->rope_theta, fl,
                              q + ((size_t)s * n_tok + t) * qw);
                vvo_matvec(&w->attn_k, xn, tmp, fl);
                add_bias(&w->attn_k_bias, tmp, kvw);
                vvo_rope_neox(tmp, nkv, hd, pos_start[s] + t, hp->rope_theta, fl, k);
                vvo_matvec(&w->attn_v, xn, v, fl);
                add_bias(&w->attn_v_bias, v, kvw);
                float* kd = m->kc + kv_off(m, li, r, m->past[r] + t);
                float* vd = m->vc + kv_off(m, li, r, m->past[r] + t);
                for (int i = 0; i < kvw; i++) { kd[i] = kv_store(m, k[i]); vd[i] = kv_store(m, v[i]); }
            }
        }
        /* 2. attention of every (row, token, head) in one parallel region,
         *    then O-proj, residual, FFN per row */
#pragma omp parallel for schedule(dynamic)
        for (int64_t i = 0; i < (int64_t)nrow * nq; i++) {
            const int st = (int)(i / nq), hh = (int)(i % nq), s = st / n_tok, t = st % n_tok;
            attend(m, q + (size_t)st * qw + (size_t)hh * hd, li, rows[s], hh / grp, m->past[rows[s]] + n_tok,
                   pos_start[s] + t, att + (size_t)st * qw + (size_t)hh * hd);
        }
        for (int s = 0; s < n_sel; s++) {
            for (int t = 0; t < n_tok; t++) {
                float* hx = h + ((size_t)s * n_tok + t) * H;
                vvo_matvec(&w->attn_o, att + ((size_t)s * n_tok + t) * qw, o, fl);
                for (int i = 0; i < H; i++) hx[i] = hx[i] + o[i];
                if (fl & VVO_NO_FFN) continue;
                vvo_rms_norm(hx, as_f32(&w->ffn_norm, nw, H), H, hp->rms_eps, xn);
                vvo_matvec(&w->ffn_gate, xn, g, fl);
                vvo_matvec(&w->ffn_up, xn, u, fl);
                for (int i = 0; i < F; i++) g[i] = silu(g[i]) * u[i];
                vvo_matvec(&w->ffn_down, g, o, fl);
                for (int i = 0; i < H; i++) hx[i] = hx[i] + o[i];
            }
        }
    }
    if (apply_output_norm && m->out_norm.data) {
        for (size_t i = 0; i < nrow; i++) {
            memcpy(xn, h + i * H, (size_t)H * sizeof(float));
            vvo_rms_norm(xn, as_f32(&m->out_norm, nw, H), H, hp->rms_eps, h + i * H);
        }
    }
    memcpy(y, h, nrow * H * sizeof(float));
    if (advance)
        for (int s = 0; s < n_sel; s++) m->past[rows[s]] += n_tok;
    free(h); free(xn); free(q); free(tmp); free(att); free(g); free(u); free(o); free(nw);
    free(k); free(v);
    return 0;
}

int vvo_lm_head(vvo_model* m, int n, const float* h, float* logits, int* argmax) {
    if (!m || !m->lm_head.data) return -2;
    const int64_t V = m->lm_head.ne1, H = m->hp.hidden;
    float* lg = (float*)malloc((size_t)V * sizeof(float));
    for (int i = 0; i < n; i++) {
        vvo_matvec(&m->lm_head, h + (size_t)i * H, lg, m->flags);
        if (logits) memcpy(logits + (size_t)i * V, lg, (size_t)V * sizeof(float));
        if (argmax) {     /* first maximum, strict > as src/vibevoice_asr.cpp:702-706 */
            int best = 0;
            for (int64_t j = 1; j < V; j++) if (lg[j] > lg[best]) best = (int)j;
            argmax[i] = best;
        }
    }
    free(lg);
    return 0;
}

int vvo_embed(vvo_model* m, int n, const int* tok, float* out) {
    if (!m || !m->tok_embd.data) return -2;
    const int64_t H = m->tok_embd.ne0;
    const size_t rb = vvo_row_bytes(m->tok_embd.type, H);
    for (int i = 0; i < n; i++) {
        if (tok[i] < 0 || tok[i] >= m->tok_embd.ne1) return -2;
        vvo_dequantize(m->tok_embd.type, (const uint8_t*)m->tok_embd.data + (size_t)tok[i] * rb, H,
                       out + (size_t)i * H);
    }
    return 0;
}
