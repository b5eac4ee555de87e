/*
 * iq_oracle_avx2.c -- the reference-order quantized dot products with AVX2,
 * several input rows per pass over a weight row.
 *
 * TEST INFRASTRUCTURE ONLY (see iq_oracle.h): the CPU baseline's fast path.
 * Bitwise equal to the scalar restatements in iq_oracle_dot.c (ref_q4k,
 * ref_q6k, ref_q80): the same exact integer sums per 32-bit lane n (bytes
 * 4n..4n+3 of every 32-byte chunk), one fused multiply-add per lane and
 * block, the same horizontal sums (Q5_K: the one-chunk block order of
 * ref_q5k).  Like the reference's tiled kernels
 * (src/qgemm.rs:175-397, 399-438), a weight block is decoded once for up to
 * eight input rows.  Used only when the CPU has AVX2, FMA and F16C.
 */
#include "iq_oracle.h"
#include <immintrin.h>
#include <math.h>
#include <string.h>

#define AVX2 __attribute__((target("avx2,fma,f16c")))

/* f16 -> f32 with the F16C instruction (exact: every f16 value is an f32) */
static inline AVX2 float f16f(const uint8_t* p) { return _cvtsh_ss((unsigned short)(p[0] | (p[1] << 8))); }
static inline float hsum8f(const float a[8]) {
    float r0 = a[4] + a[0], r1 = a[5] + a[1], r2 = a[6] + a[2], r3 = a[7] + a[3];
    return (r0 + r2) + (r1 + r3);
}
static inline float hsum4f(const float a[4]) { return (a[0] + a[2]) + (a[1] + a[3]); }

static void scales_mins(const uint8_t* s, uint8_t sc[8], uint8_t mn[8]) {
    for (int j = 0; j < 4; j++) {
        sc[j] = s[j] & 63;
        mn[j] = s[j + 4] & 63;
        sc[j + 4] = (s[j + 8] & 0xf) | ((s[j] >> 6) << 4);
        mn[j + 4] = (s[j + 8] >> 4) | ((s[j + 4] >> 6) << 4);
    }
}

int or_have_avx2(void) {
    __builtin_cpu_init();
    return __builtin_cpu_supports("avx2") && __builtin_cpu_supports("fma") && __builtin_cpu_supports("f16c");
}

/* Q4_K row against T <= 8 Q8_K input rows (blocks of 292 bytes: f32 d,
 * i8 qs[256], i16 bsums[16]); out[t]. */
static inline __attribute__((always_inline)) AVX2 void q4k_rows_t(const uint8_t* w, int nb,
                                                                 const uint8_t* const* xs, const int T, float* out) {
    const __m256i m4 = _mm256_set1_epi8(0xF);
    __m256 acc[8];
    __m128 accm[8];
    for (int t = 0; t < T; t++) { acc[t] = _mm256_setzero_ps(); accm[t] = _mm_setzero_ps(); }
    for (int b = 0; b < nb; b++) {
        const uint8_t* blk = w + 144 * b;
        uint8_t sc[8], mn[8];
        scales_mins(blk + 4, sc, mn);
        const float xd = f16f(blk), xdmin = f16f(blk + 2);
        const __m128i mins = _mm_setr_epi16(mn[0], mn[1], mn[2], mn[3], mn[4], mn[5], mn[6], mn[7]);
        __m256i sumi[8];
        for (int t = 0; t < T; t++) sumi[t] = _mm256_setzero_si256();
        for (int j = 0; j < 4; j++) {
            const __m256i q4 = _mm256_loadu_si256((const __m256i*)(blk + 16 + 32 * j));
            const __m256i lo = _mm256_and_si256(q4, m4), hi = _mm256_and_si256(_mm256_srli_epi16(q4, 4), m4);
            const __m256i sl = _mm256_set1_epi16(sc[2 * j]), sh = _mm256_set1_epi16(sc[2 * j + 1]);
            for (int t = 0; t < T; t++) {
                const uint8_t* yq = xs[t] + 292 * b + 4 + 64 * j;
                const __m256i yl = _mm256_loadu_si256((const __m256i*)yq);
                const __m256i yh = _mm256_loadu_si256((const __m256i*)(yq + 32));
                const __m256i pl = _mm256_madd_epi16(sl, _mm256_maddubs_epi16(lo, yl));
                const __m256i ph = _mm256_madd_epi16(sh, _mm256_maddubs_epi16(hi, yh));
                sumi[t] = _mm256_add_epi32(sumi[t], _mm256_add_epi32(pl, ph));
            }
        }
        for (int t = 0; t < T; t++) {
            const uint8_t* y = xs[t] + 292 * b;
            float yd;
            memcpy(&yd, y, 4);
            const float d = yd * xd, dmin = -yd * xdmin;
            acc[t] = _mm256_fmadd_ps(_mm256_set1_ps(d), _mm256_cvtepi32_ps(sumi[t]), acc[t]);
            const __m256i bs = _mm256_loadu_si256((const __m256i*)(y + 260));
            const __m128i q8s = _mm_hadd_epi16(_mm256_castsi256_si128(bs), _mm256_extracti128_si256(bs, 1));
            const __m128i prod = _mm_madd_epi16(mins, q8s);
            accm[t] = _mm_fmadd_ps(_mm_set1_ps(dmin), _mm_cvtepi32_ps(prod), accm[t]);
        }
    }
    for (int t = 0; t < T; t++) {
        float a[8], m[4];
        _mm256_storeu_ps(a, acc[t]);
        _mm_storeu_ps(m, accm[t]);
        out[t] = hsum8f(a) + hsum4f(m);
    }
}

/* Q6_K row (blocks of 210 bytes: ql[128], qh[64], i8 scales[16], f16 d). */
static inline __attribute__((always_inline)) AVX2 void q6k_rows_t(const uint8_t* w, int nb,
                                                                 const uint8_t* const* xs, const int T, float* out) {
    const __m256i m4 = _mm256_set1_epi8(0xF), m2 = _mm256_set1_epi8(3), m32s = _mm256_set1_epi8(32);
    __m256 acc[8];
    for (int t = 0; t < T; t++) acc[t] = _mm256_setzero_ps();
    for (int b = 0; b < nb; b++) {
        const uint8_t* blk = w + 210 * b;
        const uint8_t *ql = blk, *qh = blk + 128;
        const int8_t* sc = (const int8_t*)(blk + 192);
        const float xd = f16f(blk + 208);
        __m256i sumi[8];
        for (int t = 0; t < T; t++) sumi[t] = _mm256_setzero_si256();
        for (int j = 0; j < 2; j++) {
            const __m256i b1 = _mm256_loadu_si256((const __m256i*)(ql + 64 * j));
            const __m256i b2 = _mm256_loadu_si256((const __m256i*)(ql + 64 * j + 32));
            const __m256i bh = _mm256_loadu_si256((const __m256i*)(qh + 32 * j));
            __m256i q[4];
            q[0] = _mm256_or_si256(_mm256_and_si256(b1, m4), _mm256_slli_epi16(_mm256_and_si256(bh, m2), 4));
            q[1] = _mm256_or_si256(_mm256_and_si256(b2, m4),
                                   _mm256_slli_epi16(_mm256_and_si256(_mm256_srli_epi16(bh, 2), m2), 4));
            q[2] = _mm256_or_si256(_mm256_and_si256(_mm256_srli_epi16(b1, 4), m4),
                                   _mm256_slli_epi16(_mm256_and_si256(_mm256_srli_epi16(bh, 4), m2), 4));
            q[3] = _mm256_or_si256(_mm256_and_si256(_mm256_srli_epi16(b2, 4), m4),
                                   _mm256_slli_epi16(_mm256_and_si256(_mm256_srli_epi16(bh, 6), m2), 4));
            __m256i s[4];
            for (int x = 0; x < 4; x++)
                s[x] = _mm256_set_m128i(_mm_set1_epi16(sc[2 * (4 * j + x) + 1]), _mm_set1_epi16(sc[2 * (4 * j + x)]));
            for (int t = 0; t < T; t++) {
                const uint8_t* yq = xs[t] + 292 * b + 4 + 128 * j;
                __m256i part = _mm256_setzero_si256();
                for (int x = 0; x < 4; x++) {
                    const __m256i y = _mm256_loadu_si256((const __m256i*)(yq + 32 * x));
                    const __m256i p = _mm256_sub_epi16(_mm256_maddubs_epi16(q[x], y), _mm256_maddubs_epi16(m32s, y));
                    part = _mm256_add_epi32(part, _mm256_madd_epi16(s[x], p));
                }
                sumi[t] = _mm256_add_epi32(sumi[t], part);
            }
        }
        for (int t = 0; t < T; t++) {
            float yd;
            memcpy(&yd, xs[t] + 292 * b, 4);
            acc[t] = _mm256_fmadd_ps(_mm256_set1_ps(yd * xd), _mm256_cvtepi32_ps(sumi[t]), acc[t]);
        }
    }
    for (int t = 0; t < T; t++) {
        float a[8];
        _mm256_storeu_ps(a, acc[t]);
        out[t] = hsum8f(a);
    }
}

/* Q8_0 row against Q8_0 input rows (blocks of 34 bytes: f16 d, i8 qs[32]);
 * lane n = sum of the products of elements 4n..4n+3, exact in i32. */
static inline __attribute__((always_inline)) AVX2 void q80_rows_t(const uint8_t* w, int nb,
                                                                 const uint8_t* const* xs, const int T, float* out) {
    const __m256i perm = _mm256_setr_epi32(0, 1, 4, 5, 2, 3, 6, 7);
    __m256 acc[8];
    for (int t = 0; t < T; t++) acc[t] = _mm256_setzero_ps();
    for (int b = 0; b < nb; b++) {
        const uint8_t* blk = w + 34 * b;
        const float xd = f16f(blk);
        const __m128i wv0 = _mm_loadu_si128((const __m128i*)(blk + 2));
        const __m128i wv1 = _mm_loadu_si128((const __m128i*)(blk + 18));
        const __m256i w0 = _mm256_cvtepi8_epi16(wv0), w1 = _mm256_cvtepi8_epi16(wv1);
        for (int t = 0; t < T; t++) {
            const uint8_t* yb = xs[t] + 34 * b;
            const __m256i y0 = _mm256_cvtepi8_epi16(_mm_loadu_si128((const __m128i*)(yb + 2)));
            const __m256i y1 = _mm256_cvtepi8_epi16(_mm_loadu_si128((const __m128i*)(yb + 18)));
            const __m256i h = _mm256_hadd_epi32(_mm256_madd_epi16(w0, y0), _mm256_madd_epi16(w1, y1));
            const __m256i lanes = _mm256_permutevar8x32_epi32(h, perm);
            acc[t] = _mm256_fmadd_ps(_mm256_set1_ps(xd * f16f(yb)), _mm256_cvtepi32_ps(lanes), acc[t]);
        }
    }
    for (int t = 0; t < T; t++) {
        float a[8];
        _mm256_storeu_ps(a, acc[t]);
        out[t] = hsum8f(a);
    }
}

/* Q5_K row (blocks of 176 bytes: f16 d, f16 dmin, scales[12], qh[32],
 * qs[128]) against T <= 8 Q8_K input rows: per block the exact integers
 * isum = sum_s sc[s] (q_s . y_s) and msum = sum_s mn[s] (bsum_{2s} +
 * bsum_{2s+1}), then acc = fma(y.d d, isum, acc), accm = fma(y.d dmin,
 * msum, accm), result acc - accm: bitwise the scalar form (ref_q5k, one
 * chunk of the block order). */
static inline __attribute__((always_inline)) AVX2 void q5k_rows_t(const uint8_t* w, int nb,
                                                                 const uint8_t* const* xs, const int T, float* out) {
    const __m256i m4 = _mm256_set1_epi8(0xF), m1 = _mm256_set1_epi8(1), ones = _mm256_set1_epi16(1);
    float acc[8], accm[8];
    for (int t = 0; t < T; t++) { acc[t] = 0.f; accm[t] = 0.f; }
    for (int b = 0; b < nb; b++) {
        const uint8_t* blk = w + 176 * b;
        uint8_t sc[8], mn[8];
        scales_mins(blk + 4, sc, mn);
        const float xd = f16f(blk), xdmin = f16f(blk + 2);
        const __m256i qh = _mm256_loadu_si256((const __m256i*)(blk + 16));
        __m256i q[8];  /* the 5-bit weights of sub-block s as bytes */
        for (int j = 0; j < 4; j++) {
            const __m256i q4 = _mm256_loadu_si256((const __m256i*)(blk + 48 + 32 * j));
            const __m256i lo = _mm256_and_si256(q4, m4), hi = _mm256_and_si256(_mm256_srli_epi16(q4, 4), m4);
            const __m256i hb0 = _mm256_and_si256(_mm256_srli_epi16(qh, 2 * j), m1);
            const __m256i hb1 = _mm256_and_si256(_mm256_srli_epi16(qh, 2 * j + 1), m1);
            q[2 * j] = _mm256_or_si256(lo, _mm256_slli_epi16(hb0, 4));
            q[2 * j + 1] = _mm256_or_si256(hi, _mm256_slli_epi16(hb1, 4));
        }
        for (int t = 0; t < T; t++) {
            const uint8_t* y = xs[t] + 292 * b;
            __m256i isv = _mm256_setzero_si256();
            for (int s = 0; s < 8; s++) {
                const __m256i yv = _mm256_loadu_si256((const __m256i*)(y + 4 + 32 * s));
                const __m256i p = _mm256_madd_epi16(_mm256_maddubs_epi16(q[s], yv), ones);
                isv = _mm256_add_epi32(isv, _mm256_mullo_epi32(p, _mm256_set1_epi32(sc[s])));
            }
            int32_t lanes[8];
            _mm256_storeu_si256((__m256i*)lanes, isv);
            int32_t isum = 0;
            for (int i = 0; i < 8; i++) isum += lanes[i];
            int16_t bs[16];
            memcpy(bs, y + 260, 32);
            int32_t msum = 0;
            for (int s2 = 0; s2 < 8; s2++) msum += mn[s2] * (bs[2 * s2] + bs[2 * s2 + 1]);
            float yd;
            memcpy(&yd, y, 4);
            acc[t] = fmaf(yd * xd, (float)isum, acc[t]);
            accm[t] = fmaf(yd * xdmin, (float)msum, accm[t]);
        }
    }
    for (int t = 0; t < T; t++) out[t] = acc[t] - accm[t];
}

/* Exported forms: T (the input rows, 1..8) made a constant per instance, so
 * the per-row accumulators stay in registers (same operations, same order). */
#define IQ_ROWS_DISPATCH(name)                                                                 \
    AVX2 void or_##name##_rows_avx2(const uint8_t* w, int nb, const uint8_t* const* xs, int T, float* out) { \
        switch (T) {                                                                           \
            case 1: name##_rows_t(w, nb, xs, 1, out); break;                                   \
            case 2: name##_rows_t(w, nb, xs, 2, out); break;                                   \
            case 3: name##_rows_t(w, nb, xs, 3, out); break;                                   \
            case 4: name##_rows_t(w, nb, xs, 4, out); break;                                   \
            case 5: name##_rows_t(w, nb, xs, 5, out); break;                                   \
            case 6: name##_rows_t(w, nb, xs, 6, out); break;                                   \
            case 7: name##_rows_t(w, nb, xs, 7, out); break;                                   \
            default: name##_rows_t(w, nb, xs, 8, out); break;                                  \
        }                                                                                      \
    }
IQ_ROWS_DISPATCH(q4k)
IQ_ROWS_DISPATCH(q6k)
IQ_ROWS_DISPATCH(q80)
IQ_ROWS_DISPATCH(q5k)

/* The attention scan's two inner loops (quantized_attention.rs:155-178 and
 * the value sum after it) eight lanes at a time, bitwise the scalar forms:
 * dot8 keeps its eight lane partials as one vector (products and sums
 * rounded separately, as the scalar build does), and the value sum is an
 * independent sequential sum per output element d, so eight d run side by
 * side in the same position order. */
AVX2 float or_dot8_avx2(const float* a, const float* b, int n) {
    __m256 acc = _mm256_setzero_ps();
    const int full = n / 8 * 8;
    for (int i = 0; i < full; i += 8)
        acc = _mm256_add_ps(acc, _mm256_mul_ps(_mm256_loadu_ps(a + i), _mm256_loadu_ps(b + i)));
    float lanes[8];
    _mm256_storeu_ps(lanes, acc);
    float total = 0.f;
    for (int i = full; i < n; i++) total += a[i] * b[i];
    for (int l = 0; l < 8; l++) total += lanes[l];
    return total;
}

/* o[d] (zeroed by the caller) += (scores[p] / den) * v[p * stride + d] for p
 * in order; scores is overwritten with the probabilities.  One pass over the
 * value rows, o staying in L1. */
AVX2 void or_attend_values_avx2(float* o, float* scores, float den, const float* v, int64_t positions,
                                int64_t stride, int hd) {
    for (int64_t p = 0; p < positions; p++) scores[p] = scores[p] / den;
    const int full = hd / 8 * 8;
    for (int64_t p = 0; p < positions; p++) {
        const __m256 pb = _mm256_set1_ps(scores[p]);
        const float* row = v + p * stride;
        for (int d = 0; d < full; d += 8)
            _mm256_storeu_ps(o + d, _mm256_add_ps(_mm256_loadu_ps(o + d), _mm256_mul_ps(pb, _mm256_loadu_ps(row + d))));
        for (int d = full; d < hd; d++) o[d] += scores[p] * row[d];
    }
}
