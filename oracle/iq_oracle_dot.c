/*
 * iq_oracle_dot.c -- the quantized matrix-vector product in two f32 orders.
 *
 * TEST INFRASTRUCTURE ONLY (see iq_oracle.h).  Built with -ffp-contract=off.
 *
 * Integer block sums are identical in both orders (and to the reference):
 *   Q4_K/Q5_K  isum = sum_s sc[s] * sum_{e in s} q_e * x_e,
 *              msum = sum_s mn[s] * (bsums[2s] + bsums[2s+1])
 *   Q6_K       isum = sum_s sc[s] * sum_{e in s} (q_e - 32) * x_e  (16-wide s)
 *   Q8_0       isum = sum_e q_e * x_e
 * Only how the per-block f32 terms are accumulated differs.
 */
#include "iq_oracle.h"
#include <math.h>
#include <string.h>
#include <stdlib.h>

static inline uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }

static void unpack_k_scales(const uint8_t* s, uint8_t sc[8], uint8_t mn[8]) {
    for (int j = 0; j < 4; j++) {
        sc[j] = s[j] & 63;
        mn[j] = s[j + 4] & 63;
        sc[j + 4] = (s[j + 8] & 0xf) | ((s[j] >> 6) << 4);
        mn[j + 4] = (s[j + 8] >> 4) | ((s[j + 4] >> 6) << 4);
    }
}

typedef struct { float d; int8_t qs[256]; int16_t bs[16]; } q8k_t;  /* unpacked view */

static void load_q8k(const uint8_t* p, q8k_t* b) {
    memcpy(&b->d, p, 4);
    memcpy(b->qs, p + 4, 256);
    memcpy(b->bs, p + 260, 32);
}

/* Register-only horizontal sums of src/qgemm.rs:127-145. */
static inline float hsum8(const float a[8]) {
    float r0 = a[4] + a[0], r1 = a[5] + a[1], r2 = a[6] + a[2], r3 = a[7] + a[3];
    return (r0 + r2) + (r1 + r3);
}
static inline float hsum4(const float a[4]) { return (a[0] + a[2]) + (a[1] + a[3]); }

/* q of element e of a Q4_K block (0..15) and of a Q5_K block (0..31). */
static inline int q4k_q(const uint8_t* qs, int e) {
    int j = e / 64, i = e % 64;
    return i < 32 ? (qs[32 * j + i] & 0xf) : (qs[32 * j + i - 32] >> 4);
}
static inline int q5k_q(const uint8_t* qh, const uint8_t* qs, int e) {
    int s = e / 32, i = e % 32;
    return q4k_q(qs, e) | (((qh[i] >> s) & 1) << 4);
}
static inline int q6k_q(const uint8_t* ql, const uint8_t* qh, int e) {
    int half = e / 128, l = e % 128;
    int nib = (l < 64) ? (ql[half * 64 + l] & 0xf) : (ql[half * 64 + l - 64] >> 4);
    int hb = (qh[half * 32 + (l % 32)] >> (2 * (l / 32))) & 3;
    return (nib | (hb << 4)) - 32;
}

/* ---- reference order: src/qgemm.rs q4k_tile (:175-245), lane n of the
 * 256-bit accumulators covers bytes 4n..4n+3 of every 32-byte chunk. */
static float ref_q4k(const uint8_t* w, const uint8_t* xq, int nb) {
    float acc[8] = {0}, accm[4] = {0};
    for (int b = 0; b < nb; b++) {
        const uint8_t* blk = w + 144 * b;
        q8k_t y; load_q8k(xq + 292 * b, &y);
        uint8_t sc[8], mn[8]; unpack_k_scales(blk + 4, sc, mn);
        const uint8_t* qs = blk + 16;
        float xd = or_f16_to_f32(rd16(blk)), xdmin = or_f16_to_f32(rd16(blk + 2));
        int32_t sumi[8] = {0};
        for (int j = 0; j < 4; j++)
            for (int n = 0; n < 8; n++)
                for (int e = 0; e < 4; e++) {
                    int byte = 32 * j + 4 * n + e;
                    sumi[n] += sc[2 * j] * (qs[byte] & 0xf) * y.qs[64 * j + 4 * n + e]
                             + sc[2 * j + 1] * (qs[byte] >> 4) * y.qs[64 * j + 32 + 4 * n + e];
                }
        float d = y.d * xd, dmin = -y.d * xdmin;
        for (int n = 0; n < 8; n++) acc[n] = fmaf(d, (float)sumi[n], acc[n]);
        int16_t q8s[8];
        for (int i = 0; i < 8; i++) q8s[i] = (int16_t)(y.bs[2 * i] + y.bs[2 * i + 1]);
        for (int i = 0; i < 4; i++) {
            int32_t prod = mn[2 * i] * q8s[2 * i] + mn[2 * i + 1] * q8s[2 * i + 1];
            accm[i] = fmaf(dmin, (float)prod, accm[i]);
        }
    }
    return hsum8(acc) + hsum4(accm);
}

/* src/qgemm.rs q6k_tile (:249-346): lane n, chunk x of half j uses scale
 * 2*(4j+x) for n<4 and 2*(4j+x)+1 for n>=4. */
static float ref_q6k(const uint8_t* w, const uint8_t* xq, int nb) {
    float acc[8] = {0};
    for (int b = 0; b < nb; b++) {
        const uint8_t* blk = w + 210 * b;
        q8k_t y; load_q8k(xq + 292 * b, &y);
        const uint8_t *ql = blk, *qh = blk + 128;
        const int8_t* sc = (const int8_t*)(blk + 192);
        float xd = or_f16_to_f32(rd16(blk + 208));
        int32_t sumi[8] = {0};
        for (int j = 0; j < 2; j++)
            for (int x = 0; x < 4; x++)
                for (int n = 0; n < 8; n++) {
                    int scale = sc[2 * (4 * j + x) + (n >= 4)];
                    int32_t part = 0;
                    for (int e = 0; e < 4; e++) {
                        int el = 128 * j + 32 * x + 4 * n + e;
                        part += q6k_q(ql, qh, el) * y.qs[el];
                    }
                    sumi[n] += scale * part;
                }
        float d = y.d * xd;
        for (int n = 0; n < 8; n++) acc[n] = fmaf(d, (float)sumi[n], acc[n]);
    }
    return hsum8(acc);
}

/* src/qgemm.rs q80_tile (:369-397). */
static float ref_q80(const uint8_t* w, const uint8_t* xq, int nb) {
    float acc[8] = {0};
    for (int b = 0; b < nb; b++) {
        const uint8_t* blk = w + 34 * b;
        const uint8_t* yb = xq + 34 * b;
        const int8_t* wq = (const int8_t*)(blk + 2);
        const int8_t* yq = (const int8_t*)(yb + 2);
        float xd = or_f16_to_f32(rd16(blk));
        float d = xd * or_f16_to_f32(rd16(yb));
        for (int n = 0; n < 8; n++) {
            int32_t dot = 0;
            for (int e = 0; e < 4; e++) dot += wq[4 * n + e] * yq[4 * n + e];
            acc[n] = fmaf(d, (float)dot, acc[n]);
        }
    }
    return hsum8(acc);
}

/* Q5_K has no fused reference kernel (src/gguf.rs:594-596 keeps it on
 * candle's per-row vec_dot, whose source is not in the reference tree).
 * The reference order is therefore unpinned; it is restated here as the
 * plain per-block form: one f32 FMA per block, mins separately. */
static float dev_block_chunks(int dtype, const uint8_t* w, const uint8_t* xq, int nb, int ksplit);

static float ref_q5k(const uint8_t* w, const uint8_t* xq, int nb) {
    return dev_block_chunks(OR_Q5_K, w, xq, nb, 1);
}

/* ---- device order: per block exact integer sums, one FMA per block per
 * chunk, chunk partials added left to right. */
static void block_terms(int dtype, const uint8_t* blk, const uint8_t* xq, int b,
                        float* t_scale, float* t_int, float* m_scale, float* m_int) {
    *m_scale = 0.f; *m_int = 0.f;
    if (dtype == OR_Q4_K || dtype == OR_Q5_K) {
        q8k_t y; load_q8k(xq + 292 * b, &y);
        uint8_t sc[8], mn[8]; unpack_k_scales(blk + 4, sc, mn);
        const uint8_t* qs = blk + (dtype == OR_Q4_K ? 16 : 48);
        const uint8_t* qh = blk + 16;
        int32_t isum = 0, msum = 0;
        for (int s = 0; s < 8; s++) {
            int32_t p = 0;
            for (int i = 0; i < 32; i++) {
                int e = 32 * s + i;
                int q = dtype == OR_Q4_K ? q4k_q(qs, e) : q5k_q(qh, qs, e);
                p += q * y.qs[e];
            }
            isum += sc[s] * p;
            msum += mn[s] * (y.bs[2 * s] + y.bs[2 * s + 1]);
        }
        float xd = or_f16_to_f32(rd16(blk)), xdmin = or_f16_to_f32(rd16(blk + 2));
        *t_scale = y.d * xd; *t_int = (float)isum;
        *m_scale = y.d * xdmin; *m_int = (float)msum;
    } else if (dtype == OR_Q6_K) {
        q8k_t y; load_q8k(xq + 292 * b, &y);
        const uint8_t *ql = blk, *qh = blk + 128;
        const int8_t* sc = (const int8_t*)(blk + 192);
        int32_t isum = 0;
        for (int s = 0; s < 16; s++) {
            int32_t p = 0;
            for (int i = 0; i < 16; i++) p += q6k_q(ql, qh, 16 * s + i) * y.qs[16 * s + i];
            isum += sc[s] * p;
        }
        *t_scale = y.d * or_f16_to_f32(rd16(blk + 208)); *t_int = (float)isum;
    } else { /* Q8_0 */
        const uint8_t* yb = xq + 34 * b;
        const int8_t* wq = (const int8_t*)(blk + 2);
        const int8_t* yq = (const int8_t*)(yb + 2);
        int32_t isum = 0;
        for (int e = 0; e < 32; e++) isum += wq[e] * yq[e];
        *t_scale = or_f16_to_f32(rd16(blk)) * or_f16_to_f32(rd16(yb)); *t_int = (float)isum;
    }
}

/* The AVX2 forms (iq_oracle_avx2.c) and a switch to the scalar ones. */
int or_have_avx2(void);
void or_q4k_rows_avx2(const uint8_t* w, int nb, const uint8_t* const* xs, int T, float* out);
void or_q6k_rows_avx2(const uint8_t* w, int nb, const uint8_t* const* xs, int T, float* out);
void or_q80_rows_avx2(const uint8_t* w, int nb, const uint8_t* const* xs, int T, float* out);
void or_q5k_rows_avx2(const uint8_t* w, int nb, const uint8_t* const* xs, int T, float* out);
static int g_force_scalar = 0;
void or_force_scalar(int on) { g_force_scalar = on; }
int or_scalar_forced(void) { return g_force_scalar; }

static int block_bytes(int dtype) {
    return dtype == OR_Q4_K ? 144 : dtype == OR_Q5_K ? 176 : dtype == OR_Q6_K ? 210 : 34;
}

/* ksplit chunks of whole "units" (one 256-block, or four Q8_0 blocks). */
static float dev_block_chunks(int dtype, const uint8_t* w, const uint8_t* xq, int nb, int ksplit) {
    int per_unit = dtype == OR_Q8_0 ? 4 : 1;
    int units = nb / per_unit;
    float y = 0.f;
    for (int c = 0; c < ksplit; c++) {
        int u0 = c * units / ksplit, u1 = (c + 1) * units / ksplit;
        float acc = 0.f, accm = 0.f;
        for (int b = u0 * per_unit; b < u1 * per_unit; b++) {
            float ts, ti, ms, mi;
            block_terms(dtype, w + (int64_t)block_bytes(dtype) * b, xq, b, &ts, &ti, &ms, &mi);
            acc = fmaf(ts, ti, acc);
            if (dtype == OR_Q4_K || dtype == OR_Q5_K) accm = fmaf(ms, mi, accm);
        }
        float part = (dtype == OR_Q4_K || dtype == OR_Q5_K) ? acc - accm : acc;
        y = c == 0 ? part : y + part;
    }
    return y;
}

int or_qmatvec(int dtype, const void* wv, int64_t rows, int64_t cols,
               const float* x, int k, float* y, int order, int ksplit) {
    const uint8_t* w = (const uint8_t*)wv;
    if (dtype == OR_F32) { /* plain serial f32 dot (candle's f32 matmul order is unpinned) */
        const float* wf = (const float*)wv;
        #pragma omp parallel for schedule(static)
        for (int64_t r = 0; r < rows; r++)
            for (int i = 0; i < k; i++) {
                float s = 0.f;
                for (int64_t c = 0; c < cols; c++) s += wf[r * cols + c] * x[i * cols + c];
                y[i * rows + r] = s;
            }
        return 0;
    }
    if (dtype == OR_BF16) {
        /* QuantizedMatrix of BF16 (src/gguf.rs:305-316) runs candle's matmul
         * with bf16 as the vec-dot type: input rows rounded to bf16 (round to
         * nearest even), exact products summed in f32 (candle-core 0.11.0,
         * unvendored; its summation order is unpinned: serial here) */
        const uint16_t* wb = (const uint16_t*)wv;
        float* xb = (float*)malloc((size_t)(k * cols) * 4);
        for (int64_t i = 0; i < k * cols; i++) {
            uint32_t u;
            memcpy(&u, x + i, 4);
            u = (u + 0x7FFFu + ((u >> 16) & 1u)) & 0xFFFF0000u;  /* RNE to bf16 (finite inputs) */
            memcpy(xb + i, &u, 4);
        }
        #pragma omp parallel for schedule(static)
        for (int64_t r = 0; r < rows; r++)
            for (int i = 0; i < k; i++) {
                float s = 0.f;
                for (int64_t c = 0; c < cols; c++) {
                    uint32_t u = (uint32_t)wb[r * cols + c] << 16;
                    float w;
                    memcpy(&w, &u, 4);
                    s += w * xb[i * cols + c];
                }
                y[i * rows + r] = s;
            }
        free(xb);
        return 0;
    }
    int is_k = dtype == OR_Q4_K || dtype == OR_Q5_K || dtype == OR_Q6_K;
    if (!is_k && dtype != OR_Q8_0) return -1;
    int blk = is_k ? 256 : 32;
    if (cols % blk) return -2;
    int nb = (int)(cols / blk);
    int64_t xbytes = is_k ? (int64_t)nb * 292 : (int64_t)nb * 34;
    uint8_t* xq = (uint8_t*)malloc((size_t)(xbytes * k));
    for (int i = 0; i < k; i++) {
        if (is_k) or_quant_q8k(x + i * cols, cols, xq + i * xbytes);
        else or_quant_q80(x + i * cols, cols, xq + i * xbytes);
    }
    int64_t rb = or_row_bytes(dtype, cols);
    if (ksplit < 1) ksplit = 1;
    /* the AVX2 forms of the reference order: a weight row decoded once for
     * up to eight input rows (bitwise the scalar forms below) */
    static int avx2 = -1;
    if (avx2 < 0) avx2 = or_have_avx2();
    if (order == 0 && avx2 && !g_force_scalar &&
        (dtype == OR_Q4_K || dtype == OR_Q5_K || dtype == OR_Q6_K || dtype == OR_Q8_0)) {
        #pragma omp parallel for schedule(static)
        for (int64_t r = 0; r < rows; r++) {
            const uint8_t* wr = w + r * rb;
            for (int i0 = 0; i0 < k; i0 += 8) {
                const uint8_t* xs[8];
                float o[8];
                int T = k - i0 < 8 ? k - i0 : 8;
                for (int t = 0; t < T; t++) xs[t] = xq + (i0 + t) * xbytes;
                if (dtype == OR_Q4_K) or_q4k_rows_avx2(wr, nb, xs, T, o);
                else if (dtype == OR_Q6_K) or_q6k_rows_avx2(wr, nb, xs, T, o);
                else if (dtype == OR_Q5_K) or_q5k_rows_avx2(wr, nb, xs, T, o);
                else or_q80_rows_avx2(wr, nb, xs, T, o);
                for (int t = 0; t < T; t++) y[(i0 + t) * rows + r] = o[t];
            }
        }
        free(xq);
        return 0;
    }
    #pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; r++) {
        const uint8_t* wr = w + r * rb;
        for (int i = 0; i < k; i++) {
            const uint8_t* xi = xq + i * xbytes;
            float v;
            if (order == 0) {
                v = dtype == OR_Q4_K ? ref_q4k(wr, xi, nb) : dtype == OR_Q6_K ? ref_q6k(wr, xi, nb)
                  : dtype == OR_Q8_0 ? ref_q80(wr, xi, nb) : ref_q5k(wr, xi, nb);
            } else {
                v = dev_block_chunks(dtype, wr, xi, nb, ksplit);
            }
            y[i * rows + r] = v;
        }
    }
    free(xq);
    return 0;
}
