/*
 * iq_oracle_quant.c -- block formats, activation quantization and the
 * quantized matrix-vector product, restated on the CPU.
 *
 * TEST INFRASTRUCTURE ONLY (see iq_oracle.h).  Build with -ffp-contract=off:
 * every multiply-add below that is not an explicit fmaf() must round twice,
 * as the reference's Rust does.
 */
#include "iq_oracle.h"
#include <math.h>
#include <string.h>
#include <stdlib.h>

int64_t or_row_bytes(int dtype, int64_t cols) {
    switch (dtype) {
    case OR_F32: return cols * 4;
    case OR_F16: return cols * 2;
    case OR_Q8_0: return cols / 32 * 34;
    case OR_Q4_K: return cols / 256 * 144;
    case OR_Q5_K: return cols / 256 * 176;
    case OR_Q6_K: return cols / 256 * 210;
    case OR_Q8_K: return cols / 256 * 292;
    default: return -1;
    }
}

float or_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h >> 15) << 31;
    uint32_t exp = (h >> 10) & 0x1f, man = h & 0x3ff, bits;
    if (exp == 0) {
        if (man == 0) bits = sign;
        else { /* subnormal: value = man * 2^-24 */
            float f = (float)man * 5.9604644775390625e-08f;
            memcpy(&bits, &f, 4);
            bits |= sign;
        }
    } else if (exp == 31) bits = sign | 0x7f800000u | (man << 13);
    else bits = sign | ((exp + 112) << 23) | (man << 13);
    float out; memcpy(&out, &bits, 4); return out;
}

uint16_t or_f32_to_f16(float f) {
    uint32_t x; memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000;
    uint32_t ax = x & 0x7fffffff;
    if (ax >= 0x7f800000) return (uint16_t)(sign | 0x7c00 | (ax > 0x7f800000 ? 0x200 : 0));
    if (ax >= 0x477ff000) return (uint16_t)(sign | 0x7c00); /* overflow rounds to inf */
    if (ax < 0x38800000) { /* subnormal or zero in f16 */
        float a; memcpy(&a, &ax, 4);
        float s = a * 16777216.0f; /* exact scaling by 2^24 */
        /* round to nearest even integer */
        float r = rintf(s);
        return (uint16_t)(sign | (uint32_t)r);
    }
    uint32_t man = ax & 0x7fffff, e = (ax >> 23) - 112;
    uint32_t h = (e << 10) | (man >> 13);
    uint32_t rem = man & 0x1fff;
    if (rem > 0x1000 || (rem == 0x1000 && (h & 1))) h++;
    return (uint16_t)(sign | h);
}

static inline uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }

/* Twelve packed bytes -> eight 6-bit scales and eight 6-bit mins, the
 * sequence src/qgemm.rs:153-167 (unpack_k_scales) reproduces. */
static void unpack_k_scales(const uint8_t* s, uint8_t sc[8], uint8_t mn[8]) {
    for (int j = 0; j < 4; j++) {
        sc[j] = s[j] & 63;
        mn[j] = s[j + 4] & 63;
        sc[j + 4] = (s[j + 8] & 0xf) | ((s[j] >> 6) << 4);
        mn[j + 4] = (s[j + 8] >> 4) | ((s[j + 4] >> 6) << 4);
    }
}

/* ---------------------------------------------------------------- decode */

static void deq_q4k(const uint8_t* b, float* y) {
    float d = or_f16_to_f32(rd16(b)), dmin = or_f16_to_f32(rd16(b + 2));
    uint8_t sc[8], mn[8];
    unpack_k_scales(b + 4, sc, mn);
    const uint8_t* qs = b + 16;
    for (int j = 0; j < 4; j++) {
        float d1 = d * (float)sc[2 * j], m1 = dmin * (float)mn[2 * j];
        float d2 = d * (float)sc[2 * j + 1], m2 = dmin * (float)mn[2 * j + 1];
        for (int i = 0; i < 32; i++) y[64 * j + i] = d1 * (float)(qs[32 * j + i] & 0xf) - m1;
        for (int i = 0; i < 32; i++) y[64 * j + 32 + i] = d2 * (float)(qs[32 * j + i] >> 4) - m2;
    }
}

static void deq_q5k(const uint8_t* b, float* y) {
    float d = or_f16_to_f32(rd16(b)), dmin = or_f16_to_f32(rd16(b + 2));
    uint8_t sc[8], mn[8];
    unpack_k_scales(b + 4, sc, mn);
    const uint8_t* qh = b + 16;
    const uint8_t* qs = b + 48;
    for (int j = 0; j < 4; j++) {
        float d1 = d * (float)sc[2 * j], m1 = dmin * (float)mn[2 * j];
        float d2 = d * (float)sc[2 * j + 1], m2 = dmin * (float)mn[2 * j + 1];
        for (int i = 0; i < 32; i++) {
            int lo = (qs[32 * j + i] & 0xf) | (((qh[i] >> (2 * j)) & 1) << 4);
            int hi = (qs[32 * j + i] >> 4) | (((qh[i] >> (2 * j + 1)) & 1) << 4);
            y[64 * j + i] = d1 * (float)lo - m1;
            y[64 * j + 32 + i] = d2 * (float)hi - m2;
        }
    }
}

/* Q6_K element e: ql nibble, two bits of qh, minus 32, times d*scale[e/16]. */
static inline int q6k_value(const uint8_t* ql, const uint8_t* qh, int e) {
    int half = e / 128, l = e % 128;
    int nib = (l < 64) ? (ql[half * 64 + l] & 0xf) : (ql[half * 64 + l - 64] >> 4);
    int hb = (qh[half * 32 + (l % 32)] >> (2 * (l / 32))) & 3;
    return (nib | (hb << 4)) - 32;
}

static void deq_q6k(const uint8_t* b, float* y) {
    const uint8_t* ql = b;
    const uint8_t* qh = b + 128;
    const int8_t* sc = (const int8_t*)(b + 192);
    float d = or_f16_to_f32(rd16(b + 208));
    for (int e = 0; e < 256; e++) y[e] = (d * (float)sc[e / 16]) * (float)q6k_value(ql, qh, e);
}

static void deq_q80(const uint8_t* b, float* y) {
    float d = or_f16_to_f32(rd16(b));
    const int8_t* q = (const int8_t*)(b + 2);
    for (int i = 0; i < 32; i++) y[i] = (float)q[i] * d;
}

int or_dequant_rows(int dtype, const void* w, int64_t rows, int64_t cols, float* out) {
    const uint8_t* p = (const uint8_t*)w;
    int64_t n = rows * cols;
    switch (dtype) {
    case OR_F32: memcpy(out, w, (size_t)n * 4); return 0;
    case OR_F16: for (int64_t i = 0; i < n; i++) out[i] = or_f16_to_f32(rd16(p + 2 * i)); return 0;
    case OR_BF16:  /* exact widening: the bf16 bits are the top half of the f32 */
        for (int64_t i = 0; i < n; i++) { uint32_t u = (uint32_t)rd16(p + 2 * i) << 16; memcpy(out + i, &u, 4); }
        return 0;
    case OR_Q4_K: for (int64_t i = 0; i < n / 256; i++) deq_q4k(p + 144 * i, out + 256 * i); return 0;
    case OR_Q5_K: for (int64_t i = 0; i < n / 256; i++) deq_q5k(p + 176 * i, out + 256 * i); return 0;
    case OR_Q6_K: for (int64_t i = 0; i < n / 256; i++) deq_q6k(p + 210 * i, out + 256 * i); return 0;
    case OR_Q8_0: for (int64_t i = 0; i < n / 32; i++) deq_q80(p + 34 * i, out + 32 * i); return 0;
    default: return -1;
    }
}

/* ------------------------------------------------- activation quantizers */

/* candle-core 0.11 k_quants BlockQ8K::from_float (call site src/gguf.rs:650):
 * the signed value of largest magnitude (first one on ties) sets
 * iscale = -128/max; q = round-half-away(iscale*x) capped at 127;
 * d = 1/iscale; bsums are the 16-element sums of q. */
void or_quant_q8k(const float* x, int64_t cols, void* blocks) {
    uint8_t* out = (uint8_t*)blocks;
    for (int64_t b = 0; b < cols / 256; b++) {
        const float* xs = x + 256 * b;
        uint8_t* blk = out + 292 * b;
        float max = 0.f, amax = 0.f;
        for (int i = 0; i < 256; i++) {
            float a = fabsf(xs[i]);
            if (amax < a) { amax = a; max = xs[i]; }
        }
        int8_t qs[256];
        int16_t bs[16];
        float d;
        if (amax == 0.f) {
            d = 0.f;
            memset(qs, 0, sizeof qs);
        } else {
            float iscale = -128.f / max;
            for (int i = 0; i < 256; i++) {
                float v = roundf(iscale * xs[i]);
                qs[i] = (int8_t)(v < 127.f ? v : 127.f);
            }
            d = 1.f / iscale;
        }
        for (int j = 0; j < 16; j++) {
            int s = 0;
            for (int i = 0; i < 16; i++) s += qs[16 * j + i];
            bs[j] = (int16_t)s;
        }
        memcpy(blk, &d, 4);
        memcpy(blk + 4, qs, 256);
        memcpy(blk + 260, bs, 32);
    }
}

/* candle-core 0.11 BlockQ8_0::from_float: d = amax/127 stored as f16,
 * q = round-half-away(x * (1/d)) with the f32 d, not the f16 one. */
void or_quant_q80(const float* x, int64_t cols, void* blocks) {
    uint8_t* out = (uint8_t*)blocks;
    for (int64_t b = 0; b < cols / 32; b++) {
        const float* xs = x + 32 * b;
        float amax = 0.f;
        for (int i = 0; i < 32; i++) amax = fmaxf(amax, fabsf(xs[i]));
        float d = amax / 127.f;
        float id = d != 0.f ? 1.f / d : 0.f;
        uint16_t dh = or_f32_to_f16(d);
        uint8_t* blk = out + 34 * b;
        blk[0] = dh & 0xff; blk[1] = dh >> 8;
        for (int i = 0; i < 32; i++) blk[2 + i] = (uint8_t)(int8_t)roundf(xs[i] * id);
    }
}

int64_t or_argmax(const float* v, int64_t n) {
    int64_t best = -1;
    for (int64_t i = 0; i < n; i++) {
        if (!isfinite(v[i])) continue;
        if (best < 0 || v[i] >= v[best]) best = i;
    }
    return best;
}
