/* kq_oracle.c — CPU restatement of the quantized expert hot path.
 * TEST INFRASTRUCTURE ONLY: the checker for the CUDA plugin, never linked into it.
 * The header lists every reference file:line this follows and what is specified
 * here because the reference checkout has no source for it.
 *
 * Build with -ffp-contract=off: every float operation below is meant to round
 * exactly once, in the order written, so the device kernels can reproduce it.
 */
#include "kq_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------------ */
/* fp16                                                                      */
/* ------------------------------------------------------------------------ */
/* binary16 -> binary32, exact (follows V/include/katali_gguf_fp.h:14-36). */
float kqo_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h >> 15) << 31;
    uint32_t exp = (h >> 10) & 0x1Fu;
    uint32_t mant = h & 0x3FFu;
    uint32_t bits;
    if (exp == 0) {
        if (mant == 0) {
            bits = sign;
        } else {
            int e = -1;
            do { mant <<= 1; e++; } while ((mant & 0x400u) == 0);
            mant &= 0x3FFu;
            bits = sign | ((uint32_t)(127 - 15 - e) << 23) | (mant << 13);
        }
    } else if (exp == 31) {
        bits = sign | 0x7F800000u | (mant << 13);
    } else {
        bits = sign | ((exp - 15u + 127u) << 23) | (mant << 13);
    }
    float out;
    memcpy(&out, &bits, 4);
    return out;
}

/* binary32 -> binary16, IEEE round-to-nearest-even, subnormals included. */
uint16_t kqo_f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t ax = x & 0x7FFFFFFFu;
    if (ax >= 0x7F800000u) /* inf / nan */
        return (uint16_t)(sign | 0x7C00u | (ax > 0x7F800000u ? 0x200u : 0u));
    if (ax >= 0x477FF000u) /* >= 65520 rounds to inf */
        return (uint16_t)(sign | 0x7C00u);
    uint32_t e = ax >> 23;
    if (e < 113) { /* below 2^-14: half subnormal or zero */
        if (e < 102) return (uint16_t)sign;
        uint32_t m = (ax & 0x7FFFFFu) | 0x800000u;
        uint32_t shift = 126u - e; /* 14..24 */
        uint32_t q = m >> shift;
        uint32_t rem = m & ((1u << shift) - 1u);
        uint32_t half = 1u << (shift - 1u);
        if (rem > half || (rem == half && (q & 1u))) q++;
        return (uint16_t)(sign | q);
    }
    uint32_t mant = ax & 0x7FFFFFu;
    uint32_t h = ((e - 112u) << 10) | (mant >> 13);
    uint32_t rem = mant & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
    return (uint16_t)(sign | h);
}

static inline uint16_t ld16(const uint8_t *p) { uint16_t v; memcpy(&v, p, 2); return v; }
static inline void st16(uint8_t *p, uint16_t v) { memcpy(p, &v, 2); }

/* ------------------------------------------------------------------------ */
/* exp / silu                                                                */
/* ------------------------------------------------------------------------ */
/* e^x = 2^n * e^r with n = rint(x*log2 e), r = x - n*ln2 (ln2 split hi/lo,
 * Cody & Waite), and e^r from its Taylor series to degree 7 (|r| <= 0.35, so
 * the truncation error is below 1e-8 relative). Every step is one IEEE
 * operation or fmaf, which the device reproduces exactly. */
float kqo_expf(float x) {
    if (x != x) return x;
    if (x > 88.0f) x = 88.0f;
    if (x < -87.0f) x = -87.0f;
    const float n = rintf(x * 1.44269504088896341f);
    float r = fmaf(-n, 0.693145751953125f, x);
    r = fmaf(-n, 1.42860682030941723e-6f, r);
    float p = 1.98412698412698413e-4f;          /* 1/7! */
    p = fmaf(p, r, 1.38888888888888889e-3f);    /* 1/6! */
    p = fmaf(p, r, 8.33333333333333333e-3f);    /* 1/5! */
    p = fmaf(p, r, 4.16666666666666667e-2f);    /* 1/4! */
    p = fmaf(p, r, 1.66666666666666667e-1f);    /* 1/3! */
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    const uint32_t bits = (uint32_t)((int)n + 127) << 23;
    float s;
    memcpy(&s, &bits, 4);
    return p * s;
}

/* silu(x) = x / (1 + e^-x) (V/src/gguf_kernels.c:323, with kqo_expf). */
float kqo_silu(float x) { return x / (1.0f + kqo_expf(-x)); }

/* ------------------------------------------------------------------------ */
/* block layouts                                                             */
/* ------------------------------------------------------------------------ */
uint64_t kqo_row_bytes(uint32_t type, uint64_t cols) {
    switch (type) {
        case KQO_Q4_K: return cols % 256 ? 0 : cols / 256 * KQO_Q4_K_BYTES;
        case KQO_Q6_K: return cols % 256 ? 0 : cols / 256 * KQO_Q6_K_BYTES;
        case KQO_Q8_1: return cols % 32 ? 0 : cols / 32 * KQO_Q8_1_BYTES;
        default: return 0;
    }
}

/* Q4_K 6-bit sub-scale j and sub-min j from the 12 packed bytes
 * (V/src/gguf_dtype.c:350-358). */
static inline void q4k_scale_min(int j, const uint8_t *q, int *sc, int *m) {
    if (j < 4) {
        *sc = q[j] & 63;
        *m = q[j + 4] & 63;
    } else {
        *sc = (q[j + 4] & 0x0F) | ((q[j - 4] >> 6) << 4);
        *m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
    }
}

/* 4-bit value i (0..31) of 32-element group j (0..7) of a Q4_K block. */
static inline int q4k_q(const uint8_t *qs, int j, int i) {
    const uint8_t b = qs[(j >> 1) * 32 + i];
    return (j & 1) ? (b >> 4) : (b & 0x0F);
}

/* 6-bit value (0..63) of element e (0..255) of a Q6_K block
 * (layout of V/src/gguf_dtype.c:487-512). */
static inline int q6k_q(const uint8_t *blk, int e) {
    const int h = e >> 7, quarter = (e >> 5) & 3, l = e & 31;
    const uint8_t ql = blk[64 * h + 32 * (quarter & 1) + l];
    const uint8_t qh = blk[128 + 32 * h + l];
    const int lo = (quarter >= 2) ? (ql >> 4) : (ql & 0x0F);
    return lo | (((qh >> (2 * quarter)) & 3) << 4);
}

int kqo_dequant(uint32_t type, const void *src, uint64_t n, float *out) {
    const uint8_t *s = (const uint8_t *)src;
    if (!s || !out) return -1;
    if (type == KQO_Q4_K) {
        if (n % 256) return -1;
        for (uint64_t b = 0; b < n / 256; b++) {
            const uint8_t *blk = s + b * KQO_Q4_K_BYTES;
            const float d = kqo_f16_to_f32(ld16(blk));
            const float mn = kqo_f16_to_f32(ld16(blk + 2));
            for (int j = 0; j < 8; j++) {
                int sc, m;
                q4k_scale_min(j, blk + 4, &sc, &m);
                const float dl = d * (float)sc, ml = mn * (float)m;
                for (int i = 0; i < 32; i++)
                    out[b * 256 + 32 * j + i] = dl * (float)q4k_q(blk + 16, j, i) - ml;
            }
        }
        return 0;
    }
    if (type == KQO_Q6_K) {
        if (n % 256) return -1;
        for (uint64_t b = 0; b < n / 256; b++) {
            const uint8_t *blk = s + b * KQO_Q6_K_BYTES;
            const float d = kqo_f16_to_f32(ld16(blk + 208));
            for (int e = 0; e < 256; e++) {
                const int8_t sc = (int8_t)blk[192 + e / 16];
                out[b * 256 + e] = d * (float)sc * (float)(q6k_q(blk, e) - 32);
            }
        }
        return 0;
    }
    if (type == KQO_Q8_1) {
        if (n % 32) return -1;
        for (uint64_t b = 0; b < n / 32; b++) {
            const uint8_t *blk = s + b * KQO_Q8_1_BYTES;
            const float d = kqo_f16_to_f32(ld16(blk));
            for (int i = 0; i < 32; i++) out[b * 32 + i] = d * (float)(int8_t)blk[4 + i];
        }
        return 0;
    }
    return -1;
}

/* ------------------------------------------------------------------------ */
/* encoders                                                                  */
/* ------------------------------------------------------------------------ */
static inline int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

/* Q4_K: per 32-group offset M_j = max(0, -min) and step s_j = (max + M_j)/15;
 * super-scales d = max s_j / 63, dmin = max M_j / 63 stored as RNE fp16;
 * 6-bit sub-scales round(s_j/d), round(M_j/dmin) against the stored fp16
 * values; 4-bit q = round((x + dmin*m)/(d*sc)). */
int kqo_quantize_q4_K(const float *x, uint64_t n, void *out) {
    if (!x || !out || n % 256) return -1;
    uint8_t *o = (uint8_t *)out;
    for (uint64_t b = 0; b < n / 256; b++) {
        const float *xb = x + b * 256;
        uint8_t *blk = o + b * KQO_Q4_K_BYTES;
        float s[8], M[8], smax = 0.0f, Mmax = 0.0f;
        for (int j = 0; j < 8; j++) {
            float lo = xb[32 * j], hi = xb[32 * j];
            for (int i = 1; i < 32; i++) {
                const float v = xb[32 * j + i];
                if (v < lo) lo = v;
                if (v > hi) hi = v;
            }
            M[j] = lo < 0.0f ? -lo : 0.0f;
            s[j] = (hi + M[j]) / 15.0f;
            if (s[j] > smax) smax = s[j];
            if (M[j] > Mmax) Mmax = M[j];
        }
        const uint16_t dh = kqo_f32_to_f16(smax / 63.0f);
        const uint16_t mh = kqo_f32_to_f16(Mmax / 63.0f);
        const float d = kqo_f16_to_f32(dh), dmin = kqo_f16_to_f32(mh);
        int sc[8], mm[8];
        for (int j = 0; j < 8; j++) {
            sc[j] = d > 0.0f ? clampi((int)roundf(s[j] / d), 0, 63) : 0;
            mm[j] = dmin > 0.0f ? clampi((int)roundf(M[j] / dmin), 0, 63) : 0;
        }
        st16(blk, dh);
        st16(blk + 2, mh);
        uint8_t *scb = blk + 4;
        memset(scb, 0, 12);
        for (int j = 0; j < 4; j++) {
            scb[j] = (uint8_t)(sc[j] | ((sc[j + 4] >> 4) << 6));
            scb[j + 4] = (uint8_t)(mm[j] | ((mm[j + 4] >> 4) << 6));
            scb[j + 8] = (uint8_t)((sc[j + 4] & 0x0F) | ((mm[j + 4] & 0x0F) << 4));
        }
        uint8_t *qs = blk + 16;
        for (int j = 0; j < 8; j++) {
            const float ds = d * (float)sc[j];
            const float dm = dmin * (float)mm[j];
            for (int i = 0; i < 32; i++) {
                int q = 0;
                if (ds > 0.0f) q = clampi((int)roundf((xb[32 * j + i] + dm) / ds), 0, 15);
                uint8_t *p = qs + (j >> 1) * 32 + i;
                if (j & 1) *p = (uint8_t)(*p | (q << 4));
                else *p = (uint8_t)q;
            }
        }
    }
    return 0;
}

/* Q6_K: per 16-group s_k = amax/31, super-scale d = max s_k / 127 as RNE fp16,
 * int8 sub-scales round(s_k/d), 6-bit q = round(x/(d*sc)) + 32 in [0, 63]. */
int kqo_quantize_q6_K(const float *x, uint64_t n, void *out) {
    if (!x || !out || n % 256) return -1;
    uint8_t *o = (uint8_t *)out;
    for (uint64_t b = 0; b < n / 256; b++) {
        const float *xb = x + b * 256;
        uint8_t *blk = o + b * KQO_Q6_K_BYTES;
        float s[16], smax = 0.0f;
        for (int k = 0; k < 16; k++) {
            float amax = 0.0f;
            for (int i = 0; i < 16; i++) {
                const float a = fabsf(xb[16 * k + i]);
                if (a > amax) amax = a;
            }
            s[k] = amax / 31.0f;
            if (s[k] > smax) smax = s[k];
        }
        const uint16_t dh = kqo_f32_to_f16(smax / 127.0f);
        const float d = kqo_f16_to_f32(dh);
        memset(blk, 0, KQO_Q6_K_BYTES);
        for (int k = 0; k < 16; k++) {
            const int sc = d > 0.0f ? clampi((int)roundf(s[k] / d), -128, 127) : 0;
            blk[192 + k] = (uint8_t)(int8_t)sc;
            const float ds = d * (float)sc;
            for (int i = 0; i < 16; i++) {
                const int e = 16 * k + i;
                int q = 32;
                if (ds != 0.0f) q = clampi((int)roundf(xb[e] / ds), -32, 31) + 32;
                const int h = e >> 7, quarter = (e >> 5) & 3, l = e & 31;
                uint8_t *ql = blk + 64 * h + 32 * (quarter & 1) + l;
                uint8_t *qh = blk + 128 + 32 * h + l;
                if (quarter >= 2) *ql = (uint8_t)(*ql | ((q & 0x0F) << 4));
                else *ql = (uint8_t)(*ql | (q & 0x0F));
                *qh = (uint8_t)(*qh | (((q >> 4) & 3) << (2 * quarter)));
            }
        }
        st16(blk + 208, dh);
    }
    return 0;
}

/* q8_1: d = amax/127 in fp32; q = roundf(x/d) (0 when amax == 0); the block
 * stores RNE fp16 d and s = d*sum(q). */
int kqo_quantize_q8_1(const float *x, uint64_t n, void *out) {
    if (!x || !out || n % 32) return -1;
    uint8_t *o = (uint8_t *)out;
    for (uint64_t b = 0; b < n / 32; b++) {
        const float *xb = x + b * 32;
        uint8_t *blk = o + b * KQO_Q8_1_BYTES;
        float amax = 0.0f;
        for (int i = 0; i < 32; i++) {
            const float a = fabsf(xb[i]);
            if (a > amax) amax = a;
        }
        const float d = amax / 127.0f;
        int sum = 0;
        for (int i = 0; i < 32; i++) {
            const int q = amax == 0.0f ? 0 : clampi((int)roundf(xb[i] / d), -127, 127);
            blk[4 + i] = (uint8_t)(int8_t)q;
            sum += q;
        }
        st16(blk, kqo_f32_to_f16(d));
        st16(blk + 2, kqo_f32_to_f16(d * (float)sum));
    }
    return 0;
}

int kqo_quantize(uint32_t type, const float *x, uint64_t n, void *out) {
    switch (type) {
        case KQO_Q4_K: return kqo_quantize_q4_K(x, n, out);
        case KQO_Q6_K: return kqo_quantize_q6_K(x, n, out);
        case KQO_Q8_1: return kqo_quantize_q8_1(x, n, out);
        default: return -1;
    }
}

/* ------------------------------------------------------------------------ */
/* integer block dots against q8_1                                           */
/* ------------------------------------------------------------------------ */
int kqo_row_isums(uint32_t type, const void *row, const void *xq, uint64_t cols,
                  int32_t *isum, int32_t *xsum) {
    const uint8_t *w = (const uint8_t *)row, *a = (const uint8_t *)xq;
    if (!w || !a || !isum || cols % 256) return -1;
    const uint64_t nb = cols / 256;
    if (type == KQO_Q4_K) {
        for (uint64_t b = 0; b < nb; b++) {
            const uint8_t *qs = w + b * KQO_Q4_K_BYTES + 16;
            for (int j = 0; j < 8; j++) {
                const int8_t *qx = (const int8_t *)(a + (b * 8 + j) * KQO_Q8_1_BYTES + 4);
                int32_t s = 0, sx = 0;
                for (int i = 0; i < 32; i++) {
                    s += q4k_q(qs, j, i) * qx[i];
                    sx += qx[i];
                }
                isum[b * 8 + j] = s;
                if (xsum) xsum[b * 8 + j] = sx;
            }
        }
        return 0;
    }
    if (type == KQO_Q6_K) {
        for (uint64_t b = 0; b < nb; b++) {
            const uint8_t *blk = w + b * KQO_Q6_K_BYTES;
            for (int k = 0; k < 16; k++) {
                const int8_t *qx = (const int8_t *)(a + (b * 8 + k / 2) * KQO_Q8_1_BYTES + 4)
                                   + 16 * (k & 1);
                int32_t s = 0, sx = 0;
                for (int i = 0; i < 16; i++) {
                    s += (q6k_q(blk, 16 * k + i) - 32) * qx[i];
                    sx += qx[i];
                }
                isum[b * 16 + k] = s;
                if (xsum) xsum[b * 16 + k] = sx;
            }
        }
        return 0;
    }
    return -1;
}

/* Float combine, per q8_1 block (32 elements):
 *   Q4_K: ((double)d*dx) * (sc*isum) - ((double)dmin*dx) * (m*xsum)
 *   Q6_K: ((double)d*dx) * (sc_2j*isum_2j + sc_2j+1*isum_2j+1)
 * Both products are exact in double (<= 47 significant bits), so each term
 * rounds once; terms are summed in double and the row rounds once to float. */
float kqo_dot_q8(uint32_t type, const void *row, const void *xq, uint64_t cols) {
    const uint8_t *w = (const uint8_t *)row, *a = (const uint8_t *)xq;
    const uint64_t nb = cols / 256;
    double acc = 0.0;
    if (type == KQO_Q4_K) {
        for (uint64_t b = 0; b < nb; b++) {
            const uint8_t *blk = w + b * KQO_Q4_K_BYTES;
            const double d = kqo_f16_to_f32(ld16(blk));
            const double dmin = kqo_f16_to_f32(ld16(blk + 2));
            for (int j = 0; j < 8; j++) {
                const uint8_t *qb = a + (b * 8 + j) * KQO_Q8_1_BYTES;
                const int8_t *qx = (const int8_t *)(qb + 4);
                const double dx = kqo_f16_to_f32(ld16(qb));
                int sc, m;
                q4k_scale_min(j, blk + 4, &sc, &m);
                int32_t s = 0, sx = 0;
                for (int i = 0; i < 32; i++) {
                    s += q4k_q(blk + 16, j, i) * qx[i];
                    sx += qx[i];
                }
                acc += (d * dx) * (double)(sc * s) - (dmin * dx) * (double)(m * sx);
            }
        }
        return (float)acc;
    }
    if (type == KQO_Q6_K) {
        for (uint64_t b = 0; b < nb; b++) {
            const uint8_t *blk = w + b * KQO_Q6_K_BYTES;
            const double d = kqo_f16_to_f32(ld16(blk + 208));
            for (int j = 0; j < 8; j++) {
                const uint8_t *qb = a + (b * 8 + j) * KQO_Q8_1_BYTES;
                const int8_t *qx = (const int8_t *)(qb + 4);
                const double dx = kqo_f16_to_f32(ld16(qb));
                int32_t I = 0;
                for (int half = 0; half < 2; half++) {
                    const int k = 2 * j + half;
                    int32_t s = 0;
                    for (int i = 0; i < 16; i++) s += (q6k_q(blk, 16 * k + i) - 32) * qx[16 * half + i];
                    I += (int32_t)(int8_t)blk[192 + k] * s;
                }
                acc += (d * dx) * (double)I;
            }
        }
        return (float)acc;
    }
    return 0.0f;
}

int kqo_matvec_q8(uint32_t type, const void *w, uint64_t rows, uint64_t cols,
                  const void *xq, float *y) {
    const uint64_t rb = kqo_row_bytes(type, cols);
    if (!w || !xq || !y || rb == 0) return -1;
    for (uint64_t r = 0; r < rows; r++)
        y[r] = kqo_dot_q8(type, (const uint8_t *)w + r * rb, xq, cols);
    return 0;
}

/* fp32 activations. Q4_K follows the reference's scalar dot_q4_K
 * (V/src/gguf_dtype.c:594-624); Q6_K follows its fallback, a double dot over
 * the decoded row (katali_ggml_vec_dot_ref, :544-559). */
float kqo_dot_f32(uint32_t type, const void *row, const float *x, uint64_t cols) {
    const uint8_t *w = (const uint8_t *)row;
    const uint64_t nb = cols / 256;
    double acc = 0.0;
    if (type == KQO_Q4_K) {
        for (uint64_t b = 0; b < nb; b++) {
            const uint8_t *blk = w + b * KQO_Q4_K_BYTES;
            const float d = kqo_f16_to_f32(ld16(blk));
            const float mn = kqo_f16_to_f32(ld16(blk + 2));
            const float *xb = x + b * 256;
            for (int j = 0; j < 8; j++) {
                int sc, m;
                q4k_scale_min(j, blk + 4, &sc, &m);
                double sacc = 0.0, xacc = 0.0;
                for (int i = 0; i < 32; i++) {
                    sacc += (double)q4k_q(blk + 16, j, i) * (double)xb[32 * j + i];
                    xacc += (double)xb[32 * j + i];
                }
                acc += (double)(d * (float)sc) * sacc - (double)(mn * (float)m) * xacc;
            }
        }
        return (float)acc;
    }
    if (type == KQO_Q6_K) {
        float tmp[256];
        for (uint64_t b = 0; b < nb; b++) {
            kqo_dequant(KQO_Q6_K, w + b * KQO_Q6_K_BYTES, 256, tmp);
            for (int i = 0; i < 256; i++) acc += (double)tmp[i] * (double)x[b * 256 + i];
        }
        return (float)acc;
    }
    return 0.0f;
}

int kqo_matvec_f32(uint32_t type, const void *w, uint64_t rows, uint64_t cols,
                   const float *x, float *y) {
    const uint64_t rb = kqo_row_bytes(type, cols);
    if (!w || !x || !y || rb == 0) return -1;
    for (uint64_t r = 0; r < rows; r++)
        y[r] = kqo_dot_f32(type, (const uint8_t *)w + r * rb, x, cols);
    return 0;
}

/* ------------------------------------------------------------------------ */
/* routing                                                                   */
/* ------------------------------------------------------------------------ */
/* Total order used for top-k: NaN lowest, -0 == +0, larger value first, then
 * lower index. */
static inline uint32_t order_key(float f) {
    if (f != f) return 0u;
    f = f + 0.0f; /* -0 -> +0 */
    uint32_t u;
    memcpy(&u, &f, 4);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

int kqo_route_topk(const float *logits, int n, int k, int norm, int32_t *ids, float *w) {
    if (!logits || !ids || !w || n <= 0 || k <= 0 || k > n || k > 64) return -1;
    unsigned char taken[4096];
    if (n > 4096) return -1;
    memset(taken, 0, (size_t)n);
    for (int t = 0; t < k; t++) {
        int best = -1;
        uint32_t bk = 0;
        for (int i = 0; i < n; i++) {
            if (taken[i]) continue;
            const uint32_t key = order_key(logits[i]);
            if (best < 0 || key > bk) { best = i; bk = key; }
        }
        taken[best] = 1;
        ids[t] = best;
    }
    const float m = logits[ids[0]];
    float e[64];
    for (int t = 0; t < k; t++) e[t] = kqo_expf(logits[ids[t]] - m);
    double S = 0.0;
    if (norm) {
        for (int t = 0; t < k; t++) S += (double)e[t];
    } else {
        for (int i = 0; i < n; i++) S += (double)kqo_expf(logits[i] - m);
    }
    for (int t = 0; t < k; t++) w[t] = (float)((double)e[t] / S);
    return 0;
}

int kqo_argmax(const float *x, int n) {
    int best = 0;
    float bv = -3.402823466e+38f;
    for (int i = 0; i < n; i++)
        if (x[i] > bv) { bv = x[i]; best = i; }
    return best;
}

/* ------------------------------------------------------------------------ */
/* fused MoE layer                                                           */
/* ------------------------------------------------------------------------ */
int kqo_moe_layer_routed(const KqoMoe *m, const float *x, const int32_t *ids,
                         const float *w, float *y, int mode, float *h_out) {
    if (!m || !x || !ids || !w || !y) return -1;
    const int H = m->hidden, F = m->ffn, K = m->top_k;
    const uint64_t rbg = kqo_row_bytes(m->gate_type, (uint64_t)H);
    const uint64_t rbu = kqo_row_bytes(m->up_type, (uint64_t)H);
    const uint64_t rbd = kqo_row_bytes(m->down_type, (uint64_t)F);
    if (!rbg || !rbu || !rbd || H % 256 || F % 256) return -1;
    uint8_t *xq = (uint8_t *)malloc((size_t)H / 32 * KQO_Q8_1_BYTES);
    uint8_t *hq = (uint8_t *)malloc((size_t)K * F / 32 * KQO_Q8_1_BYTES);
    float *h = (float *)malloc((size_t)K * F * sizeof(float));
    if (!xq || !hq || !h) { free(xq); free(hq); free(h); return -1; }
    if (mode == 0) kqo_quantize_q8_1(x, (uint64_t)H, xq);
    for (int t = 0; t < K; t++) {
        const int e = ids[t];
        const uint8_t *G = (const uint8_t *)m->gate[e];
        const uint8_t *U = (const uint8_t *)m->up[e];
        for (int j = 0; j < F; j++) {
            float g, u;
            if (mode == 0) {
                g = kqo_dot_q8(m->gate_type, G + (uint64_t)j * rbg, xq, (uint64_t)H);
                u = kqo_dot_q8(m->up_type, U + (uint64_t)j * rbu, xq, (uint64_t)H);
            } else {
                g = kqo_dot_f32(m->gate_type, G + (uint64_t)j * rbg, x, (uint64_t)H);
                u = kqo_dot_f32(m->up_type, U + (uint64_t)j * rbu, x, (uint64_t)H);
            }
            h[(size_t)t * F + j] = kqo_silu(g) * u;
        }
        if (mode == 0)
            kqo_quantize_q8_1(h + (size_t)t * F, (uint64_t)F,
                              hq + (size_t)t * F / 32 * KQO_Q8_1_BYTES);
    }
    for (int r = 0; r < H; r++) {
        double acc = 0.0;
        for (int t = 0; t < K; t++) {
            const uint8_t *D = (const uint8_t *)m->down[ids[t]] + (uint64_t)r * rbd;
            const float v = mode == 0
                ? kqo_dot_q8(m->down_type, D, hq + (size_t)t * F / 32 * KQO_Q8_1_BYTES, (uint64_t)F)
                : kqo_dot_f32(m->down_type, D, h + (size_t)t * F, (uint64_t)F);
            acc += (double)w[t] * (double)v;
        }
        y[r] = (float)acc;
    }
    if (h_out) memcpy(h_out, h, (size_t)K * F * sizeof(float));
    free(xq); free(hq); free(h);
    return 0;
}

/* ------------------------------------------------------------------------ */
/* expert-parallel slot protocol                                             */
/* ------------------------------------------------------------------------ */
uint32_t kqo_ep_slot_bytes(int hidden, int top_k) {
    return ((uint32_t)(16 + 8 * top_k + 15) & ~15u) + (uint32_t)hidden / 32 * KQO_Q8_1_BYTES;
}

static int ep_geometry_ok(const KqoMoe *m, int n_ranks, int max_tokens) {
    return m && n_ranks > 0 && max_tokens > 0 && m->n_experts % n_ranks == 0 &&
           m->top_k > 0 && m->top_k <= 64 && m->hidden % 256 == 0;
}

int kqo_ep_dispatch(const KqoMoe *m, int n_ranks, int max_tokens, int n_tokens,
                    const float *x, const float *logits, uint8_t *send, int32_t *src_ids) {
    if (!ep_geometry_ok(m, n_ranks, max_tokens) || n_tokens < 0 || n_tokens > max_tokens)
        return -1;
    const int H = m->hidden, K = m->top_k, per = m->n_experts / n_ranks;
    const uint32_t sb = kqo_ep_slot_bytes(H, K), hdr = sb - (uint32_t)H / 32 * KQO_Q8_1_BYTES;
    uint8_t *row = (uint8_t *)malloc((size_t)H / 32 * KQO_Q8_1_BYTES);
    if (!row) return -1;
    for (int t = 0; t < max_tokens; t++) {
        int32_t ids[64];
        float w[64];
        if (t < n_tokens) {
            if (kqo_route_topk(logits + (size_t)t * m->n_experts, m->n_experts, K, m->norm_topk,
                               ids, w) != 0) {
                free(row);
                return -1;
            }
            memcpy(src_ids + (size_t)t * K, ids, sizeof(int32_t) * (size_t)K);
            kqo_quantize_q8_1(x + (size_t)t * H, (uint64_t)H, row);
        }
        for (int d = 0; d < n_ranks; d++) {
            uint8_t *slot = send + ((size_t)d * max_tokens + t) * sb;
            int32_t head[4] = {0, t, 0, 0};
            if (t < n_tokens) {
                int32_t *sid = (int32_t *)(slot + 16);
                float *sw = (float *)(slot + 16 + 4 * K);
                for (int k = 0; k < K; k++) {
                    const int own = ids[k] / per == d;
                    head[0] += own;
                    sid[k] = own ? ids[k] : -1;
                    sw[k] = w[k];
                }
                if (head[0] > 0) memcpy(slot + hdr, row, (size_t)H / 32 * KQO_Q8_1_BYTES);
            }
            memcpy(slot, head, sizeof head);
        }
    }
    free(row);
    return 0;
}

int kqo_ep_experts(const KqoMoe *m, int n_ranks, int rank, int max_tokens,
                   const uint8_t *recv, double *ret) {
    if (!ep_geometry_ok(m, n_ranks, max_tokens) || rank < 0 || rank >= n_ranks) return -1;
    const int H = m->hidden, F = m->ffn, K = m->top_k;
    const uint32_t sb = kqo_ep_slot_bytes(H, K), hdr = sb - (uint32_t)H / 32 * KQO_Q8_1_BYTES;
    const uint64_t rbg = kqo_row_bytes(m->gate_type, (uint64_t)H);
    const uint64_t rbu = kqo_row_bytes(m->up_type, (uint64_t)H);
    if (!rbg || !rbu || F % 256) return -1;
    float *h = (float *)malloc((size_t)F * sizeof(float));
    float *dv = (float *)malloc((size_t)H * sizeof(float));
    uint8_t *hq = (uint8_t *)malloc((size_t)F / 32 * KQO_Q8_1_BYTES);
    if (!h || !dv || !hq) { free(h); free(dv); free(hq); return -1; }
    for (int s = 0; s < n_ranks * max_tokens; s++) {
        const uint8_t *slot = recv + (size_t)s * sb;
        int32_t n;
        memcpy(&n, slot, 4);
        if (n <= 0) continue;
        const uint8_t *xq = slot + hdr;
        double *acc = ret + (size_t)s * H;
        for (int r = 0; r < H; r++) acc[r] = 0.0;
        for (int k = 0; k < K; k++) {
            int32_t e;
            float w;
            memcpy(&e, slot + 16 + 4 * k, 4);
            memcpy(&w, slot + 16 + 4 * K + 4 * k, 4);
            if (e < 0) continue;
            const uint8_t *G = (const uint8_t *)m->gate[e];
            const uint8_t *U = (const uint8_t *)m->up[e];
            for (int j = 0; j < F; j++) {
                const float g = kqo_dot_q8(m->gate_type, G + (uint64_t)j * rbg, xq, (uint64_t)H);
                const float u = kqo_dot_q8(m->up_type, U + (uint64_t)j * rbu, xq, (uint64_t)H);
                h[j] = kqo_silu(g) * u;
            }
            kqo_quantize_q8_1(h, (uint64_t)F, hq);
            kqo_matvec_q8(m->down_type, (const uint8_t *)m->down[e], (uint64_t)H, (uint64_t)F, hq, dv);
            for (int r = 0; r < H; r++) acc[r] += (double)w * (double)dv[r];
        }
    }
    free(h); free(dv); free(hq);
    return 0;
}

int kqo_ep_combine(const KqoMoe *m, int n_ranks, int max_tokens, int n_tokens,
                   const int32_t *src_ids, const double *back, float *y) {
    if (!ep_geometry_ok(m, n_ranks, max_tokens) || n_tokens < 0 || n_tokens > max_tokens)
        return -1;
    const int H = m->hidden, K = m->top_k, per = m->n_experts / n_ranks;
    for (int t = 0; t < n_tokens; t++) {
        for (int r = 0; r < H; r++) {
            double acc = 0.0;
            for (int d = 0; d < n_ranks; d++) {
                int own = 0;
                for (int k = 0; k < K; k++) own |= src_ids[(size_t)t * K + k] / per == d;
                if (own) acc += back[((size_t)d * max_tokens + t) * H + r];
            }
            y[(size_t)t * H + r] = (float)acc;
        }
    }
    return 0;
}

int kqo_moe_layer(const KqoMoe *m, const float *x, const float *logits,
                  float *y, int mode, int32_t *ids, float *w, float *h_out) {
    if (!m || m->top_k <= 0 || m->top_k > 64) return -1;
    int32_t idl[64];
    float wl[64];
    if (kqo_route_topk(logits, m->n_experts, m->top_k, m->norm_topk, idl, wl) != 0) return -1;
    if (ids) memcpy(ids, idl, sizeof(int32_t) * (size_t)m->top_k);
    if (w) memcpy(w, wl, sizeof(float) * (size_t)m->top_k);
    return kqo_moe_layer_routed(m, x, idl, wl, y, mode, h_out);
}
