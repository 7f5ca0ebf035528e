/* oracle/quants_oracle.c -- TEST INFRASTRUCTURE ONLY (see sepia_oracle.h).
 *
 * CPU restatement of GGML block dequantization. Each superblock decoder is
 * written as eight 32-element "parts" (part p covers elements 32p..32p+31),
 * and computes every element with the same fp32 operation sequence as the
 * reference (src/quants.c:79-248) or, for the four formats the reference
 * lacks, as gguf-py 0.19.0's numpy `dequantize_blocks` (gguf/quants.py:
 * Q2_K:404, Q3_K:431, IQ2_XXS:766, IQ1_S:1128). Products and differences are
 * kept as separate roundings: FP_CONTRACT is off, exactly as the reference
 * compiles src/quants.c (src/quants.c:6). */
#pragma STDC FP_CONTRACT OFF

#include "sepia_oracle.h"

#include <string.h>

#define SEPIA_TABLE_QUAL static const
#include "../sepia_b200/csrc/quant_tables.h"

#define QK 256

typedef struct { int type; int64_t elems; size_t bytes; } OrFmt;

/* Block geometry: src/quants.c:28-32 plus ggml's Q2_K/Q3_K/IQ2_XXS/IQ1_S. */
static const OrFmt FMTS[] = {
    { OR_T_F32, 1, 4 },      { OR_T_F16, 1, 2 },       { OR_T_Q8_0, 32, 34 },
    { OR_T_Q2_K, QK, 84 },   { OR_T_Q3_K, QK, 110 },   { OR_T_Q4_K, QK, 144 },
    { OR_T_Q5_K, QK, 176 },  { OR_T_Q6_K, QK, 210 },   { OR_T_IQ2_XXS, QK, 66 },
    { OR_T_IQ2_XS, QK, 74 }, { OR_T_IQ3_XXS, QK, 98 }, { OR_T_IQ1_S, QK, 50 },
    { OR_T_IQ4_XS, QK, 136 },
};

static const OrFmt *fmt_of(int t) {
    for (size_t i = 0; i < sizeof FMTS / sizeof FMTS[0]; i++)
        if (FMTS[i].type == t) return &FMTS[i];
    return NULL;
}

int or_supported(int t) { return fmt_of(t) != NULL; }
int64_t or_block_size(int t) { const OrFmt *f = fmt_of(t); return f ? f->elems : 0; }
size_t or_type_size(int t) { const OrFmt *f = fmt_of(t); return f ? f->bytes : 0; }
size_t or_row_bytes(int t, int64_t n) {
    const OrFmt *f = fmt_of(t);
    if (!f || n < 0 || n % f->elems) return 0;
    return (size_t)(n / f->elems) * f->bytes;
}

static uint16_t rd16(const uint8_t *p) { uint16_t v; memcpy(&v, p, 2); return v; }
static uint32_t rd32(const uint8_t *p) { uint32_t v; memcpy(&v, p, 4); return v; }

/* IEEE half -> float by bit manipulation, subnormals normalised, Inf/NaN
 * payload kept (src/quants.c:58-77). */
float or_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h >> 15) << 31;
    int32_t e = (h >> 10) & 0x1F;
    uint32_t m = h & 0x3FF, bits;
    if (e == 0x1F) {
        bits = sign | 0x7F800000u | (m << 13);
    } else if (e != 0) {
        bits = sign | ((uint32_t)(e + 112) << 23) | (m << 13);
    } else if (m == 0) {
        bits = sign;
    } else {
        int32_t E = 113;                 /* 127 - 15 + 1 */
        while (!(m & 0x400)) { m <<= 1; E--; }
        bits = sign | ((uint32_t)E << 23) | ((m & 0x3FF) << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* 6-bit scale/min pair j of the 12-byte K-quant scale field
 * (src/quants.c:96-102). */
static void kscale(const uint8_t *s, int j, int *sc, int *mn) {
    if (j < 4) {
        *sc = s[j] & 63;
        *mn = s[j + 4] & 63;
    } else {
        *sc = (s[j + 4] & 15) | ((s[j - 4] >> 6) << 4);
        *mn = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
}

/* ---- one superblock -> 256 floats, per format --------------------------- */

static void sb_q2_k(const uint8_t *b, float *y) {
    const uint8_t *sc = b, *qs = b + 16;
    const float d = or_f16_to_f32(rd16(b + 80)), dmin = or_f16_to_f32(rd16(b + 82));
    for (int p = 0; p < 8; p++) {
        const uint8_t *q = qs + 32 * (p >> 2);
        const int sh = 2 * (p & 3);
        for (int g = 0; g < 2; g++) {
            const uint8_t s = sc[2 * p + g];
            const float dl = d * (float)(s & 15), ml = dmin * (float)(s >> 4);
            for (int l = 0; l < 16; l++)
                y[32 * p + 16 * g + l] = dl * (float)((q[16 * g + l] >> sh) & 3) - ml;
        }
    }
}

/* Q3_K's sixteen 6-bit scales: low nibble from bytes 0..7, high pair from
 * bytes 8..11 (gguf/quants.py:441-457 packing diagram). */
static int q3k_scale(const uint8_t *s, int i) {
    int lo = (i < 8) ? (s[i] & 15) : (s[i - 8] >> 4);
    int hi = (s[8 + (i & 3)] >> (2 * (i >> 2))) & 3;
    return (lo | (hi << 4)) - 32;
}

static void sb_q3_k(const uint8_t *b, float *y) {
    const uint8_t *hm = b, *qs = b + 32, *sc = b + 96;
    const float d = or_f16_to_f32(rd16(b + 108));
    for (int p = 0; p < 8; p++) {
        const uint8_t *q = qs + 32 * (p >> 2);
        const int sh = 2 * (p & 3);
        for (int g = 0; g < 2; g++) {
            const float dl = d * (float)q3k_scale(sc, 2 * p + g);
            for (int l = 16 * g; l < 16 * g + 16; l++) {
                int v = ((q[l] >> sh) & 3) - (((hm[l] >> p) & 1) ? 0 : 4);
                y[32 * p + l] = dl * (float)v;
            }
        }
    }
}

static void sb_q4_k(const uint8_t *b, float *y) {
    const float d = or_f16_to_f32(rd16(b)), dmin = or_f16_to_f32(rd16(b + 2));
    const uint8_t *sc = b + 4, *qs = b + 16;
    for (int p = 0; p < 8; p++) {
        int s, m;
        kscale(sc, p, &s, &m);
        const float dl = d * (float)s, ml = dmin * (float)m;
        const uint8_t *q = qs + 32 * (p >> 1);
        const int sh = 4 * (p & 1);
        for (int l = 0; l < 32; l++) y[32 * p + l] = dl * (float)((q[l] >> sh) & 15) - ml;
    }
}

static void sb_q5_k(const uint8_t *b, float *y) {
    const float d = or_f16_to_f32(rd16(b)), dmin = or_f16_to_f32(rd16(b + 2));
    const uint8_t *sc = b + 4, *qh = b + 16, *qs = b + 48;
    for (int p = 0; p < 8; p++) {
        int s, m;
        kscale(sc, p, &s, &m);
        const float dl = d * (float)s, ml = dmin * (float)m;
        const uint8_t *q = qs + 32 * (p >> 1);
        const int sh = 4 * (p & 1);
        for (int l = 0; l < 32; l++) {
            int v = ((q[l] >> sh) & 15) + (((qh[l] >> p) & 1) ? 16 : 0);
            y[32 * p + l] = dl * (float)v - ml;
        }
    }
}

static void sb_q6_k(const uint8_t *b, float *y) {
    const uint8_t *ql = b, *qh = b + 128;
    const int8_t *sc = (const int8_t *)(b + 192);
    const float d = or_f16_to_f32(rd16(b + 208));
    for (int p = 0; p < 8; p++) {
        const int half = p >> 2, k = p & 3;
        const uint8_t *L = ql + 64 * half + 32 * (k & 1);
        const uint8_t *Hh = qh + 32 * half;
        for (int l = 0; l < 32; l++) {
            int lo = (L[l] >> (4 * (k >> 1))) & 15;
            int hi = (Hh[l] >> (2 * k)) & 3;
            int v = (lo | (hi << 4)) - 32;
            /* (d * sc) * q, as src/quants.c:166-169 */
            y[32 * p + l] = d * (float)sc[8 * half + 2 * k + l / 16] * (float)v;
        }
    }
}

static void sb_iq2_xxs(const uint8_t *b, float *y) {
    const float d = or_f16_to_f32(rd16(b));
    for (int p = 0; p < 8; p++) {
        const uint32_t idx = rd32(b + 2 + 8 * p), sgn = rd32(b + 6 + 8 * p);
        const float db = d * (0.5f + (float)(sgn >> 28)) * 0.25f;
        for (int l = 0; l < 4; l++) {
            const uint64_t row = sepia_iq2xxs_grid[(idx >> (8 * l)) & 255];
            const uint8_t s = sepia_ksigns_iq2xs[(sgn >> (7 * l)) & 127];
            for (int j = 0; j < 8; j++) {
                float gv = (float)((row >> (8 * j)) & 255);
                y[32 * p + 8 * l + j] = db * gv * ((s >> j) & 1 ? -1.0f : 1.0f);
            }
        }
    }
}

static void sb_iq2_xs(const uint8_t *b, float *y) {
    const float d = or_f16_to_f32(rd16(b));
    const uint8_t *sc = b + 66;
    for (int p = 0; p < 8; p++) {
        const float db0 = d * (0.5f + (float)(sc[p] & 15)) * 0.25f;
        const float db1 = d * (0.5f + (float)(sc[p] >> 4)) * 0.25f;
        for (int l = 0; l < 4; l++) {
            const uint16_t q = rd16(b + 2 + 2 * (4 * p + l));
            const uint64_t row = sepia_iq2xs_grid[q & 511];
            const uint8_t s = sepia_ksigns_iq2xs[q >> 9];
            const float dl = (l < 2) ? db0 : db1;
            for (int j = 0; j < 8; j++) {
                float gv = (float)((row >> (8 * j)) & 255);
                y[32 * p + 8 * l + j] = dl * gv * ((s >> j) & 1 ? -1.0f : 1.0f);
            }
        }
    }
}

static void sb_iq3_xxs(const uint8_t *b, float *y) {
    const float d = or_f16_to_f32(rd16(b));
    const uint8_t *qs = b + 2, *sas = b + 66;
    for (int p = 0; p < 8; p++) {
        const uint32_t a = rd32(sas + 4 * p);
        const float db = d * (0.5f + (float)(a >> 28)) * 0.5f;
        for (int l = 0; l < 4; l++) {
            const uint8_t s = sepia_ksigns_iq2xs[(a >> (7 * l)) & 127];
            const uint32_t g1 = sepia_iq3xxs_grid[qs[8 * p + 2 * l]];
            const uint32_t g2 = sepia_iq3xxs_grid[qs[8 * p + 2 * l + 1]];
            for (int j = 0; j < 4; j++) {
                y[32 * p + 8 * l + j] = db * (float)((g1 >> (8 * j)) & 255) * ((s >> j) & 1 ? -1.0f : 1.0f);
                y[32 * p + 8 * l + 4 + j] = db * (float)((g2 >> (8 * j)) & 255) * ((s >> (j + 4)) & 1 ? -1.0f : 1.0f);
            }
        }
    }
}

static void sb_iq1_s(const uint8_t *b, float *y) {
    const float d = or_f16_to_f32(rd16(b));
    const uint8_t *qs = b + 2;
    for (int p = 0; p < 8; p++) {
        const uint16_t h = rd16(b + 34 + 2 * p);
        const float dl = d * (float)(2 * ((h >> 12) & 7) + 1);
        const float delta = (h & 0x8000) ? -0.125f : 0.125f;
        for (int l = 0; l < 4; l++) {
            const uint64_t row = sepia_iq1s_grid[qs[4 * p + l] | (((h >> (3 * l)) & 7) << 8)];
            for (int j = 0; j < 8; j++) {
                float gv = (float)(int8_t)((row >> (8 * j)) & 255);
                y[32 * p + 8 * l + j] = dl * (gv + delta);
            }
        }
    }
}

static void sb_iq4_xs(const uint8_t *b, float *y) {
    const float d = or_f16_to_f32(rd16(b));
    const uint16_t sh = rd16(b + 2);
    const uint8_t *sl = b + 4, *qs = b + 8;
    for (int p = 0; p < 8; p++) {
        const int ls = ((sl[p >> 1] >> (4 * (p & 1))) & 15) | (((sh >> (2 * p)) & 3) << 4);
        const float dl = d * (float)(ls - 32);
        for (int j = 0; j < 16; j++) {
            y[32 * p + j] = dl * (float)sepia_kvalues_iq4nl[qs[16 * p + j] & 15];
            y[32 * p + 16 + j] = dl * (float)sepia_kvalues_iq4nl[qs[16 * p + j] >> 4];
        }
    }
}

int or_dequantize_row(int t, const void *src, float *dst, int64_t n) {
    const OrFmt *f = fmt_of(t);
    if (!f || n < 0 || n % f->elems) return 0;
    const uint8_t *p = (const uint8_t *)src;
    const int64_t nb = n / f->elems;
    switch (t) {
    case OR_T_F32: memcpy(dst, src, (size_t)n * 4); return 1;
    case OR_T_F16:
        for (int64_t i = 0; i < n; i++) dst[i] = or_f16_to_f32(rd16(p + 2 * i));
        return 1;
    case OR_T_Q8_0:
        for (int64_t b = 0; b < nb; b++, p += 34) {
            const float d = or_f16_to_f32(rd16(p));
            for (int j = 0; j < 32; j++) dst[32 * b + j] = d * (float)(int8_t)p[2 + j];
        }
        return 1;
    default: break;
    }
    void (*sb)(const uint8_t *, float *) = NULL;
    switch (t) {
    case OR_T_Q2_K: sb = sb_q2_k; break;
    case OR_T_Q3_K: sb = sb_q3_k; break;
    case OR_T_Q4_K: sb = sb_q4_k; break;
    case OR_T_Q5_K: sb = sb_q5_k; break;
    case OR_T_Q6_K: sb = sb_q6_k; break;
    case OR_T_IQ2_XXS: sb = sb_iq2_xxs; break;
    case OR_T_IQ2_XS: sb = sb_iq2_xs; break;
    case OR_T_IQ3_XXS: sb = sb_iq3_xxs; break;
    case OR_T_IQ1_S: sb = sb_iq1_s; break;
    case OR_T_IQ4_XS: sb = sb_iq4_xs; break;
    default: return 0;
    }
    for (int64_t b = 0; b < nb; b++) sb(p + (size_t)b * f->bytes, dst + QK * b);
    return 1;
}
