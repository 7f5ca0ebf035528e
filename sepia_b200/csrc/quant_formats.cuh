// sepia_b200/csrc/quant_formats.cuh -- GGML block formats on the device.
//
// Every 256-wide superblock is split into eight 32-element "parts"; part p
// covers elements 32p..32p+31 of the superblock for every format (for Q8_0
// a "superblock" is 8 consecutive 34-byte blocks and part p is block p; for
// F16/F32 it is 256 consecutive values). One lane owns one part, so eight
// lanes cover a superblock and a warp covers four.
//
// Two decoders per format:
//   decode_part_exact  fp32 values bit-identical to the reference CPU
//                      dequant (src/quants.c:79-248; gguf-py 0.19.0 for
//                      Q2_K/Q3_K/IQ2_XXS/IQ1_S) -- explicit __fmul_rn /
//                      __fadd_rn / __fsub_rn, never contracted to FMA.
// The GEMV dot products over a part live in quant_dot.cuh.
//
// Byte reads go through shared memory at whatever alignment the block has
// (blocks of 110, 50, 66, ... bytes are only 2-byte aligned); see rd_words.
#pragma once
#include "common.cuh"

#define SEPIA_TABLE_QUAL static __device__ const
#include "quant_tables.h"

namespace sepia {

enum GgmlType : int {
    T_F32 = 0, T_F16 = 1, T_Q8_0 = 8, T_Q2_K = 10, T_Q3_K = 11, T_Q4_K = 12, T_Q5_K = 13,
    T_Q6_K = 14, T_IQ2_XXS = 16, T_IQ2_XS = 17, T_IQ3_XXS = 18, T_IQ1_S = 19, T_IQ4_XS = 23,
};

// Elements and bytes of one ggml block (src/quants.c:28-32 + ggml).
__host__ __device__ constexpr int fmt_block_elems(int t) {
    switch (t) {
    case T_F32: case T_F16: return 1;
    case T_Q8_0: return 32;
    case T_Q2_K: case T_Q3_K: case T_Q4_K: case T_Q5_K: case T_Q6_K:
    case T_IQ2_XXS: case T_IQ2_XS: case T_IQ3_XXS: case T_IQ1_S: case T_IQ4_XS: return 256;
    default: return 0;
    }
}
__host__ __device__ constexpr int fmt_block_bytes(int t) {
    switch (t) {
    case T_F32: return 4;
    case T_F16: return 2;
    case T_Q8_0: return 34;
    case T_Q2_K: return 84;
    case T_Q3_K: return 110;
    case T_Q4_K: return 144;
    case T_Q5_K: return 176;
    case T_Q6_K: return 210;
    case T_IQ2_XXS: return 66;
    case T_IQ2_XS: return 74;
    case T_IQ3_XXS: return 98;
    case T_IQ1_S: return 50;
    case T_IQ4_XS: return 136;
    default: return 0;
    }
}
// Bytes of one 256-element "superblock" as the kernels index it.
__host__ __device__ inline int fmt_sb_bytes(int t) {
    return fmt_block_bytes(t) * (kQK / fmt_block_elems(t));
}

// ----------------------------------------------------------- byte access
// 4 bytes starting at any 2-byte-aligned shared-memory address.
__device__ __forceinline__ uint32_t rd32(const uint8_t *p) { return lds_u32_any(p); }
__device__ __forceinline__ uint32_t rd16(const uint8_t *p) { return lds_u16(p); }

// n consecutive 32-bit words starting at p (any alignment): n+1 aligned
// loads plus funnel shifts.
template <int N>
__device__ __forceinline__ void rd_words(const uint8_t *p, uint32_t (&w)[N]) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    const uint32_t *base = reinterpret_cast<const uint32_t *>(a & ~(uintptr_t)3);
    const uint32_t sh = (uint32_t)(a & 3) * 8;
    uint32_t prev = base[0];
#pragma unroll
    for (int i = 0; i < N; i++) {
        const uint32_t next = base[i + 1];
        w[i] = __funnelshift_r(prev, next, sh);
        prev = next;
    }
}

// ==================================================================
// Exact decoders (bitwise parity with the CPU reference)
// ==================================================================
__device__ __forceinline__ void kscale_pair(const uint8_t *s, int j, int &sc, int &mn) {
    // src/quants.c:96-102
    if (j < 4) {
        sc = s[j] & 63;
        mn = s[j + 4] & 63;
    } else {
        sc = (s[j + 4] & 15) | ((s[j - 4] >> 6) << 4);
        mn = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
}

__device__ __forceinline__ int q3k_scale(const uint8_t *s, int i) {
    const int lo = (i < 8) ? (s[i] & 15) : (s[i - 8] >> 4);
    const int hi = (s[8 + (i & 3)] >> (2 * (i >> 2))) & 3;
    return (lo | (hi << 4)) - 32;
}

__device__ __forceinline__ float sgnf(uint32_t s, int j) { return ((s >> j) & 1) ? -1.0f : 1.0f; }

// fp16 bits -> float: HW = false uses the integer restatement (NaN payloads
// kept bit for bit, for the bitwise dequant gate); HW = true uses the
// conversion instruction (identical for every finite value and infinity).
template <bool HW>
__device__ __forceinline__ float cvt16(uint32_t h) {
    if constexpr (HW) return __half2float(__ushort_as_half((unsigned short)h));
    else return f16_bits_to_f32(h);
}

// Decode part p of superblock `b` (bytes of the whole superblock) into y[32].
// For F32/F16 `n_valid` limits the elements read (ragged last superblock).
template <bool HW = false>
__device__ __forceinline__ void decode_part_exact(int t, const uint8_t *b, int p, float *y, int n_valid = 32) {
    switch (t) {
    case T_F32: {
        const uint8_t *q = b + 128 * p;
        for (int i = 0; i < n_valid; i++) y[i] = __uint_as_float(rd32(q + 4 * i));
        break;
    }
    case T_F16: {
        const uint8_t *q = b + 64 * p;
        for (int i = 0; i < n_valid; i++) y[i] = cvt16<HW>(rd16(q + 2 * i));
        break;
    }
    case T_Q8_0: {
        const uint8_t *q = b + 34 * p;
        const float d = cvt16<HW>(rd16(q));
        for (int i = 0; i < 32; i++) y[i] = __fmul_rn(d, (float)(int8_t)q[2 + i]);
        break;
    }
    case T_Q2_K: {
        const float d = cvt16<HW>(rd16(b + 80)), dmin = cvt16<HW>(rd16(b + 82));
        const uint8_t *q = b + 16 + 32 * (p >> 2);
        const int sh = 2 * (p & 3);
        for (int g = 0; g < 2; g++) {
            const int s = b[2 * p + g];
            const float dl = __fmul_rn(d, (float)(s & 15)), ml = __fmul_rn(dmin, (float)(s >> 4));
            for (int l = 0; l < 16; l++)
                y[16 * g + l] = __fsub_rn(__fmul_rn(dl, (float)((q[16 * g + l] >> sh) & 3)), ml);
        }
        break;
    }
    case T_Q3_K: {
        const float d = cvt16<HW>(rd16(b + 108));
        const uint8_t *hm = b, *q = b + 32 + 32 * (p >> 2), *sc = b + 96;
        const int sh = 2 * (p & 3);
        for (int g = 0; g < 2; g++) {
            const float dl = __fmul_rn(d, (float)q3k_scale(sc, 2 * p + g));
            for (int l = 16 * g; l < 16 * g + 16; l++) {
                const int v = ((q[l] >> sh) & 3) - (((hm[l] >> p) & 1) ? 0 : 4);
                y[l] = __fmul_rn(dl, (float)v);
            }
        }
        break;
    }
    case T_Q4_K: case T_Q5_K: {
        const float d = cvt16<HW>(rd16(b)), dmin = cvt16<HW>(rd16(b + 2));
        int s, m;
        kscale_pair(b + 4, p, s, m);
        const float dl = __fmul_rn(d, (float)s), ml = __fmul_rn(dmin, (float)m);
        const int sh = 4 * (p & 1);
        if (t == T_Q4_K) {
            const uint8_t *q = b + 16 + 32 * (p >> 1);
            for (int l = 0; l < 32; l++) y[l] = __fsub_rn(__fmul_rn(dl, (float)((q[l] >> sh) & 15)), ml);
        } else {
            const uint8_t *qh = b + 16, *q = b + 48 + 32 * (p >> 1);
            for (int l = 0; l < 32; l++) {
                const int v = ((q[l] >> sh) & 15) + (((qh[l] >> p) & 1) ? 16 : 0);
                y[l] = __fsub_rn(__fmul_rn(dl, (float)v), ml);
            }
        }
        break;
    }
    case T_Q6_K: {
        const float d = cvt16<HW>(rd16(b + 208));
        const int half = p >> 2, k = p & 3;
        const uint8_t *L = b + 64 * half + 32 * (k & 1), *Hh = b + 128 + 32 * half;
        const int8_t *sc = reinterpret_cast<const int8_t *>(b + 192 + 8 * half + 2 * k);
        for (int l = 0; l < 32; l++) {
            const int lo = (L[l] >> (4 * (k >> 1))) & 15, hi = (Hh[l] >> (2 * k)) & 3;
            const int v = (lo | (hi << 4)) - 32;
            y[l] = __fmul_rn(__fmul_rn(d, (float)sc[l >> 4]), (float)v);
        }
        break;
    }
    case T_IQ2_XXS: {
        const float d = cvt16<HW>(rd16(b));
        const uint32_t idx = rd32(b + 2 + 8 * p), sg = rd32(b + 6 + 8 * p);
        const float db = __fmul_rn(__fmul_rn(d, __fadd_rn(0.5f, (float)(sg >> 28))), 0.25f);
        for (int l = 0; l < 4; l++) {
            const uint64_t row = sepia_iq2xxs_grid[(idx >> (8 * l)) & 255];
            const uint32_t s = sepia_ksigns_iq2xs[(sg >> (7 * l)) & 127];
            for (int j = 0; j < 8; j++)
                y[8 * l + j] = __fmul_rn(__fmul_rn(db, (float)((row >> (8 * j)) & 255)), sgnf(s, j));
        }
        break;
    }
    case T_IQ2_XS: {
        const float d = cvt16<HW>(rd16(b));
        const int sc = b[66 + p];
        const float db0 = __fmul_rn(__fmul_rn(d, __fadd_rn(0.5f, (float)(sc & 15))), 0.25f);
        const float db1 = __fmul_rn(__fmul_rn(d, __fadd_rn(0.5f, (float)(sc >> 4))), 0.25f);
        for (int l = 0; l < 4; l++) {
            const uint32_t q = rd16(b + 2 + 2 * (4 * p + l));
            const uint64_t row = sepia_iq2xs_grid[q & 511];
            const uint32_t s = sepia_ksigns_iq2xs[q >> 9];
            const float dl = (l < 2) ? db0 : db1;
            for (int j = 0; j < 8; j++)
                y[8 * l + j] = __fmul_rn(__fmul_rn(dl, (float)((row >> (8 * j)) & 255)), sgnf(s, j));
        }
        break;
    }
    case T_IQ3_XXS: {
        const float d = cvt16<HW>(rd16(b));
        const uint32_t a = rd32(b + 66 + 4 * p);
        const float db = __fmul_rn(__fmul_rn(d, __fadd_rn(0.5f, (float)(a >> 28))), 0.5f);
        const uint8_t *qs = b + 2 + 8 * p;
        for (int l = 0; l < 4; l++) {
            const uint32_t s = sepia_ksigns_iq2xs[(a >> (7 * l)) & 127];
            const uint32_t g1 = sepia_iq3xxs_grid[qs[2 * l]], g2 = sepia_iq3xxs_grid[qs[2 * l + 1]];
            for (int j = 0; j < 4; j++) {
                y[8 * l + j] = __fmul_rn(__fmul_rn(db, (float)((g1 >> (8 * j)) & 255)), sgnf(s, j));
                y[8 * l + 4 + j] = __fmul_rn(__fmul_rn(db, (float)((g2 >> (8 * j)) & 255)), sgnf(s, j + 4));
            }
        }
        break;
    }
    case T_IQ1_S: {
        const float d = cvt16<HW>(rd16(b));
        const uint32_t h = rd16(b + 34 + 2 * p);
        const float dl = __fmul_rn(d, (float)(2 * ((h >> 12) & 7) + 1));
        const float delta = (h & 0x8000u) ? -0.125f : 0.125f;
        const uint8_t *qs = b + 2 + 4 * p;
        for (int l = 0; l < 4; l++) {
            const uint64_t row = sepia_iq1s_grid[qs[l] | (((h >> (3 * l)) & 7) << 8)];
            for (int j = 0; j < 8; j++)
                y[8 * l + j] = __fmul_rn(dl, __fadd_rn((float)(int8_t)((row >> (8 * j)) & 255), delta));
        }
        break;
    }
    case T_IQ4_XS: {
        const float d = cvt16<HW>(rd16(b));
        const uint32_t sh = rd16(b + 2);
        const int ls = ((b[4 + (p >> 1)] >> (4 * (p & 1))) & 15) | (((sh >> (2 * p)) & 3) << 4);
        const float dl = __fmul_rn(d, (float)(ls - 32));
        const uint8_t *qs = b + 8 + 16 * p;
        for (int j = 0; j < 16; j++) {
            y[j] = __fmul_rn(dl, (float)sepia_kvalues_iq4nl[qs[j] & 15]);
            y[16 + j] = __fmul_rn(dl, (float)sepia_kvalues_iq4nl[qs[j] >> 4]);
        }
        break;
    }
    default:
        for (int i = 0; i < 32; i++) y[i] = 0.0f;
    }
}


}  // namespace sepia
