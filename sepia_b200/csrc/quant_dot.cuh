// sepia_b200/csrc/quant_dot.cuh -- per-lane dot products of one 32-element
// part of a quantized row with the activations the lane holds in registers.
//
// Exact products without integer->float conversions
// ---------------------------------------------------
// An unpacked quant field v (2-4 bits) that sits at bit position P of a
// 32-bit word, with every other bit cleared, IS the IEEE single whose value
// is v * 2^(P-149) (a subnormal: exponent field zero, the field inside the
// mantissa). So one LOP3 (mask in place) turns packed bits into an exact
// float, and FFMA(field, x * 2^(125-P-e), acc) adds exactly v * x * 2^-(24+e)
// -- the same rounding as a plain fp32 dot of the dequantized integer with x.
// The lane pre-scales its activations once per kernel ("scaled" XPart):
// element i (byte i%4 of a packed word) is scaled for the field position
// P = {4, 12, 20, 20}[i%4], and e is the exponent of the part's largest |x|
// (clamped to [-2, 100]) so nothing overflows or underflows. Products come
// out in units of 2^-(24+e); `inv` restores them. This relies on subnormal
// FMA inputs being honoured (no -ftz / fast-math), the nvcc default.
// Q2_K, Q3_K and Q4_K use it; the other formats decode each part to floats
// exactly (decode_part_exact) and use unscaled activations.
#pragma once
#include "quant_formats.cuh"

namespace sepia {

__host__ __device__ constexpr bool fast_format(int t) { return t == T_Q2_K || t == T_Q3_K || t == T_Q4_K; }

struct XPart {
    float v[32];    // activations (scaled for the fast formats)
    float s16[2];   // unscaled sums of elements 0..15 and 16..31
    float inv;      // 2^(24+e): restores the scaled products (fast formats)
};

__device__ __forceinline__ float pow2f(int k) { return __int_as_float((127 + k) << 23); }

template <bool SCALED>
__device__ __forceinline__ void xpart_finish(XPart &x) {
    float a = 0.f, b = 0.f, m = 0.f;
#pragma unroll
    for (int i = 0; i < 16; i++) {
        a += x.v[i];
        b += x.v[16 + i];
        m = fmaxf(m, fmaxf(fabsf(x.v[i]), fabsf(x.v[16 + i])));
    }
    x.s16[0] = a;
    x.s16[1] = b;
    if constexpr (SCALED) {
        int e = (m > 0.f) ? ((__float_as_int(m) >> 23) & 0xFF) - 127 : 0;
        e = max(-2, min(e, 100));
        x.inv = pow2f(24 + e);
        const float s0 = pow2f(125 - 4 - e), s1 = pow2f(125 - 12 - e), s2 = pow2f(125 - 20 - e);
#pragma unroll
        for (int i = 0; i < 32; i++) x.v[i] *= ((i & 3) == 0) ? s0 : (((i & 3) == 1) ? s1 : s2);
    } else {
        x.inv = 1.0f;
    }
}

// 8 consecutive 32-bit words at p: plain word loads when 4-byte aligned,
// otherwise aligned loads + funnel shifts (blocks of 110/210/66/... bytes).
__device__ __forceinline__ void rd8w(const uint8_t *p, uint32_t (&w)[8]) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    const uint32_t *base = reinterpret_cast<const uint32_t *>(a & ~(uintptr_t)3);
    if ((a & 3) == 0) {
#pragma unroll
        for (int i = 0; i < 8; i++) w[i] = base[i];
    } else {
        const uint32_t sh = (uint32_t)(a & 3) * 8;
        uint32_t prev = base[0];
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const uint32_t next = base[i + 1];
            w[i] = __funnelshift_r(prev, next, sh);
            prev = next;
        }
    }
}

__device__ __forceinline__ float fbits(uint32_t u) { return __uint_as_float(u); }

// exact small-integer -> float (n < 2^23) without the slow conversion pipe
__device__ __forceinline__ float u2f_small(uint32_t n) { return __uint_as_float(0x4B000000u | n) - 8388608.0f; }

// ------------------------------------------------------------ Q2_K
// part p: 32 consecutive qs bytes (half p>>2), 2-bit field at shift
// s = 2(p&3); two 16-element groups with (scale, min) nibbles.
__device__ __forceinline__ float dot_q2_k(const uint8_t *b, int p, const XPart &x) {
    const float d = cvt16<true>(rd16(b + 80)), dmin = cvt16<true>(rd16(b + 82));
    const uint32_t rot = (uint32_t)(4 - 2 * (p & 3)) & 31u;     // field -> bits 4..5 of each byte
    uint32_t w[8];
    rd8w(b + 16 + 32 * (p >> 2), w);
    const uint32_t scw = rd16(b + 2 * p);
    float acc = 0.f;
#pragma unroll
    for (int g = 0; g < 2; g++) {
        float s0 = 0.f, s1 = 0.f;
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const uint32_t t = __funnelshift_l(w[4 * g + k], w[4 * g + k], rot);
            const float *xv = x.v + 16 * g + 4 * k;
            s0 = fmaf(fbits(t & 0x00000030u), xv[0], s0);
            s1 = fmaf(fbits(t & 0x00003000u), xv[1], s1);
            s0 = fmaf(fbits(t & 0x00300000u), xv[2], s0);
            s1 = fmaf(fbits((t >> 8) & 0x00300000u), xv[3], s1);
        }
        const uint32_t sc = (scw >> (8 * g)) & 255u;
        const float dl = d * u2f_small(sc & 15u), ml = dmin * u2f_small(sc >> 4);
        acc = fmaf(dl * x.inv, s0 + s1, acc);
        acc = fmaf(-ml, x.s16[g], acc);
    }
    return acc;
}

// ------------------------------------------------------------ Q3_K
// u = q2 + 4*hbit in 0..7 packed at bits 4..6 of each byte; value = u - 4.
__device__ __forceinline__ float dot_q3_k(const uint8_t *b, int p, const XPart &x) {
    const float d = cvt16<true>(rd16(b + 108));
    const uint32_t rot = (uint32_t)(4 - 2 * (p & 3)) & 31u;     // q2 field -> bits 4..5
    const uint32_t hrot = (uint32_t)(6 - p) & 31u;              // hmask bit p -> bit 6
    uint32_t w[8], h[8];
    rd8w(b + 32 + 32 * (p >> 2), w);
    rd8w(b, h);
    float acc = 0.f;
#pragma unroll
    for (int g = 0; g < 2; g++) {
        float s0 = 0.f, s1 = 0.f;
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const uint32_t u = (__funnelshift_l(w[4 * g + k], w[4 * g + k], rot) & 0x30303030u) |
                               (__funnelshift_l(h[4 * g + k], h[4 * g + k], hrot) & 0x40404040u);
            const float *xv = x.v + 16 * g + 4 * k;
            s0 = fmaf(fbits(u & 0x00000070u), xv[0], s0);
            s1 = fmaf(fbits(u & 0x00007000u), xv[1], s1);
            s0 = fmaf(fbits(u & 0x00700000u), xv[2], s0);
            s1 = fmaf(fbits((u >> 8) & 0x00700000u), xv[3], s1);
        }
        const float dl = d * (float)q3k_scale(b + 96, 2 * p + g);
        // sum(v x) = sum(u x) - 4 X
        acc = fmaf(dl, fmaf(s0 + s1, x.inv, -4.0f * x.s16[g]), acc);
    }
    return acc;
}

// ------------------------------------------------------------ Q4_K
// nibble (p&1) of 32 qs bytes; nibbles land at bits {0, 8, 16, 16}, the
// scaled activations' {4, 12, 20, 20} minus 4, so products carry 2^-4.
__device__ __forceinline__ float dot_q4_k(const uint8_t *b, int p, const XPart &x) {
    const float d = cvt16<true>(rd16(b)), dmin = cvt16<true>(rd16(b + 2));
    int s, m;
    kscale_pair(b + 4, p, s, m);
    const uint32_t sh = (uint32_t)(p & 1) * 4u;
    uint32_t w[8];
    rd8w(b + 16 + 32 * (p >> 1), w);
    float s0 = 0.f, s1 = 0.f;
#pragma unroll
    for (int k = 0; k < 8; k++) {
        const uint32_t t = w[k] >> sh;
        const float *xv = x.v + 4 * k;
        s0 = fmaf(fbits(t & 0x0000000Fu), xv[0], s0);
        s1 = fmaf(fbits(t & 0x00000F00u), xv[1], s1);
        s0 = fmaf(fbits(t & 0x000F0000u), xv[2], s0);
        s1 = fmaf(fbits((t >> 8) & 0x000F0000u), xv[3], s1);
    }
    const float dl = d * u2f_small((uint32_t)s), ml = dmin * u2f_small((uint32_t)m);
    return fmaf(dl * (x.inv * 16.0f), s0 + s1, -ml * (x.s16[0] + x.s16[1]));
}

// ------------------------------------------------------------ IQ codebook formats
// Codebook formats with unscaled activations: each grid byte v (0..255)
// becomes the exact float 2^23 + v by one byte permute with the exponent
// byte 0x4B, and one subtraction; signs flip the activation's sign bit. The
// part's 32 products sum in fp32 (relative error ~1e-7, far inside the
// 1e-4 parity bound) and the part scale multiplies once.
__device__ __forceinline__ float grid_byte_f(uint32_t w, int j) {
    return __uint_as_float(__byte_perm(w, 0x4B000000u, (uint32_t)j | 0x7650u)) - 8388608.0f;
}
__device__ __forceinline__ float flip_if(float x, uint32_t s, int j) {
    return __int_as_float(__float_as_int(x) ^ (int)((s << (31 - j)) & 0x80000000u));
}

// gguf IQ2_XXS: per 32 elements idx (4 grid rows of 8 bytes), signs and a
// 4-bit scale: db = d * (0.5 + s) * 0.25 (src decode: decode_part_exact).
__device__ __forceinline__ float dot_iq2_xxs(const uint8_t *b, int p, const XPart &x) {
    const float d = cvt16<true>(rd16(b));
    const uint32_t idx = rd32(b + 2 + 8 * p), sg = rd32(b + 6 + 8 * p);
    const float db = __fmul_rn(__fmul_rn(d, __fadd_rn(0.5f, (float)(sg >> 28))), 0.25f);
    float t0 = 0.f, t1 = 0.f;
#pragma unroll
    for (int l = 0; l < 4; l++) {
        const uint64_t row = sepia_iq2xxs_grid[(idx >> (8 * l)) & 255];
        const uint32_t s = sepia_ksigns_iq2xs[(sg >> (7 * l)) & 127];
        const uint32_t lo = (uint32_t)row, hi = (uint32_t)(row >> 32);
        const float *xv = x.v + 8 * l;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            t0 = fmaf(grid_byte_f(lo, j), flip_if(xv[j], s, j), t0);
            t1 = fmaf(grid_byte_f(hi, j), flip_if(xv[4 + j], s, 4 + j), t1);
        }
    }
    return db * (t0 + t1);
}

// gguf IQ2_XS: per 8 elements a 16-bit word (9-bit grid row, 7-bit sign
// index); 4-bit scales per 16 elements.
__device__ __forceinline__ float dot_iq2_xs(const uint8_t *b, int p, const XPart &x) {
    const float d = cvt16<true>(rd16(b));
    const int sc = b[66 + p];
    const float db0 = __fmul_rn(__fmul_rn(d, __fadd_rn(0.5f, (float)(sc & 15))), 0.25f);
    const float db1 = __fmul_rn(__fmul_rn(d, __fadd_rn(0.5f, (float)(sc >> 4))), 0.25f);
    float t[2] = {0.f, 0.f};
#pragma unroll
    for (int l = 0; l < 4; l++) {
        const uint32_t q = rd16(b + 2 + 2 * (4 * p + l));
        const uint64_t row = sepia_iq2xs_grid[q & 511];
        const uint32_t s = sepia_ksigns_iq2xs[q >> 9];
        const uint32_t lo = (uint32_t)row, hi = (uint32_t)(row >> 32);
        const float *xv = x.v + 8 * l;
        float a = 0.f;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            a = fmaf(grid_byte_f(lo, j), flip_if(xv[j], s, j), a);
            a = fmaf(grid_byte_f(hi, j), flip_if(xv[4 + j], s, 4 + j), a);
        }
        t[l >> 1] += a;
    }
    return fmaf(db0, t[0], db1 * t[1]);
}

// gguf IQ3_XXS: per 8 elements two 4-byte grid rows and a sign index;
// db = d * (0.5 + s) * 0.5.
__device__ __forceinline__ float dot_iq3_xxs(const uint8_t *b, int p, const XPart &x) {
    const float d = cvt16<true>(rd16(b));
    const uint32_t a = rd32(b + 66 + 4 * p);
    const float db = __fmul_rn(__fmul_rn(d, __fadd_rn(0.5f, (float)(a >> 28))), 0.5f);
    const uint8_t *qs = b + 2 + 8 * p;
    float t0 = 0.f, t1 = 0.f;
#pragma unroll
    for (int l = 0; l < 4; l++) {
        const uint32_t s = sepia_ksigns_iq2xs[(a >> (7 * l)) & 127];
        const uint32_t g1 = sepia_iq3xxs_grid[qs[2 * l]], g2 = sepia_iq3xxs_grid[qs[2 * l + 1]];
        const float *xv = x.v + 8 * l;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            t0 = fmaf(grid_byte_f(g1, j), flip_if(xv[j], s, j), t0);
            t1 = fmaf(grid_byte_f(g2, j), flip_if(xv[4 + j], s, 4 + j), t1);
        }
    }
    return db * (t0 + t1);
}

// gguf IQ1_S: grid bytes g in {-1, 0, 1}, value dl * (g + delta). The
// bytewise u = g + 1 in {0, 1, 2} (carry-free) becomes the float g exactly
// as (2^23 + u) - (2^23 + 1); sum (g + delta) x = sum g x + delta * sum x
// (summing g x directly: no cancellation against sum x).
__device__ __forceinline__ uint32_t plus1_bytes(uint32_t w) {
    return ((w & 0x7F7F7F7Fu) + 0x01010101u) ^ (w & 0x80808080u);
}
__device__ __forceinline__ float grid_g_f(uint32_t u, int j) {
    return __uint_as_float(__byte_perm(u, 0x4B000000u, (uint32_t)j | 0x7650u)) - 8388609.0f;
}
__device__ __forceinline__ float dot_iq1_s(const uint8_t *b, int p, const XPart &x) {
    const float d = cvt16<true>(rd16(b));
    const uint32_t h = rd16(b + 34 + 2 * p);
    const float dl = __fmul_rn(d, (float)(2 * ((h >> 12) & 7) + 1));
    const float delta = (h & 0x8000u) ? -0.125f : 0.125f;
    const uint8_t *qs = b + 2 + 4 * p;
    float t0 = 0.f, t1 = 0.f;
#pragma unroll
    for (int l = 0; l < 4; l++) {
        const uint64_t row = sepia_iq1s_grid[qs[l] | (((h >> (3 * l)) & 7) << 8)];
        const uint32_t lo = plus1_bytes((uint32_t)row), hi = plus1_bytes((uint32_t)(row >> 32));
        const float *xv = x.v + 8 * l;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            t0 = fmaf(grid_g_f(lo, j), xv[j], t0);
            t1 = fmaf(grid_g_f(hi, j), xv[4 + j], t1);
        }
    }
    return dl * fmaf(delta, x.s16[0] + x.s16[1], t0 + t1);
}

// ------------------------------------------------------------ generic
__device__ __forceinline__ float dot_generic(int t, const uint8_t *b, int p, const XPart &x, int n_valid) {
    float y[32];
    decode_part_exact<true>(t, b, p, y, n_valid);
    // fp64 accumulation: the part's sum rounds once (the reference
    // double-accumulates its dot, src/sepia.c:731-735)
    double s0 = 0.0, s1 = 0.0;
#pragma unroll
    for (int i = 0; i < 32; i += 2) {
        s0 = fma(i < n_valid ? (double)y[i] : 0.0, (double)x.v[i], s0);
        s1 = fma(i + 1 < n_valid ? (double)y[i + 1] : 0.0, (double)x.v[i + 1], s1);
    }
    return (float)(s0 + s1);
}

// Dot of part p for a compile-time format: the fast decoders expect scaled
// activations (load with SCALED = fast_format(T)), the others unscaled.
template <int T>
__device__ __forceinline__ float dot_part(const uint8_t *b, int p, const XPart &x, int n_valid) {
    if constexpr (T == T_Q2_K) return dot_q2_k(b, p, x);
    else if constexpr (T == T_Q3_K) return dot_q3_k(b, p, x);
    else if constexpr (T == T_Q4_K) return dot_q4_k(b, p, x);
    else if constexpr (T == T_IQ2_XXS) return dot_iq2_xxs(b, p, x);
    else if constexpr (T == T_IQ1_S) return dot_iq1_s(b, p, x);
    else if constexpr (T == T_IQ2_XS) return dot_iq2_xs(b, p, x);
    else if constexpr (T == T_IQ3_XXS) return dot_iq3_xxs(b, p, x);
    else return dot_generic(T, b, p, x, n_valid);
}

}  // namespace sepia
