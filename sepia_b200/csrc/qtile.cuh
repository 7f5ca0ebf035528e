// sepia_b200/csrc/qtile.cuh -- exact quantized dot products on the integer
// tensor cores, one 16-row tile and one 256-element superblock at a time.
//
// Why: a batch-1 GEMV over 2-4 bit weights is HBM-bound only if unpacking
// costs about one instruction per weight. Decoding to floats and running
// FMAs costs 3-7, so such a kernel is issue-bound far below the HBM
// roofline. Here the packed fields are unpacked to 8-bit integers with a few
// bit operations per 4 weights and the multiply-accumulate runs on the
// tensor cores (mma.sync m16n8k32 / m16n8k16, u8 or s8 x s8 -> s32).
//
// Exactness: each superblock's 256 activations are written as integers
// x_int = round(x * 2^(kXShift - e)), e = exponent of the superblock's
// largest |x|, split into four balanced base-256 digits ("limbs", signed
// bytes). The tensor core forms sum_k w_int[k] * limb_j[k] exactly in int32
// for each limb j (MMA columns), and the limbs recombine exactly in fp64, so
// a superblock's dot product is exact; only x's representation rounds, at
// 2^-(kXShift+1) of the superblock's largest value. Scales and mins enter as
// small integers (folded into the A operand, applied to the int32 partials
// with IMAD, or as a second MMA over group sums), and the fp16 superblock
// scales multiply once per superblock in fp64.
//
// Fragment layouts (lane = 4*gid + tig), m16n8k32:
//   A (16 x 32): a0 = row gid,   k 4tig..+3      a1 = row gid+8, same k
//                a2 = row gid,   k 16+4tig..+3   a3 = row gid+8, same k
//   B (32 x 8):  b0 = k 4tig..+3, col gid        b1 = k 16+4tig..+3, col gid
//   C (16 x 8):  c0 = (gid, 2tig) c1 = (gid, 2tig+1) c2 = (gid+8, 2tig) c3 = (gid+8, 2tig+1)
// m16n8k16 uses only a0/a1 and b0. A part's k32 MMA pairs hardware k with
// the part's elements so that each lane's 8 elements are consecutive: k
// 4tig+i <-> element 8tig+i, k 16+4tig+i <-> element 8tig+4+i (A and B
// alike). Lanes tig 0,1 thus hold elements 0-15 (one 16-element group),
// lanes tig 2,3 elements 16-31, and one scale serves both A registers.
//
// Two B arrangements come from one table entry e = (b0, b1) of limb gid&3:
//   natural: columns 0-3 = limbs 0-3 of the whole part (gid >= 4: zero);
//   split:   columns 0-3 = limbs of elements 0-15 only, columns 4-7 = limbs
//            of elements 16-31 only (B of lanes tig 0,1 kept for gid < 4,
//            of lanes tig 2,3 for gid >= 4), so one MMA yields the two
//            16-element groups' dots separately (C lanes tig 0,1: first
//            group; tig 2,3: second group) -- used where a per-group scale
//            cannot be folded into A.
// Either way lane tig's two C columns are limbs 2(tig&1) and 2(tig&1)+1, of
// weight 256^(2(tig&1)) and 256^(2(tig&1)+1).
#pragma once
#include "quant_formats.cuh"

namespace sepia {

constexpr int kXShift = 29;      // x_int = round(x * 2^(kXShift - e)), |x_int| <= 2^30
constexpr int kTabSB = 1296;     // activation-table bytes per superblock (16-byte multiple)
// Table entry of one superblock:
//   [0, 1024)     uint2 b[8 parts][tig*4 + limb]      natural k32 B fragments (4 limbs)
//   [1024, 1152)  uint32 g16[tig*8 + limb]            k16 B fragments of the 16 group sums
//   [1152, 1280)  uint32 g32[tig*8 + limb]            k16 B fragments of the 8 part sums
//   [1280, 1284)  float unit = 2^(e - kXShift)        value of one x_int unit
// Group and part sums reach 2^35 and take 5 limbs (columns 0-4 of a k16
// MMA; columns 5-7 are zero).
constexpr int kTabG16 = 1024, kTabG32 = 1152, kTabUnit = 1280;

// Five balanced base-256 digits of v (|v| < 2^38).
__device__ __forceinline__ void limbs5(long long v, int (&d)[5]) {
#pragma unroll
    for (int j = 0; j < 4; j++) {
        const int lo = (int)((v + 128) & 255) - 128;
        d[j] = lo;
        v = (v - lo) >> 8;
    }
    d[4] = (int)v;
}

// Table entry of one superblock, in two steps so that a warp can issue the
// loads of several superblocks before it computes any. Lane l owns part
// l/4 and tig l%4: positions 32*part + 8*tig + {0..7} of the superblock.
// CG: read through L2 only (x was written by another grid or other CTAs).
template <bool CG = false>
__device__ __forceinline__ void xtab_load(const float *xsb, int lane, float (&v)[8]) {
    const float *xs = xsb + 32 * (lane >> 2) + 8 * (lane & 3);
    if ((reinterpret_cast<uintptr_t>(xs) & 15) == 0) {
        const float4 lo = CG ? __ldcg(reinterpret_cast<const float4 *>(xs)) : *reinterpret_cast<const float4 *>(xs);
        const float4 hi =
            CG ? __ldcg(reinterpret_cast<const float4 *>(xs + 4)) : *reinterpret_cast<const float4 *>(xs + 4);
        v[0] = lo.x; v[1] = lo.y; v[2] = lo.z; v[3] = lo.w;
        v[4] = hi.x; v[5] = hi.y; v[6] = hi.z; v[7] = hi.w;
    } else {
#pragma unroll
        for (int j = 0; j < 8; j++) v[j] = CG ? __ldcg(xs + j) : xs[j];
    }
}

__device__ inline void xtab_emit(uint8_t *te, const float (&v)[8], int lane) {
    const int part = lane >> 2, tig = lane & 3;
    float m = 0.f;
#pragma unroll
    for (int j = 0; j < 8; j++) m = fmaxf(m, fabsf(v[j]));
    m = warp_max(m);
    int e = (m > 0.f) ? ((__float_as_int(m) >> 23) & 0xFF) - 127 : 0;
    e = max(-90, min(e, 90));
    const float scale = __int_as_float((127 + kXShift - e) << 23);
    // Balanced base-256 digits by one biased add: u = xi + 0x808080 has
    // bytes 0-2 equal to d_j + 128 (each digit in [-128, 127]) and byte 3
    // equal to d3 (|xi| <= 2^30), so each limb byte is a byte of u, the low
    // three with the bias bit flipped (d + 128 -> d as a signed byte). A
    // 4 x 4 byte transpose (8 prmt) turns the u of 4 elements into the 4
    // limb words of those elements.
    int xi[8];
    uint32_t wl[2][4];
#pragma unroll
    for (int hq = 0; hq < 2; hq++) {
        uint32_t u[4];
#pragma unroll
        for (int j = 0; j < 4; j++) {
            xi[4 * hq + j] = __float2int_rn(v[4 * hq + j] * scale);
            u[j] = (uint32_t)xi[4 * hq + j] + 0x808080u;
        }
        const uint32_t t01l = __byte_perm(u[0], u[1], 0x5140), t01h = __byte_perm(u[0], u[1], 0x7362);
        const uint32_t t23l = __byte_perm(u[2], u[3], 0x5140), t23h = __byte_perm(u[2], u[3], 0x7362);
        wl[hq][0] = __byte_perm(t01l, t23l, 0x5410) ^ 0x80808080u;
        wl[hq][1] = __byte_perm(t01l, t23l, 0x7632) ^ 0x80808080u;
        wl[hq][2] = __byte_perm(t01h, t23h, 0x5410) ^ 0x80808080u;
        wl[hq][3] = __byte_perm(t01h, t23h, 0x7632);
    }
    uint2 *bd = reinterpret_cast<uint2 *>(te) + part * 16 + tig * 4;
#pragma unroll
    for (int l = 0; l < 4; l++) bd[l] = make_uint2(wl[0][l], wl[1][l]);
    // group sums: group 2*part = elements 0-15 of the part (lanes tig
    // 0,1), group 2*part+1 = elements 16-31 (lanes tig 2,3)
    long long gs = 0;
#pragma unroll
    for (int j = 0; j < 8; j++) gs += xi[j];
    gs += __shfl_xor_sync(0xffffffffu, gs, 1);
    const long long g0 = gs, g1 = __shfl_xor_sync(0xffffffffu, gs, 2);
    // k16 fragment words: lane (gid = limb, t) holds k = 4t..4t+3
    uint8_t *g16 = te + kTabG16, *g32 = te + kTabG32;
    if (tig == 0) {
        int d0[5], d1[5], dp[5];
        limbs5(g0, d0);
        limbs5(g1, d1);
        limbs5(g0 + g1, dp);
#pragma unroll
        for (int l = 0; l < 5; l++) {
            // groups 2p, 2p+1 -> word t = p/2, bytes 2(p&1), 2(p&1)+1
            uint8_t *wp = g16 + 4 * ((part >> 1) * 8 + l);
            wp[2 * (part & 1)] = (uint8_t)(d0[l] & 255);
            wp[2 * (part & 1) + 1] = (uint8_t)(d1[l] & 255);
            // part p -> word t = p/4, byte p&3 (k 8..15 are zero)
            g32[4 * ((part >> 2) * 8 + l) + (part & 3)] = (uint8_t)(dp[l] & 255);
        }
    }
    // zero words: limbs 5-7 everywhere, and k 8..15 of the part sums
    if (lane < 12) {
        const int t = lane / 3, l = 5 + lane % 3;
        reinterpret_cast<uint32_t *>(g16)[t * 8 + l] = 0u;
        reinterpret_cast<uint32_t *>(g32)[t * 8 + l] = 0u;
    } else if (lane < 28) {
        const int t = 2 + (lane - 12) / 8, l = (lane - 12) % 8;
        reinterpret_cast<uint32_t *>(g32)[t * 8 + l] = 0u;
    }
    if (lane == 0) *reinterpret_cast<float *>(te + kTabUnit) = __int_as_float((127 - kXShift + e) << 23);
}

// Build the table entries of x[0 .. nsb*256) into tab (shared or global
// memory), one warp per superblock (x at least 4-byte aligned).
template <bool CG = false>
__device__ inline void xtab_build(uint8_t *tab, const float *x, int nsb, int warp, int nwarps, int lane) {
    for (int sb = warp; sb < nsb; sb += nwarps) {
        float v[8];
        xtab_load<CG>(x + (size_t)sb * kQK, lane, v);
        xtab_emit(tab + (size_t)sb * kTabSB, v, lane);
    }
}

// ------------------------------------------------------------ MMA wrappers
__device__ __forceinline__ void mma_k32(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                        uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
// C = A.B (no accumulator input)
__device__ __forceinline__ void mma_k32_z(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%10,%10,%10};\n"
        : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}
__device__ __forceinline__ void mma_k16(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%0,%1,%2,%3};\n"
        : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
        : "r"(a0), "r"(a1), "r"(b0));
}
__device__ __forceinline__ void mma_k16_ss(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%0,%1,%2,%3};\n"
        : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
        : "r"(a0), "r"(a1), "r"(b0));
}

// byte j of w as a 32-bit integer
__device__ __forceinline__ uint32_t byte_of(uint32_t w, int j) { return __byte_perm(w, 0u, 0x4440u + j); }
__device__ __forceinline__ uint32_t ldw(const uint8_t *p) { return *reinterpret_cast<const uint32_t *>(p); }

// Per-lane constants of a tile walk.
struct LaneCtx {
    int gid, tig;
    uint32_t boff;       // byte offset of the lane's B entry in a part's 128 bytes
    uint32_t goff;       // byte offset of the lane's k16 group-sum B word
    uint32_t msplit;     // split layout: keep this lane's B (its group matches its columns)
    uint32_t mlo;        // columns 0-3 only
    float lwn;           // natural layout: weight of the lane's first limb column (0 for tig 2,3)
    float lws;           // split layout: same, every lane
    float lwg;           // group-sum MMAs (8 limb columns): 256^(2 tig)
    uint32_t bsel;       // byte_perm selector of the lane's group scale byte (group 2p + tig/2)
    uint32_t ssel0, ssel1;   // prmt selectors: byte tig/2 (resp. 2 + tig/2), sign-extended
    int unit_off;            // two-vector units: from the lane's B table to its C columns' table
};
__device__ __forceinline__ LaneCtx lane_ctx(int lane) {
    LaneCtx L;
    L.gid = lane >> 2;
    L.tig = lane & 3;
    // columns 4-7 read the entries of limbs 0-3 again: in the natural layout
    // their results (lanes tig 2,3) are duplicates and get weight 0
    L.boff = (uint32_t)(L.tig * 4 + (L.gid & 3)) * 8u;
    L.goff = (uint32_t)(L.tig * 8 + L.gid) * 4u;
    L.msplit = ((L.gid < 4) == (L.tig < 2)) ? 0xFFFFFFFFu : 0u;
    L.mlo = (L.gid < 4) ? 0xFFFFFFFFu : 0u;
    L.lws = (L.tig & 1) ? 65536.0f : 1.0f;
    L.lwn = (L.tig < 2) ? L.lws : 0.0f;
    L.lwg = (L.tig == 0) ? 1.0f : (L.tig == 1) ? 65536.0f : (L.tig == 2) ? 4294967296.0f : 0.0f;
    L.bsel = 0x4440u + (uint32_t)(L.tig >> 1);
    const uint32_t j0 = (uint32_t)(L.tig >> 1), j1 = j0 + 2;
    L.ssel0 = j0 | ((j0 | 8) << 4) | ((j0 | 8) << 8) | ((j0 | 8) << 12);
    L.ssel1 = j1 | ((j1 | 8) << 4) | ((j1 | 8) << 8) | ((j1 | 8) << 12);
    L.unit_off = 0;
    return L;
}

__device__ __forceinline__ uint2 ld_b(const uint8_t *te, int p, const LaneCtx &C) {
    return *reinterpret_cast<const uint2 *>(te + p * 128 + C.boff);
}
__device__ __forceinline__ uint32_t ld_g(const uint8_t *te, int off, const LaneCtx &C) {
    return *reinterpret_cast<const uint32_t *>(te + off + C.goff);
}
__device__ __forceinline__ float ld_unit(const uint8_t *te) { return *reinterpret_cast<const float *>(te + kTabUnit); }

// byte j of w sign-extended to 32 bits (prmt with the sign-replicate bit
// set in the selector nibbles of bytes 1-3)
__device__ __forceinline__ int sbyte_of(uint32_t w, int j) {
    int r;
    asm("prmt.b32 %0, %1, 0, %2;" : "=r"(r) : "r"(w), "r"((uint32_t)(j | ((j | 8) << 4) | ((j | 8) << 8) | ((j | 8) << 12))));
    return r;
}

// exact value of the lane's two limb columns: (lo + 256 hi) * lw
__device__ __forceinline__ double limb_pair(int lo, int hi, float lw) {
    return ((double)lo + 256.0 * (double)hi) * (double)lw;
}

// ------------------------------------------------------------------ Q2_K
// 84-byte superblock: scales[16] (low nibble scale, high nibble min of each
// 16-element group), qs[64], d, dmin (fp16). Element 128h + 32s + l is the
// 2-bit field at shift 2s of qs[32h + l] (src/quants.c dequantize_row_q2_K).
// The scale nibble multiplies the field inside A (product <= 180 fits u8);
// fields at odd s are masked in place (x4) and accumulated separately.
__device__ __forceinline__ void sb_q2k(const uint8_t *bg, const uint8_t *bg8, const uint8_t *te, const LaneCtx &C,
                                       double &yg, double &yg8) {
    const int tig = C.tig;
    uint32_t sl[4], sl8[4];
#pragma unroll
    for (int j = 0; j < 4; j++) {
        sl[j] = ldw(bg + 4 * j) & 0x0F0F0F0Fu;
        sl8[j] = ldw(bg8 + 4 * j) & 0x0F0F0F0Fu;
    }
    int c[4] = {0, 0, 0, 0}, c2[4] = {0, 0, 0, 0};
#pragma unroll
    for (int h = 0; h < 2; h++) {
        const uint8_t *q = bg + 16 + 32 * h, *q8 = bg8 + 16 + 32 * h;
        const uint32_t w[4] = {ldw(q + 8 * tig), ldw(q8 + 8 * tig), ldw(q + 8 * tig + 4), ldw(q8 + 8 * tig + 4)};
        uint32_t w4[4];
#pragma unroll
        for (int r = 0; r < 4; r++) w4[r] = w[r] >> 4;
#pragma unroll
        for (int s = 0; s < 4; s++) {
            const int p = 4 * h + s;                                   // this lane's group: 2p + tig/2
            const uint32_t m = (s & 1) ? 0x0C0C0C0Cu : 0x03030303u;
            const uint32_t *src = (s < 2) ? w : w4;
            const uint2 b = ld_b(te, p, C);
            const uint32_t sc = __byte_perm(sl[p >> 1], 0u, C.bsel + 2 * (p & 1));
            const uint32_t sc8 = __byte_perm(sl8[p >> 1], 0u, C.bsel + 2 * (p & 1));
            const uint32_t a0 = (src[0] & m) * sc, a1 = (src[1] & m) * sc8;
            const uint32_t a2 = (src[2] & m) * sc, a3 = (src[3] & m) * sc8;
            if (s & 1) mma_k32(c2, a0, a1, a2, a3, b.x, b.y);
            else mma_k32(c, a0, a1, a2, a3, b.x, b.y);
        }
    }
    // min term: A = the 16 min nibbles per row, B = group sums
    int cm[4] = {0, 0, 0, 0};
    mma_k16(cm, (ldw(bg + 4 * tig) >> 4) & 0x0F0F0F0Fu, (ldw(bg8 + 4 * tig) >> 4) & 0x0F0F0F0Fu,
            ld_g(te, kTabG16, C));
    // |c| < 2^21: the int pairs below cannot overflow
    const int ia = (c[0] + (c2[0] >> 2)) + 256 * (c[1] + (c2[1] >> 2));
    const int ia8 = (c[2] + (c2[2] >> 2)) + 256 * (c[3] + (c2[3] >> 2));
    const int im = cm[0] + 256 * cm[1], im8 = cm[2] + 256 * cm[3];
    const uint32_t dd = ldw(bg + 80), dd8 = ldw(bg8 + 80);
    const float un = ld_unit(te);
    const float u = un * C.lwn, ug = un * C.lwg;
    yg += (double)(cvt16<true>(dd & 0xFFFFu) * u) * (double)ia - (double)(cvt16<true>(dd >> 16) * ug) * (double)im;
    yg8 += (double)(cvt16<true>(dd8 & 0xFFFFu) * u) * (double)ia8 - (double)(cvt16<true>(dd8 >> 16) * ug) * (double)im8;
}

// ------------------------------------------------------------------ Q3_K
// 110-byte superblock: hmask[32], qs[64], scales[12], d (fp16). Element
// 128h + 32s + l: u = ((qs[32h+l] >> 2s) & 3) | (bit p of hmask[l]) << 2,
// p = 4h + s; value = u - 4; group g = 2p + (l >= 16) has the signed 6-bit
// scale s_g (src/quants.c dequantize_row_q3_K). A holds u (unsigned, odd s
// in place x4); the split B layout gives per-group partials C_g, scaled by
// s_g with IMAD; the -4 offset is -4 * sum_g s_g G_g, one s8 x s8 k16 MMA
// over the group sums G_g.
// A 110-byte superblock at an odd index of a row sits 2 bytes off a 4-byte
// boundary; its words are assembled from the two aligned words around them.
template <bool ODD>
__device__ __forceinline__ uint32_t ldw2(const uint8_t *p) {
    if constexpr (ODD) return __byte_perm(ldw(p - 2), ldw(p + 2), 0x5432);
    else return ldw(p);
}

// prmt of w with a precomputed selector (sign-extending byte select)
__device__ __forceinline__ int prmt_sel(uint32_t w, uint32_t sel) {
    int r;
    asm("prmt.b32 %0, %1, 0, %2;" : "=r"(r) : "r"(w), "r"(sel));
    return r;
}

// Signed scales (sc - 32) of groups 4i..4i+3 as the bytes of one word, for
// i = tig: each lane of a quad unpacks one of the four words of its row.
template <bool ODD>
__device__ __forceinline__ uint32_t q3k_scale_word(const uint8_t *sc, int tig) {
    const uint32_t Sa = ldw2<ODD>(sc + 4 * (tig & 1)), S2 = ldw2<ODD>(sc + 8);
    const uint32_t U = ((Sa >> (2 * (tig & 2))) & 0x0F0F0F0Fu) | (((S2 >> (2 * tig)) & 0x03030303u) << 4);
    // 6-bit unsigned -> signed byte (sc - 32): flip bit 5, then copy the
    // new bit 5 into bits 6 and 7
    const uint32_t t = U ^ 0x20202020u, sg = t & 0x20202020u;
    return t | (sg * 6u);
}

template <bool ODD>
__device__ __forceinline__ void sb_q3k(const uint8_t *bg, const uint8_t *bg8, const uint8_t *te, const LaneCtx &C,
                                       double &yg, double &yg8) {
    const int tig = C.tig;
    // this lane's scale word (groups 4tig..4tig+3) of rows gid and gid+8;
    // part p's scales come from quad lane p/2
    const uint32_t Gw = q3k_scale_word<ODD>(bg + 96, tig), Gw8 = q3k_scale_word<ODD>(bg8 + 96, tig);
    const int qbase = 4 * C.gid;
    const uint32_t hm[4] = {ldw2<ODD>(bg + 8 * tig), ldw2<ODD>(bg8 + 8 * tig), ldw2<ODD>(bg + 8 * tig + 4),
                            ldw2<ODD>(bg8 + 8 * tig + 4)};
    int acc[4] = {0, 0, 0, 0}, accq[4] = {0, 0, 0, 0};
#pragma unroll
    for (int h = 0; h < 2; h++) {
        const uint8_t *q = bg + 32 + 32 * h, *q8 = bg8 + 32 + 32 * h;
        const uint32_t w[4] = {ldw2<ODD>(q + 8 * tig), ldw2<ODD>(q8 + 8 * tig), ldw2<ODD>(q + 8 * tig + 4),
                               ldw2<ODD>(q8 + 8 * tig + 4)};
        uint32_t w4[4];
#pragma unroll
        for (int r = 0; r < 4; r++) w4[r] = w[r] >> 4;
        const uint32_t ga = __shfl_sync(0xffffffffu, Gw, qbase + 2 * h);
        const uint32_t gb = __shfl_sync(0xffffffffu, Gw, qbase + 2 * h + 1);
        const uint32_t ga8 = __shfl_sync(0xffffffffu, Gw8, qbase + 2 * h);
        const uint32_t gb8 = __shfl_sync(0xffffffffu, Gw8, qbase + 2 * h + 1);
#pragma unroll
        for (int s = 0; s < 4; s++) {
            const int p = 4 * h + s;
            const uint32_t qm = (s & 1) ? 0x0C0C0C0Cu : 0x03030303u;
            const int tb = (s & 1) ? 4 : 2;                 // bit that receives the high bit
            const uint32_t hmk = 0x01010101u << tb;
            const uint32_t *src = (s < 2) ? w : w4;
            uint32_t a[4];
#pragma unroll
            for (int r = 0; r < 4; r++) {
                const uint32_t hb = (tb >= p) ? (hm[r] << (tb - p)) : (hm[r] >> (p - tb));
                a[r] = (src[r] & qm) | (hb & hmk);
            }
            const uint2 e = ld_b(te, p, C);
            int cc[4];
            mma_k32_z(cc, a[0], a[1], a[2], a[3], e.x & C.msplit, e.y & C.msplit);
            // this lane's group: 2p + t
            // group 2p + t: byte 2(p&1) + t of word p/2 (= 2h + s/2)
            const uint32_t sl = (p & 1) ? C.ssel1 : C.ssel0;
            const int sg = prmt_sel((s < 2) ? ga : gb, sl);
            const int sg8 = prmt_sel((s < 2) ? ga8 : gb8, sl);
            int *ac = (s & 1) ? accq : acc;
            ac[0] += sg * cc[0];
            ac[1] += sg * cc[1];
            ac[2] += sg8 * cc[2];
            ac[3] += sg8 * cc[3];
        }
    }
    // sum_g s_g G_g: A = signed scales of groups 4tig..4tig+3, B = the group
    // sums' 5 limbs
    int cm[4] = {0, 0, 0, 0};
    {
        mma_k16_ss(cm, Gw, Gw8, ld_g(te, kTabG16, C));
    }
    const int v0 = acc[0] + (accq[0] >> 2), v1 = acc[1] + (accq[1] >> 2);
    const int v2 = acc[2] + (accq[2] >> 2), v3 = acc[3] + (accq[3] >> 2);
    const float u = ld_unit(te);
    yg += (double)(cvt16<true>(lds_u16(bg + 108)) * u) * (limb_pair(v0, v1, C.lws) - 4.0 * limb_pair(cm[0], cm[1], C.lwg));
    yg8 += (double)(cvt16<true>(lds_u16(bg8 + 108)) * u) * (limb_pair(v2, v3, C.lws) - 4.0 * limb_pair(cm[2], cm[3], C.lwg));
}

// ------------------------------------------------------------------ Q4_K
// 144-byte superblock: d, dmin (fp16), scales[12] (6-bit scale and min of
// each 32-element part), qs[128]. Part p: nibble (p&1) of qs[32(p>>1) + l]
// (src/quants.c dequantize_row_q4_K). One MMA per part into fresh
// accumulators, scaled by the part's scale with IMAD; the mins are one k16
// MMA over the part sums.
__device__ __forceinline__ void q4k_scales(const uint8_t *s, uint32_t &sc0, uint32_t &sc1, uint32_t &m0,
                                           uint32_t &m1) {
    const uint32_t W0 = ldw(s), W1 = ldw(s + 4), W2 = ldw(s + 8);
    sc0 = W0 & 0x3F3F3F3Fu;
    m0 = W1 & 0x3F3F3F3Fu;
    sc1 = (W2 & 0x0F0F0F0Fu) | ((W0 >> 2) & 0x30303030u);
    m1 = ((W2 >> 4) & 0x0F0F0F0Fu) | ((W1 >> 2) & 0x30303030u);
}

__device__ __forceinline__ void sb_q4k(const uint8_t *bg, const uint8_t *bg8, const uint8_t *te, const LaneCtx &C,
                                       double &yg, double &yg8) {
    const int tig = C.tig;
    uint32_t sc0, sc1, m0, m1, sc08, sc18, m08, m18;
    q4k_scales(bg + 4, sc0, sc1, m0, m1);
    q4k_scales(bg8 + 4, sc08, sc18, m08, m18);
    int acc[4] = {0, 0, 0, 0};
#pragma unroll
    for (int j = 0; j < 4; j++) {
        const uint8_t *q = bg + 16 + 32 * j, *q8 = bg8 + 16 + 32 * j;
        const uint32_t w[4] = {ldw(q + 8 * tig), ldw(q8 + 8 * tig), ldw(q + 8 * tig + 4), ldw(q8 + 8 * tig + 4)};
#pragma unroll
        for (int hi = 0; hi < 2; hi++) {
            const int p = 2 * j + hi;
            uint32_t a[4];
#pragma unroll
            for (int r = 0; r < 4; r++) a[r] = hi ? ((w[r] >> 4) & 0x0F0F0F0Fu) : (w[r] & 0x0F0F0F0Fu);
            const uint2 b = ld_b(te, p, C);
            int cc[4];
            mma_k32_z(cc, a[0], a[1], a[2], a[3], b.x, b.y);
            const int s = (int)byte_of(p < 4 ? sc0 : sc1, p & 3), s8 = (int)byte_of(p < 4 ? sc08 : sc18, p & 3);
            acc[0] += s * cc[0];
            acc[1] += s * cc[1];
            acc[2] += s8 * cc[2];
            acc[3] += s8 * cc[3];
        }
    }
    int cm[4] = {0, 0, 0, 0};
    {
        // k = part: lanes tig 0,1 hold parts 0-3, 4-7; k 8..15 meet zero B
        const uint32_t am = (tig == 0) ? m0 : m1;
        const uint32_t am8 = (tig == 0) ? m08 : m18;
        mma_k16(cm, am, am8, ld_g(te, kTabG32, C));
    }
    const uint32_t dd = ldw(bg), dd8 = ldw(bg8);
    const float un = ld_unit(te);
    const float u = un * C.lwn, ug = un * C.lwg;
    yg += (double)(cvt16<true>(dd & 0xFFFFu) * u) * ((double)acc[0] + 256.0 * (double)acc[1]) -
          (double)(cvt16<true>(dd >> 16) * ug) * (double)(cm[0] + 256 * cm[1]);
    yg8 += (double)(cvt16<true>(dd8 & 0xFFFFu) * u) * ((double)acc[2] + 256.0 * (double)acc[3]) -
           (double)(cvt16<true>(dd8 >> 16) * ug) * (double)(cm[2] + 256 * cm[3]);
}

// ------------------------------------------------------------ IQ formats
// Grid-codebook formats (gguf IQ2_XXS, IQ2_XS, IQ3_XXS, IQ1_S). A lane's 8
// elements of a part (8tig..8tig+7) are exactly one codebook row, so its A
// registers are that row's bytes, signed (s8 x s8 MMA): a0 / a1 the row's
// elements 0-3, a2 / a3 elements 4-7. The per-part (2s + 1) scales multiply
// each part's int32 partial (IMAD); IQ2_XS scales its two 16-element groups
// separately (split B layout, as Q3_K). Value scales: IQ2_XXS / IQ2_XS
// d (2s+1)/8, IQ3_XXS d (2s+1)/4, IQ1_S d (2s+1)/8 (src/quants.c:179-228;
// gguf-py IQ2_XXS / IQ1_S).
//
// Codebook lookups are random per lane, so a plain shared-memory table
// costs several bank conflicts per load. The engine instead stages
// lane-private copies (iq_tabs_fill), every entry one 128-byte row:
//   IQ2_XXS / IQ2_XS: every codebook byte is 8, 25 or 43, so a row is
//               stored as 8 nibble codes (0, 1, 2) and a 7-bit sign field
//               (bit 7 = its parity, gguf ksigns_iq2xs) as 8 nibbles with
//               bit 2 = the element's sign. code | sign is then a byte
//               permute selector picking from {8, 25, 43} and {-8, -25,
//               -43}: one OR and two PRMT give the signed row. Codebooks
//               256 / 512 entries and the sign table 128 entries, each
//               entry 32 copies of its 4-byte word (lane l reads copy l:
//               conflict-free).
//   IQ3_XXS: codebook 256 entries x 32 copies of the 4-byte row; sign masks
//               128 entries x 16 copies of uint2 {m_lo, m_hi}, m = 0xFF in
//               each byte whose element is negated; (g ^ m) + (m & 1s) = -g
//               per negated byte (codebook bytes are 4..62: no carries).
//               Lane l reads mask copy l % 16 (8-byte loads are served 16
//               lanes at a time: 16 distinct bank pairs).
//   IQ1_S: 4096 entries of 8 bytes (one copy), entry e = index | (delta
//               sign << 11), bytes 8 g + 1 (or 8 g - 1) = 8 (g + delta).
// Each region is present only when a format of the launch needs it.
constexpr uint32_t kIqRow = 128;
struct IqLayout {
    uint32_t sign, spread, g2xxs, g2xs, g3xxs, g1s;   // byte offsets in the region (~0u: absent)
    uint32_t bytes;
};
constexpr uint32_t kIq2Pos = 0x002B1908u;   // bytes 8, 25, 43
constexpr uint32_t kIq2Neg = 0x00D5E7F8u;   // bytes -8, -25, -43
__host__ __device__ constexpr bool iq_format(int t) {
    return t == T_IQ2_XXS || t == T_IQ2_XS || t == T_IQ3_XXS || t == T_IQ1_S;
}
// Host: the region for a launch whose matrices have formats a and b.
inline IqLayout iq_layout(int a, int b) {
    IqLayout L{~0u, ~0u, ~0u, ~0u, ~0u, ~0u, 0u};
    auto has = [&](int t) { return a == t || b == t; };
    auto take = [&](uint32_t &off, uint32_t n) { off = L.bytes; L.bytes += n; };
    if (has(T_IQ3_XXS)) take(L.sign, 128 * kIqRow);
    if (has(T_IQ2_XXS) || has(T_IQ2_XS)) take(L.spread, 128 * kIqRow);
    if (has(T_IQ2_XXS)) take(L.g2xxs, 256 * kIqRow);
    if (has(T_IQ2_XS)) take(L.g2xs, 512 * kIqRow);
    if (has(T_IQ3_XXS)) take(L.g3xxs, 256 * kIqRow);
    if (has(T_IQ1_S)) take(L.g1s, 4096 * 8);
    return L;
}

// Sign masks of a 7-bit sign field s (bit 7 = its parity, gguf
// ksigns_iq2xs): bit j -> byte j = 0xFF (copies of a nibble 7 bits apart
// never overlap; then a sign-replicating prmt -- the __byte_perm intrinsic
// ignores the replicate bit).
__device__ __forceinline__ uint2 iq_sign_masks(uint32_t s) {
    const uint32_t b = sepia_ksigns_iq2xs[s];
    return make_uint2((uint32_t)prmt_sel((b & 15u) * 0x10204080u, 0xBA98u),
                      (uint32_t)prmt_sel((b >> 4) * 0x10204080u, 0xBA98u));
}
// bytes (each < 16) of lo, hi -> 8 nibbles
__device__ __forceinline__ uint32_t iq_nibbles(uint32_t lo, uint32_t hi) {
    const uint32_t a = (lo | (lo >> 4)) & 0x00FF00FFu, b = (hi | (hi >> 4)) & 0x00FF00FFu;
    return ((a | (a >> 8)) & 0xFFFFu) | (((b | (b >> 8)) & 0xFFFFu) << 16);
}
// IQ2 codebook row (bytes 8, 25, 43) -> nibble codes 0, 1, 2: byte * 3 >> 6
// (no byte overflows: 43 * 3 < 256)
__device__ __forceinline__ uint32_t iq2_codes(uint64_t g) {
    const uint32_t lo = (((uint32_t)g * 3u) >> 6) & 0x03030303u, hi = (((uint32_t)(g >> 32) * 3u) >> 6) & 0x03030303u;
    return iq_nibbles(lo, hi);
}
// sign field s -> nibble j bit 2 = sign of element j
__device__ __forceinline__ uint32_t iq2_spread(uint32_t s) {
    const uint32_t b = sepia_ksigns_iq2xs[s];
    const uint32_t lo = ((b & 15u) * 0x00204081u) & 0x01010101u, hi = ((b >> 4) * 0x00204081u) & 0x01010101u;
    return iq_nibbles(lo, hi) << 2;
}

// Fill the region (the calling threads, numbered 0..nthreads-1; the caller
// synchronises them before any walk reads it). Every replicated entry is
// one 128-byte row written as 8 16-byte stores.
__device__ inline void iq_tabs_fill(uint8_t *r, const IqLayout &L, int tid, int nthreads) {
    auto rows = [&](uint32_t off, int n, auto word4) {
        if (off == ~0u) return;
        uint4 *d = reinterpret_cast<uint4 *>(r + off);
        for (int i = tid; i < n * 8; i += nthreads) d[i] = word4(i >> 3);
    };
    rows(L.sign, 128, [](int e) { const uint2 m = iq_sign_masks((uint32_t)e); return make_uint4(m.x, m.y, m.x, m.y); });
    rows(L.spread, 128, [](int e) { const uint32_t w = iq2_spread((uint32_t)e); return make_uint4(w, w, w, w); });
    rows(L.g2xxs, 256, [](int e) { const uint32_t w = iq2_codes(sepia_iq2xxs_grid[e]); return make_uint4(w, w, w, w); });
    rows(L.g2xs, 512, [](int e) { const uint32_t w = iq2_codes(sepia_iq2xs_grid[e]); return make_uint4(w, w, w, w); });
    rows(L.g3xxs, 256, [](int e) { const uint32_t w = sepia_iq3xxs_grid[e]; return make_uint4(w, w, w, w); });
    if (L.g1s != ~0u) {
        for (int e = tid; e < 4096; e += nthreads) {
            const uint64_t g = sepia_iq1s_grid[e & 2047];
            // 8 g + 1 (or 8 g - 1) per byte, g in {-1, 0, 1}
            const uint32_t add = (e & 2048) ? 0xFFFFFFFFu : 0x01010101u;
            const uint32_t lo = (uint32_t)g, hi = (uint32_t)(g >> 32);
            uint32_t w[2];
#pragma unroll
            for (int h = 0; h < 2; h++) {
                const uint32_t gw = h ? hi : lo;
                uint32_t o = 0;
#pragma unroll
                for (int j = 0; j < 4; j++) o |= ((((gw >> (8 * j)) * 8u) + add) & 255u) << (8 * j);
                w[h] = o;
            }
            reinterpret_cast<uint2 *>(r + L.g1s)[e] = make_uint2(w[0], w[1]);
        }
    }
}

// A lane's views of the region: entry i of a replicated table is at
// base + i * kIqRow.
struct IqLane {
    const uint8_t *sign, *grid;
};
__device__ __forceinline__ IqLane iq_lane(const uint8_t *r, const IqLayout &L, int t, int lane) {
    IqLane q;
    q.sign = (t == T_IQ3_XXS) ? r + L.sign + 8 * (lane & 15) : r + L.spread + 4 * lane;
    q.grid = (t == T_IQ2_XXS) ? r + L.g2xxs + 4 * lane
           : (t == T_IQ2_XS)  ? r + L.g2xs + 4 * lane
           : (t == T_IQ3_XXS) ? r + L.g3xxs + 4 * lane
                              : r + L.g1s;
    return q;
}

__device__ __forceinline__ void mma_k32_ss_z(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                             uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%10,%10,%10};\n"
        : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}

__device__ __forceinline__ uint2 lds64(const uint8_t *p) { return *reinterpret_cast<const uint2 *>(p); }
__device__ __forceinline__ uint4 lds128(const uint8_t *p) { return *reinterpret_cast<const uint4 *>(p); }
__device__ __forceinline__ uint32_t ldh(const uint8_t *p) { return *reinterpret_cast<const uint16_t *>(p); }

// codebook row g (8 bytes) with the signs of mask entry m applied
__device__ __forceinline__ void iq_signed(uint2 g, uint2 m, uint32_t &lo, uint32_t &hi) {
    lo = (g.x ^ m.x) + (m.x & 0x01010101u);
    hi = (g.y ^ m.y) + (m.y & 0x01010101u);
}

// Superblock walks: ODD = the superblock starts 2 bytes past a 4-byte
// boundary (every IQ superblock size is 2 mod 4).
template <bool ODD>
__device__ __forceinline__ void sb_iq2xxs(const uint8_t *bg, const uint8_t *bg8, const uint8_t *te, const IqLane &Q,
                                          const LaneCtx &C, double &yg, double &yg8) {
    // part p: 4 codebook indices at 2+8p, then a word of four 7-bit sign
    // fields and the 4-bit scale (bits 28-31)
    const uint32_t sh = 7u * (uint32_t)C.tig;
    int acc[4] = {0, 0, 0, 0};
#pragma unroll
    for (int p = 0; p < 8; p++) {
        const uint32_t sg = ldw2<!ODD>(bg + 6 + 8 * p), sg8 = ldw2<!ODD>(bg8 + 6 + 8 * p);
        const uint32_t ix = bg[2 + 8 * p + C.tig], ix8 = bg8[2 + 8 * p + C.tig];
        const uint32_t w = ldw(Q.grid + kIqRow * ix) | ldw(Q.sign + kIqRow * ((sg >> sh) & 127u));
        const uint32_t w8 = ldw(Q.grid + kIqRow * ix8) | ldw(Q.sign + kIqRow * ((sg8 >> sh) & 127u));
        const uint32_t a0 = __byte_perm(kIq2Pos, kIq2Neg, w), a2 = __byte_perm(kIq2Pos, kIq2Neg, w >> 16);
        const uint32_t a1 = __byte_perm(kIq2Pos, kIq2Neg, w8), a3 = __byte_perm(kIq2Pos, kIq2Neg, w8 >> 16);
        const uint2 b = ld_b(te, p, C);
        int cc[4];
        mma_k32_ss_z(cc, a0, a1, a2, a3, b.x, b.y);
        const int s = (int)((sg >> 27) | 1u), s8 = (int)((sg8 >> 27) | 1u);     // 2 * scale + 1
        acc[0] += s * cc[0];
        acc[1] += s * cc[1];
        acc[2] += s8 * cc[2];
        acc[3] += s8 * cc[3];
    }
    const float u = ld_unit(te + C.unit_off) * C.lwn * 0.125f;
    yg += (double)(cvt16<true>(ldh(bg)) * u) * limb_pair(acc[0], acc[1], 1.0f);
    yg8 += (double)(cvt16<true>(ldh(bg8)) * u) * limb_pair(acc[2], acc[3], 1.0f);
}

template <bool ODD>
__device__ __forceinline__ void sb_iq2xs(const uint8_t *bg, const uint8_t *bg8, const uint8_t *te, const IqLane &Q,
                                         const LaneCtx &C, double &yg, double &yg8) {
    // part p, group l: uint16 at 2+8p+2l = 9-bit codebook index | 7-bit
    // sign field << 9; scale byte 66+p: low nibble elements 0-15, high 16-31
    const uint32_t ssh = 4u * (uint32_t)(C.tig >> 1);
    int acc[4] = {0, 0, 0, 0};
#pragma unroll
    for (int p = 0; p < 8; p++) {
        const uint32_t q = ldh(bg + 2 + 8 * p + 2 * C.tig), q8 = ldh(bg8 + 2 + 8 * p + 2 * C.tig);
        const uint32_t w = ldw(Q.grid + kIqRow * (q & 511u)) | ldw(Q.sign + kIqRow * (q >> 9));
        const uint32_t w8 = ldw(Q.grid + kIqRow * (q8 & 511u)) | ldw(Q.sign + kIqRow * (q8 >> 9));
        const uint32_t a0 = __byte_perm(kIq2Pos, kIq2Neg, w), a2 = __byte_perm(kIq2Pos, kIq2Neg, w >> 16);
        const uint32_t a1 = __byte_perm(kIq2Pos, kIq2Neg, w8), a3 = __byte_perm(kIq2Pos, kIq2Neg, w8 >> 16);
        const uint2 e = ld_b(te, p, C);
        int cc[4];
        mma_k32_ss_z(cc, a0, a1, a2, a3, e.x & C.msplit, e.y & C.msplit);
        // this lane's C columns belong to group tig/2 of the part
        const int s = (int)(((uint32_t)bg[66 + p] >> ssh) & 15u) * 2 + 1;
        const int s8 = (int)(((uint32_t)bg8[66 + p] >> ssh) & 15u) * 2 + 1;
        acc[0] += s * cc[0];
        acc[1] += s * cc[1];
        acc[2] += s8 * cc[2];
        acc[3] += s8 * cc[3];
    }
    const float u = ld_unit(te) * C.lws * 0.125f;
    yg += (double)(cvt16<true>(ldh(bg)) * u) * limb_pair(acc[0], acc[1], 1.0f);
    yg8 += (double)(cvt16<true>(ldh(bg8)) * u) * limb_pair(acc[2], acc[3], 1.0f);
}

template <bool ODD>
__device__ __forceinline__ void sb_iq3xxs(const uint8_t *bg, const uint8_t *bg8, const uint8_t *te, const IqLane &Q,
                                          const LaneCtx &C, double &yg, double &yg8) {
    // part p: 8 codebook indices at 2+8p (group l: bytes 2l, 2l+1, 4 values
    // each), word at 66+4p = four 7-bit sign fields | scale << 28
    const uint32_t sh = 7u * (uint32_t)C.tig;
    int acc[4] = {0, 0, 0, 0};
#pragma unroll
    for (int p = 0; p < 8; p++) {
        const uint32_t sw = ldw2<!ODD>(bg + 66 + 4 * p), sw8 = ldw2<!ODD>(bg8 + 66 + 4 * p);
        const uint32_t ii = ldh(bg + 2 + 8 * p + 2 * C.tig), ii8 = ldh(bg8 + 2 + 8 * p + 2 * C.tig);
        const uint2 g = make_uint2(ldw(Q.grid + kIqRow * (ii & 255u)), ldw(Q.grid + kIqRow * (ii >> 8)));
        const uint2 g8 = make_uint2(ldw(Q.grid + kIqRow * (ii8 & 255u)), ldw(Q.grid + kIqRow * (ii8 >> 8)));
        const uint2 m = lds64(Q.sign + kIqRow * ((sw >> sh) & 127u));
        const uint2 m8 = lds64(Q.sign + kIqRow * ((sw8 >> sh) & 127u));
        uint32_t a0, a1, a2, a3;
        iq_signed(g, m, a0, a2);
        iq_signed(g8, m8, a1, a3);
        const uint2 b = ld_b(te, p, C);
        int cc[4];
        mma_k32_ss_z(cc, a0, a1, a2, a3, b.x, b.y);
        const int s = (int)((sw >> 27) | 1u), s8 = (int)((sw8 >> 27) | 1u);
        acc[0] += s * cc[0];
        acc[1] += s * cc[1];
        acc[2] += s8 * cc[2];
        acc[3] += s8 * cc[3];
    }
    const float u = ld_unit(te + C.unit_off) * C.lwn * 0.25f;
    yg += (double)(cvt16<true>(ldh(bg)) * u) * limb_pair(acc[0], acc[1], 1.0f);
    yg8 += (double)(cvt16<true>(ldh(bg8)) * u) * limb_pair(acc[2], acc[3], 1.0f);
}

__device__ __forceinline__ void sb_iq1s(const uint8_t *bg, const uint8_t *bg8, const uint8_t *te, const IqLane &Q,
                                        const LaneCtx &C, double &yg, double &yg8) {
    // part p: 4 low index bytes at 2+4p; uint16 at 34+2p = four 3-bit high
    // index fields | scale << 12 | delta sign << 15
    const uint32_t sh = 3u * (uint32_t)C.tig;
    int acc[4] = {0, 0, 0, 0};
#pragma unroll
    for (int p = 0; p < 8; p++) {
        const uint32_t h = ldh(bg + 34 + 2 * p), h8 = ldh(bg8 + 34 + 2 * p);
        const uint32_t e = (uint32_t)bg[2 + 4 * p + C.tig] | (((h >> sh) & 7u) << 8) | ((h >> 4) & 0x800u);
        const uint32_t e8 = (uint32_t)bg8[2 + 4 * p + C.tig] | (((h8 >> sh) & 7u) << 8) | ((h8 >> 4) & 0x800u);
        const uint2 g = lds64(Q.grid + 8 * e), g8 = lds64(Q.grid + 8 * e8);
        const uint2 b = ld_b(te, p, C);
        int cc[4];
        mma_k32_ss_z(cc, g.x, g8.x, g.y, g8.y, b.x, b.y);
        const int s = (int)(((h >> 11) & 14u) | 1u), s8 = (int)(((h8 >> 11) & 14u) | 1u);
        acc[0] += s * cc[0];
        acc[1] += s * cc[1];
        acc[2] += s8 * cc[2];
        acc[3] += s8 * cc[3];
    }
    const float u = ld_unit(te + C.unit_off) * C.lwn * 0.125f;
    yg += (double)(cvt16<true>(ldh(bg)) * u) * limb_pair(acc[0], acc[1], 1.0f);
    yg8 += (double)(cvt16<true>(ldh(bg8)) * u) * limb_pair(acc[2], acc[3], 1.0f);
}

// ------------------------------------------------------------ dispatch
__host__ __device__ constexpr bool mma_format(int t) { return t == T_Q2_K || t == T_Q3_K || t == T_Q4_K; }

// Superblocks [i0, i1) of the staged rows (row gid at rg, row gid+8 at rg8,
// superblock i at +i*sb_bytes); table entries start at te0 for i = 0.
// Q2_K/Q4_K rows must start 4-byte aligned; Q3_K rows 2-byte aligned, with
// flip = 1 when superblock 0 sits 2 bytes off a 4-byte boundary.
template <int T>
__device__ __forceinline__ void tile_sbs(const uint8_t *rg, const uint8_t *rg8, const uint8_t *te0, int i0, int i1,
                                         int flip, const LaneCtx &C, double &yg, double &yg8,
                                         const IqLane &Q = IqLane{}) {
    constexpr int SB = fmt_block_bytes(T);
    const uint8_t *r = rg + i0 * SB, *r8 = rg8 + i0 * SB, *te = te0 + (size_t)i0 * kTabSB;
    for (int i = i0; i < i1; i++, r += SB, r8 += SB, te += kTabSB) {
        const bool odd = (i ^ flip) & 1;
        if constexpr (T == T_Q2_K) sb_q2k(r, r8, te, C, yg, yg8);
        else if constexpr (T == T_Q3_K) {
            if (odd) sb_q3k<true>(r, r8, te, C, yg, yg8);
            else sb_q3k<false>(r, r8, te, C, yg, yg8);
        } else if constexpr (T == T_Q4_K) sb_q4k(r, r8, te, C, yg, yg8);
        else if constexpr (T == T_IQ2_XXS) {
            if (odd) sb_iq2xxs<true>(r, r8, te, Q, C, yg, yg8);
            else sb_iq2xxs<false>(r, r8, te, Q, C, yg, yg8);
        } else if constexpr (T == T_IQ2_XS) {
            if (odd) sb_iq2xs<true>(r, r8, te, Q, C, yg, yg8);
            else sb_iq2xs<false>(r, r8, te, Q, C, yg, yg8);
        } else if constexpr (T == T_IQ3_XXS) {
            if (odd) sb_iq3xxs<true>(r, r8, te, Q, C, yg, yg8);
            else sb_iq3xxs<false>(r, r8, te, Q, C, yg, yg8);
        } else sb_iq1s(r, r8, te, Q, C, yg, yg8);
    }
}

// IQ: 0 = K-quant formats only; > 0 = every matrix of the launch has this
// IQ format; -1 = any format (IQ tables in the region at iq, laid out by L).
template <int IQ = 0>
__device__ __forceinline__ void tile_sbs_rt(int t, const uint8_t *rg, const uint8_t *rg8, const uint8_t *te0, int i0,
                                            int i1, int flip, const LaneCtx &C, double &yg, double &yg8,
                                            const uint8_t *iq = nullptr, const IqLayout *L = nullptr) {
    if constexpr (IQ > 0) {
        tile_sbs<IQ>(rg, rg8, te0, i0, i1, flip, C, yg, yg8, iq_lane(iq, *L, IQ, 4 * C.gid + C.tig));
        return;
    } else if constexpr (IQ < 0) {
        if (iq_format(t)) {
            const IqLane Q = iq_lane(iq, *L, t, 4 * C.gid + C.tig);
            switch (t) {
            case T_IQ2_XXS: tile_sbs<T_IQ2_XXS>(rg, rg8, te0, i0, i1, flip, C, yg, yg8, Q); return;
            case T_IQ2_XS: tile_sbs<T_IQ2_XS>(rg, rg8, te0, i0, i1, flip, C, yg, yg8, Q); return;
            case T_IQ3_XXS: tile_sbs<T_IQ3_XXS>(rg, rg8, te0, i0, i1, flip, C, yg, yg8, Q); return;
            default: tile_sbs<T_IQ1_S>(rg, rg8, te0, i0, i1, flip, C, yg, yg8, Q); return;
            }
        }
    }
    switch (t) {
    case T_Q2_K: tile_sbs<T_Q2_K>(rg, rg8, te0, i0, i1, flip, C, yg, yg8); break;
    case T_Q3_K: tile_sbs<T_Q3_K>(rg, rg8, te0, i0, i1, flip, C, yg, yg8); break;
    default: tile_sbs<T_Q4_K>(rg, rg8, te0, i0, i1, flip, C, yg, yg8); break;
    }
}

// Sum the quad's 4 lanes: afterwards every lane of the quad holds the rows'
// values (row gid in yg, gid+8 in yg8).
__device__ __forceinline__ void quad_sum(double &yg, double &yg8) {
    yg += __shfl_xor_sync(0xffffffffu, yg, 1);
    yg8 += __shfl_xor_sync(0xffffffffu, yg8, 1);
    yg += __shfl_xor_sync(0xffffffffu, yg, 2);
    yg8 += __shfl_xor_sync(0xffffffffu, yg8, 2);
}

}  // namespace sepia
