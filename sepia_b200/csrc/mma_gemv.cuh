// sepia_b200/csrc/mma_gemv.cuh -- quantized GEMV on the integer tensor cores.
//
// Why: a batch-1 GEMV over 2-3 bit weights is HBM-bound only if unpacking
// costs about one instruction per weight; on the FP32 pipe (convert + FMA
// per weight) it costs 3-7, so the kernel is issue-bound far below the HBM
// roofline. Here the weights are unpacked to 8-bit integers (a few bit ops
// per 4 weights) and the multiply-accumulate runs on the tensor cores.
//
// Exactness: each superblock's 256 activations are written as integers
// x_int = round(x * 2^(25-e)) (e = exponent of the superblock's largest
// |x|) split into four balanced base-256 digits ("limbs", signed bytes). The
// tensor core computes sum_k w_int[k] * limb_j[k] exactly in int32 for every
// limb j (the columns N of an m16n8k32 MMA, 4 of 8 used), so a superblock's
// dot is exact; recombining limbs in fp64 gives sum_k w_int[k]*x_int[k]
// exactly. Only x's representation rounds, at 2^-25 of the superblock's
// largest value. The Q2_K "min" term sum_g m_g * sum_{k in g} x_int[k] is a
// second, k16 MMA per superblock over the 16 group sums (also exact).
//
// Fragment layouts (lane = 4*gid + tig), m16n8k32 u8 x s8 -> s32:
//   A (16 x 32): a0 = row gid,   k 4tig..+3      a1 = row gid+8, same k
//                a2 = row gid,   k 16+4tig..+3   a3 = row gid+8, same k
//   B (32 x 8):  b0 = k 4tig..+3, col gid        b1 = k 16+4tig..+3, col gid
//   C (16 x 8):  c0 = (gid, 2tig) c1 = (gid, 2tig+1) c2 = (gid+8, 2tig) c3 = (gid+8, 2tig+1)
// m16n8k16 is the same with only a0/a1 and b0.
#pragma once
#include "quant_dot.cuh"

namespace sepia {

constexpr int kXShift = 25;   // x_int = round(x * 2^(kXShift - e))

// Per-CTA activation tables in shared memory.
struct XLimbs {
    uint2 *b;        // [nsb][8 parts][4 tig][4 limbs]: B fragments of the k32 MMAs
    uint32_t *bg;    // [nsb][4 tig][4 limbs]: B fragments of the group-sum k16 MMA
    float *unit;     // [nsb] 2^-(kXShift-e): value of one x_int unit
};

__host__ __device__ inline int xlimbs_bytes(int nsb) { return nsb * (8 * 4 * 4 * 8 + 4 * 4 * 4 + 4); }

__device__ __forceinline__ XLimbs xlimbs_carve(uint8_t *base, int nsb) {
    XLimbs L;
    L.b = reinterpret_cast<uint2 *>(base);
    L.bg = reinterpret_cast<uint32_t *>(base + nsb * 8 * 4 * 4 * 8);
    L.unit = reinterpret_cast<float *>(base + nsb * (8 * 4 * 4 * 8 + 4 * 4 * 4));
    return L;
}

// Balanced base-256 digits of v (|v| < 2^30): v = d0 + 256 d1 + 65536 d2 + 2^24 d3.
__device__ __forceinline__ void limbs4(int v, int (&d)[4]) {
#pragma unroll
    for (int j = 0; j < 3; j++) {
        const int lo = ((v + 128) & 255) - 128;
        d[j] = lo;
        v = (v - lo) >> 8;
    }
    d[3] = v;
}

// Build the tables for x[0..nsb*256) with every warp of the CTA (one warp
// per superblock); ends with __syncthreads(). Lane l owns part l/4 and
// tig l%4, i.e. positions 32*part + 4*tig + {0..3} and +16.
__device__ inline void xlimbs_build(const XLimbs &L, const float *x, int nsb, int warp, int nwarps, int lane) {
    const int part = lane >> 2, tig = lane & 3;
    for (int sb = warp; sb < nsb; sb += nwarps) {
        const float *xs = x + sb * kQK + 32 * part + 4 * tig;
        const float4 lo = *reinterpret_cast<const float4 *>(xs);
        const float4 hi = *reinterpret_cast<const float4 *>(xs + 16);
        const float v[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
        float m = 0.f;
#pragma unroll
        for (int j = 0; j < 8; j++) m = fmaxf(m, fabsf(v[j]));
        m = warp_max(m);
        int e = (m > 0.f) ? ((__float_as_int(m) >> 23) & 0xFF) - 127 : 0;
        e = max(-90, min(e, 90));
        const float scale = __int_as_float((127 + kXShift - e) << 23);
        int xi[8];
        uint32_t w0[4] = {0, 0, 0, 0}, w1[4] = {0, 0, 0, 0};
#pragma unroll
        for (int j = 0; j < 8; j++) {
            xi[j] = __float2int_rn(v[j] * scale);
            int d[4];
            limbs4(xi[j], d);
#pragma unroll
            for (int l = 0; l < 4; l++) {
                if (j < 4) w0[l] |= (uint32_t)(d[l] & 255) << (8 * j);
                else w1[l] |= (uint32_t)(d[l] & 255) << (8 * (j - 4));
            }
        }
        uint2 *bd = L.b + (size_t)sb * 128 + lane * 4;
#pragma unroll
        for (int l = 0; l < 4; l++) bd[l] = make_uint2(w0[l], w1[l]);
        // group sums: group 2*part (positions 4tig..+3 of the low half) and
        // 2*part+1 (high half); the 4 lanes of a part share their groups
        int g0 = xi[0] + xi[1] + xi[2] + xi[3], g1 = xi[4] + xi[5] + xi[6] + xi[7];
        g0 += __shfl_xor_sync(0xffffffffu, g0, 1);
        g0 += __shfl_xor_sync(0xffffffffu, g0, 2);
        g1 += __shfl_xor_sync(0xffffffffu, g1, 1);
        g1 += __shfl_xor_sync(0xffffffffu, g1, 2);
        // k16 B fragment: lane (gid, t) holds limb gid of groups 4t..4t+3;
        // write it from the lane that owns group pair (part): groups 2p, 2p+1
        // live in word t = (2p)/4 = p/2, bytes 2(p&1), 2(p&1)+1
        if (tig == 0) {
            int d0[4], d1[4];
            limbs4(g0, d0);
            limbs4(g1, d1);
            uint8_t *bgb = reinterpret_cast<uint8_t *>(L.bg + (size_t)sb * 16);
#pragma unroll
            for (int l = 0; l < 4; l++) {
                // word index: t = part/2, limb l -> L.bg[sb][t][l]
                uint8_t *wp = bgb + 4 * ((part >> 1) * 4 + l);
                wp[2 * (part & 1)] = (uint8_t)(d0[l] & 255);
                wp[2 * (part & 1) + 1] = (uint8_t)(d1[l] & 255);
            }
        }
        if (lane == 0) L.unit[sb] = __int_as_float((127 - kXShift + e) << 23);
    }
    __syncthreads();
}

__device__ __forceinline__ void mma_k32(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                        uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void mma_k16(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%0,%1,%2,%3};\n"
        : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
        : "r"(a0), "r"(a1), "r"(b0));
}

// byte j of w as a 32-bit integer
__device__ __forceinline__ uint32_t byte_of(uint32_t w, int j) { return __byte_perm(w, 0u, 0x4440u + j); }

// One warp, one 16-row tile of Q2_K rows (row r at tile + r*rb, 4-byte
// aligned), superblocks [sb0, sb1). Adds this lane's share of the exact
// row values to yg (row gid) and yg8 (row gid+8): the row's value is the sum
// of yg over the 4 lanes of its quad (see tile16_finish).
__device__ __forceinline__ void tile16_q2k(const uint8_t *tile, int64_t rb, int sb0, int sb1, const XLimbs &X,
                                           int lane, double &yg, double &yg8) {
    const int gid = lane >> 2, tig = lane & 3;
    // weight of this lane's limb pair (lanes tig 2, 3 hold the zero columns)
    const float lw = (tig == 0) ? 1.0f : (tig == 1 ? 65536.0f : 0.0f);
    const uint8_t *rg = tile + (int64_t)gid * rb, *rg8 = tile + (int64_t)(gid + 8) * rb;
    for (int sb = sb0; sb < sb1; sb++) {
        const uint8_t *bg = rg + sb * 84, *bg8 = rg8 + sb * 84;
        uint32_t sl[4], sl8[4];          // scale nibbles (low) of the 16 groups
#pragma unroll
        for (int j = 0; j < 4; j++) {
            sl[j] = reinterpret_cast<const uint32_t *>(bg)[j] & 0x0F0F0F0Fu;
            sl8[j] = reinterpret_cast<const uint32_t *>(bg8)[j] & 0x0F0F0F0Fu;
        }
        int c[4] = {0, 0, 0, 0}, c2[4] = {0, 0, 0, 0};
        const uint2 *bf = X.b + (size_t)sb * 128 + tig * 4 + (gid & 3);
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const uint32_t *q = reinterpret_cast<const uint32_t *>(bg + 16 + 32 * h);
            const uint32_t *q8 = reinterpret_cast<const uint32_t *>(bg8 + 16 + 32 * h);
            uint32_t w[4] = {q[tig], q8[tig], q[4 + tig], q8[4 + tig]};
            uint32_t w4[4];
#pragma unroll
            for (int r = 0; r < 4; r++) w4[r] = w[r] >> 4;
#pragma unroll
            for (int s = 0; s < 4; s++) {
                const int p = 4 * h + s;                                   // part: groups 2p, 2p+1
                // fields at shift 2s: s < 2 use w, s >= 2 use w >> 4; the mask
                // keeps them in place, so parts with odd s carry a factor 4
                // (accumulated separately in c2 and divided out exactly)
                const uint32_t m = (s & 1) ? 0x0C0C0C0Cu : 0x03030303u;
                const uint32_t *src = (s < 2) ? w : w4;
                const uint32_t sa = byte_of(sl[p >> 1], 2 * (p & 1)), sb_ = byte_of(sl[p >> 1], 2 * (p & 1) + 1);
                const uint32_t s8a = byte_of(sl8[p >> 1], 2 * (p & 1)), s8b = byte_of(sl8[p >> 1], 2 * (p & 1) + 1);
                const uint32_t a0 = (src[0] & m) * sa;
                const uint32_t a1 = (src[1] & m) * s8a;
                const uint32_t a2 = (src[2] & m) * sb_;
                const uint32_t a3 = (src[3] & m) * s8b;
                uint2 b = make_uint2(0u, 0u);
                if (gid < 4) b = bf[p * 16];
                if (s & 1) mma_k32(c2, a0, a1, a2, a3, b.x, b.y);
                else mma_k32(c, a0, a1, a2, a3, b.x, b.y);
            }
        }
        // min term: A = the 16 high nibbles (m_g) per row, B = group sums
        int cm[4] = {0, 0, 0, 0};
        {
            const uint32_t am = (reinterpret_cast<const uint32_t *>(bg)[tig] >> 4) & 0x0F0F0F0Fu;
            const uint32_t am8 = (reinterpret_cast<const uint32_t *>(bg8)[tig] >> 4) & 0x0F0F0F0Fu;
            const uint32_t bm = (gid < 4) ? X.bg[(size_t)sb * 16 + tig * 4 + gid] : 0u;
            mma_k16(cm, am, am8, bm);
        }
        // lane tig 0 holds limbs {0,1}, tig 1 limbs {2,3}: pair them in int32
        // (|c| < 2^23, so c_lo + 256*c_hi < 2^31) and convert once
        const int ia = (c[0] + (c2[0] >> 2)) + 256 * (c[1] + (c2[1] >> 2));
        const int ia8 = (c[2] + (c2[2] >> 2)) + 256 * (c[3] + (c2[3] >> 2));
        const int im = cm[0] + 256 * cm[1], im8 = cm[2] + 256 * cm[3];
        const uint32_t dd = *reinterpret_cast<const uint32_t *>(bg + 80);
        const uint32_t dd8 = *reinterpret_cast<const uint32_t *>(bg8 + 80);
        const float u = X.unit[sb] * lw;                 // exact power-of-two scaling
        yg += (double)(cvt16<true>(dd & 0xFFFFu) * u) * (double)ia - (double)(cvt16<true>(dd >> 16) * u) * (double)im;
        yg8 += (double)(cvt16<true>(dd8 & 0xFFFFu) * u) * (double)ia8 - (double)(cvt16<true>(dd8 >> 16) * u) * (double)im8;
    }
}

// Complete the quad sum: after this the row values are valid in tig 0.
__device__ __forceinline__ void tile16_finish(double &yg, double &yg8) {
    yg += __shfl_xor_sync(0xffffffffu, yg, 1);
    yg8 += __shfl_xor_sync(0xffffffffu, yg8, 1);
}

}  // namespace sepia
