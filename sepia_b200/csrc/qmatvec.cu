// sepia_b200/csrc/qmatvec.cu -- standalone dequantisation and the
// single-matrix quantized GEMV (ABI sepia_gpu_matvec_q / sepia_gpu_dequant_rows,
// src/sepia_gpu.h:147,160; Metal twin metal/matvec_q.metal:358-737).
//
// k_matvec streams row tiles of one [out_dim, in_dim] quantized matrix
// through shared memory (stream.cuh). CTA = nwc*G consumer warps + 1
// producer warp: nwc column slices of 4 superblocks each (lanes hold their
// activation parts in registers) x G row groups of TRW rows.
#include "../../include/sepia_cuda.h"
#include "runtime.h"
#include "stream.cuh"
#include "qengine.cuh"

#include <algorithm>
#include <stdlib.h>

namespace sepia {

int op_matvec_f32(const float *w, const float *x, float *y, int64_t out_dim, int64_t in_dim, cudaStream_t st);

constexpr int kMvStagesMax = 6;

struct MvParams {
    const uint8_t *w;
    int64_t row_bytes;
    const float *x;     // [n_vec, in_dim]
    float *y;           // [n_vec, out_dim]
    int64_t out_dim, in_dim;
    int n_vec;
    int nsb;            // superblocks per row
    int nwc;            // consumer warps per row group (column slices)
    int G;              // row groups
    int stages;
    uint32_t slot_bytes;
    int64_t num_units;  // ceil(out_dim / (TRW*G))
    int *err;
};

template <int T, int TRW, int C>
__global__ void __launch_bounds__(17 * 32) k_matvec(const MvParams P) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n_cons = P.nwc * P.G;
    const int TR = TRW * P.G;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem);
    uint64_t *empty = full + kMvStagesMax;
    double *red = reinterpret_cast<double *>(smem + 128);                  // [G][nwc][TRW]
    uint8_t *stage0 = smem + 128 + ((n_cons * TRW * 8 + 127) & ~127);

    if (threadIdx.x == 0) {
        for (int s = 0; s < P.stages; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], n_cons);
        }
        fence_barrier_init();
    }
    __syncthreads();

    const int sbb = fmt_sb_bytes(T);
    griddep_wait();
    griddep_launch();

    if (warp == n_cons) {
        // ---------------- producer ----------------
        if (lane == 0) {
            int64_t k = 0;
            for (int64_t u = blockIdx.x; u < P.num_units; u += gridDim.x, k++) {
                const int slot = (int)(k % P.stages);
                if (k >= P.stages && !mbar_wait(&empty[slot], (uint32_t)(((k / P.stages) - 1) & 1), P.err)) break;
                const int64_t r0 = u * TR;
                const int64_t nr = imin64(TR, P.out_dim - r0);
                ByteRange r{P.w + r0 * P.row_bytes, (uint32_t)(nr * P.row_bytes)};
                mbar_arrive_expect_tx(&full[slot], range_copy_bytes(r));
                range_issue(stage0 + (size_t)slot * P.slot_bytes, r, &full[slot]);
            }
            // drain: wait (bounded) for the copies still in flight
            const int64_t issued = k;
            for (int64_t j = (issued > P.stages ? issued - P.stages : 0); j < issued; j++)
                mbar_wait(&full[j % P.stages], (uint32_t)((j / P.stages) & 1), nullptr);
        }
        return;
    }

    // ---------------- consumers ----------------
    const int cw = warp % P.nwc, g = warp / P.nwc, p = lane & 7;
    int sb[C];
#pragma unroll
    for (int j = 0; j < C; j++) sb[j] = 4 * (j * P.nwc + cw) + (lane >> 3);
    XPart xp[C];
    if (P.n_vec == 1) {
#pragma unroll
        for (int j = 0; j < C; j++) load_xpart<fast_format(T)>(xp[j],P.x, P.in_dim, sb[j], p);
    }
    const int wlane = (32 / TRW) - 1;   // lanes sharing one row after the reduce-scatter
    const int my_row = rs_row<TRW>(lane);

    int64_t k = 0;
    for (int64_t u = blockIdx.x; u < P.num_units; u += gridDim.x, k++) {
        const int slot = (int)(k % P.stages);
        if (!mbar_wait(&full[slot], (uint32_t)((k / P.stages) & 1), P.err)) break;
        const int64_t r0 = u * TR;
        const int64_t nr = imin64(TR, P.out_dim - r0);
        const uint8_t *base = range_data(stage0 + (size_t)slot * P.slot_bytes, ByteRange{P.w + r0 * P.row_bytes, 0});
        for (int v = 0; v < P.n_vec; v++) {
            if (P.n_vec > 1) {
#pragma unroll
                for (int j = 0; j < C; j++) load_xpart<fast_format(T)>(xp[j],P.x + (int64_t)v * P.in_dim, P.in_dim, sb[j], p);
            }
            float acc[TRW];
#pragma unroll
            for (int i = 0; i < TRW; i++) {
                const int rl = g * TRW + i;
                acc[i] = (rl < nr) ? row_parts_dot<T, C>(base + rl * P.row_bytes, sbb, sb, p, xp, P.in_dim) : 0.0f;
            }
            if (v == P.n_vec - 1) {
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[slot]);
            }
            // partials are reduced in fp64 so the row sum rounds once, like
            // the reference's double-accumulated dot
            double ad[TRW];
#pragma unroll
            for (int i = 0; i < TRW; i++) ad[i] = (double)acc[i];
            warp_reduce_scatter<TRW>(ad, lane);
            if ((lane & wlane) == 0) red[(g * P.nwc + cw) * TRW + my_row] = ad[0];
            consumer_sync(n_cons * 32);
            const int t = threadIdx.x;
            if (t < nr) {
                const int gg = t / TRW, ii = t % TRW;
                double s = 0.0;
                for (int c = 0; c < P.nwc; c++) s += red[(gg * P.nwc + c) * TRW + ii];
                P.y[(int64_t)v * P.out_dim + r0 + t] = (float)s;
            }
            consumer_sync(n_cons * 32);
        }
    }
}

// ------------------------------------------------------------------ tensor-core path
// Q2_K / Q3_K / Q4_K rows through the tensor-core engine (qengine.cuh):
// units are 16-row tiles of the matrix, one activation table (x).
struct MvJob {
    const uint8_t *w;
    int64_t rb, out_dim;
    int type, nsb, sbs, nsplit;
    const float *x;
    float *y;
    __device__ void init() {}
    __device__ void setup(uint8_t *, int, bool) {}
    __device__ int64_t n_units() const { return (out_dim + 15) / 16; }
    __device__ bool needs_dep(int64_t) const { return false; }
    __device__ uint32_t tab_mask(const uint8_t *) const { return 1u; }
    __device__ int splits(const uint8_t *, int64_t) const { return nsplit; }
    __device__ void unit(const uint8_t *, int64_t u, QUnit &U) const {
        const int64_t r0 = u * 16;
        const int nr = (int)imin64(16, out_dim - r0);
        U.type = type; U.nsb = nsb; U.sbs = sbs; U.nsplit = nsplit; U.rb = rb; U.tab = 0;
        U.nlo = min(8, nr);
        U.nhi = max(0, nr - 8);
        U.lo = w + r0 * rb;
        U.hi = U.lo + 8 * rb;
    }
    __device__ int n_tab() const { return 1; }
    __device__ const float *tab_src(int) const { return x; }
    __device__ void finish(const uint8_t *, int64_t u, const QUnit &, double v, int lane) const {
        const int64_t r = u * 16 + lane;
        if (lane < 16 && r < out_dim) y[r] = (float)v;
    }
};

// The same job for the IQ grid-codebook formats (codebooks staged in shared
// memory).
template <int T>
struct MvIqJob : MvJob {
    static constexpr int kIq = T;
};

// Consumer split of an item: whole rows that fit only two stages get one
// group of up to 16 warps (one item in the consumers, one in flight), each
// warp taking two superblocks; otherwise the format-tuned choice when every
// CTA gets several units, qe_groups' (more warps per item) when it gets
// about one (the config-1 2048-row matrices measured slower with 6
// superblocks per warp).
static void mv_groups(int t, int sbs, int64_t rb, int64_t tab_bytes, int64_t units, int &cg, int &G) {
    const int64_t optin = dev_info().smem_optin;
    if (qe_row_budget_for(optin, tab_bytes, rb) > qe_row_budget(optin, tab_bytes, 3)) {
        cg = std::min(kQeMaxCons, (sbs + 1) / 2);
        G = 1;
        return;
    }
    if (units >= 4 * (int64_t)dev_info().sm_count) qe_groups_fmt(sbs, t, t, cg, G);
    else qe_groups(sbs, cg, G);
}

template <class Job>
static int launch_mv_job(const Job &J, const QeLayout &P, int64_t smem, int64_t out_dim, cudaStream_t st) {
    const DevInfo &di = dev_info();
    const void *fn = (const void *)k_qengine<Job>;
    if (!ensure_smem(fn, (int)smem)) return 0;
    const int64_t units = (out_dim + 15) / 16;
    const int64_t grid = std::min<int64_t>(units, (int64_t)di.sm_count);
    return check(launch_pdl(k_qengine<Job>, (unsigned)grid, (P.G * P.cg + 2) * 32, (size_t)smem, st, J, P),
                 "matvec_q (tensor cores) launch");
}

static int launch_matvec_engine(int t, const void *w, const float *x, float *y, int64_t out_dim, int64_t in_dim,
                                int64_t rb, cudaStream_t st, long long wait_cycles = kWaitCycles,
                                uint32_t test_extra_tx = 0) {
    DevInfo &di = dev_info();
    MvJob J;
    J.w = reinterpret_cast<const uint8_t *>(w);
    J.rb = rb; J.out_dim = out_dim; J.type = t;
    J.nsb = (int)(in_dim / kQK);
    J.x = x; J.y = y;
    const IqLayout iql = iq_layout(t, t);
    const uint32_t iqb = iql.bytes;
    J.sbs = qe_sbs(t, J.nsb, qe_row_budget_for(di.smem_optin, (int64_t)J.nsb * kTabSB + iqb, rb), J.nsplit);
    if (!J.sbs) return fail("matvec_q: no tensor-core split for type %d", t);
    QeLayout P;
    int cg, G;
    mv_groups(t, J.sbs, rb, (int64_t)J.nsb * kTabSB + iqb, (out_dim + 15) / 16, cg, G);
    int64_t smem = 0;
    if (!qe_layout(P, G, cg, (uint32_t)J.sbs * qe_sb_bytes(t), 1, J.nsb, di.smem_optin, smem, iqb ? &iql : nullptr))
        return fail("matvec_q: tensor-core tile needs %lld B of shared memory", (long long)smem);
    P.err = di.err;
    P.wait_cycles = wait_cycles;
    P.test_extra_tx = test_extra_tx;
    if (iqb) {
        auto run = [&](auto JI) {
            static_cast<MvJob &>(JI) = J;
            return launch_mv_job(JI, P, smem, out_dim, st);
        };
        switch (t) {
        case T_IQ2_XXS: return run(MvIqJob<T_IQ2_XXS>{});
        case T_IQ2_XS: return run(MvIqJob<T_IQ2_XS>{});
        case T_IQ3_XXS: return run(MvIqJob<T_IQ3_XXS>{});
        default: return run(MvIqJob<T_IQ1_S>{});
        }
    }
    return launch_mv_job(J, P, smem, out_dim, st);
}

// Two activation vectors per pass over the weights (formats with
// dual_format): MMA columns 0-3 carry vector 0's limbs, 4-7 vector 1's, so
// each codebook row unpacked into A serves both.
template <int T>
struct MvPairJob : MvJob {
    static constexpr int kIq = T;
    static constexpr bool kDual = true;
    int64_t in_dim;
    float *y2;
    __device__ uint32_t tab_mask(const uint8_t *) const { return 3u; }
    __device__ int n_tab() const { return 2; }
    __device__ const float *tab_src(int t) const { return x + (int64_t)t * in_dim; }
    __device__ void finish(const uint8_t *, int64_t u, const QUnit &, double v, int lane) const {
        const int64_t r = u * 16 + (lane & 15);
        if (r < out_dim) (lane < 16 ? y : y2)[r] = (float)v;
    }
};

// n_vec >= 2 on the engine: vectors in pairs (one launch per pair; an odd
// last vector runs alone). Each pair reads the weights once.
static int launch_matvec_pairs(int t, const void *w, const float *x, float *y, int64_t out_dim, int64_t in_dim,
                               int64_t rb, int64_t n_vec, cudaStream_t st) {
    DevInfo &di = dev_info();
    const IqLayout iql = iq_layout(t, t);
    const int nsb = (int)(in_dim / kQK);
    const int64_t tabs = 2 * (int64_t)nsb * kTabSB + iql.bytes;
    int nsplit = 0;
    const int sbs = qe_sbs(t, nsb, qe_row_budget(di.smem_optin, tabs, 3), nsplit);
    if (!sbs) return fail("matvec_q: no tensor-core split for type %d (pairs)", t);
    QeLayout P;
    int cg, G;
    mv_groups(t, sbs, (int64_t)sbs * qe_sb_bytes(t), tabs, (out_dim + 15) / 16, cg, G);
    int64_t smem = 0;
    if (!qe_layout(P, G, cg, (uint32_t)sbs * qe_sb_bytes(t), 2, nsb, di.smem_optin, smem, &iql, 32))
        return fail("matvec_q: paired tile needs %lld B of shared memory", (long long)smem);
    P.err = di.err;
    for (int64_t v = 0; v < n_vec; v += 2) {
        if (v + 1 == n_vec) {
            if (!launch_matvec_engine(t, w, x + v * in_dim, y + v * out_dim, out_dim, in_dim, rb, st)) return 0;
            break;
        }
        auto run = [&](auto J) {
            J.w = reinterpret_cast<const uint8_t *>(w);
            J.rb = rb; J.out_dim = out_dim; J.type = t; J.nsb = nsb; J.sbs = sbs; J.nsplit = nsplit;
            J.x = x + v * in_dim; J.y = y + v * out_dim; J.y2 = y + (v + 1) * out_dim; J.in_dim = in_dim;
            return launch_mv_job(J, P, smem, out_dim, st);
        };
        int ok = 0;
        switch (t) {
        case T_IQ2_XXS: ok = run(MvPairJob<T_IQ2_XXS>{}); break;
        case T_IQ3_XXS: ok = run(MvPairJob<T_IQ3_XXS>{}); break;
        default: ok = run(MvPairJob<T_IQ1_S>{}); break;
        }
        if (!ok) return 0;
    }
    return 1;
}

// Up to kMvMulti matrices of one format and input width sharing one input x
// (the q/k/v/r projections of an attention layer) in one engine launch: the
// matrices' 16-row tiles are numbered consecutively, so small matrices do
// not leave SMs idle and the launch count drops.
constexpr int kMvMulti = 4;
struct MvNJob {
    const uint8_t *w[kMvMulti];
    float *y[kMvMulti];
    int64_t rows[kMvMulti];
    int64_t u0[kMvMulti + 1];          // first unit of each matrix
    int n;
    int64_t rb;
    int type, nsb, sbs, nsplit;
    const float *x;
    __device__ void init() {}
    __device__ void setup(uint8_t *, int, bool) {}
    __device__ int64_t n_units() const { return u0[n]; }
    __device__ bool needs_dep(int64_t) const { return false; }
    __device__ uint32_t tab_mask(const uint8_t *) const { return 1u; }
    __device__ int splits(const uint8_t *, int64_t) const { return nsplit; }
    __device__ int which(int64_t u) const {
        int m = 0;
#pragma unroll
        for (int i = 1; i < kMvMulti; i++) m += (i < n && u >= u0[i]) ? 1 : 0;
        return m;
    }
    __device__ void unit(const uint8_t *, int64_t u, QUnit &U) const {
        const int m = which(u);
        const int64_t r0 = (u - u0[m]) * 16;
        const int nr = (int)imin64(16, rows[m] - r0);
        U.type = type; U.nsb = nsb; U.sbs = sbs; U.nsplit = nsplit; U.rb = rb; U.tab = 0;
        U.nlo = min(8, nr);
        U.nhi = max(0, nr - 8);
        U.lo = w[m] + r0 * rb;
        U.hi = U.lo + 8 * rb;
    }
    __device__ int n_tab() const { return 1; }
    __device__ const float *tab_src(int) const { return x; }
    __device__ void finish(const uint8_t *, int64_t u, const QUnit &, double v, int lane) const {
        const int m = which(u);
        const int64_t r = (u - u0[m]) * 16 + lane;
        if (lane < 16 && r < rows[m]) y[m][r] = (float)v;
    }
};

// Can this call run on the engine? in_dim whole superblocks, x 16-byte
// aligned (float4 table loads), every row at the same address mod 4 with
// 4-byte aligned superblocks (2-byte for Q3_K).
static bool engine_ok(int t, const void *w, const float *x, int64_t in_dim, int64_t rb, int64_t n_vec) {
    const uintptr_t wa = reinterpret_cast<uintptr_t>(w);
    return (mma_format(t) || iq_format(t)) && n_vec == 1 && in_dim % kQK == 0 && in_dim / kQK <= 80 &&
           rb % 4 == 0 && (wa & ((t == T_Q3_K || iq_format(t)) ? 1 : 3)) == 0 &&
           (reinterpret_cast<uintptr_t>(x) & 15) == 0;
}

// Exact dequantisation: one thread per 32-element part.
__global__ void k_dequant(int t, const uint8_t *raw, float *out, int64_t n) {
    const int64_t part = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t first = part * 32;
    if (first >= n) return;
    const int64_t sb = first / kQK;
    const int p = (int)((first % kQK) / 32);
    const int nvalid = (int)imin64(32, n - first);
    float y[32];
    decode_part_exact(t, raw + sb * fmt_sb_bytes(t), p, y, nvalid);
    for (int i = 0; i < nvalid; i++) out[first + i] = y[i];
}

// ------------------------------------------------------- batched IQ path
// n_vec > 1 for the IQ grid formats. k_matvec decodes every weight once per
// vector; here a lane decodes its 32-weight part once into exact floats
// (grid byte with the sign folded into the weight instead of the
// activation: the product is bit-identical) and reuses it for up to kIqVB
// vectors staged in shared memory. Per vector the part's fp32 accumulation
// order is the one of dot_iq2_xxs / dot_iq2_xs / dot_iq3_xxs / dot_iq1_s, so
// each row's value equals the n_vec = 1 result of that vector.
//
// Shared layout: x[v][in_dim] with the 16-byte chunk c of part P stored at
// chunk c ^ (P & 7) (8 consecutive parts -- one quarter-warp of 16-byte
// loads -- hit distinct banks), then the IQ1_S part sums S[v][P] =
// sum(x[0..15]) + sum(x[16..31]) in dot_iq1_s's order.
// Grid (vector groups, row blocks): the groups of one row block are
// adjacent block indices, so the later groups read the rows from L2.
constexpr int kIqVB = 8;
constexpr int kIqWarps = 16;
constexpr int kIqRowsPerWarp = 4;
constexpr int kIqPL = 4;    // parts a lane loads ahead

__device__ __forceinline__ uint32_t g16(const uint8_t *p) { return __ldg(reinterpret_cast<const unsigned short *>(p)); }
__device__ __forceinline__ uint32_t g32(const uint8_t *p) { return g16(p) | (g16(p + 2) << 16); }
__device__ __forceinline__ float g_half(const uint8_t *p) { return __half2float(__ushort_as_half((unsigned short)g16(p))); }

// Raw bytes of part p (0..7) of block b, loaded before any decode so a
// lane's loads for a whole row are in flight together.
struct IqRaw { uint32_t d, a, b, c; };

template <int T>
__device__ __forceinline__ IqRaw iq_load(const uint8_t *b, int p) {
    IqRaw r;
    r.d = g16(b);
    if constexpr (T == T_IQ2_XXS) {
        r.a = g32(b + 2 + 8 * p); r.b = g32(b + 6 + 8 * p); r.c = 0;
    } else if constexpr (T == T_IQ2_XS) {
        r.a = g32(b + 2 + 8 * p); r.b = g32(b + 6 + 8 * p); r.c = g16(b + 66 + (p & ~1)) >> (8 * (p & 1)) & 255;
    } else if constexpr (T == T_IQ3_XXS) {
        r.a = g32(b + 66 + 4 * p); r.b = g32(b + 2 + 8 * p); r.c = g32(b + 6 + 8 * p);
    } else {   // T_IQ1_S
        r.a = g16(b + 34 + 2 * p); r.b = g32(b + 2 + 4 * p); r.c = 0;
    }
    return r;
}

// 32 weights w of a loaded part (exact floats) and the scale terms the
// combine needs (sa, sb: see iq_combine).
template <int T>
__device__ __forceinline__ void iq_decode(const IqRaw &r, float (&w)[32], float &sa, float &sb) {
    const float d = __half2float(__ushort_as_half((unsigned short)r.d));
    if constexpr (T == T_IQ2_XXS) {
        const uint32_t idx = r.a, sg = r.b;
        sa = __fmul_rn(__fmul_rn(d, __fadd_rn(0.5f, (float)(sg >> 28))), 0.25f);
        sb = 0.f;
#pragma unroll
        for (int l = 0; l < 4; l++) {
            const uint64_t row = sepia_iq2xxs_grid[(idx >> (8 * l)) & 255];
            const uint32_t s = sepia_ksigns_iq2xs[(sg >> (7 * l)) & 127];
#pragma unroll
            for (int j = 0; j < 4; j++) {
                w[8 * l + j] = flip_if(grid_byte_f((uint32_t)row, j), s, j);
                w[8 * l + 4 + j] = flip_if(grid_byte_f((uint32_t)(row >> 32), j), s, 4 + j);
            }
        }
    } else if constexpr (T == T_IQ2_XS) {
        const uint32_t sc = r.c;
        sa = __fmul_rn(__fmul_rn(d, __fadd_rn(0.5f, (float)(sc & 15))), 0.25f);
        sb = __fmul_rn(__fmul_rn(d, __fadd_rn(0.5f, (float)(sc >> 4))), 0.25f);
#pragma unroll
        for (int l = 0; l < 4; l++) {
            const uint32_t q = ((l < 2 ? r.a : r.b) >> (16 * (l & 1))) & 0xFFFFu;
            const uint64_t row = sepia_iq2xs_grid[q & 511];
            const uint32_t s = sepia_ksigns_iq2xs[q >> 9];
#pragma unroll
            for (int j = 0; j < 4; j++) {
                w[8 * l + j] = flip_if(grid_byte_f((uint32_t)row, j), s, j);
                w[8 * l + 4 + j] = flip_if(grid_byte_f((uint32_t)(row >> 32), j), s, 4 + j);
            }
        }
    } else if constexpr (T == T_IQ3_XXS) {
        const uint32_t a = r.a;
        sa = __fmul_rn(__fmul_rn(d, __fadd_rn(0.5f, (float)(a >> 28))), 0.5f);
        sb = 0.f;
#pragma unroll
        for (int l = 0; l < 4; l++) {
            const uint32_t qq = (l < 2) ? r.b : r.c;
            const uint32_t s = sepia_ksigns_iq2xs[(a >> (7 * l)) & 127];
            const uint32_t g1 = sepia_iq3xxs_grid[(qq >> (16 * (l & 1))) & 255];
            const uint32_t g2 = sepia_iq3xxs_grid[(qq >> (16 * (l & 1) + 8)) & 255];
#pragma unroll
            for (int j = 0; j < 4; j++) {
                w[8 * l + j] = flip_if(grid_byte_f(g1, j), s, j);
                w[8 * l + 4 + j] = flip_if(grid_byte_f(g2, j), s, 4 + j);
            }
        }
    } else {   // T_IQ1_S
        const uint32_t h = r.a, qs = r.b;
        sa = __fmul_rn(d, (float)(2 * ((h >> 12) & 7) + 1));
        sb = (h & 0x8000u) ? -0.125f : 0.125f;
#pragma unroll
        for (int l = 0; l < 4; l++) {
            const uint64_t row = sepia_iq1s_grid[((qs >> (8 * l)) & 255) | (((h >> (3 * l)) & 7) << 8)];
            const uint32_t lo = plus1_bytes((uint32_t)row), hi = plus1_bytes((uint32_t)(row >> 32));
#pragma unroll
            for (int j = 0; j < 4; j++) {
                w[8 * l + j] = grid_g_f(lo, j);
                w[8 * l + 4 + j] = grid_g_f(hi, j);
            }
        }
    }
}

// Dot of decoded part w with one vector's part (swizzled chunks at xs).
template <int T>
__device__ __forceinline__ float iq_combine(const float (&w)[32], const float *xs, int sw, float sa, float sb,
                                            float S) {
    float x[32];
#pragma unroll
    for (int c = 0; c < 8; c++) {
        const float4 f = *reinterpret_cast<const float4 *>(xs + 4 * (c ^ sw));
        x[4 * c] = f.x; x[4 * c + 1] = f.y; x[4 * c + 2] = f.z; x[4 * c + 3] = f.w;
    }
    if constexpr (T == T_IQ2_XS) {
        float t[2] = {0.f, 0.f};
#pragma unroll
        for (int l = 0; l < 4; l++) {
            float a = 0.f;
#pragma unroll
            for (int j = 0; j < 4; j++) {
                a = fmaf(w[8 * l + j], x[8 * l + j], a);
                a = fmaf(w[8 * l + 4 + j], x[8 * l + 4 + j], a);
            }
            t[l >> 1] += a;
        }
        return fmaf(sa, t[0], sb * t[1]);
    } else {
        float t0 = 0.f, t1 = 0.f;
#pragma unroll
        for (int l = 0; l < 4; l++)
#pragma unroll
            for (int j = 0; j < 4; j++) {
                t0 = fmaf(w[8 * l + j], x[8 * l + j], t0);
                t1 = fmaf(w[8 * l + 4 + j], x[8 * l + 4 + j], t1);
            }
        if constexpr (T == T_IQ1_S) return sa * fmaf(sb, S, t0 + t1);
        else return sa * (t0 + t1);
    }
}

struct IqbParams {
    const uint8_t *w;
    int64_t row_bytes, out_dim, in_dim;
    const float *x;
    float *y;
    int n_vec, vb;   // vectors in all, vectors per group (<= kIqVB)
    int rpw;         // rows per warp (<= kIqRowsPerWarp)
};

template <int T>
__global__ void __launch_bounds__(kIqWarps * 32) k_matvec_iqb(const IqbParams P) {
    extern __shared__ __align__(16) float xsm[];
    const int nparts = (int)(P.in_dim / 32);
    float *ssum = xsm + (size_t)P.vb * P.in_dim;
    const int v0 = blockIdx.x * P.vb;
    const int nv = min(P.vb, P.n_vec - v0);
    const int64_t in4 = P.in_dim / 4;
    griddep_wait();
    griddep_launch();
    for (int64_t i = threadIdx.x; i < nv * in4; i += blockDim.x) {
        const int v = (int)(i / in4);
        const int64_t c4 = i - v * in4;
        const int64_t part = c4 >> 3;
        const int c = (int)(c4 & 7);
        const float4 f = __ldg(reinterpret_cast<const float4 *>(P.x + (int64_t)(v0 + v) * P.in_dim) + c4);
        *reinterpret_cast<float4 *>(xsm + (size_t)v * P.in_dim + part * 32 + 4 * (c ^ (int)(part & 7))) = f;
    }
    __syncthreads();
    if constexpr (T == T_IQ1_S) {
        for (int i = threadIdx.x; i < nv * nparts; i += blockDim.x) {
            const int v = i / nparts, part = i - v * nparts;
            const float *xp = xsm + (size_t)v * P.in_dim + part * 32;
            float a = 0.f, b = 0.f;
#pragma unroll
            for (int k = 0; k < 16; k++) {
                a += xp[4 * ((k >> 2) ^ (part & 7)) + (k & 3)];
                b += xp[4 * (((k + 16) >> 2) ^ (part & 7)) + (k & 3)];
            }
            ssum[i] = a + b;
        }
        __syncthreads();
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int bb = fmt_block_bytes(T);
    const int64_t rbase = (int64_t)blockIdx.y * (kIqWarps * P.rpw);
    for (int rr = 0; rr < P.rpw; rr++) {
        const int64_t row = rbase + (int64_t)rr * kIqWarps + warp;
        if (row >= P.out_dim) break;
        const uint8_t *wr = P.w + row * P.row_bytes;
        double acc[kIqVB];
#pragma unroll
        for (int v = 0; v < kIqVB; v++) acc[v] = 0.0;
        for (int pc = lane; pc < nparts; pc += 32 * kIqPL) {
            IqRaw raw[kIqPL];
#pragma unroll
            for (int i = 0; i < kIqPL; i++) {
                const int part = pc + 32 * i;
                if (part < nparts) raw[i] = iq_load<T>(wr + (int64_t)(part >> 3) * bb, part & 7);
            }
#pragma unroll
            for (int i = 0; i < kIqPL; i++) {
                const int part = pc + 32 * i;
                if (part < nparts) {
                    float wv[32], sa, sb;
                    iq_decode<T>(raw[i], wv, sa, sb);
#pragma unroll
                    for (int v = 0; v < kIqVB; v++) {
                        if (v < nv) {
                            const float S = (T == T_IQ1_S) ? ssum[v * nparts + part] : 0.f;
                            acc[v] += (double)iq_combine<T>(wv, xsm + (size_t)v * P.in_dim + part * 32, part & 7,
                                                            sa, sb, S);
                        }
                    }
                }
            }
        }
#pragma unroll
        for (int v = 0; v < kIqVB; v++) {
            if (v < nv) {
                double a = acc[v];
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
                if (lane == 0) P.y[(int64_t)(v0 + v) * P.out_dim + row] = (float)a;
            }
        }
    }
}

static bool iqb_type(int t) { return t == T_IQ2_XXS || t == T_IQ2_XS || t == T_IQ3_XXS || t == T_IQ1_S; }

static int launch_matvec_iqb(int t, const void *w, const float *x, float *y, int64_t out_dim, int64_t in_dim,
                             int64_t rb, int64_t n_vec, cudaStream_t st) {
    DevInfo &di = dev_info();
    const int64_t nparts = in_dim / 32;
    const int64_t per_vec = 4 * (in_dim + (t == T_IQ1_S ? nparts : 0));   // x (+ IQ1_S part sums)
    const int vb = (int)std::min<int64_t>(kIqVB, std::min<int64_t>(n_vec, di.smem_optin / per_vec));
    const size_t smem = (size_t)vb * per_vec;
    const void *fn = nullptr;
    switch (t) {
    case T_IQ2_XXS: fn = (const void *)k_matvec_iqb<T_IQ2_XXS>; break;
    case T_IQ2_XS: fn = (const void *)k_matvec_iqb<T_IQ2_XS>; break;
    case T_IQ3_XXS: fn = (const void *)k_matvec_iqb<T_IQ3_XXS>; break;
    default: fn = (const void *)k_matvec_iqb<T_IQ1_S>; break;
    }
    if (!ensure_smem(fn, (int)smem)) return 0;
    IqbParams P;
    P.w = reinterpret_cast<const uint8_t *>(w);
    P.row_bytes = rb; P.out_dim = out_dim; P.in_dim = in_dim;
    P.x = x; P.y = y; P.n_vec = (int)n_vec; P.vb = vb;
    // rows per warp: as many as keep >= 2 CTAs per SM in the grid (each CTA
    // stages its vectors once, so fewer, longer CTAs save L2 reads)
    const int64_t groups = (n_vec + vb - 1) / vb;
    P.rpw = (int)std::max<int64_t>(1, std::min<int64_t>(kIqRowsPerWarp,
                                                        out_dim * groups / ((int64_t)kIqWarps * 2 * di.sm_count)));
    const int64_t rows_per_cta = (int64_t)kIqWarps * P.rpw;
    dim3 grid((unsigned)groups, (unsigned)((out_dim + rows_per_cta - 1) / rows_per_cta));
    switch (t) {
    case T_IQ2_XXS: k_matvec_iqb<T_IQ2_XXS><<<grid, kIqWarps * 32, smem, st>>>(P); break;
    case T_IQ2_XS: k_matvec_iqb<T_IQ2_XS><<<grid, kIqWarps * 32, smem, st>>>(P); break;
    case T_IQ3_XXS: k_matvec_iqb<T_IQ3_XXS><<<grid, kIqWarps * 32, smem, st>>>(P); break;
    default: k_matvec_iqb<T_IQ1_S><<<grid, kIqWarps * 32, smem, st>>>(P); break;
    }
    return check(cudaGetLastError(), "matvec_q (batched IQ) launch");
}

// Can this call take the batched IQ path? Several vectors, whole
// superblocks, 2-byte aligned weights and rows, 16-byte aligned x, and at
// least one vector's x (plus part sums) fits in shared memory.
static bool iqb_ok(int t, const void *w, const float *x, int64_t in_dim, int64_t rb, int64_t n_vec) {
    return iqb_type(t) && n_vec > 1 && in_dim % kQK == 0 && rb % 2 == 0 &&
           (reinterpret_cast<uintptr_t>(w) & 1) == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0 &&
           4 * (in_dim + in_dim / 32) <= (int64_t)dev_info().smem_optin && (n_vec + kIqVB - 1) / kIqVB < 65536;
}

// ----------------------------------------------------------------- host side
typedef void (*MvKernel)(const MvParams);

template <int T>
static MvKernel pick_mv(int trw, int c) {
    if (trw == 8) return c == 1 ? k_matvec<T, 8, 1> : k_matvec<T, 8, 2>;
    return c == 1 ? k_matvec<T, 2, 1> : k_matvec<T, 2, 2>;
}

static MvKernel mv_kernel(int t, int trw, int c) {
    switch (t) {
    case T_F32: return pick_mv<T_F32>(trw, c);
    case T_F16: return pick_mv<T_F16>(trw, c);
    case T_Q8_0: return pick_mv<T_Q8_0>(trw, c);
    case T_Q2_K: return pick_mv<T_Q2_K>(trw, c);
    case T_Q3_K: return pick_mv<T_Q3_K>(trw, c);
    case T_Q4_K: return pick_mv<T_Q4_K>(trw, c);
    case T_Q5_K: return pick_mv<T_Q5_K>(trw, c);
    case T_Q6_K: return pick_mv<T_Q6_K>(trw, c);
    case T_IQ2_XXS: return pick_mv<T_IQ2_XXS>(trw, c);
    case T_IQ2_XS: return pick_mv<T_IQ2_XS>(trw, c);
    case T_IQ3_XXS: return pick_mv<T_IQ3_XXS>(trw, c);
    case T_IQ1_S: return pick_mv<T_IQ1_S>(trw, c);
    case T_IQ4_XS: return pick_mv<T_IQ4_XS>(trw, c);
    default: return nullptr;
    }
}

int launch_matvec_q(int t, const void *w, const float *x, float *y, int64_t out_dim, int64_t in_dim,
                    int64_t n_vec, cudaStream_t st) {
    if (out_dim <= 0 || in_dim <= 0 || n_vec <= 0 || n_vec > (1 << 20))
        return fail("matvec_q: bad dims out=%lld in=%lld n_vec=%lld", (long long)out_dim, (long long)in_dim,
                    (long long)n_vec);
    const int64_t rb = host_row_bytes(t, in_dim);
    if (rb <= 0) return fail("matvec_q: unsupported ggml type %d or in_dim %lld not block-aligned", t, (long long)in_dim);
    if (!w || !x || !y) return fail("matvec_q: null pointer");
    // K-quants with aligned rows run on the integer tensor cores
    if (engine_ok(t, w, x, in_dim, rb, n_vec)) return launch_matvec_engine(t, w, x, y, out_dim, in_dim, rb, st);
    // (with fewer rows the fixed cost of one launch per pair loses to the
    // CUDA-core batch kernel: measured at 2048 rows x 16 vectors)
    if (n_vec > 1 && out_dim >= 4096 && dual_format(t) && engine_ok(t, w, x, in_dim, rb, 1))
        return launch_matvec_pairs(t, w, x, y, out_dim, in_dim, rb, n_vec, st);
    if (iqb_ok(t, w, x, in_dim, rb, n_vec)) return launch_matvec_iqb(t, w, x, y, out_dim, in_dim, rb, n_vec, st);
    DevInfo &di = dev_info();
    const int nsb = (int)((in_dim + kQK - 1) / kQK);
    int c = 1, nwc = (nsb + 3) / 4;
    if (nwc > 16) { c = 2; nwc = (nsb + 7) / 8; }
    if (nwc > 16) return fail("matvec_q: in_dim %lld too large (max 32768)", (long long)in_dim);
    int G = 1;
    while (nwc * G * 2 <= 16) G *= 2;         // up to 16 consumer warps: latency hiding
    int trw = 8;
    if ((int64_t)trw * G * rb > 80 * 1024) trw = 2;
    while (G > 1 && (int64_t)trw * G * rb > 80 * 1024) G /= 2;
    if ((int64_t)trw * G * rb > 160 * 1024) return fail("matvec_q: rows of %lld bytes too large", (long long)rb);
    if (t == T_F32 && 2 * (int64_t)slot_bytes_for((uint64_t)trw * G * rb) + 4096 > (int64_t)di.smem_optin) {
        // f32 rows too long to double-buffer: one warp per row straight from
        // global memory (same double-accumulated dot)
        for (int64_t v = 0; v < n_vec; v++)
            if (!op_matvec_f32(reinterpret_cast<const float *>(w), x + v * in_dim, y + v * out_dim, out_dim, in_dim, st))
                return 0;
        return 1;
    }
    const int TR = trw * G;
    const uint32_t slot = slot_bytes_for((uint64_t)TR * rb);
    const int n_cons = nwc * G;
    const int head = 128 + ((n_cons * trw * 8 + 127) & ~127);
    int stages = kMvStagesMax;
    while (stages > 2 && head + (int64_t)stages * slot > (int64_t)di.smem_optin) stages--;
    const int64_t smem = head + (int64_t)stages * slot;
    if (smem > di.smem_optin) return fail("matvec_q: tile needs %lld B of shared memory", (long long)smem);
    MvKernel kern = mv_kernel(t, trw, c);
    if (!kern) return fail("matvec_q: unsupported ggml type %d", t);
    if (!ensure_smem((const void *)kern, (int)smem)) return 0;
    MvParams P;
    P.w = reinterpret_cast<const uint8_t *>(w);
    P.row_bytes = rb;
    P.x = x; P.y = y;
    P.out_dim = out_dim; P.in_dim = in_dim; P.n_vec = (int)n_vec;
    P.nsb = nsb; P.nwc = nwc; P.G = G; P.stages = stages; P.slot_bytes = slot;
    P.num_units = (out_dim + TR - 1) / TR;
    P.err = di.err;
    int per_sm = 0;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, (n_cons + 1) * 32, (size_t)smem);
    if (per_sm < 1) per_sm = 1;
    const int64_t grid = std::min<int64_t>(P.num_units, (int64_t)di.sm_count * per_sm);
    if (!check(launch_pdl(kern, (unsigned)grid, (n_cons + 1) * 32, (size_t)smem, st, P), "matvec_q launch")) return 0;
    return check(cudaGetLastError(), "matvec_q launch");
}

// y_i = W_i x for n <= 4 matrices of one format and input width: one engine
// launch when every matrix can run on it, else one launch per matrix.
int launch_matvec_q_multi(int n, int t, const void *const *w, const int64_t *rows, int64_t in_dim, const float *x,
                          float *const *y, cudaStream_t st) {
    if (n < 1 || n > kMvMulti) return fail("matvec_q_multi: %d matrices (1..%d)", n, kMvMulti);
    const int64_t rb = host_row_bytes(t, in_dim);
    bool eng = rb > 0 && mma_format(t);     // (the multi job stages no IQ codebooks)
    for (int i = 0; i < n && eng; i++) eng = rows[i] > 0 && engine_ok(t, w[i], x, in_dim, rb, 1);
    if (!eng) {
        for (int i = 0; i < n; i++)
            if (!launch_matvec_q(t, w[i], x, y[i], rows[i], in_dim, 1, st)) return 0;
        return 1;
    }
    DevInfo &di = dev_info();
    MvNJob J;
    J.n = n; J.rb = rb; J.type = t; J.nsb = (int)(in_dim / kQK); J.x = x;
    J.u0[0] = 0;
    for (int i = 0; i < kMvMulti; i++) {
        J.w[i] = i < n ? reinterpret_cast<const uint8_t *>(w[i]) : nullptr;
        J.y[i] = i < n ? y[i] : nullptr;
        J.rows[i] = i < n ? rows[i] : 0;
        J.u0[i + 1] = J.u0[i] + (i < n ? (rows[i] + 15) / 16 : 0);
    }
    J.sbs = qe_sbs(t, J.nsb, qe_row_budget_for(di.smem_optin, (int64_t)J.nsb * kTabSB, rb), J.nsplit);
    if (!J.sbs) return fail("matvec_q_multi: no tensor-core split for type %d", t);
    QeLayout P;
    int cg, G;
    mv_groups(t, J.sbs, rb, (int64_t)J.nsb * kTabSB, J.u0[n], cg, G);
    int64_t smem = 0;
    if (!qe_layout(P, G, cg, (uint32_t)J.sbs * qe_sb_bytes(t), 1, J.nsb, di.smem_optin, smem))
        return fail("matvec_q_multi: tensor-core tile needs %lld B of shared memory", (long long)smem);
    P.err = di.err;
    const void *fn = (const void *)k_qengine<MvNJob>;
    if (!ensure_smem(fn, (int)smem)) return 0;
    const int64_t grid = std::min<int64_t>(J.u0[n], (int64_t)di.sm_count);
    return check(launch_pdl(k_qengine<MvNJob>, (unsigned)grid, (P.G * P.cg + 2) * 32, (size_t)smem, st, J, P),
                 "matvec_q_multi launch");
}

int launch_dequant(int t, const void *raw, float *out, int64_t n, cudaStream_t st) {
    const int e = host_block_elems(t);
    if (e == 0) return fail("dequant: unsupported ggml type %d", t);
    if (n <= 0 || n % e) return fail("dequant: n=%lld not a multiple of block size %d (type %d)", (long long)n, e, t);
    if (!raw || !out) return fail("dequant: null pointer");
    const int64_t parts = (n + 31) / 32;
    const int threads = 128;
    k_dequant<<<(unsigned)((parts + threads - 1) / threads), threads, 0, st>>>(t, reinterpret_cast<const uint8_t *>(raw), out, n);
    return check(cudaGetLastError(), "dequant launch");
}

}  // namespace sepia

extern "C" int sepia_cuda_matvec_q(int ggml_type, const void *w, const float *x, float *y, int64_t out_dim,
                                   int64_t in_dim, int64_t n_vec, void *stream) {
    return sepia::launch_matvec_q(ggml_type, w, x, y, out_dim, in_dim, n_vec, sepia::as_stream(stream));
}

extern "C" int sepia_cuda_dequant(int ggml_type, const void *raw, float *out, int64_t n, void *stream) {
    return sepia::launch_dequant(ggml_type, raw, out, n, sepia::as_stream(stream));
}

// ------------------------------------------------------------ test hook
// Failure detection without a GPU fault: the engine's producer announces 16
// more bytes than it copies, so the first stage never completes; every
// waiting role gives up after `wait_cycles` clock cycles, records
// kErrWaitTimeout in the device error word and returns. The copies it did
// issue all land before the CTA exits. Used only by the tests.
extern "C" int sepia_cuda_test_engine_timeout(int ggml_type, const void *w, const float *x, float *y,
                                              int64_t out_dim, int64_t in_dim, long long wait_cycles,
                                              void *stream) {
    using namespace sepia;
    const int64_t rb = host_row_bytes(ggml_type, in_dim);
    if (rb <= 0 || !engine_ok(ggml_type, w, x, in_dim, rb, 1))
        return fail("test_engine_timeout: shape not on the tensor-core engine");
    if (wait_cycles <= 0 || wait_cycles > kWaitCycles) return fail("test_engine_timeout: bad wait limit");
    return launch_matvec_engine(ggml_type, w, x, y, out_dim, in_dim, rb, as_stream(stream), wait_cycles, 16u);
}

extern "C" void *sepia_cuda_lib_stream(void) { return (void *)sepia::lib_stream(); }
