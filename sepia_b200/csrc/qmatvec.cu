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


static int launch_matvec_engine(int t, const void *w, const float *x, float *y, int64_t out_dim, int64_t in_dim,
                                int64_t rb, cudaStream_t st) {
    DevInfo &di = dev_info();
    MvJob J;
    J.w = reinterpret_cast<const uint8_t *>(w);
    J.rb = rb; J.out_dim = out_dim; J.type = t;
    J.nsb = (int)(in_dim / kQK);
    J.x = x; J.y = y;
    J.sbs = qe_sbs(t, J.nsb, qe_row_budget(di.smem_optin, (int64_t)J.nsb * kTabSB), J.nsplit);
    if (!J.sbs) return fail("matvec_q: no tensor-core split for type %d", t);
    QeLayout P;
    int cg, G;
    qe_groups(J.sbs, cg, G);
    int64_t smem = 0;
    if (!qe_layout(P, G, cg, (uint32_t)J.sbs * qe_sb_bytes(t), 1, J.nsb, di.smem_optin, smem))
        return fail("matvec_q: tensor-core tile needs %lld B of shared memory", (long long)smem);
    P.err = di.err;
    const void *fn = (const void *)k_qengine<MvJob>;
    if (!ensure_smem(fn, (int)smem)) return 0;
    const int64_t units = (out_dim + 15) / 16;
    const int64_t grid = std::min<int64_t>(units, (int64_t)di.sm_count);
    k_qengine<MvJob><<<(unsigned)grid, (P.G * P.cg + 2) * 32, (size_t)smem, st>>>(J, P);
    return check(cudaGetLastError(), "matvec_q (tensor cores) launch");
}

// Can this call run on the engine? in_dim whole superblocks, x 16-byte
// aligned (float4 table loads), every row at the same address mod 4 with
// 4-byte aligned superblocks (2-byte for Q3_K).
static bool engine_ok(int t, const void *w, const float *x, int64_t in_dim, int64_t rb, int64_t n_vec) {
    const uintptr_t wa = reinterpret_cast<uintptr_t>(w);
    return mma_format(t) && n_vec == 1 && in_dim % kQK == 0 && in_dim / kQK <= 64 && rb % 4 == 0 &&
           (wa & (t == T_Q3_K ? 1 : 3)) == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0;
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
    kern<<<(unsigned)grid, (n_cons + 1) * 32, (size_t)smem, st>>>(P);
    return check(cudaGetLastError(), "matvec_q launch");
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
