// sepia_b200/csrc/moe.cu -- one MoE layer for one token, entirely on device.
//
// Replaces the reference's host-synchronised sequence in
// real_mlp_moe_forward_gpu (src/sepia.c:3831-3974: router matvec, SYNC,
// host moe_route_select, per-expert gate/up/silu/down dispatches, SYNC, host
// combine) with three kernels and no host round trip:
//   k_router      logits = W_r x (fp64 accumulation, as dotf does), then the
//                 last CTA to finish runs moe_route_select (src/sepia.c:
//                 1329-1375): sigmoid + selection bias, top-k by the strict
//                 '>' scan (lowest index wins ties), log-sigmoid/LSE weights
//                 over the k raw logits plus the shared-sink logits.
//   k_gateup      for every selected routed expert and every shared expert,
//                 gate and up row tiles stream through shared memory and the
//                 epilogue writes h = silu(g)*u (times gamma for shared
//                 experts, mlp_moe_forward's order, src/sepia.c:1432-1444).
//   k_down        row tiles of every active expert's down matrix; the
//                 epilogue sums sum_j w_j*E_j + sum_s S_s in the reference
//                 order (routed j = 0..k-1, then shared) -- or, for expert
//                 sharding, writes each slot's term separately so an
//                 all-reduce plus k_combine reproduces the same sums bit for
//                 bit on any number of GPUs.
#include "moe_dev.cuh"
#include "stream.cuh"

#include <algorithm>
#include <cstring>
#include <mutex>

namespace sepia {

// Router GEMV: the [n_total, hidden] f32 matrix is cut into chunks of
// kRouterChunk consecutive elements of one row; one warp per chunk, every
// lane issuing all of its 16-byte loads before the first FMA, so the whole
// matrix is in flight at once (a decode router is too small to reach HBM
// bandwidth any other way). Chunk partials are fp64 and are summed per row
// in chunk order by the last CTA, so the result does not depend on
// scheduling. That CTA then runs the selection (one warp: the serial parts
// are short and __syncthreads rounds would dominate).
__global__ void __launch_bounds__(kRouterMaxChunks * 32) k_router(const MoeDev L, const float *x, float *logits,
                                                                   int32_t *topk_idx, float *weights,
                                                                   unsigned int *counter, float2 *row_out) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n_total = L.n_routed + L.n_shared;
    const int cpr = router_chunks(L.hidden);
    const int row = blockIdx.x;
    __shared__ double s_part[kRouterMaxChunks];
    if (warp < cpr) {
        const int64_t c0 = (int64_t)warp * kRouterChunk;
        const int64_t n = imin64(kRouterChunk, L.hidden - c0);
        const float *w = L.router_w + (int64_t)row * L.hidden + c0;
        const float *xc = x + c0;
        double acc = 0.0;
        if (n == kRouterChunk && ((reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(xc)) & 15) == 0) {
            constexpr int kV = kRouterChunk / 128;      // float4 per lane
            float4 wv[kV], xv[kV];
            // the weights do not depend on the previous kernel: load them
            // before waiting for it (x does)
#pragma unroll
            for (int i = 0; i < kV; i++) wv[i] = __ldcs(reinterpret_cast<const float4 *>(w) + lane + 32 * i);
            griddep_wait();
#pragma unroll
            for (int i = 0; i < kV; i++) xv[i] = __ldg(reinterpret_cast<const float4 *>(xc) + lane + 32 * i);
            double a2[2] = {0.0, 0.0};
#pragma unroll
            for (int i = 0; i < kV; i++) {
                a2[i & 1] = fma((double)wv[i].x, (double)xv[i].x, a2[i & 1]);
                a2[i & 1] = fma((double)wv[i].y, (double)xv[i].y, a2[i & 1]);
                a2[i & 1] = fma((double)wv[i].z, (double)xv[i].z, a2[i & 1]);
                a2[i & 1] = fma((double)wv[i].w, (double)xv[i].w, a2[i & 1]);
            }
            acc = a2[0] + a2[1];
        } else {
            griddep_wait();
            for (int64_t i = lane; i < n; i += 32) acc = fma((double)w[i], (double)xc[i], acc);
        }
        acc = warp_sum_d(acc);
        if (lane == 0) s_part[warp] = acc;
    }
    // the row's selection score and log-sigmoid, computed here so that the
    // serial tail below only selects and normalises
    const float bias = (row < L.n_routed && threadIdx.x == 0) ? L.router_bias[row] : 0.0f;
    __syncthreads();
    // every warp is past its dependency wait: the successor may launch (it
    // reads x, final since this kernel's predecessor completed)
    griddep_launch();
    if (warp != 0) return;
    unsigned int last = 0;
    if (lane == 0) {
        if (row < n_total) {
            double t = 0.0;
            for (int c = 0; c < cpr; c++) t += s_part[c];       // chunk order
            const float l = (float)t;
            logits[row] = l;
            const float score = row < L.n_routed ? __fadd_rn(sigmoid_ref(l), bias) : 0.0f;
            row_out[row] = make_float2(score, logsigmoid_ref(l));
        }
        __threadfence();     // release this CTA's writes before counting it
        last = (atomicAdd(counter, 1u) == gridDim.x - 1) ? 1u : 0u;
    }
    if (!__shfl_sync(0xffffffffu, last, 0)) return;
    __threadfence();
    // ---- last CTA, one warp: top-k and the weights ----
    if (L.n_routed <= 8 * 32) router_select<8>(L, row_out, topk_idx, weights, lane);
    else router_select<kRouterMaxExperts / 32>(L, row_out, topk_idx, weights, lane);
    if (lane == 0) {
        *counter = 0u;   // ready for the next launch
        __threadfence();
    }
}

// Router GEMV, bulk-copy form: each CTA owns `rpc` consecutive rows of the
// [n_total, hidden] f32 matrix (contiguous bytes), fetched with one 1-D
// cp.async.bulk (TMA engine, no multicast) into shared memory before the
// dependency wait -- the weights do not depend on the previous kernel. A
// single request per CTA keeps the whole matrix in flight without the
// per-load queueing of thousands of 16-byte loads. Thread t then dots
// float4 t, t + T, ... of each row with x (held in registers) in four fp64
// chains, the warps' partials are summed in warp order, and the last CTA
// selects.
constexpr int kRouter2Threads = 256;
constexpr int kRouter2MaxPerThread = 64;       // hidden <= 64 * 256
// Optional phase timestamps for profiling builds (-DSEPIA_ROUTER_STAMPS):
// [CTA][phase] of the last router2 launch, in globaltimer nanoseconds.
#ifdef SEPIA_ROUTER_STAMPS
__device__ unsigned long long g_rstamps[256][8];
#define RS(i)                                                                        \
    do {                                                                             \
        if (threadIdx.x == 0 && blockIdx.x < 256) {                                  \
            unsigned long long t_;                                                   \
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));                   \
            g_rstamps[blockIdx.x][i] = t_;                                           \
        }                                                                            \
    } while (0)
#else
#define RS(i) do { } while (0)
#endif
__global__ void __launch_bounds__(kRouter2Threads) k_router2(const MoeDev L, const float *x, float *logits,
                                                              int32_t *topk_idx, float *weights,
                                                              unsigned int *counter, float2 *row_out, int rpc) {
    extern __shared__ __align__(128) float w_sm[];
    RS(0);
    __shared__ __align__(8) uint64_t bar;
    __shared__ double s_w[kRouter2Threads / 32], s_w2[kRouter2Threads / 32];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n_total = L.n_routed + L.n_shared;
    const int r0 = blockIdx.x * rpc;
    const int nr = min(rpc, n_total - r0);
    const int64_t H = L.hidden;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_barrier_init();
        const uint32_t bytes = (uint32_t)(nr * H * 4);
        mbar_arrive_expect_tx(&bar, bytes);
        bulk_g2s(w_sm, L.router_w + (int64_t)r0 * H, bytes, &bar);
    }
    // the successor (gate/up) may launch once this kernel's own predecessor,
    // which wrote x, has completed: it reads x before its dependency wait
    griddep_wait();
    griddep_launch();
    RS(1);
    // x as float4 (H % 4 == 0): thread t holds float4 t, t + T, ...
    constexpr int kV = kRouter2MaxPerThread / 4;
    const int64_t H4 = H / 4;
    float4 xv[kV];
#pragma unroll
    for (int j = 0; j < kV; j++) {
        const int64_t f = threadIdx.x + (int64_t)j * kRouter2Threads;
        xv[j] = f < H4 ? __ldg(reinterpret_cast<const float4 *>(x) + f) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    const int rl = lane;     // warp 0, lane q finalises row q of each pair
    __syncthreads();                       // the barrier's init is visible
    RS(2);
    const bool ok = mbar_wait(&bar, 0, L.err);
    RS(3);
    // rows two at a time: four fp64 chains per row and thread, one block
    // reduction per pair, the pair's rows finalised by two lanes at once
    for (int r = 0; r < nr; r += 2) {
        const int nrr = min(2, nr - r);
        double acc[2] = {0.0, 0.0};
        if (ok) {
#pragma unroll
            for (int q = 0; q < 2; q++) {
                if (q < nrr) {
                    const float4 *wr = reinterpret_cast<const float4 *>(w_sm + (int64_t)(r + q) * H);
                    double c[4] = {0.0, 0.0, 0.0, 0.0};
#pragma unroll
                    for (int j = 0; j < kV; j++) {
                        const int64_t f = threadIdx.x + (int64_t)j * kRouter2Threads;
                        if (f < H4) {
                            const float4 w4 = wr[f];
                            c[0] = fma((double)w4.x, (double)xv[j].x, c[0]);
                            c[1] = fma((double)w4.y, (double)xv[j].y, c[1]);
                            c[2] = fma((double)w4.z, (double)xv[j].z, c[2]);
                            c[3] = fma((double)w4.w, (double)xv[j].w, c[3]);
                        }
                    }
                    acc[q] = (c[0] + c[1]) + (c[2] + c[3]);
                }
            }
        }
        acc[0] = warp_sum_d(acc[0]);
        acc[1] = warp_sum_d(acc[1]);
        if (lane == 0) {
            s_w[warp] = acc[0];
            s_w2[warp] = acc[1];
        }
        __syncthreads();
        RS(7);
        if (warp == 0 && rl < nrr) {
            const double *sw = rl == 0 ? s_w : s_w2;
            double t = 0.0;
            for (int w = 0; w < kRouter2Threads / 32; w++) t += sw[w];       // warp order
            const int row = r0 + r + rl;
            const float l = (float)t;
            logits[row] = l;
            const float score = row < L.n_routed ? __fadd_rn(sigmoid_ref(l), L.router_bias[row]) : 0.0f;
            row_out[row] = make_float2(score, logsigmoid_ref(l));
        }
        __syncthreads();
    }
    RS(4);
    if (warp != 0) return;
    unsigned int last = 0;
    if (lane == 0) {
        __threadfence();     // release this CTA's writes before counting it
        last = (atomicAdd(counter, 1u) == gridDim.x - 1) ? 1u : 0u;
    }
    RS(5);
    if (!__shfl_sync(0xffffffffu, last, 0)) return;
    __threadfence();
    if (L.n_routed <= 8 * 32) router_select<8>(L, row_out, topk_idx, weights, lane);
    else router_select<kRouterMaxExperts / 32>(L, row_out, topk_idx, weights, lane);
    // ready for the next launch (kernel completion publishes it)
    if (lane == 0) *counter = 0u;
    RS(6);
}

// Selection only (bit-exact part of the router): top-k of given scores.
__global__ void k_topk(const float *scores, int n, int topk, int32_t *idx) {
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    for (int j = 0; j < topk; j++) {
        int best = -1;
        for (int i = 0; i < n; i++) {
            bool used = false;
            for (int q = 0; q < j; q++) used |= (idx[q] == i);
            if (used) continue;
            if (best < 0 || scores[i] > scores[best]) best = i;
        }
        idx[j] = best;
    }
}

// ============================================================== shared GEMV pieces
template <int T, int TRW>
__device__ __forceinline__ void rows_dot(const uint8_t *base, int64_t rb, int nr, int sb, int p,
                                         const XPart &xp, int64_t in_dim, float (&acc)[TRW]) {
    const int sbb = fmt_sb_bytes(T);
    const int sbs[1] = {sb};
    const XPart(&xa)[1] = *reinterpret_cast<const XPart(*)[1]>(&xp);
#pragma unroll
    for (int i = 0; i < TRW; i++)
        acc[i] = (i < nr) ? row_parts_dot<T, 1>(base + i * rb, sbb, sbs, p, xa, in_dim) : 0.0f;
}

// Generic rows: exact per-part decode + FFMA with UNSCALED activations
// (any format, including the fast ones when the kernel is runtime-typed).
template <int T, int TRW>
__device__ __forceinline__ void rows_dot_generic(const uint8_t *base, int64_t rb, int nr, int sb, int p,
                                                 const XPart &xp, int64_t in_dim, float (&acc)[TRW]) {
    const int sbb = fmt_sb_bytes(T);
    const int64_t first = (int64_t)sb * kQK + 32 * p;
    const int nvalid = first < in_dim ? (int)imin64(32, in_dim - first) : 0;
#pragma unroll
    for (int i = 0; i < TRW; i++)
        acc[i] = (i < nr && nvalid > 0) ? dot_generic(T, base + i * rb + (int64_t)sb * sbb, p, xp, nvalid) : 0.0f;
}

template <int TRW>
__device__ __forceinline__ void rows_dot_rt(int t, const uint8_t *base, int64_t rb, int nr, int sb, int p,
                                            const XPart &xp, int64_t in_dim, float (&acc)[TRW]) {
    switch (t) {
#define SEPIA_RT_CASE(TT) case TT: rows_dot_generic<TT, TRW>(base, rb, nr, sb, p, xp, in_dim, acc); break;
    SEPIA_RT_CASE(T_F32) SEPIA_RT_CASE(T_F16) SEPIA_RT_CASE(T_Q8_0) SEPIA_RT_CASE(T_Q2_K) SEPIA_RT_CASE(T_Q3_K)
    SEPIA_RT_CASE(T_Q4_K) SEPIA_RT_CASE(T_Q5_K) SEPIA_RT_CASE(T_Q6_K) SEPIA_RT_CASE(T_IQ2_XXS)
    SEPIA_RT_CASE(T_IQ2_XS) SEPIA_RT_CASE(T_IQ3_XXS) SEPIA_RT_CASE(T_IQ1_S) SEPIA_RT_CASE(T_IQ4_XS)
#undef SEPIA_RT_CASE
    default:
        for (int i = 0; i < TRW; i++) acc[i] = 0.0f;
    }
}

// TK >= 0: compile-time fast format (the kernel's activations are scaled);
// TK < 0: runtime format t through the generic decoder.
template <int TK, int TRW>
__device__ __forceinline__ void rows_dot_k(int t, const uint8_t *base, int64_t rb, int nr, int sb, int p,
                                           const XPart &xp, int64_t in_dim, float (&acc)[TRW]) {
    if constexpr (TK >= 0) rows_dot<TK, TRW>(base, rb, nr, sb, p, xp, in_dim, acc);
    else rows_dot_rt<TRW>(t, base, rb, nr, sb, p, xp, in_dim, acc);
}

// ============================================================== gate/up + SwiGLU
struct GuParams {
    MoeDev L;
    const float *x;
    const int32_t *idx;
    const float *weights;
    float *h;                 // [slots, ff]
    int tr_routed, tr_shared; // rows per unit for each kind
    int nwc;                  // column warps (per matrix group)
    int stages;
    uint32_t slot_bytes, up_off;
};

__device__ __forceinline__ void gu_unit(const GuParams &P, const int (&slots)[kMaxSlots], int n_act, int64_t u,
                                        int &slot, int64_t &r0, int &nr, const uint8_t *&g_src,
                                        const uint8_t *&u_src, int64_t &rbg, int64_t &rbu, int &tg, int &tu) {
    const MoeDev &L = P.L;
    const int64_t tiles_r = (L.ff + P.tr_routed - 1) / P.tr_routed;
    const int64_t tiles_s = (L.ff + P.tr_shared - 1) / P.tr_shared;
    int64_t rem = u;
    for (int a = 0; a < n_act; a++) {
        const int s = slots[a];
        const bool routed = s < L.topk;
        const int64_t tiles = routed ? tiles_r : tiles_s;
        if (rem < tiles) {
            const int tr = routed ? P.tr_routed : P.tr_shared;
            slot = s;
            r0 = rem * tr;
            nr = (int)imin64(tr, L.ff - r0);
            if (routed) {
                const int64_t le = local_expert(L, P.idx[s]);
                rbg = L.rb_gate; rbu = L.rb_up; tg = L.gate_type; tu = L.up_type;
                g_src = L.gate + le * L.gate_stride + r0 * rbg;
                u_src = L.up + le * L.up_stride + r0 * rbu;
            } else {
                const int64_t sh = s - L.topk;
                rbg = L.rb_sh_gate; rbu = L.rb_sh_up; tg = L.sh_gate_type; tu = L.sh_up_type;
                g_src = L.sh_gate + sh * L.sh_gate_stride + r0 * rbg;
                u_src = L.sh_up + sh * L.sh_up_stride + r0 * rbu;
            }
            return;
        }
        rem -= tiles;
    }
    slot = -1;
}

template <int TG, int TS>   // gate/up format of routed / shared experts; -1 = any (runtime)
__global__ void __launch_bounds__(17 * 32, 1) k_gateup(const GuParams P) {
    constexpr bool kScaled = TG >= 0 && TS >= 0;
    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n_cons = 2 * P.nwc;
    const MoeDev &L = P.L;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem);
    uint64_t *empty = full + kGuStagesMax;
    double *red = reinterpret_cast<double *>(smem + 256);   // [2][nwc][kTRG]
    uint8_t *stage0 = smem + 256 + ((2 * 16 * kTRG * 8 + 127) & ~127);

    int slots[kMaxSlots];
    const int n_act = active_slots(L, P.idx, slots);
    int64_t n_units = 0;
    {
        const int64_t tiles_r = (L.ff + P.tr_routed - 1) / P.tr_routed;
        const int64_t tiles_s = (L.ff + P.tr_shared - 1) / P.tr_shared;
        for (int a = 0; a < n_act; a++) n_units += (slots[a] < L.topk) ? tiles_r : tiles_s;
    }

    if (threadIdx.x == 0) {
        for (int s = 0; s < P.stages; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], n_cons);
        }
        fence_barrier_init();
    }
    __syncthreads();

    if (warp == n_cons) {
        if (lane == 0) {
            int64_t k = 0;
            for (int64_t u = blockIdx.x; u < n_units; u += gridDim.x, k++) {
                const int st = (int)(k % P.stages);
                if (k >= P.stages && !mbar_wait(&empty[st], (uint32_t)(((k / P.stages) - 1) & 1), L.err)) break;
                int slot, nr, tg, tu;
                int64_t r0, rbg, rbu;
                const uint8_t *gs, *us;
                gu_unit(P, slots, n_act, u, slot, r0, nr, gs, us, rbg, rbu, tg, tu);
                const ByteRange rg{gs, (uint32_t)(nr * rbg)}, ru{us, (uint32_t)(nr * rbu)};
                uint8_t *dst = stage0 + (size_t)st * P.slot_bytes;
                mbar_arrive_expect_tx(&full[st], range_copy_bytes(rg) + range_copy_bytes(ru));
                range_issue(dst, rg, &full[st]);
                range_issue(dst + P.up_off, ru, &full[st]);
            }
            const int64_t issued = k;
            for (int64_t j = (issued > P.stages ? issued - P.stages : 0); j < issued; j++)
                mbar_wait(&full[j % P.stages], (uint32_t)((j / P.stages) & 1), nullptr);
        }
        return;
    }

    const int grp = warp / P.nwc, cw = warp % P.nwc, p = lane & 7;
    const int sb = 4 * cw + (lane >> 3);
    XPart xp;
    load_xpart<kScaled>(xp, P.x, L.hidden, sb, p);
    const int my_row = rs_row<kTRG>(lane);

    int64_t k = 0;
    for (int64_t u = blockIdx.x; u < n_units; u += gridDim.x, k++) {
        const int st = (int)(k % P.stages);
        if (!mbar_wait(&full[st], (uint32_t)((k / P.stages) & 1), L.err)) break;
        int slot, nr, tg, tu;
        int64_t r0, rbg, rbu;
        const uint8_t *gs, *us;
        gu_unit(P, slots, n_act, u, slot, r0, nr, gs, us, rbg, rbu, tg, tu);
        const uint8_t *dst = stage0 + (size_t)st * P.slot_bytes;
        float acc[kTRG];
        const bool shared = slot >= L.topk;
        const uint8_t *gsrc = range_data(dst, ByteRange{gs, 0}), *usrc = range_data(dst + P.up_off, ByteRange{us, 0});
        if (grp == 0) {
            if (shared) rows_dot_k<TS, kTRG>(tg, gsrc, rbg, nr, sb, p, xp, L.hidden, acc);
            else rows_dot_k<TG, kTRG>(tg, gsrc, rbg, nr, sb, p, xp, L.hidden, acc);
        } else {
            if (shared) rows_dot_k<TS, kTRG>(tu, usrc, rbu, nr, sb, p, xp, L.hidden, acc);
            else rows_dot_k<TG, kTRG>(tu, usrc, rbu, nr, sb, p, xp, L.hidden, acc);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[st]);
        double ad[kTRG];
#pragma unroll
        for (int i = 0; i < kTRG; i++) ad[i] = (double)acc[i];
        warp_reduce_scatter<kTRG>(ad, lane);
        if ((lane & 3) == 0) red[(grp * P.nwc + cw) * kTRG + my_row] = ad[0];
        consumer_sync(n_cons * 32);
        const int t = threadIdx.x;
        if (t < nr) {
            double gd = 0.0, ud = 0.0;
            for (int c = 0; c < P.nwc; c++) {
                gd += red[c * kTRG + t];
                ud += red[(P.nwc + c) * kTRG + t];
            }
            const float gsum = (float)gd, usum = (float)ud;
            const float sig = __fdiv_rn(1.0f, __fadd_rn(1.0f, (float)exp(-(double)gsum)));
            float hv = __fmul_rn(__fmul_rn(gsum, sig), usum);
            if (slot >= L.topk) hv = __fmul_rn(hv, P.weights[slot]);   // shared: gamma inside h
            P.h[(int64_t)slot * L.ff + r0 + t] = hv;
        }
        consumer_sync(n_cons * 32);
    }
}

// ============================================================== down + combine
struct DnParams {
    MoeDev L;
    const int32_t *idx;
    const float *weights;
    const float *h;          // [slots, ff]
    float *out;              // [hidden]            (combine mode)
    float *slots_out;        // [slots, hidden]     (slot mode) or nullptr
    int nwc;                 // column warps (ceil(nsb_ff / 4))
    int stages;
    uint32_t slot_bytes;
    int64_t n_units;
};

// TD / TSD: down format of routed / shared experts (-1 = any, runtime);
// SPW: slots per consumer warp (the slots are split over groups = 8 / SPW
// warp groups, each warp keeps its slots' activations in registers).
template <int TD, int TSD, int SPW>
__global__ void __launch_bounds__(17 * 32, 1) k_down(const DnParams P) {
    constexpr bool kScaled = TD >= 0 && TSD >= 0;
    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    constexpr int kGroups = kDnMaxSlots / SPW;
    const int n_cons = kGroups * P.nwc;
    const MoeDev &L = P.L;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem);
    uint64_t *empty = full + kDnStagesMax;
    double *red = reinterpret_cast<double *>(smem + 256);   // [kMaxSlots][nwc][kTRD]
    uint8_t *stage0 = smem + 256 + ((kMaxSlots * 16 * kTRD * 8 + 127) & ~127);

    int slots[kMaxSlots];
    const int n_act = active_slots(L, P.idx, slots);
    // per-active-slot source base, row bytes, type and stage offset
    const uint8_t *sbase[kMaxSlots];
    int64_t srb[kMaxSlots];
    int stype[kMaxSlots];
    uint32_t soff[kMaxSlots];
    {
        uint32_t off = 0;
        for (int a = 0; a < n_act; a++) {
            const int s = slots[a];
            if (s < L.topk) {
                sbase[a] = L.down + local_expert(L, P.idx[s]) * L.down_stride;
                srb[a] = L.rb_down; stype[a] = L.down_type;
            } else {
                sbase[a] = L.sh_down + (int64_t)(s - L.topk) * L.sh_down_stride;
                srb[a] = L.rb_sh_down; stype[a] = L.sh_down_type;
            }
            soff[a] = off;
            off += slot_bytes_for((uint64_t)kTRD * srb[a]);
        }
    }

    if (threadIdx.x == 0) {
        for (int s = 0; s < P.stages; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], n_cons);
        }
        fence_barrier_init();
    }
    __syncthreads();

    if (warp == n_cons) {
        if (lane == 0) {
            int64_t k = 0;
            for (int64_t u = blockIdx.x; u < P.n_units; u += gridDim.x, k++) {
                const int st = (int)(k % P.stages);
                if (k >= P.stages && !mbar_wait(&empty[st], (uint32_t)(((k / P.stages) - 1) & 1), L.err)) break;
                const int64_t r0 = u * kTRD;
                const int nr = (int)imin64(kTRD, L.hidden - r0);
                uint32_t tx = 0;
                for (int a = 0; a < n_act; a++) tx += range_copy_bytes(ByteRange{sbase[a] + r0 * srb[a], (uint32_t)(nr * srb[a])});
                mbar_arrive_expect_tx(&full[st], tx);
                uint8_t *dst = stage0 + (size_t)st * P.slot_bytes;
                for (int a = 0; a < n_act; a++)
                    range_issue(dst + soff[a], ByteRange{sbase[a] + r0 * srb[a], (uint32_t)(nr * srb[a])}, &full[st]);
            }
            const int64_t issued = k;
            for (int64_t j = (issued > P.stages ? issued - P.stages : 0); j < issued; j++)
                mbar_wait(&full[j % P.stages], (uint32_t)((j / P.stages) & 1), nullptr);
        }
        return;
    }

    const int sg = warp / P.nwc, cw = warp % P.nwc, p = lane & 7;
    const int sb = 4 * cw + (lane >> 3);
    // this warp's slots: active indices a = sg, sg + G, ...
    XPart xp[SPW];
#pragma unroll
    for (int q = 0; q < SPW; q++) {
        const int a = sg + q * kGroups;
        if (a < n_act) load_xpart<kScaled>(xp[q], P.h + (int64_t)slots[a] * L.ff, L.ff, sb, p);
    }
    const int my_row = rs_row<kTRD>(lane);

    int64_t k = 0;
    for (int64_t u = blockIdx.x; u < P.n_units; u += gridDim.x, k++) {
        const int st = (int)(k % P.stages);
        if (!mbar_wait(&full[st], (uint32_t)((k / P.stages) & 1), L.err)) break;
        const int64_t r0 = u * kTRD;
        const int nr = (int)imin64(kTRD, L.hidden - r0);
        const uint8_t *dst = stage0 + (size_t)st * P.slot_bytes;
        float acc[SPW][kTRD];
#pragma unroll
        for (int q = 0; q < SPW; q++) {
            const int a = sg + q * kGroups;
            if (a < n_act) {
                const uint8_t *src = range_data(dst + soff[a], ByteRange{sbase[a] + r0 * srb[a], 0});
                if (slots[a] >= L.topk) rows_dot_k<TSD, kTRD>(stype[a], src, srb[a], nr, sb, p, xp[q], L.ff, acc[q]);
                else rows_dot_k<TD, kTRD>(stype[a], src, srb[a], nr, sb, p, xp[q], L.ff, acc[q]);
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[st]);
#pragma unroll
        for (int q = 0; q < SPW; q++) {
            const int a = sg + q * kGroups;
            if (a < n_act) {
                double ad[kTRD];
#pragma unroll
                for (int i = 0; i < kTRD; i++) ad[i] = (double)acc[q][i];
                warp_reduce_scatter<kTRD>(ad, lane);
                if ((lane & 7) == 0) red[(a * P.nwc + cw) * kTRD + my_row] = ad[0];
            }
        }
        consumer_sync(n_cons * 32);
        const int t = threadIdx.x;
        if (t < nr) {
            float o = 0.0f;
            int a = 0;
            const int n_slots = L.topk + L.n_shared;
            for (int s = 0; s < n_slots; s++) {
                float term = 0.0f;
                if (a < n_act && slots[a] == s) {
                    double ed = 0.0;
                    for (int c = 0; c < P.nwc; c++) ed += red[(a * P.nwc + c) * kTRD + t];
                    const float e = (float)ed;
                    term = (s < L.topk) ? __fmul_rn(e, P.weights[s]) : e;
                    a++;
                    if (!P.slots_out) o = __fadd_rn(o, term);
                }
                if (P.slots_out) P.slots_out[(int64_t)s * L.hidden + r0 + t] = term;
            }
            if (!P.slots_out) P.out[r0 + t] = o;
        }
        consumer_sync(n_cons * 32);
    }
}

// out[r] = sum over slots in order (after an all-reduce of the slot terms).
__global__ void k_combine(const float *slots, int n_slots, int64_t hidden, float *out) {
    const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    griddep_wait();
    griddep_launch();
    if (r >= hidden) return;
    float o = 0.0f;
    for (int s = 0; s < n_slots; s++) o = __fadd_rn(o, slots[(int64_t)s * hidden + r]);
    out[r] = o;
}

// ============================================================== tensor-core path
// Gate/up and down of every selected expert on the engine of qengine.cuh,
// chained router -> gate/up -> down by programmatic dependent launch: each
// kernel starts streaming weights that do not depend on its predecessor
// (shared experts for gate/up, every down matrix) while the predecessor
// finishes.


// Units: (slot, 8-row block of ff): MMA rows 0-7 are the gate rows, 8-15 the
// matching up rows. Shared slots come first: they do not depend on the router.
// The x tables are built before the dependency wait: x was written before
// the router's predecessor completed, and the routers let this kernel launch
// only after their own dependency wait.
struct GuJob {
    static constexpr bool kTabsEarly = true;
    MoeDev L;
    const int32_t *idx;
    const float *weights;
    float *h;
    const float *x;
    int nsb_h, tpu, n_slots;
    float inv_tpu;      // 1/tpu (qe_div; n_units < kQeDivMax)
    int sbs_r, nsplit_r, sbs_s, nsplit_s;
    __device__ void init() {}
    __device__ void setup(uint8_t *jsm, int tid, bool after_dep) {
        MoeSlot *S = reinterpret_cast<MoeSlot *>(jsm);
        if (!after_dep && tid < L.n_shared) {
            MoeSlot &m = S[L.topk + tid];
            m.a = L.sh_gate + (int64_t)tid * L.sh_gate_stride;
            m.b = L.sh_up + (int64_t)tid * L.sh_up_stride;
            m.rb = L.rb_sh_gate; m.type = L.sh_gate_type; m.sbs = sbs_s;
            m.nsplit = (tid % L.world == L.rank) ? nsplit_s : 0;
        }
        if (after_dep && tid < L.topk) {
            MoeSlot &m = S[tid];
            const int e = idx[tid];
            const bool own = e >= 0 && e < L.n_routed && e % L.world == L.rank;
            const int64_t le = own ? local_expert(L, e) : 0;
            m.a = L.gate + le * L.gate_stride;
            m.b = L.up + le * L.up_stride;
            m.rb = L.rb_gate; m.type = L.gate_type; m.sbs = sbs_r;
            m.nsplit = own ? nsplit_r : 0;
        }
    }
    __device__ int64_t n_units() const { return (int64_t)n_slots * tpu; }
    __device__ int slot_of(int a) const { return a < L.n_shared ? L.topk + a : a - L.n_shared; }
    __device__ bool needs_dep(int64_t u) const { return slot_of(qe_div((int)u, inv_tpu)) < L.topk; }
    __device__ int splits(const uint8_t *jsm, int64_t u) const {
        return reinterpret_cast<const MoeSlot *>(jsm)[slot_of(qe_div((int)u, inv_tpu))].nsplit;
    }
    __device__ void unit(const uint8_t *jsm, int64_t u, QUnit &U) const {
        const int a = qe_div((int)u, inv_tpu), r = (int)u - a * tpu;
        const MoeSlot &m = reinterpret_cast<const MoeSlot *>(jsm)[slot_of(a)];
        U.type = m.type; U.rb = m.rb; U.sbs = m.sbs; U.nsplit = m.nsplit;
        U.nsb = nsb_h;
        U.tab = 0;
        U.nlo = U.nhi = 8;
        U.lo = m.a + (int64_t)r * 8 * m.rb;
        U.hi = m.b + (int64_t)r * 8 * m.rb;
    }
    __device__ int n_tab() const { return 1; }
    __device__ uint32_t tab_mask(const uint8_t *) const { return 1u; }
    __device__ const float *tab_src(int) const { return x; }
    // lanes 0-7: h = silu(g) * u in the reference's float arithmetic
    // (src/sepia.c:1405-1410; shared experts: * gamma, src/sepia.c:1432-1444)
    __device__ void finish(const uint8_t *, int64_t u, const QUnit &, double v, int lane) const {
        const int a = qe_div((int)u, inv_tpu), r = (int)u - a * tpu;
        const int s = slot_of(a);
        const float uv = (float)__shfl_sync(0xffffffffu, v, (lane + 8) & 31);
        if (lane < 8) {
            const float gv = (float)v;
            const float sig = __fdiv_rn(1.0f, __fadd_rn(1.0f, (float)exp(-(double)gv)));
            float hv = __fmul_rn(__fmul_rn(gv, sig), uv);
            if (s >= L.topk) hv = __fmul_rn(hv, weights[s]);
            h[(int64_t)s * L.ff + (int64_t)r * 8 + lane] = hv;
        }
    }
};

// Units: (16-row tile of hidden, slot), slot-minor. The reducer writes each
// slot's term (routed: E_j * w_j; shared: S_s, gamma already inside h);
// k_combine sums them in slot order.
struct DnJob {
    MoeDev L;
    const int32_t *idx;
    const float *weights;
    const float *h;
    float *slots_out;
    int nsb_f, n_slots, n_tiles;
    float inv_slots;    // 1/n_slots (qe_div; n_units < kQeDivMax)
    int sbs_r, nsplit_r, sbs_s, nsplit_s;
    __device__ void init() {}
    // the router finished before the gate/up kernel let its successors
    // launch, so the expert ids and weights are final already
    __device__ void setup(uint8_t *jsm, int tid, bool after_dep) {
        if (after_dep || tid >= n_slots) return;
        MoeSlot &m = reinterpret_cast<MoeSlot *>(jsm)[tid];
        if (tid >= L.topk) {
            const int e = tid - L.topk;
            m.a = L.sh_down + (int64_t)e * L.sh_down_stride;
            m.rb = L.rb_sh_down; m.type = L.sh_down_type; m.sbs = sbs_s;
            m.nsplit = (e % L.world == L.rank) ? nsplit_s : 0;
            m.w = 1.0f;
        } else {
            const int e = __ldcg(idx + tid);
            m.w = __ldcg(weights + tid);
            const bool own = e >= 0 && e < L.n_routed && e % L.world == L.rank;
            m.a = L.down + (own ? local_expert(L, e) : 0) * L.down_stride;
            m.rb = L.rb_down; m.type = L.down_type; m.sbs = sbs_r;
            m.nsplit = own ? nsplit_r : 0;
        }
        m.b = m.a;
    }
    __device__ int64_t n_units() const { return (int64_t)n_slots * n_tiles; }
    __device__ bool needs_dep(int64_t) const { return false; }
    __device__ int splits(const uint8_t *jsm, int64_t u) const {
        const int t = qe_div((int)u, inv_slots);
        return reinterpret_cast<const MoeSlot *>(jsm)[(int)u - t * n_slots].nsplit;
    }
    __device__ void unit(const uint8_t *jsm, int64_t u, QUnit &U) const {
        const int t = qe_div((int)u, inv_slots), s = (int)u - t * n_slots;
        const MoeSlot &m = reinterpret_cast<const MoeSlot *>(jsm)[s];
        const int64_t r0 = (int64_t)t * 16;
        const int nr = (int)imin64(16, L.hidden - r0);
        U.type = m.type; U.rb = m.rb; U.sbs = m.sbs; U.nsplit = m.nsplit;
        U.nsb = nsb_f;
        U.tab = s;
        U.nlo = min(8, nr);
        U.nhi = max(0, nr - 8);
        U.lo = m.a + r0 * m.rb;
        U.hi = U.lo + 8 * m.rb;
    }
    __device__ int n_tab() const { return n_slots; }
    // units u = blockIdx.x + k*gridDim.x read table u % n_slots: the slots
    // repeat with period at most n_slots, and inactive slots need none
    __device__ uint32_t tab_mask(const uint8_t *jsm) const {
        const MoeSlot *m = reinterpret_cast<const MoeSlot *>(jsm);
        uint32_t mask = 0;
        const int64_t nu = n_units();
        for (int k = 0; k < n_slots; k++) {
            const int64_t u = blockIdx.x + (int64_t)k * gridDim.x;
            if (u >= nu) break;
            const int s = (int)(u % n_slots);
            if (m[s].nsplit) mask |= 1u << s;
        }
        return mask;
    }
    __device__ const float *tab_src(int t) const { return h + (int64_t)t * L.ff; }
    __device__ void finish(const uint8_t *jsm, int64_t u, const QUnit &, double v, int lane) const {
        const int t = qe_div((int)u, inv_slots), s = (int)u - t * n_slots;
        const int64_t r0 = (int64_t)t * 16;
        if (lane < 16 && r0 + lane < L.hidden) {
            const float e = (float)v;
            const float w = reinterpret_cast<const MoeSlot *>(jsm)[s].w;
            slots_out[(int64_t)s * L.hidden + r0 + lane] = (s < L.topk) ? __fmul_rn(e, w) : e;
        }
    }
};

// The same jobs for launches that carry IQ grid-codebook formats (the
// engine stages their codebooks in shared memory).
struct GuIqJob : GuJob {
    static constexpr int kIq = -1;
};
struct DnIqJob : DnJob {
    static constexpr int kIq = -1;
};
// Gate/up whose x may be written by the kernel right before it (no router in
// between): the tables wait for the dependency.
struct GuLateJob : GuJob {
    static constexpr bool kTabsEarly = false;
};
struct GuIqLateJob : GuJob {
    static constexpr int kIq = -1;
    static constexpr bool kTabsEarly = false;
};

static bool engine_format(int t) { return mma_format(t) || iq_format(t); }

// ============================================================== host side
int to_dev(const SepiaMoeLayer *in, MoeDev &L) {
    if (!in) return fail("moe: null layer");
    L.hidden = in->hidden; L.ff = in->ff;
    L.n_routed = in->n_routed; L.n_shared = in->n_shared; L.topk = in->topk;
    L.route_scale = in->route_scale; L.global_scale = in->global_scale;
    L.router_w = in->router_w; L.router_bias = in->router_bias;
    L.gate_type = in->gate_type; L.up_type = in->up_type; L.down_type = in->down_type;
    L.sh_gate_type = in->sh_gate_type; L.sh_up_type = in->sh_up_type; L.sh_down_type = in->sh_down_type;
    L.gate = (const uint8_t *)in->gate; L.up = (const uint8_t *)in->up; L.down = (const uint8_t *)in->down;
    L.sh_gate = (const uint8_t *)in->sh_gate; L.sh_up = (const uint8_t *)in->sh_up; L.sh_down = (const uint8_t *)in->sh_down;
    L.gate_stride = in->gate_stride; L.up_stride = in->up_stride; L.down_stride = in->down_stride;
    L.sh_gate_stride = in->sh_gate_stride; L.sh_up_stride = in->sh_up_stride; L.sh_down_stride = in->sh_down_stride;
    L.rank = in->rank; L.world = in->world < 1 ? 1 : in->world;
    L.expert_slot = in->expert_slot;
    L.err = dev_info().err;
    if (L.hidden <= 0 || L.ff <= 0 || L.n_routed <= 0 || L.topk <= 0 || L.topk > L.n_routed || L.n_shared < 0 ||
        L.topk + L.n_shared > kMaxSlots || L.n_routed > 1024)
        return fail("moe: bad geometry hidden=%lld ff=%lld routed=%d shared=%d topk=%d (max %d slots, 1024 experts)",
                    (long long)L.hidden, (long long)L.ff, L.n_routed, L.n_shared, L.topk, kMaxSlots);
    if (L.rank < 0 || L.rank >= L.world) return fail("moe: rank %d outside world %d", L.rank, L.world);
    if (!L.router_w || !L.router_bias) return fail("moe: router weights missing");
    L.rb_gate = host_row_bytes(L.gate_type, L.hidden);
    L.rb_up = host_row_bytes(L.up_type, L.hidden);
    L.rb_down = host_row_bytes(L.down_type, L.ff);
    if (L.rb_gate <= 0 || L.rb_up <= 0 || L.rb_down <= 0) return fail("moe: unsupported routed expert types/dims");
    if (L.n_shared > 0) {
        L.rb_sh_gate = host_row_bytes(L.sh_gate_type, L.hidden);
        L.rb_sh_up = host_row_bytes(L.sh_up_type, L.hidden);
        L.rb_sh_down = host_row_bytes(L.sh_down_type, L.ff);
        if (L.rb_sh_gate <= 0 || L.rb_sh_up <= 0 || L.rb_sh_down <= 0) return fail("moe: unsupported shared expert types/dims");
    } else {
        L.rb_sh_gate = L.rb_sh_up = L.rb_sh_down = 0;
    }
    if ((L.hidden + kQK - 1) / kQK > 64 || (L.ff + kQK - 1) / kQK > 16)
        return fail("moe: hidden <= 16384 and ff <= 4096 supported (hidden=%lld ff=%lld)", (long long)L.hidden, (long long)L.ff);
    return 1;
}

typedef void (*GuKernel)(const GuParams);
typedef void (*DnKernel)(const DnParams);

// Kernel instances: every (routed, shared) pair of the fast formats gets a
// specialised kernel; anything else runs the runtime-typed generic kernel.
template <int A>
static GuKernel gu_for_shared(int b) {
    if (b == T_Q2_K) return k_gateup<A, T_Q2_K>;
    if (b == T_Q3_K) return k_gateup<A, T_Q3_K>;
    if (b == T_Q4_K) return k_gateup<A, T_Q4_K>;
    return k_gateup<-1, -1>;
}
template <int A>
static DnKernel dn_for_shared(int b) {
    if (b == T_Q2_K) return k_down<A, T_Q2_K, 1>;
    if (b == T_Q3_K) return k_down<A, T_Q3_K, 1>;
    if (b == T_Q4_K) return k_down<A, T_Q4_K, 1>;
    return k_down<-1, -1, 1>;
}

static GuKernel pick_gateup(const MoeDev &L) {
    const int a = L.gate_type;
    const int b = L.n_shared ? L.sh_gate_type : a;
    const bool same = L.up_type == a && (!L.n_shared || L.sh_up_type == b);
    if (same && fast_format(a) && fast_format(b)) {
        if (a == T_Q2_K) return gu_for_shared<T_Q2_K>(b);
        if (a == T_Q3_K) return gu_for_shared<T_Q3_K>(b);
        if (a == T_Q4_K) return gu_for_shared<T_Q4_K>(b);
    }
    return k_gateup<-1, -1>;
}

static DnKernel pick_down(const MoeDev &L, int spw) {
    const int a = L.down_type;
    const int b = L.n_shared ? L.sh_down_type : a;
    if (spw == 2) return k_down<-1, -1, 2>;
    if (fast_format(a) && fast_format(b)) {
        if (a == T_Q2_K) return dn_for_shared<T_Q2_K>(b);
        if (a == T_Q3_K) return dn_for_shared<T_Q3_K>(b);
        if (a == T_Q4_K) return dn_for_shared<T_Q4_K>(b);
    }
    return k_down<-1, -1, 1>;
}

static int pick_tr(int64_t rb_pair, int64_t budget) {
    int tr = kTRG;
    while (tr > 1 && (int64_t)tr * rb_pair > budget) tr >>= 1;
    return tr;
}

// Tensor-core engine eligibility: K-quant formats it decodes, whole
// superblocks, rows at 4-byte aligned addresses that agree mod 4 between
// the gate and up matrices, and the tables in the work area.
static bool rows_ok(const void *base, int64_t stride, int64_t rb) {
    return ((reinterpret_cast<uintptr_t>(base) | (uintptr_t)stride | (uintptr_t)rb) & 3) == 0;
}
bool engine_gateup_ok(const MoeDev &L, const SepiaMoeWork *ws) {
    if (L.hidden % kQK || L.ff % kQK || L.hidden / kQK > 64 || L.ff / kQK > 16) return false;
    if (!engine_format(L.gate_type) || L.up_type != L.gate_type) return false;
    if (!rows_ok(L.gate, L.gate_stride, L.rb_gate) || !rows_ok(L.up, L.up_stride, L.rb_up) ||
        ((reinterpret_cast<uintptr_t>(L.gate) ^ reinterpret_cast<uintptr_t>(L.up)) & 3))
        return false;
    if (L.n_shared > 0) {
        if (!engine_format(L.sh_gate_type) || L.sh_up_type != L.sh_gate_type) return false;
        if (!rows_ok(L.sh_gate, L.sh_gate_stride, L.rb_sh_gate) || !rows_ok(L.sh_up, L.sh_up_stride, L.rb_sh_up) ||
            ((reinterpret_cast<uintptr_t>(L.sh_gate) ^ reinterpret_cast<uintptr_t>(L.sh_up)) & 3))
            return false;
    }
    return true;
}
bool engine_down_ok(const MoeDev &L, const SepiaMoeWork *ws) {
    if (L.ff % kQK || L.ff / kQK > 16) return false;
    if (!engine_format(L.down_type) || !rows_ok(L.down, L.down_stride, L.rb_down)) return false;
    if (L.n_shared > 0 && (!engine_format(L.sh_down_type) || !rows_ok(L.sh_down, L.sh_down_stride, L.rb_sh_down)))
        return false;
    return true;
}


static int launch_gateup_engine(const MoeDev &L, const float *x, const SepiaMoeWork *ws, cudaStream_t st,
                                bool early = true) {
    DevInfo &di = dev_info();
    GuJob J;
    J.L = L; J.idx = ws->topk_idx; J.weights = ws->weights; J.h = ws->h;
    J.x = x;
    J.nsb_h = (int)(L.hidden / kQK); J.tpu = (int)(L.ff / 8);
    J.inv_tpu = 1.0f / (float)J.tpu;
    J.n_slots = L.topk + L.n_shared;
    const IqLayout iql = iq_layout(L.gate_type, L.n_shared ? L.sh_gate_type : L.gate_type);
    const uint32_t iqb = iql.bytes;
    const uint32_t budget = qe_row_budget(di.smem_optin, (int64_t)J.nsb_h * kTabSB + iqb);
    J.sbs_r = qe_sbs(L.gate_type, J.nsb_h, budget, J.nsplit_r);
    J.sbs_s = J.sbs_r; J.nsplit_s = J.nsplit_r;
    if (L.n_shared) J.sbs_s = qe_sbs(L.sh_gate_type, J.nsb_h, budget, J.nsplit_s);
    if (!J.sbs_r || !J.sbs_s) return fail("moe: no tensor-core split for the gate/up rows");
    const uint32_t row_max = std::max((uint32_t)J.sbs_r * qe_sb_bytes(L.gate_type),
                                      L.n_shared ? (uint32_t)J.sbs_s * qe_sb_bytes(L.sh_gate_type) : 0u);
    int cg, G;
    qe_groups_fmt(std::max(J.sbs_r, J.sbs_s), L.gate_type, L.n_shared ? L.sh_gate_type : L.gate_type, cg, G);
    QeLayout P;
    int64_t smem = 0;
    if (!qe_layout(P, G, cg, row_max, 1, J.nsb_h, di.smem_optin, smem, iqb ? &iql : nullptr))
        return fail("moe: gate/up tile needs %lld B of shared memory", (long long)smem);
    P.err = di.err;
    const int64_t units = (int64_t)J.n_slots * J.tpu;
    if (units >= kQeDivMax) return fail("moe: %lld gate/up units exceed the engine's index range", (long long)units);
    const unsigned grid = (unsigned)std::min<int64_t>(units, di.sm_count);
    auto run = [&](auto JV) {
        using JT = decltype(JV);
        static_cast<GuJob &>(JV) = J;
        if (!ensure_smem((const void *)k_qengine<JT>, (int)smem)) return 0;
        return check(launch_pdl(k_qengine<JT>, grid, (P.G * P.cg + 2) * 32, (size_t)smem, st, JV, P),
                     "moe gate/up (tensor cores) launch");
    };
    if (iqb) return early ? run(GuIqJob{}) : run(GuIqLateJob{});
    return early ? run(GuJob{}) : run(GuLateJob{});
}

static int launch_down_engine(const MoeDev &L, const SepiaMoeWork *ws, float *out, float *slots_out, bool clear,
                              cudaStream_t st) {
    DevInfo &di = dev_info();
    DnJob J;
    J.L = L; J.idx = ws->topk_idx; J.weights = ws->weights; J.h = ws->h;
    J.slots_out = slots_out ? slots_out : ws->slots;
    J.nsb_f = (int)(L.ff / kQK);
    J.n_slots = L.topk + L.n_shared;
    J.n_tiles = (int)((L.hidden + 15) / 16);
    J.inv_slots = 1.0f / (float)J.n_slots;
    if ((int64_t)J.n_slots * J.n_tiles >= kQeDivMax) return fail("moe: too many down units");
    const IqLayout iql = iq_layout(L.down_type, L.n_shared ? L.sh_down_type : L.down_type);
    const uint32_t iqb = iql.bytes;
    const uint32_t budget = qe_row_budget(di.smem_optin, (int64_t)J.n_slots * J.nsb_f * kTabSB + iqb);
    J.sbs_r = qe_sbs(L.down_type, J.nsb_f, budget, J.nsplit_r);
    J.sbs_s = J.sbs_r; J.nsplit_s = J.nsplit_r;
    if (L.n_shared) J.sbs_s = qe_sbs(L.sh_down_type, J.nsb_f, budget, J.nsplit_s);
    if (!J.sbs_r || !J.sbs_s) return fail("moe: no tensor-core split for the down rows");
    const uint32_t row_max = std::max((uint32_t)J.sbs_r * qe_sb_bytes(L.down_type),
                                      L.n_shared ? (uint32_t)J.sbs_s * qe_sb_bytes(L.sh_down_type) : 0u);
    int cg, G;
    qe_groups_fmt(std::max(J.sbs_r, J.sbs_s), L.down_type, L.n_shared ? L.sh_down_type : L.down_type, cg, G);
    QeLayout P;
    int64_t smem = 0;
    if (!qe_layout(P, G, cg, row_max, J.n_slots, J.nsb_f, di.smem_optin, smem, iqb ? &iql : nullptr))
        return fail("moe: down tile needs %lld B of shared memory", (long long)smem);
    P.err = di.err;
    const void *fn = iqb ? (const void *)k_qengine<DnIqJob> : (const void *)k_qengine<DnJob>;
    if (!ensure_smem(fn, (int)smem)) return 0;
    if (slots_out && clear &&
        !check(cudaMemsetAsync(slots_out, 0, (size_t)J.n_slots * L.hidden * sizeof(float), st), "moe slot clear"))
        return 0;
    // the down projections (each CTA builds the h tables it reads), then
    // the combine
    const int64_t units = (int64_t)J.n_slots * J.n_tiles;
    const unsigned grid = (unsigned)std::min<int64_t>(units, di.sm_count);
    if (iqb) {
        DnIqJob JI;
        static_cast<DnJob &>(JI) = J;
        if (!check(launch_pdl(k_qengine<DnIqJob>, grid, (P.G * P.cg + 2) * 32, (size_t)smem, st, JI, P),
                   "moe down (tensor cores) launch"))
            return 0;
    } else if (!check(launch_pdl(k_qengine<DnJob>, grid, (P.G * P.cg + 2) * 32, (size_t)smem, st, J, P),
                      "moe down (tensor cores) launch"))
        return 0;
    if (slots_out) return 1;
    return check(launch_pdl(k_combine, (unsigned)((L.hidden + 255) / 256), 256, 0, st, (const float *)J.slots_out,
                            J.n_slots, L.hidden, out),
                 "moe combine launch");
}

int launch_router(const MoeDev &L, const float *x, const SepiaMoeWork *ws, cudaStream_t st) {
    const int n_total = L.n_routed + L.n_shared;
    if (n_total > kRouterMaxExperts) return fail("moe: %d experts exceed the router's %d", n_total, kRouterMaxExperts);
    if (router_chunks(L.hidden) > kRouterMaxChunks)
        return fail("moe: hidden %lld exceeds the router's %d", (long long)L.hidden, kRouterMaxChunks * kRouterChunk);
    if (!ws->router_part) return fail("moe: work area has no router scratch (carve it with moe_work_carve)");
    // bulk-copy form: ~one CTA per SM, each fetching its rows in one request
    const DevInfo &di = dev_info();
    const int sms = di.sm_count > 0 ? di.sm_count : 148;
    const int rpc = (n_total + sms - 1) / sms;
    const int64_t smem = (int64_t)rpc * L.hidden * 4;
    if ((L.hidden * 4) % 16 == 0 && ((reinterpret_cast<uintptr_t>(L.router_w) | reinterpret_cast<uintptr_t>(x)) & 15) == 0 &&
        L.hidden <= (int64_t)kRouter2MaxPerThread * kRouter2Threads && smem <= di.smem_optin - 2048 &&
        smem < (1 << 20)) {
        if (!ensure_smem((const void *)k_router2, (int)smem)) return 0;
        const unsigned grid = (unsigned)((n_total + rpc - 1) / rpc);
        return check(launch_pdl(k_router2, grid, kRouter2Threads, (size_t)smem, st, L, x, ws->logits, ws->topk_idx,
                                ws->weights, ws->counter, reinterpret_cast<float2 *>(ws->router_part), rpc),
                     "moe router launch");
    }
    // one CTA per logit row, a warp per 1024-element chunk
    const int nw = std::max(kRouterWarps, router_chunks(L.hidden));
    return check(launch_pdl(k_router, (unsigned)n_total, nw * 32, 0, st, L, x, ws->logits, ws->topk_idx, ws->weights,
                            ws->counter, reinterpret_cast<float2 *>(ws->router_part)),
                 "moe router launch");
}

int launch_gateup(const MoeDev &L, const float *x, const SepiaMoeWork *ws, cudaStream_t st) {
    if (engine_gateup_ok(L, ws)) return launch_gateup_engine(L, x, ws, st);
    DevInfo &di = dev_info();
    GuParams G;
    G.L = L; G.x = x; G.idx = ws->topk_idx; G.weights = ws->weights; G.h = ws->h;
    G.nwc = (int)((L.hidden + kQK - 1) / kQK + 3) / 4;
    if (2 * G.nwc > 16) return fail("moe: hidden %lld too large for the gate/up kernel (max 8192)", (long long)L.hidden);
    const int64_t budget = 40 * 1024;
    G.tr_routed = pick_tr(L.rb_gate + L.rb_up, budget);
    G.tr_shared = L.n_shared ? pick_tr(L.rb_sh_gate + L.rb_sh_up, budget) : G.tr_routed;
    const uint32_t sr_g = slot_bytes_for((uint64_t)G.tr_routed * L.rb_gate), sr_u = slot_bytes_for((uint64_t)G.tr_routed * L.rb_up);
    const uint32_t ss_g = L.n_shared ? slot_bytes_for((uint64_t)G.tr_shared * L.rb_sh_gate) : 0;
    const uint32_t ss_u = L.n_shared ? slot_bytes_for((uint64_t)G.tr_shared * L.rb_sh_up) : 0;
    G.up_off = std::max(sr_g, ss_g);
    G.slot_bytes = G.up_off + std::max(sr_u, ss_u);
    const int head_g = 256 + ((2 * 16 * kTRG * 8 + 127) & ~127);
    G.stages = kGuStagesMax;
    while (G.stages > 2 && head_g + (int64_t)G.stages * G.slot_bytes > di.smem_optin) G.stages--;
    const int64_t smem_g = head_g + (int64_t)G.stages * G.slot_bytes;
    if (smem_g > di.smem_optin) return fail("moe: gate/up tile needs %lld B of shared memory", (long long)smem_g);
    const GuKernel kern = pick_gateup(L);
    if (!ensure_smem((const void *)kern, (int)smem_g)) return 0;
    const int n_slots = L.topk + L.n_shared;
    const int64_t max_units = (int64_t)n_slots * ((L.ff + G.tr_routed - 1) / std::min(G.tr_routed, G.tr_shared));
    const int grid_g = (int)std::min<int64_t>(max_units, di.sm_count);
    kern<<<grid_g, (2 * G.nwc + 1) * 32, (size_t)smem_g, st>>>(G);
    return check(cudaGetLastError(), "moe gate/up launch");
}

// The down engine reads the h tables that only the gate/up engine builds.
// clear: zero the slot buffer first (slots other ranks own stay zero, as a
// sum all-reduce of the buffer needs); an owner-only exchange skips it.
int launch_down(const MoeDev &L, const SepiaMoeWork *ws, float *out, float *slots_out, cudaStream_t st,
                bool clear = true) {
    if (engine_gateup_ok(L, ws) && engine_down_ok(L, ws)) return launch_down_engine(L, ws, out, slots_out, clear, st);
    DevInfo &di = dev_info();
    const int n_slots = L.topk + L.n_shared;
    DnParams D;
    D.L = L; D.idx = ws->topk_idx; D.weights = ws->weights; D.h = ws->h; D.out = out; D.slots_out = slots_out;
    D.nwc = (int)((L.ff + kQK - 1) / kQK + 3) / 4;
    if (n_slots > kDnMaxSlots) return fail("moe: topk + n_shared = %d > %d", n_slots, kDnMaxSlots);
    const int spw = (8 * D.nwc <= 16) ? 1 : 2;       // one slot per warp when the warps fit
    if ((kDnMaxSlots / spw) * D.nwc > 16) return fail("moe: ff %lld too large for the down kernel (max 4096)", (long long)L.ff);
    // worst-case stage: every slot active, each with its own row bytes
    uint64_t sbytes = 0;
    for (int s = 0; s < n_slots; s++)
        sbytes += slot_bytes_for((uint64_t)kTRD * (s < L.topk ? L.rb_down : L.rb_sh_down));
    D.slot_bytes = (uint32_t)sbytes;
    const int head_d = 256 + ((kMaxSlots * 16 * kTRD * 8 + 127) & ~127);
    D.stages = kDnStagesMax;
    while (D.stages > 2 && head_d + (int64_t)D.stages * D.slot_bytes > di.smem_optin) D.stages--;
    const int64_t smem_d = head_d + (int64_t)D.stages * D.slot_bytes;
    if (smem_d > di.smem_optin) return fail("moe: down tile needs %lld B of shared memory", (long long)smem_d);
    const DnKernel kern = pick_down(L, spw);
    if (!ensure_smem((const void *)kern, (int)smem_d)) return 0;
    D.n_units = (L.hidden + kTRD - 1) / kTRD;
    const int grid_d = (int)std::min<int64_t>(D.n_units, di.sm_count);
    kern<<<grid_d, ((kDnMaxSlots / spw) * D.nwc + 1) * 32, (size_t)smem_d, st>>>(D);
    return check(cudaGetLastError(), "moe down launch");
}

int launch_experts(const MoeDev &L, const float *x, const SepiaMoeWork *ws, float *out, float *slots_out,
                   cudaStream_t st) {
    // the down engine reads the h tables that only the gate/up engine builds
    return launch_gateup(L, x, ws, st) && launch_down(L, ws, out, slots_out, st);
}

}  // namespace sepia

using namespace sepia;

extern "C" size_t sepia_cuda_moe_work_bytes(const SepiaMoeLayer *L) {
    if (!L) return 0;
    const size_t n_total = (size_t)L->n_routed + (size_t)L->n_shared;
    const size_t n_slots = (size_t)L->topk + (size_t)L->n_shared;
    size_t b = 0;
    auto add = [&](size_t n) { b += (n + 255) & ~(size_t)255; };
    add(n_total * 4);                 // logits
    add((size_t)L->topk * 4);         // topk_idx
    add(n_slots * 4);                 // weights
    add(n_slots * (size_t)L->ff * 4); // h
    add(n_slots * (size_t)L->hidden * 4);  // slots
    add(256);                         // counter
    add(n_total * (size_t)router_chunks(L->hidden) * 8);  // router_part
    add(moe_fused_sync_bytes(L));     // sync
    add(moe_fused_htab_bytes(L));     // htab
    return b;
}


extern "C" int sepia_cuda_moe_work_carve(const SepiaMoeLayer *L, void *base, size_t bytes, SepiaMoeWork *ws) {
    if (!L || !base || !ws) return fail("moe_work_carve: null argument");
    if (bytes < sepia_cuda_moe_work_bytes(L)) return fail("moe_work_carve: %zu bytes < %zu needed", bytes, sepia_cuda_moe_work_bytes(L));
    if (reinterpret_cast<uintptr_t>(base) & 255) return fail("moe_work_carve: base must be 256-byte aligned");
    const size_t n_total = (size_t)L->n_routed + (size_t)L->n_shared;
    const size_t n_slots = (size_t)L->topk + (size_t)L->n_shared;
    uint8_t *p = (uint8_t *)base;
    auto take = [&](size_t n) { uint8_t *r = p; p += (n + 255) & ~(size_t)255; return r; };
    ws->logits = (float *)take(n_total * 4);
    ws->topk_idx = (int32_t *)take((size_t)L->topk * 4);
    ws->weights = (float *)take(n_slots * 4);
    ws->h = (float *)take(n_slots * (size_t)L->ff * 4);
    ws->slots = (float *)take(n_slots * (size_t)L->hidden * 4);
    ws->counter = (unsigned int *)take(256);
    ws->router_part = (double *)take(n_total * (size_t)router_chunks(L->hidden) * 8);
    ws->sync = (unsigned int *)take(moe_fused_sync_bytes(L));
    ws->htab = take(moe_fused_htab_bytes(L));
    return 1;
}

extern "C" int sepia_cuda_moe_router(const SepiaMoeLayer *Lh, const float *x, const SepiaMoeWork *ws, void *stream) {
    MoeDev L;
    if (!to_dev(Lh, L)) return 0;
    if (!x || !ws) return fail("moe_router: null argument");
    return launch_router(L, x, ws, as_stream(stream));
}

namespace sepia {
// Router already run: every slot this rank owns gets its term in ws->slots
// (other slots are left as they are); for an exchange that moves owned rows
// only (csrc/model.cu).
int moe_experts_owned_slots(const SepiaMoeLayer *Lh, const float *x, const SepiaMoeWork *ws, cudaStream_t st) {
    MoeDev L;
    if (!to_dev(Lh, L)) return 0;
    if (!x || !ws) return fail("moe_experts: null argument");
    return launch_gateup(L, x, ws, st) && launch_down(L, ws, nullptr, ws->slots, st, false);
}
}  // namespace sepia

extern "C" int sepia_cuda_moe_experts(const SepiaMoeLayer *Lh, const float *x, const SepiaMoeWork *ws, float *out,
                                      int write_slots, void *stream) {
    MoeDev L;
    if (!to_dev(Lh, L)) return 0;
    if (!x || !ws || (!out && !write_slots)) return fail("moe_experts: null argument");
    return launch_experts(L, x, ws, out, write_slots ? ws->slots : nullptr, as_stream(stream));
}

extern "C" int sepia_cuda_moe_gateup(const SepiaMoeLayer *Lh, const float *x, const SepiaMoeWork *ws, void *stream) {
    MoeDev L;
    if (!to_dev(Lh, L)) return 0;
    if (!x || !ws) return fail("moe_gateup: null argument");
    return launch_gateup(L, x, ws, as_stream(stream));
}

extern "C" int sepia_cuda_moe_down(const SepiaMoeLayer *Lh, const SepiaMoeWork *ws, float *out, int write_slots,
                                   void *stream) {
    MoeDev L;
    if (!to_dev(Lh, L)) return 0;
    if (!ws || (!out && !write_slots)) return fail("moe_down: null argument");
    return launch_down(L, ws, out, write_slots ? ws->slots : nullptr, as_stream(stream));
}

extern "C" int sepia_cuda_moe_combine(const SepiaMoeLayer *Lh, const SepiaMoeWork *ws, float *out, void *stream) {
    if (!Lh || !ws || !out) return fail("moe_combine: null argument");
    const int n_slots = Lh->topk + Lh->n_shared;
    const int threads = 256;
    k_combine<<<(unsigned)((Lh->hidden + threads - 1) / threads), threads, 0, as_stream(stream)>>>(ws->slots, n_slots,
                                                                                                  Lh->hidden, out);
    return check(cudaGetLastError(), "moe combine launch");
}

extern "C" int sepia_cuda_moe_layer(const SepiaMoeLayer *Lh, const float *x, const SepiaMoeWork *ws, float *out,
                                    void *stream) {
    MoeDev L;
    if (!to_dev(Lh, L)) return 0;
    if (!x || !ws || !out) return fail("moe_layer: null argument");
    cudaStream_t st = as_stream(stream);
    if (!launch_router(L, x, ws, st)) return 0;
    return launch_experts(L, x, ws, out, nullptr, st);
}

// ------------------------------------------------ one expert's SwiGLU slab
// The expert kernels with a fixed one-slot selection (expert 0, weight 1)
// kept in device constants: the slab runs as two engine launches (gate+up
// with the SwiGLU epilogue, then down writing y) instead of three matvecs
// and an elementwise kernel.
static __device__ int32_t g_slab_idx = 0;
static __device__ float g_slab_w = 1.0f;

extern "C" int sepia_cuda_expert_swiglu(int gate_type, const void *gate, int up_type, const void *up, int down_type,
                                        const void *down, int64_t hidden, int64_t ff, const float *x, float *h,
                                        float *y, void *stream) {
    using namespace sepia;
    if (!gate || !up || !down || !x || !h || !y || hidden <= 0 || ff <= 0) return fail("expert_swiglu: bad arguments");
    cudaStream_t st = as_stream(stream);
    MoeDev L;
    memset(&L, 0, sizeof L);
    L.hidden = hidden; L.ff = ff;
    L.n_routed = 1; L.n_shared = 0; L.topk = 1;
    L.route_scale = 1.0; L.global_scale = 1.0f;
    L.gate_type = gate_type; L.up_type = up_type; L.down_type = down_type;
    L.gate = (const uint8_t *)gate; L.up = (const uint8_t *)up; L.down = (const uint8_t *)down;
    L.rb_gate = host_row_bytes(gate_type, hidden); L.rb_up = host_row_bytes(up_type, hidden);
    L.rb_down = host_row_bytes(down_type, ff);
    if (L.rb_gate <= 0 || L.rb_up <= 0 || L.rb_down <= 0) return fail("expert_swiglu: unsupported types or dims");
    L.gate_stride = L.rb_gate * ff; L.up_stride = L.rb_up * ff; L.down_stride = L.rb_down * hidden;
    L.rank = 0; L.world = 1; L.expert_slot = nullptr;
    L.err = dev_info().err;
    const bool eng = gate_type == up_type && engine_gateup_ok(L, nullptr) && engine_down_ok(L, nullptr) &&
                     (reinterpret_cast<uintptr_t>(x) & 15) == 0 && (reinterpret_cast<uintptr_t>(h) & 15) == 0;
    if (!eng)
        return fail("expert_swiglu: types %d/%d/%d or alignment not on the tensor-core engine "
                    "(use matvec_q + silu_mul)", gate_type, up_type, down_type);
    // the one-slot selection, looked up once per device
    static std::mutex mu;
    static int32_t *idx_d[64] = {};
    static float *w_d[64] = {};
    int dev = 0;
    if (!check(cudaGetDevice(&dev), "expert_swiglu: cudaGetDevice")) return 0;
    if (dev < 0 || dev >= 64) return fail("expert_swiglu: device %d out of range", dev);
    {
        std::lock_guard<std::mutex> lk(mu);
        if (!idx_d[dev]) {
            void *a = nullptr, *b = nullptr;
            if (!check(cudaGetSymbolAddress(&a, g_slab_idx), "expert_swiglu: cudaGetSymbolAddress") ||
                !check(cudaGetSymbolAddress(&b, g_slab_w), "expert_swiglu: cudaGetSymbolAddress"))
                return 0;
            idx_d[dev] = (int32_t *)a;
            w_d[dev] = (float *)b;
        }
    }
    SepiaMoeWork ws;
    memset(&ws, 0, sizeof ws);
    ws.topk_idx = idx_d[dev];
    ws.weights = w_d[dev];
    ws.h = h;
    ws.slots = y;
    return launch_gateup_engine(L, x, &ws, st, false) && launch_down_engine(L, &ws, y, y, false, st);
}

extern "C" int sepia_cuda_topk_select(const float *scores, int32_t n, int32_t topk, int32_t *idx, void *stream) {
    if (!scores || !idx || n <= 0 || topk <= 0 || topk > n) return fail("topk_select: bad arguments");
    k_topk<<<1, 32, 0, as_stream(stream)>>>(scores, n, topk, idx);
    return check(cudaGetLastError(), "topk launch");
}

#ifdef SEPIA_ROUTER_STAMPS
extern "C" __attribute__((visibility("default"))) int sepia_router_stamps(void *dst) {
    return cudaMemcpyFromSymbol(dst, sepia::g_rstamps, sizeof(sepia::g_rstamps)) == cudaSuccess;
}
#endif
#ifdef SEPIA_QE_STAMPS
extern "C" __attribute__((visibility("default"))) int sepia_qe_stamps(void *dst) {
    return cudaMemcpyFromSymbol(dst, sepia::g_qe_stamps, sizeof(sepia::g_qe_stamps)) == cudaSuccess;
}
#endif
