// sepia_b200/csrc/moe_dev.cuh -- the device-side description of one MoE
// layer and the router pieces shared by the layer kernels (moe.cu) and the
// fused single-launch layer (moe_fused.cu).
#pragma once
#include "../../include/sepia_cuda.h"
#include "runtime.h"
#include "qengine.cuh"

namespace sepia {

constexpr int kMaxSlots = 16;      // topk + n_shared
constexpr int kRouterWarps = 8;
constexpr int kRouterChunk = 1024;       // router row elements per warp
constexpr int kRouterMaxExperts = 1024;  // n_routed + n_shared
constexpr int kRouterMaxChunks = 16;     // hidden <= 16384
__host__ __device__ inline int router_chunks(int64_t hidden) { return (int)((hidden + kRouterChunk - 1) / kRouterChunk); }
constexpr int kGuStagesMax = 8;
constexpr int kDnStagesMax = 8;
constexpr int kTRG = 8;            // max rows per gate/up unit
constexpr int kTRD = 4;            // rows per down unit
constexpr int kDnMaxSlots = 8;     // topk + n_shared handled by the down kernel

// --------------------------------------------------------------- device-side layer
struct MoeDev {
    int64_t hidden, ff;
    int n_routed, n_shared, topk;
    double route_scale;
    float global_scale;
    const float *router_w, *router_bias;
    int gate_type, up_type, down_type, sh_gate_type, sh_up_type, sh_down_type;
    const uint8_t *gate, *up, *down, *sh_gate, *sh_up, *sh_down;
    int64_t gate_stride, up_stride, down_stride, sh_gate_stride, sh_up_stride, sh_down_stride;
    int64_t rb_gate, rb_up, rb_down, rb_sh_gate, rb_sh_up, rb_sh_down;
    int rank, world;
    const int32_t *expert_slot;
    int *err;
};

// Active slots of this rank, in the reference's combine order.
// slot j < topk: routed expert idx[j]; slot topk+s: shared expert s.
__device__ __forceinline__ int active_slots(const MoeDev &L, const int32_t *idx, int (&slots)[kMaxSlots]) {
    int n = 0;
    for (int j = 0; j < L.topk; j++) {
        const int e = idx[j];
        if (e >= 0 && e < L.n_routed && (e % L.world) == L.rank) slots[n++] = j;
    }
    for (int s = 0; s < L.n_shared; s++)
        if ((s % L.world) == L.rank) slots[n++] = L.topk + s;
    return n;
}

__device__ __forceinline__ int64_t local_expert(const MoeDev &L, int e) {
    if (L.expert_slot) return L.expert_slot[e];
    return L.world > 1 ? e / L.world : e;
}

// ============================================================== router
// sigmoid as the reference computes it (1/(1+expf(-x)) in float), with
// expf taken as the correctly rounded float of the double exponential.
__device__ __forceinline__ float sigmoid_ref(float x) {
    const float e = (float)exp(-(double)x);
    return __fdiv_rn(1.0f, __fadd_rn(1.0f, e));
}
__device__ __forceinline__ float logsigmoid_ref(float x) {
    if (x >= 0.0f) return -log1pf((float)exp(-(double)x));
    return x - log1pf((float)exp((double)x));
}

// Order-preserving 32-bit key of a score: larger key = larger score, +0 and
// -0 equal (they compare equal in the reference's scan). 0 is below every
// score's key and marks a taken or absent entry.
__device__ __forceinline__ uint32_t score_key(float f) {
    const uint32_t u = __float_as_uint(f == 0.0f ? 0.0f : f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// moe_route_select (src/sepia.c:1329-1375) on one warp. Expert e's key sits
// in lane e % 32, register e / 32. The reference's repeated strict-'>' scan
// picks, at each step, the highest remaining score and the lowest index
// among equal ones: per step a warp max of the keys (redux.sync), then a
// warp min of the indices holding that key. Weights: log-sigmoid softmax
// over the k raw logits and the shared-sink logits, in slot order.
template <int KPL>
__device__ __forceinline__ void router_select(const MoeDev &L, const float2 *row_out, int32_t *topk_idx,
                                              float *weights, int lane) {
    // one round of loads: every entry's (score, log-sigmoid), plus the
    // shared-sink log-sigmoids (lanes 0 .. n_shared-1)
    uint32_t key[KPL];
    float lpv[KPL];
#pragma unroll
    for (int j = 0; j < KPL; j++) {
        const int e = lane + 32 * j;
        const float2 ro = e < L.n_routed ? __ldcg(&row_out[e]) : make_float2(0.0f, 0.0f);
        key[j] = e < L.n_routed ? score_key(ro.x) : 0u;
        lpv[j] = ro.y;
    }
    const float lp_sh = lane < L.n_shared ? __ldcg(&row_out[L.n_routed + lane].y) : 0.0f;
    int my_sel = -1;        // lane j < topk: the j-th pick
    float my_lp = -INFINITY;
    for (int k = 0; k < L.topk; k++) {
        uint32_t m = 0;
#pragma unroll
        for (int j = 0; j < KPL; j++) m = max(m, key[j]);
        m = __reduce_max_sync(0xffffffffu, m);
        uint32_t cand = 0xFFFFFFFFu;
#pragma unroll
        for (int j = KPL - 1; j >= 0; j--)
            if (key[j] == m) cand = (uint32_t)(lane + 32 * j);
        const int e = (int)__reduce_min_sync(0xffffffffu, cand);
        float lpe = 0.0f;
#pragma unroll
        for (int j = 0; j < KPL; j++) {
            if (lane + 32 * j == e) key[j] = 0u;
            if (j == (e >> 5)) lpe = lpv[j];
        }
        lpe = __shfl_sync(0xffffffffu, lpe, e & 31);
        if (lane == k) {
            my_sel = e;
            my_lp = lpe;
        }
    }
    const int n_sel = L.topk + L.n_shared;
    float lp = -INFINITY;
    {
        const float shv = __shfl_sync(0xffffffffu, lp_sh, (lane - L.topk) & 31);
        if (lane < L.topk) lp = my_lp;
        else if (lane < n_sel) lp = shv;
    }
    float lmax = lp;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) lmax = fmaxf(lmax, __shfl_xor_sync(0xffffffffu, lmax, o));
    const double ex = (lane < n_sel) ? exp((double)(lp - lmax)) : 0.0;
    double se = 0.0;
    for (int j = 0; j < n_sel; j++) se += __shfl_sync(0xffffffffu, ex, j);   // slot order
    const double lse = (double)lmax + log(se);
    const double scl = (double)L.route_scale * (double)L.global_scale;
    if (lane < n_sel) weights[lane] = (float)(exp((double)lp - lse) * scl);
    if (lane < L.topk) topk_idx[lane] = my_sel;
}

// Per-slot row sources of one launch, kept in the engine's shared job
// scratch: matrix bases (gate/up, or down), row bytes, format and splits;
// nsplit = 0 for slots this rank does not own; w = the slot's combine
// weight (down kernel: routed slots' router weights, 1 for shared ones).
struct MoeSlot {
    const uint8_t *a, *b;
    int64_t rb;
    int type, sbs, nsplit;
    float w;
};
static_assert(kMaxSlots * sizeof(MoeSlot) <= (size_t)kQeJobSmem, "slot table exceeds the job scratch");

// Host: SepiaMoeLayer -> MoeDev with geometry checks (0 + message on error).
int to_dev(const SepiaMoeLayer *in, MoeDev &L);
// Host: whether the tensor-core engine takes the gate/up resp. down rows.
bool engine_gateup_ok(const MoeDev &L, const SepiaMoeWork *ws);
bool engine_down_ok(const MoeDev &L, const SepiaMoeWork *ws);
// Single-launch layer (moe_fused.cu): work-area parts and the launch
// (1 launched, 0 error, -1 layer not eligible).
size_t moe_fused_sync_bytes(const SepiaMoeLayer *L);
size_t moe_fused_htab_bytes(const SepiaMoeLayer *L);
int launch_moe_fused(const MoeDev &L, const float *x, const SepiaMoeWork *ws, float *out, cudaStream_t st);

}  // namespace sepia
