// sepia_b200/csrc/moe_fused.cu -- one MoE layer for one token as ONE
// persistent kernel: router matvec and top-k selection, gate/up + SwiGLU of
// every selected routed expert and every shared expert, the down
// projections and the slot combine.
//
// Replaces the reference's real_mlp_moe_forward_gpu (src/sepia.c:3831-3974),
// which dispatches the router, synchronises the host for moe_route_select
// (src/sepia.c:1329-1375), dispatches each expert's gate/up/silu/down and
// synchronises again to combine on the host. The multi-kernel chain in
// moe.cu already keeps all of that on the device; this kernel also removes
// its kernel boundaries, where the weight stream stopped while one grid
// drained and the next one built its activation tables.
//
// One CTA per SM, all CTAs resident (cooperative launch). Every CTA walks
// the same kind of item sequence:
//   router rows      rows c, c+P, ... of the f32 router matrix (one bulk
//                    copy per row, issued before anything else), fp64 dot
//                    with x in 1024-element chunks;
//   gate/up units    slot-major list (shared experts first: they need no
//                    router), unit u = (slot, 8-row block of ff), CTA c takes
//                    u = c, c+P, ...; 8 gate rows + the matching 8 up rows
//                    form one 16-row MMA tile;
//   down items       slot-major list of 32-row blocks of each active slot's
//                    down matrix, CTA c takes one contiguous range (so it
//                    touches at most two slots' activation tables).
// Roles (as in qengine.cuh): one producer thread streams items into a ring
// of shared-memory stages with 1-D cp.async.bulk; consumer warps take the
// items' "pieces" (a piece = a few superblocks of one 16-row tile, or one
// 1024-element router chunk) round robin over the whole sequence, so warps
// stay busy whatever the item sizes; one reducer warp sums each item's
// piece partials in piece order (deterministic) and runs its epilogue.
//
// Cross-CTA dependencies go through counters in the work area (released
// with __threadfence + atomics, acquired with ld.acquire.gpu):
//   router rows done -> once all are counted, every CTA's producer reads the
//     rows' selection scores and runs the top-k selection itself (the
//     selection is deterministic, so all CTAs agree; CTA 0 also writes it
//     out) before its first routed item; the shared experts' epilogue waits
//     for the same selection (gamma);
//   gate/up blocks done per (slot, h superblock) -> the signaller whose
//     increment completes a superblock builds its tensor-core activation
//     table into global memory once; tables ready per slot -> producers
//     bulk-copy a slot's tables into shared memory before its first down
//     item;
//   down items done per 16-row tile -> the signaller completing a tile sums
//     its slot terms in the reference's order (routed j = 0..k-1, then
//     shared; src/sepia.c:1432-1470) into the output.
// Under a saturated memory system every dependent global access (a fence,
// an atomic, an L2 read) takes microseconds, so the kernel keeps as few of
// them as possible on the path of the weight stream: the reducer hands
// finished rows to a signaller warp that batches its fences.
// The last CTA to finish zeroes every counter, so each launch starts from
// zero. Every wait is bounded (kWaitCycles): on timeout the kernel records
// kErrWaitTimeout in the device error word and the waiting role stops; the
// work area's counters must then be zeroed again before the next call.
#include "moe_dev.cuh"
#include "stream.cuh"

#include <algorithm>

namespace sepia {

constexpr int kFCons = 13;            // consumer warps
constexpr int kFThreads = (kFCons + 3) * 32;   // + producer, reducer, signaller
constexpr int kFRecs = 32;            // reducer -> signaller record ring
constexpr int kFBatch = 16;           // signals per fence
constexpr int kFMaxPieces = 8;        // pieces per item (partials per stage)
constexpr int kFStagesMax = 8;
constexpr int kFTabSlots = 2;         // h table sets a CTA holds
constexpr int kFSyncHead = 4;         // router rows done, unused, CTAs done, unused

struct FArgs {
    MoeDev L;
    const float *x;
    float *out;
    float *logits;
    int32_t *topk_idx;
    float *weights;
    float *h;
    float *slots;          // [n_slots, hidden] slot terms
    float2 *row_out;       // [n_total] router (selection score, log-sigmoid)
    uint8_t *gtab;         // [n_slots, nsb_f, kTabSB] activation tables of h
    uint32_t *sync;
    int n_total, n_slots, nsb_h, nsb_f, tpu, n_tiles;
    int dn_rows, nd_slot, nd_total;      // rows per down item, items per slot, all slots
    int sbs_r, nsplit_r, sbs_s, nsplit_s;  // gate/up item splits (routed, shared)
    int rt_pieces, dn_ppt;               // router chunks; down pieces per 16-row tile
    int stages;
    uint32_t slot_bytes, red_off, xtab_off, htab_off, stage_off;
    long long wait_cycles;
};

__host__ __device__ inline uint32_t *f_rt_cnt(uint32_t *s) { return s; }
__host__ __device__ inline uint32_t *f_fin(uint32_t *s) { return s + 2; }
__host__ __device__ inline uint32_t *f_hc(uint32_t *s) { return s + kFSyncHead; }
__host__ __device__ inline uint32_t *f_tab(uint32_t *s, int n_slots, int nsb_f) {
    return s + kFSyncHead + n_slots * nsb_f;
}
__host__ __device__ inline uint32_t *f_dn(uint32_t *s, int n_slots, int nsb_f) {
    return s + kFSyncHead + n_slots * nsb_f + n_slots;
}
__host__ __device__ inline size_t f_sync_words(int n_slots, int nsb_f, int n_tiles) {
    return (size_t)kFSyncHead + (size_t)n_slots * nsb_f + n_slots + n_tiles;
}

__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_gpu(uint32_t *p, uint32_t v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// Orders this thread's generic-proxy accesses to global memory against its
// later async-proxy (bulk copy) accesses.
__device__ __forceinline__ void fence_proxy_async_global() {
    asm volatile("fence.proxy.async.global;" ::: "memory");
}

// Bounded wait until *p >= target (acquire). false + error code on timeout.
__device__ __noinline__ bool wait_counter(const uint32_t *p, uint32_t target, int *err, long long limit) {
    if (ld_acquire_gpu(p) >= target) return true;
    const long long t0 = clock64();
    while (ld_acquire_gpu(p) < target) {
        if (clock64() - t0 > limit) {
            set_error(err, kErrWaitTimeout);
            return false;
        }
        __nanosleep(100);
    }
    return true;
}

// (a * n) / d for small non-negative a, n, d (d > 0) without an integer
// division: the +0.5 keeps the float quotient 0.5/d away from integers,
// beyond its rounding error for products below 2^22.
__device__ __forceinline__ int f_part(int a, int n, float inv_d) {
    return __float2int_rz(((float)(a * n) + 0.5f) * inv_d);
}

// Optional phase timestamps (-DSEPIA_QE_STAMPS): [CTA][phase] of the last
// launch in globaltimer nanoseconds.
#ifdef SEPIA_QE_STAMPS
__device__ unsigned long long g_fu_stamps[1024][16];
#define FU_STAMP(k)                                                                 \
    do {                                                                            \
        unsigned long long t_;                                                      \
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));                      \
        if (blockIdx.x < 1024) g_fu_stamps[blockIdx.x][k] = t_;                     \
    } while (0)
#else
#define FU_STAMP(k) \
    do {            \
    } while (0)
#endif

enum FKind : int { kFRouter = 0, kFX = 1, kFGateUp = 2, kFDown = 3 };

// A finished item, from the reducer to the signaller: row values of up to
// two 16-row tiles (router: v[0][0]).
struct FRec {
    double v[2][16];
    int kind, a, b, np;
};

struct FItem {
    int kind;
    int a;        // router: row; gate/up, down: slot-order index (shared slots first)
    int b;        // gate/up: 8-row block of ff; down: item within the slot
    int sp;       // gate/up split
};

// The item sequence of one CTA. Every role walks its own copy in the same
// order.
struct FSeq {
    int phase;         // an FKind, or 4 when done
    int r;             // router row
    int ga, gb, gsp;   // gate/up: slot-order index, block, split
    int d, d_end;      // down: global item index and end
    int da, db;        // down: slot-order index, item within slot

    __device__ void start(const FArgs &A) {
        phase = kFRouter;
        r = blockIdx.x;
        // gate/up unit blockIdx.x: slot-order index and block
        ga = 0;
        gb = blockIdx.x;
        while (ga < A.n_slots && gb >= A.tpu) { gb -= A.tpu; ga++; }
        gsp = 0;
        const int64_t P = gridDim.x;
        d = (int)((int64_t)blockIdx.x * A.nd_total / P);
        d_end = (int)((int64_t)(blockIdx.x + 1) * A.nd_total / P);
        da = 0;
        db = d;
        while (da < A.n_slots && db >= A.nd_slot) { db -= A.nd_slot; da++; }
        settle(A);
    }
    // advance phases that are empty for this CTA
    __device__ void settle(const FArgs &A) {
        if (phase == kFRouter && r >= A.n_total) phase = kFX;
        if (phase == kFGateUp && ga >= A.n_slots) phase = kFDown;
        if (phase == kFDown && d >= d_end) phase = 4;
    }
    __device__ bool done() const { return phase == 4; }
    __device__ FItem item() const {
        FItem it;
        it.kind = phase;
        it.sp = 0;
        it.a = it.b = 0;
        if (phase == kFRouter) it.a = r;
        else if (phase == kFGateUp) { it.a = ga; it.b = gb; it.sp = gsp; }
        else if (phase == kFDown) { it.a = da; it.b = db; }
        return it;
    }
    __device__ void next(const FArgs &A) {
        if (phase == kFRouter) {
            r += gridDim.x;
        } else if (phase == kFX) {
            phase = kFGateUp;
        } else if (phase == kFGateUp) {
            const int ns = (ga < A.L.n_shared) ? A.nsplit_s : A.nsplit_r;
            if (++gsp >= ns) {
                gsp = 0;
                gb += gridDim.x;
                while (ga < A.n_slots && gb >= A.tpu) { gb -= A.tpu; ga++; }
            }
        } else if (phase == kFDown) {
            d++;
            if (++db == A.nd_slot) { db = 0; da++; }
        }
        settle(A);
    }
};

// Router rows of this CTA (they precede the x item in its sequence).
__device__ __forceinline__ int f_router_rows(const FArgs &A) {
    return (int)blockIdx.x < A.n_total ? (A.n_total - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
}

// slot-order index -> slot (routed j < topk, then shared): shared first
__device__ __forceinline__ int f_slot(const FArgs &A, int a) {
    return a < A.L.n_shared ? A.L.topk + a : a - A.L.n_shared;
}

// Pieces of a gate/up item of n superblocks: about half the consumer warps
// per item, so that about two items are in consumption and the rest of the
// stage ring is loading.
constexpr int kFGuPieces = 7;
__host__ __device__ __forceinline__ int f_gu_pieces(int n) { return n < kFGuPieces ? n : kFGuPieces; }

__device__ __forceinline__ int f_pieces(const FArgs &A, const FItem &it) {
    if (it.kind == kFRouter) return A.rt_pieces;
    if (it.kind == kFX) return 1;
    if (it.kind == kFGateUp) {
        const bool sh = it.a < A.L.n_shared;
        const int sbs = sh ? A.sbs_s : A.sbs_r;
        const int s0 = it.sp * sbs;
        const int n = min(A.nsb_h, s0 + sbs) - s0;
        return f_gu_pieces(n);
    }
    const int r0 = it.b * A.dn_rows;
    const int ntile = (min(A.dn_rows, (int)A.L.hidden - r0) + 15) >> 4;
    return ntile * A.dn_ppt;
}

// Stage layout of a gate/up item (the engine's copy shapes: whole rows as
// two 8-row blocks, or per-row copies of a superblock range).
struct FGu {
    const uint8_t *lo, *hi;   // first superblock of the item, row 0 / row 8
    int64_t rb;
    int type, s0, n;          // superblocks [s0, s0 + n)
    bool block;
};
__device__ __forceinline__ FGu f_gu(const FArgs &A, const MoeSlot *S, const FItem &it) {
    const MoeSlot &m = S[f_slot(A, it.a)];
    FGu g;
    g.rb = m.rb;
    g.type = m.type;
    g.block = m.nsplit == 1;
    g.s0 = it.sp * m.sbs;
    g.n = min(A.nsb_h, g.s0 + m.sbs) - g.s0;
    const int64_t off = (int64_t)it.b * 8 * m.rb + (int64_t)g.s0 * qe_sb_bytes(m.type);
    g.lo = m.a + off;
    g.hi = m.b + off;
    return g;
}

// Issue the copies of a router row or gate/up item; called by the whole
// producer warp. A bulk copy costs its issuing thread ~200 ns, so the 16
// per-row copies of a split item go out from 16 lanes at once.
__device__ __forceinline__ void f_issue(const FArgs &A, const MoeSlot *S, const FItem &it, uint8_t *dst,
                                        uint64_t *full, int lane) {
    const MoeDev &L = A.L;
    if (it.kind == kFRouter || it.kind == kFX) {
        // a router row, or the layer input x (one copy for the whole CTA
        // instead of thousands of loads of the same lines by every CTA)
        if (lane == 0) {
            const uint32_t bytes = (uint32_t)(L.hidden * 4);
            mbar_arrive_expect_tx(full, bytes);
            bulk_g2s(dst, it.kind == kFX ? A.x : L.router_w + (int64_t)it.a * L.hidden, bytes, full);
        }
        return;
    }
    const FGu g = f_gu(A, S, it);
    if (g.block) {
        if (lane == 0) {
            const ByteRange rl{g.lo, (uint32_t)(8 * g.rb)}, rh{g.hi, (uint32_t)(8 * g.rb)};
            mbar_arrive_expect_tx(full, range_copy_bytes(rl) + range_copy_bytes(rh));
            range_issue(dst, rl, full);
            range_issue(dst + qe_hi_off(g.rb), rh, full);
        }
        return;
    }
    const uint32_t bytes = (uint32_t)g.n * (uint32_t)qe_sb_bytes(g.type);
    const uint32_t pitch = qe_pitch(bytes);
    // lane i < 16: row i (rows 8-15 are the up rows)
    const int i = lane & 15;
    const ByteRange r{(i < 8 ? g.lo : g.hi) + (i & 7) * g.rb, bytes};
    uint32_t tx = lane < 16 ? range_copy_bytes(r) : 0u;
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) tx += __shfl_xor_sync(0xffffffffu, tx, o);
    if (lane == 0) mbar_arrive_expect_tx(full, tx);
    __syncwarp();
    if (lane < 16) range_issue(dst + i * pitch, r, full);
}

__global__ void __launch_bounds__(kFThreads, 1) k_moe_fused(const FArgs A) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ __align__(16) MoeSlot S[kMaxSlots];
    __shared__ const uint8_t *Sd[kMaxSlots];       // down matrix of each slot
    __shared__ int32_t sel_idx[kMaxSlots];         // this CTA's copy of the top-k selection
    __shared__ float sel_w[kMaxSlots];             // routed weights, then shared gammas
    __shared__ volatile int sel_ready;             // set once sel_* hold the selection
    const MoeDev &L = A.L;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int prod = kFCons, redw = kFCons + 1, sigw = kFCons + 2;
    if (threadIdx.x == 0) FU_STAMP(0);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem);
    uint64_t *ready = full + kFStagesMax;
    uint64_t *empty = ready + kFStagesMax;
    uint64_t *tabb = empty + kFStagesMax;            // [kFTabSlots] h table arrival
    uint64_t *sig_full = tabb + kFTabSlots;          // [kFRecs] record written
    uint64_t *sig_empty = sig_full + kFRecs;         // [kFRecs] record consumed
    __shared__ FRec recs[kFRecs];
    double *red = reinterpret_cast<double *>(smem + A.red_off);     // [stages][kFMaxPieces][16]
    uint8_t *xtab = smem + A.xtab_off;
    uint8_t *htab = smem + A.htab_off;
    uint8_t *stage0 = smem + A.stage_off;
    uint32_t *sync = A.sync;
    const int nsb_tab = A.nsb_f;

    // shared-expert slot descriptors need nothing from a predecessor
    if (threadIdx.x < L.n_shared) {
        MoeSlot &m = S[L.topk + threadIdx.x];
        const int e = threadIdx.x;
        m.a = L.sh_gate + (int64_t)e * L.sh_gate_stride;
        m.b = L.sh_up + (int64_t)e * L.sh_up_stride;
        m.rb = L.rb_sh_gate; m.type = L.sh_gate_type; m.sbs = A.sbs_s; m.nsplit = A.nsplit_s;
        m.w = 1.0f;
        Sd[L.topk + e] = L.sh_down + (int64_t)e * L.sh_down_stride;
    }
    if (threadIdx.x == 0) {
        sel_ready = 0;
        for (int s = 0; s < A.stages; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&ready[s], kFCons);
            mbar_init(&empty[s], 1);
        }
        for (int t = 0; t < kFTabSlots; t++) mbar_init(&tabb[t], 1);
        for (int r = 0; r < kFRecs; r++) {
            mbar_init(&sig_full[r], 1);
            mbar_init(&sig_empty[r], 1);
        }
        fence_barrier_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) FU_STAMP(15);

    // the slot-order index of this CTA's first down item: its h tables go to
    // table set (slot-order index - da0)
    const int da0 = (int)((int64_t)blockIdx.x * A.nd_total / gridDim.x) / max(1, A.nd_slot);

    // ------------------------------------------------------------ producer
    // The whole warp runs the loop (lane 0 waits and signals, the lanes
    // share the per-row copies of split items).
    if (warp == prod) {
        FSeq q;
        q.start(A);
        QeRing ring;
        int64_t k = 0;
        int *err = L.err;
        // lane 0 waits, the warp follows
        auto wwait = [&](bool ok_lane0) -> bool {
            const bool ok = __shfl_sync(0xffffffffu, ok_lane0 ? 1 : 0, 0) != 0;
            __syncwarp();
            return ok;
        };
        // Router rows depend on nothing and go out before the dependency
        // wait; the x item (the layer input) is the first one after it.
        while (!q.done() && k < A.stages) {
            const FItem it = q.item();
            if (it.kind != kFRouter) break;
            f_issue(A, S, it, stage0 + (size_t)ring.slot * A.slot_bytes, &full[ring.slot], lane);
            k++;
            ring.next(A.stages);
            q.next(A);
        }
        griddep_wait();
        if (lane == 0) FU_STAMP(1);
        bool have_topk = false;
        while (!q.done()) {
            const FItem it = q.item();
            q.next(A);
            if (k >= A.stages &&
                !wwait(lane != 0 || mbar_wait(&empty[ring.slot], ring.phase ^ 1u, err, A.wait_cycles)))
                break;
            if (!have_topk && (it.kind == kFDown || (it.kind == kFGateUp && it.a >= L.n_shared))) {
                // Every router row is counted: this warp runs the (deterministic)
                // selection itself on the rows' scores -- one dependent read
                // instead of waiting for another CTA to select and publish.
                if (lane == 0) FU_STAMP(11);
                if (!wwait(lane != 0 || wait_counter(f_rt_cnt(sync), (uint32_t)A.n_total, err, A.wait_cycles))) break;
                __threadfence();
                if (L.n_routed <= 8 * 32) router_select<8>(L, A.row_out, sel_idx, sel_w, lane);
                else router_select<kRouterMaxExperts / 32>(L, A.row_out, sel_idx, sel_w, lane);
                __syncwarp();
                if (blockIdx.x == 0) {
                    // the selection as the layer's outputs
                    if (lane < L.topk) A.topk_idx[lane] = sel_idx[lane];
                    if (lane < A.n_slots) A.weights[lane] = sel_w[lane];
                }
                if (lane == 0) {
                    for (int j = 0; j < L.topk; j++) {
                        MoeSlot &m = S[j];
                        const int e = sel_idx[j];
                        const int64_t le = (e >= 0 && e < L.n_routed) ? local_expert(L, e) : 0;
                        m.a = L.gate + le * L.gate_stride;
                        m.b = L.up + le * L.up_stride;
                        m.rb = L.rb_gate; m.type = L.gate_type; m.sbs = A.sbs_r; m.nsplit = A.nsplit_r;
                        m.w = sel_w[j];
                        Sd[j] = L.down + le * L.down_stride;
                    }
                    __threadfence_block();
                    sel_ready = 1;
                    FU_STAMP(2);
                }
                __syncwarp();
                have_topk = true;
            }
            uint8_t *dst = stage0 + (size_t)ring.slot * A.slot_bytes;
            if (it.kind == kFDown) {
                if (lane == 0) {
                    const int s = f_slot(A, it.a);
                    const int64_t rb = s < L.topk ? L.rb_down : L.rb_sh_down;
                    const int r0 = it.b * A.dn_rows;
                    const int nr = min(A.dn_rows, (int)L.hidden - r0);
                    const ByteRange rg{Sd[s] + (int64_t)r0 * rb, (uint32_t)(nr * rb)};
                    mbar_arrive_expect_tx(&full[ring.slot], range_copy_bytes(rg));
                    range_issue(dst, rg, &full[ring.slot]);
                }
            } else {
                f_issue(A, S, it, dst, &full[ring.slot], lane);
            }
            k++;
            ring.next(A.stages);
        }
        if (!have_topk) {
            // no routed item here: the signaller may still need the gammas
            if (wwait(lane != 0 || wait_counter(f_rt_cnt(sync), (uint32_t)A.n_total, err, A.wait_cycles))) {
                __threadfence();
                if (L.n_routed <= 8 * 32) router_select<8>(L, A.row_out, sel_idx, sel_w, lane);
                else router_select<kRouterMaxExperts / 32>(L, A.row_out, sel_idx, sel_w, lane);
                __syncwarp();
                if (blockIdx.x == 0) {
                    if (lane < L.topk) A.topk_idx[lane] = sel_idx[lane];
                    if (lane < A.n_slots) A.weights[lane] = sel_w[lane];
                }
                if (lane == 0) {
                    __threadfence_block();
                    sel_ready = 1;
                }
            }
        }
        if (lane == 0) {
            FU_STAMP(4);
            // no bulk copy may be in flight when the CTA exits
            for (int64_t j = (k > A.stages ? k - A.stages : 0); j < k; j++)
                mbar_wait(&full[j % A.stages], (uint32_t)((j / A.stages) & 1), nullptr, A.wait_cycles);
        }
        return;
    }

    griddep_wait();

    // ------------------------------------------------------------ reducer
    // Sums each item's piece partials in piece order, frees the stage and
    // hands the finished row values to the signaller through a record ring.
    if (warp == redw) {
        FSeq q;
        q.start(A);
        QeRing ring;
        int *err = L.err;
        double gacc = 0.0;             // gate/up unit value across its splits (lane < 16)
        int64_t nrec = 0;
        while (!q.done()) {
            const FItem it = q.item();
            q.next(A);
            const int np = f_pieces(A, it);
            if (!mbar_wait(&ready[ring.slot], ring.phase, err, A.wait_cycles)) break;
            const double *rs = red + (size_t)ring.slot * kFMaxPieces * 16;
            double v0 = 0.0, v1 = 0.0;
            if (it.kind == kFDown) {
                const int ppt = A.dn_ppt;
                if (lane < 16) {
                    for (int j = 0; j < ppt; j++) v0 += rs[j * 16 + lane];
                    for (int j = ppt; j < np; j++) v1 += rs[j * 16 + lane];
                }
            } else if (lane < 16) {
                for (int j = 0; j < np; j++) v0 += rs[j * 16 + lane];
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[ring.slot]);
            ring.next(A.stages);
            if (it.kind == kFGateUp) {
                const int ns = (it.a < L.n_shared) ? A.nsplit_s : A.nsplit_r;
                gacc = (it.sp == 0 ? 0.0 : gacc) + v0;
                if (it.sp + 1 < ns) continue;
                v0 = gacc;
            }
            if (it.kind == kFX) continue;
            if (it.kind == kFRouter) {
                // router rows are on the critical path: publish and count now
                if (lane == 0) {
                    const int row = it.a;
                    const float l = (float)v0;
                    A.logits[row] = l;
                    const float score = row < L.n_routed ? __fadd_rn(sigmoid_ref(l), L.router_bias[row]) : 0.0f;
                    A.row_out[row] = make_float2(score, logsigmoid_ref(l));
                    __threadfence();
                    atomicAdd(f_rt_cnt(sync), 1u);
                    FU_STAMP(8);
                }
                continue;
            }
            const int ri = (int)(nrec % kFRecs);
            if (nrec >= kFRecs && !mbar_wait(&sig_empty[ri], (uint32_t)(((nrec / kFRecs) - 1) & 1), err, A.wait_cycles))
                break;
            FRec &rc = recs[ri];
            if (lane < 16) {
                rc.v[0][lane] = v0;
                rc.v[1][lane] = v1;
            }
            if (lane == 0) {
                rc.kind = it.kind;
                rc.a = it.a;
                rc.b = it.b;
                rc.np = np;
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&sig_full[ri]);
            nrec++;
        }
        return;
    }

    // ------------------------------------------------------------ signaller
    // Runs the gate/up and down epilogues (h = silu(g)*u, slot terms) and
    // their cross-CTA signals. Signals are batched: the stores of the
    // records at hand go out, then one fence, then their counter increments
    // (one lane each), then the actions of the counters that completed (an
    // h table, a tile's combine). Under a saturated memory system a fence or
    // an atomic takes microseconds, so the signaller flushes only when its
    // batch is full or the CTA moves on to another phase; the reducer hands
    // it records through a ring and never waits for it unless the ring is
    // full.
    if (warp == sigw) {
        FSeq q;
        q.start(A);
        int *err = L.err;
        bool have_sel = false, ok = true;
        int64_t nrec = 0;
        auto wwait_sig = [&](bool ok_lane0) -> bool {
            const bool r = __shfl_sync(0xffffffffu, ok_lane0 ? 1 : 0, 0) != 0;
            __syncwarp();
            return r;
        };
        // pending counter increments
        uint32_t *pc[kFBatch];
        int npend = 0;
        int prev_slot = -1;
        auto flush = [&]() {
            if (npend == 0) return;
            __syncwarp();
            __threadfence();
            if (lane < npend) atomicAdd(pc[lane], 1u);
            npend = 0;
        };
        auto push = [&](uint32_t *c) {
            if (npend == kFBatch) flush();
            pc[npend] = c;
            npend++;
        };
        // Designated work, spread over the CTAs so that it runs in parallel
        // (j = c, c + P, ... for CTA c): build h table j (slot * nsb_f + sb)
        // once all gate/up blocks of that superblock are counted; combine the
        // 16-row tile j once every slot's term of it is counted.
        bool tables_done = false;
        auto build_tables = [&]() {
            tables_done = true;
            for (int j = blockIdx.x; j < A.n_slots * A.nsb_f; j += gridDim.x) {
                const int s = j / A.nsb_f, sb = j - s * A.nsb_f;
                const uint32_t need = (uint32_t)(min(kQK, (int)L.ff - sb * kQK) / 8);
                if (!wwait_sig(lane != 0 || wait_counter(f_hc(sync) + j, need, err, A.wait_cycles))) return false;
                __threadfence();
                float hv8[8];
                xtab_load<true>(A.h + (int64_t)s * L.ff + (int64_t)sb * kQK, lane, hv8);
                xtab_emit(A.gtab + (size_t)j * kTabSB, hv8, lane);
                __threadfence();
                fence_proxy_async_global();
                __syncwarp();
                if (lane == 0) atomicAdd(f_tab(sync, A.n_slots, A.nsb_f) + s, 1u);
            }
            return true;
        };
        auto combine_tiles = [&]() {
            // this CTA's tiles t = c + i P (i < nt), one per lane, polled together
            const int nt = ((int)A.n_tiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;
            for (int i0 = 0; i0 < nt; i0 += 32) {
                const int i = i0 + lane;
                const uint32_t *cnt = f_dn(sync, A.n_slots, A.nsb_f) + blockIdx.x + (int64_t)i * gridDim.x;
                bool mine = i >= nt;
                const long long t0 = clock64();
                while (!__all_sync(0xffffffffu, mine)) {
                    if (!mine) mine = ld_acquire_gpu(cnt) >= (uint32_t)A.n_slots;
                    if (clock64() - t0 > A.wait_cycles) {
                        if (lane == 0) set_error(err, kErrWaitTimeout);
                        return false;
                    }
                    __nanosleep(100);
                }
                __threadfence();
                const int ntl = min(32, nt - i0);
                for (int q = lane; q < ntl * 16; q += 32) {
                    const int t = blockIdx.x + (i0 + (q >> 4)) * gridDim.x;
                    const int r = t * 16 + (q & 15);
                    if (r < L.hidden) {
                        float o = 0.0f;
                        for (int j = 0; j < A.n_slots; j++) o = __fadd_rn(o, __ldcg(A.slots + (int64_t)j * L.hidden + r));
                        A.out[r] = o;
                    }
                }
            }
            return true;
        };
        // h table sets this CTA's down items read: set ts holds slot-order
        // index da0 + ts; copied in by this warp as soon as they are built
        uint32_t tab_need = 0, tab_done = 0;
        {
            const int64_t P = gridDim.x;
            const int d0 = (int)((int64_t)blockIdx.x * A.nd_total / P);
            const int d1 = (int)((int64_t)(blockIdx.x + 1) * A.nd_total / P);
            if (d1 > d0) {
                const int a1 = (d1 - 1) / A.nd_slot;
                for (int a = da0; a <= a1; a++) tab_need |= 1u << (a - da0);
            }
        }
        auto try_tables = [&](bool block) -> bool {
            for (int ts = 0; ts < kFTabSlots; ts++) {
                if (!((tab_need & ~tab_done) >> ts & 1u)) continue;
                const int s = f_slot(A, da0 + ts);
                const uint32_t *tr = f_tab(sync, A.n_slots, A.nsb_f) + s;
                bool ready;
                if (block) {
                    if (!wwait_sig(lane != 0 || wait_counter(tr, (uint32_t)A.nsb_f, err, A.wait_cycles))) return false;
                    ready = true;
                } else {
                    ready = __shfl_sync(0xffffffffu, lane == 0 ? (ld_acquire_gpu(tr) >= (uint32_t)A.nsb_f ? 1 : 0) : 0, 0);
                }
                if (!ready) continue;
                if (lane == 0) {
                    fence_proxy_async_global();
                    const uint32_t tb = (uint32_t)A.nsb_f * kTabSB;
                    mbar_arrive_expect_tx(&tabb[ts], tb);
                    bulk_g2s(htab + (size_t)ts * tb, A.gtab + (size_t)s * tb, tb, &tabb[ts]);
                }
                __syncwarp();
                tab_done |= 1u << ts;
            }
            return true;
        };
        int prev_kind = kFRouter;
        while (!q.done()) {
            const FItem it = q.item();
            q.next(A);
            if (it.kind == kFRouter || it.kind == kFX) continue;   // the reducer handles these
            if (it.kind == kFGateUp) {
                const int ns = (it.a < L.n_shared) ? A.nsplit_s : A.nsplit_r;
                if (it.sp + 1 < ns) continue;
            }
            // a phase change flushes what the previous phase left pending; this
            // CTA's gate/up signals are then all out, and its designated tables
            // come before its own down records (which may need other tables)
            if (it.kind != prev_kind) {
                flush();
                if (it.kind == kFDown) {
                    if (!tables_done && !build_tables()) { ok = false; break; }
                    if (!try_tables(true)) { ok = false; break; }
                }
            }
            prev_kind = it.kind;
            const int ri = (int)(nrec % kFRecs);
            const uint32_t par = (uint32_t)((nrec / kFRecs) & 1);
            if (!mbar_wait(&sig_full[ri], par, err, A.wait_cycles)) { ok = false; break; }
            const FRec &rc = recs[ri];
            const double v0 = lane < 16 ? rc.v[0][lane] : 0.0;
            const double v1 = lane < 16 ? rc.v[1][lane] : 0.0;
            const int kind = rc.kind, ra = rc.a, rb = rc.b, np = rc.np;
            __syncwarp();
            if (lane == 0) mbar_arrive(&sig_empty[ri]);
            nrec++;
            if (kind == kFGateUp) {
                const int s = f_slot(A, ra);
                const bool sh = s >= L.topk;
                if (sh && !have_sel) {
                    // gamma comes from the selection (this CTA's producer runs it)
                    flush();
                    const long long t0 = clock64();
                    while (!sel_ready) {
                        if (clock64() - t0 > A.wait_cycles) break;
                        __nanosleep(200);
                    }
                    if (!sel_ready) {
                        set_error(err, kErrWaitTimeout);
                        ok = false;
                        break;
                    }
                    __threadfence_block();
                    have_sel = true;
                }
                const float uv = (float)__shfl_sync(0xffffffffu, v0, (lane + 8) & 31);
                if (lane < 8) {
                    const float gv = (float)v0;
                    const float sig = __fdiv_rn(1.0f, __fadd_rn(1.0f, (float)exp(-(double)gv)));
                    float hv = __fmul_rn(__fmul_rn(gv, sig), uv);
                    if (sh) hv = __fmul_rn(hv, sel_w[s]);
                    A.h[(int64_t)s * L.ff + (int64_t)rb * 8 + lane] = hv;
                }
                const int sb = (rb * 8) / kQK;
                // a CTA's gate/up units are slot-major: flush at each slot change so
                // that early slots' tables (and their down items) need not wait
                // for the end of the gate/up phase
                if (s != prev_slot) {
                    flush();
                    if (tab_need & ~tab_done) try_tables(false);
                }
                prev_slot = s;
                push(f_hc(sync) + s * A.nsb_f + sb);
            } else {
                const int s = f_slot(A, ra);
                const float w = S[s].w;
                const int r0 = rb * A.dn_rows;
                const int ntile = np / A.dn_ppt;
                for (int tt = 0; tt < ntile; tt++) {
                    const int rr = r0 + 16 * tt;
                    const double v = tt == 0 ? v0 : v1;
                    if (lane < 16 && rr + lane < L.hidden) {
                        const float e = (float)v;
                        A.slots[(int64_t)s * L.hidden + rr + lane] = (s < L.topk) ? __fmul_rn(e, w) : e;
                    }
                    push(f_dn(sync, A.n_slots, A.nsb_f) + (rr >> 4));
                }
            }
        }
        flush();
        if (ok && !tables_done) ok = build_tables();
        if (ok) ok = combine_tiles();
        // no bulk copy may be in flight when the CTA exits
        if (lane == 0)
            for (int ts = 0; ts < kFTabSlots; ts++)
                if (tab_done >> ts & 1u) mbar_wait(&tabb[ts], 0, nullptr, A.wait_cycles);
        (void)ok;
        // the last CTA to finish zeroes every counter for the next launch
        __syncwarp();
        unsigned int last = 0;
        if (lane == 0) {
            __threadfence();
            last = (atomicAdd(f_fin(sync), 1u) == gridDim.x - 1u) ? 1u : 0u;
        }
        if (__shfl_sync(0xffffffffu, last, 0)) {
            __threadfence();
            const size_t nw = f_sync_words(A.n_slots, A.nsb_f, A.n_tiles);
            for (size_t i = lane; i < nw; i += 32) sync[i] = 0u;
            __threadfence();
        }
        if (lane == 0) FU_STAMP(7);
        griddep_launch();
        return;
    }

    // ------------------------------------------------------------ consumers
    // The x item (the layer input, one bulk copy) comes right after this
    // CTA's router rows; the x table for the gate/up items is built from it
    // first, and the router rows read x from it too.
    const int nr_rows = f_router_rows(A);
    const float *xs = reinterpret_cast<const float *>(stage0 + (size_t)(nr_rows % A.stages) * A.slot_bytes);
    if (warp == 0 && lane == 0) FU_STAMP(12);
    if (!mbar_wait(&full[nr_rows % A.stages], (uint32_t)((nr_rows / A.stages) & 1), L.err, A.wait_cycles)) return;
    {
        const int n_build = A.nsb_h;
        for (int sb = warp; sb < n_build; sb += kFCons) {
            float v[8];
            xtab_load<false>(xs + (size_t)sb * kQK, lane, v);
            xtab_emit(xtab + (size_t)sb * kTabSB, v, lane);
        }
        named_bar_sync(1, kFCons * 32);
        if (warp == 0 && lane == 0) FU_STAMP(5);
    }
    const LaneCtx C = lane_ctx(lane);
    FSeq q;
    q.start(A);
    QeRing ring;
    int bm = 0;                      // first piece of the current item, mod kFCons
    uint32_t tab_seen = 0;
    int *err = L.err;
    while (!q.done()) {
        const FItem it = q.item();
        q.next(A);
        const int np = f_pieces(A, it);
        int j = warp - bm;
        if (j < 0) j += kFCons;
        bm += np;
        if (bm >= kFCons) bm -= kFCons;
        const int slot = ring.slot;
        if (it.kind == kFDown && !tab_seen && warp == 0 && lane == 0) FU_STAMP(9);
        if (!mbar_wait(&full[slot], ring.phase, err, A.wait_cycles)) return;
        ring.next(A.stages);
        if (j < np) {
            const uint8_t *st = stage0 + (size_t)slot * A.slot_bytes;
            double *rs = red + ((size_t)slot * kFMaxPieces + j) * 16;
            if (it.kind == kFX) {
                // the x item has one (empty) piece: its owner only arrives
            } else if (it.kind == kFRouter) {
                const int64_t c0 = (int64_t)j * kRouterChunk;
                const int64_t n = imin64(kRouterChunk, L.hidden - c0);
                const float *w = reinterpret_cast<const float *>(st) + c0;
                const float *xc = xs + c0;
                double acc = 0.0;
                if (n == kRouterChunk) {
                    constexpr int kV = kRouterChunk / 128;
                    double a2[2] = {0.0, 0.0};
#pragma unroll
                    for (int i = 0; i < kV; i++) {
                        const float4 wv = reinterpret_cast<const float4 *>(w)[lane + 32 * i];
                        const float4 xv = reinterpret_cast<const float4 *>(xc)[lane + 32 * i];
                        a2[i & 1] = fma((double)wv.x, (double)xv.x, a2[i & 1]);
                        a2[i & 1] = fma((double)wv.y, (double)xv.y, a2[i & 1]);
                        a2[i & 1] = fma((double)wv.z, (double)xv.z, a2[i & 1]);
                        a2[i & 1] = fma((double)wv.w, (double)xv.w, a2[i & 1]);
                    }
                    acc = a2[0] + a2[1];
                } else {
                    for (int64_t i = lane; i < n; i += 32) acc = fma((double)w[i], (double)xc[i], acc);
                }
                acc = warp_sum_d(acc);
                if (lane == 0) rs[0] = acc;
            } else {
                const uint8_t *rg, *rg8, *te;
                int type, i0, i1, flip;
                if (it.kind == kFGateUp) {
                    const FGu g = f_gu(A, S, it);
                    type = g.type;
                    const int npc = f_gu_pieces(g.n);
                    const float inv = 1.0f / (float)npc;
                    i0 = f_part(j, g.n, inv);
                    i1 = f_part(j + 1, g.n, inv);
                    const uintptr_t a_lo = reinterpret_cast<uintptr_t>(g.lo + C.gid * g.rb);
                    if (g.block) {
                        rg = st + (reinterpret_cast<uintptr_t>(g.lo) & 15) + C.gid * g.rb;
                        rg8 = st + qe_hi_off(g.rb) + (reinterpret_cast<uintptr_t>(g.hi) & 15) + C.gid * g.rb;
                    } else {
                        const uint32_t pitch = qe_pitch((uint32_t)g.n * (uint32_t)qe_sb_bytes(g.type));
                        const uintptr_t a_hi = reinterpret_cast<uintptr_t>(g.hi + C.gid * g.rb);
                        rg = st + C.gid * pitch + (a_lo & 15);
                        rg8 = st + (C.gid + 8) * pitch + (a_hi & 15);
                    }
                    te = xtab + (size_t)g.s0 * kTabSB;
                    flip = (int)(a_lo & 2) >> 1;
                } else {
                    const int s = f_slot(A, it.a);
                    const int ts = it.a - da0;
                    if (!(tab_seen >> ts & 1u)) {
                        if (!mbar_wait(&tabb[ts], 0, err, A.wait_cycles)) return;
                        tab_seen |= 1u << ts;
                    }
                    const int64_t rb = s < L.topk ? L.rb_down : L.rb_sh_down;
                    const uint8_t *base = Sd[s];
                    type = s < L.topk ? L.down_type : L.sh_down_type;
                    const int tt = j >= A.dn_ppt ? 1 : 0;
                    const int jj = j - tt * A.dn_ppt;
                    const int r0 = it.b * A.dn_rows;
                    base += (int64_t)r0 * rb;
                    const float inv = 1.0f / (float)A.dn_ppt;
                    i0 = f_part(jj, A.nsb_f, inv);
                    i1 = f_part(jj + 1, A.nsb_f, inv);
                    rg = st + (reinterpret_cast<uintptr_t>(base) & 15) + (16 * tt + C.gid) * rb;
                    rg8 = rg + 8 * rb;
                    te = htab + (size_t)ts * A.nsb_f * kTabSB;
                    flip = (int)(reinterpret_cast<uintptr_t>(base + (16 * tt + C.gid) * rb) & 2) >> 1;
                }
                double yg = 0.0, yg8 = 0.0;
                tile_sbs_rt(type, rg, rg8, te, i0, i1, flip, C, yg, yg8);
                quad_sum(yg, yg8);
                if (C.tig == 0) {
                    rs[C.gid] = yg;
                    rs[C.gid + 8] = yg8;
                }
            }
        }
        // Only the piece owners arrive (the owner of piece 0 also for the
        // warps without a piece): a warp busy with an earlier piece must not
        // hold up the completion of items it takes no part in.
        __syncwarp();
        if (lane == 0 && j < np) mbar_arrive_cnt(&ready[slot], j == 0 ? (uint32_t)(kFCons - np + 1) : 1u);
    }
    if (warp == 0 && lane == 0) FU_STAMP(6);
}

// ------------------------------------------------------------------ host
static int fused_plan(const MoeDev &L, FArgs &A, int64_t &smem, int &grid) {
    const DevInfo &di = dev_info();
    if (L.world != 1 || L.expert_slot) return 0;
    if (L.hidden % kQK || L.ff % kQK) return 0;
    A.nsb_h = (int)(L.hidden / kQK);
    A.nsb_f = (int)(L.ff / kQK);
    A.n_total = L.n_routed + L.n_shared;
    A.n_slots = L.topk + L.n_shared;
    A.tpu = (int)(L.ff / 8);
    A.n_tiles = (int)((L.hidden + 15) / 16);
    A.rt_pieces = router_chunks(L.hidden);
    if (A.rt_pieces > kFMaxPieces || A.nsb_h > 4 * kFMaxPieces) return 0;
    if ((reinterpret_cast<uintptr_t>(L.router_w) & 15) || (L.hidden * 4) % 16) return 0;
    if (A.n_total > kRouterMaxExperts) return 0;
    grid = di.sm_count > 0 ? di.sm_count : 148;
    // fixed shared memory: barriers, partials, x table, two h table sets
    const uint32_t bar_bytes = 8 * (3 * kFStagesMax + kFTabSlots + 2 * kFRecs);
    const uint32_t xtab = (uint32_t)A.nsb_h * kTabSB, htab = (uint32_t)kFTabSlots * A.nsb_f * kTabSB;
    // static shared memory of the kernel: slot descriptors, down bases, records
    const int64_t stat = (int64_t)(sizeof(MoeSlot) + sizeof(void *)) * kMaxSlots + (int64_t)sizeof(FRec) * kFRecs + 256;
    const int64_t avail = (int64_t)di.smem_optin - stat;
    const int64_t per_stage_red = kFMaxPieces * 16 * 8;
    const int64_t fixed = bar_bytes + xtab + htab + 3 * 128;
    // gate/up: whole rows if 16 rows fit a slot of a 4-stage ring
    const int64_t slot_cap = (avail - fixed) / 4 - per_stage_red;
    auto gu_split = [&](int t, int &sbs, int &nsplit) -> uint32_t {
        const int64_t rb = host_row_bytes(t, L.hidden);
        const uint32_t blk = qe_hi_off(rb) + (uint32_t)(8 * rb) + 32;
        if (blk <= slot_cap) { sbs = A.nsb_h; nsplit = 1; return blk; }
        const int sb = qe_sb_bytes(t);
        for (nsplit = 2; nsplit <= A.nsb_h; nsplit++) {
            sbs = (A.nsb_h + nsplit - 1) / nsplit;
            const uint32_t b = 16 * qe_pitch((uint32_t)sbs * sb);
            if (b <= slot_cap) { nsplit = (A.nsb_h + sbs - 1) / sbs; return b; }
        }
        return 0;
    };
    uint32_t need = (uint32_t)(L.hidden * 4) + 32;
    const uint32_t gr = gu_split(L.gate_type, A.sbs_r, A.nsplit_r);
    A.sbs_s = A.sbs_r; A.nsplit_s = A.nsplit_r;
    uint32_t gs = 0;
    if (L.n_shared) gs = gu_split(L.sh_gate_type, A.sbs_s, A.nsplit_s);
    if (!gr || (L.n_shared && !gs)) return 0;
    if ((A.sbs_r + 6) / 7 > 4 || (A.sbs_s + 6) / 7 > 4) return 0;      // at most 4 superblocks a piece
    need = std::max(need, std::max(gr, gs));
    const int64_t rbd = std::max<int64_t>(L.rb_down, L.n_shared ? L.rb_sh_down : 0);
    A.dn_rows = (32 * rbd + 32 <= slot_cap) ? 32 : 16;
    if (A.dn_rows * rbd + 32 > slot_cap) return 0;
    need = std::max(need, (uint32_t)(A.dn_rows * rbd + 32));
    A.dn_ppt = std::min(A.nsb_f, kFMaxPieces / (A.dn_rows / 16));
    A.nd_slot = (int)((L.hidden + A.dn_rows - 1) / A.dn_rows);
    A.nd_total = A.n_slots * A.nd_slot;
    // a CTA's down range must touch at most kFTabSlots slots
    if ((A.nd_total + grid - 1) / grid > A.nd_slot + 1) return 0;
    A.slot_bytes = (need + 127) & ~127u;
    A.stages = 0;
    for (int s = kFStagesMax; s >= 3; s--) {
        const int64_t tot = fixed + (int64_t)s * (A.slot_bytes + per_stage_red);
        if (tot <= avail) { A.stages = s; break; }
    }
    if (!A.stages) return 0;
    // the x item sits behind this CTA's router rows in the first ring round
    if ((A.n_total + grid - 1) / grid >= A.stages) return 0;
    A.red_off = bar_bytes;
    A.xtab_off = (A.red_off + (uint32_t)(A.stages * per_stage_red) + 127) & ~127u;
    A.htab_off = (A.xtab_off + xtab + 127) & ~127u;
    A.stage_off = (A.htab_off + htab + 127) & ~127u;
    smem = A.stage_off + (int64_t)A.stages * A.slot_bytes;
    return smem <= avail;
}

size_t moe_fused_sync_bytes(const SepiaMoeLayer *L) {
    const int n_slots = L->topk + L->n_shared;
    const int nsb_f = (int)((L->ff + kQK - 1) / kQK);
    const int n_tiles = (int)((L->hidden + 15) / 16);
    return f_sync_words(n_slots, nsb_f, n_tiles) * 4;
}

size_t moe_fused_htab_bytes(const SepiaMoeLayer *L) {
    const int n_slots = L->topk + L->n_shared;
    const int nsb_f = (int)((L->ff + kQK - 1) / kQK);
    return (size_t)n_slots * nsb_f * kTabSB;
}

// 1 = launched, 0 = error (message set), -1 = this layer does not take the
// fused path (the caller runs the kernel chain).
// The fused kernel walks the K-quant tiles only (no IQ codebook staging).
static bool fused_formats_ok(const MoeDev &L) {
    return mma_format(L.gate_type) && mma_format(L.down_type) &&
           (L.n_shared == 0 || (mma_format(L.sh_gate_type) && mma_format(L.sh_down_type)));
}

int launch_moe_fused(const MoeDev &L, const float *x, const SepiaMoeWork *ws, float *out, cudaStream_t st) {
    if (!ws->sync || !ws->htab || !fused_formats_ok(L)) return -1;
    if (!engine_gateup_ok(L, ws) || !engine_down_ok(L, ws)) return -1;
    FArgs A;
    int64_t smem = 0;
    int grid = 0;
    if (!fused_plan(L, A, smem, grid)) return -1;
    if (reinterpret_cast<uintptr_t>(x) & 15) return -1;      // x arrives by one bulk copy
    A.L = L;
    A.x = x; A.out = out;
    A.logits = ws->logits; A.topk_idx = ws->topk_idx; A.weights = ws->weights; A.h = ws->h;
    A.slots = ws->slots;
    A.row_out = reinterpret_cast<float2 *>(ws->router_part);
    A.gtab = reinterpret_cast<uint8_t *>(ws->htab);
    A.sync = ws->sync;
    A.wait_cycles = kWaitCycles;
    if (!ensure_smem((const void *)k_moe_fused, (int)smem)) return 0;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(kFThreads);
    cfg.dynamicSmemBytes = (size_t)smem;
    cfg.stream = st;
    cudaLaunchAttribute at[2];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    at[1].id = cudaLaunchAttributeCooperative;
    at[1].val.cooperative = 1;
    cfg.attrs = at;
    cfg.numAttrs = 2;
    return check(cudaLaunchKernelEx(&cfg, k_moe_fused, A), "moe fused layer launch");
}

}  // namespace sepia

extern "C" int sepia_cuda_moe_fused_eligible(const SepiaMoeLayer *Lh, const SepiaMoeWork *ws) {
    sepia::MoeDev L;
    if (!Lh || !ws || !sepia::to_dev(Lh, L)) return 0;
    if (!ws->sync || !ws->htab || !sepia::fused_formats_ok(L) || !sepia::engine_gateup_ok(L, ws) ||
        !sepia::engine_down_ok(L, ws))
        return 0;
    sepia::FArgs A;
    int64_t smem = 0;
    int grid = 0;
    return sepia::fused_plan(L, A, smem, grid);
}

extern "C" int sepia_cuda_moe_layer_fused(const SepiaMoeLayer *Lh, const float *x, const SepiaMoeWork *ws, float *out,
                                          void *stream) {
    sepia::MoeDev L;
    if (!sepia::to_dev(Lh, L)) return 0;
    if (!x || !ws || !out) return sepia::fail("moe_layer_fused: null argument");
    const int r = sepia::launch_moe_fused(L, x, ws, out, sepia::as_stream(stream));
    if (r < 0) return sepia::fail("moe_layer_fused: layer not eligible (see sepia_cuda_moe_fused_eligible)");
    return r;
}

#ifdef SEPIA_QE_STAMPS
extern "C" __attribute__((visibility("default"))) int sepia_fu_stamps(void *dst) {
    return cudaMemcpyFromSymbol(dst, sepia::g_fu_stamps, sizeof(sepia::g_fu_stamps)) == cudaSuccess;
}
#endif
