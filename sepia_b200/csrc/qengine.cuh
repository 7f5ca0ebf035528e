// sepia_b200/csrc/qengine.cuh -- the streaming tensor-core GEMV engine
// behind matvec_q and the MoE gate/up and down projections.
//
// Work is a list of units; a unit is one 16-row tile (rows 0-7 and 8-15 may
// come from two matrices, e.g. 8 gate rows and the 8 matching up rows) over
// all superblocks of the input, possibly cut into `nsplit` items along the
// superblocks so that one item fits a shared-memory stage. CTAs take units
// round robin (unit u goes to CTA u % grid) and walk every item of a unit in
// order, so one CTA owns a unit's whole row sum (deterministic).
//
// Warps of a CTA:
//   producer   one thread copies each item's rows into a stage slot with
//              1-D cp.async.bulk (one copy per row, 16-byte aligned rows,
//              padded pitch so the 8 rows of an MMA tile hit distinct
//              shared-memory banks), completing on the slot's "full" mbarrier;
//              the other warps build the activation tables first;
//   consumers  G groups of cg warps; group k % G takes item k, its warps
//              splitting the item's superblocks into cg chunks; each warp
//              runs the format's tile walk (qtile.cuh) and stores its fp64
//              row partials, then arrives on the slot's "ready" mbarrier;
//   reducer    sums the cg partials of every row in chunk order, adds the
//              unit's splits in order, runs the job's epilogue on the
//              finished rows and releases the slot on its "empty" mbarrier.
// Every wait is bounded (mbar_wait): on timeout the kernel records an error
// code and the waiting role stops.
#pragma once
#include "qtile.cuh"
#include "stream.cuh"

#include <algorithm>
#include <type_traits>

namespace sepia {

constexpr int kQeMaxCons = 16;
constexpr int kQeMaxStages = 8;
constexpr int kQeThreadsMax = (kQeMaxCons + 2) * 32;
constexpr int kQeBuildBatch = 4;           // table superblocks a warp loads before computing

struct QUnit {
    int type;              // quant format of both halves
    int nsb;               // superblocks per row
    int sbs;               // superblocks per split (the last split may be shorter)
    int nsplit;
    int nlo, nhi;          // valid rows in 0-7 and 8-15
    const uint8_t *lo;     // row i < 8 starts at lo + i*rb
    const uint8_t *hi;     // row 8+i starts at hi + i*rb
    int64_t rb;
    int tab;               // activation table index
};

__host__ __device__ inline int qe_sb_bytes(int t) { return fmt_block_bytes(t); }

// Whether a job may carry IQ formats (Job::kIq; 0 = none, an IQ type = only
// that format, -1 = any): only such launches stage the IQ codebooks in
// shared memory and compile the IQ tile walks.
template <class J, class = void> struct JobIq { static constexpr int v = 0; };
template <class J> struct JobIq<J, std::void_t<decltype(J::kIq)>> { static constexpr int v = J::kIq; };
// Whether a job's activation tables may be built before its dependency wait
// (Job::kTabsEarly): their sources were complete before the predecessor
// kernel let this one launch.
template <class J, class = void> struct JobTabsEarly { static constexpr bool v = false; };
template <class J> struct JobTabsEarly<J, std::void_t<decltype(J::kTabsEarly)>> { static constexpr bool v = J::kTabsEarly; };
// Whether a job's units carry two activation vectors (Job::kDual): tables
// U.tab and U.tab + 1 feed MMA columns 0-3 and 4-7, so one pass over the
// weights yields both vectors' rows (formats whose walks use only the
// natural B layout and no group-sum MMA, which needs all 8 columns:
// IQ2_XXS, IQ3_XXS, IQ1_S). finish() then sees 32 lanes: row lane % 16 of
// vector lane / 16.
template <class J, class = void> struct JobDual { static constexpr bool v = false; };
template <class J> struct JobDual<J, std::void_t<decltype(J::kDual)>> { static constexpr bool v = J::kDual; };
__host__ __device__ constexpr bool dual_format(int t) {
    return t == T_IQ2_XXS || t == T_IQ3_XXS || t == T_IQ1_S;
}
// Row pitch in a stage for `bytes` bytes per row: 16-byte multiple with an
// odd number of 16-byte granules (8 consecutive rows -> 8 distinct banks).
__host__ __device__ inline uint32_t qe_pitch(uint32_t bytes) {
    uint32_t p = (bytes + 32 + 15) & ~15u;     // + the partial granules around an unaligned row
    if (((p >> 4) & 1) == 0) p += 16;
    return p;
}

// Items of whole rows are copied as two blocks of 8 consecutive rows -- two
// bulk copies instead of 16: the copy engine's per-request cost dominates for
// rows of a few kilobytes, more than the shared-memory bank conflicts that a
// row stride with an even number of 16-byte granules brings.
__host__ __device__ inline bool qe_block_mode(const QUnit &U) {
    return U.nsplit == 1;
}
// Offset of the second block (rows 8-15) in a stage slot.
__host__ __device__ inline uint32_t qe_hi_off(int64_t rb) { return (uint32_t)((8 * rb + 30 + 15) & ~(int64_t)15); }

// Slot and phase of a stage ring, advanced item by item (no divisions).
struct QeRing {
    int slot = 0;
    uint32_t phase = 0;
    __device__ __forceinline__ void next(int stages) {
        if (++slot == stages) {
            slot = 0;
            phase ^= 1u;
        }
    }
};

struct QeLayout {
    int G, cg, stages;
    uint32_t slot_bytes, red_off, tab_off, stage_off;
    int n_tab, tab_nsb;    // tables x superblocks each
    uint32_t iq_off = 0;   // IQ codebook region (qtile.cuh), 0 = none
    IqLayout iq{};         // its layout
    int *err;
    long long wait_cycles = kWaitCycles;   // bound of every mbarrier wait
    uint32_t test_extra_tx = 0;            // test hook only: extra bytes the producer announces
};

// u / n for 0 <= u < 2^22 without an integer division: (u + 0.5) / n lies
// at least 0.5/n from an integer, more than the float product's error
// ((u + 0.5) / n * 2^-23) for such u; inv_n = 1/n rounded to float.
constexpr int kQeDivMax = 1 << 22;
__device__ __forceinline__ int qe_div(int u, float inv_n) { return __float2int_rz(((float)u + 0.5f) * inv_n); }

// Optional phase timestamps for profiling builds (-DSEPIA_QE_STAMPS):
// [job kind][CTA][phase] of the last launch, in globaltimer nanoseconds.
#ifdef SEPIA_QE_STAMPS
__device__ unsigned long long g_qe_stamps[2][1024][8];
#define QE_STAMP(k)                                                                 \
    do {                                                                            \
        unsigned long long t_;                                                      \
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));                      \
        if (blockIdx.x < 1024) g_qe_stamps[J.n_tab() > 1][blockIdx.x][k] = t_;      \
    } while (0)
#else
#define QE_STAMP(k) \
    do {            \
    } while (0)
#endif

constexpr int kQeJobSmem = 1024;     // shared scratch of a job (per-CTA unit tables)

// Job interface (see k_qengine):
//   void init();                              // per-thread setup (reads only data
//                                             //   that exists before griddep_wait)
//   void setup(uint8_t *jsm, int tid, bool after_dep);
//                                             // fill the job's shared scratch; called by
//                                             //   every thread before and after griddep_wait
//   int64_t n_units() const;
//   bool needs_dep(int64_t u) const;          // unit u's rows depend on the predecessor
//   void unit(const uint8_t *jsm, int64_t u, QUnit &U) const;   // U.nsplit = 0: nothing to do
//   int splits(const uint8_t *jsm, int64_t u) const;             // U.nsplit alone (cheap)
//   int n_tab() const;                        // activation tables (<= QeLayout.n_tab)
//   uint32_t tab_mask(const uint8_t *jsm) const;  // bit t: this CTA's units read table t (n_tab <= 32)
//   const float *tab_src(int t) const;       // activations of table t, written before the
//                                             //   predecessor completed (read through L2)
//   void finish(const uint8_t *jsm, int64_t u, const QUnit &U, double v, int lane) const;
//       called by the 32 reducer lanes with v = row `lane`'s value (lane < 16)
template <class Job>
__global__ void __launch_bounds__(kQeThreadsMax, 1) k_qengine(const Job Jp, const QeLayout P) {
    Job J = Jp;
    J.init();
    constexpr bool DUAL = JobDual<Job>::v;
    constexpr int RW = DUAL ? 32 : 16;          // reduction rows per consumer partial
    if (threadIdx.x == 0) QE_STAMP(0);
    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n_cons = P.G * P.cg, prod = n_cons, redw = n_cons + 1;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem);
    uint64_t *ready = full + kQeMaxStages;
    uint64_t *empty = ready + kQeMaxStages;
    double *red = reinterpret_cast<double *>(smem + P.red_off);      // [stages][cg][RW]
    uint8_t *tab = smem + P.tab_off;
    uint8_t *stage0 = smem + P.stage_off;
    const int64_t n_units = J.n_units();
    __shared__ __align__(16) uint8_t jsm[kQeJobSmem];
    J.setup(jsm, threadIdx.x, false);

    if (threadIdx.x == 0) {
        for (int s = 0; s < P.stages; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&ready[s], P.cg);
            mbar_init(&empty[s], 1);
        }
        fence_barrier_init();
    }
    __syncthreads();

    // producer: item k of this CTA goes to slot k % stages. Each row's bytes
    // are fetched as the 16-byte granules that cover them (range_issue), so
    // row i's data starts at stage + i*pitch + (its address & 15).
    auto issue = [&](const QUnit &U, int sp, int slot) {
        const int sbB = qe_sb_bytes(U.type);
        const int s0 = sp * U.sbs, s1 = min(U.nsb, s0 + U.sbs);
        const uint32_t bytes = (uint32_t)(s1 - s0) * (uint32_t)sbB;
        uint8_t *dst = stage0 + (size_t)slot * P.slot_bytes;
        if (qe_block_mode(U)) {
            // whole rows with a bank-friendly stride: two copies of 8 rows
            const ByteRange rl{U.lo, (uint32_t)(U.nlo * U.rb)}, rh{U.hi, (uint32_t)(U.nhi * U.rb)};
            mbar_arrive_expect_tx(&full[slot], range_copy_bytes(rl) + (U.nhi ? range_copy_bytes(rh) : 0u) + P.test_extra_tx);
            range_issue(dst, rl, &full[slot]);
            if (U.nhi) range_issue(dst + qe_hi_off(U.rb), rh, &full[slot]);
            return;
        }
        const uint32_t pitch = qe_pitch(bytes);
        const int64_t off = (int64_t)s0 * sbB;
        uint32_t tx = 0;
        for (int i = 0; i < U.nlo; i++) tx += range_copy_bytes(ByteRange{U.lo + i * U.rb + off, bytes});
        for (int i = 0; i < U.nhi; i++) tx += range_copy_bytes(ByteRange{U.hi + i * U.rb + off, bytes});
        mbar_arrive_expect_tx(&full[slot], tx + P.test_extra_tx);
        for (int i = 0; i < U.nlo; i++) range_issue(dst + i * pitch, ByteRange{U.lo + i * U.rb + off, bytes}, &full[slot]);
        for (int i = 0; i < U.nhi; i++)
            range_issue(dst + (8 + i) * pitch, ByteRange{U.hi + i * U.rb + off, bytes}, &full[slot]);
    };

    // Producer state: next (unit, split) to issue, item count, ring position.
    int64_t pu = blockIdx.x;
    int psp = 0;
    int64_t pk = 0;
    QeRing pring;
    QUnit PU;
    PU.nsplit = 0;
    // The first `stages` items need no empty-wait. Up to half of them, of
    // units that do not depend on the predecessor kernel, are issued before
    // waiting for it: more would only queue the table loads that follow the
    // wait behind weight data (measured +1 % on the MoE layer).
    if (warp == prod && lane == 0) {
        const int pre = max(1, P.stages / 2);
        while (pu < n_units && pk < pre && !J.needs_dep(pu)) {
            if (psp == 0) J.unit(jsm, pu, PU);
            if (psp < PU.nsplit) {
                issue(PU, psp, pring.slot);
                pk++;
                pring.next(P.stages);
            }
            if (++psp >= PU.nsplit) {
                psp = 0;
                pu += gridDim.x;
            }
        }
    }
    if (warp == prod && lane == 0) QE_STAMP(7);
    // IQ codebooks: constant data, staged by the non-producer warps before
    // the dependency wait; barrier 2 below publishes them to the consumers
    if constexpr (JobIq<Job>::v != 0) {
        if (P.iq_off && warp != prod) {
            const int t = warp < prod ? threadIdx.x : threadIdx.x - 32;
            iq_tabs_fill(smem + P.iq_off, P.iq, t, (n_cons + 1) * 32);
        }
    }
    // Build the activation tables this CTA's units read (non-producer warps).
    auto build_tabs = [&]() {
        // superblock q of the needed tables (in table order) goes to warp
        // q % nbw; a warp loads up to kQeBuildBatch of them before it
        // computes any, so their L2 latencies overlap
        const uint32_t mask = J.tab_mask(jsm);
        const int n_build = __popc(mask) * P.tab_nsb;
        const int bw = warp < prod ? warp : warp - 1, nbw = n_cons + 1;
        for (int q0 = bw; q0 < n_build; q0 += kQeBuildBatch * nbw) {
            float v[kQeBuildBatch][8];
            uint8_t *te[kQeBuildBatch];
#pragma unroll
            for (int i = 0; i < kQeBuildBatch; i++) {
                const int q = q0 + i * nbw;
                te[i] = nullptr;
                if (q < n_build) {
                    const int k = q / P.tab_nsb, sb = q - k * P.tab_nsb;
                    uint32_t m = mask;
                    for (int j = 0; j < k; j++) m &= m - 1;      // drop the k lowest tables
                    const int t = __ffs(m) - 1;
                    te[i] = tab + ((size_t)t * P.tab_nsb + sb) * kTabSB;
                    xtab_load<true>(J.tab_src(t) + (size_t)sb * kQK, lane, v[i]);
                }
            }
#pragma unroll
            for (int i = 0; i < kQeBuildBatch; i++)
                if (te[i]) xtab_emit(te[i], v[i], lane);
        }
    };
    // Jobs whose tables read only data that was final before their
    // predecessor started (kTabsEarly) build them before the dependency
    // wait, while the predecessor finishes.
    if constexpr (JobTabsEarly<Job>::v) {
        if (warp != prod) build_tabs();
    }
    griddep_wait();
    if (threadIdx.x == 0) {
        QE_STAMP(1);
        griddep_launch();
    }
    J.setup(jsm, threadIdx.x, true);
    // The producer needs only warp 0's post-dependency job scratch (named
    // barrier 1: warp 0 arrives, the producer waits); the other warps build
    // the activation tables their units read and meet on barrier 2. The
    // producer, possibly still blocked issuing its first copies, holds
    // nobody up.
    if (warp == prod) {
        named_bar_sync(1, 64);
    } else {
        if (warp == 0) named_bar_arrive(1, 64);
        if constexpr (!JobTabsEarly<Job>::v) build_tabs();
        named_bar_sync(2, (n_cons + 1) * 32);
    }

    if (warp == prod) {
        if (lane == 0) {
            // from round 1 on, item k waits for its slot's release in round - 1
            bool ok = true;
            while (pu < n_units) {
                if (psp == 0) J.unit(jsm, pu, PU);
                if (psp < PU.nsplit) {
                    if (pk >= P.stages && !mbar_wait(&empty[pring.slot], pring.phase ^ 1u, P.err, P.wait_cycles)) { ok = false; break; }
                    issue(PU, psp, pring.slot);
                    pk++;
                    pring.next(P.stages);
                }
                if (++psp >= PU.nsplit) {
                    psp = 0;
                    pu += gridDim.x;
                }
            }
            QE_STAMP(6);
            // No bulk copy may be in flight when the CTA exits, on the error
            // path too: the copies already issued complete on their "full"
            // barriers whatever the consumers do, so wait for each (bounded).
            (void)ok;
            for (int64_t j = (pk > P.stages ? pk - P.stages : 0); j < pk; j++)
                mbar_wait(&full[j % P.stages], (uint32_t)((j / P.stages) & 1), nullptr, P.wait_cycles);
        }
        return;
    }

    if (warp == redw) {
        QeRing ring;
        for (int64_t u = blockIdx.x; u < n_units; u += gridDim.x) {
            QUnit U;
            J.unit(jsm, u, U);
            if (U.nsplit == 0) continue;
            double acc = 0.0;
            bool ok = true;
            for (int sp = 0; sp < U.nsplit; sp++) {
                if (!mbar_wait(&ready[ring.slot], ring.phase, P.err, P.wait_cycles)) { ok = false; break; }
                if (lane < RW) {
                    const double *rs = red + (size_t)ring.slot * P.cg * RW + lane;
                    for (int c = 0; c < P.cg; c++) acc += rs[c * RW];
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[ring.slot]);
                ring.next(P.stages);
            }
            if (!ok) break;
            J.finish(jsm, u, U, acc, lane);
        }
        if (lane == 0) QE_STAMP(5);
        return;
    }

    // consumers
    if (warp == 0 && lane == 0) QE_STAMP(2);
    bool first = true;
    const int grp = warp / P.cg, cw = warp % P.cg;
    LaneCtx C = lane_ctx(lane);
    if constexpr (DUAL) {
        // columns 4-7 carry the second vector's limbs, not duplicates; a
        // lane's B operand comes from the table of its column gid, its C
        // columns (2tig, 2tig+1) belong to vector tig / 2, whose x unit
        // scales them
        C.lwn = C.lws;
        C.unit_off = ((C.tig >= 2 ? 1 : 0) - (C.gid >= 4 ? 1 : 0)) * P.tab_nsb * kTabSB;
    }
    QeRing ring;
    int g = 0;                        // group of the current item (item index % G)
    const float inv_cg = 1.0f / (float)P.cg;
    for (int64_t u = blockIdx.x; u < n_units; u += gridDim.x) {
        // units whose items all go to other groups need only their split count
        const int ns = J.splits(jsm, u);
        if (P.G > 1 && ns == 1 && g != grp) {
            ring.next(P.stages);
            if (++g == P.G) g = 0;
            continue;
        }
        QUnit U;
        J.unit(jsm, u, U);
        // DUAL: lanes that supply MMA columns 4-7 (gid >= 4) read the second
        // vector's table
        const uint8_t *te_base = tab + ((size_t)U.tab + ((DUAL && C.gid >= 4) ? 1 : 0)) * P.tab_nsb * kTabSB;
        const int sbB = qe_sb_bytes(U.type);
        const int rb = (int)U.rb;
        for (int sp = 0; sp < U.nsplit; sp++) {
            const int slot = ring.slot;
            const uint32_t phase = ring.phase;
            ring.next(P.stages);
            const bool mine = (g == grp);
            if (++g == P.G) g = 0;
            if (!mine) continue;
            if (!mbar_wait(&full[slot], phase, P.err, P.wait_cycles)) return;
            if (first && warp == 0 && lane == 0) QE_STAMP(3);
            first = false;
            const int s0 = sp * U.sbs, s1 = min(U.nsb, s0 + U.sbs), n = s1 - s0;
            const uint32_t pitch = qe_pitch((uint32_t)n * (uint32_t)sbB);
            // (cw*n)/cg exactly: the +0.5 keeps the float product away from
            // integers by 0.5/cg, far beyond its rounding error
            const int i0 = __float2int_rz(((float)(cw * n) + 0.5f) * inv_cg);
            const int i1 = __float2int_rz(((float)((cw + 1) * n) + 0.5f) * inv_cg);
            const uint8_t *st = stage0 + (size_t)slot * P.slot_bytes;
            const int off = s0 * sbB;
            // rows past the tile's end hold stale bytes: their results are
            // never read (rows are independent in the MMA)
            const uintptr_t a_lo = reinterpret_cast<uintptr_t>(U.lo + (C.gid * rb + off));
            const uintptr_t a_hi = reinterpret_cast<uintptr_t>(U.hi + (C.gid * rb + off));
            double yg = 0.0, yg8 = 0.0;
            const bool blk = qe_block_mode(U);
            const uint8_t *rg = blk ? st + (reinterpret_cast<uintptr_t>(U.lo) & 15) + C.gid * rb
                                    : st + C.gid * pitch + (a_lo & 15);
            const uint8_t *rg8 = blk ? st + qe_hi_off(rb) + (reinterpret_cast<uintptr_t>(U.hi) & 15) + C.gid * rb
                                     : st + (C.gid + 8) * pitch + (a_hi & 15);
            tile_sbs_rt<JobIq<Job>::v>(U.type, rg, rg8, te_base + (size_t)s0 * kTabSB, i0, i1, (int)(a_lo & 2) >> 1,
                                       C, yg, yg8, smem + P.iq_off, &P.iq);
            if constexpr (DUAL) {
                // lanes tig 0,1 hold the first vector's columns, tig 2,3 the second's
                yg += __shfl_xor_sync(0xffffffffu, yg, 1);
                yg8 += __shfl_xor_sync(0xffffffffu, yg8, 1);
                if ((C.tig & 1) == 0) {
                    double *rs = red + ((size_t)slot * P.cg + cw) * RW + (C.tig == 2 ? 16 : 0);
                    rs[C.gid] = yg;
                    rs[C.gid + 8] = yg8;
                }
            } else {
                quad_sum(yg, yg8);
                if (C.tig == 0) {
                    double *rs = red + ((size_t)slot * P.cg + cw) * RW;
                    rs[C.gid] = yg;
                    rs[C.gid + 8] = yg8;
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&ready[slot]);   // release: the partials above are visible to the reducer
        }
    }
    if (warp == 0 && lane == 0) QE_STAMP(4);
}

// Host: the largest row an item may carry whole, given the activation-table
// bytes the CTA keeps in shared memory: `stages` stages of 16 rows must fit.
inline uint32_t qe_row_budget(int64_t smem_optin, int64_t tab_bytes, int stages = 3) {
    const int64_t b = (smem_optin - kQeJobSmem - tab_bytes - 8192) / (stages * 16) - 48;
    return (uint32_t)std::max<int64_t>(512, std::min<int64_t>(stages >= 3 ? 4000 : 6000, b));
}
// Host: the row budget for rows of rb bytes: three stages, or two when that
// keeps rows of up to 4 KB whole (whole rows move as two bulk copies per
// item; split rows need one copy per row and slice, and the copy engine's
// per-request cost then dominates). Measured on Q4_K rows of 7168 columns
// (4032 B): 2495 -> 3717 GB/s at 65536 rows; rows of 4608 B measured
// slower with two stages.
inline uint32_t qe_row_budget_for(int64_t smem_optin, int64_t tab_bytes, int64_t rb) {
    const uint32_t b3 = qe_row_budget(smem_optin, tab_bytes, 3);
    if (rb <= (int64_t)b3 || rb > 4096) return b3;
    const uint32_t b2 = qe_row_budget(smem_optin, tab_bytes, 2);
    return rb <= (int64_t)b2 ? b2 : b3;
}

// Host: superblocks per split for a row of `nsb` superblocks of format t so
// that one row's item bytes stay within `row_budget`; 0 if impossible.
inline int qe_sbs(int t, int nsb, uint32_t row_budget, int &nsplit) {
    const int sb = qe_sb_bytes(t);
    int sbs = std::min(nsb, (int)(row_budget / (uint32_t)sb));
    if (sbs <= 0) return 0;
    nsplit = (nsb + sbs - 1) / sbs;
    sbs = (nsb + nsplit - 1) / nsplit;          // balanced splits (the last may be shorter)
    nsplit = (nsb + sbs - 1) / sbs;
    return sbs;
}

// Host: consumers per group (cg) for items of at most `maxn` superblocks,
// and groups G (items in flight), cg * G <= kQeMaxCons. Each consumer takes
// up to 4 superblocks of an item (fewer when that leaves warps idle): the
// per-item bookkeeping is then small against the superblocks' work.
inline void qe_groups(int maxn, int &cg, int &G) {
    for (int per = 4; per >= 1; per--) {
        cg = (maxn + per - 1) / per;
        if (cg > kQeMaxCons) { cg = kQeMaxCons; G = 1; return; }
        G = std::min(4, kQeMaxCons / cg);
        if (cg * G >= 12 || per == 1) return;
    }
}

// Host: the same for items whose rows have formats a and b. Long rows
// (>= 16 superblocks) get a format-tuned share per warp, measured on 65536 x
// 7168 matrices and the config-2 gate/up: the cheap Q2_K walk does best with
// 6 superblocks per warp and 3 groups (3430 -> 3721 GB/s; gate/up 28.7 ->
// 26.9 us), the costly Q3_K and IQ2_XS / IQ3_XXS walks with 2 superblocks
// per warp in one group of 14 (Q3_K 2586 -> 2807, IQ2_XS 1386 -> 1597
// GB/s). IQ2_XXS and IQ1_S measured 3-4 % slower that way and keep
// qe_groups' choice, as do short rows (the 8-superblock down projections).
inline void qe_groups_fmt(int maxn, int a, int b, int &cg, int &G) {
    auto heavy = [](int t) { return t == T_Q3_K || t == T_IQ2_XS || t == T_IQ3_XXS; };
    int per = 0;
    if (maxn >= 16) {
        if (heavy(a) || heavy(b)) per = 2;
        else if (a == T_Q2_K || b == T_Q2_K) per = 6;
    }
    if (!per) {
        qe_groups(maxn, cg, G);
        return;
    }
    cg = std::min(kQeMaxCons, (maxn + per - 1) / per);
    G = std::max(1, std::min(4, kQeMaxCons / cg));
}

// Host: shared-memory layout for a launch. item_bytes_max = the largest
// item's row bytes (one row); returns 0 if nothing fits.
inline int qe_layout(QeLayout &P, int G, int cg, uint32_t item_row_bytes_max, int n_tab, int tab_nsb,
                     int64_t smem_optin, int64_t &smem, const IqLayout *iq = nullptr, int red_w = 16) {
    const uint32_t iq_bytes = iq ? iq->bytes : 0u;
    if (iq) P.iq = *iq;
    P.G = G;
    P.cg = cg;
    P.n_tab = n_tab;
    P.tab_nsb = tab_nsb;
    P.slot_bytes = 16 * qe_pitch(item_row_bytes_max);
    smem_optin -= kQeJobSmem;          // the kernel's static shared memory
    P.stages = kQeMaxStages;
    for (;;) {
        P.red_off = ((3 * kQeMaxStages + 1) * 8 + 127) & ~127u;
        P.tab_off = P.red_off + ((P.stages * cg * red_w * 8 + 127) & ~127u);
        P.stage_off = P.tab_off + (((uint32_t)n_tab * tab_nsb * kTabSB + 127) & ~127u);
        P.iq_off = iq_bytes ? P.stage_off : 0u;
        P.stage_off += (iq_bytes + 127) & ~127u;
        smem = P.stage_off + (int64_t)P.stages * P.slot_bytes;
        if (smem <= smem_optin || P.stages <= 2) break;
        P.stages--;
    }
    // items in flight in the consumer groups, plus two being filled
    while (P.G > 1 && P.stages < P.G + 2) P.G--;
    return smem <= smem_optin;
}

}  // namespace sepia
