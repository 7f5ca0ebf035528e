// sepia_b200/csrc/attn.cu -- banded relative-position attention
// (ABI sepia_gpu_rel_project / sepia_gpu_banded_attn, src/sepia_gpu.h:
// 209-231; CPU oracle attn_forward_chunk, src/sepia.c:1195-1262; Metal twin
// metal/banded_attn.metal).
//
// Per query token t (position q_pos = q_pos_base + t) and head h:
//   s[kv] = dot(q[t,h], k[kv,hk]) * inv_head_dim
//           + (q_pos - kv < rel_extent ? rel_logits[t,h,q_pos-kv] * tau[t] : 0)
//   out[t,h] = softmax_kv(s) . v[kv,hk],  kv in [kv_lo[t], kv_hi[t]],
// with hk = h / (H/Hkv) (GQA) and q already scaled by tau by the caller.
//
// Decode at long context is a read of the whole K/V band, so the kernel is
// split-KV ("flash decoding"): grid (splits, Hkv, T); one CTA owns a chunk
// of kv positions of one KV head and ALL query heads of that GQA group, so
// each K/V row crosses HBM exactly once. Each CTA writes (m, l, acc[Dh])
// per head; k_attn_combine merges the splits in split order (deterministic).
// K/V may be fp32 (the reference cache) or fp16 (the decode configuration).
#include "../../include/sepia_cuda.h"
#include "runtime.h"
#include "common.cuh"

#include <cuda_fp16.h>
#include <algorithm>
#include <mutex>

namespace sepia {

constexpr int kAttnThreads = 256;
constexpr int kAttnWarps = kAttnThreads / 32;
constexpr int kAttnKT = 64;          // kv positions per tile
constexpr int kAttnMaxDh = 128;
constexpr int kAttnMaxG = 16;        // query heads per KV head
// K/V tile buffers per tensor: fp32 tiles single-buffered, so that two CTAs
// fit an SM (more warps hide the copy: decode 270 -> 273.5 tok/s); fp16
// tiles double-buffered (single measured 4 % slower at 32768 keys)
template <typename KV>
constexpr int attn_bufs() { return sizeof(KV) == 4 ? 1 : 2; }

struct AttnParams {
    const float *q;            // [T, H, Dh]
    const void *k, *v;         // [cap, kv_dim]
    const float *rel_logits;   // [T, H, E]
    const int64_t *kv_lo, *kv_hi;
    const float *tau;
    const double *tau64;       // tau in double (the reference's type); overrides tau when set
    const int32_t *qpos_dev;   // q_pos_base read on the device (decode graphs); overrides q_pos_base
    double *part;              // [T, H, S, Dh + 2]: m, l, acc[Dh] (fp64: no rounding before the combine)
    int64_t T, H, Hkv, Dh, E, q_pos_base, kv_dim;
    double inv_head_dim;       // 1.0/(double)Dh when the caller passed that value rounded to float
    int S;
    int64_t max_chunk;         // kv positions per split (upper bound)
};


template <typename KV>
__device__ __forceinline__ double kv_d(const KV *p);
template <>
__device__ __forceinline__ double kv_d<float>(const float *p) { return (double)*p; }
template <>
__device__ __forceinline__ double kv_d<__half>(const __half *p) { return (double)__half2float(*p); }

// Shared-memory row length (elements) of a staged K/V tile: 16-byte multiple.
template <typename KV>
__host__ __device__ constexpr int attn_ldk(int Dh) { return Dh + 16 / (int)sizeof(KV); }

// One CTA per (kv split, KV head, token). K/V tiles of kAttnKT rows are
// staged in their own type with 16-byte cp.async copies, double buffered
// (the next tile is in flight while this one is used); VEC = false stages
// element by element (rows not 16-byte aligned).
template <typename KV, bool VEC, int GM>
__global__ void __launch_bounds__(kAttnThreads, sizeof(KV) == 4 ? 3 : 2) k_attn_split(const AttnParams P) {
    extern __shared__ __align__(16) uint8_t smraw[];
    const int s = blockIdx.x, hk = blockIdx.y;
    const int64_t t = blockIdx.z;
    const int G = (int)(P.H / P.Hkv), Dh = (int)P.Dh;
    const int ldq = Dh + 2, ldk = attn_ldk<KV>(Dh);
    double *sq = reinterpret_cast<double *>(smraw);               // [G][ldq] (converted once)
    KV *skb = reinterpret_cast<KV *>(sq + G * ldq);              // [2][KT][ldk]
    constexpr int kAttnBufs = attn_bufs<KV>();
    KV *svb = skb + kAttnBufs * kAttnKT * ldk;                   // [bufs][KT][ldk]
    float *ss = reinterpret_cast<float *>(svb + kAttnBufs * kAttnKT * ldk);   // [G][KT]
    float *sml = ss + G * kAttnKT;                               // [G][2] running m, l

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    griddep_wait();
    griddep_launch();
    const int64_t lo = P.kv_lo[t], hi = P.kv_hi[t];
    const int64_t n = hi - lo + 1;
    const int64_t chunk = (n + P.S - 1) / P.S;
    const int64_t c0 = lo + (int64_t)s * chunk;
    const int64_t c1 = min(hi + 1, c0 + chunk);
    const int64_t q_pos = (P.qpos_dev ? (int64_t)*P.qpos_dev : P.q_pos_base) + t;
    const double tau = P.tau64 ? P.tau64[t] : (double)P.tau[t];
    const KV *K = reinterpret_cast<const KV *>(P.k);
    const KV *V = reinterpret_cast<const KV *>(P.v);

    for (int i = tid; i < G * Dh; i += kAttnThreads) {
        const int g = i / Dh, d = i - g * Dh;
        sq[g * ldq + d] = (double)P.q[(t * P.H + (int64_t)hk * G + g) * P.Dh + d];
    }
    if (tid < G) { sml[2 * tid] = -INFINITY; sml[2 * tid + 1] = 0.0f; }

    // stage rows [base, base+nt) of this KV head into buffer b
    const int gpr = Dh * (int)sizeof(KV) / 16;                     // 16-byte granules per row
    auto stage = [&](int64_t base, int nt, int b) {
        KV *sk = skb + b * kAttnKT * ldk, *sv = svb + b * kAttnKT * ldk;
        if constexpr (VEC) {
            for (int i = tid; i < nt * gpr; i += kAttnThreads) {
                const int r = i / gpr, c = i - r * gpr;
                const int64_t off = (base + r) * P.kv_dim + (int64_t)hk * Dh;
                cp_async16(reinterpret_cast<uint8_t *>(sk + r * ldk) + 16 * c,
                           reinterpret_cast<const uint8_t *>(K + off) + 16 * c);
                cp_async16(reinterpret_cast<uint8_t *>(sv + r * ldk) + 16 * c,
                           reinterpret_cast<const uint8_t *>(V + off) + 16 * c);
            }
            cp_async_commit();
        } else {
            for (int i = tid; i < nt * Dh; i += kAttnThreads) {
                const int r = i / Dh, d = i - r * Dh;
                const int64_t off = (base + r) * P.kv_dim + (int64_t)hk * Dh + d;
                sk[r * ldk + d] = K[off];
                sv[r * ldk + d] = V[off];
            }
        }
    };

    // PV ownership: warp w owns heads g = w, w+8, ...; lane owns dims lane + 32j
    constexpr int kHPW = (GM + kAttnWarps - 1) / kAttnWarps;   // heads per warp (GM >= G)
    constexpr int kHPT = (GM + (kAttnThreads / kAttnKT) - 1) / (kAttnThreads / kAttnKT);   // score heads per thread
    double acc[kHPW][kAttnMaxDh / 32];   // fp64, as the reference accumulates
    double acc_b[kHPW][kAttnMaxDh / 32]; // VEC: the odd rows' accumulators
#pragma unroll
    for (int a = 0; a < kHPW; a++)
#pragma unroll
        for (int j = 0; j < kAttnMaxDh / 32; j++) acc[a][j] = acc_b[a][j] = 0.0;

    if (kAttnBufs == 2 && c0 < c1) stage(c0, (int)min((int64_t)kAttnKT, c1 - c0), 0);
    int buf = 0;
    for (int64_t base = c0; base < c1; base += kAttnKT, buf ^= (kAttnBufs - 1)) {
        const int nt = (c1 - base < kAttnKT) ? (int)(c1 - base) : kAttnKT;
        const int64_t nb = base + kAttnKT;
        if constexpr (kAttnBufs == 1) {
            // one buffer per tensor (more CTAs per SM hide the copy instead)
            stage(base, nt, 0);
            if constexpr (VEC) cp_async_wait<0>();
        } else if constexpr (VEC) {
            if (nb < c1) {
                stage(nb, (int)min((int64_t)kAttnKT, c1 - nb), buf ^ 1);
                cp_async_wait<1>();
            } else {
                cp_async_wait<0>();
            }
        } else {
            if (base != c0) stage(base, nt, buf);
        }
        __syncthreads();
        const KV *sk = skb + buf * kAttnKT * ldk, *sv = svb + buf * kAttnKT * ldk;
        // ---- scores: thread -> kv row r, heads g0, g0+gstep, ... ----
        {
            const int r = tid % kAttnKT;
            const int g0 = tid / kAttnKT;
            const int gstep = kAttnThreads / kAttnKT;
            if (r < nt) {
                const int64_t kv = base + r;
                const int64_t dist = q_pos - kv;
                // the reference's score arithmetic (src/sepia.c:1216-1220):
                // fp64 dot rounded to float, then content + bias in fp64,
                // rounded once -- a one-ulp score change moves exp() by
                // ~1e-6 relative, more than the whole error budget. Each k
                // element is converted once for all of the thread's heads.
                double dd[kHPT];
#pragma unroll
                for (int j = 0; j < kHPT; j++) dd[j] = 0.0;
                const KV *kr = sk + r * ldk;
                if constexpr (VEC) {
                    // one 16-byte shared load per granule: rows sit 16 bytes
                    // past a multiple of 128, so 8 consecutive rows (one
                    // quarter-warp phase) cover all 32 banks without conflict.
                    // Each dot runs as 4 interleaved fp64 partial sums
                    // (element pairs 2c, 2c+1 of every 8 go to chain c),
                    // added pairwise at the end: 4x shorter dependent FMA
                    // chains; the fp64 result moves by ~1e-16 relative,
                    // far inside the float rounding that follows.
                    constexpr int EPG = 16 / (int)sizeof(KV);
                    double dc[kHPT][4];
#pragma unroll
                    for (int j = 0; j < kHPT; j++)
#pragma unroll
                        for (int c = 0; c < 4; c++) dc[j][c] = 0.0;
                    for (int d0 = 0; d0 < Dh; d0 += EPG) {
                        const uint4 raw = *reinterpret_cast<const uint4 *>(kr + d0);
                        double kd[EPG];
                        if constexpr (sizeof(KV) == 2) {
                            const __half2 *h2 = reinterpret_cast<const __half2 *>(&raw);
#pragma unroll
                            for (int e = 0; e < 4; e++) {
                                const float2 f = __half22float2(h2[e]);
                                kd[2 * e] = (double)f.x;
                                kd[2 * e + 1] = (double)f.y;
                            }
                        } else {
                            const float *f4 = reinterpret_cast<const float *>(&raw);
#pragma unroll
                            for (int e = 0; e < EPG; e++) kd[e] = (double)f4[e];
                        }
#pragma unroll
                        for (int j = 0; j < kHPT; j++) {
                            const int g = g0 + gstep * j;
                            if (g < G) {
                                const double *qg = sq + g * ldq + d0;
#pragma unroll
                                for (int e = 0; e < EPG; e += 2) {
                                    const double2 q2 = *reinterpret_cast<const double2 *>(qg + e);
                                    double &a = dc[j][(e >> 1) & 3];
                                    a = fma(q2.x, kd[e], a);
                                    a = fma(q2.y, kd[e + 1], a);
                                }
                            }
                        }
                    }
#pragma unroll
                    for (int j = 0; j < kHPT; j++) dd[j] = (dc[j][0] + dc[j][1]) + (dc[j][2] + dc[j][3]);
                } else {
                    for (int d = 0; d < Dh; d++) {
                        const double kd = kv_d<KV>(kr + d);
#pragma unroll
                        for (int j = 0; j < kHPT; j++) {
                            const int g = g0 + gstep * j;
                            if (g < G) dd[j] = fma(sq[g * ldq + d], kd, dd[j]);
                        }
                    }
                }
#pragma unroll
                for (int j = 0; j < kHPT; j++) {
                    const int g = g0 + gstep * j;
                    if (g < G) {
                        double sc = (double)(float)dd[j] * P.inv_head_dim;
                        if (dist < P.E && dist >= 0)
                            sc += (double)P.rel_logits[(t * P.H + (int64_t)hk * G + g) * P.E + dist] * tau;
                        ss[g * kAttnKT + r] = (float)sc;
                    }
                }
            } else {
                for (int g = g0; g < G; g += gstep) ss[g * kAttnKT + r] = -INFINITY;
            }
        }
        __syncthreads();
        // ---- online softmax update, per head owned by this warp ----
#pragma unroll
        for (int a = 0; a < kHPW; a++) {
            const int g = warp + kAttnWarps * a;
            if (g < G) {
                const float v0 = ss[g * kAttnKT + lane], v1 = ss[g * kAttnKT + lane + 32];
                const float tmax = warp_max(fmaxf(v0, v1));
                const float m_old = sml[2 * g];
                const float m_new = fmaxf(m_old, tmax);
                const float corr = (m_old == -INFINITY) ? 0.0f : (float)exp((double)(m_old - m_new));
                const float p0 = (v0 == -INFINITY) ? 0.0f : (float)exp((double)(v0 - m_new));
                const float p1 = (v1 == -INFINITY) ? 0.0f : (float)exp((double)(v1 - m_new));
                ss[g * kAttnKT + lane] = p0;
                ss[g * kAttnKT + lane + 32] = p1;
                const float psum = warp_sum(p0 + p1);
                __syncwarp();
                if (lane == 0) { sml[2 * g] = m_new; sml[2 * g + 1] = sml[2 * g + 1] * corr + psum; }
#pragma unroll
                for (int j = 0; j < kAttnMaxDh / 32; j++) {
                    acc[a][j] *= (double)corr;
                    acc_b[a][j] *= (double)corr;
                }
            }
        }
        __syncwarp();
        // ---- P.V: each v element is converted once for all of the warp's heads ----
        // Products accumulate in fp64 as in the reference (src/sepia.c:1247-
        // 1252): an fp32 running sum over a tile loses ~1e-7 of its
        // magnitude per tile, which at 32k keys puts outputs near zero past
        // the 1e-4 bar. VEC: even and odd rows go to two accumulator sets
        // (twice the independent fp64 chains), added when the split ends.
        for (int r = 0; r < nt; r++) {
            double pr[kHPW];
#pragma unroll
            for (int a = 0; a < kHPW; a++) {
                const int g = warp + kAttnWarps * a;
                pr[a] = (g < G) ? (double)ss[g * kAttnKT + r] : 0.0;
            }
            if constexpr (VEC) {
                // lane owns dims 4*lane .. 4*lane+3: one 8- or 16-byte load
                if (4 * lane < Dh) {
                    double vd[4];
                    if constexpr (sizeof(KV) == 2) {
                        const uint2 raw = *reinterpret_cast<const uint2 *>(sv + r * ldk + 4 * lane);
                        const float2 f0 = __half22float2(*reinterpret_cast<const __half2 *>(&raw.x));
                        const float2 f1 = __half22float2(*reinterpret_cast<const __half2 *>(&raw.y));
                        vd[0] = f0.x; vd[1] = f0.y; vd[2] = f1.x; vd[3] = f1.y;
                    } else {
                        const float4 f = *reinterpret_cast<const float4 *>(sv + r * ldk + 4 * lane);
                        vd[0] = f.x; vd[1] = f.y; vd[2] = f.z; vd[3] = f.w;
                    }
                    if (r & 1) {
#pragma unroll
                        for (int jj = 0; jj < 4; jj++)
#pragma unroll
                            for (int a = 0; a < kHPW; a++) acc_b[a][jj] = fma(pr[a], vd[jj], acc_b[a][jj]);
                    } else {
#pragma unroll
                        for (int jj = 0; jj < 4; jj++)
#pragma unroll
                            for (int a = 0; a < kHPW; a++) acc[a][jj] = fma(pr[a], vd[jj], acc[a][jj]);
                    }
                }
            } else {
#pragma unroll
                for (int jj = 0; jj < kAttnMaxDh / 32; jj++) {
                    const int d = lane + 32 * jj;
                    if (d < Dh) {
                        const double vdd = kv_d<KV>(sv + r * ldk + d);
#pragma unroll
                        for (int a = 0; a < kHPW; a++)
                            if (warp + kAttnWarps * a < G) acc[a][jj] = fma(pr[a], vdd, acc[a][jj]);
                    }
                }
            }
        }
        __syncthreads();
    }
    // ---- write this split's partial per head ----
#pragma unroll
    for (int a = 0; a < kHPW; a++) {
        const int g = warp + kAttnWarps * a;
        if (g < G) {
            const int64_t h = (int64_t)hk * G + g;
            double *pp = P.part + ((t * P.H + h) * P.S + s) * (P.Dh + 2);
            if (lane == 0) { pp[0] = sml[2 * g]; pp[1] = sml[2 * g + 1]; }
#pragma unroll
            for (int j = 0; j < kAttnMaxDh / 32; j++) {
                const int d = VEC ? 4 * lane + j : lane + 32 * j;
                if (d < Dh) pp[2 + d] = acc[a][j] + acc_b[a][j];
            }
        }
    }
}

template <typename KV>
static size_t attn_smem(int G, int Dh) {
    return sizeof(double) * (size_t)G * (Dh + 2) + sizeof(KV) * 2 * attn_bufs<KV>() * (size_t)kAttnKT * attn_ldk<KV>(Dh) +
           sizeof(float) * ((size_t)G * kAttnKT + 2 * G);
}

template <typename KV, bool VEC, int GM>
static int attn_launch_g(const AttnParams &P, size_t smem, cudaStream_t st) {
    const void *fn = (const void *)k_attn_split<KV, VEC, GM>;
    if (!ensure_smem(fn, (int)smem)) return 0;
    dim3 grid((unsigned)P.S, (unsigned)P.Hkv, (unsigned)P.T);
    return check(launch_pdl(k_attn_split<KV, VEC, GM>, grid, dim3(kAttnThreads), smem, st, P), "banded_attn launch");
}

template <typename KV, bool VEC>
static int attn_launch_v(const AttnParams &P, int G, size_t smem, cudaStream_t st) {
    if (G <= 2) return attn_launch_g<KV, VEC, 2>(P, smem, st);
    if (G <= 4) return attn_launch_g<KV, VEC, 4>(P, smem, st);
    if (G <= 8) return attn_launch_g<KV, VEC, 8>(P, smem, st);
    return attn_launch_g<KV, VEC, kAttnMaxG>(P, smem, st);
}

template <typename KV>
static int attn_launch_split(const AttnParams &P, int G, cudaStream_t st) {
    const int Dh = (int)P.Dh;
    const size_t smem = attn_smem<KV>(G, Dh);
    const bool vec = (Dh * (int)sizeof(KV)) % 16 == 0 && (P.kv_dim * (int64_t)sizeof(KV)) % 16 == 0 &&
                     ((reinterpret_cast<uintptr_t>(P.k) | reinterpret_cast<uintptr_t>(P.v)) & 15) == 0;
    return vec ? attn_launch_v<KV, true>(P, G, smem, st) : attn_launch_v<KV, false>(P, G, smem, st);
}

// out[t,h,:] = sum_s acc_s e^(m_s - M) / sum_s l_s e^(m_s - M), splits in order.
// The split weights e^(m_s - M) are computed once per (t, h) into shared memory.
constexpr int kAttnMaxSplits = 256;
__global__ void k_attn_combine(const double *part, float *out, int64_t TH, int S, int64_t Dh) {
    const int64_t th = blockIdx.x;
    griddep_wait();
    griddep_launch();
    if (th >= TH) return;
    __shared__ double s_w[kAttnMaxSplits];
    __shared__ double s_M, s_L;
    const double *pp = part + th * S * (Dh + 2);
    const int lane = threadIdx.x & 31;
    // M and L by warp 0: lane-strided loads, then a fixed shuffle tree
    // (deterministic; L's fp64 order differs from a serial sum by ~1e-16)
    if (threadIdx.x < 32) {
        double M = -INFINITY;
        for (int s = lane; s < S; s += 32) M = fmax(M, pp[s * (Dh + 2)]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) M = fmax(M, __shfl_xor_sync(0xffffffffu, M, o));
        if (lane == 0) s_M = M;
    }
    __syncthreads();
    const double M = s_M;
    for (int s = threadIdx.x; s < S; s += blockDim.x) {
        const double m = pp[s * (Dh + 2)];
        s_w[s] = (m != -INFINITY) ? exp(m - M) : 0.0;
    }
    __syncthreads();
    if (threadIdx.x < 32) {
        double L = 0.0;
        for (int s = lane; s < S; s += 32) L += pp[s * (Dh + 2) + 1] * s_w[s];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
        if (lane == 0) s_L = L;
    }
    __syncthreads();
    const double L = s_L;
    for (int64_t d = threadIdx.x; d < Dh; d += blockDim.x) {
        double a = 0.0;
        for (int s = 0; s < S; s++) a += pp[s * (Dh + 2) + 2 + d] * s_w[s];
        out[th * Dh + d] = (float)(a / L);
    }
}

// rel_logits[t,h,r] = sum_d r_vec[t,h,d] * rel_proj[d,r] (double accumulation)
__global__ void k_rel_project(const float *r_vec, const float *rel_proj, float *rel_logits, int64_t TH,
                              int64_t d_rel, int64_t E) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    griddep_wait();
    griddep_launch();
    if (i >= TH * E) return;
    const int64_t th = i / E, r = i % E;
    const float *rv = r_vec + th * d_rel;
    double acc = 0.0;
    for (int64_t d = 0; d < d_rel; d++) acc = fma((double)rv[d], (double)rel_proj[d * E + r], acc);
    rel_logits[i] = (float)acc;
}

int attn_splits(int64_t T, int64_t Hkv, int64_t max_n) {
    const int sms = dev_info().sm_count > 0 ? dev_info().sm_count : 148;
    int64_t want = (4 * (int64_t)sms + T * Hkv - 1) / (T * Hkv);
    const int64_t by_len = (max_n + kAttnKT - 1) / kAttnKT;   // at least one tile per split
    want = std::max<int64_t>(1, std::min<int64_t>(want, by_len));
    return (int)std::min<int64_t>(want, 256);
}

size_t attn_part_bytes(int64_t T, int64_t H, int S, int64_t Dh) {
    return (size_t)T * (size_t)H * (size_t)S * (size_t)(Dh + 2) * sizeof(double);
}

int launch_banded_attn_ex(int kv_f16, const float *q, const void *k, const void *v, const float *rel_logits,
                          float *out, const int64_t *kv_lo_d, const int64_t *kv_hi_d, const float *tau_d,
                          const double *tau64_d, const int32_t *qpos_d, int64_t T, int64_t H, int64_t Hkv,
                          int64_t Dh, int64_t E, int64_t q_pos_base, int64_t kv_dim, float inv_head_dim, int S,
                          double *part, cudaStream_t st);

int launch_banded_attn(int kv_f16, const float *q, const void *k, const void *v, const float *rel_logits, float *out,
                       const int64_t *kv_lo_d, const int64_t *kv_hi_d, const float *tau_d, int64_t T, int64_t H,
                       int64_t Hkv, int64_t Dh, int64_t E, int64_t q_pos_base, int64_t kv_dim, float inv_head_dim,
                       int S, double *part, cudaStream_t st) {
    return launch_banded_attn_ex(kv_f16, q, k, v, rel_logits, out, kv_lo_d, kv_hi_d, tau_d, nullptr, nullptr, T, H,
                                 Hkv, Dh, E, q_pos_base, kv_dim, inv_head_dim, S, part, st);
}

// tau64_d / qpos_d (either may be null): tau in double and the position of
// token 0 read on the device, for decode steps replayed from a CUDA graph.
int launch_banded_attn_ex(int kv_f16, const float *q, const void *k, const void *v, const float *rel_logits,
                          float *out, const int64_t *kv_lo_d, const int64_t *kv_hi_d, const float *tau_d,
                          const double *tau64_d, const int32_t *qpos_d, int64_t T, int64_t H, int64_t Hkv,
                          int64_t Dh, int64_t E, int64_t q_pos_base, int64_t kv_dim, float inv_head_dim, int S,
                          double *part, cudaStream_t st) {
    if (T <= 0 || H <= 0 || Hkv <= 0 || H % Hkv || Dh <= 0 || E < 0 || kv_dim < Hkv * Dh)
        return fail("banded_attn: bad geometry T=%lld H=%lld Hkv=%lld Dh=%lld E=%lld kv_dim=%lld", (long long)T,
                    (long long)H, (long long)Hkv, (long long)Dh, (long long)E, (long long)kv_dim);
    if (Dh > kAttnMaxDh) return fail("banded_attn: Dh=%lld exceeds %d", (long long)Dh, kAttnMaxDh);
    if (H / Hkv > kAttnMaxG) return fail("banded_attn: %lld query heads per KV head exceeds %d", (long long)(H / Hkv), kAttnMaxG);
    if (!q || !k || !v || !out || !kv_lo_d || !kv_hi_d || (!tau_d && !tau64_d) || !part || (E > 0 && !rel_logits))
        return fail("banded_attn: null pointer");
    if (S < 1) return fail("banded_attn: bad split count");
    AttnParams P;
    P.q = q; P.k = k; P.v = v; P.rel_logits = rel_logits; P.kv_lo = kv_lo_d; P.kv_hi = kv_hi_d; P.tau = tau_d;
    P.tau64 = tau64_d; P.qpos_dev = qpos_d;
    P.part = part; P.T = T; P.H = H; P.Hkv = Hkv; P.Dh = Dh; P.E = E; P.q_pos_base = q_pos_base; P.kv_dim = kv_dim;
    // The reference scales by 1.0/(double)Dh (src/sepia.c:1217); the ABI
    // carries a float, so a float equal to that value rounded stands for it.
    const double inv_exact = 1.0 / (double)Dh;
    P.inv_head_dim = ((float)inv_exact == inv_head_dim) ? inv_exact : (double)inv_head_dim;
    P.S = S; P.max_chunk = 0;
    const int G = (int)(H / Hkv);
    if (!(kv_f16 ? attn_launch_split<__half>(P, G, st) : attn_launch_split<float>(P, G, st))) return 0;
    if (!check(launch_pdl(k_attn_combine, (unsigned)(T * H), 128, 0, st, (const double *)part, out, T * H, S, Dh),
               "banded_attn combine launch"))
        return 0;
    return check(cudaGetLastError(), "banded_attn combine launch");
}

int launch_rel_project(const float *r_vec, const float *rel_proj, float *rel_logits, int64_t T, int64_t H,
                       int64_t d_rel, int64_t E, cudaStream_t st) {
    if (T <= 0 || H <= 0 || d_rel <= 0 || E <= 0 || !r_vec || !rel_proj || !rel_logits)
        return fail("rel_project: bad arguments");
    const int64_t n = T * H * E;
    if (!check(launch_pdl(k_rel_project, (unsigned)((n + 255) / 256), 256, 0, st, r_vec, rel_proj, rel_logits, T * H,
                          d_rel, E), "rel_project launch"))
        return 0;
    return check(cudaGetLastError(), "rel_project launch");
}

}  // namespace sepia

using namespace sepia;

extern "C" size_t sepia_cuda_banded_attn_ws_bytes(int64_t T, int64_t H, int64_t Hkv, int64_t Dh, int64_t max_kv) {
    if (T <= 0 || H <= 0 || Hkv <= 0 || Dh <= 0) return 0;
    return attn_part_bytes(T, H, attn_splits(T, Hkv, max_kv), Dh);
}

extern "C" int sepia_cuda_banded_attn(int kv_f16, const float *q, const void *k, const void *v, const float *rel_logits,
                                      float *out, const int64_t *kv_lo, const int64_t *kv_hi, const float *tau,
                                      int64_t T, int64_t H, int64_t Hkv, int64_t Dh, int64_t rel_extent,
                                      int64_t q_pos_base, int64_t kv_dim, float inv_head_dim, int64_t max_kv,
                                      void *ws, size_t ws_bytes, void *stream) {
    const int S = attn_splits(T, Hkv, max_kv > 0 ? max_kv : 1);
    if (!ws || ws_bytes < attn_part_bytes(T, H, S, Dh))
        return fail("banded_attn: workspace of %zu bytes < %zu needed", ws_bytes, attn_part_bytes(T, H, S, Dh));
    return launch_banded_attn(kv_f16, q, k, v, rel_logits, out, kv_lo, kv_hi, tau, T, H, Hkv, Dh, rel_extent,
                              q_pos_base, kv_dim, inv_head_dim, S, (double *)ws, as_stream(stream));
}

// ------------------------------------------------ allocation-free variant
// Some callers cannot allocate device memory at all: hosts whose device heap
// is owned by another allocator that reserved it up front, plugin hosts that
// only hand the library their own input/output buffers, and latency-critical
// loops that must not call cudaMalloc/cudaFree because those can synchronize
// the whole device. For them the split partials live in a fixed array
// compiled into the library instead of a caller workspace.
//
// The first call on each device looks up the array's device address (one
// cudaGetDevice + cudaGetSymbolAddress, with that device current); make that
// first call before any stream capture begins. The array is a module global, so every GPU that loads the
// library holds its kNoAllocScratchBytes from module load until the process
// exits.
//
// Nothing in it must start at zero: every (token, head, split) record is
// fully written by k_attn_split before k_attn_combine reads it. All calls on
// one device share the one array, so two calls whose kernels overlap on the
// GPU (different streams with no ordering between them) race and corrupt
// each other's result; calls on one stream are ordered and safe.
constexpr size_t kNoAllocScratchBytes = (size_t)8 << 20;   // 8 MiB of fp64 partials
constexpr int kNoAllocMaxDevices = 64;

static __device__ __align__(256) double g_attn_noalloc_part[kNoAllocScratchBytes / sizeof(double)];

// Device address of g_attn_noalloc_part on the current device. In host code
// the symbol is only a host-side handle, never a device address, so the
// address is looked up once per device (with that device current) through
// cudaGetSymbolAddress and cached.
static double *noalloc_part_ptr() {
    static std::mutex mu;
    static double *ptrs[kNoAllocMaxDevices] = {};
    int dev = -1;
    if (!check(cudaGetDevice(&dev), "banded_attn_noalloc: cudaGetDevice")) return nullptr;
    if (dev < 0 || dev >= kNoAllocMaxDevices) {
        fail("banded_attn_noalloc: device %d out of range (max %d)", dev, kNoAllocMaxDevices);
        return nullptr;
    }
    std::lock_guard<std::mutex> lock(mu);
    if (!ptrs[dev]) {
        void *p = nullptr;
        if (!check(cudaGetSymbolAddress(&p, g_attn_noalloc_part), "banded_attn_noalloc: cudaGetSymbolAddress"))
            return nullptr;
        ptrs[dev] = (double *)p;
    }
    return ptrs[dev];
}

extern "C" size_t sepia_cuda_banded_attn_noalloc_max_bytes(void) { return kNoAllocScratchBytes; }

extern "C" int sepia_cuda_banded_attn_noalloc(int kv_f16, const float *q, const void *k, const void *v,
                                              const float *rel_logits, float *out, const int64_t *kv_lo,
                                              const int64_t *kv_hi, const float *tau, int64_t T, int64_t H,
                                              int64_t Hkv, int64_t Dh, int64_t rel_extent, int64_t q_pos_base,
                                              int64_t kv_dim, float inv_head_dim, int64_t max_kv, void *stream) {
    if (T <= 0 || H <= 0 || Hkv <= 0 || Dh <= 0)
        return fail("banded_attn_noalloc: bad geometry T=%lld H=%lld Hkv=%lld Dh=%lld", (long long)T, (long long)H,
                    (long long)Hkv, (long long)Dh);
    const int S = attn_splits(T, Hkv, max_kv > 0 ? max_kv : 1);
    const size_t need = attn_part_bytes(T, H, S, Dh);
    if (need > kNoAllocScratchBytes)
        return fail("banded_attn_noalloc: T=%lld H=%lld Dh=%lld needs %zu bytes of partials, above the fixed "
                    "%zu-byte scratch; use sepia_cuda_banded_attn with a caller workspace",
                    (long long)T, (long long)H, (long long)Dh, need, kNoAllocScratchBytes);
    double *part = noalloc_part_ptr();
    if (!part) return 0;
    return launch_banded_attn(kv_f16, q, k, v, rel_logits, out, kv_lo, kv_hi, tau, T, H, Hkv, Dh, rel_extent,
                              q_pos_base, kv_dim, inv_head_dim, S, part, as_stream(stream));
}

extern "C" int sepia_cuda_rel_project(const float *r_vec, const float *rel_proj, float *rel_logits, int64_t T,
                                      int64_t H, int64_t d_rel, int64_t rel_extent, void *stream) {
    return launch_rel_project(r_vec, rel_proj, rel_logits, T, H, d_rel, rel_extent, as_stream(stream));
}
