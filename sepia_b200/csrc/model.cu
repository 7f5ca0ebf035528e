// sepia_b200/csrc/model.cu -- the whole-token decode engine (include/sepia_model.h).
//
// A token's path on the device, per decoder layer (decoder_layer_forward,
// src/sepia.c:1483-1552; attention attn_forward_chunk, src/sepia.c:1077-1276):
//   xn -> q,k,v,r projections (matvec_q, four launches)
//      -> k_attn_prep: K/V short convolutions with history roll, per-head
//         RMSNorm of q and k, cache write, q scaled by tau, the kv range
//         and the relative-position band (rel_project)
//      -> split-KV banded attention -> wo projection
//      -> k_residual: attention-output short convolution + residual, then
//         the MLP norm of the new residual stream (one CTA)
//      -> MoE layer (router, top-k, experts; moe.cu) or dense SwiGLU
//      -> k_residual: MLP-output short convolution + residual, then the next
//         layer's attention norm (or the final norm / mup for the head)
// then the logits head (matvec_q over the unpadded rows) and k_argmax, whose
// 64-bit (value, index) key feeds the next step's k_embed. Token ids,
// positions and the argmax live in device memory, so a decode step needs no
// host value and is replayed from one CUDA graph.
#include "../../include/sepia_model.h"
#include "runtime.h"
#include "common.cuh"
#include "quant_formats.cuh"

#include <cooperative_groups.h>
#include <cmath>
#include <cstring>
#include <vector>

namespace cg = cooperative_groups;

namespace sepia {

int launch_matvec_q(int t, const void *w, const float *x, float *y, int64_t out_dim, int64_t in_dim, int64_t n_vec,
                    cudaStream_t st);
int launch_matvec_q_multi(int n, int t, const void *const *w, const int64_t *rows, int64_t in_dim, const float *x,
                          float *const *y, cudaStream_t st);
int launch_banded_attn_ex(int kv_f16, const float *q, const void *k, const void *v, const float *rel_logits,
                          float *out, const int64_t *kv_lo_d, const int64_t *kv_hi_d, const float *tau_d,
                          const double *tau64_d, const int32_t *qpos_d, int64_t T, int64_t H, int64_t Hkv,
                          int64_t Dh, int64_t E, int64_t q_pos_base, int64_t kv_dim, float inv_head_dim, int S,
                          double *part, cudaStream_t st);
int attn_splits(int64_t T, int64_t Hkv, int64_t max_n);
size_t attn_part_bytes(int64_t T, int64_t H, int S, int64_t Dh);
int op_silu_mul(const float *g, const float *u, float *z, int64_t n, cudaStream_t st);

constexpr int kMaxConvK = 16;

// Device-resident decode state.
struct ModelState {
    unsigned long long best;   // argmax key of the last logits (0: none)
    int32_t pos;               // position of the next token
    int32_t fed;               // teacher-forced tokens consumed by the current prefill
    int32_t gen;               // generated tokens written by decode steps
    int32_t bad_token;         // set when an input token id is out of range
    int64_t kv_lo, kv_hi;      // attention range of the current token (this layer)
    double tau;                // tau of the current token (this layer)
};

// ------------------------------------------------------------ reductions
__device__ double block_sum_d2(double v, double *sh) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
    v = warp_sum_d(v);
    if (lane == 0) sh[warp] = v;
    __syncthreads();
    if (warp == 0) {
        double t = lane < nw ? sh[lane] : 0.0;
        t = warp_sum_d(t);
        if (lane == 0) sh[32] = t;
    }
    __syncthreads();
    const double r = sh[32];
    __syncthreads();
    return r;
}

// RMSNorm scale of n values spread over the block (src/sepia.c:720-729):
// squares rounded to float, summed in double, mean rounded to float,
// 1/sqrtf(var + eps).
__device__ float rms_inv(const float *v, int64_t n, float eps, double *sh) {
    double acc = 0.0;
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) acc += (double)__fmul_rn(v[i], v[i]);
    acc = block_sum_d2(acc, sh);
    const float var = (float)(acc / (double)n);
    return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
}

// The residual stream's kernels run as one cluster of kClusterCtas CTAs
// (each owns hidden/kClusterCtas channels); a norm's sum of squares is a
// block reduction per CTA, then every CTA adds the partials of the whole
// cluster through distributed shared memory in rank order (deterministic).
constexpr int kClusterCtas = 8;
constexpr int kClThreads = 1024;

__device__ double cluster_sum_d(double v, double *sh, double *part) {
    cg::cluster_group cl = cg::this_cluster();
    v = block_sum_d2(v, sh);
    if (threadIdx.x == 0) part[0] = v;
    cl.sync();
    double t = 0.0;
    for (unsigned r = 0; r < cl.num_blocks(); r++) t += *cl.map_shared_rank(part, r);
    cl.sync();       // no CTA leaves (or reuses part) while another still reads it
    return t;
}

__device__ __forceinline__ float rms_inv_from(double sumsq, int64_t n, float eps) {
    const float var = (float)(sumsq / (double)n);
    return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
}

// ------------------------------------------------------------ embedding
struct EmbedArgs {
    int type;
    const uint8_t *w;           // token_embd.weight
    int64_t rb, hidden;
    int32_t vocab;
    const int32_t *ids;         // teacher-forced ids (mode 0)
    int mode;                   // 0: ids[st->fed]; 1: the pending argmax
    int32_t *out_ids;           // mode 1: where the consumed token goes
    ModelState *st;
    const float *embed_norm, *norm0;
    float eps;
    float *x, *xn;              // residual stream, normed input of layer 0
    int *err;
};

// Token id -> dequantized row (qrow, src/sepia.c:742-746) -> rmsnorm with
// embed_norm = x (src/sepia.c:3352-3355) -> rmsnorm with layer 0's
// attention norm = xn. One cluster; CTA rank r owns a contiguous run of
// 32-element parts. Every CTA reads the pending token before rank 0
// updates the decode state.
__global__ void __launch_bounds__(kClThreads) k_embed(const EmbedArgs A) {
    cg::cluster_group cl = cg::this_cluster();
    __shared__ double sh[33];
    __shared__ double part;
    __shared__ int tok_sh;
    __shared__ float e_sm[32 * 32];
    griddep_wait();
    griddep_launch();
    const unsigned rank = cl.block_rank(), nr = cl.num_blocks();
    if (threadIdx.x == 0) {
        const ModelState *st = A.st;
        int tok = A.mode == 0 ? A.ids[st->fed] : (int)(0xFFFFFFFFu - (uint32_t)(st->best & 0xFFFFFFFFull));
        tok_sh = tok;
    }
    cl.sync();
    int tok = tok_sh;
    if (rank == 0 && threadIdx.x == 0) {
        ModelState *st = A.st;
        if (A.mode == 0) {
            st->fed += 1;
        } else {
            A.out_ids[st->gen] = tok;
            st->gen += 1;
        }
        st->best = 0ull;
        if (tok < 0 || tok >= A.vocab) {
            st->bad_token = 1;
            set_error(A.err, kErrBadArgs);
        }
    }
    if (tok < 0 || tok >= A.vocab) tok = 0;
    const int64_t nparts = (A.hidden + 31) / 32;
    const int64_t pp = (nparts + nr - 1) / nr;             // parts per CTA (<= 32)
    const int64_t p0 = rank * pp, p1 = imin64(nparts, p0 + pp);
    const int64_t e0 = p0 * 32, e1 = imin64(A.hidden, p1 * 32);
    const uint8_t *row = A.w + (int64_t)tok * A.rb;
    const int sbB = fmt_sb_bytes(A.type);
    if (threadIdx.x < p1 - p0) {
        const int64_t first = (p0 + threadIdx.x) * 32;
        float y[32];
        const int nvalid = (int)imin64(32, A.hidden - first);
        decode_part_exact(A.type, row + (first / kQK) * sbB, (int)((first % kQK) / 32), y, nvalid);
        for (int i = 0; i < nvalid; i++) e_sm[first - e0 + i] = y[i];
    }
    __syncthreads();
    const int64_t c = e0 + threadIdx.x;
    const bool mine = c < e1;
    const float ev = mine ? e_sm[threadIdx.x] : 0.0f;
    const float inv = rms_inv_from(cluster_sum_d(mine ? (double)__fmul_rn(ev, ev) : 0.0, sh, &part), A.hidden, A.eps);
    const float xv = mine ? __fmul_rn(A.embed_norm[c], __fmul_rn(ev, inv)) : 0.0f;
    if (mine) A.x[c] = xv;
    const float inv2 = rms_inv_from(cluster_sum_d(mine ? (double)__fmul_rn(xv, xv) : 0.0, sh, &part), A.hidden, A.eps);
    if (mine) A.xn[c] = __fmul_rn(A.norm0[c], __fmul_rn(xv, inv2));
}

// ------------------------------------------------------- attention prep
struct PrepArgs {
    const float *q_raw, *k_raw, *v_raw;
    float *q_out;
    float *k_cache, *v_cache;   // [cap, kv_dim] fp32
    float *k_hist, *v_hist;     // [K-1, kv_dim]
    const float *q_norm, *k_norm, *k_sconv, *v_sconv;
    int H, Hkv, Dh, K;
    int64_t kv_dim;
    float eps;
    int is_sliding, window;
    const double *tau_table;    // per position (global layers)
    ModelState *st;
    // relative-position band: rel_logits[h, r] = sum_d r_vec[h, d] rel_proj[d, r]
    const float *r_vec, *rel_proj;
    float *rel_logits;
    int d_rel, E;
};

// Depthwise causal convolution of one channel at T = 1 with its history,
// plus the history roll (sconv_apply, src/sepia.c:801-816).
__device__ __forceinline__ float sconv1(const float *w, float *hist, int64_t C, int K, int64_t c, float in) {
    // window = hist[0..K-2] then `in`; the history moves one frame down
    // (no local array: K is a runtime value)
    double acc = 0.0;
    const float *wc = w + c * K;
    for (int j = 0; j < K - 1; j++) {
        const float h = hist[(int64_t)j * C + c];
        acc += (double)wc[j] * (double)h;
        if (j > 0) hist[(int64_t)(j - 1) * C + c] = h;
    }
    acc += (double)wc[K - 1] * (double)in;
    if (K > 1) hist[(int64_t)(K - 2) * C + c] = in;
    return __fadd_rn(in, (float)acc);
}

// Blocks 0..H-1: query head h (RMSNorm, then (float)((double)q * tau),
// src/sepia.c:1153-1166, 1209). Blocks H..H+Hkv-1: KV head (K and V short
// convolutions, K RMSNorm, cache write at pos, src/sepia.c:1124-1180).
__global__ void __launch_bounds__(128) k_attn_prep(const PrepArgs A) {
    __shared__ double sh[33];
    __shared__ float v_sm[128];
    const int d = threadIdx.x;
    griddep_wait();
    griddep_launch();
    if ((int)blockIdx.x >= A.H + A.Hkv) {
        // the band projection (rel_project, src/sepia.c:1188-1194; the
        // same double accumulation as k_rel_project), one entry per thread
        const int64_t i = (int64_t)(blockIdx.x - A.H - A.Hkv) * blockDim.x + threadIdx.x;
        if (i >= (int64_t)A.H * A.E) return;
        const int64_t h = i / A.E, r = i - h * A.E;
        const float *rv = A.r_vec + h * A.d_rel;
        double acc = 0.0;
        for (int d = 0; d < A.d_rel; d++) acc = fma((double)rv[d], (double)A.rel_proj[(int64_t)d * A.E + r], acc);
        A.rel_logits[i] = (float)acc;
        return;
    }
    const int64_t pos = A.st->pos;
    const double tau = (A.is_sliding || !A.tau_table) ? 1.0 : A.tau_table[pos];
    if ((int)blockIdx.x < A.H) {
        const int h = blockIdx.x;
        const float qw = d < A.Dh ? A.q_norm[d] : 0.0f;
        if (d < A.Dh) v_sm[d] = A.q_raw[(int64_t)h * A.Dh + d];
        __syncthreads();
        const float inv = rms_inv(v_sm, A.Dh, A.eps, sh);
        if (d < A.Dh) {
            const float qn = __fmul_rn(qw, __fmul_rn(v_sm[d], inv));
            A.q_out[(int64_t)h * A.Dh + d] = (float)((double)qn * tau);
        }
        if (h == 0 && d == 0) {
            int64_t lo = A.is_sliding ? pos - A.window + 1 : 0;
            A.st->kv_lo = lo < 0 ? 0 : lo;
            A.st->kv_hi = pos;
            A.st->tau = tau;
        }
        return;
    }
    const int hk = blockIdx.x - A.H;
    const int64_t c = (int64_t)hk * A.Dh + d;
    const float kw = d < A.Dh ? A.k_norm[d] : 0.0f;
    float kv = 0.0f;
    if (d < A.Dh) {
        kv = sconv1(A.k_sconv, A.k_hist, A.kv_dim, A.K, c, A.k_raw[c]);
        const float vv = sconv1(A.v_sconv, A.v_hist, A.kv_dim, A.K, c, A.v_raw[c]);
        A.v_cache[pos * A.kv_dim + c] = vv;
        v_sm[d] = kv;
    }
    __syncthreads();
    const float inv = rms_inv(v_sm, A.Dh, A.eps, sh);
    if (d < A.Dh) A.k_cache[pos * A.kv_dim + c] = __fmul_rn(kw, __fmul_rn(kv, inv));
}

// --------------------------------------------------------- residual join
struct ResArgs {
    float *x;                   // residual stream [C], updated
    const float *in;            // block output [C]
    float scale;                // in * scale first (dense MLP global scale)
    int use_scale;
    const float *w;             // [C, K]
    float *hist;                // [K-1, C]
    int64_t C;
    int K;
    const float *norm_w;        // next norm
    float eps;
    float mup;                  // > 0: xn = normed / mup (logits input)
    float *xn;
    ModelState *st;
    int advance;                // pos += 1 at the end
};

// x += sconv(in) (src/sepia.c:1506-1519, 1535-1549), then xn = rmsnorm(x)
// for the next block. One cluster; each thread owns one channel per pass.
__global__ void __launch_bounds__(kClThreads) k_residual(const ResArgs A) {
    cg::cluster_group cl = cg::this_cluster();
    __shared__ double sh[33];
    __shared__ double part;
    griddep_wait();
    griddep_launch();
    const unsigned rank = cl.block_rank(), nr = cl.num_blocks();
    const int64_t per = (A.C + nr - 1) / nr;
    const int64_t c0 = rank * per, c1 = imin64(A.C, c0 + per);
    constexpr int kMaxPer = 8;          // channels per thread (hidden <= 8 * 1024 * kClusterCtas)
    float xs[kMaxPer], nw[kMaxPer];
    double sq = 0.0;
#pragma unroll
    for (int k = 0; k < kMaxPer; k++) {
        const int64_t c = c0 + threadIdx.x + (int64_t)k * blockDim.x;
        xs[k] = 0.0f;
        nw[k] = 0.0f;
        if (c < c1) {
            nw[k] = A.norm_w[c];      // fetched with the inputs: one memory round trip less
            const float v = A.use_scale ? __fmul_rn(A.in[c], A.scale) : A.in[c];
            const float o = sconv1(A.w, A.hist, A.C, A.K, c, v);
            const float xv = __fadd_rn(A.x[c], o);
            A.x[c] = xv;
            xs[k] = xv;
            sq += (double)__fmul_rn(xv, xv);
        }
    }
    const float inv = rms_inv_from(cluster_sum_d(sq, sh, &part), A.C, A.eps);
#pragma unroll
    for (int k = 0; k < kMaxPer; k++) {
        const int64_t c = c0 + threadIdx.x + (int64_t)k * blockDim.x;
        if (c < c1) {
            float v = __fmul_rn(nw[k], __fmul_rn(xs[k], inv));
            if (A.mup > 0.0f) v = __fdiv_rn(v, A.mup);
            A.xn[c] = v;
        }
    }
    if (A.advance && rank == 0 && threadIdx.x == 0) A.st->pos += 1;
}

// ---------------------------------------------------------------- argmax
// Order-preserving key: the float's bits mapped to an unsigned order in the
// high word, the bitwise complement of the index in the low word, so the
// largest value wins and among equal values the lowest index (argmax_f's
// strict '>' scan, src/sepia.c:764-773).
__device__ __forceinline__ unsigned long long argmax_key(float v, uint32_t i) {
    uint32_t u = __float_as_uint(v);
    u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ((unsigned long long)u << 32) | (unsigned long long)(0xFFFFFFFFu - i);
}

__global__ void __launch_bounds__(256) k_argmax(const float *logits, int32_t n, ModelState *st, int advance) {
    __shared__ unsigned long long sh[8];
    unsigned long long best = 0ull;
    griddep_wait();
    griddep_launch();
    for (int32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const float v = logits[i];
        if (v == v) {
            const unsigned long long k = argmax_key(v, (uint32_t)i);
            best = k > best ? k : best;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long t = __shfl_xor_sync(0xffffffffu, best, o);
        best = t > best ? t : best;
    }
    if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < (int)(blockDim.x >> 5); w++) best = sh[w] > best ? sh[w] : best;
        atomicMax(&st->best, best);
        if (advance && blockIdx.x == 0) st->pos += 1;
    }
}

__global__ void k_state_reset(ModelState *st) {
    st->best = 0ull;
    st->pos = 0;
    st->fed = 0;
    st->gen = 0;
    st->bad_token = 0;
}
__global__ void k_state_new_call(ModelState *st) {
    st->fed = 0;
    st->gen = 0;
}

}  // namespace sepia

using namespace sepia;

// ============================================================== host side
struct SepiaModel {
    SepiaModelDesc d;
    std::vector<SepiaModelLayer> layers;
    int device = -1;
    // device memory: one allocation carved into pieces
    void *mem = nullptr;
    size_t mem_bytes = 0;
    ModelState *st = nullptr;
    double *tau = nullptr;           // [max_positions]
    float *x = nullptr, *xn = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *r = nullptr, *qs = nullptr;
    float *rl = nullptr, *att = nullptr, *blk = nullptr, *g = nullptr, *u = nullptr, *h = nullptr;
    float *logits = nullptr;
    double *part = nullptr;
    size_t part_bytes = 0;
    std::vector<float *> kc, vc, kh, vh, ah, mh;   // per layer caches and histories
    std::vector<int> splits;                       // per layer attention split count
    void *moe_ws_mem = nullptr;
    SepiaMoeWork ws{};
    int64_t max_q = 0, max_kv = 0, max_r = 0, max_rl = 0, max_ff = 0;
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    int32_t *graph_out = nullptr;    // out_ids array baked into the graph
    // expert sharding (world > 1)
    int rank = 0, world = 1;
    SepiaExchange *xchg = nullptr;   // the sharded MoE layers' exchange
};

namespace {

size_t align256(size_t n) { return (n + 255) & ~(size_t)255; }

int check_q(const SepiaQTensor &t, int64_t rows, int64_t cols, const char *what, int l) {
    if (!t.data) return fail("model: layer %d %s: null weights", l, what);
    if (t.rows != rows || t.cols != cols)
        return fail("model: layer %d %s: shape [%lld, %lld], expected [%lld, %lld]", l, what, (long long)t.rows,
                    (long long)t.cols, (long long)rows, (long long)cols);
    if (host_row_bytes(t.type, cols) <= 0) return fail("model: layer %d %s: type %d unsupported", l, what, t.type);
    return 1;
}

// One cluster of kClusterCtas CTAs, launched with programmatic dependent
// launch like the rest of the chain.
template <typename Args>
int launch_cluster(void (*kern)(const Args), cudaStream_t st, const Args &a) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(kClusterCtas);
    cfg.blockDim = dim3(kClThreads);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = st;
    cudaLaunchAttribute at[2];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = kClusterCtas;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 2;
    return check(cudaLaunchKernelEx(&cfg, kern, a), "model: cluster kernel launch");
}

int mv(const SepiaQTensor &t, const float *x, float *y, int64_t rows, cudaStream_t st) {
    return launch_matvec_q(t.type, t.data, x, y, rows, t.cols, 1, st);
}

// Everything of one token after its embedding: the layers, then (want_logits)
// the head and the argmax. `last_advance`: which kernel moves pos.
int run_layers(SepiaModel *m, bool want_logits, cudaStream_t st) {
    const SepiaModelDesc &d = m->d;
    const int64_t hidden = d.hidden;
    const int K = d.conv_k;
    for (int l = 0; l < d.n_layers; l++) {
        const SepiaModelLayer &L = m->layers[l];
        const int H = L.n_heads, Hkv = L.n_kv_heads, Dh = L.head_dim;
        const int64_t q_dim = (int64_t)H * Dh, kv_dim = (int64_t)Hkv * Dh, r_dim = (int64_t)H * d.d_rel;
        if (L.wq.type == L.wk.type && L.wq.type == L.wv.type && L.wq.type == L.wr.type) {
            const void *w4[4] = {L.wq.data, L.wk.data, L.wv.data, L.wr.data};
            const int64_t r4[4] = {q_dim, kv_dim, kv_dim, r_dim};
            float *y4[4] = {m->q, m->k, m->v, m->r};
            if (!launch_matvec_q_multi(4, L.wq.type, w4, r4, hidden, m->xn, y4, st)) return 0;
        } else if (!mv(L.wq, m->xn, m->q, q_dim, st) || !mv(L.wk, m->xn, m->k, kv_dim, st) ||
                   !mv(L.wv, m->xn, m->v, kv_dim, st) || !mv(L.wr, m->xn, m->r, r_dim, st)) {
            return 0;
        }
        PrepArgs P;
        P.q_raw = m->q; P.k_raw = m->k; P.v_raw = m->v; P.q_out = m->qs;
        P.k_cache = m->kc[l]; P.v_cache = m->vc[l]; P.k_hist = m->kh[l]; P.v_hist = m->vh[l];
        P.q_norm = L.q_norm; P.k_norm = L.k_norm; P.k_sconv = L.k_sconv; P.v_sconv = L.v_sconv;
        P.H = H; P.Hkv = Hkv; P.Dh = Dh; P.K = K; P.kv_dim = kv_dim; P.eps = d.eps;
        P.is_sliding = L.is_sliding; P.window = d.window; P.tau_table = d.has_log_scaling ? m->tau : nullptr;
        P.st = m->st;
        P.r_vec = m->r; P.rel_proj = L.rel_proj; P.rel_logits = m->rl; P.d_rel = (int)d.d_rel;
        P.E = L.rel_extent;
        if (L.rel_extent <= 0 || d.d_rel <= 0 || !L.rel_proj) return fail("model: layer %d has no relative band", l);
        const unsigned rel_blocks = (unsigned)(((int64_t)H * L.rel_extent + 127) / 128);
        launch_pdl(k_attn_prep, (unsigned)(H + Hkv) + rel_blocks, 128, 0, st, P);
        if (!check(cudaGetLastError(), "model: attn_prep launch")) return 0;
        if (!launch_banded_attn_ex(0, m->qs, m->kc[l], m->vc[l], m->rl, m->att, &m->st->kv_lo, &m->st->kv_hi,
                                   nullptr, &m->st->tau, &m->st->pos, 1, H, Hkv, Dh, L.rel_extent, 0, kv_dim,
                                   (float)(1.0 / Dh), m->splits[l], m->part, st))
            return 0;
        if (!mv(L.wo, m->att, m->blk, hidden, st)) return 0;
        ResArgs R;
        R.x = m->x; R.in = m->blk; R.scale = 1.0f; R.use_scale = 0; R.w = L.attn_sconv; R.hist = m->ah[l];
        R.C = hidden; R.K = K; R.norm_w = L.mlp_norm; R.eps = d.eps; R.mup = 0.0f; R.xn = m->xn; R.st = m->st;
        R.advance = 0;
        if (!launch_cluster(k_residual, st, R)) return 0;
        if (L.is_sparse && m->world > 1) {
            if (!sepia_cuda_moe_layer_sharded(m->xchg, &L.moe, m->xn, &m->ws, m->blk, (void *)st)) return 0;
        } else if (L.is_sparse) {
            if (!sepia_cuda_moe_layer(&L.moe, m->xn, &m->ws, m->blk, (void *)st)) return 0;
        } else {
            const int64_t ff = L.dense_gate.rows;
            if (!mv(L.dense_gate, m->xn, m->g, ff, st) || !mv(L.dense_up, m->xn, m->u, ff, st)) return 0;
            if (!op_silu_mul(m->g, m->u, m->h, ff, st)) return 0;
            if (!mv(L.dense_down, m->h, m->blk, hidden, st)) return 0;
        }
        const bool last = (l == d.n_layers - 1);
        R.in = m->blk; R.use_scale = L.is_sparse ? 0 : 1; R.scale = L.dense_gscale; R.w = L.mlp_sconv;
        R.hist = m->mh[l];
        R.norm_w = last ? d.final_norm : m->layers[l + 1].attn_norm;
        R.mup = last ? d.mup : 0.0f;
        R.advance = (last && !want_logits) ? 1 : 0;
        if (!launch_cluster(k_residual, st, R)) return 0;
    }
    if (want_logits) {
        if (!launch_matvec_q(d.unembed.type, d.unembed.data, m->xn, m->logits, d.unpadded_vocab, hidden, 1, st))
            return 0;
        const int sms = dev_info().sm_count > 0 ? dev_info().sm_count : 148;
        launch_pdl(k_argmax, (unsigned)sms, 256, 0, st, (const float *)m->logits, d.unpadded_vocab, m->st, 1);
        if (!check(cudaGetLastError(), "model: argmax launch")) return 0;
    }
    return 1;
}

int embed(SepiaModel *m, int mode, const int32_t *ids, int32_t *out_ids, cudaStream_t st) {
    const SepiaModelDesc &d = m->d;
    EmbedArgs E;
    E.type = d.embed.type; E.w = (const uint8_t *)d.embed.data; E.rb = host_row_bytes(d.embed.type, d.hidden);
    E.hidden = d.hidden; E.vocab = d.vocab; E.ids = ids; E.mode = mode; E.out_ids = out_ids; E.st = m->st;
    E.embed_norm = d.embed_norm; E.norm0 = m->layers[0].attn_norm; E.eps = d.eps; E.x = m->x; E.xn = m->xn;
    E.err = dev_info().err;
    return launch_cluster(k_embed, st, E);
}

int setup_kernels(const SepiaModelDesc &d) {
    (void)d;
    return 1;
}

}  // namespace

extern "C" int sepia_model_create(const SepiaModelDesc *d, SepiaModel **out) {
    if (!d || !out) return fail("model: null argument");
    *out = nullptr;
    if (d->n_layers <= 0 || !d->layers) return fail("model: no layers");
    if (d->hidden <= 0 || d->hidden % 32 || d->hidden > 8 * kClThreads * kClusterCtas ||
        (d->hidden + kClusterCtas - 1) / kClusterCtas > kClThreads)
        return fail("model: hidden %lld unsupported (a multiple of 32, at most %d)", (long long)d->hidden,
                    kClThreads * kClusterCtas);
    if (d->conv_k < 1 || d->conv_k > kMaxConvK) return fail("model: conv kernel %d outside 1..%d", d->conv_k, kMaxConvK);
    if (d->max_positions <= 0) return fail("model: max_positions must be positive");
    if (d->unpadded_vocab <= 0 || d->unpadded_vocab > d->vocab) return fail("model: bad vocab sizes");
    if (!d->embed_norm || !d->final_norm) return fail("model: null norm weights");
    if (d->has_log_scaling && d->log_scaling_n_floor <= 0) return fail("model: log scaling needs n_floor > 0");
    if (d->mup == 0.0f) return fail("model: mup multiplier is zero");
    SepiaModel *m = new SepiaModel();
    m->d = *d;
    m->layers.assign(d->layers, d->layers + d->n_layers);
    m->d.layers = m->layers.data();
    const int64_t hidden = d->hidden;
    int ok = check_q(d->embed, d->vocab, hidden, "token_embd", -1) && check_q(d->unembed, d->vocab, hidden, "output", -1);
    if (ok && host_block_elems(d->embed.type) > 32 && hidden % host_block_elems(d->embed.type))
        ok = fail("model: hidden not a multiple of the embedding's block");
    size_t moe_ws = 0;
    const SepiaMoeLayer *moe0 = nullptr;
    for (int l = 0; ok && l < d->n_layers; l++) {
        const SepiaModelLayer &L = m->layers[l];
        if (L.n_heads <= 0 || L.n_kv_heads <= 0 || L.n_heads % L.n_kv_heads || L.head_dim <= 0 || L.head_dim > 128 ||
            L.rel_extent <= 0)
            { ok = fail("model: layer %d: bad attention geometry", l); break; }
        const int64_t q_dim = (int64_t)L.n_heads * L.head_dim, kv_dim = (int64_t)L.n_kv_heads * L.head_dim;
        const int64_t r_dim = (int64_t)L.n_heads * d->d_rel;
        ok = check_q(L.wq, q_dim, hidden, "attn_q", l) && check_q(L.wk, kv_dim, hidden, "attn_k", l) &&
             check_q(L.wv, kv_dim, hidden, "attn_v", l) && check_q(L.wr, r_dim, hidden, "attn_r", l) &&
             check_q(L.wo, hidden, q_dim, "attn_output", l);
        if (!ok) break;
        if (!L.attn_norm || !L.mlp_norm || !L.q_norm || !L.k_norm || !L.rel_proj || !L.k_sconv || !L.v_sconv ||
            !L.attn_sconv || !L.mlp_sconv)
            { ok = fail("model: layer %d: null f32 weights", l); break; }
        m->max_q = std::max(m->max_q, q_dim);
        m->max_kv = std::max(m->max_kv, kv_dim);
        m->max_r = std::max(m->max_r, r_dim);
        m->max_rl = std::max(m->max_rl, (int64_t)L.n_heads * L.rel_extent);
        if (L.is_sparse) {
            if (L.moe.hidden != hidden) { ok = fail("model: layer %d: MoE hidden differs", l); break; }
            const size_t b = sepia_cuda_moe_work_bytes(&L.moe);
            if (!b) { ok = fail("model: layer %d: bad MoE layer: %s", l, sepia_cuda_last_error()); break; }
            if (moe0 && (L.moe.ff != moe0->ff || L.moe.n_routed != moe0->n_routed ||
                         L.moe.n_shared != moe0->n_shared || L.moe.topk != moe0->topk))
                { ok = fail("model: layer %d: MoE shape differs from the first MoE layer", l); break; }
            if (!moe0) { moe_ws = b; moe0 = &L.moe; }
        } else {
            const int64_t ff = L.dense_gate.rows;
            ok = check_q(L.dense_gate, ff, hidden, "ffn_gate", l) && check_q(L.dense_up, ff, hidden, "ffn_up", l) &&
                 check_q(L.dense_down, hidden, ff, "ffn_down", l);
            m->max_ff = std::max(m->max_ff, ff);
        }
    }
    if (!ok) { delete m; return 0; }
    if (!check(cudaGetDevice(&m->device), "model: cudaGetDevice")) { delete m; return 0; }
    m->rank = d->rank;
    m->world = d->world < 1 ? 1 : d->world;
    if (m->rank < 0 || m->rank >= m->world) { fail("model: rank %d outside world %d", d->rank, d->world); delete m; return 0; }
    if (m->world > 1 && moe0) {
        for (int l = 0; l < d->n_layers; l++)
            if (m->layers[l].is_sparse && (m->layers[l].moe.rank != m->rank || m->layers[l].moe.world != m->world)) {
                fail("model: layer %d's MoE shard is not rank %d of %d", l, m->rank, m->world);
                delete m;
                return 0;
            }
        if (!sepia_cuda_exchange_create(moe0->topk + moe0->n_shared, hidden, m->rank, m->world, &m->xchg)) {
            delete m;
            return 0;
        }
    }
    // carve one allocation
    const int64_t cap = d->max_positions;
    const int K = d->conv_k;
    size_t part = 0;
    m->splits.resize(d->n_layers);
    for (int l = 0; l < d->n_layers; l++) {
        const SepiaModelLayer &L = m->layers[l];
        const int64_t span = L.is_sliding ? std::min<int64_t>(cap, d->window) : cap;
        m->splits[l] = attn_splits(1, L.n_kv_heads, span);
        part = std::max(part, attn_part_bytes(1, L.n_heads, m->splits[l], L.head_dim));
    }
    m->part_bytes = part;
    std::vector<std::pair<void **, size_t>> plan;
    auto add = [&](void **p, size_t bytes) { plan.push_back({p, align256(bytes)}); };
    add((void **)&m->st, sizeof(ModelState));
    add((void **)&m->tau, sizeof(double) * cap);
    add((void **)&m->x, 4 * hidden); add((void **)&m->xn, 4 * hidden); add((void **)&m->blk, 4 * hidden);
    add((void **)&m->q, 4 * m->max_q); add((void **)&m->qs, 4 * m->max_q); add((void **)&m->att, 4 * m->max_q);
    add((void **)&m->k, 4 * m->max_kv); add((void **)&m->v, 4 * m->max_kv);
    add((void **)&m->r, 4 * m->max_r); add((void **)&m->rl, 4 * m->max_rl);
    add((void **)&m->g, 4 * std::max<int64_t>(1, m->max_ff)); add((void **)&m->u, 4 * std::max<int64_t>(1, m->max_ff));
    add((void **)&m->h, 4 * std::max<int64_t>(1, m->max_ff));
    add((void **)&m->logits, 4 * (size_t)d->unpadded_vocab);
    add((void **)&m->part, part);
    add((void **)&m->moe_ws_mem, std::max<size_t>(moe_ws, 256));
    m->kc.resize(d->n_layers); m->vc.resize(d->n_layers); m->kh.resize(d->n_layers); m->vh.resize(d->n_layers);
    m->ah.resize(d->n_layers); m->mh.resize(d->n_layers);
    for (int l = 0; l < d->n_layers; l++) {
        const int64_t kv_dim = (int64_t)m->layers[l].n_kv_heads * m->layers[l].head_dim;
        add((void **)&m->kc[l], 4 * cap * kv_dim); add((void **)&m->vc[l], 4 * cap * kv_dim);
        add((void **)&m->kh[l], 4 * std::max(1, K - 1) * kv_dim); add((void **)&m->vh[l], 4 * std::max(1, K - 1) * kv_dim);
        add((void **)&m->ah[l], 4 * std::max(1, K - 1) * hidden); add((void **)&m->mh[l], 4 * std::max(1, K - 1) * hidden);
    }
    size_t total = 0;
    for (auto &p : plan) total += p.second;
    if (!check(cudaMalloc(&m->mem, total), "model: cudaMalloc")) { sepia_model_destroy(m); return 0; }
    m->mem_bytes = total;
    size_t off = 0;
    for (auto &p : plan) { *p.first = (char *)m->mem + off; off += p.second; }
    if (!check(cudaMemset(m->mem, 0, total), "model: clear")) { sepia_model_destroy(m); return 0; }
    if (moe0 && !sepia_cuda_moe_work_carve(moe0, m->moe_ws_mem, moe_ws, &m->ws)) { sepia_model_destroy(m); return 0; }
    // tau per position in double, as attn_forward_chunk computes it
    // (src/sepia.c:1188-1194), with the host's libm log
    std::vector<double> tau(cap, 1.0);
    if (d->has_log_scaling)
        for (int64_t p = 0; p < cap; p++) {
            double ratio = (double)(p + 1) / (double)d->log_scaling_n_floor;
            if (ratio < 1.0) ratio = 1.0;
            tau[p] = 1.0 + d->log_scaling_alpha * log(ratio);
        }
    if (!check(cudaMemcpy(m->tau, tau.data(), sizeof(double) * cap, cudaMemcpyHostToDevice), "model: tau upload") ||
        !setup_kernels(*d)) {
        sepia_model_destroy(m);
        return 0;
    }
    *out = m;
    return 1;
}

extern "C" void sepia_model_destroy(SepiaModel *m) {
    if (!m) return;
    if (m->exec) cudaGraphExecDestroy(m->exec);
    if (m->graph) cudaGraphDestroy(m->graph);
    if (m->mem) cudaFree(m->mem);
    if (m->xchg) sepia_cuda_exchange_destroy(m->xchg);
    delete m;
}

extern "C" int sepia_model_exchange_handle(SepiaModel *m, void *handle) {
    if (!m || !m->xchg) return fail("model: no exchange (world 1 or no MoE layer)");
    return sepia_cuda_exchange_handle(m->xchg, handle);
}

extern "C" int sepia_model_connect(SepiaModel *m, const void *handles) {
    if (!m || !m->xchg) return fail("model: no exchange (world 1 or no MoE layer)");
    return sepia_cuda_exchange_connect(m->xchg, handles);
}

extern "C" size_t sepia_model_device_bytes(const SepiaModel *m) { return m ? m->mem_bytes : 0; }

extern "C" int sepia_model_reset(SepiaModel *m, void *stream) {
    if (!m) return fail("model: null model");
    cudaStream_t st = as_stream(stream);
    const SepiaModelDesc &d = m->d;
    const int64_t cap = d.max_positions, K = d.conv_k, hidden = d.hidden;
    for (int l = 0; l < d.n_layers; l++) {
        const int64_t kv_dim = (int64_t)m->layers[l].n_kv_heads * m->layers[l].head_dim;
        const int64_t km1 = std::max<int64_t>(1, K - 1);
        if (!check(cudaMemsetAsync(m->kc[l], 0, 4 * cap * kv_dim, st), "model: reset") ||
            !check(cudaMemsetAsync(m->vc[l], 0, 4 * cap * kv_dim, st), "model: reset") ||
            !check(cudaMemsetAsync(m->kh[l], 0, 4 * km1 * kv_dim, st), "model: reset") ||
            !check(cudaMemsetAsync(m->vh[l], 0, 4 * km1 * kv_dim, st), "model: reset") ||
            !check(cudaMemsetAsync(m->ah[l], 0, 4 * km1 * hidden, st), "model: reset") ||
            !check(cudaMemsetAsync(m->mh[l], 0, 4 * km1 * hidden, st), "model: reset"))
            return 0;
    }
    k_state_reset<<<1, 1, 0, st>>>(m->st);
    return check(cudaGetLastError(), "model: reset");
}

extern "C" int sepia_model_prefill(SepiaModel *m, const int32_t *ids, int32_t n, int32_t want_logits, void *stream) {
    if (!m || !ids || n <= 0) return fail("model: prefill needs ids and n > 0");
    cudaStream_t st = as_stream(stream);
    k_state_new_call<<<1, 1, 0, st>>>(m->st);
    for (int32_t i = 0; i < n; i++) {
        if (!embed(m, 0, ids, nullptr, st)) return 0;
        if (!run_layers(m, want_logits && i == n - 1, st)) return 0;
    }
    return 1;
}

extern "C" int sepia_model_decode(SepiaModel *m, int32_t n, int32_t *out_ids, void *stream) {
    if (!m || !out_ids || n <= 0) return fail("model: decode needs out_ids and n > 0");
    cudaStream_t st = as_stream(stream);
    k_state_new_call<<<1, 1, 0, st>>>(m->st);
    if (!check(cudaGetLastError(), "model: decode")) return 0;
    if (m->exec && m->graph_out != out_ids) {
        cudaGraphExecDestroy(m->exec);
        cudaGraphDestroy(m->graph);
        m->exec = nullptr;
        m->graph = nullptr;
    }
    int32_t i0 = 0;
    if (!m->exec) {
        // The first step runs eagerly (it sets every kernel's attributes
        // outside any capture), the rest replay its captured twin.
        if (!embed(m, 1, nullptr, out_ids, st) || !run_layers(m, true, st)) return 0;
        i0 = 1;
        cudaStream_t cs;
        if (!check(cudaStreamCreateWithFlags(&cs, cudaStreamNonBlocking), "model: capture stream")) return 0;
        if (!check(cudaStreamBeginCapture(cs, cudaStreamCaptureModeThreadLocal), "model: begin capture")) {
            cudaStreamDestroy(cs);
            return 0;
        }
        int ok = embed(m, 1, nullptr, out_ids, cs) && run_layers(m, true, cs);
        cudaGraph_t g = nullptr;
        const cudaError_t e = cudaStreamEndCapture(cs, &g);
        cudaStreamDestroy(cs);
        if (!ok) { if (g) cudaGraphDestroy(g); return 0; }
        if (!check(e, "model: end capture")) return 0;
        if (!check(cudaGraphInstantiate(&m->exec, g, 0), "model: graph instantiate")) { cudaGraphDestroy(g); return 0; }
        m->graph = g;
        m->graph_out = out_ids;
    }
    for (int32_t i = i0; i < n; i++)
        if (!check(cudaGraphLaunch(m->exec, st), "model: graph launch")) return 0;
    return 1;
}

extern "C" const float *sepia_model_logits(const SepiaModel *m) { return m ? m->logits : nullptr; }

extern "C" int sepia_model_copy_logits(const SepiaModel *m, float *dst, void *stream) {
    if (!m || !dst) return fail("model: copy_logits needs a destination");
    return check(cudaMemcpyAsync(dst, m->logits, sizeof(float) * (size_t)m->d.unpadded_vocab,
                                 cudaMemcpyDeviceToDevice, as_stream(stream)), "model: copy logits");
}

extern "C" int sepia_model_position(SepiaModel *m, void *stream) {
    if (!m) return -1;
    if (!check(cudaStreamSynchronize(as_stream(stream)), "model: sync")) return -1;
    ModelState s;
    if (!check(cudaMemcpy(&s, m->st, sizeof s, cudaMemcpyDeviceToHost), "model: read state")) return -1;
    return s.pos;
}
