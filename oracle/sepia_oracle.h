/* oracle/sepia_oracle.h -- TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C, single-precision-storage / double-accumulation restatement of
 * the reference CPU path (rinaldofesta/sepia src/quants.c and src/sepia.c)
 * for the quantized-matvec decode path. It is the checker for the CUDA
 * library, never part of it: only tests/, __graft_entry__.smoke() and
 * bench.py's CPU-baseline leg load it. Nothing in sepia_b200/ links it.
 *
 * Parity status:
 *   - F32, F16, Q8_0, Q4_K, Q5_K, Q6_K, IQ2_XS, IQ3_XXS, IQ4_XS dequant:
 *     pinned bitwise to the reference's own SQFX fixtures
 *     (tools/fixtures/quants/*.bin) and to src/quants.c compiled from the
 *     reference sources (oracle/_ref).
 *   - Q2_K, Q3_K, IQ2_XXS, IQ1_S: absent from the reference; pinned bitwise
 *     to gguf-py 0.19.0 `dequantize` through committed SQFX fixtures
 *     (tests/golden/make_golden.py).
 *   - qlinear / router selection / sconv / rmsnorm / banded attention:
 *     pinned against the reference's static functions compiled from
 *     src/sepia.c (oracle/ref_shim.c) when the reference checkout is present.
 */
#ifndef SEPIA_ORACLE_H
#define SEPIA_ORACLE_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ggml type ids (src/quants.h:6-10 for the nine the reference has; ggml's own
 * numbering for Q2_K=10, Q3_K=11, IQ2_XXS=16, IQ1_S=19). */
enum {
    OR_T_F32 = 0, OR_T_F16 = 1, OR_T_Q8_0 = 8, OR_T_Q2_K = 10, OR_T_Q3_K = 11,
    OR_T_Q4_K = 12, OR_T_Q5_K = 13, OR_T_Q6_K = 14, OR_T_IQ2_XXS = 16,
    OR_T_IQ2_XS = 17, OR_T_IQ3_XXS = 18, OR_T_IQ1_S = 19, OR_T_IQ4_XS = 23,
};

/* --- formats (src/quants.c:28-56, 250-265) ------------------------------ */
int     or_supported(int type);
int64_t or_block_size(int type);            /* 0 if unsupported */
size_t  or_type_size(int type);             /* 0 if unsupported */
size_t  or_row_bytes(int type, int64_t n);  /* 0 if unsupported or ragged */
float   or_f16_to_f32(uint16_t h);          /* src/quants.c:58-77 */
/* Returns 1 on success, 0 on an unsupported type or a ragged n. */
int     or_dequantize_row(int type, const void *src, float *dst, int64_t n);

/* --- qlinear (src/sepia.c:742-753) -------------------------------------- */
/* y[o] = (float) sum_double dequant(W[o,:]) * x. Rows split over nthreads
 * pthreads (nthreads <= 1: the reference's single-threaded loop). */
int or_qlinear(int type, const void *w, int64_t out_dim, int64_t in_dim,
               const float *x, float *y, int nthreads);
int or_qlinear_batch(int type, const void *w, int64_t out_dim, int64_t in_dim, int64_t n_vec,
                     const float *x, float *y, int nthreads);
/* f32 linear (src/sepia.c:731-740). */
void or_linear(const float *w, int64_t out_dim, int64_t in_dim, const float *x, float *y, int nthreads);

/* --- elementwise and norms (src/sepia.c:720-729, 755-760, 801-816) -------- */
void or_rmsnorm(const float *x, const float *w, int64_t n, float eps, float *out);
float or_sigmoid(float x);
float or_silu(float x);
float or_logsigmoid(float x);
void or_silu_mul(const float *g, const float *u, float *z, int64_t n);
void or_softmax_rows(const float *x, float *y, int64_t rows, int64_t n);
/* sconv_apply: updates hist [K-1,C] in place, writes out [T,C]. */
void or_sconv_apply(const float *w, int64_t C, int64_t K, float *hist, const float *in, int64_t T, float *out);
/* GPU-ABI sconv (no history write-back): out = in + sum_k w[c,k]*window[t+k]. */
void or_sconv_nohist(const float *w, const float *hist, const float *in, float *out, int64_t C, int64_t K, int64_t T);
/* sconv_hist_roll: the tail update of sconv_apply on its own. */
void or_sconv_hist_roll(float *hist, const float *in, int64_t C, int64_t K, int64_t T);

/* --- router (src/sepia.c:1329-1375) --------------------------------------- */
/* scores = sigmoid(logit)+bias over the n_routed first logits, top-k by the
 * strict-greater scan (lowest index wins ties), weights over the k selected
 * raw logits plus the n_shared sink logits. weights has topk+n_shared slots. */
void or_route_select(int n_routed, int n_shared, int topk, double route_scale, float global_scale,
                     const float *logits, const float *bias, int *topk_idx, float *weights);
/* Selection only, given precomputed scores (the bit-exact part). */
void or_topk_scores(int n, int topk, const float *scores, int *topk_idx);

/* --- MoE layer (src/sepia.c:1377-1470 + real_expert_ffn 2993-3022) ------- */
typedef struct {
    int64_t hidden, ff;              /* x is [hidden]; each expert is [ff,hidden]/[hidden,ff] */
    int n_routed, n_shared, topk;
    double route_scale;
    float global_scale;
    const float *router_w;           /* [n_routed+n_shared, hidden] f32 */
    const float *router_bias;        /* [n_routed] */
    int gate_type, up_type, down_type;             /* routed expert quant types */
    const uint8_t *gate, *up, *down;               /* expert e at base + e*stride */
    size_t gate_stride, up_stride, down_stride;
    int sh_gate_type, sh_up_type, sh_down_type;    /* shared expert quant types */
    const uint8_t *sh_gate, *sh_up, *sh_down;
    size_t sh_gate_stride, sh_up_stride, sh_down_stride;
} OrMoeLayer;

/* out = sum_j w_j * E_j(x) + sum_s S_s(x) with gamma folded into the shared
 * activation (mlp_moe_forward's order). Optional outputs (may be NULL):
 * logits [n_routed+n_shared], topk_idx [topk], weights [topk+n_shared]. */
int or_moe_layer(const OrMoeLayer *L, const float *x, float *out,
                 float *logits, int *topk_idx, float *weights, int nthreads);
/* One expert SwiGLU: y = down(silu(gate x) * (up x)) * (scale on h). */
int or_expert_swiglu(int gt, const void *g, int ut, const void *u, int dt, const void *d,
                     int64_t hidden, int64_t ff, float h_scale, const float *x, float *y, int nthreads);

/* --- banded attention (src/sepia.c:1195-1262) ------------------------------ */
void or_rel_project(const float *r_vec, const float *rel_proj, float *rel_logits,
                    int64_t T, int64_t H, int64_t d_rel, int64_t rel_extent);
/* q already tau-scaled; k/v are [cap, kv_dim] f32 caches. */
void or_banded_attn(const float *q, const float *k, const float *v, const float *rel_logits,
                    float *out, const int64_t *kv_lo, const int64_t *kv_hi, const float *tau,
                    int64_t T, int64_t H, int64_t Hkv, int64_t Dh, int64_t rel_extent,
                    int64_t q_pos_base, int64_t kv_dim, float inv_head_dim, int nthreads);
void or_banded_attn64(const float *q, const float *k, const float *v, const float *rel_logits,
                      float *out, const int64_t *kv_lo, const int64_t *kv_hi, const double *tau,
                      int64_t T, int64_t H, int64_t Hkv, int64_t Dh, int64_t rel_extent,
                      int64_t q_pos_base, int64_t kv_dim, float inv_head_dim, int nthreads);

#ifdef __cplusplus
}
#endif
#endif
