/* oracle/ref_shim.c -- TEST INFRASTRUCTURE ONLY.
 *
 * Compiles the reference's own CPU implementation (rinaldofesta/sepia
 * src/sepia.c, read in place from the reference checkout through -I, never
 * copied into this repository) and exports thin C wrappers around the static
 * functions the quantized-matvec path uses, so tests can pin the restatement
 * in oracle/*.c against the real thing and bench.py can time it:
 *   qlinear            src/sepia.c:748-753 (+ dequantize_row src/quants.c:250)
 *   moe_route_select   src/sepia.c:1329-1375
 *   rmsnorm            src/sepia.c:720-729
 *   sconv_apply        src/sepia.c:801-816
 *   attn_forward_chunk src/sepia.c:1077-1276
 *   real_load + real_forward_chunk + real_generate's greedy loop
 *                      src/sepia.c:2647, 3345, 4114 (token ids in and out:
 *                      the tokenizer file real_load opens is not needed, so
 *                      its loader is replaced by one that returns NULL)
 * Built by oracle/Makefile into oracle/_ref/libsepia_ref.so. */
#include "src/tokenizer.h"
#include "src/quants.h"
static Tokenizer *shim_tokenizer_load(const char *path) { (void)path; return (Tokenizer *)0; }

/* src/quants.c has no Q2_K, Q3_K, IQ2_XXS or IQ1_S (src/quants.h:6-10). For
 * the decoder (sepia.c) only, rows of those four formats are dequantized by
 * this directory's restatement, pinned bitwise to gguf-py 0.19.0
 * (quants_oracle.c); every other format still goes through src/quants.c.
 * The ref_dequantize_row / ref_qlinear exports below are not redirected. */
int or_dequantize_row(int type, const void *src, float *dst, int64_t n);
size_t or_row_bytes(int type, int64_t n);
static int shim_extra_type(int t) { return t == 10 || t == 11 || t == 16 || t == 19; }
static size_t shim_row_bytes(int t, int64_t ne) {
    return shim_extra_type(t) ? or_row_bytes(t, ne) : quants_row_bytes(t, ne);
}
static void shim_dequantize_row(int t, const void *src, float *dst, int64_t n) {
    if (shim_extra_type(t)) or_dequantize_row(t, src, dst, n);
    else dequantize_row(t, src, dst, n);
}
#define tokenizer_load shim_tokenizer_load
#define quants_row_bytes shim_row_bytes
#define dequantize_row shim_dequantize_row
#define main sepia_reference_main
#include "src/sepia.c"
#undef main
#undef tokenizer_load
#undef quants_row_bytes
#undef dequantize_row

#include <pthread.h>

int ref_quants_supported(int t) { return quants_supported(t); }

int ref_dequantize_row(int t, const void *src, float *dst, int64_t n) {
    if (!quants_supported(t) || n % quants_block_size(t) != 0) return 0;
    dequantize_row(t, src, dst, n);
    return 1;
}

typedef struct { QTensor w; const float *x; float *y; int64_t r0, r1; } RefQlJob;

static void *ref_ql_job(void *arg) {
    RefQlJob *j = (RefQlJob *)arg;
    float *scratch = xmalloc(sizeof(float) * (size_t)j->w.in_dim);
    size_t rb = quants_row_bytes(j->w.ggml_type, j->w.in_dim);
    QTensor part = j->w;
    part.data = (const uint8_t *)j->w.data + (size_t)j->r0 * rb;
    part.out_dim = j->r1 - j->r0;
    qlinear(&part, j->x, j->y + j->r0, scratch);
    free(scratch);
    return NULL;
}

/* The reference's qlinear loop, unchanged per row; nthreads > 1 splits the
 * output rows over pthreads (each thread runs qlinear on its own row range). */
int ref_qlinear(int t, const void *w, int64_t out_dim, int64_t in_dim, const float *x, float *y, int nthreads) {
    if (!quants_supported(t) || in_dim % quants_block_size(t) != 0) return 0;
    if (nthreads < 1) nthreads = 1;
    if (nthreads > 256) nthreads = 256;
    if (nthreads > out_dim) nthreads = (int)(out_dim > 0 ? out_dim : 1);
    RefQlJob jobs[256];
    pthread_t th[256];
    for (int i = 0; i < nthreads; i++) {
        jobs[i].w = (QTensor){ t, w, out_dim, in_dim };
        jobs[i].x = x; jobs[i].y = y;
        jobs[i].r0 = out_dim * i / nthreads; jobs[i].r1 = out_dim * (i + 1) / nthreads;
    }
    for (int i = 1; i < nthreads; i++) pthread_create(&th[i], NULL, ref_ql_job, &jobs[i]);
    ref_ql_job(&jobs[0]);
    for (int i = 1; i < nthreads; i++) pthread_join(th[i], NULL);
    return 1;
}

void ref_route_select(int n_routed, int n_shared, int topk, double route_scale, float global_scale,
                      const float *logits, const float *bias, int *topk_idx, float *weights) {
    Config cfg;
    memset(&cfg, 0, sizeof cfg);
    cfg.n_routed_experts = n_routed;
    cfg.n_shared_experts = n_shared;
    cfg.num_experts_per_tok = topk;
    cfg.route_scale = route_scale;
    LayerWeights lw;
    memset(&lw, 0, sizeof lw);
    lw.router_bias = bias;
    lw.router_global_scale = &global_scale;
    moe_route_select(&cfg, &lw, logits, topk_idx, weights);
}

void ref_rmsnorm(const float *x, const float *w, int n, float eps, float *out) { rmsnorm(x, w, n, eps, out); }

void ref_sconv_apply(const float *w, int C, int K, float *hist, const float *in, int T, float *out) {
    sconv_apply(w, C, K, hist, in, T, out);
}

/* One attention layer call (projections, sconv, per-head norms, cache write,
 * banded attention, wo) on fp32 weights. k_cache/v_cache are [cap, kv_dim]
 * and hold positions [0, start_pos) on entry; k_hist/v_hist are [K-1, kv_dim]
 * and are updated in place, exactly as LayerCache is. */
void ref_attn_chunk(int hidden, int H, int Hkv, int Dh, int d_rel, int rel_extent, int K,
                    int is_sliding, int window, float eps,
                    int has_log_scaling, double log_alpha, long log_n_floor,
                    const float *wq, const float *wk, const float *wv, const float *wr, const float *wo,
                    const float *q_norm, const float *k_norm, const float *rel_proj,
                    const float *k_sconv_w, const float *v_sconv_w,
                    float *k_cache, float *v_cache, float *k_hist, float *v_hist,
                    const float *x_normed, int T, int start_pos, float *out) {
    Config cfg;
    memset(&cfg, 0, sizeof cfg);
    cfg.hidden_size = hidden;
    cfg.conv_kernel_size = K;
    cfg.d_rel = d_rel;
    cfg.rms_norm_eps = eps;
    cfg.sliding_window_size = window;
    cfg.has_log_scaling_floor = has_log_scaling;
    cfg.log_scaling_alpha = log_alpha;
    cfg.log_scaling_n_floor = log_n_floor;
    LayerWeights lw;
    memset(&lw, 0, sizeof lw);
    lw.is_sliding = is_sliding;
    lw.num_heads = H; lw.num_kv_heads = Hkv; lw.head_dim = Dh; lw.rel_extent = rel_extent;
    lw.q_dim = H * Dh; lw.kv_dim = Hkv * Dh; lw.r_dim = H * d_rel;
    lw.wq = wq; lw.wk = wk; lw.wv = wv; lw.wr = wr; lw.wo = wo;
    lw.q_norm = q_norm; lw.k_norm = k_norm; lw.rel_proj = rel_proj;
    lw.k_sconv_w = k_sconv_w; lw.v_sconv_w = v_sconv_w;
    LayerCache lc;
    memset(&lc, 0, sizeof lc);
    lc.len = start_pos;
    lc.k = k_cache; lc.v = v_cache; lc.k_hist = k_hist; lc.v_hist = v_hist;
    attn_forward_chunk(&cfg, &lw, &lc, x_normed, T, start_pos, out);
}

/* Greedy generation on a container, token ids in and out: real_load
 * (page-cache expert reads), real_forward_chunk over the prompt, then
 * real_generate's loop (src/sepia.c:4131-4151): argmax of the current
 * logits, forward that token, n_gen times (no eos stop). out_ids[n_gen];
 * out_logits (optional) [n_gen, unpadded_vocab] = the logits each id was
 * taken from. Returns unpadded_vocab_size. Dies (exits) on a bad container,
 * as real_load does. */
int ref_generate_ids(const char *config_path, const char *manifest_path, const char *index_path,
                     const int *prompt, int n_prompt, int n_gen, int *out_ids, float *out_logits) {
    RealModel m = real_load(config_path, manifest_path, index_path, "unused-tokenizer", 0, 0, 1);
    const int unpadded = m.cfg.unpadded_vocab_size;
    Cache *cache = cache_create_cfg(&m.cfg, n_prompt + n_gen + 8);
    float *logits = xmalloc(sizeof(float) * (size_t)n_prompt * (size_t)unpadded);
    real_forward_chunk(&m, cache, prompt, n_prompt, 0, logits);
    float *cur = xmalloc(sizeof(float) * (size_t)unpadded);
    memcpy(cur, logits + (size_t)(n_prompt - 1) * unpadded, sizeof(float) * (size_t)unpadded);
    free(logits);
    int pos = n_prompt;
    for (int i = 0; i < n_gen; i++) {
        int tok = argmax_f(cur, unpadded);
        out_ids[i] = tok;
        if (out_logits) memcpy(out_logits + (size_t)i * unpadded, cur, sizeof(float) * (size_t)unpadded);
        real_forward_chunk(&m, cache, &tok, 1, pos, cur);
        pos++;
    }
    cache_free(cache);
    free(cur);
    return unpadded;
}
