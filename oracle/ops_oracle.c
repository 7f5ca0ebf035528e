/* oracle/ops_oracle.c -- TEST INFRASTRUCTURE ONLY (see sepia_oracle.h).
 *
 * CPU restatement of the reference math around the quantized matvec:
 * qlinear, rmsnorm, SwiGLU, the sigmoid top-k router, the MoE combine,
 * short convolution and the banded relative-position attention. Storage is
 * fp32, reductions accumulate in double, as src/sepia.c does. Each function
 * names the reference lines it restates. The optional pthread split only
 * partitions independent output rows; every row's arithmetic is unchanged. */
#pragma STDC FP_CONTRACT OFF

#include "sepia_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* ---- tiny row-parallel helper ------------------------------------------- */
typedef void (*RowFn)(void *ctx, int64_t r0, int64_t r1);
typedef struct { RowFn fn; void *ctx; int64_t r0, r1; } RowJob;

static void *row_job_main(void *a) {
    RowJob *j = (RowJob *)a;
    j->fn(j->ctx, j->r0, j->r1);
    return NULL;
}

static void parallel_rows(RowFn fn, void *ctx, int64_t rows, int nthreads) {
    if (nthreads <= 1 || rows < 2) { fn(ctx, 0, rows); return; }
    if (nthreads > 256) nthreads = 256;
    if (nthreads > rows) nthreads = (int)rows;
    pthread_t th[256];
    RowJob jobs[256];
    for (int i = 0; i < nthreads; i++) {
        jobs[i].fn = fn; jobs[i].ctx = ctx;
        jobs[i].r0 = rows * i / nthreads; jobs[i].r1 = rows * (i + 1) / nthreads;
    }
    int started = 0;
    for (int i = 1; i < nthreads; i++) {
        if (pthread_create(&th[i], NULL, row_job_main, &jobs[i]) != 0) break;
        started = i;
    }
    fn(ctx, jobs[0].r0, jobs[0].r1);
    for (int i = 1; i <= started; i++) pthread_join(th[i], NULL);
    for (int i = started + 1; i < nthreads; i++) fn(ctx, jobs[i].r0, jobs[i].r1);
}

/* ---- dot / linear / qlinear (src/sepia.c:731-753) ----------------------- */
static float dot_d(const float *a, const float *b, int64_t n) {
    double acc = 0.0;
    for (int64_t i = 0; i < n; i++) acc += (double)a[i] * (double)b[i];
    return (float)acc;
}

typedef struct { int type; const uint8_t *w; size_t rb; int64_t in; const float *x; float *y; int ok; } QlCtx;

static void ql_rows(void *c, int64_t r0, int64_t r1) {
    QlCtx *q = (QlCtx *)c;
    float *row = (float *)malloc(sizeof(float) * (size_t)(q->in ? q->in : 1));
    if (!row) { q->ok = 0; return; }
    for (int64_t o = r0; o < r1; o++) {
        if (!or_dequantize_row(q->type, q->w + (size_t)o * q->rb, row, q->in)) { q->ok = 0; break; }
        q->y[o] = dot_d(row, q->x, q->in);
    }
    free(row);
}

int or_qlinear(int type, const void *w, int64_t out_dim, int64_t in_dim, const float *x, float *y, int nthreads) {
    size_t rb = or_row_bytes(type, in_dim);
    if (!rb) return 0;
    QlCtx c = { type, (const uint8_t *)w, rb, in_dim, x, y, 1 };
    parallel_rows(ql_rows, &c, out_dim, nthreads);
    return c.ok;
}

/* Several vectors through one matrix: each row is dequantized once and
 * dotted with every vector by the same per-row arithmetic as or_qlinear
 * (src/sepia.c:748-753), so y[v] equals or_qlinear(x[v]) bit for bit. */
typedef struct { int type; const uint8_t *w; size_t rb; int64_t in, out, nv; const float *x; float *y; int ok; } QlbCtx;

static void qlb_rows(void *c, int64_t r0, int64_t r1) {
    QlbCtx *q = (QlbCtx *)c;
    float *row = (float *)malloc(sizeof(float) * (size_t)(q->in ? q->in : 1));
    if (!row) { q->ok = 0; return; }
    for (int64_t o = r0; o < r1; o++) {
        if (!or_dequantize_row(q->type, q->w + (size_t)o * q->rb, row, q->in)) { q->ok = 0; break; }
        for (int64_t v = 0; v < q->nv; v++) q->y[v * q->out + o] = dot_d(row, q->x + v * q->in, q->in);
    }
    free(row);
}

int or_qlinear_batch(int type, const void *w, int64_t out_dim, int64_t in_dim, int64_t n_vec,
                     const float *x, float *y, int nthreads) {
    size_t rb = or_row_bytes(type, in_dim);
    if (!rb) return 0;
    QlbCtx c = { type, (const uint8_t *)w, rb, in_dim, out_dim, n_vec, x, y, 1 };
    parallel_rows(qlb_rows, &c, out_dim, nthreads);
    return c.ok;
}

typedef struct { const float *w; int64_t in; const float *x; float *y; } LinCtx;
static void lin_rows(void *c, int64_t r0, int64_t r1) {
    LinCtx *l = (LinCtx *)c;
    for (int64_t o = r0; o < r1; o++) l->y[o] = dot_d(l->w + (size_t)o * (size_t)l->in, l->x, l->in);
}

void or_linear(const float *w, int64_t out_dim, int64_t in_dim, const float *x, float *y, int nthreads) {
    LinCtx c = { w, in_dim, x, y };
    parallel_rows(lin_rows, &c, out_dim, nthreads);
}

/* ---- norms and activations (src/sepia.c:720-729, 755-760) --------------- */
void or_rmsnorm(const float *x, const float *w, int64_t n, float eps, float *out) {
    double acc = 0.0;
    for (int64_t i = 0; i < n; i++) { float sq = x[i] * x[i]; acc += (double)sq; }
    const float var = (float)(acc / (double)n);
    const float inv = 1.0f / sqrtf(var + eps);
    for (int64_t i = 0; i < n; i++) out[i] = w[i] * (x[i] * inv);
}

float or_sigmoid(float x) { return 1.0f / (1.0f + expf(-x)); }
float or_silu(float x) { return x * or_sigmoid(x); }
float or_logsigmoid(float x) {
    if (x >= 0.0f) return -log1pf(expf(-x));
    return x - log1pf(expf(x));
}

void or_silu_mul(const float *g, const float *u, float *z, int64_t n) {
    for (int64_t i = 0; i < n; i++) z[i] = or_silu(g[i]) * u[i];
}

/* Row softmax in the structure of attn_forward_chunk's inline softmax
 * (src/sepia.c:1232-1245): max, exp in double, normalise. */
void or_softmax_rows(const float *x, float *y, int64_t rows, int64_t n) {
    for (int64_t r = 0; r < rows; r++) {
        const float *xr = x + r * n;
        float *yr = y + r * n;
        float m = -INFINITY;
        for (int64_t i = 0; i < n; i++) if (xr[i] > m) m = xr[i];
        double s = 0.0;
        for (int64_t i = 0; i < n; i++) { double e = exp((double)(xr[i] - m)); yr[i] = (float)e; s += e; }
        for (int64_t i = 0; i < n; i++) yr[i] = (float)((double)yr[i] / s);
    }
}

/* ---- short convolution (src/sepia.c:801-816) ----------------------------- */
void or_sconv_apply(const float *w, int64_t C, int64_t K, float *hist, const float *in, int64_t T, float *out) {
    const int64_t Km1 = K - 1;
    float *win = (float *)malloc(sizeof(float) * (size_t)(Km1 + T + 1));
    if (!win) return;
    for (int64_t c = 0; c < C; c++) {
        for (int64_t j = 0; j < Km1; j++) win[j] = hist[j * C + c];
        for (int64_t t = 0; t < T; t++) win[Km1 + t] = in[t * C + c];
        for (int64_t t = 0; t < T; t++) {
            double acc = 0.0;
            for (int64_t k = 0; k < K; k++) acc += (double)w[c * K + k] * (double)win[t + k];
            out[t * C + c] = in[t * C + c] + (float)acc;
        }
        for (int64_t j = 0; j < Km1; j++) hist[j * C + c] = win[T + j];
    }
    free(win);
}

void or_sconv_nohist(const float *w, const float *hist, const float *in, float *out, int64_t C, int64_t K, int64_t T) {
    const int64_t Km1 = K - 1;
    for (int64_t t = 0; t < T; t++)
        for (int64_t c = 0; c < C; c++) {
            double acc = 0.0;
            for (int64_t k = 0; k < K; k++) {
                int64_t i = t + k;
                float v = (i < Km1) ? hist[i * C + c] : in[(i - Km1) * C + c];
                acc += (double)w[c * K + k] * (double)v;
            }
            out[t * C + c] = in[t * C + c] + (float)acc;
        }
}

void or_sconv_hist_roll(float *hist, const float *in, int64_t C, int64_t K, int64_t T) {
    const int64_t Km1 = K - 1;
    for (int64_t c = 0; c < C; c++) {
        /* window = hist ++ in; new hist = its last Km1 rows */
        for (int64_t j = 0; j < Km1; j++) {
            int64_t src = T + j; /* index into the window */
            float v = (src < Km1) ? hist[src * C + c] : in[(src - Km1) * C + c];
            /* src >= j always, so rows are read before they are overwritten */
            hist[j * C + c] = v;
        }
    }
}

/* ---- router (src/sepia.c:1329-1375) -------------------------------------- */
void or_topk_scores(int n, int topk, const float *scores, int *idx) {
    unsigned char *used = (unsigned char *)calloc((size_t)n, 1);
    for (int j = 0; j < topk; j++) {
        int best = -1;
        for (int i = 0; i < n; i++) {
            if (used && used[i]) continue;
            if (best < 0 || scores[i] > scores[best]) best = i;
        }
        idx[j] = best;
        if (used && best >= 0) used[best] = 1;
    }
    free(used);
}

void or_route_select(int n_routed, int n_shared, int topk, double route_scale, float global_scale,
                     const float *logits, const float *bias, int *idx, float *weights) {
    float *sc = (float *)malloc(sizeof(float) * (size_t)n_routed);
    for (int i = 0; i < n_routed; i++) sc[i] = or_sigmoid(logits[i]) + bias[i];
    or_topk_scores(n_routed, topk, sc, idx);
    free(sc);

    const int n_sel = topk + n_shared;
    float lp[64];
    for (int j = 0; j < n_sel && j < 64; j++)
        lp[j] = or_logsigmoid(j < topk ? logits[idx[j]] : logits[n_routed + (j - topk)]);
    float lmax = lp[0];
    for (int j = 1; j < n_sel; j++) if (lp[j] > lmax) lmax = lp[j];
    double se = 0.0;
    for (int j = 0; j < n_sel; j++) se += exp((double)(lp[j] - lmax));
    const double lse = lmax + log(se);
    const double gs = (double)global_scale;
    for (int j = 0; j < n_sel; j++) {
        double w = exp((double)lp[j] - lse);
        w *= route_scale * gs;
        weights[j] = (float)w;
    }
}

/* ---- experts and the MoE layer ------------------------------------------ */
int or_expert_swiglu(int gt, const void *g, int ut, const void *u, int dt, const void *d,
                     int64_t hidden, int64_t ff, float h_scale, const float *x, float *y, int nthreads) {
    float *gv = (float *)malloc(sizeof(float) * (size_t)ff);
    float *uv = (float *)malloc(sizeof(float) * (size_t)ff);
    float *h = (float *)malloc(sizeof(float) * (size_t)ff);
    int ok = gv && uv && h;
    ok = ok && or_qlinear(gt, g, ff, hidden, x, gv, nthreads);
    ok = ok && or_qlinear(ut, u, ff, hidden, x, uv, nthreads);
    if (ok) {
        /* routed: h = silu(g)*u (src/sepia.c:3020); shared: *gamma inside h
         * (src/sepia.c:1442) -- h_scale == 1 reproduces the routed case. */
        for (int64_t i = 0; i < ff; i++) h[i] = (h_scale == 1.0f) ? or_silu(gv[i]) * uv[i]
                                                                   : or_silu(gv[i]) * uv[i] * h_scale;
        ok = or_qlinear(dt, d, hidden, ff, h, y, nthreads);
    }
    free(gv); free(uv); free(h);
    return ok;
}

int or_moe_layer(const OrMoeLayer *L, const float *x, float *out,
                 float *logits_out, int *idx_out, float *w_out, int nthreads) {
    const int n_total = L->n_routed + L->n_shared;
    const int n_sel = L->topk + L->n_shared;
    float *logits = (float *)malloc(sizeof(float) * (size_t)n_total);
    float *eo = (float *)malloc(sizeof(float) * (size_t)L->hidden);
    int idx[64];
    float w[64];
    if (!logits || !eo || n_sel > 64) { free(logits); free(eo); return 0; }
    or_linear(L->router_w, n_total, L->hidden, x, logits, nthreads);
    or_route_select(L->n_routed, L->n_shared, L->topk, L->route_scale, L->global_scale,
                    logits, L->router_bias, idx, w);
    for (int64_t i = 0; i < L->hidden; i++) out[i] = 0.0f;
    int ok = 1;
    for (int j = 0; j < L->topk && ok; j++) {
        const size_t e = (size_t)idx[j];
        ok = or_expert_swiglu(L->gate_type, L->gate + e * L->gate_stride, L->up_type, L->up + e * L->up_stride,
                              L->down_type, L->down + e * L->down_stride, L->hidden, L->ff, 1.0f, x, eo, nthreads);
        for (int64_t i = 0; i < L->hidden; i++) out[i] += eo[i] * w[j];
    }
    for (int s = 0; s < L->n_shared && ok; s++) {
        ok = or_expert_swiglu(L->sh_gate_type, L->sh_gate + (size_t)s * L->sh_gate_stride,
                              L->sh_up_type, L->sh_up + (size_t)s * L->sh_up_stride,
                              L->sh_down_type, L->sh_down + (size_t)s * L->sh_down_stride,
                              L->hidden, L->ff, w[L->topk + s], x, eo, nthreads);
        for (int64_t i = 0; i < L->hidden; i++) out[i] += eo[i];
    }
    if (logits_out) memcpy(logits_out, logits, sizeof(float) * (size_t)n_total);
    if (idx_out) memcpy(idx_out, idx, sizeof(int) * (size_t)L->topk);
    if (w_out) memcpy(w_out, w, sizeof(float) * (size_t)n_sel);
    free(logits); free(eo);
    return ok;
}

/* ---- banded attention (src/sepia.c:1195-1262) ------------------------------ */
void or_rel_project(const float *r_vec, const float *rel_proj, float *rel_logits,
                    int64_t T, int64_t H, int64_t d_rel, int64_t rel_extent) {
    for (int64_t th = 0; th < T * H; th++) {
        const float *rv = r_vec + th * d_rel;
        for (int64_t r = 0; r < rel_extent; r++) {
            double acc = 0.0;
            for (int64_t d = 0; d < d_rel; d++) acc += (double)rv[d] * (double)rel_proj[d * rel_extent + r];
            rel_logits[th * rel_extent + r] = (float)acc;
        }
    }
}

typedef struct {
    const float *q, *k, *v, *rl; float *out; const int64_t *lo, *hi; const float *tau; const double *tau64;
    int64_t H, Hkv, Dh, E, base, kv_dim; double inv;
} AttnCtx;

static void attn_rows(void *c, int64_t r0, int64_t r1) {
    AttnCtx *a = (AttnCtx *)c;
    const int64_t group = a->H / a->Hkv;
    double *acc = (double *)malloc(sizeof(double) * (size_t)a->Dh);
    for (int64_t th = r0; th < r1; th++) {
        const int64_t t = th / a->H, h = th % a->H, hk = h / group;
        const int64_t q_pos = a->base + t, lo = a->lo[t], hi = a->hi[t], n = hi - lo + 1;
        const double tau = a->tau64 ? a->tau64[t] : (double)a->tau[t];
        const float *qv = a->q + th * a->Dh;
        const float *rl = a->rl + th * a->E;
        float *sc = (float *)malloc(sizeof(float) * (size_t)(n > 0 ? n : 1));
        float mx = -INFINITY;
        for (int64_t kv = lo; kv <= hi; kv++) {
            const float *kvv = a->k + kv * a->kv_dim + hk * a->Dh;
            double content = (double)dot_d(qv, kvv, a->Dh) * a->inv;
            int64_t dist = q_pos - kv;
            double bias = (dist < a->E) ? (double)rl[dist] * tau : 0.0;
            float s = (float)(content + bias);
            sc[kv - lo] = s;
            if (s > mx) mx = s;
        }
        double se = 0.0;
        for (int64_t i = 0; i < n; i++) { double e = exp((double)(sc[i] - mx)); sc[i] = (float)e; se += e; }
        for (int64_t d = 0; d < a->Dh; d++) acc[d] = 0.0;
        for (int64_t i = 0; i < n; i++) {
            const double wg = (double)sc[i] / se;
            const float *vv = a->v + (lo + i) * a->kv_dim + hk * a->Dh;
            for (int64_t d = 0; d < a->Dh; d++) acc[d] += wg * (double)vv[d];
        }
        for (int64_t d = 0; d < a->Dh; d++) a->out[th * a->Dh + d] = (float)acc[d];
        free(sc);
    }
    free(acc);
}

static void banded_attn_any(const float *q, const float *k, const float *v, const float *rel_logits,
                            float *out, const int64_t *kv_lo, const int64_t *kv_hi, const float *tau,
                            const double *tau64, int64_t T, int64_t H, int64_t Hkv, int64_t Dh, int64_t rel_extent,
                            int64_t q_pos_base, int64_t kv_dim, float inv_head_dim, int nthreads) {
    /* the reference scales by 1.0/(double)Dh (src/sepia.c:1217); a float equal
     * to that value rounded stands for it */
    const double inv_exact = 1.0 / (double)Dh;
    AttnCtx c = { q, k, v, rel_logits, out, kv_lo, kv_hi, tau, tau64, H, Hkv, Dh, rel_extent,
                  q_pos_base, kv_dim, ((float)inv_exact == inv_head_dim) ? inv_exact : (double)inv_head_dim };
    parallel_rows(attn_rows, &c, T * H, nthreads);
}

void or_banded_attn(const float *q, const float *k, const float *v, const float *rel_logits,
                    float *out, const int64_t *kv_lo, const int64_t *kv_hi, const float *tau,
                    int64_t T, int64_t H, int64_t Hkv, int64_t Dh, int64_t rel_extent,
                    int64_t q_pos_base, int64_t kv_dim, float inv_head_dim, int nthreads) {
    banded_attn_any(q, k, v, rel_logits, out, kv_lo, kv_hi, tau, NULL, T, H, Hkv, Dh, rel_extent, q_pos_base,
                    kv_dim, inv_head_dim, nthreads);
}

/* The same with tau in double, as attn_forward_chunk holds it
 * (src/sepia.c:1188-1194: the bias is rel_logits * tau in double). */
void or_banded_attn64(const float *q, const float *k, const float *v, const float *rel_logits,
                      float *out, const int64_t *kv_lo, const int64_t *kv_hi, const double *tau,
                      int64_t T, int64_t H, int64_t Hkv, int64_t Dh, int64_t rel_extent,
                      int64_t q_pos_base, int64_t kv_dim, float inv_head_dim, int nthreads) {
    banded_attn_any(q, k, v, rel_logits, out, kv_lo, kv_hi, NULL, tau, T, H, Hkv, Dh, rel_extent, q_pos_base,
                    kv_dim, inv_head_dim, nthreads);
}
