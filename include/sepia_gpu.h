/* include/sepia_gpu.h -- the GPU backend contract of rinaldofesta/sepia,
 * implemented by libsepia_cuda.so for NVIDIA B200 (sm_100a).
 *
 * The 30 functions below keep the exact names, argument lists and return
 * conventions of the reference's src/sepia_gpu.h, so the reference's
 * src/sepia.c links against this library in place of src/sepia_metal.m or
 * src/sepia_gpu_stub.c without a source change. Each declaration cites the
 * reference line it replaces. Conventions (src/sepia_gpu.h:1-3):
 *   - every function returns 1 / non-NULL on success and 0 / NULL on failure,
 *     after printing "sepia: cuda: ..." to stderr; nothing calls exit();
 *   - every op requires an open batch (sepia_gpu_begin) and never opens one
 *     implicitly (src/sepia_gpu.h:63-85);
 *   - single host thread only, like the Metal backend.
 *
 * Buffer model on a discrete GPU (the reference's Metal buffers are
 * unified memory; here they are mirrored):
 *   - alloc(len, 0) "Shared": device memory plus a pinned host mirror
 *     returned by host_ptr. The first op of a batch that names a Shared
 *     buffer uploads its host mirror (so a buffer filled after begin(), as
 *     src/sepia.c:4941 does, is seen); sepia_gpu_end() downloads every
 *     Shared or wrapped buffer the GPU wrote during the batch. Host writes
 *     therefore belong before the first op that uses the buffer and host
 *     reads after end() -- the reference's calling discipline
 *     (src/sepia_gpu.h:86-88 and every caller in src/sepia.c).
 *   - alloc(len, 1) "Private": device memory only, host_ptr NULL.
 *   - wrap_mmap(base, len): the bytes are copied into device memory once, at
 *     wrap time (the reference wraps the read-only resident.bin mapping);
 *     host_ptr returns `base`; GPU writes are copied back at end().
 */
#ifndef SEPIA_GPU_H
#define SEPIA_GPU_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif
#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

/* ----------------------------------------------------------- lifecycle */
int  sepia_gpu_available(void);                 /* src/sepia_gpu.h:9  */
int  sepia_gpu_init(const char *metal_dir);     /* src/sepia_gpu.h:10 (dir ignored: kernels are compiled in) */
void sepia_gpu_shutdown(void);                  /* src/sepia_gpu.h:11 */
const char *sepia_gpu_device_name(void);        /* src/sepia_gpu.h:12 */

/* ------------------------------------------------------------- buffers */
typedef struct SepiaGpuBuf SepiaGpuBuf;         /* src/sepia_gpu.h:19 (opaque) */
SepiaGpuBuf *sepia_gpu_wrap_mmap(void *base, size_t len);   /* src/sepia_gpu.h:33; NULL unless base is page-aligned */
SepiaGpuBuf *sepia_gpu_alloc(size_t len, int gpu_private);  /* src/sepia_gpu.h:38 */
void sepia_gpu_free(SepiaGpuBuf *b);                         /* src/sepia_gpu.h:43 */
void *sepia_gpu_host_ptr(SepiaGpuBuf *b);                    /* src/sepia_gpu.h:48 */
uint64_t sepia_gpu_gpu_addr(SepiaGpuBuf *b);                 /* src/sepia_gpu.h:52 (a CUDA device pointer) */
int sepia_gpu_selftest_touch(SepiaGpuBuf *buf, size_t n_floats); /* src/sepia_gpu.h:61 */

/* ------------------------------------------------------------ batching */
int sepia_gpu_begin(void);                      /* src/sepia_gpu.h:86 */
int sepia_gpu_flush(void);                      /* src/sepia_gpu.h:87 */
int sepia_gpu_end(void);                        /* src/sepia_gpu.h:88; 0 on device error or watchdog timeout */

/* ----------------------------------------------------------------- ops */
int sepia_gpu_rmsnorm(SepiaGpuBuf *w, SepiaGpuBuf *x, SepiaGpuBuf *y, int64_t rows, int64_t n, float eps);   /* :102 */
int sepia_gpu_matvec(SepiaGpuBuf *w, SepiaGpuBuf *x, SepiaGpuBuf *y, int64_t out_dim, int64_t in_dim);       /* :108 */
int sepia_gpu_silu_mul(SepiaGpuBuf *g, SepiaGpuBuf *u, SepiaGpuBuf *z, int64_t n);                            /* :113 */
int sepia_gpu_add(SepiaGpuBuf *a, SepiaGpuBuf *b, SepiaGpuBuf *out, int64_t n);                              /* :116 */
int sepia_gpu_softmax(SepiaGpuBuf *x, SepiaGpuBuf *y, int64_t rows, int64_t n);                               /* :122 */
int sepia_gpu_sconv(SepiaGpuBuf *w, SepiaGpuBuf *hist, SepiaGpuBuf *in, SepiaGpuBuf *out,
                    int64_t C, int64_t K, int64_t T);                                                          /* :128 */
int sepia_gpu_matvec_q(int ggml_type, SepiaGpuBuf *w, size_t w_off, SepiaGpuBuf *x, SepiaGpuBuf *y,
                       int64_t out_dim, int64_t in_dim);                                                       /* :147 */
int sepia_gpu_dequant_rows(int ggml_type, SepiaGpuBuf *raw, size_t raw_off, SepiaGpuBuf *out, int64_t n);     /* :160 */
int sepia_gpu_rel_project(SepiaGpuBuf *r_vec, SepiaGpuBuf *rel_proj, SepiaGpuBuf *rel_logits,
                          int64_t T, int64_t H, int64_t d_rel, int64_t rel_extent);                            /* :209 */
int sepia_gpu_banded_attn(SepiaGpuBuf *q, SepiaGpuBuf *k, SepiaGpuBuf *v, SepiaGpuBuf *rel_logits,
                          SepiaGpuBuf *attn_out, const int64_t *kv_lo, const int64_t *kv_hi, const float *tau,
                          int64_t T, int64_t H, int64_t Hkv, int64_t Dh, int64_t rel_extent,
                          int64_t q_pos_base, int64_t kv_dim, float inv_head_dim);                             /* :226 */
int sepia_gpu_matvec_off(SepiaGpuBuf *w, size_t w_off, SepiaGpuBuf *x, SepiaGpuBuf *y, int64_t out_dim, int64_t in_dim); /* :249 */
int sepia_gpu_rmsnorm_off(SepiaGpuBuf *w, size_t w_off, SepiaGpuBuf *x, SepiaGpuBuf *y, int64_t rows, int64_t n, float eps); /* :250 */
int sepia_gpu_sconv_off(SepiaGpuBuf *w, size_t w_off, SepiaGpuBuf *hist, SepiaGpuBuf *in, SepiaGpuBuf *out,
                        int64_t C, int64_t K, int64_t T);                                                      /* :251 */
int sepia_gpu_rel_project_off(SepiaGpuBuf *r_vec, SepiaGpuBuf *rel_proj, size_t rel_proj_off, SepiaGpuBuf *rel_logits,
                              int64_t T, int64_t H, int64_t d_rel, int64_t rel_extent);                        /* :253 */
int sepia_gpu_copy(SepiaGpuBuf *src, size_t src_off, SepiaGpuBuf *dst, size_t dst_off, int64_t n);           /* :264 */
int sepia_gpu_scale(float scale, SepiaGpuBuf *x, SepiaGpuBuf *y, int64_t n);                                  /* :272 */
int sepia_gpu_sconv_hist_roll(SepiaGpuBuf *hist, SepiaGpuBuf *in, int64_t C, int64_t K, int64_t T);          /* :285 */

/* ----------------------------------------------------- ggml type ids
 * src/quants.h:6-10 defines F32=0 F16=1 Q8_0=8 Q4_K=12 Q5_K=13 Q6_K=14
 * IQ2_XS=17 IQ3_XXS=18 IQ4_XS=23. This backend also accepts ggml's Q2_K=10,
 * Q3_K=11, IQ2_XXS=16 and IQ1_S=19 in matvec_q / dequant_rows. */

/* ---------------------------------------------- extension: MoE layer
 * No counterpart in the reference's header: it replaces the host-side
 * sequence of real_mlp_moe_forward_gpu (src/sepia.c:3831-3974 -- router
 * matvec_off, SYNC, moe_route_select, per-expert matvec_q/silu_mul, SYNC,
 * host combine) with one device-resident call and zero host syncs.
 * Weights are (buffer, byte offset) pairs; routed expert e's gate matrix
 * starts at gate_off + e*gate_stride, and so on. Result semantics follow
 * mlp_moe_forward (src/sepia.c:1377-1470). Requires an open batch. */
typedef struct {
    int64_t hidden, ff;
    int32_t n_routed, n_shared, topk;
    double route_scale;        /* double, as the reference reads it from the config (src/sepia.c:434) */
    float global_scale;
    SepiaGpuBuf *router_w; size_t router_w_off;       /* f32 [n_routed+n_shared, hidden] */
    SepiaGpuBuf *router_bias; size_t router_bias_off; /* f32 [n_routed] */
    int32_t gate_type, up_type, down_type;
    SepiaGpuBuf *experts; size_t gate_off, up_off, down_off;
    int64_t gate_stride, up_stride, down_stride;
    int32_t sh_gate_type, sh_up_type, sh_down_type;
    SepiaGpuBuf *shared; size_t sh_gate_off, sh_up_off, sh_down_off;
    int64_t sh_gate_stride, sh_up_stride, sh_down_stride;
} SepiaGpuMoeDesc;

/* out[hidden] = MoE(x[hidden]). Optional topk_idx (int32[topk]) and
 * weights (f32[topk+n_shared]) buffers receive the routing decision. */
int sepia_gpu_moe_layer(const SepiaGpuMoeDesc *d, SepiaGpuBuf *x, SepiaGpuBuf *out,
                        SepiaGpuBuf *topk_idx, SepiaGpuBuf *weights);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif
#ifdef __cplusplus
}
#endif
#endif
