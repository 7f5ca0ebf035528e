/* oracle/ref_gpu_noop.c -- TEST INFRASTRUCTURE ONLY.
 * Inert definitions of the 30 GPU-ABI symbols so the reference's CPU code
 * (oracle/ref_shim.c) links without any GPU backend. Every call reports
 * "unavailable" the way the reference's non-Darwin stub does. */
#include <stddef.h>
#include <stdint.h>
typedef struct SepiaGpuBuf SepiaGpuBuf;
int sepia_gpu_available(void) { return 0; }
int sepia_gpu_init(const char *d) { (void)d; return 0; }
void sepia_gpu_shutdown(void) {}
const char *sepia_gpu_device_name(void) { return NULL; }
SepiaGpuBuf *sepia_gpu_wrap_mmap(void *b, size_t n) { (void)b; (void)n; return NULL; }
SepiaGpuBuf *sepia_gpu_alloc(size_t n, int p) { (void)n; (void)p; return NULL; }
void sepia_gpu_free(SepiaGpuBuf *b) { (void)b; }
void *sepia_gpu_host_ptr(SepiaGpuBuf *b) { (void)b; return NULL; }
uint64_t sepia_gpu_gpu_addr(SepiaGpuBuf *b) { (void)b; return 0; }
int sepia_gpu_selftest_touch(SepiaGpuBuf *b, size_t n) { (void)b; (void)n; return 0; }
int sepia_gpu_begin(void) { return 0; }
int sepia_gpu_flush(void) { return 0; }
int sepia_gpu_end(void) { return 0; }
#define NOOP(name, ...) int name(__VA_ARGS__) { return 0; }
NOOP(sepia_gpu_rmsnorm, SepiaGpuBuf *w, SepiaGpuBuf *x, SepiaGpuBuf *y, int64_t r, int64_t n, float e)
NOOP(sepia_gpu_matvec, SepiaGpuBuf *w, SepiaGpuBuf *x, SepiaGpuBuf *y, int64_t o, int64_t i)
NOOP(sepia_gpu_silu_mul, SepiaGpuBuf *g, SepiaGpuBuf *u, SepiaGpuBuf *z, int64_t n)
NOOP(sepia_gpu_add, SepiaGpuBuf *a, SepiaGpuBuf *b, SepiaGpuBuf *o, int64_t n)
NOOP(sepia_gpu_softmax, SepiaGpuBuf *x, SepiaGpuBuf *y, int64_t r, int64_t n)
NOOP(sepia_gpu_sconv, SepiaGpuBuf *w, SepiaGpuBuf *h, SepiaGpuBuf *i, SepiaGpuBuf *o, int64_t C, int64_t K, int64_t T)
NOOP(sepia_gpu_matvec_q, int t, SepiaGpuBuf *w, size_t wo, SepiaGpuBuf *x, SepiaGpuBuf *y, int64_t o, int64_t i)
NOOP(sepia_gpu_dequant_rows, int t, SepiaGpuBuf *r, size_t ro, SepiaGpuBuf *o, int64_t n)
NOOP(sepia_gpu_rel_project, SepiaGpuBuf *r, SepiaGpuBuf *p, SepiaGpuBuf *l, int64_t T, int64_t H, int64_t d, int64_t e)
NOOP(sepia_gpu_banded_attn, SepiaGpuBuf *q, SepiaGpuBuf *k, SepiaGpuBuf *v, SepiaGpuBuf *rl, SepiaGpuBuf *o,
     const int64_t *lo, const int64_t *hi, const float *tau, int64_t T, int64_t H, int64_t Hkv, int64_t Dh,
     int64_t e, int64_t b, int64_t kd, float ih)
NOOP(sepia_gpu_matvec_off, SepiaGpuBuf *w, size_t wo, SepiaGpuBuf *x, SepiaGpuBuf *y, int64_t o, int64_t i)
NOOP(sepia_gpu_rmsnorm_off, SepiaGpuBuf *w, size_t wo, SepiaGpuBuf *x, SepiaGpuBuf *y, int64_t r, int64_t n, float e)
NOOP(sepia_gpu_sconv_off, SepiaGpuBuf *w, size_t wo, SepiaGpuBuf *h, SepiaGpuBuf *i, SepiaGpuBuf *o, int64_t C, int64_t K, int64_t T)
NOOP(sepia_gpu_rel_project_off, SepiaGpuBuf *r, SepiaGpuBuf *p, size_t po, SepiaGpuBuf *l, int64_t T, int64_t H, int64_t d, int64_t e)
NOOP(sepia_gpu_copy, SepiaGpuBuf *s, size_t so, SepiaGpuBuf *d, size_t dof, int64_t n)
int sepia_gpu_scale(float s, SepiaGpuBuf *x, SepiaGpuBuf *y, int64_t n) { (void)s; (void)x; (void)y; (void)n; return 0; }
NOOP(sepia_gpu_sconv_hist_roll, SepiaGpuBuf *h, SepiaGpuBuf *i, int64_t C, int64_t K, int64_t T)
