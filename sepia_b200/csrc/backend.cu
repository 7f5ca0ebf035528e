// sepia_b200/csrc/backend.cu -- the reference GPU ABI (include/sepia_gpu.h,
// the 30 functions of rinaldofesta/sepia src/sepia_gpu.h) on CUDA.
//
// Functional model: src/sepia_metal.m (device init :103-160, buffers
// :184-298, batching :339-399, per-op dispatch :431-1085) re-designed for a
// discrete B200: Shared buffers are device memory with a pinned host
// mirror, synchronised at the batch boundaries the reference already has;
// a batch is the library stream; end() waits on an event under a watchdog
// and checks the device error word instead of blocking forever.
#include "../../include/sepia_cuda.h"
#include "../../include/sepia_gpu.h"
#include "runtime.h"

#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>
#include <unistd.h>

#include <algorithm>
#include <set>
#include <vector>

namespace sepia {
int launch_matvec_q(int t, const void *w, const float *x, float *y, int64_t out_dim, int64_t in_dim, int64_t n_vec,
                    cudaStream_t st);
int launch_dequant(int t, const void *raw, float *out, int64_t n, cudaStream_t st);
int op_rmsnorm(const float *w, const float *x, float *y, int64_t rows, int64_t n, float eps, cudaStream_t st);
int op_matvec_f32(const float *w, const float *x, float *y, int64_t out_dim, int64_t in_dim, cudaStream_t st);
int op_silu_mul(const float *g, const float *u, float *z, int64_t n, cudaStream_t st);
int op_add(const float *a, const float *b, float *o, int64_t n, cudaStream_t st);
int op_scale(float s, const float *x, float *y, int64_t n, cudaStream_t st);
int op_touch(float *x, int64_t n, cudaStream_t st);
int op_softmax(const float *x, float *y, int64_t rows, int64_t n, cudaStream_t st);
int op_sconv(const float *w, const float *hist, const float *in, float *out, int64_t C, int64_t K, int64_t T,
             cudaStream_t st);
int op_sconv_hist_roll(float *hist, const float *in, int64_t C, int64_t K, int64_t T, cudaStream_t st);
int launch_rel_project(const float *r_vec, const float *rel_proj, float *rel_logits, int64_t T, int64_t H,
                       int64_t d_rel, int64_t E, cudaStream_t st);
int launch_banded_attn(int kv_f16, const float *q, const void *k, const void *v, const float *rel_logits, float *out,
                       const int64_t *kv_lo_d, const int64_t *kv_hi_d, const float *tau_d, int64_t T, int64_t H,
                       int64_t Hkv, int64_t Dh, int64_t E, int64_t q_pos_base, int64_t kv_dim, float inv_head_dim,
                       int S, double *part, cudaStream_t st);
int attn_splits(int64_t T, int64_t Hkv, int64_t max_n);
size_t attn_part_bytes(int64_t T, int64_t H, int S, int64_t Dh);
}  // namespace sepia

using namespace sepia;

enum BufKind { kShared = 0, kPrivate = 1, kWrapped = 2 };

struct SepiaGpuBuf {
    void *dev = nullptr;
    void *host = nullptr;    // pinned mirror (Shared), caller mapping (Wrapped), NULL (Private)
    size_t len = 0;          // device bytes
    BufKind kind = kShared;
    bool dev_dirty = false;  // written by the GPU in the open batch
    bool synced = false;     // Shared: host mirror uploaded in the open batch
};

namespace {

struct Arena {   // bump allocator over device chunks, recycled at end()
    std::vector<std::pair<char *, size_t>> chunks;
    size_t cur = 0, off = 0;
    void *take(size_t n) {
        n = (n + 255) & ~(size_t)255;
        while (cur < chunks.size() && off + n > chunks[cur].second) { cur++; off = 0; }
        if (cur == chunks.size()) {
            size_t sz = n > ((size_t)64 << 20) ? n : ((size_t)64 << 20);
            char *p = nullptr;
            if (cudaMalloc(&p, sz) != cudaSuccess) return nullptr;
            chunks.push_back({p, sz});
            off = 0;
        }
        void *r = chunks[cur].first + off;
        off += n;
        return r;
    }
    void reset() { cur = 0; off = 0; }
    void release() {
        for (auto &c : chunks) cudaFree(c.first);
        chunks.clear();
        reset();
    }
};

struct HostArena {  // pinned staging for host arrays uploaded inside a batch
    std::vector<std::pair<char *, size_t>> chunks;
    size_t cur = 0, off = 0;
    void *take(size_t n) {
        n = (n + 63) & ~(size_t)63;
        while (cur < chunks.size() && off + n > chunks[cur].second) { cur++; off = 0; }
        if (cur == chunks.size()) {
            size_t sz = n > ((size_t)1 << 20) ? n : ((size_t)1 << 20);
            char *p = nullptr;
            if (cudaMallocHost(&p, sz) != cudaSuccess) return nullptr;
            chunks.push_back({p, sz});
            off = 0;
        }
        void *r = chunks[cur].first + off;
        off += n;
        return r;
    }
    void reset() { cur = 0; off = 0; }
    void release() {
        for (auto &c : chunks) cudaFreeHost(c.first);
        chunks.clear();
        reset();
    }
};

struct Backend {
    bool ready = false;
    int device = 0;
    char name[256] = {0};
    bool batch_open = false;
    cudaStream_t stream = nullptr;
    cudaEvent_t done = nullptr;
    unsigned *moe_counter = nullptr;   // the router's CTA counter (zeroed once; the router resets it)
    std::set<SepiaGpuBuf *> bufs;
    Arena arena;
    HostArena harena;
};

Backend g;

bool need_batch(const char *op) {
    if (!g.ready) { fail("%s: GPU not initialized", op); return false; }
    if (!g.batch_open) { fail("%s: no active batch (call sepia_gpu_begin first)", op); return false; }
    return true;
}

template <typename T = float>
T *dptr(SepiaGpuBuf *b, size_t off = 0) {
    return reinterpret_cast<T *>(static_cast<char *>(b->dev) + off);
}

// Bounds-checks a buffer argument of an op and, for a Shared buffer the
// batch has not touched yet, enqueues the upload of its host mirror first:
// the reference (unified memory) may fill a Shared buffer after
// sepia_gpu_begin(), right before the op that reads it (src/sepia.c:4941).
bool fits(SepiaGpuBuf *b, size_t off, size_t bytes, const char *op, const char *what) {
    if (!b || !b->dev) { fail("%s: %s buffer is NULL", op, what); return false; }
    if (off > b->len || bytes > b->len - off) {
        fail("%s: %s needs %zu bytes at offset %zu but the buffer holds %zu", op, what, bytes, off, b->len);
        return false;
    }
    if (b->kind == kShared && g.batch_open && !b->synced) {
        if (!check(cudaMemcpyAsync(b->dev, b->host, b->len, cudaMemcpyHostToDevice, g.stream), "upload Shared buffer"))
            return false;
        b->synced = true;
    }
    return true;
}

// An op's output that overwrites the whole of a Shared buffer: its mirror
// need not be uploaded first.
bool fits_out(SepiaGpuBuf *b, size_t bytes, const char *op, const char *what) {
    if (b && b->dev && b->kind == kShared && g.batch_open && !b->synced && bytes == b->len) {
        b->synced = true;
        return true;
    }
    return fits(b, 0, bytes, op, what);
}

void mark(SepiaGpuBuf *b) {
    if (b) { b->dev_dirty = true; b->synced = true; }
}

double now_s() {
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return ts.tv_sec + ts.tv_nsec * 1e-9;
}

// Wait for the stream under a deadline (SEPIA_CUDA_END_TIMEOUT_S, default
// 120 s): never blocks forever on a wedged kernel.
int wait_stream(const char *what) {
    if (!check(cudaEventRecord(g.done, g.stream), "cudaEventRecord")) return 0;
    double limit = 120.0;
    if (const char *e = getenv("SEPIA_CUDA_END_TIMEOUT_S")) limit = atof(e) > 0 ? atof(e) : limit;
    // spin for the first 2 ms (decode steps finish in tens of microseconds),
    // then back off to sleeping polls
    const double t0 = now_s();
    for (;;) {
        cudaError_t q = cudaEventQuery(g.done);
        if (q == cudaSuccess) break;
        if (q != cudaErrorNotReady) return check(q, what);
        const double el = now_s() - t0;
        if (el > limit) return fail("%s: device did not finish within %.0f s", what, limit);
        if (el > 2e-3) usleep(50);
    }
    DevInfo &di = dev_info();
    if (di.err) {
        int code = 0;
        if (!check(cudaMemcpy(&code, di.err, sizeof(int), cudaMemcpyDeviceToHost), "read device error word")) return 0;
        if (code) {
            cudaMemset(di.err, 0, sizeof(int));
            return fail("%s: a kernel reported device error %d (bounded wait expired)", what, code);
        }
    }
    return 1;
}

}  // namespace

// =========================================================== lifecycle
extern "C" int sepia_gpu_available(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) return 0;
    return n > 0 ? 1 : 0;
}

extern "C" int sepia_gpu_init(const char *metal_dir) {
    (void)metal_dir;
    if (g.ready) return 1;
    int n = 0;
    if (!check(cudaGetDeviceCount(&n), "cudaGetDeviceCount")) return 0;
    if (n <= 0) return fail("init: no CUDA device");
    if (!check(cudaGetDevice(&g.device), "cudaGetDevice")) return 0;
    cudaDeviceProp prop;
    if (!check(cudaGetDeviceProperties(&prop, g.device), "cudaGetDeviceProperties")) return 0;
    if (prop.major < 10) return fail("init: %s is sm_%d%d; this library is built for sm_100a", prop.name, prop.major, prop.minor);
    snprintf(g.name, sizeof g.name, "%s", prop.name);
    g.stream = lib_stream();
    if (!check(cudaEventCreateWithFlags(&g.done, cudaEventDisableTiming), "cudaEventCreate")) return 0;
    if (!check(cudaMalloc((void **)&g.moe_counter, 256), "init: cudaMalloc") ||
        !check(cudaMemset(g.moe_counter, 0, 256), "init: cudaMemset"))
        return 0;
    dev_info();
    g.ready = true;
    return 1;
}

extern "C" void sepia_gpu_shutdown(void) {
    if (!g.ready) return;
    if (g.batch_open) { cudaStreamSynchronize(g.stream); g.batch_open = false; }
    std::vector<SepiaGpuBuf *> live(g.bufs.begin(), g.bufs.end());
    for (SepiaGpuBuf *b : live) sepia_gpu_free(b);
    g.arena.release();
    g.harena.release();
    if (g.done) cudaEventDestroy(g.done);
    g.done = nullptr;
    if (g.moe_counter) cudaFree(g.moe_counter);
    g.moe_counter = nullptr;
    g.ready = false;
    g.name[0] = 0;
}

extern "C" const char *sepia_gpu_device_name(void) { return g.ready ? g.name : nullptr; }

// ============================================================= buffers
extern "C" SepiaGpuBuf *sepia_gpu_wrap_mmap(void *base, size_t len) {
    if (!g.ready) { fail("wrap_mmap: GPU not initialized"); return nullptr; }
    if (!base || len == 0) { fail("wrap_mmap: invalid base/len"); return nullptr; }
    const size_t page = (size_t)sysconf(_SC_PAGESIZE);
    if ((uintptr_t)base % page) { fail("wrap_mmap: base %p is not page-aligned (page=%zu)", base, page); return nullptr; }
    const size_t rounded = (len + page - 1) & ~(page - 1);
    SepiaGpuBuf *b = new SepiaGpuBuf;
    b->kind = kWrapped;
    b->host = base;
    b->len = rounded;
    if (!check(cudaMalloc(&b->dev, rounded), "wrap_mmap: cudaMalloc") ||
        !check(cudaMemcpy(b->dev, base, rounded, cudaMemcpyHostToDevice), "wrap_mmap: upload")) {
        if (b->dev) cudaFree(b->dev);
        delete b;
        return nullptr;
    }
    g.bufs.insert(b);
    return b;
}

extern "C" SepiaGpuBuf *sepia_gpu_alloc(size_t len, int gpu_private) {
    if (!g.ready) { fail("alloc: GPU not initialized"); return nullptr; }
    if (len == 0) { fail("alloc: zero length"); return nullptr; }
    SepiaGpuBuf *b = new SepiaGpuBuf;
    b->kind = gpu_private ? kPrivate : kShared;
    b->len = len;
    if (!check(cudaMalloc(&b->dev, len), "alloc: cudaMalloc")) { delete b; return nullptr; }
    if (!gpu_private) {
        if (!check(cudaMallocHost(&b->host, len), "alloc: cudaMallocHost")) {
            cudaFree(b->dev);
            delete b;
            return nullptr;
        }
        memset(b->host, 0, len);
    }
    cudaMemset(b->dev, 0, len);
    g.bufs.insert(b);
    return b;
}

extern "C" void sepia_gpu_free(SepiaGpuBuf *b) {
    if (!b) return;
    if (g.bufs.erase(b) == 0) return;   // not ours / already freed
    if (g.batch_open) cudaStreamSynchronize(g.stream);   // the open batch may still read it
    if (b->dev) cudaFree(b->dev);
    if (b->kind == kShared && b->host) cudaFreeHost(b->host);
    delete b;
}

extern "C" void *sepia_gpu_host_ptr(SepiaGpuBuf *b) {
    if (!b || b->kind == kPrivate) return nullptr;
    return b->host;
}

extern "C" uint64_t sepia_gpu_gpu_addr(SepiaGpuBuf *b) { return b ? (uint64_t)(uintptr_t)b->dev : 0; }

extern "C" int sepia_gpu_selftest_touch(SepiaGpuBuf *b, size_t n_floats) {
    if (!g.ready) return fail("selftest_touch: GPU not initialized");
    if (!fits(b, 0, n_floats * 4, "selftest_touch", "buf")) return 0;
    if (n_floats == 0) return 1;
    if (b->host && !check(cudaMemcpyAsync(b->dev, b->host, n_floats * 4, cudaMemcpyHostToDevice, g.stream), "touch upload"))
        return 0;
    if (!op_touch(dptr(b), (int64_t)n_floats, g.stream)) return 0;
    if (b->host && !check(cudaMemcpyAsync(b->host, b->dev, n_floats * 4, cudaMemcpyDeviceToHost, g.stream), "touch download"))
        return 0;
    return wait_stream("selftest_touch");
}

// ============================================================ batching
extern "C" int sepia_gpu_begin(void) {
    if (!g.ready) return fail("begin: GPU not initialized");
    if (g.batch_open) return fail("begin: a batch is already active");
    // Shared buffers are uploaded lazily, by the first op of the batch that
    // names them (see fits()).
    for (SepiaGpuBuf *b : g.bufs) {
        b->dev_dirty = false;
        b->synced = false;
    }
    g.batch_open = true;
    return 1;
}

extern "C" int sepia_gpu_flush(void) {
    if (!g.batch_open) return fail("flush: no active batch");
    // Work is already queued on the stream in order; nothing to commit.
    return 1;
}

extern "C" int sepia_gpu_end(void) {
    if (!g.batch_open) return fail("end: no active batch");
    g.batch_open = false;
    int ok = 1;
    for (SepiaGpuBuf *b : g.bufs) {
        if (b->dev_dirty && b->host && b->kind != kPrivate)
            ok &= check(cudaMemcpyAsync(b->host, b->dev, b->len, cudaMemcpyDeviceToHost, g.stream), "end: download");
        b->dev_dirty = false;
        b->synced = false;
    }
    ok &= wait_stream("end");
    g.arena.reset();
    g.harena.reset();
    return ok;
}

// ================================================================= ops
extern "C" int sepia_gpu_rmsnorm(SepiaGpuBuf *w, SepiaGpuBuf *x, SepiaGpuBuf *y, int64_t rows, int64_t n, float eps) {
    return sepia_gpu_rmsnorm_off(w, 0, x, y, rows, n, eps);
}

extern "C" int sepia_gpu_rmsnorm_off(SepiaGpuBuf *w, size_t w_off, SepiaGpuBuf *x, SepiaGpuBuf *y, int64_t rows,
                                     int64_t n, float eps) {
    if (!need_batch("rmsnorm")) return 0;
    if (rows <= 0 || n <= 0) return fail("rmsnorm: bad dims rows=%lld n=%lld", (long long)rows, (long long)n);
    const size_t rb = (size_t)rows * (size_t)n * 4;
    if (!fits(w, w_off, (size_t)n * 4, "rmsnorm", "w") || !fits(x, 0, rb, "rmsnorm", "x") || !fits(y, 0, rb, "rmsnorm", "y"))
        return 0;
    if (!op_rmsnorm(dptr(w, w_off), dptr(x), dptr(y), rows, n, eps, g.stream)) return 0;
    mark(y);
    return 1;
}

extern "C" int sepia_gpu_matvec(SepiaGpuBuf *w, SepiaGpuBuf *x, SepiaGpuBuf *y, int64_t out_dim, int64_t in_dim) {
    return sepia_gpu_matvec_off(w, 0, x, y, out_dim, in_dim);
}

extern "C" int sepia_gpu_matvec_off(SepiaGpuBuf *w, size_t w_off, SepiaGpuBuf *x, SepiaGpuBuf *y, int64_t out_dim,
                                    int64_t in_dim) {
    if (!need_batch("matvec")) return 0;
    if (out_dim <= 0 || in_dim <= 0) return fail("matvec: bad dims");
    if (!fits(w, w_off, (size_t)out_dim * (size_t)in_dim * 4, "matvec", "w") ||
        !fits(x, 0, (size_t)in_dim * 4, "matvec", "x") || !fits(y, 0, (size_t)out_dim * 4, "matvec", "y"))
        return 0;
    if (w_off % 4) return fail("matvec: w_off %zu not 4-byte aligned", w_off);
    if (!op_matvec_f32(dptr(w, w_off), dptr(x), dptr(y), out_dim, in_dim, g.stream)) return 0;
    mark(y);
    return 1;
}

extern "C" int sepia_gpu_silu_mul(SepiaGpuBuf *gb, SepiaGpuBuf *u, SepiaGpuBuf *z, int64_t n) {
    if (!need_batch("silu_mul")) return 0;
    const size_t nb = (size_t)(n > 0 ? n : 0) * 4;
    if (!fits(gb, 0, nb, "silu_mul", "g") || !fits(u, 0, nb, "silu_mul", "u") || !fits(z, 0, nb, "silu_mul", "z")) return 0;
    if (!op_silu_mul(dptr(gb), dptr(u), dptr(z), n, g.stream)) return 0;
    mark(z);
    return 1;
}

extern "C" int sepia_gpu_add(SepiaGpuBuf *a, SepiaGpuBuf *b, SepiaGpuBuf *out, int64_t n) {
    if (!need_batch("add")) return 0;
    const size_t nb = (size_t)(n > 0 ? n : 0) * 4;
    if (!fits(a, 0, nb, "add", "a") || !fits(b, 0, nb, "add", "b") || !fits(out, 0, nb, "add", "out")) return 0;
    if (!op_add(dptr(a), dptr(b), dptr(out), n, g.stream)) return 0;
    mark(out);
    return 1;
}

extern "C" int sepia_gpu_softmax(SepiaGpuBuf *x, SepiaGpuBuf *y, int64_t rows, int64_t n) {
    if (!need_batch("softmax")) return 0;
    const size_t nb = (size_t)(rows > 0 ? rows : 0) * (size_t)(n > 0 ? n : 0) * 4;
    if (!fits(x, 0, nb, "softmax", "x") || !fits(y, 0, nb, "softmax", "y")) return 0;
    if (!op_softmax(dptr(x), dptr(y), rows, n, g.stream)) return 0;
    mark(y);
    return 1;
}

extern "C" int sepia_gpu_sconv(SepiaGpuBuf *w, SepiaGpuBuf *hist, SepiaGpuBuf *in, SepiaGpuBuf *out, int64_t C,
                               int64_t K, int64_t T) {
    return sepia_gpu_sconv_off(w, 0, hist, in, out, C, K, T);
}

extern "C" int sepia_gpu_sconv_off(SepiaGpuBuf *w, size_t w_off, SepiaGpuBuf *hist, SepiaGpuBuf *in, SepiaGpuBuf *out,
                                   int64_t C, int64_t K, int64_t T) {
    if (!need_batch("sconv")) return 0;
    if (C <= 0 || K <= 0 || T <= 0) return fail("sconv: bad dims");
    const size_t tb = (size_t)C * (size_t)T * 4;
    if (!fits(w, w_off, (size_t)C * (size_t)K * 4, "sconv", "w") || !fits(in, 0, tb, "sconv", "in") ||
        !fits(out, 0, tb, "sconv", "out"))
        return 0;
    if (K > 1 && !fits(hist, 0, (size_t)(K - 1) * (size_t)C * 4, "sconv", "hist")) return 0;
    if (!op_sconv(dptr(w, w_off), K > 1 ? dptr(hist) : nullptr, dptr(in), dptr(out), C, K, T, g.stream)) return 0;
    mark(out);
    return 1;
}

extern "C" int sepia_gpu_matvec_q(int ggml_type, SepiaGpuBuf *w, size_t w_off, SepiaGpuBuf *x, SepiaGpuBuf *y,
                                  int64_t out_dim, int64_t in_dim) {
    if (!need_batch("matvec_q")) return 0;
    const int64_t rb = host_row_bytes(ggml_type, in_dim);
    if (rb <= 0 || out_dim <= 0)
        return fail("matvec_q: unsupported ggml type %d or bad dims out=%lld in=%lld", ggml_type, (long long)out_dim,
                    (long long)in_dim);
    if (!fits(w, w_off, (size_t)rb * (size_t)out_dim, "matvec_q", "w") || !fits(x, 0, (size_t)in_dim * 4, "matvec_q", "x") ||
        !fits(y, 0, (size_t)out_dim * 4, "matvec_q", "y"))
        return 0;
    if (!launch_matvec_q(ggml_type, dptr<char>(w, w_off), dptr(x), dptr(y), out_dim, in_dim, 1, g.stream)) return 0;
    mark(y);
    return 1;
}

extern "C" int sepia_gpu_dequant_rows(int ggml_type, SepiaGpuBuf *raw, size_t raw_off, SepiaGpuBuf *out, int64_t n) {
    if (!need_batch("dequant_rows")) return 0;
    const int64_t rb = host_row_bytes(ggml_type, n);
    if (rb <= 0) return fail("dequant_rows: unsupported ggml type %d or n=%lld not block-aligned", ggml_type, (long long)n);
    if (!fits(raw, raw_off, (size_t)rb, "dequant_rows", "raw") || !fits(out, 0, (size_t)n * 4, "dequant_rows", "out"))
        return 0;
    if (!launch_dequant(ggml_type, dptr<char>(raw, raw_off), dptr(out), n, g.stream)) return 0;
    mark(out);
    return 1;
}

extern "C" int sepia_gpu_rel_project(SepiaGpuBuf *r_vec, SepiaGpuBuf *rel_proj, SepiaGpuBuf *rel_logits, int64_t T,
                                     int64_t H, int64_t d_rel, int64_t rel_extent) {
    return sepia_gpu_rel_project_off(r_vec, rel_proj, 0, rel_logits, T, H, d_rel, rel_extent);
}

extern "C" int sepia_gpu_rel_project_off(SepiaGpuBuf *r_vec, SepiaGpuBuf *rel_proj, size_t rel_proj_off,
                                         SepiaGpuBuf *rel_logits, int64_t T, int64_t H, int64_t d_rel,
                                         int64_t rel_extent) {
    if (!need_batch("rel_project")) return 0;
    if (T <= 0 || H <= 0 || d_rel <= 0 || rel_extent <= 0) return fail("rel_project: bad dims");
    if (!fits(r_vec, 0, (size_t)T * H * d_rel * 4, "rel_project", "r_vec") ||
        !fits(rel_proj, rel_proj_off, (size_t)d_rel * rel_extent * 4, "rel_project", "rel_proj") ||
        !fits(rel_logits, 0, (size_t)T * H * rel_extent * 4, "rel_project", "rel_logits"))
        return 0;
    if (!launch_rel_project(dptr(r_vec), dptr(rel_proj, rel_proj_off), dptr(rel_logits), T, H, d_rel, rel_extent,
                            g.stream))
        return 0;
    mark(rel_logits);
    return 1;
}

extern "C" int sepia_gpu_banded_attn(SepiaGpuBuf *q, SepiaGpuBuf *k, SepiaGpuBuf *v, SepiaGpuBuf *rel_logits,
                                     SepiaGpuBuf *attn_out, const int64_t *kv_lo, const int64_t *kv_hi, const float *tau,
                                     int64_t T, int64_t H, int64_t Hkv, int64_t Dh, int64_t rel_extent,
                                     int64_t q_pos_base, int64_t kv_dim, float inv_head_dim) {
    if (!need_batch("banded_attn")) return 0;
    if (T <= 0 || H <= 0 || Hkv <= 0 || Dh <= 0 || !kv_lo || !kv_hi || !tau) return fail("banded_attn: bad arguments");
    if (Dh > 128) return fail("banded_attn: Dh=%lld exceeds 128", (long long)Dh);
    int64_t max_n = 1, max_hi = 0;
    for (int64_t t = 0; t < T; t++) {
        if (kv_lo[t] < 0 || kv_hi[t] < kv_lo[t]) return fail("banded_attn: bad kv range at t=%lld", (long long)t);
        max_n = std::max<int64_t>(max_n, kv_hi[t] - kv_lo[t] + 1);
        max_hi = std::max<int64_t>(max_hi, kv_hi[t]);
    }
    const size_t cache_bytes = (size_t)(max_hi + 1) * (size_t)kv_dim * 4;
    if (!fits(q, 0, (size_t)T * H * Dh * 4, "banded_attn", "q") || !fits(k, 0, cache_bytes, "banded_attn", "k") ||
        !fits(v, 0, cache_bytes, "banded_attn", "v") || !fits(attn_out, 0, (size_t)T * H * Dh * 4, "banded_attn", "out") ||
        (rel_extent > 0 && !fits(rel_logits, 0, (size_t)T * H * rel_extent * 4, "banded_attn", "rel_logits")))
        return 0;
    // host arrays -> pinned staging -> device (stream-ordered)
    const size_t nb64 = (size_t)T * 8, nb32 = (size_t)T * 4;
    char *hs = (char *)g.harena.take(2 * nb64 + nb32);
    char *ds = (char *)g.arena.take(2 * nb64 + nb32);
    if (!hs || !ds) return fail("banded_attn: out of staging memory");
    memcpy(hs, kv_lo, nb64);
    memcpy(hs + nb64, kv_hi, nb64);
    memcpy(hs + 2 * nb64, tau, nb32);
    if (!check(cudaMemcpyAsync(ds, hs, 2 * nb64 + nb32, cudaMemcpyHostToDevice, g.stream), "banded_attn upload")) return 0;
    const int S = attn_splits(T, Hkv, max_n);
    double *part = (double *)g.arena.take(attn_part_bytes(T, H, S, Dh));
    if (!part) return fail("banded_attn: out of scratch memory");
    if (!launch_banded_attn(0, dptr(q), dptr(k), dptr(v), rel_extent > 0 ? dptr(rel_logits) : nullptr, dptr(attn_out),
                            (const int64_t *)ds, (const int64_t *)(ds + nb64), (const float *)(ds + 2 * nb64), T, H, Hkv,
                            Dh, rel_extent, q_pos_base, kv_dim, inv_head_dim, S, part, g.stream))
        return 0;
    mark(attn_out);
    return 1;
}

extern "C" int sepia_gpu_copy(SepiaGpuBuf *src, size_t src_off, SepiaGpuBuf *dst, size_t dst_off, int64_t n) {
    if (!need_batch("copy")) return 0;
    if (n < 0) return fail("copy: negative n");
    const size_t nb = (size_t)n * 4;
    if (!fits(src, src_off, nb, "copy", "src") || !fits(dst, dst_off, nb, "copy", "dst")) return 0;
    if (nb && !check(cudaMemcpyAsync(dptr<char>(dst, dst_off), dptr<char>(src, src_off), nb, cudaMemcpyDeviceToDevice,
                                     g.stream),
                     "copy"))
        return 0;
    mark(dst);
    return 1;
}

extern "C" int sepia_gpu_scale(float scale, SepiaGpuBuf *x, SepiaGpuBuf *y, int64_t n) {
    if (!need_batch("scale")) return 0;
    const size_t nb = (size_t)(n > 0 ? n : 0) * 4;
    if (!fits(x, 0, nb, "scale", "x") || !fits(y, 0, nb, "scale", "y")) return 0;
    if (!op_scale(scale, dptr(x), dptr(y), n, g.stream)) return 0;
    mark(y);
    return 1;
}

extern "C" int sepia_gpu_sconv_hist_roll(SepiaGpuBuf *hist, SepiaGpuBuf *in, int64_t C, int64_t K, int64_t T) {
    if (!need_batch("sconv_hist_roll")) return 0;
    if (C <= 0 || K <= 0 || T <= 0) return fail("sconv_hist_roll: bad dims");
    if (K - 1 > 15) return fail("sconv_hist_roll: K-1 = %lld exceeds 15", (long long)(K - 1));
    if (!fits(in, 0, (size_t)C * T * 4, "sconv_hist_roll", "in") ||
        (K > 1 && !fits(hist, 0, (size_t)(K - 1) * C * 4, "sconv_hist_roll", "hist")))
        return 0;
    if (!op_sconv_hist_roll(K > 1 ? dptr(hist) : nullptr, dptr(in), C, K, T, g.stream)) return 0;
    mark(hist);
    return 1;
}

// ------------------------------------------------- extension: MoE layer
extern "C" int sepia_gpu_moe_layer(const SepiaGpuMoeDesc *d, SepiaGpuBuf *x, SepiaGpuBuf *out, SepiaGpuBuf *topk_idx,
                                   SepiaGpuBuf *weights) {
    if (!need_batch("moe_layer")) return 0;
    if (!d || !d->router_w || !d->router_bias || !d->experts || (d->n_shared > 0 && !d->shared))
        return fail("moe_layer: incomplete descriptor");
    if (!fits(x, 0, (size_t)d->hidden * 4, "moe_layer", "x") || !fits_out(out, (size_t)d->hidden * 4, "moe_layer", "out"))
        return 0;
    SepiaMoeLayer L;
    memset(&L, 0, sizeof L);
    L.hidden = d->hidden; L.ff = d->ff;
    L.n_routed = d->n_routed; L.n_shared = d->n_shared; L.topk = d->topk;
    L.route_scale = d->route_scale; L.global_scale = d->global_scale;
    if (!fits(d->router_w, d->router_w_off, (size_t)(d->n_routed + d->n_shared) * d->hidden * 4, "moe_layer", "router_w") ||
        !fits(d->router_bias, d->router_bias_off, (size_t)d->n_routed * 4, "moe_layer", "router_bias"))
        return 0;
    L.router_w = dptr(d->router_w, d->router_w_off);
    L.router_bias = dptr(d->router_bias, d->router_bias_off);
    L.gate_type = d->gate_type; L.up_type = d->up_type; L.down_type = d->down_type;
    const int64_t rbg = host_row_bytes(d->gate_type, d->hidden), rbu = host_row_bytes(d->up_type, d->hidden);
    const int64_t rbd = host_row_bytes(d->down_type, d->ff);
    if (rbg <= 0 || rbu <= 0 || rbd <= 0) return fail("moe_layer: unsupported routed expert types");
    const size_t last = (size_t)(d->n_routed - 1);
    if (!fits(d->experts, d->gate_off + last * d->gate_stride, (size_t)rbg * d->ff, "moe_layer", "gate") ||
        !fits(d->experts, d->up_off + last * d->up_stride, (size_t)rbu * d->ff, "moe_layer", "up") ||
        !fits(d->experts, d->down_off + last * d->down_stride, (size_t)rbd * d->hidden, "moe_layer", "down"))
        return 0;
    L.gate = dptr<char>(d->experts, d->gate_off); L.up = dptr<char>(d->experts, d->up_off);
    L.down = dptr<char>(d->experts, d->down_off);
    L.gate_stride = d->gate_stride; L.up_stride = d->up_stride; L.down_stride = d->down_stride;
    L.sh_gate_type = d->sh_gate_type; L.sh_up_type = d->sh_up_type; L.sh_down_type = d->sh_down_type;
    if (d->n_shared > 0) {
        const int64_t sg = host_row_bytes(d->sh_gate_type, d->hidden), su = host_row_bytes(d->sh_up_type, d->hidden);
        const int64_t sd = host_row_bytes(d->sh_down_type, d->ff);
        if (sg <= 0 || su <= 0 || sd <= 0) return fail("moe_layer: unsupported shared expert types");
        const size_t ls = (size_t)(d->n_shared - 1);
        if (!fits(d->shared, d->sh_gate_off + ls * d->sh_gate_stride, (size_t)sg * d->ff, "moe_layer", "shared gate") ||
            !fits(d->shared, d->sh_up_off + ls * d->sh_up_stride, (size_t)su * d->ff, "moe_layer", "shared up") ||
            !fits(d->shared, d->sh_down_off + ls * d->sh_down_stride, (size_t)sd * d->hidden, "moe_layer", "shared down"))
            return 0;
        L.sh_gate = dptr<char>(d->shared, d->sh_gate_off); L.sh_up = dptr<char>(d->shared, d->sh_up_off);
        L.sh_down = dptr<char>(d->shared, d->sh_down_off);
        L.sh_gate_stride = d->sh_gate_stride; L.sh_up_stride = d->sh_up_stride; L.sh_down_stride = d->sh_down_stride;
    }
    L.rank = 0; L.world = 1; L.expert_slot = nullptr;
    const size_t wb = sepia_cuda_moe_work_bytes(&L);
    void *wsmem = g.arena.take(wb);
    if (!wsmem) return fail("moe_layer: out of scratch memory");
    SepiaMoeWork ws;
    if (!sepia_cuda_moe_work_carve(&L, wsmem, wb, &ws)) return 0;
    // the kernel chain below uses only the router's CTA counter: a
    // persistent one, zero between calls (the router's last CTA resets it),
    // so no clearing op precedes the router (calls are serialised on the
    // backend's one stream)
    ws.counter = g.moe_counter;
    if (!sepia_cuda_moe_layer(&L, dptr(x), &ws, dptr(out), g.stream)) return 0;
    mark(out);
    if (topk_idx) {
        if (!fits(topk_idx, 0, (size_t)d->topk * 4, "moe_layer", "topk_idx")) return 0;
        if (!check(cudaMemcpyAsync(topk_idx->dev, ws.topk_idx, (size_t)d->topk * 4, cudaMemcpyDeviceToDevice, g.stream), "copy idx"))
            return 0;
        mark(topk_idx);
    }
    if (weights) {
        const size_t nb = (size_t)(d->topk + d->n_shared) * 4;
        if (!fits(weights, 0, nb, "moe_layer", "weights")) return 0;
        if (!check(cudaMemcpyAsync(weights->dev, ws.weights, nb, cudaMemcpyDeviceToDevice, g.stream), "copy weights"))
            return 0;
        mark(weights);
    }
    return 1;
}

// ----------------------------------------------------- runtime extras
extern "C" const char *sepia_cuda_last_error(void);
extern "C" int sepia_cuda_sm_count(void) { return dev_info().sm_count; }
extern "C" int sepia_cuda_block_elems(int t) { return host_block_elems(t); }
extern "C" int sepia_cuda_block_bytes(int t) { return host_block_bytes(t); }
extern "C" int64_t sepia_cuda_row_bytes(int t, int64_t n) { return host_row_bytes(t, n); }

extern "C" int sepia_cuda_device_error(void *stream) {
    cudaStream_t st = as_stream(stream);
    if (cudaStreamSynchronize(st) != cudaSuccess) return -1;
    DevInfo &di = dev_info();
    if (!di.err) return 0;
    int code = 0;
    if (cudaMemcpy(&code, di.err, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return -1;
    if (code) cudaMemset(di.err, 0, sizeof(int));
    return code;
}
