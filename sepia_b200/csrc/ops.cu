// sepia_b200/csrc/ops.cu -- the f32 ops of the GPU ABI (src/sepia_gpu.h:
// 102-128, 249-285; Metal twins in metal/ops.metal). Reductions accumulate
// in double like the CPU reference (src/sepia.c:720-740, 801-816), so
// results sit within a rounding of the reference rather than within the
// looser f32-accumulation gap the Metal kernels have.
#include "../../include/sepia_cuda.h"
#include "runtime.h"
#include "common.cuh"

namespace sepia {

constexpr int kRowThreads = 256;

__device__ __forceinline__ double block_sum_d(double v, double *sh) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    v = warp_sum_d(v);
    if (lane == 0) sh[warp] = v;
    __syncthreads();
    double t = 0.0;
    if (warp == 0) {
        t = (lane < (int)(blockDim.x >> 5)) ? sh[lane] : 0.0;
        t = warp_sum_d(t);
        if (lane == 0) sh[0] = t;
    }
    __syncthreads();
    t = sh[0];
    __syncthreads();
    return t;
}

// y[r,i] = w[i] * (x[r,i] * (1/sqrtf(mean(x^2)+eps)))   (src/sepia.c:720-729)
__global__ void k_rmsnorm(const float *w, const float *x, float *y, int64_t n, float eps) {
    __shared__ double sh[32];
    const float *xr = x + (int64_t)blockIdx.x * n;
    float *yr = y + (int64_t)blockIdx.x * n;
    double acc = 0.0;
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
        const float v = xr[i];
        acc += (double)__fmul_rn(v, v);
    }
    acc = block_sum_d(acc, sh);
    const float var = (float)(acc / (double)n);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) yr[i] = __fmul_rn(w[i], __fmul_rn(xr[i], inv));
}

// y[o] = dot(w[o,:], x), double accumulation; one warp per row.
__global__ void k_matvec_f32(const float *w, const float *x, float *y, int64_t out_dim, int64_t in_dim) {
    const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= out_dim) return;
    const float *wr = w + row * in_dim;
    double acc = 0.0;
    const bool vec = ((reinterpret_cast<uintptr_t>(wr) | reinterpret_cast<uintptr_t>(x)) & 15) == 0;
    const int64_t n4 = vec ? in_dim / 4 : 0;
    for (int64_t i = lane; i < n4; i += 32) {
        const float4 a = __ldg(reinterpret_cast<const float4 *>(wr) + i);
        const float4 b = __ldg(reinterpret_cast<const float4 *>(x) + i);
        acc = fma((double)a.x, (double)b.x, acc);
        acc = fma((double)a.y, (double)b.y, acc);
        acc = fma((double)a.z, (double)b.z, acc);
        acc = fma((double)a.w, (double)b.w, acc);
    }
    for (int64_t i = n4 * 4 + lane; i < in_dim; i += 32) acc = fma((double)wr[i], (double)x[i], acc);
    acc = warp_sum_d(acc);
    if (lane == 0) y[row] = (float)acc;
}

// z = silu(g) * u with silu(v) = v * (1/(1+expf(-v)))   (src/sepia.c:755-756)
__global__ void k_silu_mul(const float *g, const float *u, float *z, int64_t n) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    griddep_wait();
    griddep_launch();
    if (i >= n) return;
    const float gv = g[i];
    const float sig = __fdiv_rn(1.0f, __fadd_rn(1.0f, (float)exp(-(double)gv)));
    z[i] = __fmul_rn(__fmul_rn(gv, sig), u[i]);
}

__global__ void k_add(const float *a, const float *b, float *o, int64_t n) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) o[i] = __fadd_rn(a[i], b[i]);
}

__global__ void k_scale(float s, const float *x, float *y, int64_t n) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) y[i] = __fmul_rn(x[i], s);
}

__global__ void k_touch(float *x, int64_t n) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) x[i] += 0.0f;
}

// Row softmax: max, exp in double, normalise (src/sepia.c:1232-1245).
__global__ void k_softmax(const float *x, float *y, int64_t n) {
    __shared__ double sh[32];
    __shared__ float shm[32];
    const float *xr = x + (int64_t)blockIdx.x * n;
    float *yr = y + (int64_t)blockIdx.x * n;
    float m = -INFINITY;
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) m = fmaxf(m, xr[i]);
    m = warp_max(m);
    if ((threadIdx.x & 31) == 0) shm[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x < 32) {
        float t = (threadIdx.x < (blockDim.x >> 5)) ? shm[threadIdx.x] : -INFINITY;
        t = warp_max(t);
        if (threadIdx.x == 0) shm[0] = t;
    }
    __syncthreads();
    m = shm[0];
    double s = 0.0;
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
        const double e = exp((double)__fsub_rn(xr[i], m));
        s += e;
    }
    s = block_sum_d(s, sh);
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
        const double e = exp((double)__fsub_rn(xr[i], m));
        yr[i] = (float)((double)(float)e / s);
    }
}

// out[t,c] = in[t,c] + sum_k w[c,k] * window[t+k,c], window = hist ++ in.
__global__ void k_sconv(const float *w, const float *hist, const float *in, float *out, int64_t C, int64_t K,
                        int64_t T) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= C * T) return;
    const int64_t t = i / C, c = i % C, Km1 = K - 1;
    double acc = 0.0;
    for (int64_t k = 0; k < K; k++) {
        const int64_t j = t + k;
        const float v = (j < Km1) ? hist[j * C + c] : in[(j - Km1) * C + c];
        acc = fma((double)w[c * K + k], (double)v, acc);
    }
    out[i] = __fadd_rn(in[i], (float)acc);
}

// hist <- last K-1 rows of (hist ++ in), per channel (src/sepia.c:814).
__global__ void k_sconv_hist_roll(float *hist, const float *in, int64_t C, int64_t K, int64_t T) {
    const int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= C) return;
    const int64_t Km1 = K - 1;
    float keep[16];
    for (int64_t j = 0; j < Km1; j++) {
        const int64_t src = T + j;   // row of the concatenated window
        keep[j] = (src < Km1) ? hist[src * C + c] : in[(src - Km1) * C + c];
    }
    for (int64_t j = 0; j < Km1; j++) hist[j * C + c] = keep[j];
}

static inline unsigned blocks_for(int64_t n, int t) { return (unsigned)((n + t - 1) / t); }

int op_rmsnorm(const float *w, const float *x, float *y, int64_t rows, int64_t n, float eps, cudaStream_t st) {
    if (rows <= 0 || n <= 0 || !w || !x || !y) return fail("rmsnorm: bad arguments");
    k_rmsnorm<<<(unsigned)rows, kRowThreads, 0, st>>>(w, x, y, n, eps);
    return check(cudaGetLastError(), "rmsnorm launch");
}
int op_matvec_f32(const float *w, const float *x, float *y, int64_t out_dim, int64_t in_dim, cudaStream_t st) {
    if (out_dim <= 0 || in_dim <= 0 || !w || !x || !y) return fail("matvec: bad arguments");
    k_matvec_f32<<<blocks_for(out_dim, 8), 256, 0, st>>>(w, x, y, out_dim, in_dim);
    return check(cudaGetLastError(), "matvec launch");
}
int op_silu_mul(const float *g, const float *u, float *z, int64_t n, cudaStream_t st) {
    if (n <= 0 || !g || !u || !z) return fail("silu_mul: bad arguments");
    if (!check(launch_pdl(k_silu_mul, blocks_for(n, 256), 256, 0, st, g, u, z, n), "silu_mul launch")) return 0;
    return check(cudaGetLastError(), "silu_mul launch");
}
int op_add(const float *a, const float *b, float *o, int64_t n, cudaStream_t st) {
    if (n <= 0 || !a || !b || !o) return fail("add: bad arguments");
    k_add<<<blocks_for(n, 256), 256, 0, st>>>(a, b, o, n);
    return check(cudaGetLastError(), "add launch");
}
int op_scale(float s, const float *x, float *y, int64_t n, cudaStream_t st) {
    if (n <= 0 || !x || !y) return fail("scale: bad arguments");
    k_scale<<<blocks_for(n, 256), 256, 0, st>>>(s, x, y, n);
    return check(cudaGetLastError(), "scale launch");
}
int op_touch(float *x, int64_t n, cudaStream_t st) {
    if (n <= 0 || !x) return fail("touch: bad arguments");
    k_touch<<<blocks_for(n, 256), 256, 0, st>>>(x, n);
    return check(cudaGetLastError(), "touch launch");
}
int op_softmax(const float *x, float *y, int64_t rows, int64_t n, cudaStream_t st) {
    if (rows <= 0 || n <= 0 || !x || !y) return fail("softmax: bad arguments");
    k_softmax<<<(unsigned)rows, kRowThreads, 0, st>>>(x, y, n);
    return check(cudaGetLastError(), "softmax launch");
}
int op_sconv(const float *w, const float *hist, const float *in, float *out, int64_t C, int64_t K, int64_t T,
             cudaStream_t st) {
    if (C <= 0 || K <= 0 || T <= 0 || !w || !in || !out || (K > 1 && !hist)) return fail("sconv: bad arguments");
    k_sconv<<<blocks_for(C * T, 256), 256, 0, st>>>(w, hist, in, out, C, K, T);
    return check(cudaGetLastError(), "sconv launch");
}
int op_sconv_hist_roll(float *hist, const float *in, int64_t C, int64_t K, int64_t T, cudaStream_t st) {
    if (C <= 0 || K <= 0 || T <= 0 || !in) return fail("sconv_hist_roll: bad arguments");
    if (K - 1 > 15) return fail("sconv_hist_roll: K-1 = %lld exceeds 15", (long long)(K - 1));
    if (K == 1) return 1;
    if (!hist) return fail("sconv_hist_roll: null hist");
    k_sconv_hist_roll<<<blocks_for(C, 256), 256, 0, st>>>(hist, in, C, K, T);
    return check(cudaGetLastError(), "sconv_hist_roll launch");
}

}  // namespace sepia

using namespace sepia;

extern "C" int sepia_cuda_rmsnorm(const float *w, const float *x, float *y, int64_t rows, int64_t n, float eps,
                                  void *stream) {
    return op_rmsnorm(w, x, y, rows, n, eps, as_stream(stream));
}
extern "C" int sepia_cuda_matvec_f32(const float *w, const float *x, float *y, int64_t out_dim, int64_t in_dim,
                                     void *stream) {
    return op_matvec_f32(w, x, y, out_dim, in_dim, as_stream(stream));
}
extern "C" int sepia_cuda_silu_mul(const float *g, const float *u, float *z, int64_t n, void *stream) {
    return op_silu_mul(g, u, z, n, as_stream(stream));
}
extern "C" int sepia_cuda_sconv(const float *w, const float *hist, const float *in, float *out, int64_t C, int64_t K,
                                int64_t T, void *stream) {
    return op_sconv(w, hist, in, out, C, K, T, as_stream(stream));
}
extern "C" int sepia_cuda_sconv_hist_roll(float *hist, const float *in, int64_t C, int64_t K, int64_t T, void *stream) {
    return op_sconv_hist_roll(hist, in, C, K, T, as_stream(stream));
}
