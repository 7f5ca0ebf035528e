// sepia_b200/csrc/runtime.cu -- implementation of runtime.h.
#include "runtime.h"
#include "../../include/sepia_cuda.h"

#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <mutex>
#include <unordered_map>

#include "quant_formats.cuh"

namespace sepia {

thread_local char g_last_error[512];

int fail(const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_last_error, sizeof g_last_error, fmt, ap);
    va_end(ap);
    fprintf(stderr, "sepia: cuda: %s\n", g_last_error);
    return 0;
}

int check(cudaError_t err, const char *what) {
    if (err == cudaSuccess) return 1;
    return fail("%s: %s", what, cudaGetErrorString(err));
}

static std::mutex g_mu;
static DevInfo g_infos[64];

DevInfo &dev_info() {
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) dev = 0;
    DevInfo &d = g_infos[dev];
    if (d.device == dev) return d;
    std::lock_guard<std::mutex> lk(g_mu);
    if (d.device != dev) {
        cudaDeviceGetAttribute(&d.sm_count, cudaDevAttrMultiProcessorCount, dev);
        cudaDeviceGetAttribute(&d.smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
        if (cudaMalloc(&d.err, sizeof(int)) != cudaSuccess) d.err = nullptr;
        else cudaMemset(d.err, 0, sizeof(int));
        d.device = dev;
    }
    return d;
}

static cudaStream_t g_streams[64];

cudaStream_t lib_stream() {
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) dev = 0;
    if (!g_streams[dev]) {
        std::lock_guard<std::mutex> lk(g_mu);
        if (!g_streams[dev]) cudaStreamCreateWithFlags(&g_streams[dev], cudaStreamNonBlocking);
    }
    return g_streams[dev];
}

int ensure_smem(const void *fn, int bytes) {
    static std::mutex mu;
    static std::unordered_map<uint64_t, int> done;   // (device, fn) -> bytes set
    int dev = 0;
    cudaGetDevice(&dev);
    const uint64_t key = (reinterpret_cast<uint64_t>(fn) << 6) ^ (uint64_t)dev;
    {
        std::lock_guard<std::mutex> lk(mu);
        auto it = done.find(key);
        if (it != done.end() && it->second >= bytes) return 1;
    }
    if (!check(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes),
               "cudaFuncSetAttribute(max dynamic smem)"))
        return 0;
    std::lock_guard<std::mutex> lk(mu);
    done[key] = bytes;
    return 1;
}

int host_block_elems(int t) { return fmt_block_elems(t); }
int host_block_bytes(int t) { return fmt_block_bytes(t); }
int64_t host_row_bytes(int t, int64_t n) {
    const int e = fmt_block_elems(t);
    if (e == 0 || n < 0 || n % e) return -1;
    return (n / e) * (int64_t)fmt_block_bytes(t);
}

}  // namespace sepia

extern "C" const char *sepia_cuda_last_error(void) { return sepia::g_last_error; }
