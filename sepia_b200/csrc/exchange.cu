// sepia_b200/csrc/exchange.cu -- the expert-sharded MoE exchange
// (include/sepia_cuda.h: sepia_cuda_exchange_*; used by csrc/model.cu).
//
// With experts sharded by index (routed expert e on rank e % world, shared
// expert s on rank s % world), each rank computes the slot terms it owns.
// One kernel then replaces the collective: every rank stores its owned slot
// rows into every rank's receive buffer (plain stores through peer mappings,
// over NVLink; no TMA, no multicast), bumps a per-source arrival counter on
// each rank, waits until every source has arrived for this exchange
// (bounded), and sums the slots in the reference's combine order (routed
// j = 0..k-1, then shared; mlp_moe_forward, src/sepia.c:1420-1466). Each
// slot has exactly one writer, so the sum is bit-identical to one GPU.
//
// Exchange e (1-based, the same sequence on every rank) uses receive buffer
// e & 1 and waits for counter[src] >= e * CTAs. A rank writes buffer e & 1
// again only at exchange e + 2, after every rank arrived at e + 1, i.e.
// after every rank finished reading exchange e. Counters are cumulative and
// per source, so an early arrival of a fast rank at e + 1 cannot satisfy a
// wait for e. The epoch lives on the device: the last CTA of an exchange
// increments it, after every CTA of this rank has read it (each CTA waits
// for its own rank's arrivals, which every CTA makes after reading it).
#include "../../include/sepia_cuda.h"
#include "runtime.h"
#include "common.cuh"

#include <cstring>
#include <vector>

namespace sepia {

constexpr int kXchgCtas = 16;
constexpr int kXchgThreads = 256;
constexpr long long kXchgSpinLimit = 10000000;   // x ~200 ns sleeps: about 2 s

struct XchgArgs {
    const float *slots;                  // this rank's slot terms [n_slots, hidden]
    const int32_t *topk_idx;
    int topk, n_shared, n_routed;
    int64_t hidden;
    int rank, world;
    float *const *peer_recv;             // [world] receive bases (2 buffers each)
    unsigned long long *const *peer_cnt; // [world] counter arrays ([world] each)
    const float *my_recv;
    unsigned long long *my_cnt;
    unsigned long long *epoch;           // exchanges completed on this rank
    unsigned int *done;                  // CTAs finished in the current exchange
    float *out;
    int *err;
    long long spin_limit;
};

__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void red_release_sys_add(unsigned long long *p, unsigned long long v) {
    asm volatile("red.release.sys.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__global__ void __launch_bounds__(kXchgThreads) k_exchange(const XchgArgs A) {
    __shared__ int owned[32];
    __shared__ int n_owned, ok_sh;
    griddep_wait();
    griddep_launch();
    const unsigned long long e = *(volatile unsigned long long *)A.epoch + 1ull;
    const int buf = (int)(e & 1ull);
    const int n_slots = A.topk + A.n_shared;
    if (threadIdx.x == 0) {
        int n = 0;
        for (int j = 0; j < A.topk; j++) {
            const int ex = A.topk_idx[j];
            if (ex >= 0 && ex < A.n_routed && ex % A.world == A.rank) owned[n++] = j;
        }
        for (int s = 0; s < A.n_shared; s++)
            if (s % A.world == A.rank) owned[n++] = A.topk + s;
        n_owned = n;
        ok_sh = 1;
    }
    __syncthreads();
    // this CTA's columns of every owned row, to every rank (itself included)
    const int64_t per = (A.hidden + gridDim.x - 1) / gridDim.x;
    const int64_t c0 = (int64_t)blockIdx.x * per, c1 = imin64(A.hidden, c0 + per);
    for (int k = 0; k < n_owned; k++) {
        const int sl = owned[k];
        const float *src = A.slots + (int64_t)sl * A.hidden;
        for (int p = 0; p < A.world; p++) {
            float *dst = A.peer_recv[p] + ((int64_t)buf * n_slots + sl) * A.hidden;
            for (int64_t c = c0 + threadIdx.x; c < c1; c += blockDim.x) dst[c] = __ldcg(src + c);
        }
    }
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int p = 0; p < A.world; p++) red_release_sys_add(A.peer_cnt[p] + A.rank, 1ull);
        const unsigned long long want = e * (unsigned long long)gridDim.x;
        for (int src = 0; src < A.world && ok_sh; src++) {
            long long spins = 0;
            while (ld_acquire_sys(A.my_cnt + src) < want) {
                if (++spins > A.spin_limit) {
                    set_error(A.err, kErrWaitTimeout);
                    ok_sh = 0;
                    break;
                }
                __nanosleep(200);
            }
        }
    }
    __syncthreads();
    if (ok_sh) {
        const float *rb = A.my_recv + (int64_t)buf * n_slots * A.hidden;
        for (int64_t c = c0 + threadIdx.x; c < c1; c += blockDim.x) {
            float o = 0.0f;
            for (int sl = 0; sl < n_slots; sl++) o = __fadd_rn(o, __ldcg(rb + (int64_t)sl * A.hidden + c));
            A.out[c] = o;
        }
    }
    // the last CTA moves the epoch on (every CTA of this rank read it before
    // arriving, and every CTA has passed its wait or given up)
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        if (atomicAdd(A.done, 1u) == gridDim.x - 1) {
            *A.done = 0u;
            *(volatile unsigned long long *)A.epoch = e;
            __threadfence();
        }
    }
}

int moe_experts_owned_slots(const SepiaMoeLayer *Lh, const float *x, const SepiaMoeWork *ws, cudaStream_t st);

}  // namespace sepia

using namespace sepia;

struct SepiaExchange {
    int n_slots = 0, rank = 0, world = 1;
    int64_t hidden = 0;
    void *mem = nullptr;             // recv[2][n_slots][hidden] floats | counters[world] | epoch, done
    float *recv = nullptr;
    unsigned long long *cnt = nullptr, *epoch = nullptr;
    unsigned int *done = nullptr;
    size_t recv_bytes = 0;
    void *tables = nullptr;          // device arrays peer_recv[world], peer_cnt[world]
    std::vector<void *> opened;
    bool connected = false;
};

static size_t xa(size_t n) { return (n + 255) & ~(size_t)255; }

extern "C" int sepia_cuda_exchange_create(int32_t n_slots, int64_t hidden, int32_t rank, int32_t world,
                                          SepiaExchange **out) {
    if (!out) return fail("exchange: null output");
    *out = nullptr;
    if (n_slots <= 0 || n_slots > 32 || hidden <= 0 || world < 1 || rank < 0 || rank >= world)
        return fail("exchange: bad geometry (slots %d, hidden %lld, rank %d of %d)", n_slots, (long long)hidden, rank,
                    world);
    SepiaExchange *x = new SepiaExchange();
    x->n_slots = n_slots; x->hidden = hidden; x->rank = rank; x->world = world;
    x->recv_bytes = xa(sizeof(float) * 2 * (size_t)n_slots * (size_t)hidden);
    const size_t bytes = x->recv_bytes + xa(sizeof(unsigned long long) * world) + 256;
    if (!check(cudaMalloc(&x->mem, bytes), "exchange: cudaMalloc") ||
        !check(cudaMemset(x->mem, 0, bytes), "exchange: clear")) {
        if (x->mem) cudaFree(x->mem);
        delete x;
        return 0;
    }
    x->recv = (float *)x->mem;
    x->cnt = (unsigned long long *)((char *)x->mem + x->recv_bytes);
    x->epoch = (unsigned long long *)((char *)x->cnt + xa(sizeof(unsigned long long) * world));
    x->done = (unsigned int *)(x->epoch + 1);
    *out = x;
    return 1;
}

extern "C" void sepia_cuda_exchange_destroy(SepiaExchange *x) {
    if (!x) return;
    for (void *p : x->opened) cudaIpcCloseMemHandle(p);
    if (x->tables) cudaFree(x->tables);
    if (x->mem) cudaFree(x->mem);
    delete x;
}

extern "C" int sepia_cuda_exchange_handle(SepiaExchange *x, void *handle) {
    if (!x || !handle) return fail("exchange: handle needs an exchange and an output");
    cudaIpcMemHandle_t h;
    if (!check(cudaIpcGetMemHandle(&h, x->mem), "exchange: cudaIpcGetMemHandle")) return 0;
    memcpy(handle, &h, sizeof h);
    return 1;
}

extern "C" int sepia_cuda_exchange_connect(SepiaExchange *x, const void *handles) {
    if (!x || (!handles && x->world > 1)) return fail("exchange: connect needs the handles");
    if (x->connected) return 1;
    std::vector<float *> recv(x->world);
    std::vector<unsigned long long *> cnt(x->world);
    for (int p = 0; p < x->world; p++) {
        void *base = nullptr;
        if (p == x->rank) {
            base = x->mem;
        } else {
            cudaIpcMemHandle_t h;
            memcpy(&h, (const char *)handles + (size_t)p * sizeof h, sizeof h);
            if (!check(cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess), "exchange: cudaIpcOpenMemHandle"))
                return 0;
            x->opened.push_back(base);
        }
        recv[p] = (float *)base;
        cnt[p] = (unsigned long long *)((char *)base + x->recv_bytes);
    }
    const size_t n = sizeof(void *) * (size_t)x->world;
    if (!check(cudaMalloc(&x->tables, 2 * n), "exchange: peer tables")) return 0;
    if (!check(cudaMemcpy(x->tables, recv.data(), n, cudaMemcpyHostToDevice), "exchange: table upload") ||
        !check(cudaMemcpy((char *)x->tables + n, cnt.data(), n, cudaMemcpyHostToDevice), "exchange: table upload"))
        return 0;
    x->connected = true;
    return 1;
}

extern "C" int sepia_cuda_moe_exchange(SepiaExchange *x, const SepiaMoeLayer *L, const SepiaMoeWork *ws, float *out,
                                       void *stream) {
    if (!x || !L || !ws || !out) return fail("moe_exchange: null argument");
    if (!x->connected) return fail("moe_exchange: call sepia_cuda_exchange_connect first");
    if (L->topk + L->n_shared != x->n_slots || L->hidden != x->hidden || L->rank != x->rank || L->world != x->world)
        return fail("moe_exchange: the layer's slots/hidden/rank/world differ from the exchange's");
    XchgArgs A;
    A.slots = ws->slots; A.topk_idx = ws->topk_idx;
    A.topk = L->topk; A.n_shared = L->n_shared; A.n_routed = L->n_routed; A.hidden = L->hidden;
    A.rank = x->rank; A.world = x->world;
    A.peer_recv = (float *const *)x->tables;
    A.peer_cnt = (unsigned long long *const *)((char *)x->tables + sizeof(void *) * x->world);
    A.my_recv = x->recv; A.my_cnt = x->cnt; A.epoch = x->epoch; A.done = x->done;
    A.out = out; A.err = dev_info().err; A.spin_limit = kXchgSpinLimit;
    if (!check(launch_pdl(k_exchange, kXchgCtas, kXchgThreads, 0, as_stream(stream), A), "moe_exchange launch"))
        return 0;
    return check(cudaGetLastError(), "moe_exchange launch");
}

extern "C" int sepia_cuda_moe_layer_sharded(SepiaExchange *x, const SepiaMoeLayer *L, const float *xin,
                                            const SepiaMoeWork *ws, float *out, void *stream) {
    if (!x) return fail("moe_layer_sharded: null exchange");
    cudaStream_t st = as_stream(stream);
    return sepia_cuda_moe_router(L, xin, ws, stream) && moe_experts_owned_slots(L, xin, ws, st) &&
           sepia_cuda_moe_exchange(x, L, ws, out, stream);
}
