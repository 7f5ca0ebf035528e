// sepia_b200/csrc/common.cuh -- device helpers shared by every kernel file:
// error reporting, exact fp16 widening, warp reductions, and the sm_100a
// async-copy primitives (mbarrier + cp.async.bulk) the streaming GEMVs use.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>

#ifndef __CUDACC__
#error "common.cuh is CUDA-only"
#endif

namespace sepia {

// ------------------------------------------------------------------ limits
constexpr int kWarp = 32;
constexpr int kQK = 256;                 // superblock width of every K/IQ format
// A kernel that waits on an mbarrier gives up after this many cycles
// (~1-2 s at B200 clocks), records the failure in the device error word
// and returns.
constexpr long long kWaitCycles = 4000000000LL;
// try_wait may suspend the waiting thread up to this long (ns) instead of
// returning at once: waiting warps stop taking issue slots
constexpr int kWaitSuspendNs = 1000000;

// Device-side error word: 0 = ok. Kernels set a nonzero code instead of
// trapping; the host reads it at sepia_gpu_end() / sepia_cuda_check().
enum DevError : int {
    kErrNone = 0,
    kErrWaitTimeout = 1,
    kErrBadArgs = 2,
};

__device__ __forceinline__ void set_error(int *err, int code) {
    if (err) atomicCAS(err, 0, code);
}

// ------------------------------------------------------------ fp16 widening
// IEEE half bits -> float, exact, NaN payload preserved: the reference's
// software conversion (src/quants.c:58-77) restated with integer ops so the
// result does not depend on how the hardware canonicalises NaNs.
__device__ __forceinline__ float f16_bits_to_f32(uint32_t h) {
    const uint32_t sign = (h & 0x8000u) << 16;
    const uint32_t e = (h >> 10) & 0x1Fu;
    uint32_t m = h & 0x3FFu;
    uint32_t bits;
    if (e == 0x1Fu) {
        bits = sign | 0x7F800000u | (m << 13);
    } else if (e != 0) {
        bits = sign | ((e + 112u) << 23) | (m << 13);
    } else if (m == 0) {
        bits = sign;
    } else {
        // subnormal: normalise (m has at most 10 significant bits)
        const int lz = __clz(m) - 21;          // shifts until bit 10 is set
        m = (m << lz) & 0x3FFu;
        bits = sign | ((uint32_t)(113 - lz) << 23) | (m << 13);
    }
    return __uint_as_float(bits);
}

__host__ __device__ __forceinline__ int64_t imin64(int64_t a, int64_t b) { return a < b ? a : b; }

// ------------------------------------------------------------ reductions
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Reduce-scatter of N per-lane partial sums across the warp (N a power of
// two <= 32). On return v[0] in lane L holds the full warp sum of row
// rs_row<N>(L). Costs N-1 + log2(32/N) shuffles instead of N*5.
template <int N, typename T>
__device__ __forceinline__ void warp_reduce_scatter(T (&v)[N], int lane) {
    int n = N;
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) {
        if (n > 1) {
            const bool upper = (lane & off) != 0;
#pragma unroll
            for (int i = 0; i < N / 2; i++) {
                if (i < n / 2) {
                    const T lo = v[i], hi = v[i + n / 2];
                    const T send = upper ? lo : hi;
                    const T keep = upper ? hi : lo;
                    v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
                }
            }
            n >>= 1;
        } else {
            v[0] += __shfl_xor_sync(0xffffffffu, v[0], off);
        }
    }
}
// Row index whose total lane L holds after warp_reduce_scatter<N>.
template <int N>
__device__ __forceinline__ int rs_row(int lane) {
    int row = 0, n = N;
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) {
        if (n > 1) {
            if (lane & off) row += n / 2;
            n >>= 1;
        }
    }
    return row;
}

// --------------------------------------------------- mbarrier + bulk copy
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Named barriers (ids 1-15; 0 is __syncthreads): nthreads counts every
// thread that arrives or syncs, a multiple of 32.
__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}
__device__ __forceinline__ void named_bar_arrive(int id, int nthreads) {
    asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
                 : "memory");
}

// Arrival counted `count` times (count >= 1).
__device__ __forceinline__ void mbar_arrive_cnt(uint64_t *bar, uint32_t count) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(smem_u32(bar)),
                 "r"(count)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
                     smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "n"(kWaitSuspendNs)
        : "memory");
    return ok != 0;
}

// Bounded wait: returns false (and records kErrWaitTimeout) if the phase
// does not complete within kWaitCycles.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, int *err,
                                          long long limit = kWaitCycles) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, parity)) {
        if (clock64() - t0 > limit) {
            set_error(err, kErrWaitTimeout);
            return false;
        }
    }
    return true;
}

// 16-byte asynchronous copy global -> shared (L2 only); groups of them are
// committed and waited for with cp_async_commit / cp_async_wait<N> (at most
// N groups still in flight).
__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// 1-D bulk copy global -> shared, completion signalled on `bar` as
// transaction bytes. dst/src 16-byte aligned, bytes a multiple of 16.
// No multicast: every CTA fetches its own bytes.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// Byte-granular shared-memory reads at arbitrary alignment (the K/IQ
// blocks of 84/110/50/66/... bytes are only 2-byte aligned in a row).
__device__ __forceinline__ uint32_t lds_u8(const uint8_t *p) { return *p; }
__device__ __forceinline__ uint32_t lds_u16(const uint8_t *p) {
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8);
}
// 4 bytes from a 2-byte-aligned address (two 16-bit loads).
__device__ __forceinline__ uint32_t lds_u32_a2(const uint8_t *p) {
    const uint16_t *q = reinterpret_cast<const uint16_t *>(p);
    return (uint32_t)q[0] | ((uint32_t)q[1] << 16);
}
// 4 bytes from any address: aligned word pair + funnel shift.
__device__ __forceinline__ uint32_t lds_u32_any(const uint8_t *p) {
    // Never touches a word that holds none of the 4 bytes, so it is safe at
    // the very end of a global allocation too.
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    const uint32_t *w = reinterpret_cast<const uint32_t *>(a & ~(uintptr_t)3);
    if ((a & 3) == 0) return w[0];
    const uint32_t sh = (uint32_t)(a & 3) * 8;
    return __funnelshift_r(w[0], w[1], sh);
}

// ------------------------------------------- programmatic dependent launch
// A kernel launched with the programmatic stream serialization attribute
// (launch_pdl) may start while its predecessor in the stream still runs:
// griddep_wait() blocks until the predecessor grid completed and its writes
// are visible (a no-op for a normal launch), griddep_launch() lets the
// successor start launching. Every kernel launched by launch_pdl calls
// griddep_wait() in every CTA before it reads its inputs or writes anything
// a predecessor may still read, so completion stays transitive along the
// stream.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename Kern, typename... Args>
static cudaError_t launch_pdl(Kern kern, dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, args...);
}

}  // namespace sepia
