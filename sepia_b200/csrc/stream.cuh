// sepia_b200/csrc/stream.cuh -- the row-streaming pipeline shared by every
// quantized GEMV kernel.
//
// Shape of a streaming kernel:
//   * the weight bytes of a "unit" (a tile of consecutive rows of one or
//     more matrices) are contiguous byte ranges in HBM;
//   * one producer thread moves each range into a shared-memory stage with
//     a 1-D cp.async.bulk (TMA engine, no tensor map, no multicast), signalled
//     on a per-stage "full" mbarrier with transaction bytes;
//   * consumer warps split the K dimension: each lane owns one 32-element
//     part of a 256-wide superblock and keeps the matching activations in
//     registers for the whole kernel, so only weight bytes cross shared
//     memory; after a tile each warp reduce-scatters its per-row partials and
//     the warps' partials are summed in a fixed order (deterministic);
//   * consumers release a stage on a per-stage "empty" mbarrier.
// A bulk copy needs 16-byte aligned addresses and sizes, so a range is
// fetched from floor16(src) to ceil16(end) and lands at stage + (src & 15):
// the shared-memory copy keeps the global address modulo 16.
#pragma once
#include "quant_dot.cuh"

namespace sepia {

struct ByteRange {
    const uint8_t *src;
    uint32_t bytes;
};

__device__ __forceinline__ uint32_t range_copy_bytes(const ByteRange &r) {
    const uintptr_t a0 = reinterpret_cast<uintptr_t>(r.src) & ~(uintptr_t)15;
    const uintptr_t a1 = (reinterpret_cast<uintptr_t>(r.src) + r.bytes + 15) & ~(uintptr_t)15;
    return (uint32_t)(a1 - a0);
}

// Issue the copy of one range into `dst` (16-aligned); returns the bytes moved.
__device__ __forceinline__ uint32_t range_issue(uint8_t *dst, const ByteRange &r, uint64_t *full) {
    const uint32_t n = range_copy_bytes(r);
    const uint8_t *a0 = reinterpret_cast<const uint8_t *>(reinterpret_cast<uintptr_t>(r.src) & ~(uintptr_t)15);
    bulk_g2s(dst, a0, n, full);
    return n;
}

// Where the first byte of a range sits inside its stage slot.
__device__ __forceinline__ const uint8_t *range_data(const uint8_t *dst, const ByteRange &r) {
    return dst + (reinterpret_cast<uintptr_t>(r.src) & 15);
}

// Shared-memory bytes a slot needs for a range of `bytes` bytes: the copy
// may start up to 15 bytes early and end up to 15 bytes late, and decoders
// may read one word past the last byte.
__host__ __device__ inline uint32_t slot_bytes_for(uint64_t bytes) {
    return (uint32_t)(((bytes + 15 + 15 + 16) + 15) & ~(uint64_t)15);
}

// Named barrier among the consumer warps only (id 1; id 0 is __syncthreads).
__device__ __forceinline__ void consumer_sync(int nthreads) {
    asm volatile("bar.sync 1, %0;" ::"r"(nthreads) : "memory");
}

// Load the activation part a lane owns: x[sb*256 + 32p + i] for i < 32,
// zero beyond in_dim; also the two 16-element sums and, for the fast
// formats (SCALED), the per-position pre-scaling of quant_dot.cuh.
template <bool SCALED>
__device__ __forceinline__ void load_xpart(XPart &xp, const float *x, int64_t in_dim, int sb, int p) {
    const int64_t base = (int64_t)sb * kQK + 32 * p;
    if (base + 32 <= in_dim && ((reinterpret_cast<uintptr_t>(x + base) & 15) == 0)) {
        const float4 *v = reinterpret_cast<const float4 *>(x + base);
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const float4 q = __ldg(v + i);
            xp.v[4 * i] = q.x; xp.v[4 * i + 1] = q.y; xp.v[4 * i + 2] = q.z; xp.v[4 * i + 3] = q.w;
        }
    } else {
#pragma unroll
        for (int i = 0; i < 32; i++) xp.v[i] = (base + i < in_dim) ? __ldg(x + base + i) : 0.0f;
    }
    xpart_finish<SCALED>(xp);
}

// Dot of one row's parts owned by this lane: superblocks sb_j, part p.
// Returns 0 for parts beyond in_dim (never touches those bytes).
template <int T, int C>
__device__ __forceinline__ float row_parts_dot(const uint8_t *row, int sbb, const int (&sb)[C], int p,
                                               const XPart (&xp)[C], int64_t in_dim) {
    float acc = 0.0f;
#pragma unroll
    for (int j = 0; j < C; j++) {
        const int64_t first = (int64_t)sb[j] * kQK + 32 * p;
        if (first < in_dim) {
            const int nvalid = (int)imin64(32, in_dim - first);
            acc += dot_part<T>(row + (int64_t)sb[j] * sbb, p, xp[j], nvalid);
        }
    }
    return acc;
}

}  // namespace sepia
