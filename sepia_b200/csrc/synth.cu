// sepia_b200/csrc/synth.cu -- seeded synthetic weights generated in HBM.
//
// The benchmark models (BASELINE configurations 2 and 5: up to ~317 GB of
// quantized experts) are random-init; generating them on the host and
// copying them in would dominate a run. Here every byte of a unit (one
// expert matrix, one resident tensor) is a hash of (seed, global unit id,
// byte offset), so a rank's shard holds exactly the bytes the same units
// have on any other number of GPUs. Distribution: the block bytes uniform
// (scale/min nibbles, grid indices, sign bits all uniform), then every fp16
// scale field of every block set to a value uniform in [d_lo, d_hi]
// (BASELINE: [1e-3, 4e-3]).
#include "../../include/sepia_cuda.h"
#include "runtime.h"
#include "common.cuh"
#include "quant_formats.cuh"

namespace sepia {

__device__ __forceinline__ uint64_t mix64(uint64_t z) {
    // SplitMix64 finaliser (Steele, Lea, Flood: "Fast splittable
    // pseudorandom number generators", OOPSLA 2014)
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

struct FillArgs {
    uint8_t *dst;
    int64_t n_units, unit_stride, unit_bytes;
    int64_t id0, id_step;
    uint64_t seed;
};

// 16 random bytes per thread-iteration over every unit's byte range.
__global__ void k_fill_bytes(const FillArgs A) {
    const int64_t chunks = (A.unit_bytes + 15) / 16;
    const int64_t total = A.n_units * chunks;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t u = i / chunks, c = i - u * chunks;
        const uint64_t g = (uint64_t)(A.id0 + u * A.id_step);
        const uint64_t key = A.seed * 0x100000001B3ull ^ (g << 32) ^ (uint64_t)c;
        const uint64_t a = mix64(key), b = mix64(key ^ 0xD6E8FEB86659FD93ull);
        uint8_t *p = A.dst + u * A.unit_stride + c * 16;
        if (c * 16 + 16 <= A.unit_bytes && (reinterpret_cast<uintptr_t>(p) & 15) == 0) {
            *reinterpret_cast<uint4 *>(p) = make_uint4((uint32_t)a, (uint32_t)(a >> 32), (uint32_t)b, (uint32_t)(b >> 32));
        } else {
            const int n = (int)imin64(16, A.unit_bytes - c * 16);
            for (int k = 0; k < n; k++) p[k] = (uint8_t)((k < 8 ? a >> (8 * k) : b >> (8 * (k - 8))) & 0xFF);
        }
    }
}

struct ScaleArgs {
    uint8_t *dst;
    int64_t n_units, unit_stride, blocks_per_unit;
    int block_bytes;
    int n_fields, f0, f1;
    int64_t id0, id_step;
    uint64_t seed;
    float d_lo, d_hi;
};

__global__ void k_fill_scales(const ScaleArgs A) {
    const int64_t total = A.n_units * A.blocks_per_unit;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t u = i / A.blocks_per_unit, b = i - u * A.blocks_per_unit;
        const uint64_t g = (uint64_t)(A.id0 + u * A.id_step);
        uint8_t *blk = A.dst + u * A.unit_stride + b * A.block_bytes;
        for (int f = 0; f < A.n_fields; f++) {
            const uint64_t h = mix64(A.seed * 0x9E3779B97F4A7C15ull ^ (g << 34) ^ ((uint64_t)b << 2) ^ (uint64_t)f ^
                                     0xA24BAED4963EE407ull);
            const float r = (float)(h >> 40) * (1.0f / 16777216.0f);       // [0, 1)
            const __half d = __float2half_rn(A.d_lo + r * (A.d_hi - A.d_lo));
            const unsigned short bits = __half_as_ushort(d);
            uint8_t *q = blk + (f == 0 ? A.f0 : A.f1);
            q[0] = (uint8_t)(bits & 0xFF);
            q[1] = (uint8_t)(bits >> 8);
        }
    }
}

// Byte offsets of the fp16 scale fields in one block (d, then dmin).
static int scale_fields(int t, int &f0, int &f1) {
    switch (t) {
    case T_Q8_0: case T_IQ2_XXS: case T_IQ2_XS: case T_IQ3_XXS: case T_IQ1_S: case T_IQ4_XS: f0 = 0; return 1;
    case T_Q2_K: f0 = 80; f1 = 82; return 2;
    case T_Q3_K: f0 = 108; return 1;
    case T_Q4_K: case T_Q5_K: f0 = 0; f1 = 2; return 2;
    case T_Q6_K: f0 = 208; return 1;
    default: return -1;
    }
}

}  // namespace sepia

using namespace sepia;

extern "C" int sepia_cuda_fill_blocks(int ggml_type, void *dst, int64_t n_units, int64_t unit_stride,
                                      int64_t blocks_per_unit, uint64_t seed, int64_t unit_id0, int64_t unit_id_step,
                                      float d_lo, float d_hi, void *stream) {
    int f0 = 0, f1 = 0;
    const int nf = scale_fields(ggml_type, f0, f1);
    const int bb = host_block_bytes(ggml_type);
    if (nf < 0 || bb <= 0) return fail("fill_blocks: type %d is not a quantized block format", ggml_type);
    if (!dst || n_units <= 0 || blocks_per_unit <= 0 || unit_stride < blocks_per_unit * bb)
        return fail("fill_blocks: bad arguments");
    cudaStream_t st = as_stream(stream);
    const int sms = dev_info().sm_count > 0 ? dev_info().sm_count : 148;
    FillArgs A{(uint8_t *)dst, n_units, unit_stride, blocks_per_unit * bb, unit_id0, unit_id_step, seed};
    k_fill_bytes<<<(unsigned)(sms * 8), 256, 0, st>>>(A);
    if (!check(cudaGetLastError(), "fill_blocks launch")) return 0;
    ScaleArgs S{(uint8_t *)dst, n_units, unit_stride, blocks_per_unit, bb, nf, f0, f1, unit_id0, unit_id_step,
                seed, d_lo, d_hi};
    k_fill_scales<<<(unsigned)(sms * 8), 256, 0, st>>>(S);
    return check(cudaGetLastError(), "fill_blocks scales launch");
}
