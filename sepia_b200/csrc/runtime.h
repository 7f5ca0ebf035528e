// sepia_b200/csrc/runtime.h -- host-side runtime shared by the CUDA files:
// per-device facts (SM count, opt-in shared memory), the device error word,
// the last-error string and the library's default stream.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace sepia {

struct DevInfo {
    int device = -1;
    int sm_count = 0;
    int smem_optin = 0;      // max dynamic shared memory per block (opt-in)
    int *err = nullptr;      // device error word (DevError codes)
};

// Facts for the current device (initialised on first use per device).
DevInfo &dev_info();
// printf-style: records the message returned by sepia_cuda_last_error()
// and prints "sepia: cuda: <msg>" to stderr. Always returns 0.
int fail(const char *fmt, ...);
// Maps a CUDA error to fail(); returns 1 when err == cudaSuccess.
int check(cudaError_t err, const char *what);
// The library's own stream (non-blocking, created on first use).
cudaStream_t lib_stream();
// Stream argument of the raw entry points: NULL is the legacy default stream
// (stream 0), as everywhere in CUDA -- torch's current stream is usually 0.
inline cudaStream_t as_stream(void *s) { return (cudaStream_t)s; }

// Sets the dynamic shared-memory limit of `fn` to at least `bytes` (cached).
int ensure_smem(const void *fn, int bytes);

// Quant-format geometry on the host (same table as quant_formats.cuh).
int host_block_elems(int type);
int host_block_bytes(int type);
int64_t host_row_bytes(int type, int64_t n);   // -1 if unsupported/ragged

}  // namespace sepia
