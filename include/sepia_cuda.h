/* include/sepia_cuda.h -- CUDA-native entry points of libsepia_cuda.so.
 *
 * These take raw device pointers and a cudaStream_t (passed as void*; NULL
 * is the legacy default stream, as in the CUDA runtime) and are
 * stream-ordered: nothing here
 * synchronises, allocates, or touches host memory, so a caller may capture
 * sequences of them in a CUDA graph. They are what the reference-shaped
 * ABI in sepia_gpu.h is built on, and what bench.py and the multi-GPU
 * expert-sharded path call directly. All return 1 on success and 0 on a
 * rejected argument or launch failure (message in sepia_cuda_last_error()).
 * Each cites the reference code whose semantics it reproduces.
 */
#ifndef SEPIA_CUDA_H
#define SEPIA_CUDA_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif
#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

/* ggml type ids (src/quants.h:6-10 plus ggml's numbering for the four
 * formats the reference lacks) */
enum {
    SEPIA_CUDA_T_F32 = 0, SEPIA_CUDA_T_F16 = 1, SEPIA_CUDA_T_Q8_0 = 8, SEPIA_CUDA_T_Q2_K = 10,
    SEPIA_CUDA_T_Q3_K = 11, SEPIA_CUDA_T_Q4_K = 12, SEPIA_CUDA_T_Q5_K = 13, SEPIA_CUDA_T_Q6_K = 14,
    SEPIA_CUDA_T_IQ2_XXS = 16, SEPIA_CUDA_T_IQ2_XS = 17, SEPIA_CUDA_T_IQ3_XXS = 18,
    SEPIA_CUDA_T_IQ1_S = 19, SEPIA_CUDA_T_IQ4_XS = 23
};

/* ------------------------------------------------------------ runtime */
const char *sepia_cuda_last_error(void);
/* Synchronises `stream`, then returns and clears the device error word
 * (0 = none, 1 = a kernel's bounded wait timed out, 2 = bad arguments seen
 * on the device). Returns -1 if the synchronisation itself failed. */
int sepia_cuda_device_error(void *stream);
int sepia_cuda_sm_count(void);
/* ggml geometry: elements per block, bytes per block, bytes per row of n
 * elements (-1 when unsupported or ragged). src/quants.c:28-56. */
int sepia_cuda_block_elems(int ggml_type);
int sepia_cuda_block_bytes(int ggml_type);
int64_t sepia_cuda_row_bytes(int ggml_type, int64_t n);

/* ------------------------------------------------ quantized matvec */
/* out[0..n) = dequant(raw) bit-exactly (src/quants.c:250 dequantize_row). */
int sepia_cuda_dequant(int ggml_type, const void *raw, float *out, int64_t n, void *stream);
/* y[v, o] = sum_i dequant(W[o, :])[i] * x[v, i] for v < n_vec, fp32
 * accumulation (src/sepia.c:742-753 qlinear; metal/matvec_q.metal). W is
 * row-major [out_dim, in_dim] ggml blocks at any byte alignment. */
int sepia_cuda_matvec_q(int ggml_type, const void *w, const float *x, float *y,
                        int64_t out_dim, int64_t in_dim, int64_t n_vec, void *stream);
/* f32 helpers with double accumulation (src/sepia.c:720-740, 755, 801-816) */
int sepia_cuda_matvec_f32(const float *w, const float *x, float *y, int64_t out_dim, int64_t in_dim, void *stream);
int sepia_cuda_rmsnorm(const float *w, const float *x, float *y, int64_t rows, int64_t n, float eps, void *stream);
int sepia_cuda_silu_mul(const float *g, const float *u, float *z, int64_t n, void *stream);
/* One expert's SwiGLU slab, y = down(silu(gate x) * (up x)) with h the
 * [ff] intermediate (real_expert_ffn, src/sepia.c:2993-3022): gate/up
 * [ff, hidden] and down [hidden, ff] in a format of the tensor-core engine
 * (Q2_K/Q3_K/Q4_K, IQ2_XXS/IQ2_XS/IQ3_XXS/IQ1_S), x and h 16-byte aligned.
 * Two launches (gate+up with the SwiGLU epilogue, then down). */
int sepia_cuda_expert_swiglu(int gate_type, const void *gate, int up_type, const void *up, int down_type,
                             const void *down, int64_t hidden, int64_t ff, const float *x, float *h, float *y,
                             void *stream);
int sepia_cuda_sconv(const float *w, const float *hist, const float *in, float *out,
                     int64_t C, int64_t K, int64_t T, void *stream);
int sepia_cuda_sconv_hist_roll(float *hist, const float *in, int64_t C, int64_t K, int64_t T, void *stream);

/* ----------------------------------------------------------- MoE layer */
/* Device description of one MoE layer (src/sepia.c:583-626 LayerWeights'
 * MoE fields, with the experts quantized as in real mode). Routed expert e
 * lives at gate + slot(e)*gate_stride (likewise up/down) where slot(e) =
 * expert_slot[e] if expert_slot is non-NULL, else e / world when world > 1,
 * else e. Expert sharding: routed expert e is computed on rank
 * e % world, shared expert s on rank s % world; every rank computes the same
 * router output. */
typedef struct {
    int64_t hidden, ff;
    int32_t n_routed, n_shared, topk;
    double route_scale;        /* double, as the reference reads it from the config (src/sepia.c:434) */
    float global_scale;
    const float *router_w;     /* [n_routed + n_shared, hidden] */
    const float *router_bias;  /* [n_routed] selection-only bias */
    int32_t gate_type, up_type, down_type;
    const void *gate, *up, *down;
    int64_t gate_stride, up_stride, down_stride;
    int32_t sh_gate_type, sh_up_type, sh_down_type;
    const void *sh_gate, *sh_up, *sh_down;
    int64_t sh_gate_stride, sh_up_stride, sh_down_stride;
    int32_t rank, world;
    const int32_t *expert_slot;
} SepiaMoeLayer;

/* Device scratch of one layer call, carved from one caller allocation. */
typedef struct {
    float *logits;          /* [n_routed + n_shared] */
    int32_t *topk_idx;      /* [topk] */
    float *weights;         /* [topk + n_shared] routed weights then shared gammas */
    float *h;               /* [topk + n_shared, ff] SwiGLU activations */
    float *slots;           /* [topk + n_shared, hidden] per-slot terms (sharded mode) */
    unsigned int *counter;  /* router completion counter; zero before first use */
    double *router_part;    /* [n_routed + n_shared, ceil(hidden/1024)] router scratch (per-row scores) */
    unsigned int *sync;     /* single-launch layer: progress counters; zero before first use, every
                               completed launch leaves them zero (re-zero after a device error) */
    void *htab;             /* single-launch layer: tensor-core activation tables of h */
} SepiaMoeWork;

size_t sepia_cuda_moe_work_bytes(const SepiaMoeLayer *L);
/* base: 256-byte aligned device memory of at least moe_work_bytes(L) bytes,
 * zeroed once by the caller (the router counter resets itself). */
int sepia_cuda_moe_work_carve(const SepiaMoeLayer *L, void *base, size_t bytes, SepiaMoeWork *ws);
/* Router logits (fp64 accumulation) + on-device moe_route_select
 * (src/sepia.c:1329-1375) -> ws->logits, ws->topk_idx, ws->weights. */
int sepia_cuda_moe_router(const SepiaMoeLayer *L, const float *x, const SepiaMoeWork *ws, void *stream);
/* Experts after the router: gate/up+SwiGLU then down. write_slots = 0:
 * out = sum_j w_j E_j(x) + sum_s S_s(x) in the reference order.
 * write_slots = 1: ws->slots[j] = this rank's term for slot j (zero for
 * slots owned by other ranks); after a sum all-reduce of ws->slots across
 * ranks, sepia_cuda_moe_combine gives the same bits as world = 1. */
int sepia_cuda_moe_experts(const SepiaMoeLayer *L, const float *x, const SepiaMoeWork *ws, float *out,
                           int write_slots, void *stream);
/* The two halves of sepia_cuda_moe_experts, separately launchable (used to
 * time each kernel): gate/up+SwiGLU into ws->h, then down + combine.
 * Ordering: the expert kernels run after sepia_cuda_moe_router on the same
 * stream, and x must not be rewritten between the router and them (the
 * gate/up kernel reads x while the router is still finishing). */
int sepia_cuda_moe_gateup(const SepiaMoeLayer *L, const float *x, const SepiaMoeWork *ws, void *stream);
int sepia_cuda_moe_down(const SepiaMoeLayer *L, const SepiaMoeWork *ws, float *out, int write_slots, void *stream);
int sepia_cuda_moe_combine(const SepiaMoeLayer *L, const SepiaMoeWork *ws, float *out, void *stream);
/* router + experts (world must be 1 or the layer already sharded with
 * write_slots handled by the caller). */
int sepia_cuda_moe_layer(const SepiaMoeLayer *L, const float *x, const SepiaMoeWork *ws, float *out, void *stream);
/* The same layer as ONE persistent cooperative kernel (router, top-k,
 * gate/up, down and combine; no kernel boundary). Opt-in: on B200 it
 * measured slower than the kernel chain of sepia_cuda_moe_layer (96 us
 * against 72 us for BASELINE configuration 2), because under a saturated
 * memory system each of its cross-CTA dependencies costs 2-4 us. Same
 * results as the chain (ids and weights equal, outputs within 1e-6).
 * eligible: 1 when the fused kernel takes this layer (world = 1,
 * tensor-core expert formats, hidden <= 8192, a shared-memory plan that
 * fits). No reference counterpart: the reference synchronises the host
 * inside every MoE layer (src/sepia.c:3831-3974). */
int sepia_cuda_moe_fused_eligible(const SepiaMoeLayer *L, const SepiaMoeWork *ws);
int sepia_cuda_moe_layer_fused(const SepiaMoeLayer *L, const float *x, const SepiaMoeWork *ws, float *out,
                               void *stream);
/* Selection only: top-k of given scores by the reference's strict-'>' scan
 * (src/sepia.c:1336-1347; lowest index wins ties). */
int sepia_cuda_topk_select(const float *scores, int32_t n, int32_t topk, int32_t *idx, void *stream);

/* ------------------------------------------- expert-sharded exchange */
/* With experts sharded by index over the GPUs of one box (one process per
 * GPU, routed expert e on rank e % world, shared expert s on rank
 * s % world), every rank computes the same router and only the slot terms
 * it owns. The exchange replaces the collective with one kernel: owned slot
 * rows are stored into every rank's receive buffer through peer mappings
 * (NVLink), a per-source arrival counter is bumped on every rank, each rank
 * waits until all sources arrived (bounded, about 2 s; on timeout the device
 * error word is set and `out` is left unwritten) and sums the slots in the
 * reference's combine order, so the result is bit-identical to one GPU.
 * No counterpart in the reference (its expert store is one process on one
 * GPU, src/sepia.c:2216-2470; combine order src/sepia.c:1420-1466).
 * Setup: create on every rank, export the 64-byte IPC handle
 * (cudaIpcMemHandle_t), gather all ranks' handles in rank order by any host
 * channel, connect. Every rank must then run the same sequence of
 * exchanges; calls are stream-ordered and may be captured in CUDA graphs. */
typedef struct SepiaExchange SepiaExchange;
int sepia_cuda_exchange_create(int32_t n_slots, int64_t hidden, int32_t rank, int32_t world, SepiaExchange **out);
void sepia_cuda_exchange_destroy(SepiaExchange *x);
int sepia_cuda_exchange_handle(SepiaExchange *x, void *handle);
int sepia_cuda_exchange_connect(SepiaExchange *x, const void *handles);
/* out = combine of every rank's owned slot terms in ws->slots (after
 * sepia_cuda_moe_router + the owned-slot experts). */
int sepia_cuda_moe_exchange(SepiaExchange *x, const SepiaMoeLayer *L, const SepiaMoeWork *ws, float *out,
                            void *stream);
/* Router + this rank's experts + exchange: one sharded MoE layer. */
int sepia_cuda_moe_layer_sharded(SepiaExchange *x, const SepiaMoeLayer *L, const float *xin, const SepiaMoeWork *ws,
                                 float *out, void *stream);

/* ------------------------------------------------- banded attention */
/* rel_logits[t,h,r] = sum_d r_vec[t,h,d] * rel_proj[d,r] (src/sepia.c:1201-1208) */
int sepia_cuda_rel_project(const float *r_vec, const float *rel_proj, float *rel_logits,
                           int64_t T, int64_t H, int64_t d_rel, int64_t rel_extent, void *stream);
/* Split-KV banded attention (src/sepia.c:1210-1262). kv_f16 selects fp16
 * K/V caches (else fp32); kv_lo/kv_hi/tau are DEVICE arrays of length T;
 * max_kv bounds kv_hi-kv_lo+1 and sizes the split; ws holds the per-split
 * partials (sepia_cuda_banded_attn_ws_bytes). */
size_t sepia_cuda_banded_attn_ws_bytes(int64_t T, int64_t H, int64_t Hkv, int64_t Dh, int64_t max_kv);
int sepia_cuda_banded_attn(int kv_f16, const float *q, const void *k, const void *v, const float *rel_logits,
                           float *out, const int64_t *kv_lo, const int64_t *kv_hi, const float *tau,
                           int64_t T, int64_t H, int64_t Hkv, int64_t Dh, int64_t rel_extent,
                           int64_t q_pos_base, int64_t kv_dim, float inv_head_dim, int64_t max_kv,
                           void *ws, size_t ws_bytes, void *stream);

/* Allocation-free banded attention. No counterpart in the reference (its
 * Metal backend allocates per call): for callers that cannot allocate device
 * memory -- a host whose device heap belongs to another allocator, a plugin
 * host that only passes its own input/output buffers, or a loop that must not
 * call cudaMalloc/cudaFree because they can synchronize the device. Same
 * arguments and result as sepia_cuda_banded_attn minus the workspace: the
 * split partials go to a fixed 8 MiB array inside the library
 * (sepia_cuda_banded_attn_noalloc_max_bytes), held on every GPU that loads
 * the library until exit. Shapes whose partials exceed it return 0 with a
 * "needs N bytes" error. The first call on each device resolves the array's
 * address and caches it; make it before any stream capture begins. A
 * cudaDeviceReset makes the cached address stale and the library does not
 * notice: do not call this entry point on a device after resetting it in
 * the same process. All calls on a device
 * share the array: calls whose kernels overlap on the GPU (unordered
 * streams) race; calls on one stream are safe. */
size_t sepia_cuda_banded_attn_noalloc_max_bytes(void);
int sepia_cuda_banded_attn_noalloc(int kv_f16, const float *q, const void *k, const void *v,
                                   const float *rel_logits, float *out, const int64_t *kv_lo,
                                   const int64_t *kv_hi, const float *tau, int64_t T, int64_t H, int64_t Hkv,
                                   int64_t Dh, int64_t rel_extent, int64_t q_pos_base, int64_t kv_dim,
                                   float inv_head_dim, int64_t max_kv, void *stream);

/* ------------------------------------------------------ synthetic weights */
/* Fills n_units units (unit u at dst + u*unit_stride, blocks_per_unit
 * blocks of ggml_type each) with seeded random blocks: bytes uniform, every
 * fp16 scale field (d, dmin) uniform in [d_lo, d_hi]. Unit u's bytes depend
 * only on (seed, unit_id0 + u*unit_id_step), so a shard holding every
 * world-th expert gets exactly the bytes those experts have unsharded.
 * No counterpart in the reference (its models are real checkpoints); used
 * to build the random-init benchmark models in HBM. */
int sepia_cuda_fill_blocks(int ggml_type, void *dst, int64_t n_units, int64_t unit_stride, int64_t blocks_per_unit,
                           uint64_t seed, int64_t unit_id0, int64_t unit_id_step, float d_lo, float d_hi,
                           void *stream);

/* ---------------------------------------------------------- test hooks */
/* The stream that the sepia_gpu_* batch API (sepia_gpu.h) enqueues on. */
void *sepia_cuda_lib_stream(void);
/* Failure detection without a GPU fault (no counterpart in the reference):
 * runs the tensor-core matvec engine with its producer announcing 16 bytes
 * more than it copies, so no stage ever completes. Every waiting role gives
 * up after wait_cycles SM clock cycles (<= about 4e9), records error 1 in
 * the device error word (read by sepia_cuda_device_error or sepia_gpu_end)
 * and returns; y is left unwritten. The context stays usable. */
int sepia_cuda_test_engine_timeout(int ggml_type, const void *w, const float *x, float *y,
                                   int64_t out_dim, int64_t in_dim, long long wait_cycles, void *stream);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif
#ifdef __cplusplus
}
#endif
#endif
