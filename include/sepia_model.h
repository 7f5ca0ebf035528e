/* include/sepia_model.h -- the whole-token decode engine of libsepia_cuda.so.
 *
 * One call runs a token through every decoder layer on the device: embedding
 * row + norm, per layer the attention block (q/k/v/r projections, K/V short
 * convolutions, per-head norms, cache write, relative-position band, banded
 * attention, output projection), its short convolution and residual, the
 * MoE (router, top-k, routed + shared experts) or dense MLP block, its short
 * convolution and residual, then the final norm, the logits head and an
 * on-device argmax that feeds the next token. Decode steps are captured
 * once as a CUDA graph and replayed: no host synchronisation per token.
 *
 * It replaces the reference's host-driven token loop: real_forward_chunk
 * (src/sepia.c:3345-3390, CPU) and real_forward_chunk_gpu
 * (src/sepia.c:4042-4102, 196 host syncs per token), driven by
 * real_generate / real_generate_gpu (src/sepia.c:4114-4158, 4219-4272).
 * Arithmetic follows the CPU path: fp32 storage, double accumulation, the
 * KV cache in fp32, tau in double (src/sepia.c:1188-1194).
 *
 * Weights stay where the caller put them (device memory, GGUF block
 * layout); the engine allocates its own caches and scratch at create time
 * and nothing per token. All calls are stream-ordered and return 1 on
 * success, 0 on error (message in sepia_cuda_last_error()).
 */
#ifndef SEPIA_MODEL_H
#define SEPIA_MODEL_H
#include <stddef.h>
#include <stdint.h>

#include "sepia_cuda.h"

#ifdef __cplusplus
extern "C" {
#endif
#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

/* A weight matrix [rows, cols] in ggml block layout on the device
 * (src/sepia.c:559 QTensor with out_dim = rows, in_dim = cols). */
typedef struct {
    int32_t type;
    int32_t reserved;
    const void *data;
    int64_t rows, cols;
} SepiaQTensor;

/* One decoder layer (src/sepia.c:2111-2135 RealLayer, resolved per layer as
 * real_fill_layer does, src/sepia.c:2922-2979). Device pointers. */
typedef struct {
    int32_t is_sliding, is_sparse;
    int32_t n_heads, n_kv_heads, head_dim, rel_extent;
    const float *attn_norm, *mlp_norm;      /* [hidden] */
    const float *q_norm, *k_norm;           /* [head_dim] */
    const float *rel_proj;                  /* [d_rel, rel_extent] */
    const float *k_sconv, *v_sconv;         /* [n_kv_heads*head_dim, conv_k] */
    const float *attn_sconv, *mlp_sconv;    /* [hidden, conv_k] */
    SepiaQTensor wq, wk, wv, wr, wo;
    /* dense layers */
    SepiaQTensor dense_gate, dense_up, dense_down;
    float dense_gscale;                     /* ffn_gscale.weight[0] */
    /* sparse layers: router, experts (this rank's shard), shared experts */
    SepiaMoeLayer moe;
} SepiaModelLayer;

typedef struct {
    int64_t hidden;
    int32_t n_layers;
    int32_t vocab, unpadded_vocab;
    int32_t d_rel, conv_k, window;
    int32_t max_positions;                  /* KV cache capacity */
    float eps;                              /* (float)rms_norm_eps */
    float mup;                              /* (float)logits_mup_width_multiplier */
    int32_t has_log_scaling;
    double log_scaling_alpha;
    int64_t log_scaling_n_floor;
    SepiaQTensor embed, unembed;            /* token_embd.weight, output.weight */
    const float *embed_norm, *final_norm;   /* [hidden] */
    const SepiaModelLayer *layers;          /* host array of n_layers */
    /* expert sharding over the GPUs of one box: this process is rank `rank`
     * of `world`; every sparse layer's moe must be that rank's shard */
    int32_t rank, world;
} SepiaModelDesc;

typedef struct SepiaModel SepiaModel;

/* Validates the description, allocates the KV caches, convolution
 * histories and scratch on the current device, and computes the tau table
 * (double, per position). The layer array is copied; weights are not. */
int sepia_model_create(const SepiaModelDesc *d, SepiaModel **out);
void sepia_model_destroy(SepiaModel *m);
/* Device bytes the engine allocated (caches + scratch). */
size_t sepia_model_device_bytes(const SepiaModel *m);
/* Clears caches, histories and the position (a new sequence). */
int sepia_model_reset(SepiaModel *m, void *stream);
/* Teacher-forced tokens ids[0..n) (DEVICE int32 array) at positions
 * pos .. pos+n-1, one token at a time through every layer (identical to the
 * reference's chunked prefill: every op is causal per token). With
 * want_logits, the last token's logits are computed and their argmax
 * becomes the next input token. */
int sepia_model_prefill(SepiaModel *m, const int32_t *ids, int32_t n, int32_t want_logits, void *stream);
/* n greedy steps: each step consumes the pending argmax token, writes it
 * to out_ids[i] (DEVICE int32 array), runs it through the model and takes
 * the argmax of its logits. Replays a CUDA graph captured on first use
 * (capture happens on `stream`; make the first call outside any capture). */
int sepia_model_decode(SepiaModel *m, int32_t n, int32_t *out_ids, void *stream);
/* Device pointer to the last computed logits [unpadded_vocab]. */
const float *sepia_model_logits(const SepiaModel *m);
/* Copies the last logits into dst (device, unpadded_vocab floats). */
int sepia_model_copy_logits(const SepiaModel *m, float *dst, void *stream);
/* Expert sharding (world > 1). Every rank exports the IPC handle of its
 * exchange buffers (64 bytes, cudaIpcMemHandle_t) and passes all ranks'
 * handles, in rank order, to sepia_model_connect before its first token.
 * Each sparse layer then ends with a one-kernel exchange instead of a
 * collective: owned slot rows are stored into every rank's buffers over
 * NVLink, a per-source arrival counter is bumped, and each rank waits
 * (bounded, ~2 s; on timeout the device error word is set and the layer's
 * output is left unwritten) before summing the slots in the reference's
 * order -- bit-identical to one GPU. No counterpart in the reference (its
 * expert store is one process on one GPU, src/sepia.c:2216-2470). */
int sepia_model_exchange_handle(SepiaModel *m, void *handle);
int sepia_model_connect(SepiaModel *m, const void *handles);
/* Position of the next token (synchronises `stream`). */
int sepia_model_position(SepiaModel *m, void *stream);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif
#ifdef __cplusplus
}
#endif
#endif
