/*
 * veda_train.h — C ABI of libveda.so (the C++23 host library) for callers that are not C++:
 * the Python tests and bench.py bind it with ctypes. It drives veda::train::Trainer — the
 * reference's training loop (zero_grad, TinyTransformer::forward, cross_entropy, backward,
 * clip_gradient_norm, AdamW::step; tests/TinyModelTest.cpp:290-299) on one GPU of a
 * data-parallel job — and exposes the flat parameter / gradient vectors in the reference's
 * parameter order (src/libs/train/Model.cpp:120-140, GQA k/v shapes [Hkv*Dh, D]).
 * Every entry point returns 0 or a negative status; veda_train_last_error() has the message
 * (the C++ exception's what()).
 */
#ifndef VEDA_TRAIN_H
#define VEDA_TRAIN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* veda_stream_t;
typedef struct veda_trainer veda_trainer;

/* io::ModelConfig's fields (src/libs/io/ModelConfig.h) used by training. */
typedef struct
{
    int64_t vocab, hidden, intermediate, layers, heads, kv_heads, head_dim;
    float eps, theta;
} veda_model_config;

/* optim::AdamWConfig (src/libs/optim/AdamW.h:23-30) plus the clip threshold. */
typedef struct
{
    float lr, beta1, beta2, eps, weight_decay, max_norm;
} veda_optim_config;

const char* veda_train_last_error(void);
/* Sets the stream every subsequent call of this thread launches on (NULL = default stream). */
int veda_train_set_stream(veda_stream_t stream);

/* dtype: 0 fp32 (weights, activations, GEMMs in fp32), 1 bf16 (bf16 weights and activations,
 * fp32 master weights, moments and gradients). Weights ~ N(0, 0.02) from seed, gains 1. */
int veda_trainer_create(const veda_model_config* model, const veda_optim_config* optim, int dtype,
                        int64_t batch, int64_t seq_len, uint64_t seed, veda_trainer** out);
int veda_trainer_destroy(veda_trainer* t);
int64_t veda_trainer_param_count(const veda_trainer* t);
/* Host fp32 flat vectors in parameter order. set_params writes the master weights (and their
 * bf16 rounding into the model in bf16 mode); get_params reads the master weights; get_grads
 * reads the last step's pre-clip gradients, summed over the data-parallel ranks. With a sharded
 * optimizer (veda_trainer_init_dp_sharded) get_params and get_grads are collective: every rank
 * calls them together. */
int veda_trainer_set_params(veda_trainer* t, const float* host);
int veda_trainer_get_params(veda_trainer* t, float* host);
int veda_trainer_get_grads(veda_trainer* t, float* host);

/* Data parallel: 128-byte NCCL unique id (made by rank 0, shared by the caller). */
int veda_nccl_unique_id(void* out128);
int veda_trainer_init_dp(veda_trainer* t, const void* unique_id128, int rank, int world,
                         size_t bucket_bytes);
/* The same with the optimizer state sharded across the ranks (ZeRO stage 1; no reference
 * counterpart: the reference trains on one CPU, AdamW.cpp:38-93 and Clip.cpp:12-61 give the
 * arithmetic): buckets are reduce-scattered, each rank clips (global norm from one all-reduced
 * sum of squares) and updates its 1/world of the parameters, and the updated weights are
 * all-gathered. world <= 8. */
int veda_trainer_init_dp_sharded(veda_trainer* t, const void* unique_id128, int rank, int world,
                                 size_t bucket_bytes);

/* Checkpoints (a writer the reference lacks; its reader is src/libs/io/Safetensors.cpp:106-257):
 * dir/model.safetensors holds the weights under the reference's parameter names
 * (Model.cpp:120-140) in the model's dtype; dir/optimizer.safetensors holds per parameter the fp32
 * master weights, first and second moments ("<name>.master", ".exp_avg", ".exp_avg_sq") and the
 * step count (metadata "step"). Loading restores all of it, so training resumes bit-exactly; a
 * directory without optimizer.safetensors loads the weights and starts the optimizer afresh.
 * Data-parallel: rank 0 writes; with a sharded optimizer both calls are collective. */
int veda_trainer_save_checkpoint(veda_trainer* t, const char* dir);
int veda_trainer_load_checkpoint(veda_trainer* t, const char* dir);
/* Writes host tensors as one safetensors file (the checkpoint writer's format): count tensors with
 * names, dtype names ("BF16", "F32", "I64", ...), ranks and their dims back to back, raw
 * little-endian data; meta_count string pairs of metadata. No device is touched. */
int veda_safetensors_write(const char* path, int64_t count, const char* const* names,
                           const char* const* dtypes, const int64_t* ranks, const int64_t* dims,
                           const void* const* data, int64_t meta_count, const char* const* meta_keys,
                           const char* const* meta_values);

/* A corpus on the device (data::Corpus, src/libs/data/Corpus.cpp:25-107): the same split rule,
 * generator and draw order as the reference, so the same ids and seed give bit-identical batches.
 * next_batch writes batch*length int64 inputs and targets into device buffers on the current
 * stream (split 0 = train, 1 = validation), ready for veda_trainer_step_device. */
typedef struct veda_corpus veda_corpus;
int veda_corpus_create(const int64_t* ids, int64_t n, double validation_fraction, uint64_t seed,
                       veda_corpus** out);
int veda_corpus_destroy(veda_corpus* c);
int64_t veda_corpus_boundary(const veda_corpus* c);
int veda_corpus_next_batch(veda_corpus* c, int64_t batch, int64_t length, int split,
                           int64_t* inputs, int64_t* targets);

/* Greedy generation with the trainer's current weights (generate::Generator with a
 * GreedySampler, src/libs/generate/Generator.cpp:20-109, Sampling.cpp:97-113): cached = 1
 * prefills a device KV cache once and feeds one token per step; cached = 0 reruns the forward over
 * the whole sequence. Writes up to max_new_tokens ids to out, their count, whether a stop token
 * ended it (never emitted) and the number of forward passes. A NaN logit is an error. */
int veda_trainer_generate(veda_trainer* t, const int32_t* prompt, int64_t n, int64_t max_new_tokens,
                          const int32_t* stop_tokens, int64_t n_stop, int cached, int32_t* out,
                          int64_t* out_count, int* stopped, int64_t* forward_passes);
/* The fp32 logits [vocab] of the last of n ids after a forward with the current weights. */
int veda_trainer_last_logits(veda_trainer* t, const int32_t* ids, int64_t n, float* out);

/* The current stream waits for all communication the trainer has queued: a step with a sharded
 * optimizer returns with the all-gather of its updated weights still running (the next step's
 * forward waits for each bucket where it first reads it). Call before timing the end of a run or
 * reading the weights on the device by other means. */
int veda_trainer_sync(veda_trainer* t);

/* On one GPU a step is captured once into a CUDA graph (after one eager step) and replayed: one
 * host call per step instead of ~850 launches. on = 0 keeps this trainer's steps eager. */
int veda_trainer_set_step_graph(veda_trainer* t, int on);

/* One step from host ids/targets (int64 [batch*seq_len], targets = next ids); copies them in,
 * steps and reads back loss and pre-clip grad norm (synchronous). */
int veda_trainer_step_host(veda_trainer* t, const int64_t* ids, const int64_t* targets,
                           float* loss, float* grad_norm);
/* One step on device-resident ids/targets; asynchronous on the current stream. */
int veda_trainer_step_device(veda_trainer* t, const int64_t* ids, const int64_t* targets);
/* Loss and grad norm of the last step (synchronises). Data-parallel, the wait polls the stream and
 * the NCCL communicator (ncclCommGetAsyncError) instead of blocking: an asynchronous error, or no
 * progress within the communication timeout, aborts the communicator (ncclCommAbort) and returns
 * an error instead of hanging on a failed peer. */
int veda_trainer_last_stats(veda_trainer* t, float* loss, float* grad_norm);

/* Failure handling (no reference counterpart: the reference is one CPU process).
 * set_comm_timeout: the data-parallel communication timeout of those waits in seconds (default
 * 600, or VEDA_DP_TIMEOUT_S). abort_comm: aborts the communicator without waiting for the peers,
 * for a caller that has learned on the host (a heartbeat, a store) that a peer is gone; every
 * later step returns an error. set_skip_nonfinite (default off, the reference's behaviour): on,
 * a step whose global gradient norm is not finite updates nothing and is not counted (the next
 * uses the same bias corrections); step_skipped reports whether the step read by the last
 * step_host / last_stats was such a step. */
int veda_trainer_set_comm_timeout(veda_trainer* t, double seconds);
int veda_trainer_abort_comm(veda_trainer* t);
int veda_trainer_set_skip_nonfinite(veda_trainer* t, int on);
int veda_trainer_step_skipped(veda_trainer* t, int* skipped);

/* Activation recompute of attention (default off): each layer keeps its fused q|k|v projection and
 * the attention log-sum-exp only, and the backward forms q, k (norm + RoPE) and the attention
 * output again before the output projection's and the attention's backward. */
int veda_trainer_set_recompute_attention(veda_trainer* t, int on);

/* Device-time profile of kernel classes (gemm_fwd, gemm_dx, gemm_dw, attn_fwd, attn_bwd,
 * cross_entropy, rmsnorm_bwd, swiglu_bwd, adamw), recorded with CUDA events while enabled. */
int veda_profile_enable(int on);
/* Writes up to `cap` entries; returns the number of classes (synchronises; resets the totals). */
int veda_profile_collect(char (*names)[32], double* ms, double* flops, double* bytes,
                         uint64_t* launches, int cap);

#ifdef __cplusplus
}
#endif

#endif /* VEDA_TRAIN_H */
