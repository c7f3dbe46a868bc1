// veda::train — the reference's trainable Qwen3-architecture decoder
// (src/libs/train/Model.h:34-72, Model.cpp:72-255) on the device, and the training step driver.
//
// TinyTransformer keeps the reference's parameter names, shapes and order
// (model.embed_tokens.weight, then per layer input_layernorm, q/k/v/o_proj, q/k_norm,
// post_attention_layernorm, gate/up/down_proj, then model.norm.weight; tied LM head) and its
// forward (pre-norm residual blocks, QK-norm before RoPE, causal softmax attention, SwiGLU). It
// differs where the B200 build needs it to:
//   * GQA is allowed (Hkv < H; k/v_proj are [Hkv*Dh, D]); the reference refuses it in training;
//   * weights live in one flat value arena (fp32 or bf16) and gradients in one flat fp32 arena,
//     in parameter order, so q|k|v and gate|up are single [.., D] matrices and the optimiser and
//     the all-reduce see whole buckets;
//   * the forward uses the fused modules of veda::autograd (rms_norm, linear, attention,
//     swiglu, cross_entropy) — one tape node each.
// Trainer runs one step (zero_grad, forward, cross-entropy, backward, data-parallel gradient
// all-reduce overlapped with the backward, fused clip + AdamW) on one GPU of a data-parallel job.
#pragma once

#include <functional>

#include "veda/autograd.hpp"
#include "veda/optim.hpp"

#include <cstdint>
#include <map>
#include <memory>
#include <string>
#include <utility>
#include <vector>

struct CUgraphExec_st;

namespace veda::generate
{
class Generator;
}

namespace veda::train
{

struct ModelConfig
{
    size_t hidden_size = 0;              // D
    size_t intermediate_size = 0;        // F
    size_t num_layers = 0;
    size_t num_heads = 0;                // H
    size_t num_kv_heads = 0;             // Hkv
    size_t head_dim = 0;                 // Dh
    size_t vocab_size = 0;               // V
    size_t max_position_embeddings = 0;
    float rms_norm_eps = 1e-6f;
    float rope_theta = 10000.0f;
    bool tie_word_embeddings = true;

    size_t queries_per_kv_head() const { return num_heads / num_kv_heads; }
};

// The reference's tiny_config() (src/libs/train/Model.cpp:72-89).
ModelConfig tiny_config();

// RoPE tables [T, Dh] in fp32 from angles computed in double (src/libs/model/Rope.cpp:17-63).
std::pair<core::Tensor, core::Tensor> rope_tables(size_t positions, size_t head_dim, float theta);

class TinyTransformer
{
public:
    // Weights ~ N(0, 0.02) from `seed` (device hash generator), norm gains 1.
    TinyTransformer(ModelConfig config, uint64_t seed, core::DType dtype = core::DType::F32);

    // ids are B*T token ids; the result is logits [B*T, V] on the tape.
    autograd::Variable forward(const std::vector<int64_t>& ids, size_t batch, size_t length);
    // ids already on the device (int64 [B*T]).
    autograd::Variable forward_device(const core::Tensor& ids, size_t batch, size_t length);

    // Every trainable leaf, once each, in the reference's order (views into the arenas).
    const std::vector<autograd::Variable>& parameters() const noexcept { return parameters_; }
    std::vector<std::pair<std::string, core::Tensor>> named_parameters() const;
    const ModelConfig& config() const noexcept { return config_; }
    core::DType dtype() const noexcept { return dtype_; }

    // The leaves the forward graph consumes (q|k|v and gate|up fused), with their arena ranges.
    struct GraphLeaf
    {
        autograd::Variable var;
        size_t offset, count;   // in elements of the arenas
    };
    const std::vector<GraphLeaf>& graph_leaves() const noexcept { return graph_leaves_; }
    const core::Tensor& value_arena() const noexcept { return values_; }
    const core::Tensor& grad_arena() const noexcept { return grads_; }
    size_t parameter_count() const noexcept { return total_; }
    // Elements the arenas hold: parameter_count() rounded up to a multiple of kArenaAlign, so a
    // data-parallel job of up to 8 ranks can cut them into equal shards of whole 16-byte rows.
    static constexpr size_t kArenaAlign = 8 * 840;   // 8 x lcm(1, ..., 8)
    size_t arena_length() const noexcept { return arena_len_; }
    // Clears the whole gradient arena in one memset and marks every leaf's gradient as zero.
    void zero_grad();
    // zero_grad without the memset: every leaf is only marked as holding zeros, so the backward's
    // first write to it overwrites (a GEMM with beta 0, a copy, a kernel that clears its target
    // first). clear_untouched_grads() then clears the leaves the backward never reached; between
    // the two calls the arena holds the previous step's values.
    void mark_grads_zero();
    void clear_untouched_grads();
    // Called with an arena range [lo, hi) before the forward first reads the weights in it, so
    // that a data-parallel step whose updated weights are still arriving waits only for them.
    void set_weight_gate(std::function<void(size_t, size_t)> gate) { gate_ = std::move(gate); }
    // forward_device looks the tokens up through autograd::embedding_device_rows with this sink
    // (empty: the plain embedding, whose backward scatters into the table's gradient).
    void set_embedding_rows_sink(autograd::RowsSink sink) { rows_sink_ = std::move(sink); }
    // The embedding table's range in the arenas, in elements.
    std::pair<size_t, size_t> embedding_range() const noexcept { return embed_range_; }
    // Activation recompute of attention: each layer's attention and output projection become one
    // node that keeps the fused projection and the log-sum-exp only, and forms q, k and the
    // context again in the backward (off by default).
    void set_recompute_attention(bool on) noexcept { recompute_attention_ = on; }
    bool recompute_attention() const noexcept { return recompute_attention_; }

private:
    autograd::Variable forward_from(const autograd::Variable& x, size_t batch, size_t length);

    friend class generate::Generator;   // reads the weights for inference
    ModelConfig config_;
    core::DType dtype_;
    core::Tensor values_, grads_;
    size_t total_ = 0;
    size_t arena_len_ = 0;
    std::function<void(size_t, size_t)> gate_;
    bool recompute_attention_ = false;
    autograd::RowsSink rows_sink_;
    std::pair<size_t, size_t> embed_range_, final_range_;
    std::vector<std::pair<size_t, size_t>> layer_ranges_;
    std::vector<autograd::Variable> parameters_;
    std::vector<std::string> names_;
    std::vector<GraphLeaf> graph_leaves_;
    struct Layer
    {
        autograd::Variable in_norm, qkv, o, q_norm, k_norm, post_norm, gate_up, down;
    };
    autograd::Variable embed_, final_norm_;
    std::vector<Layer> layers_;
    std::map<size_t, std::pair<core::Tensor, core::Tensor>> rope_cache_;
};

class DataParallel;

struct StepStats
{
    float loss = 0.0f;
    float grad_norm = 0.0f;
    bool skipped = false;   // set_skip_nonfinite: the norm was not finite and nothing was updated
};

class Trainer
{
public:
    Trainer(ModelConfig config, optim::AdamWConfig adam, float max_norm, core::DType dtype,
            size_t batch, size_t length, uint64_t seed);
    ~Trainer();

    // One process per GPU: NCCL communicator from a unique id shared by the caller; gradients
    // are all-reduced in buckets of `bucket_bytes` as soon as the backward finishes them.
    // sharded: the optimizer state is split across the ranks instead (ZeRO stage 1): each bucket
    // is reduce-scattered, every rank clips and updates its shard of every bucket, and the
    // updated weights are all-gathered. The host-side reads of the full master weights and
    // gradients (read_master_weights / read_gradients) are then collective.
    void init_data_parallel(const void* nccl_unique_id, int rank, int world, size_t bucket_bytes,
                            bool sharded = false);
    int world() const noexcept;
    bool sharded() const noexcept;
    // Device pointer of the fp32 master weights in arena order (the value arena for fp32).
    float* master_weights() noexcept;
    // The current stream waits for all communication the trainer has queued (a sharded step
    // leaves the all-gather of the updated weights running into the next step's forward).
    void sync();
    // Brings master_weights() (and, sharded, the gradient arena) up to date on every rank;
    // collective when sharded, a no-op otherwise.
    void gather_master_weights();
    void gather_gradients();
    // After master_weights() was written from the host: refresh this rank's shard of it.
    void master_weights_changed();
    // Checkpoint: dir/model.safetensors (the weights under the reference's parameter names, bf16
    // or fp32 as the model computes) and dir/optimizer.safetensors (per parameter its fp32
    // master weights, first and second moments as "<name>.master", ".exp_avg", ".exp_avg_sq";
    // metadata "step"). Data-parallel: rank 0 writes; collective when sharded. Loading without
    // an optimizer file starts the optimizer afresh from the file's weights.
    void save_checkpoint(const std::string& dir);
    void load_checkpoint(const std::string& dir);

    // One training step on device-resident ids/targets (int64 [B*T]); asynchronous.
    void step(const core::Tensor& ids, const core::Tensor& targets);
    // Single-GPU steps are captured once into a CUDA graph and replayed (on by default; the
    // environment variable VEDA_STEP_GRAPH=0 turns it off for the process).
    void set_step_graph(bool on);
    // One step from host buffers: copies in, steps, reads loss and grad norm back (synchronous).
    StepStats step_host(const int64_t* ids, const int64_t* targets);
    // Loss and pre-clip grad norm of the last step (synchronises). Data-parallel, the wait polls
    // the stream and the communicator (ncclCommGetAsyncError) instead of blocking: an error, or
    // no progress within the communication timeout, aborts the communicator (ncclCommAbort) and
    // throws std::runtime_error instead of hanging on a failed peer.
    StepStats last_stats();
    // Data-parallel: the communication timeout of those waits (default 600 s, or
    // VEDA_DP_TIMEOUT_S).
    void set_comm_timeout(double seconds);
    // Data-parallel: abort the communicator without waiting for the peers (for a caller that has
    // learned on the host that a peer is gone); every later step throws.
    void abort_communication();
    // On: a step whose global gradient norm is not finite updates nothing, last_stats() reports
    // it as skipped, and the step is not counted (the next uses the same bias corrections).
    // Off (the default): the reference's behaviour, the update runs with the unclipped gradient.
    void set_skip_nonfinite(bool on);
    // Activation recompute of attention in the model (TinyTransformer::set_recompute_attention);
    // a captured step graph is dropped and captured again with the new path.
    void set_recompute_attention(bool on);

    TinyTransformer& model() noexcept { return *model_; }
    optim::AdamW& optimizer() noexcept { return *opt_; }
    size_t batch() const noexcept { return batch_; }
    size_t length() const noexcept { return length_; }

private:
    std::unique_ptr<TinyTransformer> model_;
    std::unique_ptr<optim::AdamW> opt_;
    std::unique_ptr<DataParallel> dp_;
    float max_norm_;
    size_t batch_, length_;
    core::Tensor ids_, targets_, loss_;
    core::Tensor pinned_;   // host-side staging is done by the caller; kept for symmetry
    bool graph_eligible() const;
    void step_impl(const core::Tensor& ids, const core::Tensor& targets);
    ::CUgraphExec_st* graph_exec_ = nullptr;
    int64_t graph_launches_ = 0;
    int eager_steps_ = 0;
    bool use_graph_ = true;
    bool skip_nonfinite_ = false;
    void* capture_stream_ = nullptr;   // cudaStream_t the step is captured on
};

} // namespace veda::train
