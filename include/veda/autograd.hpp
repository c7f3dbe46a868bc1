// veda::autograd — the reference's reverse-mode tape (src/libs/autograd/Variable.h:31-119,
// Loss.h:43) over device tensors, plus fused training modules.
//
// Kept from the reference (same names, argument meaning and exception types):
//   Variable::leaf, backward() (starts at a scalar, reverse topological order, intermediate
//   gradients reset each pass, leaf gradients accumulate across passes), zero_grad(); the ops
//   add, mul, mul(scalar), sum, matmul, matmul_nt, silu, gelu, softmax, rms_normalize,
//   embedding, reshape, transpose, rope, cross_entropy; detail::unbroadcast.
// Changed for the device:
//   * an intermediate gradient is allocated on first contribution, and the first contribution is
//     aliased rather than copied (a node whose gradient is an alias copies before mutating), so
//     residual fan-out costs nothing;
//   * producers that can add in place (GEMM epilogues with beta = 1, the norm backward's
//     residual input, the embedding scatter) write straight into the destination gradient;
//   * a parameter's gradient may be a view into one flat fp32 arena (Variable::parameter), which
//     is what lets the optimiser and the data-parallel all-reduce work on whole buckets.
// Fused modules (one node each, B200 kernels): rms_norm (norm + gain), linear (x W^T over
// flattened tokens), attention (QK-norm + RoPE + causal GQA attention on a fused q|k|v buffer),
// swiglu (on a fused gate|up buffer), cross_entropy (streaming softmax-CE with the gradient
// formed in the same pass).
#pragma once

#include "veda/tensor.hpp"

#include <cstdint>
#include <functional>
#include <memory>
#include <string>
#include <vector>

namespace veda::autograd
{

struct Node
{
    core::Tensor value;
    core::Tensor grad;   // undefined until the first contribution (intermediates)
    std::vector<std::shared_ptr<Node>> parents;
    std::function<void(const core::Tensor& out_grad)> backward;
    bool requires_grad = false;
    bool grad_owned = true;    // false: grad aliases another tensor; copy before mutating
    bool grad_zero = false;    // leaf gradient buffer currently holds zeros
    bool is_leaf = false;

    explicit Node(core::Tensor v);
};

struct BackwardOptions
{
    // Keep intermediate gradients after the pass (the reference does); false frees each one as
    // soon as its node has propagated it.
    bool retain_intermediate_grads = true;
    // Called once per leaf when its gradient is final for this pass (every consumer has run).
    std::function<void(Node*)> on_leaf_ready;
};

class Variable
{
public:
    static Variable leaf(core::Tensor value, bool requires_grad = true);
    // A trainable leaf whose gradient is the given fp32 buffer (e.g. a view into a gradient
    // arena); the buffer is taken to hold zeros.
    static Variable parameter(core::Tensor value, core::Tensor grad);
    Variable() = default;
    explicit Variable(std::shared_ptr<Node> node) : node_(std::move(node)) {}

    const core::Tensor& value() const noexcept { return node_->value; }
    // The gradient (a zero tensor if nothing has been accumulated yet).
    const core::Tensor& grad() const;
    bool requires_grad() const noexcept { return node_->requires_grad; }
    const std::shared_ptr<Node>& node() const noexcept { return node_; }

    void backward();
    void backward(const BackwardOptions& options);
    void zero_grad();

private:
    std::shared_ptr<Node> node_;
};

Variable add(const Variable& a, const Variable& b);
Variable mul(const Variable& a, const Variable& b);
Variable mul(const Variable& a, float scalar);
Variable sum(const Variable& x);
Variable matmul(const Variable& a, const Variable& b);
Variable matmul_nt(const Variable& a, const Variable& b);
Variable silu(const Variable& x);
Variable gelu(const Variable& x);
Variable softmax(const Variable& x, size_t dim);
Variable rms_normalize(const Variable& x, float eps);
Variable embedding(const Variable& table, const std::vector<int64_t>& ids,
                   const core::Shape& id_shape);
Variable reshape(const Variable& x, const core::Shape& shape);
Variable transpose(const Variable& x, size_t a, size_t b);
Variable rope(const Variable& x, const core::Tensor& cosines, const core::Tensor& sines);
// Mean cross-entropy over lanes; targets on the host, validated like Loss.cpp:21-47.
Variable cross_entropy(const Variable& logits, const std::vector<int64_t>& targets);

// ---- fused modules --------------------------------------------------------------------------
// mul(rms_normalize(x, eps), gamma) over the last dim.
Variable rms_norm(const Variable& x, const Variable& gamma, float eps);
// rms_norm(add(x, r), gamma, eps) with the sum formed in the same pass; *sum receives the
// add(x, r) node (the residual stream), which the result's node takes as its input.
Variable add_rms_norm(const Variable& x, const Variable& r, const Variable& gamma, float eps,
                      Variable* sum);
// matmul_nt(x, w) with x [.., in] flattened to rows and w [out, in].
Variable linear(const Variable& x, const Variable& w);
// Qwen3 attention core on a fused projection qkv [B*T, (H + 2 Hkv) * Dh] (q | k | v columns):
// rope(mul(rms_normalize(q_h), q_norm)) and the same for k, causal softmax(q k^T / sqrt(Dh)) v
// with GQA; returns the context [B*T, H*Dh] (src/libs/train/Model.cpp:154-194).
Variable attention(const Variable& qkv, const Variable& q_norm, const Variable& k_norm,
                   const core::Tensor& cosines, const core::Tensor& sines, size_t batch,
                   size_t length, size_t heads, size_t kv_heads, size_t head_dim, float eps);
// attention(...) followed by linear(context, o), as one node that keeps only the projection, the
// gains and the log-sum-exp: the backward forms q, k (norm + RoPE) and the context again before
// the output projection's and the attention's backward (activation recompute of attention).
Variable attention_output(const Variable& qkv, const Variable& q_norm, const Variable& k_norm,
                          const Variable& o, const core::Tensor& cosines, const core::Tensor& sines,
                          size_t batch, size_t length, size_t heads, size_t kv_heads,
                          size_t head_dim, float eps);
// mul(silu(gate), up) on a fused gate|up buffer [rows, 2F] -> [rows, F].
Variable swiglu(const Variable& gate_up);
// The feed-forward block linear(swiglu(linear(x, gate_up)), down) with gate_up [2F, D] (gate rows,
// then up rows) and down [D, F], as one node: in bf16 the gate|up GEMM writes h as well and the
// down projection's input-gradient GEMM writes dgate|up (SwiGLU in the GEMM epilogues, the same
// bits); other dtypes and shapes run the three ops.
Variable mlp(const Variable& x, const Variable& gate_up, const Variable& down);
// Token ids already on the device (int64 [count]); ids are checked on the device and an
// out-of-range id raises std::out_of_range at the next synchronisation point.
Variable embedding_device(const Variable& table, const core::Tensor& ids);
// Receives the ids (int64 [count] on the device) and the output gradient rows [count, D] of an
// embedding_device_rows node.
using RowsSink = std::function<void(const core::Tensor& ids, size_t count, const core::Tensor& rows)>;
// embedding_device whose backward hands the ids and the gradient rows to `sink` instead of
// scattering them into the table's gradient. The table is not an input of the node, so with a
// tied LM head the table's gradient is final as soon as the head's backward has run (a
// data-parallel step exchanges it then, and the scattered rows separately at the end).
Variable embedding_device_rows(const Variable& table, const core::Tensor& ids, RowsSink sink);
// Mean cross-entropy with device targets (int64 [lanes]).
Variable cross_entropy_device(const Variable& logits, const core::Tensor& targets);

// Central finite differences against the tape's gradient (src/libs/autograd/GradientCheck.h):
// dL/dx_i ~ (L(x + h e_i) - L(x - h e_i)) / 2h for every element of `at`, compared relatively per
// element with max(|numeric|, |analytic|, 1e-3) as the scale. ok iff the worst relative
// difference is within `tolerance`; loss_of must return a scalar. Costs 2n forward passes: for
// small tensors in tests.
struct GradientCheck
{
    bool ok = true;
    double worst_relative = 0.0;
    size_t worst_index = 0;
    double analytic = 0.0;
    double numeric = 0.0;
    std::string message;
};

GradientCheck check_gradient(const std::function<Variable(const Variable&)>& loss_of,
                             const core::Tensor& at, float step = 1e-2f, double tolerance = 2e-2);

namespace detail
{
core::Tensor unbroadcast(const core::Tensor& gradient, const core::Shape& target);
// The node's gradient made private and ready to be written: *fresh is true when the buffer
// holds no contribution yet (an overwrite is then correct), false when it must be added to.
core::Tensor& grad_target(Node& node, bool* fresh, core::DType dtype);
// node.grad += g (the first contribution is aliased).
void accumulate(Node& node, const core::Tensor& g);
// Device error flag checked after launches that validate indices on the device.
int* device_flag();
void raise_device_flag();
} // namespace detail

} // namespace veda::autograd
