// veda::autograd on the device: the tape of src/libs/autograd/Variable.cpp and the op
// backwards of Variable.cpp / NonLinear.cpp / Views.cpp / Loss.cpp, each launching the kernels
// behind include/veda_cuda.h. The arithmetic of every op is the reference's; see the kernels for
// the line-by-line correspondence.
#include "veda/autograd.hpp"
#include "veda/ops.hpp"

#include "veda/profile.hpp"
#include "veda_cuda.h"

#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <limits>
#include <mutex>
#include <stdexcept>
#include <unordered_map>
#include <unordered_set>

namespace veda::autograd
{

using core::DType;
using core::Shape;
using core::Tensor;

namespace
{

veda_stream_t S() { return current_stream(); }
int dt(DType d) { return static_cast<int>(d); }

thread_local const core::Storage* g_seed_storage = nullptr;

void cuda_check(cudaError_t e, const char* what)
{
    if (e != cudaSuccess)
    {
        throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
    }
}

Tensor make_contiguous(const Tensor& t) { return t.is_contiguous() ? t : core::contiguous(t); }

// A second stream per device for work that may run beside the current stream (a Linear's weight
// gradient beside its input gradient), with the two events that fork it off and join it back.
struct SideStream
{
    cudaStream_t stream = nullptr;
    cudaEvent_t fork = nullptr, join = nullptr;
};

SideStream& side_stream()
{
    thread_local SideStream sides[64];
    int device = 0;
    cuda_check(cudaGetDevice(&device), "side stream: device");
    SideStream& f = sides[device & 63];
    if (f.stream == nullptr)
    {
        cuda_check(cudaStreamCreateWithFlags(&f.stream, cudaStreamNonBlocking), "side stream");
        cuda_check(cudaEventCreateWithFlags(&f.fork, cudaEventDisableTiming), "fork event");
        cuda_check(cudaEventCreateWithFlags(&f.join, cudaEventDisableTiming), "join event");
    }
    return f;
}

// The input- and weight-gradient GEMMs of a Linear run concurrently (VEDA_GEMM_OVERLAP=0 runs
// them one after the other): both are persistent kernels, so the second one's tiles fill the SMs
// the first one's last partial wave leaves idle.
bool gemm_overlap_enabled()
{
    static const bool on = [] {
        const char* v = std::getenv("VEDA_GEMM_OVERLAP");
        return !(v != nullptr && v[0] == '0');
    }();
    return on;
}

Tensor as_dtype(const Tensor& t, DType d)
{
    return t.dtype() == d ? make_contiguous(t) : core::to_dtype(t, d);
}

void memset_zero(const Tensor& t)
{
    if (t.numel() == 0)
    {
        return;
    }
    if (!t.is_contiguous())
    {
        throw std::logic_error("autograd: cannot clear a non-contiguous gradient");
    }
    cuda_check(cudaMemsetAsync(t.data_ptr(), 0, t.numel() * core::dtype_size(t.dtype()),
                               reinterpret_cast<cudaStream_t>(S())),
               "cudaMemsetAsync");
}

Variable make(const std::vector<Variable>& inputs, Tensor value,
              std::function<void(const Tensor&)> backward)
{
    bool any = false;
    for (const Variable& v : inputs)
    {
        any = any || v.requires_grad();
    }
    if (!any)
    {
        return Variable::leaf(std::move(value), false);
    }
    auto node = std::make_shared<Node>(std::move(value));
    node->requires_grad = true;
    for (const Variable& v : inputs)
    {
        node->parents.push_back(v.node());
    }
    node->backward = std::move(backward);
    return Variable(std::move(node));
}

// numpy broadcasting: output shape and per-input strides (0 on broadcast axes), aligned right.
Shape broadcast_shape(const Shape& a, const Shape& b)
{
    const size_t r = std::max(a.rank(), b.rank());
    std::vector<size_t> out(r);
    for (size_t k = 0; k < r; ++k)
    {
        const size_t da = k < r - a.rank() ? 1 : a[k - (r - a.rank())];
        const size_t db = k < r - b.rank() ? 1 : b[k - (r - b.rank())];
        if (da != db && da != 1 && db != 1)
        {
            throw std::invalid_argument("broadcast: shapes " + a.to_string() + " and " +
                                        b.to_string() + " do not broadcast");
        }
        out[k] = da == 1 ? db : da;
    }
    return Shape(out);
}

std::vector<int64_t> broadcast_strides(const Tensor& t, const Shape& out)
{
    const size_t r = out.rank();
    std::vector<int64_t> s(r, 0);
    for (size_t k = 0; k < t.rank(); ++k)
    {
        const size_t o = k + (r - t.rank());
        s[o] = t.shape()[k] == 1 && out[o] != 1 ? 0 : static_cast<int64_t>(t.strides()[k]);
    }
    return s;
}

Tensor binary(int op, const Tensor& a, const Tensor& b0)
{
    const Tensor b = b0.dtype() == a.dtype() ? b0 : core::to_dtype(b0, a.dtype());
    const Shape out_shape = broadcast_shape(a.shape(), b.shape());
    Tensor out = Tensor::empty(out_shape, a.dtype());
    if (out.numel() == 0)
    {
        return out;
    }
    std::vector<int64_t> shape(out_shape.dims().begin(), out_shape.dims().end());
    std::vector<int64_t> sa = broadcast_strides(a, out_shape);
    std::vector<int64_t> sb = broadcast_strides(b, out_shape);
    if (shape.empty())
    {
        shape = {1};
        sa = {0};
        sb = {0};
    }
    // strides are relative to each tensor's own first element
    check(veda_binary(op, a.data_ptr(), sa.data(), b.data_ptr(), sb.data(), out.data_ptr(),
                      shape.data(), static_cast<int>(shape.size()), dt(a.dtype()), S()),
          op == 0 ? "add" : "mul");
    return out;
}

Tensor scale(const Tensor& x, float s)
{
    const Tensor c = make_contiguous(x);
    Tensor out = Tensor::empty(c.shape(), c.dtype());
    check(veda_scale(c.data_ptr(), s, out.data_ptr(), static_cast<int64_t>(c.numel()),
                     dt(c.dtype()), S()),
          "mul(scalar)");
    return out;
}

// ---- matmul helpers ----------------------------------------------------------------------------
struct MatView
{
    Tensor t;          // contiguous in its last two dims
    size_t rows, cols;
    int64_t batch_stride;   // elements between batch entries (0 = broadcast)
};

std::vector<size_t> batch_dims(const Shape& s)
{
    return std::vector<size_t>(s.dims().begin(), s.dims().end() - 2);
}

Shape batch_broadcast(const Shape& a, const Shape& b)
{
    return broadcast_shape(Shape(batch_dims(a)), Shape(batch_dims(b)));
}

// Prepares an operand for a batched GEMM over `out_batch` entries: contiguous, with a single
// batch stride (0 when the operand is not batched); materialises any other broadcast pattern.
MatView mat_operand(const Tensor& t0, const Shape& out_batch)
{
    Tensor t = make_contiguous(t0);
    const size_t rows = t.shape()[t.rank() - 2], cols = t.shape()[t.rank() - 1];
    const Shape own(batch_dims(t.shape()));
    if (own.size() == 1)
    {
        return {t, rows, cols, 0};
    }
    if (own.size() == out_batch.size() && batch_dims(t.shape()).size() == out_batch.rank() &&
        own == out_batch)
    {
        return {t, rows, cols, static_cast<int64_t>(rows * cols)};
    }
    // expand to the full batch shape
    std::vector<size_t> full = out_batch.dims();
    full.push_back(rows);
    full.push_back(cols);
    const Shape fs(full);
    std::vector<int64_t> shape(full.begin(), full.end());
    std::vector<int64_t> strides = broadcast_strides(t, fs);
    Tensor e = Tensor::empty(fs, t.dtype());
    check(veda_copy_strided(t.data_ptr(), dt(t.dtype()), strides.data(), 0, e.data_ptr(),
                            dt(t.dtype()), shape.data(), static_cast<int>(shape.size()), S()),
          "matmul: broadcast");
    return {e, rows, cols, static_cast<int64_t>(rows * cols)};
}

// C = op(A) op(B) over a broadcast batch; op 0 NT (B is [N,K]), 1 NN (B is [K,N]).
Tensor batched_product(int op, const Tensor& a, const Tensor& b, DType out_dtype)
{
    if (a.rank() < 2 || b.rank() < 2)
    {
        throw std::invalid_argument("matmul: operands need rank >= 2, got " +
                                    a.shape().to_string() + " and " + b.shape().to_string());
    }
    const size_t M = a.shape()[a.rank() - 2], K = a.shape()[a.rank() - 1];
    const size_t kb = op == 0 ? b.shape()[b.rank() - 1] : b.shape()[b.rank() - 2];
    const size_t N = op == 0 ? b.shape()[b.rank() - 2] : b.shape()[b.rank() - 1];
    if (K != kb)
    {
        throw std::invalid_argument("matmul: inner dimensions differ: " + a.shape().to_string() +
                                    " and " + b.shape().to_string());
    }
    if (a.dtype() != b.dtype())
    {
        throw std::invalid_argument("matmul: operand dtypes differ");
    }
    const Shape out_batch = batch_broadcast(a.shape(), b.shape());
    std::vector<size_t> od = out_batch.dims();
    od.push_back(M);
    od.push_back(N);
    Tensor out = Tensor::empty(Shape(od), out_dtype);
    if (out.numel() == 0)
    {
        return out;
    }
    const Tensor bc = make_contiguous(b);
    // a batched activation times an unbatched matrix: one GEMM over all rows
    if (Shape(batch_dims(bc.shape())).size() == 1 && Shape(batch_dims(a.shape())) == out_batch)
    {
        const Tensor ac = make_contiguous(a);
        const int64_t rows = static_cast<int64_t>(ac.numel() / K);
        const int rc = op == 0 ? veda_gemm_nt(rows, N, K, ac.data_ptr(), K, bc.data_ptr(), K,
                                              out.data_ptr(), N, dt(a.dtype()), dt(out_dtype),
                                              1.0f, 0.0f, S())
                               : veda_gemm_nn(rows, N, K, ac.data_ptr(), K, bc.data_ptr(), N,
                                              out.data_ptr(), N, dt(a.dtype()), dt(out_dtype),
                                              1.0f, 0.0f, S());
        check(rc, "matmul");
        return out;
    }
    const MatView A = mat_operand(a, out_batch);
    const MatView B = mat_operand(b, out_batch);
    check(veda_gemm_batched(op == 0 ? 0 : 1, static_cast<int64_t>(out_batch.size()), M, N, K,
                            A.t.data_ptr(), K, A.batch_stride, B.t.data_ptr(),
                            op == 0 ? K : N, B.batch_stride, out.data_ptr(), N,
                            static_cast<int64_t>(M * N), dt(a.dtype()), dt(out_dtype), 1.0f,
                            0.0f, S()),
          "matmul");
    return out;
}

// dW-style product: C[P, Q] = sum over all leading rows of X[.., P]^T Y[.., Q] (the TN GEMM),
// which is matmul(transpose(x), y) followed by the unbroadcast batch sum of Variable.cpp:342-343.
Tensor weight_product(const Tensor& x, const Tensor& y, DType out_dtype)
{
    const Tensor xc = make_contiguous(x), yc = make_contiguous(y);
    const size_t P = xc.shape()[xc.rank() - 1], Q = yc.shape()[yc.rank() - 1];
    const int64_t rows = static_cast<int64_t>(xc.numel() / P);
    Tensor out = Tensor::empty(Shape({P, Q}), out_dtype);
    check(veda_gemm_tn(P, Q, rows, xc.data_ptr(), P, yc.data_ptr(), Q, out.data_ptr(), Q,
                       dt(xc.dtype()), dt(out_dtype), 1.0f, 0.0f, S()),
          "matmul backward");
    return out;
}

Tensor transpose_last(const Tensor& t) { return t.transpose(t.rank() - 2, t.rank() - 1); }

} // namespace

// ---- tape ----------------------------------------------------------------------------------------
Node::Node(Tensor v) : value(std::move(v)) {}

Variable Variable::leaf(Tensor value, bool requires_grad)
{
    auto node = std::make_shared<Node>(std::move(value));
    node->requires_grad = requires_grad;
    node->is_leaf = true;
    if (requires_grad)
    {
        // as in the reference, a leaf that takes a gradient has a zero fp32 gradient buffer from
        // the start (callers may read or write node()->grad before any backward)
        node->grad = Tensor(node->value.shape(), DType::F32);
        node->grad_owned = true;
        node->grad_zero = true;
    }
    return Variable(std::move(node));
}

Variable Variable::parameter(Tensor value, Tensor grad)
{
    if (grad.shape() != value.shape() || grad.dtype() != DType::F32)
    {
        throw std::invalid_argument("Variable::parameter: the gradient must be fp32 of shape " +
                                    value.shape().to_string());
    }
    auto node = std::make_shared<Node>(std::move(value));
    node->requires_grad = true;
    node->is_leaf = true;
    node->grad = std::move(grad);
    node->grad_zero = true;
    return Variable(std::move(node));
}

const Tensor& Variable::grad() const
{
    if (!node_->grad.defined())
    {
        node_->grad = Tensor(node_->value.shape(),
                             node_->is_leaf ? DType::F32 : node_->value.dtype());
        node_->grad_owned = true;
        node_->grad_zero = true;
    }
    return node_->grad;
}

void Variable::zero_grad()
{
    std::unordered_set<Node*> seen;
    std::vector<Node*> pending{node_.get()};
    while (!pending.empty())
    {
        Node* node = pending.back();
        pending.pop_back();
        if (!seen.insert(node).second)
        {
            continue;
        }
        if (node->is_leaf && node->grad.defined() && node->grad_owned)
        {
            memset_zero(node->grad);
            node->grad_zero = true;
        }
        else
        {
            node->grad = Tensor();
            node->grad_owned = true;
            node->grad_zero = false;
        }
        for (const auto& parent : node->parents)
        {
            pending.push_back(parent.get());
        }
    }
}

void Variable::backward() { backward(BackwardOptions{}); }

void Variable::backward(const BackwardOptions& options)
{
    if (node_->value.numel() != 1)
    {
        throw std::runtime_error("autograd: backward() starts at a scalar, got " +
                                 node_->value.shape().to_string());
    }
    // reverse topological order (iterative post-order DFS)
    std::vector<Node*> order;
    std::unordered_set<Node*> seen;
    std::vector<std::pair<Node*, size_t>> stack{{node_.get(), 0}};
    seen.insert(node_.get());
    while (!stack.empty())
    {
        auto& [node, next] = stack.back();
        if (next < node->parents.size())
        {
            Node* parent = node->parents[next++].get();
            if (seen.insert(parent).second)
            {
                stack.push_back({parent, 0});
            }
            continue;
        }
        order.push_back(node);
        stack.pop_back();
    }
    std::unordered_map<Node*, int> pending;
    for (Node* node : order)
    {
        if (node->backward)
        {
            node->grad = Tensor();   // intermediates are scratch for one pass
            node->grad_owned = true;
            node->grad_zero = false;
            for (const auto& parent : node->parents)
            {
                if (parent->is_leaf && parent->requires_grad)
                {
                    ++pending[parent.get()];
                }
            }
        }
    }
    // seed 1 at the scalar
    {
        Tensor seed = Tensor::empty(node_->value.shape(), node_->value.dtype());
        check(veda_fill(seed.data_ptr(), 1.0f, 1, dt(seed.dtype()), S()), "backward: seed");
        g_seed_storage = seed.storage().get();
        if (node_->backward)
        {
            node_->grad = seed;
        }
        else
        {
            detail::accumulate(*node_, seed);
        }
    }
    for (auto it = order.rbegin(); it != order.rend(); ++it)
    {
        Node* node = *it;
        if (!node->backward)
        {
            continue;
        }
        if (node->grad.defined())
        {
            node->backward(node->grad);
        }
        for (const auto& parent : node->parents)
        {
            if (parent->is_leaf && parent->requires_grad)
            {
                auto p = pending.find(parent.get());
                if (p != pending.end() && --p->second == 0 && options.on_leaf_ready)
                {
                    options.on_leaf_ready(parent.get());
                }
            }
        }
        if (!options.retain_intermediate_grads && node != node_.get())
        {
            node->grad = Tensor();
        }
    }
    g_seed_storage = nullptr;
}

namespace detail
{

Tensor& grad_target(Node& node, bool* fresh, DType dtype)
{
    if (!node.grad.defined())
    {
        node.grad = Tensor::empty(node.value.shape(), node.is_leaf ? DType::F32 : dtype);
        node.grad_owned = true;
        node.grad_zero = false;
        *fresh = true;
        return node.grad;
    }
    if (!node.grad_owned)
    {
        node.grad = core::contiguous(node.grad);
        node.grad_owned = true;
    }
    *fresh = node.grad_zero;
    node.grad_zero = false;
    return node.grad;
}

void accumulate(Node& node, const Tensor& g)
{
    if (g.shape() != node.value.shape())
    {
        throw std::runtime_error("autograd: a gradient of shape " + g.shape().to_string() +
                                 " does not fit a value of shape " +
                                 node.value.shape().to_string());
    }
    const DType want = node.is_leaf ? DType::F32 : node.value.dtype();
    if (!node.grad.defined())
    {
        node.grad = g.dtype() == want ? g : core::to_dtype(g, want);
        node.grad_owned = g.dtype() != want;
        node.grad_zero = false;
        return;
    }
    if (node.grad_zero)
    {
        // the buffer holds zeros: a copy is the sum
        std::vector<int64_t> shape(g.shape().dims().begin(), g.shape().dims().end());
        std::vector<int64_t> strides(g.strides().begin(), g.strides().end());
        if (shape.empty())
        {
            shape = {1};
            strides = {1};
        }
        if (!node.grad.is_contiguous())
        {
            throw std::logic_error("autograd: gradient buffer is not contiguous");
        }
        check(veda_copy_strided(g.storage()->data(), dt(g.dtype()), strides.data(),
                                static_cast<int64_t>(g.offset()), node.grad.data_ptr(),
                                dt(node.grad.dtype()), shape.data(),
                                static_cast<int>(shape.size()), S()),
              "accumulate");
        node.grad_zero = false;
        return;
    }
    if (!node.grad_owned)
    {
        node.grad = core::contiguous(node.grad);
        node.grad_owned = true;
    }
    const Tensor gc = make_contiguous(g);
    check(veda_accumulate(node.grad.data_ptr(), dt(node.grad.dtype()), gc.data_ptr(),
                          dt(gc.dtype()), static_cast<int64_t>(gc.numel()), S()),
          "accumulate");
}

Tensor unbroadcast(const Tensor& gradient, const Shape& target)
{
    if (gradient.shape() == target)
    {
        return gradient;
    }
    const Tensor g = make_contiguous(gradient);
    const size_t r = g.rank();
    if (target.rank() > r)
    {
        throw std::runtime_error("unbroadcast: target " + target.to_string() +
                                 " has more axes than " + g.shape().to_string());
    }
    std::vector<int64_t> shape(g.shape().dims().begin(), g.shape().dims().end());
    std::vector<int64_t> tgt(r, 1);
    for (size_t k = 0; k < target.rank(); ++k)
    {
        tgt[k + (r - target.rank())] = static_cast<int64_t>(target[k]);
    }
    Tensor out = Tensor::empty(target, g.dtype());
    check(veda_unbroadcast(g.data_ptr(), shape.data(), tgt.data(), static_cast<int>(r),
                           out.data_ptr(), dt(g.dtype()), S()),
          "unbroadcast");
    return out;
}

int* device_flag()
{
    static int* flags[64] = {nullptr};
    static std::mutex mu;
    int device = 0;
    cudaGetDevice(&device);
    std::lock_guard<std::mutex> lock(mu);
    if (flags[device] == nullptr)
    {
        cuda_check(cudaMalloc(&flags[device], sizeof(int)), "device flag");
        cuda_check(cudaMemset(flags[device], 0, sizeof(int)), "device flag");
    }
    return flags[device];
}

void raise_device_flag()
{
    int* f = device_flag();
    int value = 0;
    cuda_check(cudaMemcpyAsync(&value, f, sizeof(int), cudaMemcpyDeviceToHost,
                               reinterpret_cast<cudaStream_t>(S())),
               "device flag");
    cuda_check(cudaStreamSynchronize(reinterpret_cast<cudaStream_t>(S())), "device flag");
    if (value != 0)
    {
        cuda_check(cudaMemsetAsync(f, 0, sizeof(int), reinterpret_cast<cudaStream_t>(S())),
                   "device flag");
        if (value == VEDA_ERR_OUT_OF_RANGE)
        {
            throw std::out_of_range("a token id or target is outside the vocabulary");
        }
        throw std::runtime_error("device-side check failed (status " + std::to_string(value) + ")");
    }
}

} // namespace detail

using detail::accumulate;
using detail::grad_target;
using detail::unbroadcast;

// ---- reference ops ----------------------------------------------------------------------------
Variable add(const Variable& a, const Variable& b)
{
    Tensor value = binary(0, a.value(), b.value());
    auto left = a.node(), right = b.node();
    return make({a, b}, std::move(value), [left, right](const Tensor& g) {
        if (left->requires_grad) accumulate(*left, unbroadcast(g, left->value.shape()));
        if (right->requires_grad) accumulate(*right, unbroadcast(g, right->value.shape()));
    });
}

Variable mul(const Variable& a, const Variable& b)
{
    Tensor value = binary(1, a.value(), b.value());
    auto left = a.node(), right = b.node();
    return make({a, b}, std::move(value), [left, right](const Tensor& g) {
        if (left->requires_grad)
            accumulate(*left, unbroadcast(binary(1, g, right->value), left->value.shape()));
        if (right->requires_grad)
            accumulate(*right, unbroadcast(binary(1, g, left->value), right->value.shape()));
    });
}

Variable mul(const Variable& a, float scalar)
{
    Tensor value = scale(a.value(), scalar);
    auto input = a.node();
    return make({a}, std::move(value), [input, scalar](const Tensor& g) {
        accumulate(*input, scale(g, scalar));
    });
}

Variable sum(const Variable& x)
{
    Tensor total = Tensor::empty(Shape({}), DType::F32);
    const Tensor c = make_contiguous(x.value());
    check(veda_sum(c.data_ptr(), static_cast<int64_t>(c.numel()), static_cast<float*>(total.data_ptr()),
                   dt(c.dtype()), S()),
          "sum");
    auto input = x.node();
    return make({x}, std::move(total), [input](const Tensor& g) {
        // every element contributed once: broadcast the scalar back (Variable.cpp:277-285)
        const Shape& s = input->value.shape();
        Tensor spread = Tensor::empty(s, input->value.dtype());
        if (spread.numel() > 0)
        {
            std::vector<int64_t> shape(s.dims().begin(), s.dims().end());
            std::vector<int64_t> zeros(shape.size(), 0);
            if (shape.empty())
            {
                shape = {1};
                zeros = {0};
            }
            check(veda_copy_strided(g.storage()->data(), dt(g.dtype()), zeros.data(),
                                    static_cast<int64_t>(g.offset()), spread.data_ptr(),
                                    dt(spread.dtype()), shape.data(),
                                    static_cast<int>(shape.size()), S()),
                  "sum backward");
        }
        accumulate(*input, spread);
    });
}

Variable matmul(const Variable& a, const Variable& b)
{
    Tensor value = batched_product(1, a.value(), b.value(), a.value().dtype());
    auto left = a.node(), right = b.node();
    return make({a, b}, std::move(value), [left, right](const Tensor& g) {
        if (left->requires_grad)
        {
            // dA = G . B^T  (Variable.cpp:307-312)
            accumulate(*left,
                       unbroadcast(batched_product(0, g, right->value, g.dtype()),
                                   left->value.shape()));
        }
        if (right->requires_grad)
        {
            // dB = A^T . G, summed over broadcast batch axes (Variable.cpp:313-319)
            const bool flat = right->value.rank() == 2;
            if (flat)
            {
                accumulate(*right, weight_product(left->value, g,
                                                  right->is_leaf ? DType::F32 : g.dtype()));
            }
            else
            {
                const Tensor at = make_contiguous(transpose_last(left->value));
                accumulate(*right, unbroadcast(batched_product(1, at, g, g.dtype()),
                                               right->value.shape()));
            }
        }
    });
}

Variable matmul_nt(const Variable& a, const Variable& b)
{
    Tensor value = batched_product(0, a.value(), b.value(), a.value().dtype());
    auto left = a.node(), right = b.node();
    return make({a, b}, std::move(value), [left, right](const Tensor& g) {
        if (left->requires_grad)
        {
            // dA = G . B  (Variable.cpp:334-339)
            accumulate(*left, unbroadcast(batched_product(1, g, right->value, g.dtype()),
                                          left->value.shape()));
        }
        if (right->requires_grad)
        {
            // dB = G^T . A (Variable.cpp:340-344)
            if (right->value.rank() == 2)
            {
                accumulate(*right, weight_product(g, left->value,
                                                  right->is_leaf ? DType::F32 : g.dtype()));
            }
            else
            {
                const Tensor gt = make_contiguous(transpose_last(g));
                accumulate(*right, unbroadcast(batched_product(1, gt, left->value, g.dtype()),
                                               right->value.shape()));
            }
        }
    });
}

Variable silu(const Variable& x)
{
    const Tensor xc = make_contiguous(x.value());
    Tensor value = Tensor::empty(xc.shape(), xc.dtype());
    check(veda_silu_fwd(xc.data_ptr(), value.data_ptr(), static_cast<int64_t>(xc.numel()),
                        dt(xc.dtype()), S()),
          "silu");
    auto input = x.node();
    return make({x}, std::move(value), [input, xc](const Tensor& g) {
        const Tensor gc = as_dtype(g, xc.dtype());
        Tensor d = Tensor::empty(xc.shape(), xc.dtype());
        check(veda_silu_bwd(xc.data_ptr(), gc.data_ptr(), d.data_ptr(),
                            static_cast<int64_t>(xc.numel()), dt(xc.dtype()), S()),
              "silu backward");
        accumulate(*input, d);
    });
}

Variable gelu(const Variable& x)
{
    const Tensor xc = make_contiguous(x.value());
    Tensor value = Tensor::empty(xc.shape(), xc.dtype());
    check(veda_gelu_fwd(xc.data_ptr(), value.data_ptr(), static_cast<int64_t>(xc.numel()),
                        dt(xc.dtype()), S()),
          "gelu");
    auto input = x.node();
    return make({x}, std::move(value), [input, xc](const Tensor& g) {
        const Tensor gc = as_dtype(g, xc.dtype());
        Tensor d = Tensor::empty(xc.shape(), xc.dtype());
        check(veda_gelu_bwd(xc.data_ptr(), gc.data_ptr(), d.data_ptr(),
                            static_cast<int64_t>(xc.numel()), dt(xc.dtype()), S()),
              "gelu backward");
        accumulate(*input, d);
    });
}

namespace
{
// Moves axis `dim` last (materialised) so a per-lane kernel sees contiguous lanes.
Tensor to_last(const Tensor& t, size_t dim)
{
    return dim + 1 == t.rank() ? make_contiguous(t)
                               : core::contiguous(t.transpose(dim, t.rank() - 1));
}
Tensor from_last(const Tensor& t, size_t dim)
{
    return dim + 1 == t.rank() ? t : core::contiguous(t.transpose(dim, t.rank() - 1));
}
} // namespace

Variable softmax(const Variable& x, size_t dim)
{
    if (dim >= x.value().rank())
    {
        throw std::invalid_argument("softmax: dimension " + std::to_string(dim) +
                                    " is out of range for shape " + x.value().shape().to_string());
    }
    const Tensor xl = to_last(x.value(), dim);
    const size_t len = xl.shape()[xl.rank() - 1];
    const size_t lanes = len == 0 ? 0 : xl.numel() / len;
    Tensor yl = Tensor::empty(xl.shape(), xl.dtype());
    check(veda_softmax_fwd(xl.data_ptr(), yl.data_ptr(), lanes, len, dt(xl.dtype()), S()),
          "softmax");
    Tensor value = from_last(yl, dim);
    auto input = x.node();
    return make({x}, std::move(value), [input, yl, dim, lanes, len](const Tensor& g) {
        const Tensor gl = to_last(as_dtype(g, yl.dtype()), dim);
        Tensor dl = Tensor::empty(yl.shape(), yl.dtype());
        check(veda_softmax_bwd(yl.data_ptr(), gl.data_ptr(), dl.data_ptr(), lanes, len,
                               dt(yl.dtype()), S()),
              "softmax backward");
        accumulate(*input, from_last(dl, dim));
    });
}

Variable rms_normalize(const Variable& x, float eps)
{
    if (x.value().rank() == 0)
    {
        throw std::invalid_argument("rms_normalize: a rank-0 tensor has no last dimension");
    }
    const Tensor xc = make_contiguous(x.value());
    const size_t n = xc.shape()[xc.rank() - 1];
    const size_t rows = n == 0 ? 0 : xc.numel() / n;
    Tensor value = Tensor::empty(xc.shape(), xc.dtype());
    if (rows > 0)
    {
        check(veda_rmsnorm_fwd(xc.data_ptr(), n, nullptr, value.data_ptr(), n, rows, n, eps,
                               dt(xc.dtype()), S()),
              "rms_normalize");
    }
    auto input = x.node();
    return make({x}, std::move(value), [input, xc, n, rows, eps](const Tensor& g) {
        if (rows == 0) return;
        const Tensor gc = as_dtype(g, xc.dtype());
        Tensor d = Tensor::empty(xc.shape(), xc.dtype());
        check(veda_rmsnorm_bwd(xc.data_ptr(), n, nullptr, gc.data_ptr(), n, nullptr, 0,
                               d.data_ptr(), n, nullptr, nullptr, 0, rows, n, eps, dt(xc.dtype()),
                               S()),
              "rms_normalize backward");
        accumulate(*input, d);
    });
}

namespace
{
// int64 ids on the device, carried by an fp32 tensor of twice the length (8 bytes per id).
Tensor upload_ids(const std::vector<int64_t>& ids)
{
    Tensor raw = Tensor::empty(Shape({ids.size() * 2}), DType::F32);
    if (!ids.empty())
    {
        cuda_check(cudaMemcpyAsync(raw.data_ptr(), ids.data(), ids.size() * sizeof(int64_t),
                                   cudaMemcpyHostToDevice, reinterpret_cast<cudaStream_t>(S())),
                   "ids upload");
    }
    return raw;
}

Variable embedding_impl(const Variable& table, const Tensor& ids_raw, size_t count,
                        const Shape& out_shape, bool device_check)
{
    const size_t V = table.value().shape()[0], D = table.value().shape()[1];
    const Tensor tc = make_contiguous(table.value());
    Tensor value = Tensor::empty(out_shape, tc.dtype());
    const int64_t* ids = static_cast<const int64_t*>(ids_raw.data_ptr());
    check(veda_embedding_fwd(ids, count, tc.data_ptr(), V, D, value.data_ptr(), D,
                             device_check ? detail::device_flag() : nullptr, dt(tc.dtype()), S()),
          "embedding");
    auto input = table.node();
    return make({table}, std::move(value), [input, ids_raw, count, V, D](const Tensor& g) {
        // scatter-add in position order (NonLinear.cpp:245-252): deterministic, bit-exact
        bool fresh = false;
        Tensor& dt_ = grad_target(*input, &fresh, DType::F32);
        if (dt_.dtype() != DType::F32)
        {
            throw std::logic_error("embedding: the table gradient must be fp32");
        }
        if (fresh)
        {
            memset_zero(dt_);
        }
        const Tensor gc = make_contiguous(g);
        const size_t ws_bytes = veda_embedding_bwd_workspace(count);
        Tensor ws = Tensor::empty(Shape({(ws_bytes + 3) / 4}), DType::F32);
        check(veda_embedding_bwd(static_cast<const int64_t*>(ids_raw.data_ptr()), count,
                                 gc.data_ptr(), D, V, D, static_cast<float*>(dt_.data_ptr()), 1,
                                 ws.data_ptr(), ws_bytes, dt(gc.dtype()), S()),
              "embedding backward");
    });
}
} // namespace

Variable embedding(const Variable& table, const std::vector<int64_t>& ids, const Shape& id_shape)
{
    if (table.value().rank() != 2)
    {
        throw std::invalid_argument("autograd::embedding: the table must be rank 2 [V, D], got " +
                                    table.value().shape().to_string());
    }
    if (ids.size() != id_shape.size())
    {
        throw std::invalid_argument("autograd::embedding: " + std::to_string(ids.size()) +
                                    " ids for a shape " + id_shape.to_string());
    }
    const size_t V = table.value().shape()[0];
    for (int64_t id : ids)
    {
        if (id < 0 || static_cast<size_t>(id) >= V)
        {
            throw std::out_of_range("autograd::embedding: token id " + std::to_string(id) +
                                    " is outside a vocabulary of " + std::to_string(V));
        }
    }
    std::vector<size_t> dims = id_shape.dims();
    dims.push_back(table.value().shape()[1]);
    return embedding_impl(table, upload_ids(ids), ids.size(), Shape(dims), false);
}

Variable embedding_device(const Variable& table, const Tensor& ids)
{
    if (table.value().rank() != 2)
    {
        throw std::invalid_argument("embedding_device: the table must be rank 2 [V, D]");
    }
    const size_t count = ids.numel() * core::dtype_size(ids.dtype()) / sizeof(int64_t);
    return embedding_impl(table, ids, count, Shape({count, table.value().shape()[1]}), true);
}

Variable embedding_device_rows(const Variable& table, const Tensor& ids, RowsSink sink)
{
    if (table.value().rank() != 2)
    {
        throw std::invalid_argument("embedding_device_rows: the table must be rank 2 [V, D]");
    }
    const size_t V = table.value().shape()[0], D = table.value().shape()[1];
    const size_t count = ids.numel() * core::dtype_size(ids.dtype()) / sizeof(int64_t);
    const Tensor tc = make_contiguous(table.value());
    Tensor value = Tensor::empty(Shape({count, D}), tc.dtype());
    check(veda_embedding_fwd(static_cast<const int64_t*>(ids.data_ptr()), count, tc.data_ptr(), V,
                             D, value.data_ptr(), D, detail::device_flag(), dt(tc.dtype()), S()),
          "embedding");
    if (!table.requires_grad())
    {
        return Variable::leaf(std::move(value), false);
    }
    // on the tape (it receives its gradient) but with no parents: the table's gradient does not
    // wait for this node
    auto node = std::make_shared<Node>(std::move(value));
    node->requires_grad = true;
    node->backward = [sink = std::move(sink), ids, count](const Tensor& g) {
        sink(ids, count, make_contiguous(g));
    };
    return Variable(std::move(node));
}

Variable reshape(const Variable& x, const Shape& shape)
{
    Tensor value = x.value().reshape(shape);
    auto input = x.node();
    const Shape original = x.value().shape();
    return make({x}, std::move(value), [input, original](const Tensor& g) {
        accumulate(*input, make_contiguous(g).reshape(original));
    });
}

Variable transpose(const Variable& x, size_t a, size_t b)
{
    Tensor value = core::contiguous(x.value().transpose(a, b));
    auto input = x.node();
    return make({x}, std::move(value), [input, a, b](const Tensor& g) {
        accumulate(*input, core::contiguous(g.transpose(a, b)));
    });
}

Variable rope(const Variable& x, const Tensor& cosines, const Tensor& sines)
{
    const Shape& shape = x.value().shape();
    if (shape.rank() < 2)
    {
        throw std::invalid_argument("autograd::rope: expected [.., T, Dh], got " + shape.to_string());
    }
    const size_t Dh = shape[shape.rank() - 1], T = shape[shape.rank() - 2];
    if (cosines.shape() != Shape({T, Dh}) || sines.shape() != Shape({T, Dh}))
    {
        throw std::invalid_argument("autograd::rope: tables do not match (" + std::to_string(T) +
                                    ", " + std::to_string(Dh) + ")");
    }
    if (!x.value().is_contiguous())
    {
        throw std::invalid_argument("autograd::rope: expects a contiguous input");
    }
    const Tensor c = as_dtype(cosines, DType::F32), s = as_dtype(sines, DType::F32);
    const size_t lanes = (T == 0 || Dh == 0) ? 0 : x.value().numel() / (T * Dh);
    Tensor value = Tensor::empty(shape, x.value().dtype());
    check(veda_rope(x.value().data_ptr(), value.data_ptr(), static_cast<const float*>(c.data_ptr()),
                    static_cast<const float*>(s.data_ptr()), lanes, T, Dh, 0,
                    dt(x.value().dtype()), S()),
          "rope");
    auto input = x.node();
    return make({x}, std::move(value), [input, c, s, lanes, T, Dh](const Tensor& g) {
        const Tensor gc = as_dtype(g, input->value.dtype());
        Tensor d = Tensor::empty(gc.shape(), gc.dtype());
        check(veda_rope(gc.data_ptr(), d.data_ptr(), static_cast<const float*>(c.data_ptr()),
                        static_cast<const float*>(s.data_ptr()), lanes, T, Dh, 1, dt(gc.dtype()),
                        S()),
              "rope backward");
        accumulate(*input, d);
    });
}

namespace
{
Variable cross_entropy_impl(const Variable& logits, const Tensor& targets_raw, size_t lanes,
                            bool device_check)
{
    const Tensor& scores = logits.value();
    const size_t V = scores.shape()[scores.rank() - 1];
    const Tensor lc = make_contiguous(scores);
    Tensor rows = Tensor::empty(Shape({lanes}), DType::F32);
    Tensor loss = Tensor::empty(Shape({}), DType::F32);
    Tensor dlogits;
    const bool grad = logits.requires_grad();
    if (grad)
    {
        dlogits = Tensor::empty(lc.shape(), lc.dtype());
    }
    profile::Scope scope("cross_entropy", 0.0,
                         static_cast<double>(lc.numel()) * core::dtype_size(lc.dtype()) *
                             (grad ? 2.0 : 1.0));
    check(veda_cross_entropy(lc.data_ptr(), V, static_cast<const int64_t*>(targets_raw.data_ptr()),
                             static_cast<float*>(rows.data_ptr()), grad ? dlogits.data_ptr() : nullptr,
                             V, lanes, V, 1.0f / static_cast<float>(lanes),
                             device_check ? detail::device_flag() : nullptr, dt(lc.dtype()), S()),
          "cross_entropy");
    check(veda_mean_f64(static_cast<const float*>(rows.data_ptr()), lanes,
                        static_cast<float*>(loss.data_ptr()), nullptr, S()),
          "cross_entropy mean");
    if (!grad)
    {
        return Variable::leaf(std::move(loss), false);
    }
    auto input = logits.node();
    auto node = std::make_shared<Node>(std::move(loss));
    node->requires_grad = true;
    node->parents = {input};
    node->backward = [input, dlogits](const Tensor& g) {
        // (p - onehot) / lanes was formed in the forward pass for an upstream gradient of 1;
        // any other upstream value rescales it (Loss.cpp:80-99).
        if (g.storage().get() == g_seed_storage)
        {
            accumulate(*input, dlogits);
        }
        else
        {
            accumulate(*input, binary(1, dlogits, g));
        }
    };
    return Variable(std::move(node));
}
} // namespace

Variable cross_entropy(const Variable& logits, const std::vector<int64_t>& targets)
{
    const Tensor& scores = logits.value();
    if (scores.rank() == 0)
    {
        throw std::invalid_argument("cross_entropy: logits must have at least one dimension");
    }
    const size_t V = scores.shape()[scores.rank() - 1];
    const size_t lanes = V == 0 ? 0 : scores.numel() / V;
    if (targets.size() != lanes)
    {
        throw std::invalid_argument("cross_entropy: " + std::to_string(targets.size()) +
                                    " targets for " + std::to_string(lanes) + " lanes of shape " +
                                    scores.shape().to_string());
    }
    if (lanes == 0)
    {
        throw std::invalid_argument("cross_entropy: nothing to average over");
    }
    for (size_t lane = 0; lane < lanes; ++lane)
    {
        if (targets[lane] < 0 || static_cast<size_t>(targets[lane]) >= V)
        {
            throw std::invalid_argument("cross_entropy: target " + std::to_string(targets[lane]) +
                                        " at lane " + std::to_string(lane) +
                                        " is outside [0, " + std::to_string(V) + ")");
        }
    }
    return cross_entropy_impl(logits, upload_ids(targets), lanes, false);
}

Variable cross_entropy_device(const Variable& logits, const Tensor& targets)
{
    const Tensor& scores = logits.value();
    const size_t V = scores.shape()[scores.rank() - 1];
    const size_t lanes = scores.numel() / V;
    const size_t count = targets.numel() * core::dtype_size(targets.dtype()) / sizeof(int64_t);
    if (count != lanes || lanes == 0)
    {
        throw std::invalid_argument("cross_entropy_device: " + std::to_string(count) +
                                    " targets for " + std::to_string(lanes) + " lanes");
    }
    return cross_entropy_impl(logits, targets, lanes, true);
}

// ---- fused modules ----------------------------------------------------------------------------
namespace
{
// The node of y = rms_norm(x) * gamma over rows of n, given its forward value; xs is x's value
// (rows at stride ld) and gv the gain in x's dtype, both kept for the backward.
Variable rms_norm_node(const Variable& x, const Variable& gamma, Tensor value, const Tensor& xs,
                       int64_t ld, const Tensor& gv, size_t n, float eps)
{
    const size_t rows = xs.numel() / n;
    auto xin = x.node(), gin = gamma.node();
    return make({x, gamma}, std::move(value), [xin, gin, xs, gv, ld, n, rows, eps](const Tensor& g) {
        const Tensor gc = as_dtype(g, xs.dtype());
        float* dgamma = nullptr;
        if (gin->requires_grad)
        {
            bool fresh = false;
            Tensor& gg = grad_target(*gin, &fresh, DType::F32);
            if (gg.dtype() != DType::F32)
            {
                throw std::logic_error("rms_norm: the gain gradient must be fp32");
            }
            if (fresh)
            {
                memset_zero(gg);
            }
            dgamma = static_cast<float*>(gg.data_ptr());
        }
        const size_t ws_bytes = dgamma ? veda_rmsnorm_bwd_workspace(rows, n) : 0;
        Tensor ws = Tensor::empty(Shape({(ws_bytes + 3) / 4 + 1}), DType::F32);
        if (xin->requires_grad)
        {
            // the residual gradient already on x enters the kernel as dresid: dx = dresid + ...
            const bool has = xin->grad.defined() && !xin->grad_zero && !xin->is_leaf;
            const Tensor resid = has ? make_contiguous(xin->grad) : Tensor();
            Tensor d = Tensor::empty(xin->value.shape(), xs.dtype());
            profile::Scope scope("rmsnorm_bwd", 0.0,
                                 static_cast<double>(rows) * n * core::dtype_size(xs.dtype()) *
                                     (has ? 4.0 : 3.0));
            check(veda_rmsnorm_bwd(xs.data_ptr(), ld, gv.data_ptr(), gc.data_ptr(), n,
                                   has ? resid.data_ptr() : nullptr, n, d.data_ptr(), n, dgamma,
                                   ws.data_ptr(), ws_bytes, rows, n, eps, dt(xs.dtype()), S()),
                  "rms_norm backward");
            if (has)
            {
                xin->grad = d;
                xin->grad_owned = true;
            }
            else
            {
                accumulate(*xin, d);
            }
        }
        else if (dgamma)
        {
            Tensor d = Tensor::empty(xs.shape(), xs.dtype());
            check(veda_rmsnorm_bwd(xs.data_ptr(), ld, gv.data_ptr(), gc.data_ptr(), n, nullptr, 0,
                                   d.data_ptr(), n, dgamma, ws.data_ptr(), ws_bytes, rows, n, eps,
                                   dt(xs.dtype()), S()),
                  "rms_norm backward");
        }
    });
}

void check_gain(const Variable& gamma, size_t n, const char* what)
{
    if (gamma.value().shape() != Shape({n}))
    {
        throw std::invalid_argument(std::string(what) + ": gain of shape " +
                                    gamma.value().shape().to_string() + " for rows of " +
                                    std::to_string(n));
    }
}
} // namespace

Variable rms_norm(const Variable& x, const Variable& gamma, float eps)
{
    const Tensor& xv = x.value();
    const size_t n = xv.shape()[xv.rank() - 1];
    check_gain(gamma, n, "rms_norm");
    const Tensor xc = xv.rank() >= 2 ? (xv.strides().back() == 1 ? xv : make_contiguous(xv))
                                     : make_contiguous(xv);
    int64_t ld = static_cast<int64_t>(n);
    Tensor xs = xc;
    try
    {
        if (xc.rank() >= 2) ld = xc.ld();
    }
    catch (const std::invalid_argument&)
    {
        xs = make_contiguous(xc);
        ld = static_cast<int64_t>(n);
    }
    const size_t rows = xs.numel() / n;
    const Tensor gv = as_dtype(gamma.value(), xs.dtype());
    Tensor value = Tensor::empty(xs.shape(), xs.dtype());
    check(veda_rmsnorm_fwd(xs.data_ptr(), ld, gv.data_ptr(), value.data_ptr(), n, rows, n, eps,
                           dt(xs.dtype()), S()),
          "rms_norm");
    return rms_norm_node(x, gamma, std::move(value), xs, ld, gv, n, eps);
}

Variable add_rms_norm(const Variable& x, const Variable& r, const Variable& gamma, float eps,
                      Variable* sum)
{
    const Tensor& xv = x.value();
    const Tensor& rv = r.value();
    if (xv.shape() != rv.shape() || xv.dtype() != rv.dtype() || xv.rank() < 1)
    {
        throw std::invalid_argument("add_rms_norm: operands " + xv.shape().to_string() + " and " +
                                    rv.shape().to_string() + " differ");
    }
    if (sum == nullptr)
    {
        throw std::invalid_argument("add_rms_norm: no place for the sum");
    }
    const size_t n = xv.shape()[xv.rank() - 1];
    check_gain(gamma, n, "add_rms_norm");
    const Tensor xs = make_contiguous(xv);
    const Tensor rs = make_contiguous(rv);
    const size_t rows = xs.numel() / n;
    const Tensor gv = as_dtype(gamma.value(), xs.dtype());
    Tensor total = Tensor::empty(xs.shape(), xs.dtype());
    Tensor value = Tensor::empty(xs.shape(), xs.dtype());
    const int64_t ld = static_cast<int64_t>(n);
    check(veda_add_rmsnorm_fwd(xs.data_ptr(), ld, rs.data_ptr(), ld, gv.data_ptr(), total.data_ptr(),
                               ld, value.data_ptr(), ld, rows, n, eps, dt(xs.dtype()), S()),
          "add_rms_norm");
    // the sum node is add(x, r)'s (Variable.cpp:195-216): the gradient passes to both operands
    auto left = x.node(), right = r.node();
    const Tensor stored = total;
    Variable s = make({x, r}, std::move(total), [left, right](const Tensor& g) {
        if (left->requires_grad) accumulate(*left, g);
        if (right->requires_grad) accumulate(*right, g);
    });
    *sum = s;
    return rms_norm_node(s, gamma, std::move(value), stored, ld, gv, n, eps);
}

namespace
{
// What the linear backward reads: the input (rows of `in`, leading dimension ldx) and the
// contiguous weight [out, in], with the nodes the gradients go to.
struct LinearSaved
{
    std::shared_ptr<Node> xin, win;
    Tensor xs, wc;
    int64_t ldx = 0;
    size_t rows = 0, in = 0, out = 0;
};

LinearSaved linear_setup(const Tensor& xv, std::shared_ptr<Node> xin, const Variable& w)
{
    const Tensor& wv = w.value();
    if (wv.rank() != 2 || xv.rank() < 1)
    {
        throw std::invalid_argument("linear: weight must be [out, in], got " + wv.shape().to_string());
    }
    const size_t out = wv.shape()[0], in = wv.shape()[1];
    if (xv.shape()[xv.rank() - 1] != in)
    {
        throw std::invalid_argument("linear: input " + xv.shape().to_string() + " for weight " +
                                    wv.shape().to_string());
    }
    if (xv.dtype() != wv.dtype())
    {
        throw std::invalid_argument("linear: input and weight dtypes differ");
    }
    LinearSaved l;
    l.xin = std::move(xin);
    l.win = w.node();
    l.xs = xv;
    l.ldx = static_cast<int64_t>(in);
    if (xv.rank() >= 2 && xv.strides().back() == 1)
    {
        try
        {
            l.ldx = xv.ld();
        }
        catch (const std::invalid_argument&)
        {
            l.xs = make_contiguous(xv);
            l.ldx = static_cast<int64_t>(in);
        }
    }
    else
    {
        l.xs = make_contiguous(xv);
    }
    l.wc = make_contiguous(wv);
    l.rows = l.xs.numel() / in;
    l.in = in;
    l.out = out;
    return l;
}

Tensor linear_forward(const LinearSaved& l, const Shape& input_shape)
{
    std::vector<size_t> od = input_shape.dims();
    od.back() = l.out;
    Tensor value = Tensor::empty(Shape(od), l.xs.dtype());
    const double es = static_cast<double>(core::dtype_size(l.xs.dtype()));
    profile::Scope scope("gemm_fwd", 2.0 * l.rows * l.in * l.out,
                         es * (static_cast<double>(l.rows) * l.in + static_cast<double>(l.out) * l.in +
                               static_cast<double>(l.rows) * l.out));
    check(veda_gemm_nt(l.rows, l.out, l.in, l.xs.data_ptr(), l.ldx, l.wc.data_ptr(), l.in,
                       value.data_ptr(), l.out, dt(l.xs.dtype()), dt(l.xs.dtype()), 1.0f, 0.0f, S()),
          "linear");
    return value;
}

void linear_backward(const LinearSaved& l, const Tensor& g)
{
    const auto& xin = l.xin;
    const auto& win = l.win;
    const Tensor& xs = l.xs;
    const Tensor& wc = l.wc;
    const int64_t ldx = l.ldx;
    const size_t rows = l.rows, in = l.in, out = l.out;
    const Tensor gc = as_dtype(g, xs.dtype());
    const double es = static_cast<double>(core::dtype_size(xs.dtype()));
    if (xin->requires_grad && win->requires_grad && gemm_overlap_enabled())
    {
        // dW (+)= G^T X on the side stream, dX = G W on this one, then join: everything
        // after this (including the release of G and X) is ordered after both.
        bool fresh = false;
        Tensor& gw = grad_target(*win, &fresh, DType::F32);
        profile::Scope scope("gemm_bwd", 4.0 * rows * in * out,
                             es * (2.0 * static_cast<double>(rows) * out +
                                   static_cast<double>(out) * in +
                                   2.0 * static_cast<double>(rows) * in) +
                                 4.0 * static_cast<double>(out) * in * (fresh ? 1.0 : 2.0));
        SideStream& side = side_stream();
        const cudaStream_t main = reinterpret_cast<cudaStream_t>(S());
        cuda_check(cudaEventRecord(side.fork, main), "gemm fork");
        cuda_check(cudaStreamWaitEvent(side.stream, side.fork, 0), "gemm fork wait");
        check(veda_gemm_tn(out, in, rows, gc.data_ptr(), out, xs.data_ptr(), ldx,
                           gw.data_ptr(), in, dt(xs.dtype()), dt(gw.dtype()), 1.0f,
                           fresh ? 0.0f : 1.0f, side.stream),
              "linear backward (weight)");
        if (!xin->grad.defined() || xin->is_leaf || xin->grad_zero || !xin->grad_owned)
        {
            Tensor d = Tensor::empty(xin->value.shape(), xs.dtype());
            check(veda_gemm_nn(rows, in, out, gc.data_ptr(), out, wc.data_ptr(), in,
                               d.data_ptr(), in, dt(xs.dtype()), dt(xs.dtype()), 1.0f, 0.0f,
                               S()),
                  "linear backward (input)");
            accumulate(*xin, d);
        }
        else
        {
            check(veda_gemm_nn(rows, in, out, gc.data_ptr(), out, wc.data_ptr(), in,
                               xin->grad.data_ptr(), in, dt(xs.dtype()),
                               dt(xin->grad.dtype()), 1.0f, 1.0f, S()),
                  "linear backward (input)");
        }
        cuda_check(cudaEventRecord(side.join, side.stream), "gemm join");
        cuda_check(cudaStreamWaitEvent(main, side.join, 0), "gemm join wait");
        return;
    }
    if (xin->requires_grad)
    {
        // dX = G W  (NN)
        profile::Scope scope("gemm_dx", 2.0 * rows * in * out,
                             es * (static_cast<double>(rows) * out +
                                   static_cast<double>(out) * in +
                                   static_cast<double>(rows) * in));
        if (!xin->grad.defined() || xin->is_leaf || xin->grad_zero || !xin->grad_owned)
        {
            Tensor d = Tensor::empty(xin->value.shape(), xs.dtype());
            check(veda_gemm_nn(rows, in, out, gc.data_ptr(), out, wc.data_ptr(), in,
                               d.data_ptr(), in, dt(xs.dtype()), dt(xs.dtype()), 1.0f, 0.0f,
                               S()),
                  "linear backward (input)");
            accumulate(*xin, d);
        }
        else
        {
            check(veda_gemm_nn(rows, in, out, gc.data_ptr(), out, wc.data_ptr(), in,
                               xin->grad.data_ptr(), in, dt(xs.dtype()),
                               dt(xin->grad.dtype()), 1.0f, 1.0f, S()),
                  "linear backward (input)");
        }
    }
    if (win->requires_grad)
    {
        // dW (+)= G^T X  (TN), straight into the fp32 parameter gradient
        bool fresh = false;
        Tensor& gw = grad_target(*win, &fresh, DType::F32);
        profile::Scope scope("gemm_dw", 2.0 * rows * in * out,
                             es * (static_cast<double>(rows) * out +
                                   static_cast<double>(rows) * in) +
                                 4.0 * static_cast<double>(out) * in * (fresh ? 1.0 : 2.0));
        check(veda_gemm_tn(out, in, rows, gc.data_ptr(), out, xs.data_ptr(), ldx,
                           gw.data_ptr(), in, dt(xs.dtype()), dt(gw.dtype()), 1.0f,
                           fresh ? 0.0f : 1.0f, S()),
              "linear backward (weight)");
    }
}

// What the attention backward reads: the fused projection and its leading dimension, the gains
// and RoPE tables, the normalised rotated q and k, the output and the forward's log-sum-exp.
struct AttentionSaved
{
    std::shared_ptr<Node> xin, qn, kn;
    Tensor x, qg, kg, c, s;
    int64_t ld = 0;
    Tensor qr, kr, out, lse;
    size_t B = 0, T = 0, H = 0, Hkv = 0, Dh = 0;
    float eps = 0.0f, scale = 0.0f;
};

AttentionSaved attention_setup(const Variable& qkv, const Variable& q_norm, const Variable& k_norm,
                               const Tensor& cosines, const Tensor& sines, size_t B, size_t T,
                               size_t H, size_t Hkv, size_t Dh, float eps)
{
    const Tensor& xv = qkv.value();
    const size_t N = B * T;
    const size_t W = (H + 2 * Hkv) * Dh;
    if (xv.rank() != 2 || xv.shape()[0] != N || xv.shape()[1] != W)
    {
        throw std::invalid_argument("attention: expected a fused projection [" + std::to_string(N) +
                                    ", " + std::to_string(W) + "], got " + xv.shape().to_string());
    }
    if (H % Hkv != 0)
    {
        throw std::invalid_argument("attention: heads must be a multiple of kv_heads");
    }
    AttentionSaved a;
    a.xin = qkv.node();
    a.qn = q_norm.node();
    a.kn = k_norm.node();
    a.x = xv.strides().back() == 1 ? xv : make_contiguous(xv);
    a.ld = a.x.ld();
    const DType d = a.x.dtype();
    a.qg = as_dtype(q_norm.value(), d);
    a.kg = as_dtype(k_norm.value(), d);
    a.c = as_dtype(cosines, DType::F32);
    a.s = as_dtype(sines, DType::F32);
    a.lse = Tensor::empty(Shape({B * H * T}), DType::F32);
    a.B = B;
    a.T = T;
    a.H = H;
    a.Hkv = Hkv;
    a.Dh = Dh;
    a.eps = eps;
    a.scale = 1.0f / std::sqrt(static_cast<float>(Dh));
    return a;
}

// q and k: RMS norm with their gains, then RoPE, into a.qr and a.kr; then causal GQA attention
// into a.out, its log-sum-exp into `lse`. Deterministic, so a second run gives the same bits.
void attention_forward(AttentionSaved& a, float* lse, const char* scope_name)
{
    const DType d = a.x.dtype();
    const size_t es = core::dtype_size(d);
    const size_t N = a.B * a.T, H = a.H, Hkv = a.Hkv, Dh = a.Dh;
    char* base = static_cast<char*>(a.x.data_ptr());
    const float* cp = static_cast<const float*>(a.c.data_ptr());
    const float* sp = static_cast<const float*>(a.s.data_ptr());
    a.qr = Tensor::empty(Shape({N, H * Dh}), d);
    a.kr = Tensor::empty(Shape({N, Hkv * Dh}), d);
    check(veda_qknorm_rope_fwd_qk(base, base + H * Dh * es, a.ld, a.qg.data_ptr(), a.kg.data_ptr(),
                                  cp, sp, a.qr.data_ptr(), H * Dh, a.kr.data_ptr(), Hkv * Dh, N, H, Hkv,
                                  a.T, Dh, a.eps, dt(d), S()),
          "attention: q and k norm + rope");
    a.out = Tensor::empty(Shape({N, H * Dh}), d);
    // causal: half of the 2 T^2 Dh products per (batch, head) for each of QK^T and PV
    profile::Scope scope(scope_name, 2.0 * a.B * H * static_cast<double>(a.T) * a.T * Dh, 0.0);
    check(veda_attention_fwd(a.qr.data_ptr(), H * Dh, a.kr.data_ptr(), Hkv * Dh,
                             base + (H + Hkv) * Dh * es, a.ld, a.out.data_ptr(), H * Dh, lse, a.B,
                             a.T, H, Hkv, Dh, a.scale, 1, dt(d), S()),
          "attention");
}

void attention_backward(const AttentionSaved& a, const Tensor& g)
{
    const DType d = a.x.dtype();
    const size_t es = core::dtype_size(d);
    const size_t B = a.B, T = a.T, H = a.H, Hkv = a.Hkv, Dh = a.Dh;
    const size_t N = B * T, W = (H + 2 * Hkv) * Dh;
    const int64_t ld = a.ld;
    const char* base = static_cast<const char*>(a.x.data_ptr());
    const Tensor gc = as_dtype(g, d);
    Tensor dqr;
    Tensor dkr = Tensor::empty(Shape({N, Hkv * Dh}), d);
    Tensor dx = Tensor::empty(Shape({N, W}), d);
    char* dbase = static_cast<char*>(dx.data_ptr());
    const size_t ws_bytes = veda_attention_bwd_workspace(B, T, H, Hkv, Dh, dt(d));
    Tensor ws = Tensor::empty(Shape({(ws_bytes + 3) / 4}), DType::F32);
    // where the norm backward reads dQ: the fused kernel's fp32 accumulator (no separate pass
    // rounding it into a bf16 dQ), or a dQ written by the general path
    const void* dq_src = nullptr;
    int64_t dq_ld = H * Dh;
    bool dq_f32 = false;
    {
        // causal backward with the softmax recomputed: 5 products of T^2 Dh per (batch, head)
        profile::Scope scope("attn_bwd", 5.0 * B * H * static_cast<double>(T) * T * Dh, 0.0);
        const int rc = veda_attention_bwd_dq_f32(
            a.qr.data_ptr(), H * Dh, a.kr.data_ptr(), Hkv * Dh, base + (H + Hkv) * Dh * es, ld,
            a.out.data_ptr(), H * Dh, gc.data_ptr(), H * Dh, static_cast<const float*>(a.lse.data_ptr()),
            dkr.data_ptr(), Hkv * Dh, dbase + (H + Hkv) * Dh * es, W, ws.data_ptr(), ws_bytes, B, T, H,
            Hkv, Dh, a.scale, 1, dt(d), S());
        if (rc == VEDA_OK)
        {
            dq_src = static_cast<const char*>(ws.data_ptr()) + veda_attention_bwd_dq_offset(B, T, H);
            dq_f32 = true;
        }
        else if (rc == VEDA_ERR_UNSUPPORTED)
        {
            dqr = Tensor::empty(Shape({N, H * Dh}), d);
            check(veda_attention_bwd(a.qr.data_ptr(), H * Dh, a.kr.data_ptr(), Hkv * Dh,
                                     base + (H + Hkv) * Dh * es, ld, a.out.data_ptr(), H * Dh,
                                     gc.data_ptr(), H * Dh, static_cast<const float*>(a.lse.data_ptr()),
                                     dqr.data_ptr(), H * Dh, dkr.data_ptr(), Hkv * Dh,
                                     dbase + (H + Hkv) * Dh * es, W, ws.data_ptr(), ws_bytes, B, T,
                                     H, Hkv, Dh, a.scale, 1, dt(d), S()),
                  "attention backward");
            dq_src = dqr.data_ptr();
        }
        else
        {
            check(rc, "attention backward");
        }
    }
    // q_norm and k_norm backward in one launch: dq, dk into their columns of the fused gradient
    auto gain_target = [&](const std::shared_ptr<Node>& gain) -> float* {
        if (!gain->requires_grad)
        {
            return nullptr;
        }
        bool fresh = false;
        Tensor& gg = grad_target(*gain, &fresh, DType::F32);
        if (fresh) memset_zero(gg);
        return static_cast<float*>(gg.data_ptr());
    };
    float* dqg = gain_target(a.qn);
    float* dkg = gain_target(a.kn);
    const size_t wsb = veda_qknorm_rope_bwd_qk_workspace(N, H, Hkv, Dh);
    Tensor w2 = Tensor::empty(Shape({(wsb + 3) / 4 + 1}), DType::F32);
    {
        // reads x and dy, writes dx over [N, (H + Hkv) * Dh]; the q part of dy is the attention
        // backward's fp32 dQ accumulator when it kept one
        const double elems = static_cast<double>(N) * Dh;
        profile::Scope scope("qknorm_bwd", 0.0,
                             elems * ((H + Hkv) * 2.0 * es + H * (dq_f32 ? 4.0 : es) + Hkv * es));
        check(veda_qknorm_rope_bwd_qk(base, base + H * Dh * es, ld, a.qg.data_ptr(), a.kg.data_ptr(),
                                      static_cast<const float*>(a.c.data_ptr()),
                                      static_cast<const float*>(a.s.data_ptr()), dq_src, dq_ld,
                                      dq_f32 ? 1 : 0, a.scale, dkr.data_ptr(), Hkv * Dh, dbase,
                                      dbase + H * Dh * es, W, dqg, dkg,
                                      w2.data_ptr(), wsb, N, H, Hkv, T, Dh, a.eps, dt(d), S()),
              "attention backward: norm + rope");
    }
    if (a.xin->requires_grad)
    {
        accumulate(*a.xin, dx);
    }
}
} // namespace

Variable linear(const Variable& x, const Variable& w)
{
    LinearSaved l = linear_setup(x.value(), x.node(), w);
    Tensor value = linear_forward(l, x.value().shape());
    return make({x, w}, std::move(value), [l](const Tensor& g) { linear_backward(l, g); });
}

Variable attention(const Variable& qkv, const Variable& q_norm, const Variable& k_norm,
                   const Tensor& cosines, const Tensor& sines, size_t B, size_t T, size_t H,
                   size_t Hkv, size_t Dh, float eps)
{
    AttentionSaved a = attention_setup(qkv, q_norm, k_norm, cosines, sines, B, T, H, Hkv, Dh, eps);
    attention_forward(a, static_cast<float*>(a.lse.data_ptr()), "attn_fwd");
    Tensor ctx = a.out;
    return make({qkv, q_norm, k_norm}, std::move(ctx),
                [a](const Tensor& g) { attention_backward(a, g); });
}

Variable attention_output(const Variable& qkv, const Variable& q_norm, const Variable& k_norm,
                          const Variable& o, const Tensor& cosines, const Tensor& sines, size_t B,
                          size_t T, size_t H, size_t Hkv, size_t Dh, float eps)
{
    AttentionSaved a = attention_setup(qkv, q_norm, k_norm, cosines, sines, B, T, H, Hkv, Dh, eps);
    attention_forward(a, static_cast<float*>(a.lse.data_ptr()), "attn_fwd");
    LinearSaved l = linear_setup(a.out, nullptr, o);
    Tensor value = linear_forward(l, a.out.shape());
    // keep the projection, the gains and the log-sum-exp; q, k after norm + RoPE and the
    // context are dropped here and formed again by the backward
    a.qr = Tensor();
    a.kr = Tensor();
    a.out = Tensor();
    l.xs = Tensor();
    return make({qkv, q_norm, k_norm, o}, std::move(value), [a, l](const Tensor& g) {
        AttentionSaved r = a;
        Tensor lse = Tensor::empty(Shape({r.B * r.H * r.T}), DType::F32);
        attention_forward(r, static_cast<float*>(lse.data_ptr()), "attn_recompute");
        // the output projection's backward with the recomputed context as its input, whose
        // gradient a node of its own collects for the attention backward
        auto ctx = std::make_shared<Node>(r.out);
        ctx->requires_grad = true;
        LinearSaved lr = l;
        lr.xin = ctx;
        lr.xs = r.out;
        lr.ldx = static_cast<int64_t>(r.H * r.Dh);
        linear_backward(lr, g);
        attention_backward(r, ctx->grad);
    });
}

Variable swiglu(const Variable& gate_up)
{
    const Tensor& v = gate_up.value();
    if (v.rank() != 2 || v.shape()[1] % 2 != 0)
    {
        throw std::invalid_argument("swiglu: expected [rows, 2F], got " + v.shape().to_string());
    }
    const Tensor x = make_contiguous(v);
    const size_t rows = x.shape()[0], F = x.shape()[1] / 2;
    const size_t es = core::dtype_size(x.dtype());
    Tensor value = Tensor::empty(Shape({rows, F}), x.dtype());
    char* base = static_cast<char*>(x.data_ptr());
    check(veda_swiglu_fwd(base, 2 * F, base + F * es, 2 * F, value.data_ptr(), F, rows, F,
                          dt(x.dtype()), S()),
          "swiglu");
    auto input = gate_up.node();
    return make({gate_up}, std::move(value), [input, x, rows, F, es](const Tensor& g) {
        const Tensor gc = as_dtype(g, x.dtype());
        Tensor d = Tensor::empty(x.shape(), x.dtype());
        const char* base = static_cast<const char*>(x.data_ptr());
        char* db = static_cast<char*>(d.data_ptr());
        profile::Scope scope("swiglu_bwd", 0.0, 5.0 * static_cast<double>(rows) * F * es);
        check(veda_swiglu_bwd(base, 2 * F, base + F * es, 2 * F, gc.data_ptr(), F, db, 2 * F,
                              db + F * es, 2 * F, rows, F, dt(x.dtype()), S()),
              "swiglu backward");
        accumulate(*input, d);
    });
}

// VEDA_FUSED_MLP=0 runs the feed-forward block as its three ops even where the fused form applies
// (read at every call, so a process can compare the two).
bool fused_mlp_enabled()
{
    const char* v = std::getenv("VEDA_FUSED_MLP");
    return !(v != nullptr && v[0] == '0');
}

Variable mlp(const Variable& x, const Variable& gate_up, const Variable& down)
{
    // Model.cpp:199-203: down(silu(gate(x)) * up(x)). The fused form needs bf16 throughout, F a
    // multiple of 256 and at least 256 rows; otherwise the three ops run one by one.
    const Tensor& xv = x.value();
    const Tensor& wg = gate_up.value();
    const Tensor& wd = down.value();
    const size_t D = xv.rank() >= 1 ? xv.shape()[xv.rank() - 1] : 0;
    const size_t rows = D > 0 ? xv.numel() / D : 0;
    const bool fusable = xv.dtype() == DType::BF16 && wg.dtype() == DType::BF16 &&
                         wd.dtype() == DType::BF16 && wg.rank() == 2 && wd.rank() == 2 &&
                         wg.shape()[1] == D && wg.shape()[0] % 512 == 0 && wd.shape()[0] == D &&
                         2 * wd.shape()[1] == wg.shape()[0] && rows >= 256 && D % 8 == 0 &&
                         fused_mlp_enabled();
    if (!fusable)
    {
        return linear(swiglu(linear(x, gate_up)), down);
    }
    const LinearSaved l1 = linear_setup(xv, x.node(), gate_up);
    const size_t F = l1.out / 2;
    Tensor gu = Tensor::empty(Shape({rows, 2 * F}), DType::BF16);
    Tensor h = Tensor::empty(Shape({rows, F}), DType::BF16);
    int rc = VEDA_OK;
    {
        // a class of its own: the GEMM with SwiGLU in its epilogue
        profile::Scope scope("mlp_fwd", 4.0 * rows * D * F,
                             2.0 * (static_cast<double>(rows) * D + 2.0 * F * D + 3.0 * rows * F));
        rc = veda_gemm_swiglu_fwd(rows, F, D, l1.xs.data_ptr(), l1.ldx, l1.wc.data_ptr(), D,
                                  gu.data_ptr(), 2 * F, h.data_ptr(), F, S());
    }
    if (rc == VEDA_ERR_UNSUPPORTED)
    {
        return linear(swiglu(linear(x, gate_up)), down);
    }
    check(rc, "mlp (gate|up projection and SwiGLU)");
    LinearSaved l2 = linear_setup(h, nullptr, down);
    Tensor value = linear_forward(l2, xv.shape());
    return make({x, gate_up, down}, std::move(value), [l1, l2, gu, rows, F, D](const Tensor& g) {
        // the down projection's backward: dW (+)= G^T h beside dgate|up = SwiGLU'(G W) (one GEMM
        // whose epilogue applies SwiGLU's backward, so dh is never stored); then the gate|up
        // projection's backward with dgate|up
        const Tensor gc = as_dtype(g, DType::BF16);
        Tensor dgu = Tensor::empty(Shape({rows, 2 * F}), DType::BF16);
        const auto& win = l2.win;
        {
            profile::Scope scope("mlp_bwd", 4.0 * rows * D * F,
                                 2.0 * (2.0 * static_cast<double>(rows) * D + 2.0 * D * F + 5.0 * rows * F) +
                                     8.0 * static_cast<double>(D) * F);
            const cudaStream_t main = reinterpret_cast<cudaStream_t>(S());
            const bool side = win->requires_grad && gemm_overlap_enabled();
            SideStream* ss = side ? &side_stream() : nullptr;
            auto weight_grad = [&](cudaStream_t st) {
                bool fresh = false;
                Tensor& gw = grad_target(*win, &fresh, DType::F32);
                check(veda_gemm_tn(D, F, rows, gc.data_ptr(), D, l2.xs.data_ptr(), F, gw.data_ptr(), F,
                                   VEDA_BF16, dt(gw.dtype()), 1.0f, fresh ? 0.0f : 1.0f, st),
                      "mlp backward (down projection weight)");
            };
            if (side)
            {
                cuda_check(cudaEventRecord(ss->fork, main), "gemm fork");
                cuda_check(cudaStreamWaitEvent(ss->stream, ss->fork, 0), "gemm fork wait");
                weight_grad(ss->stream);
            }
            int rc = veda_gemm_swiglu_bwd(rows, F, D, gc.data_ptr(), D, l2.wc.data_ptr(), F,
                                          gu.data_ptr(), 2 * F, dgu.data_ptr(), 2 * F, S());
            if (rc == VEDA_ERR_UNSUPPORTED)
            {
                Tensor dh = Tensor::empty(Shape({rows, F}), DType::BF16);
                check(veda_gemm_nn(rows, F, D, gc.data_ptr(), D, l2.wc.data_ptr(), F, dh.data_ptr(), F,
                                   VEDA_BF16, VEDA_BF16, 1.0f, 0.0f, S()),
                      "mlp backward (down projection input)");
                const char* base = static_cast<const char*>(gu.data_ptr());
                char* db = static_cast<char*>(dgu.data_ptr());
                rc = veda_swiglu_bwd(base, 2 * F, base + 2 * F, 2 * F, dh.data_ptr(), F, db, 2 * F,
                                     db + 2 * F, 2 * F, rows, F, VEDA_BF16, S());
            }
            check(rc, "mlp backward (SwiGLU)");
            if (side)
            {
                cuda_check(cudaEventRecord(ss->join, ss->stream), "gemm join");
                cuda_check(cudaStreamWaitEvent(main, ss->join, 0), "gemm join wait");
            }
            else if (win->requires_grad)
            {
                weight_grad(main);
            }
        }
        linear_backward(l1, dgu);
    });
}

GradientCheck check_gradient(const std::function<Variable(const Variable&)>& loss_of,
                             const Tensor& at, float step, double tolerance)
{
    // the restatement of src/libs/autograd/GradientCheck.cpp:14-64: one analytic gradient from
    // the tape, then a central difference per element of `at`
    GradientCheck result;
    Variable x = Variable::leaf(core::contiguous(core::to_dtype(at, DType::F32)));
    Variable loss = loss_of(x);
    if (loss.value().numel() != 1)
    {
        result.ok = false;
        result.message = "check_gradient: the function must return a scalar, got " +
                         loss.value().shape().to_string();
        return result;
    }
    loss.backward();
    const std::vector<float> analytic = x.grad().to_host();
    const Tensor base = core::contiguous(core::to_dtype(at, DType::F32));
    std::vector<float> point = base.to_host();
    auto value_at = [&](const std::vector<float>& p) {
        const Variable v = loss_of(Variable::leaf(Tensor::from_host(p, base.shape()), false));
        return static_cast<double>(v.value().to_host()[0]);
    };
    for (size_t i = 0; i < point.size(); ++i)
    {
        const float keep = point[i];
        point[i] = keep + step;
        const double up = value_at(point);
        point[i] = (keep + step) - 2.0f * step;
        const double down = value_at(point);
        point[i] = keep;
        const double numeric = (up - down) / (2.0 * static_cast<double>(step));
        const double a = analytic[i];
        const double scale = std::max({std::fabs(numeric), std::fabs(a), 1e-3});
        const double relative = std::fabs(numeric - a) / scale;
        if (relative > result.worst_relative)
        {
            result.worst_relative = relative;
            result.worst_index = i;
            result.analytic = a;
            result.numeric = numeric;
        }
    }
    result.ok = result.worst_relative <= tolerance;
    if (!result.ok)
    {
        result.message = "gradient mismatch at index " + std::to_string(result.worst_index) +
                         ": analytic " + std::to_string(result.analytic) + ", numeric " +
                         std::to_string(result.numeric) + ", relative " +
                         std::to_string(result.worst_relative);
    }
    return result;
}

} // namespace veda::autograd

namespace veda::ops
{

using core::DType;
using core::Shape;
using core::Tensor;

Tensor add(const Tensor& a, const Tensor& b) { return autograd::binary(0, a, b); }
Tensor mul(const Tensor& a, const Tensor& b) { return autograd::binary(1, a, b); }

Tensor add(const Tensor& a, float scalar)
{
    return autograd::binary(0, a, Tensor::from_host({scalar}, Shape({}), a.dtype()));
}

Tensor mul(const Tensor& a, float scalar) { return autograd::scale(a, scalar); }

namespace
{
// f over the last dim of a contiguous [lanes, length] view of `tensor` with `dim` moved last
Tensor along(const Tensor& tensor, size_t dim, const char* what,
             int (*f)(const void*, void*, int64_t, int64_t, int, veda_stream_t))
{
    if (dim >= tensor.rank())
    {
        throw std::invalid_argument(std::string(what) + ": dimension " + std::to_string(dim) +
                                    " is out of range for shape " + tensor.shape().to_string());
    }
    const size_t last = tensor.rank() - 1;
    const Tensor moved = core::contiguous(dim == last ? tensor : tensor.transpose(dim, last));
    Tensor out = Tensor::empty(moved.shape(), moved.dtype());
    const size_t length = moved.shape()[last];
    const size_t lanes = length == 0 ? 0 : moved.numel() / length;
    check(f(moved.data_ptr(), out.data_ptr(), static_cast<int64_t>(lanes),
            static_cast<int64_t>(length), static_cast<int>(moved.dtype()), current_stream()),
          what);
    return dim == last ? out : core::contiguous(out.transpose(dim, last));
}
} // namespace

Tensor softmax(const Tensor& tensor, size_t dim)
{
    return along(tensor, dim, "softmax", veda_softmax_fwd);
}

Tensor log_softmax(const Tensor& tensor, size_t dim)
{
    return along(tensor, dim, "log_softmax", veda_log_softmax_fwd);
}

} // namespace veda::ops
