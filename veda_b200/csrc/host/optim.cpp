// veda::optim on the device (src/libs/optim/AdamW.cpp, Clip.cpp).
#include "veda/optim.hpp"

#include "veda_cuda.h"

#include <cuda_runtime.h>

#include <cmath>
#include <stdexcept>

namespace veda::optim
{

using core::DType;
using core::Shape;
using core::Tensor;

namespace
{
cudaStream_t cs() { return reinterpret_cast<cudaStream_t>(current_stream()); }

float* fptr(const Tensor& t) { return static_cast<float*>(t.data_ptr()); }

// The runs launch through device addresses taken once: bring any value or gradient the host wrote
// through Tensor::data() since then back to the device first (a no-op without host mirrors).
void flush_host_writes(const std::vector<autograd::Variable>& parameters)
{
    for (const auto& p : parameters)
    {
        p.value().storage()->data();
        if (p.node()->grad.defined())
        {
            p.node()->grad.storage()->data();
        }
    }
}
} // namespace

AdamW::AdamW(std::vector<autograd::Variable> parameters, AdamWConfig config)
    : parameters_(std::move(parameters)), config_(config)
{
    if (config_.learning_rate < 0.0f || config_.eps <= 0.0f || config_.weight_decay < 0.0f)
    {
        throw std::invalid_argument("AdamW: learning rate, eps and weight decay must be positive");
    }
    if (config_.beta1 < 0.0f || config_.beta1 >= 1.0f || config_.beta2 < 0.0f ||
        config_.beta2 >= 1.0f)
    {
        throw std::invalid_argument("AdamW: betas must lie in [0, 1)");
    }
    size_t total = 0, lowp_total = 0;
    for (const auto& p : parameters_)
    {
        total += p.value().numel();
        if (p.value().dtype() == DType::BF16)
        {
            lowp_total += p.value().numel();
        }
    }
    m_arena_ = Tensor(Shape({total > 0 ? total : 1}), DType::F32);
    v_arena_ = Tensor(Shape({total > 0 ? total : 1}), DType::F32);
    if (lowp_total > 0)
    {
        master_arena_ = Tensor::empty(Shape({lowp_total}), DType::F32);
    }
    size_t at = 0;
    for (const auto& p : parameters_)
    {
        if (p.value().dtype() == DType::BF16)
        {
            Tensor mview = Tensor::view(master_arena_.storage(), at, p.value().shape(), DType::F32);
            // the master starts at the parameter's (bf16) value, widened exactly
            std::vector<int64_t> shape(p.value().shape().dims().begin(), p.value().shape().dims().end());
            std::vector<int64_t> strides(p.value().strides().begin(), p.value().strides().end());
            if (shape.empty()) { shape = {1}; strides = {1}; }
            check(veda_copy_strided(p.value().storage()->data(), VEDA_BF16, strides.data(),
                                    static_cast<int64_t>(p.value().offset()), mview.data_ptr(),
                                    VEDA_F32, shape.data(), static_cast<int>(shape.size()),
                                    current_stream()),
                  "AdamW: master copy");
            masters_.push_back(mview);
            at += p.value().numel();
        }
        else
        {
            masters_.push_back(p.value());
        }
    }
    sumsq_ = Tensor(Shape({2}), DType::F32);   // 8 bytes: one double
    bias_ = Tensor(Shape({4}), DType::F32);    // two doubles
    build_runs();
}

AdamW::~AdamW() = default;

void AdamW::build_runs()
{
    runs_.clear();
    size_t offset = 0;
    for (size_t i = 0; i < parameters_.size(); ++i)
    {
        const auto& p = parameters_[i];
        const size_t n = p.value().numel();
        if (!p.requires_grad() || n == 0)
        {
            offset += n;
            continue;
        }
        const Tensor& g = p.grad();   // allocates zeros for a leaf that has none yet
        if (g.dtype() != DType::F32 || !g.is_contiguous() || !p.value().is_contiguous())
        {
            throw std::invalid_argument("AdamW: parameters need contiguous values and fp32 gradients");
        }
        Run r{i, 1, static_cast<int64_t>(n), fptr(g), fptr(masters_[i]), fptr(m_arena_) + offset,
              fptr(v_arena_) + offset,
              p.value().dtype() == DType::BF16 ? p.value().data_ptr() : nullptr};
        if (!runs_.empty())
        {
            Run& last = runs_.back();
            const bool adjacent = last.first + last.count == i &&
                                  last.grad + last.n == r.grad && last.master + last.n == r.master &&
                                  last.m + last.n == r.m &&
                                  ((last.lowp == nullptr && r.lowp == nullptr) ||
                                   (last.lowp != nullptr && r.lowp != nullptr &&
                                    static_cast<char*>(last.lowp) + last.n * 2 ==
                                        static_cast<char*>(r.lowp)));
            if (adjacent)
            {
                last.count += 1;
                last.n += r.n;
                offset += n;
                continue;
            }
        }
        runs_.push_back(r);
        offset += n;
    }
    int64_t largest = 1;
    for (const Run& r : runs_)
    {
        largest = std::max<int64_t>(largest, r.n);
    }
    const size_t ws = veda_sumsq_workspace(largest);
    workspace_ = Tensor::empty(Shape({(ws + 3) / 4 + 1}), DType::F32);
}

void AdamW::advance()
{
    ++steps_;
    bias_host_[0] = 1.0 - std::pow(static_cast<double>(config_.beta1), static_cast<double>(steps_));
    bias_host_[1] = 1.0 - std::pow(static_cast<double>(config_.beta2), static_cast<double>(steps_));
    if (cudaMemcpyAsync(bias_.data_ptr(), bias_host_, sizeof(bias_host_), cudaMemcpyHostToDevice, cs()) !=
        cudaSuccess)
    {
        throw std::runtime_error("AdamW: bias correction upload failed");
    }
}

void AdamW::launch(const double* sumsq, float max_norm, float grad_scale)
{
    flush_host_writes(parameters_);
    const double* bias = static_cast<const double*>(bias_.data_ptr());
    for (const Run& r : runs_)
    {
        check(veda_adamw_step_dev(r.master, r.m, r.v, r.grad, r.lowp, r.n, config_.learning_rate,
                                  config_.beta1, config_.beta2, config_.eps, config_.weight_decay,
                                  bias, sumsq, max_norm, grad_scale,
                                  skip_nonfinite_ && sumsq != nullptr ? VEDA_ADAMW_SKIP_NONFINITE : 0,
                                  current_stream()),
              "AdamW::step");
    }
}

void AdamW::step()
{
    advance();
    launch(nullptr, 1.0f, 1.0f);
}

void AdamW::step_clipped(float max_norm, float grad_scale)
{
    advance();
    launch_clipped(max_norm, grad_scale);
}

void AdamW::launch_clipped(float max_norm, float grad_scale)
{
    if (!(max_norm > 0.0f))
    {
        throw std::invalid_argument("clip_gradient_norm: max_norm must be positive");
    }
    flush_host_writes(parameters_);
    double* ss = static_cast<double*>(sumsq_.data_ptr());
    for (size_t k = 0; k < runs_.size(); ++k)
    {
        check(veda_sumsq(runs_[k].grad, runs_[k].n, ss, k == 0 ? 0 : 1, workspace_.data_ptr(),
                         workspace_.numel() * 4, current_stream()),
              "AdamW::step_clipped (norm)");
    }
    last_scale_ = grad_scale;
    launch(ss, max_norm, grad_scale);
}

float AdamW::last_grad_norm()
{
    double ss = 0.0;
    if (cudaMemcpyAsync(&ss, sumsq_.data_ptr(), sizeof(double), cudaMemcpyDeviceToHost, cs()) !=
            cudaSuccess ||
        cudaStreamSynchronize(cs()) != cudaSuccess)
    {
        throw std::runtime_error("AdamW::last_grad_norm: read failed");
    }
    return static_cast<float>(std::sqrt(ss) * std::fabs(static_cast<double>(last_scale_)));
}

void AdamW::zero_grad()
{
    for (auto& p : parameters_)
    {
        if (!p.requires_grad())
        {
            continue;
        }
        auto& node = *p.node();
        if (node.grad.defined())
        {
            if (cudaMemsetAsync(node.grad.data_ptr(), 0, node.grad.numel() * 4, cs()) != cudaSuccess)
            {
                throw std::runtime_error("AdamW::zero_grad: memset failed");
            }
            node.grad_zero = true;
            node.grad_owned = true;
        }
    }
}

float clip_gradient_norm(const std::vector<autograd::Variable>& parameters, float max_norm)
{
    if (!(max_norm > 0.0f))
    {
        throw std::invalid_argument("clip_gradient_norm: max_norm must be positive");
    }
    int64_t largest = 1;
    for (const auto& p : parameters)
    {
        largest = std::max<int64_t>(largest, static_cast<int64_t>(p.value().numel()));
    }
    const size_t ws = veda_sumsq_workspace(largest);
    Tensor work = Tensor::empty(Shape({(ws + 3) / 4 + 1}), DType::F32);
    Tensor sumsq(Shape({2}), DType::F32);
    double* ss = static_cast<double*>(sumsq.data_ptr());
    bool first = true;
    std::vector<Tensor> grads;
    for (const auto& p : parameters)
    {
        if (!p.requires_grad())
        {
            continue;
        }
        Tensor g = p.grad();
        if (g.dtype() != DType::F32 || !g.is_contiguous())
        {
            throw std::invalid_argument("clip_gradient_norm: gradients must be contiguous fp32");
        }
        check(veda_sumsq(fptr(g), static_cast<int64_t>(g.numel()), ss, first ? 0 : 1,
                         work.data_ptr(), work.numel() * 4, current_stream()),
              "clip_gradient_norm");
        first = false;
        grads.push_back(g);
    }
    double host = 0.0;
    if (cudaMemcpyAsync(&host, ss, sizeof(double), cudaMemcpyDeviceToHost, cs()) != cudaSuccess ||
        cudaStreamSynchronize(cs()) != cudaSuccess)
    {
        throw std::runtime_error("clip_gradient_norm: read failed");
    }
    const double total = std::sqrt(host);
    if (!std::isfinite(total) || total <= static_cast<double>(max_norm))
    {
        return static_cast<float>(total);   // reported, nothing written
    }
    for (const Tensor& g : grads)
    {
        check(veda_clip_apply(fptr(g), static_cast<int64_t>(g.numel()), ss, max_norm,
                              current_stream()),
              "clip_gradient_norm");
    }
    return static_cast<float>(total);
}

} // namespace veda::optim
