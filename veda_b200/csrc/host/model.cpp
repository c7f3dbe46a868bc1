// veda::train::TinyTransformer on the device (src/libs/train/Model.cpp:72-255, with GQA).
#include "veda/model.hpp"
#include "veda/train.hpp"

#include "veda_cuda.h"

#include <cuda_runtime.h>

#include <cmath>
#include <stdexcept>

namespace veda::train
{

using autograd::Variable;
using core::DType;
using core::Shape;
using core::Tensor;

ModelConfig tiny_config()
{
    ModelConfig c;
    c.hidden_size = 128;
    c.intermediate_size = 512;
    c.num_layers = 4;
    c.num_heads = 4;
    c.num_kv_heads = 4;
    c.head_dim = 32;
    c.vocab_size = 256;
    c.max_position_embeddings = 256;
    c.rms_norm_eps = 1e-6f;
    c.rope_theta = 10000.0f;
    c.tie_word_embeddings = true;
    return c;
}

std::pair<Tensor, Tensor> rope_tables(size_t positions, size_t head_dim, float theta)
{
    model::RopeTables t = model::rope_tables(positions, head_dim, theta, 0);
    return {t.cosines, t.sines};
}

} // namespace veda::train

namespace veda::model
{

using core::Shape;
using core::Tensor;

RopeTables rope_tables(size_t positions, size_t head_dim, float theta, size_t first_position)
{
    if (head_dim == 0 || head_dim % 2 != 0)
    {
        throw std::invalid_argument("rope_tables: head_dim must be even, got " +
                                    std::to_string(head_dim));
    }
    if (!(theta > 0.0f))
    {
        throw std::invalid_argument("rope_tables: theta must be positive");
    }
    // angles in double, cast per element, each written to both halves (Rope.cpp:37-59)
    const size_t pairs = head_dim / 2;
    std::vector<float> c(positions * head_dim), s(positions * head_dim);
    for (size_t p = 0; p < positions; ++p)
    {
        for (size_t i = 0; i < pairs; ++i)
        {
            const double freq = std::pow(static_cast<double>(theta),
                                         -2.0 * static_cast<double>(i) / static_cast<double>(head_dim));
            const double angle = static_cast<double>(first_position + p) * freq;
            const float cv = static_cast<float>(std::cos(angle));
            const float sv = static_cast<float>(std::sin(angle));
            c[p * head_dim + i] = c[p * head_dim + i + pairs] = cv;
            s[p * head_dim + i] = s[p * head_dim + i + pairs] = sv;
        }
    }
    return {Tensor::from_host(c, Shape({positions, head_dim})),
            Tensor::from_host(s, Shape({positions, head_dim}))};
}

Tensor apply_rope(const Tensor& x, const RopeTables& tables)
{
    if (x.rank() < 2 || tables.cosines.rank() != 2 || tables.sines.shape() != tables.cosines.shape())
    {
        throw std::invalid_argument("apply_rope: expected x [.., T, Dh] and tables [T, Dh], got " +
                                    x.shape().to_string() + " and " +
                                    tables.cosines.shape().to_string());
    }
    const size_t T = x.shape()[x.rank() - 2], Dh = x.shape()[x.rank() - 1];
    if (tables.cosines.shape()[0] != T || tables.cosines.shape()[1] != Dh)
    {
        throw std::invalid_argument("apply_rope: tables " + tables.cosines.shape().to_string() +
                                    " do not match x " + x.shape().to_string());
    }
    const Tensor c = core::contiguous(x);
    Tensor out = Tensor::empty(c.shape(), c.dtype());
    const Tensor cs = core::to_dtype(tables.cosines, core::DType::F32);
    const Tensor sn = core::to_dtype(tables.sines, core::DType::F32);
    const size_t lanes = T * Dh == 0 ? 0 : c.numel() / (T * Dh);
    check(veda_rope(c.data_ptr(), out.data_ptr(), static_cast<const float*>(cs.data_ptr()),
                    static_cast<const float*>(sn.data_ptr()), static_cast<int64_t>(lanes),
                    static_cast<int64_t>(T), static_cast<int64_t>(Dh), 0,
                    static_cast<int>(c.dtype()), current_stream()),
          "apply_rope");
    return out;
}

} // namespace veda::model

namespace veda::train
{

namespace
{
std::string layer_name(size_t layer, const std::string& suffix)
{
    return "model.layers." + std::to_string(layer) + "." + suffix + ".weight";
}
} // namespace

TinyTransformer::TinyTransformer(ModelConfig config, uint64_t seed, DType dtype)
    : config_(std::move(config)), dtype_(dtype)
{
    const size_t D = config_.hidden_size, F = config_.intermediate_size, H = config_.num_heads,
                 Hk = config_.num_kv_heads, Dh = config_.head_dim, V = config_.vocab_size,
                 L = config_.num_layers;
    if (H == 0 || Hk == 0 || H % Hk != 0)
    {
        throw std::invalid_argument("TinyTransformer: heads must be a positive multiple of kv_heads");
    }
    if (!config_.tie_word_embeddings)
    {
        throw std::invalid_argument("TinyTransformer: only tied embeddings are supported");
    }
    if (D == 0 || F == 0 || Dh == 0 || V == 0)
    {
        throw std::invalid_argument("TinyTransformer: zero-sized dimension");
    }
    // parameter table in the reference's order (Model.cpp:120-140)
    struct Spec
    {
        std::string name;
        Shape shape;
        bool gain;
    };
    std::vector<Spec> specs;
    specs.push_back({"model.embed_tokens.weight", Shape({V, D}), false});
    for (size_t l = 0; l < L; ++l)
    {
        specs.push_back({layer_name(l, "input_layernorm"), Shape({D}), true});
        specs.push_back({layer_name(l, "self_attn.q_proj"), Shape({H * Dh, D}), false});
        specs.push_back({layer_name(l, "self_attn.k_proj"), Shape({Hk * Dh, D}), false});
        specs.push_back({layer_name(l, "self_attn.v_proj"), Shape({Hk * Dh, D}), false});
        specs.push_back({layer_name(l, "self_attn.o_proj"), Shape({D, H * Dh}), false});
        specs.push_back({layer_name(l, "self_attn.q_norm"), Shape({Dh}), true});
        specs.push_back({layer_name(l, "self_attn.k_norm"), Shape({Dh}), true});
        specs.push_back({layer_name(l, "post_attention_layernorm"), Shape({D}), true});
        specs.push_back({layer_name(l, "mlp.gate_proj"), Shape({F, D}), false});
        specs.push_back({layer_name(l, "mlp.up_proj"), Shape({F, D}), false});
        specs.push_back({layer_name(l, "mlp.down_proj"), Shape({D, F}), false});
    }
    specs.push_back({"model.norm.weight", Shape({D}), true});

    // offsets rounded to 8 elements (16-byte aligned rows for both dtypes)
    std::vector<size_t> offsets;
    total_ = 0;
    for (const Spec& s : specs)
    {
        offsets.push_back(total_);
        total_ += s.shape.size();
    }
    arena_len_ = (total_ + kArenaAlign - 1) / kArenaAlign * kArenaAlign;
    values_ = Tensor(Shape({arena_len_}), dtype_);
    grads_ = Tensor(Shape({arena_len_}), DType::F32);
    for (size_t i = 0; i < specs.size(); ++i)
    {
        Tensor v = Tensor::view(values_.storage(), offsets[i], specs[i].shape, dtype_);
        Tensor g = Tensor::view(grads_.storage(), offsets[i], specs[i].shape, DType::F32);
        if (specs[i].gain)
        {
            check(veda_fill(v.data_ptr(), 1.0f, static_cast<int64_t>(v.numel()),
                            static_cast<int>(dtype_), current_stream()),
                  "TinyTransformer: init");
        }
        else
        {
            check(veda_randn(v.data_ptr(), static_cast<int64_t>(v.numel()), 0.02f,
                             seed * 1000003ull + i, static_cast<int>(dtype_), current_stream()),
                  "TinyTransformer: init");
        }
        parameters_.push_back(Variable::parameter(v, g));
        names_.push_back(specs[i].name);
    }
    // graph leaves: q|k|v and gate|up fused
    auto group = [&](size_t first, size_t count, Shape shape) {
        Tensor v = Tensor::view(values_.storage(), offsets[first], shape, dtype_);
        Tensor g = Tensor::view(grads_.storage(), offsets[first], shape, DType::F32);
        (void)count;
        return Variable::parameter(v, g);
    };
    embed_ = parameters_[0];
    graph_leaves_.push_back({embed_, offsets[0], specs[0].shape.size()});
    for (size_t l = 0; l < L; ++l)
    {
        const size_t b = 1 + l * 11;
        Layer layer{parameters_[b],
                    group(b + 1, 3, Shape({(H + 2 * Hk) * Dh, D})),
                    parameters_[b + 4],
                    parameters_[b + 5],
                    parameters_[b + 6],
                    parameters_[b + 7],
                    group(b + 8, 2, Shape({2 * F, D})),
                    parameters_[b + 10]};
        graph_leaves_.push_back({layer.in_norm, offsets[b], D});
        graph_leaves_.push_back({layer.qkv, offsets[b + 1], (H + 2 * Hk) * Dh * D});
        graph_leaves_.push_back({layer.o, offsets[b + 4], D * H * Dh});
        graph_leaves_.push_back({layer.q_norm, offsets[b + 5], Dh});
        graph_leaves_.push_back({layer.k_norm, offsets[b + 6], Dh});
        graph_leaves_.push_back({layer.post_norm, offsets[b + 7], D});
        graph_leaves_.push_back({layer.gate_up, offsets[b + 8], 2 * F * D});
        graph_leaves_.push_back({layer.down, offsets[b + 10], D * F});
        layer_ranges_.push_back({offsets[b], offsets[b + 10] + D * F});
        layers_.push_back(std::move(layer));
    }
    final_norm_ = parameters_.back();
    graph_leaves_.push_back({final_norm_, offsets.back(), D});
    embed_range_ = {offsets[0], offsets[0] + specs[0].shape.size()};
    final_range_ = {offsets.back(), offsets.back() + D};
}

std::vector<std::pair<std::string, Tensor>> TinyTransformer::named_parameters() const
{
    std::vector<std::pair<std::string, Tensor>> named;
    for (size_t i = 0; i < parameters_.size(); ++i)
    {
        named.emplace_back(names_[i], parameters_[i].value());
    }
    return named;
}

void TinyTransformer::zero_grad()
{
    if (cudaMemsetAsync(grads_.data_ptr(), 0, total_ * sizeof(float),
                        reinterpret_cast<cudaStream_t>(current_stream())) != cudaSuccess)
    {
        throw std::runtime_error("TinyTransformer::zero_grad: memset failed");
    }
    for (auto& p : parameters_)
    {
        p.node()->grad_zero = true;
    }
    for (auto& g : graph_leaves_)
    {
        g.var.node()->grad_zero = true;
    }
}

void TinyTransformer::mark_grads_zero()
{
    for (auto& p : parameters_)
    {
        p.node()->grad_zero = true;
    }
    for (auto& g : graph_leaves_)
    {
        g.var.node()->grad_zero = true;
    }
}

void TinyTransformer::clear_untouched_grads()
{
    float* base = static_cast<float*>(grads_.data_ptr());
    for (auto& g : graph_leaves_)
    {
        if (g.var.node()->grad_zero &&
            cudaMemsetAsync(base + g.offset, 0, g.count * sizeof(float),
                            reinterpret_cast<cudaStream_t>(current_stream())) != cudaSuccess)
        {
            throw std::runtime_error("TinyTransformer::clear_untouched_grads: memset failed");
        }
    }
}

Variable TinyTransformer::forward(const std::vector<int64_t>& ids, size_t batch, size_t length)
{
    if (ids.size() != batch * length)
    {
        throw std::invalid_argument("TinyTransformer::forward: " + std::to_string(ids.size()) +
                                    " ids for a [" + std::to_string(batch) + ", " +
                                    std::to_string(length) + "] window");
    }
    if (config_.max_position_embeddings != 0 && length > config_.max_position_embeddings)
    {
        throw std::invalid_argument("TinyTransformer::forward: window of " +
                                    std::to_string(length) + " exceeds the context limit " +
                                    std::to_string(config_.max_position_embeddings));
    }
    if (gate_) gate_(embed_range_.first, embed_range_.second);
    Variable x = autograd::embedding(embed_, ids, Shape({batch * length}));
    return autograd::reshape(forward_from(x, batch, length),
                             Shape({batch, length, config_.vocab_size}));
}

Variable TinyTransformer::forward_device(const Tensor& ids, size_t batch, size_t length)
{
    if (config_.max_position_embeddings != 0 && length > config_.max_position_embeddings)
    {
        throw std::invalid_argument("TinyTransformer::forward: window exceeds the context limit");
    }
    if (gate_) gate_(embed_range_.first, embed_range_.second);
    Variable x = rows_sink_ ? autograd::embedding_device_rows(embed_, ids, rows_sink_)
                            : autograd::embedding_device(embed_, ids);
    return forward_from(x, batch, length);
}

Variable TinyTransformer::forward_from(const Variable& x0, size_t B, size_t T)
{
    const size_t H = config_.num_heads, Hk = config_.num_kv_heads, Dh = config_.head_dim;
    const float eps = config_.rms_norm_eps;
    auto it = rope_cache_.find(T);
    if (it == rope_cache_.end())
    {
        it = rope_cache_.emplace(T, rope_tables(T, Dh, config_.rope_theta)).first;
    }
    const Tensor& cosines = it->second.first;
    const Tensor& sines = it->second.second;
    // pre-norm residual blocks (Model.cpp:238-249); each residual add is fused with the norm
    // that reads its sum (the next block's input norm, or the final norm)
    Variable x = x0;
    if (gate_ && layers_.empty()) gate_(final_range_.first, final_range_.second);
    if (gate_ && !layers_.empty()) gate_(layer_ranges_[0].first, layer_ranges_[0].second);
    Variable a = autograd::rms_norm(x, layers_.empty() ? final_norm_ : layers_[0].in_norm, eps);
    for (size_t l = 0; l < layers_.size(); ++l)
    {
        const Layer& L = layers_[l];
        if (gate_ && l > 0) gate_(layer_ranges_[l].first, layer_ranges_[l].second);
        if (gate_ && l + 1 == layers_.size()) gate_(final_range_.first, final_range_.second);
        Variable qkv = autograd::linear(a, L.qkv);
        Variable proj =
            recompute_attention_
                ? autograd::attention_output(qkv, L.q_norm, L.k_norm, L.o, cosines, sines, B, T, H,
                                             Hk, Dh, eps)
                : autograd::linear(autograd::attention(qkv, L.q_norm, L.k_norm, cosines, sines, B,
                                                       T, H, Hk, Dh, eps),
                                   L.o);
        Variable b = autograd::add_rms_norm(x, proj, L.post_norm, eps, &x);
        const Variable& next = l + 1 < layers_.size() ? layers_[l + 1].in_norm : final_norm_;
        a = autograd::add_rms_norm(x, autograd::mlp(b, L.gate_up, L.down), next, eps, &x);
    }
    // tied LM head: the embedding matrix read the other way round (Model.cpp:253-254)
    return autograd::linear(a, embed_);
}

} // namespace veda::train
