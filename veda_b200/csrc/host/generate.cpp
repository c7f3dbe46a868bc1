// Greedy generation on the device (include/veda/generate.hpp).
#include "veda/generate.hpp"

#include "veda_cuda.h"

#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <stdexcept>
#include <string>

namespace veda::generate
{

using core::DType;
using core::Shape;
using core::Tensor;

namespace
{
cudaStream_t cs() { return reinterpret_cast<cudaStream_t>(current_stream()); }

void cuda_check(cudaError_t e, const char* what)
{
    if (e != cudaSuccess)
    {
        throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
    }
}

int dt(DType d) { return d == DType::BF16 ? VEDA_BF16 : VEDA_F32; }

// element `i` of a tensor's storage, as a byte pointer
char* at(const Tensor& t, size_t i)
{
    return static_cast<char*>(t.data_ptr()) + i * core::dtype_size(t.dtype());
}

// One row through a Linear layer: y[n] = x[k] . w[n, k] (the decode step's projections).
void gemv(const void* x, const void* w, size_t ldw, void* y, size_t n, size_t k, int d)
{
    check(veda_gemv_nt(x, w, static_cast<int64_t>(ldw), y, static_cast<int64_t>(n), static_cast<int64_t>(k), d,
                       current_stream()),
          "generate: gemv");
}

void gemm_nt(size_t m, size_t n, size_t k, const void* a, size_t lda, const void* b, size_t ldb,
             void* c, size_t ldc, int dtype)
{
    check(veda_gemm_nt(static_cast<int64_t>(m), static_cast<int64_t>(n), static_cast<int64_t>(k), a,
                       static_cast<int64_t>(lda), b, static_cast<int64_t>(ldb), c, static_cast<int64_t>(ldc),
                       dtype, dtype, 1.0f, 0.0f, current_stream()),
          "generate: linear");
}
} // namespace

// Keys and values of every layer, after QK-norm and RoPE, one row per position
// (src/libs/model/KVCache.h): [capacity, Hkv * Dh] each.
struct Generator::Cache
{
    std::vector<Tensor> k, v;
};

// One recorded decode step: its graph, the stream it was recorded on, and the fixed buffers it
// reads and writes. io holds the token id (int64) at [0, 8) and the argmax status (int) at [8, 12);
// pos the position (int64) of the token being fed.
struct Generator::DecodeStep
{
    Tensor io, pos, x, xs, a, qkv, qr, ctx, o, hb, dn, logits, workspace, pick;
    cudaGraphExec_t exec = nullptr;
    cudaStream_t stream = nullptr;

    DecodeStep() = default;
    DecodeStep(const DecodeStep&) = delete;
    DecodeStep& operator=(const DecodeStep&) = delete;
    ~DecodeStep()
    {
        if (exec != nullptr) cudaGraphExecDestroy(exec);
        if (stream != nullptr) cudaStreamDestroy(stream);
    }
};

Generator::Generator(const train::TinyTransformer& model) : model_(model) {}

void Generator::record_step(DecodeStep& st, Cache& cache, const Tensor& cosines,
                            const Tensor& sines) const
{
    const train::ModelConfig& c = model_.config_;
    const size_t D = c.hidden_size, F = c.intermediate_size, H = c.num_heads, Hk = c.num_kv_heads,
                 Dh = c.head_dim, V = c.vocab_size;
    const size_t W = (H + 2 * Hk) * Dh, KV = Hk * Dh;
    const DType dtype = model_.dtype_;
    const int d = dt(dtype);
    const float eps = c.rms_norm_eps;
    const float scale = 1.0f / std::sqrt(static_cast<float>(Dh));
    st.io = Tensor(Shape({4}), DType::F32);
    st.pos = Tensor(Shape({2}), DType::F32);
    st.x = Tensor::empty(Shape({1, D}), dtype);
    st.xs = Tensor::empty(Shape({1, D}), dtype);
    st.a = Tensor::empty(Shape({1, D}), dtype);
    st.qkv = Tensor::empty(Shape({1, W}), dtype);
    st.qr = Tensor::empty(Shape({1, H * Dh}), dtype);
    st.ctx = Tensor::empty(Shape({1, H * Dh}), dtype);
    st.o = Tensor::empty(Shape({1, D}), dtype);
    st.hb = Tensor::empty(Shape({1, F}), dtype);
    st.dn = Tensor::empty(Shape({1, D}), dtype);
    st.logits = Tensor::empty(Shape({V}), dtype);
    // q/k/v handling and attention in one launch where its kernel takes the shape
    const bool fused = Dh == 128 && (H / Hk == 1 || H / Hk == 2 || H / Hk == 4 || H / Hk == 8) && KV % 8 == 0 &&
                       !cache.k.empty();
    const int64_t capacity = cache.k.empty() ? 0 : static_cast<int64_t>(cache.k[0].shape()[0]);
    const int64_t ws =
        fused ? veda_decode_attention_workspace(static_cast<int64_t>(H), static_cast<int64_t>(Hk), capacity) : 0;
    if (fused)
    {
        st.workspace = Tensor(Shape({static_cast<size_t>(ws + 3) / 4}), DType::F32);   // zero-filled
    }
    const int64_t pick_ws = veda_gemv_argmax_workspace(static_cast<int64_t>(V));
    st.pick = Tensor(Shape({static_cast<size_t>(pick_ws + 3) / 4}), DType::F32);
    cuda_check(cudaStreamSynchronize(cs()), "decode step buffers");
    cuda_check(cudaStreamCreateWithFlags(&st.stream, cudaStreamNonBlocking), "decode stream");
    const veda_stream_t caller = current_stream();
    set_current_stream(st.stream);
    cudaGraph_t graph = nullptr;
    cuda_check(cudaStreamBeginCapture(st.stream, cudaStreamCaptureModeThreadLocal), "decode capture");
    try
    {
        int64_t* token = static_cast<int64_t*>(st.io.data_ptr());
        int* status = reinterpret_cast<int*>(token + 1);
        const int64_t* pos = static_cast<const int64_t*>(st.pos.data_ptr());
        const float* cp = static_cast<const float*>(cosines.data_ptr());
        const float* sp = static_cast<const float*>(sines.data_ptr());
        Tensor* x = &st.x;
        Tensor* xs = &st.xs;
        check(veda_embedding_fwd(token, 1, model_.embed_.value().data_ptr(), static_cast<int64_t>(V),
                                 static_cast<int64_t>(D), x->data_ptr(), static_cast<int64_t>(D), nullptr, d,
                                 current_stream()),
              "generate: embedding");
        const auto& layers = model_.layers_;
        // Each pre-norm runs inside the projection that follows it; `delta` is the sublayer output
        // still to be added to the residual x (none before the first layer).
        const void* delta = nullptr;
        auto normed_gemv = [&](const Tensor& gain, const Tensor& w, size_t n, void* y, bool swiglu) {
            void* sum = delta != nullptr ? xs->data_ptr() : nullptr;
            const int rc = swiglu ? veda_gemv_rmsnorm_swiglu(x->data_ptr(), delta, gain.data_ptr(), eps, sum,
                                                             w.data_ptr(), static_cast<int64_t>(D), y,
                                                             static_cast<int64_t>(n), static_cast<int64_t>(D), d,
                                                             current_stream())
                                  : veda_gemv_rmsnorm(x->data_ptr(), delta, gain.data_ptr(), eps, sum,
                                                      w.data_ptr(), static_cast<int64_t>(D), y,
                                                      static_cast<int64_t>(n), static_cast<int64_t>(D), d,
                                                      current_stream());
            check(rc, "generate: norm + projection");
            if (delta != nullptr) std::swap(x, xs);
            delta = nullptr;
        };
        for (size_t l = 0; l < layers.size(); ++l)
        {
            const auto& L = layers[l];
            normed_gemv(L.in_norm.value(), L.qkv.value(), W, st.qkv.data_ptr(), false);
            if (fused)
            {
                check(veda_decode_attention_at(st.qkv.data_ptr(), L.q_norm.value().data_ptr(),
                                               L.k_norm.value().data_ptr(), cp, sp, pos, cache.k[l].data_ptr(),
                                               cache.v[l].data_ptr(), static_cast<int64_t>(KV), capacity,
                                               static_cast<int64_t>(H), static_cast<int64_t>(Hk),
                                               static_cast<int64_t>(Dh), eps, scale, st.ctx.data_ptr(),
                                               st.workspace.data_ptr(), ws, d, current_stream()),
                      "generate: q/k/v + attention");
            }
            else
            {
                check(veda_decode_qkv_at(st.qkv.data_ptr(), L.q_norm.value().data_ptr(),
                                         L.k_norm.value().data_ptr(), cp, sp, pos, st.qr.data_ptr(),
                                         cache.k[l].data_ptr(), cache.v[l].data_ptr(), static_cast<int64_t>(KV),
                                         static_cast<int64_t>(H), static_cast<int64_t>(Hk),
                                         static_cast<int64_t>(Dh), eps, d, current_stream()),
                      "generate: q/k/v");
                check(veda_attention_decode_at(st.qr.data_ptr(), cache.k[l].data_ptr(), cache.v[l].data_ptr(),
                                               static_cast<int64_t>(KV), pos, static_cast<int64_t>(H),
                                               static_cast<int64_t>(Hk), static_cast<int64_t>(Dh), scale,
                                               st.ctx.data_ptr(), d, current_stream()),
                      "generate: attention");
            }
            gemv(st.ctx.data_ptr(), L.o.value().data_ptr(), H * Dh, st.o.data_ptr(), D, H * Dh, d);
            delta = st.o.data_ptr();
            normed_gemv(L.post_norm.value(), L.gate_up.value(), F, st.hb.data_ptr(), true);
            gemv(st.hb.data_ptr(), L.down.value().data_ptr(), F, st.dn.data_ptr(), D, F, d);
            delta = st.dn.data_ptr();
        }
        // the final norm, the tied LM head and the greedy choice in one launch
        check(veda_gemv_rmsnorm_argmax(x->data_ptr(), delta, model_.final_norm_.value().data_ptr(), eps, nullptr,
                                       model_.embed_.value().data_ptr(), static_cast<int64_t>(D),
                                       st.logits.data_ptr(), static_cast<int64_t>(V), static_cast<int64_t>(D),
                                       token, status, st.pick.data_ptr(), pick_ws, d, current_stream()),
              "generate: norm + LM head + argmax");
        check(veda_decode_advance(static_cast<int64_t*>(st.pos.data_ptr()), current_stream()), "generate: position");
    }
    catch (...)
    {
        set_current_stream(caller);
        cudaStreamEndCapture(st.stream, &graph);
        if (graph != nullptr) cudaGraphDestroy(graph);
        throw;
    }
    set_current_stream(caller);
    cuda_check(cudaStreamEndCapture(st.stream, &graph), "decode capture");
    const cudaError_t e = cudaGraphInstantiate(&st.exec, graph, 0);
    cudaGraphDestroy(graph);
    cuda_check(e, "decode graph instantiate");
}

Tensor Generator::forward(const std::vector<int32_t>& ids, size_t pos0, Cache* cache,
                          const Tensor& cosines, const Tensor& sines) const
{
    const train::ModelConfig& c = model_.config_;
    const size_t n = ids.size(), D = c.hidden_size, F = c.intermediate_size, H = c.num_heads,
                 Hk = c.num_kv_heads, Dh = c.head_dim, V = c.vocab_size;
    const size_t W = (H + 2 * Hk) * Dh, KV = Hk * Dh;
    const DType dtype = model_.dtype_;
    const int d = dt(dtype);
    const size_t es = core::dtype_size(dtype);
    const float eps = c.rms_norm_eps;
    const float scale = 1.0f / std::sqrt(static_cast<float>(Dh));
    std::vector<int64_t> host(ids.begin(), ids.end());
    Tensor idt = Tensor::empty(Shape({2 * n}), DType::F32);   // int64 payloads
    cuda_check(cudaMemcpyAsync(idt.data_ptr(), host.data(), n * sizeof(int64_t), cudaMemcpyHostToDevice, cs()),
               "generate: ids");
    Tensor x = Tensor::empty(Shape({n, D}), dtype), xs = Tensor::empty(Shape({n, D}), dtype),
           a = Tensor::empty(Shape({n, D}), dtype);
    check(veda_embedding_fwd(static_cast<const int64_t*>(idt.data_ptr()), static_cast<int64_t>(n),
                             model_.embed_.value().data_ptr(), static_cast<int64_t>(V), static_cast<int64_t>(D),
                             x.data_ptr(), static_cast<int64_t>(D), nullptr, d, current_stream()),
          "generate: embedding");
    const auto& layers = model_.layers_;
    const Tensor& first_gain = layers.empty() ? model_.final_norm_.value() : layers[0].in_norm.value();
    check(veda_rmsnorm_fwd(x.data_ptr(), static_cast<int64_t>(D), first_gain.data_ptr(), a.data_ptr(),
                           static_cast<int64_t>(D), static_cast<int64_t>(n), static_cast<int64_t>(D), eps, d,
                           current_stream()),
          "generate: norm");
    Tensor qkv = Tensor::empty(Shape({n, W}), dtype), qr = Tensor::empty(Shape({n, H * Dh}), dtype),
           kr = Tensor::empty(Shape({n, KV}), dtype), ctx = Tensor::empty(Shape({n, H * Dh}), dtype),
           lse = Tensor::empty(Shape({H * n}), DType::F32), o = Tensor::empty(Shape({n, D}), dtype),
           gu = Tensor::empty(Shape({n, 2 * F}), dtype), hb = Tensor::empty(Shape({n, F}), dtype),
           dn = Tensor::empty(Shape({n, D}), dtype);
    const float* cp = static_cast<const float*>(cosines.data_ptr()) + pos0 * Dh;
    const float* sp = static_cast<const float*>(sines.data_ptr()) + pos0 * Dh;
    const auto N = static_cast<int64_t>(n);
    for (size_t l = 0; l < layers.size(); ++l)
    {
        const auto& L = layers[l];
        gemm_nt(n, W, D, a.data_ptr(), D, L.qkv.value().data_ptr(), D, qkv.data_ptr(), W, d);
        check(veda_qknorm_rope_fwd(qkv.data_ptr(), static_cast<int64_t>(W), L.q_norm.value().data_ptr(), cp, sp,
                                   qr.data_ptr(), static_cast<int64_t>(H * Dh), N, static_cast<int64_t>(H), N,
                                   static_cast<int64_t>(Dh), eps, d, current_stream()),
              "generate: q norm");
        void* kdst = cache ? at(cache->k[l], pos0 * KV) : kr.data_ptr();
        check(veda_qknorm_rope_fwd(at(qkv, H * Dh), static_cast<int64_t>(W), L.k_norm.value().data_ptr(), cp, sp,
                                   kdst, static_cast<int64_t>(KV), N, static_cast<int64_t>(Hk), N,
                                   static_cast<int64_t>(Dh), eps, d, current_stream()),
              "generate: k norm");
        const void* ksrc = cache ? cache->k[l].data_ptr() : kr.data_ptr();
        const void* vsrc = at(qkv, (H + Hk) * Dh);
        int64_t ldv = static_cast<int64_t>(W);
        if (cache)
        {
            cuda_check(cudaMemcpy2DAsync(at(cache->v[l], pos0 * KV), KV * es, vsrc, W * es, KV * es, n,
                                         cudaMemcpyDeviceToDevice, cs()),
                       "generate: cache values");
            vsrc = cache->v[l].data_ptr();
            ldv = static_cast<int64_t>(KV);
        }
        if (cache && pos0 > 0)
        {
            if (n != 1)
            {
                throw std::logic_error("generate: a cached step feeds one token");
            }
            check(veda_attention_decode(qr.data_ptr(), ksrc, vsrc, static_cast<int64_t>(KV),
                                        static_cast<int64_t>(pos0 + 1), static_cast<int64_t>(H),
                                        static_cast<int64_t>(Hk), static_cast<int64_t>(Dh), scale, ctx.data_ptr(), d,
                                        current_stream()),
                  "generate: attention");
        }
        else
        {
            check(veda_attention_fwd(qr.data_ptr(), static_cast<int64_t>(H * Dh), ksrc, static_cast<int64_t>(KV),
                                     vsrc, ldv, ctx.data_ptr(), static_cast<int64_t>(H * Dh),
                                     static_cast<float*>(lse.data_ptr()), 1, N, static_cast<int64_t>(H),
                                     static_cast<int64_t>(Hk), static_cast<int64_t>(Dh), scale, 1, d,
                                     current_stream()),
                  "generate: attention");
        }
        gemm_nt(n, D, H * Dh, ctx.data_ptr(), H * Dh, L.o.value().data_ptr(), H * Dh, o.data_ptr(), D, d);
        check(veda_add_rmsnorm_fwd(x.data_ptr(), static_cast<int64_t>(D), o.data_ptr(), static_cast<int64_t>(D),
                                   L.post_norm.value().data_ptr(), xs.data_ptr(), static_cast<int64_t>(D),
                                   a.data_ptr(), static_cast<int64_t>(D), N, static_cast<int64_t>(D), eps, d,
                                   current_stream()),
              "generate: residual + norm");
        std::swap(x, xs);
        gemm_nt(n, 2 * F, D, a.data_ptr(), D, L.gate_up.value().data_ptr(), D, gu.data_ptr(), 2 * F, d);
        check(veda_swiglu_fwd(gu.data_ptr(), static_cast<int64_t>(2 * F), at(gu, F), static_cast<int64_t>(2 * F),
                              hb.data_ptr(), static_cast<int64_t>(F), N, static_cast<int64_t>(F), d,
                              current_stream()),
              "generate: swiglu");
        gemm_nt(n, D, F, hb.data_ptr(), F, L.down.value().data_ptr(), F, dn.data_ptr(), D, d);
        const Tensor& next = l + 1 < layers.size() ? layers[l + 1].in_norm.value() : model_.final_norm_.value();
        check(veda_add_rmsnorm_fwd(x.data_ptr(), static_cast<int64_t>(D), dn.data_ptr(), static_cast<int64_t>(D),
                                   next.data_ptr(), xs.data_ptr(), static_cast<int64_t>(D), a.data_ptr(),
                                   static_cast<int64_t>(D), N, static_cast<int64_t>(D), eps, d, current_stream()),
              "generate: residual + norm");
        std::swap(x, xs);
    }
    // the tied LM head on the last position only (LMHead.cpp forward_last)
    Tensor logits = Tensor::empty(Shape({V}), dtype);
    gemm_nt(1, V, D, at(a, (n - 1) * D), D, model_.embed_.value().data_ptr(), D, logits.data_ptr(), V, d);
    return logits;
}

int32_t Generator::pick(const Tensor& logits) const
{
    Tensor out = Tensor(Shape({4}), DType::F32);   // int64 index + int status
    int64_t* index = static_cast<int64_t*>(out.data_ptr());
    int* status = reinterpret_cast<int*>(index + 1);
    const auto V = static_cast<int64_t>(logits.numel());
    check(veda_argmax(logits.data_ptr(), V, 1, V, index, status, dt(logits.dtype()), current_stream()),
          "generate: argmax");
    int64_t host[2] = {0, 0};
    cuda_check(cudaMemcpyAsync(host, out.data_ptr(), sizeof(host), cudaMemcpyDeviceToHost, cs()), "generate: argmax");
    cuda_check(cudaStreamSynchronize(cs()), "generate: argmax");
    int st = 0;
    std::memcpy(&st, &host[1], sizeof(int));
    if (st != 0)
    {
        throw std::runtime_error("generate: a logit is NaN");
    }
    return static_cast<int32_t>(host[0]);
}

namespace
{
void validate(const train::ModelConfig& c, const std::vector<int32_t>& prompt, const Options& o)
{
    if (prompt.empty())
    {
        throw std::invalid_argument("generate: the prompt is empty — there is nothing to condition on");
    }
    for (const int32_t id : prompt)
    {
        if (id < 0 || static_cast<size_t>(id) >= c.vocab_size)
        {
            throw std::invalid_argument("generate: token id " + std::to_string(id) + " is outside the vocabulary");
        }
    }
    const size_t longest = prompt.size() + o.max_new_tokens;
    if (c.max_position_embeddings != 0 && longest > c.max_position_embeddings)
    {
        throw std::invalid_argument("generate: " + std::to_string(longest) + " positions exceed the context");
    }
}

bool stops(const Options& o, int32_t id)
{
    return std::find(o.stop_tokens.begin(), o.stop_tokens.end(), id) != o.stop_tokens.end();
}
} // namespace

Result Generator::generate(const std::vector<int32_t>& prompt, const Options& options) const
{
    const train::ModelConfig& c = model_.config_;
    validate(c, prompt, options);
    const auto tables = train::rope_tables(prompt.size() + options.max_new_tokens + 1, c.head_dim, c.rope_theta);
    Result result;
    std::vector<int32_t> ids(prompt);
    for (size_t step = 0; step < options.max_new_tokens; ++step)
    {
        const int32_t next = pick(forward(ids, 0, nullptr, tables.first, tables.second));
        ++result.forward_passes;
        if (stops(options, next))
        {
            result.stopped_on_token = true;
            break;
        }
        result.generated.push_back(next);
        ids.push_back(next);
    }
    return result;
}

Result Generator::generate_cached(const std::vector<int32_t>& prompt, const Options& options) const
{
    const train::ModelConfig& c = model_.config_;
    validate(c, prompt, options);
    const size_t capacity = prompt.size() + options.max_new_tokens + 1;
    const auto tables = train::rope_tables(capacity, c.head_dim, c.rope_theta);
    Cache cache;
    for (size_t l = 0; l < c.num_layers; ++l)
    {
        cache.k.push_back(Tensor::empty(Shape({capacity, c.num_kv_heads * c.head_dim}), model_.dtype_));
        cache.v.push_back(Tensor::empty(Shape({capacity, c.num_kv_heads * c.head_dim}), model_.dtype_));
    }
    static const bool use_graph = [] {
        const char* v = std::getenv("VEDA_DECODE_GRAPH");
        return v == nullptr || std::atoi(v) != 0;
    }();
    Result result;
    // the prefill (Generator.cpp:73-78 with the whole prompt pending)
    Tensor logits = forward(prompt, 0, &cache, tables.first, tables.second);
    ++result.forward_passes;
    size_t pos = prompt.size();
    if (options.max_new_tokens == 0)
    {
        return result;   // the prefill still had to run; this is the limit, not an extra token
    }
    int32_t next = pick(logits);
    DecodeStep st;
    for (size_t step = 1;; ++step)
    {
        if (stops(options, next))
        {
            result.stopped_on_token = true;
            break;
        }
        result.generated.push_back(next);
        // feed the token just chosen (one token per step after the prefill)
        if (use_graph)
        {
            if (st.exec == nullptr)
            {
                record_step(st, cache, tables.first, tables.second);
                const int64_t init[2] = {next, 0};
                const auto p = static_cast<int64_t>(pos);
                cuda_check(cudaMemcpyAsync(st.io.data_ptr(), init, sizeof(init), cudaMemcpyHostToDevice, cs()),
                           "decode token");
                cuda_check(cudaMemcpyAsync(st.pos.data_ptr(), &p, sizeof(p), cudaMemcpyHostToDevice, cs()),
                           "decode position");
            }
            cuda_check(cudaGraphLaunch(st.exec, cs()), "decode step");
        }
        else
        {
            logits = forward({next}, pos, &cache, tables.first, tables.second);
        }
        ++pos;
        ++result.forward_passes;
        if (step == options.max_new_tokens)
        {
            break;   // the limit: the last token was fed, none is chosen from it
        }
        if (use_graph)
        {
            int64_t io[2] = {0, 0};
            cuda_check(cudaMemcpyAsync(io, st.io.data_ptr(), sizeof(io), cudaMemcpyDeviceToHost, cs()),
                       "decode token");
            cuda_check(cudaStreamSynchronize(cs()), "decode token");
            int status = 0;
            std::memcpy(&status, &io[1], sizeof(int));
            if (status != 0)
            {
                throw std::runtime_error("generate: a logit is NaN");
            }
            next = static_cast<int32_t>(io[0]);
        }
        else
        {
            next = pick(logits);
        }
    }
    cuda_check(cudaStreamSynchronize(cs()), "decode");
    return result;
}

std::vector<float> Generator::last_logits(const std::vector<int32_t>& ids) const
{
    const train::ModelConfig& c = model_.config_;
    validate(c, ids, Options{0, {}});
    const auto tables = train::rope_tables(ids.size(), c.head_dim, c.rope_theta);
    const Tensor logits = forward(ids, 0, nullptr, tables.first, tables.second);
    const size_t V = c.vocab_size;
    std::vector<float> out(V);
    if (logits.dtype() == DType::F32)
    {
        cuda_check(cudaMemcpyAsync(out.data(), logits.data_ptr(), V * 4, cudaMemcpyDeviceToHost, cs()), "logits");
        cuda_check(cudaStreamSynchronize(cs()), "logits");
    }
    else
    {
        std::vector<uint16_t> raw(V);
        cuda_check(cudaMemcpyAsync(raw.data(), logits.data_ptr(), V * 2, cudaMemcpyDeviceToHost, cs()), "logits");
        cuda_check(cudaStreamSynchronize(cs()), "logits");
        for (size_t i = 0; i < V; ++i)
        {
            const uint32_t w = static_cast<uint32_t>(raw[i]) << 16;
            std::memcpy(&out[i], &w, 4);
        }
    }
    return out;
}

} // namespace veda::generate
