// C ABI of libveda.so (include/veda_train.h): exceptions become status codes.
#include "veda_train.h"
#include "veda/checkpoint.hpp"
#include "veda/data.hpp"
#include "veda/generate.hpp"

#include "veda/profile.hpp"
#include "veda/train.hpp"

#include "veda_cuda.h"

#include <cuda_runtime.h>
#include <nccl.h>

#include <algorithm>
#include <cstring>
#include <memory>
#include <stdexcept>
#include <string>

struct veda_trainer
{
    std::unique_ptr<veda::train::Trainer> impl;
    int last_skipped = 0;   // the step read by the last step_host / last_stats was skipped
};

namespace
{
thread_local std::string g_error;

template <class F>
int guarded(F&& body)
{
    try
    {
        body();
        return VEDA_OK;
    }
    catch (const std::out_of_range& e)
    {
        g_error = e.what();
        return VEDA_ERR_OUT_OF_RANGE;
    }
    catch (const std::invalid_argument& e)
    {
        g_error = e.what();
        return VEDA_ERR_INVALID_ARGUMENT;
    }
    catch (const std::exception& e)
    {
        g_error = e.what();
        return VEDA_ERR_CUDA;
    }
}

void cuda_check(cudaError_t e, const char* what)
{
    if (e != cudaSuccess)
    {
        throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
    }
}

cudaStream_t cs() { return reinterpret_cast<cudaStream_t>(veda::current_stream()); }

// The fp32 flat vector of master weights: the model's values in fp32 mode, AdamW's master arena
// in bf16 mode (both contiguous in parameter order).
void* master_base(veda::train::Trainer& t) { return t.master_weights(); }
} // namespace

extern "C" {

const char* veda_train_last_error(void) { return g_error.c_str(); }

int veda_train_set_stream(veda_stream_t stream)
{
    veda::set_current_stream(stream);
    return VEDA_OK;
}

int veda_trainer_create(const veda_model_config* m, const veda_optim_config* o, int dtype,
                        int64_t batch, int64_t seq_len, uint64_t seed, veda_trainer** out)
{
    return guarded([&] {
        if (m == nullptr || o == nullptr || out == nullptr)
        {
            throw std::invalid_argument("veda_trainer_create: null argument");
        }
        if (dtype != 0 && dtype != 1)
        {
            throw std::invalid_argument("veda_trainer_create: dtype must be 0 (fp32) or 1 (bf16)");
        }
        veda::train::ModelConfig c;
        c.vocab_size = static_cast<size_t>(m->vocab);
        c.hidden_size = static_cast<size_t>(m->hidden);
        c.intermediate_size = static_cast<size_t>(m->intermediate);
        c.num_layers = static_cast<size_t>(m->layers);
        c.num_heads = static_cast<size_t>(m->heads);
        c.num_kv_heads = static_cast<size_t>(m->kv_heads);
        c.head_dim = static_cast<size_t>(m->head_dim);
        c.max_position_embeddings = 0;   // no context limit for synthetic training
        c.rms_norm_eps = m->eps;
        c.rope_theta = m->theta;
        veda::optim::AdamWConfig a{o->lr, o->beta1, o->beta2, o->eps, o->weight_decay};
        auto t = std::make_unique<veda_trainer>();
        t->impl = std::make_unique<veda::train::Trainer>(
            c, a, o->max_norm, dtype == 1 ? veda::core::DType::BF16 : veda::core::DType::F32,
            static_cast<size_t>(batch), static_cast<size_t>(seq_len), seed);
        *out = t.release();
    });
}

int veda_trainer_destroy(veda_trainer* t)
{
    return guarded([&] {
        if (t != nullptr)
        {
            cuda_check(cudaStreamSynchronize(cs()), "veda_trainer_destroy");
            delete t;
        }
    });
}

int64_t veda_trainer_param_count(const veda_trainer* t)
{
    return t ? static_cast<int64_t>(t->impl->model().parameter_count()) : -1;
}

int veda_trainer_set_params(veda_trainer* t, const float* host)
{
    return guarded([&] {
        auto& tr = *t->impl;
        tr.sync();   // no weight gather may still be writing the arena
        const size_t n = tr.model().parameter_count();
        void* master = master_base(tr);
        cuda_check(cudaMemcpyAsync(master, host, n * sizeof(float), cudaMemcpyHostToDevice, cs()),
                   "veda_trainer_set_params");
        if (tr.model().dtype() == veda::core::DType::BF16)
        {
            veda::check(veda_f32_to_bf16(static_cast<const float*>(master),
                                         tr.model().value_arena().data_ptr(),
                                         static_cast<int64_t>(n), veda::current_stream()),
                        "veda_trainer_set_params");
        }
        tr.master_weights_changed();
        cuda_check(cudaStreamSynchronize(cs()), "veda_trainer_set_params");
    });
}

int veda_trainer_get_params(veda_trainer* t, float* host)
{
    return guarded([&] {
        auto& tr = *t->impl;
        tr.gather_master_weights();
        cuda_check(cudaMemcpyAsync(host, master_base(tr),
                                   tr.model().parameter_count() * sizeof(float),
                                   cudaMemcpyDeviceToHost, cs()),
                   "veda_trainer_get_params");
        cuda_check(cudaStreamSynchronize(cs()), "veda_trainer_get_params");
    });
}

int veda_trainer_get_grads(veda_trainer* t, float* host)
{
    return guarded([&] {
        auto& tr = *t->impl;
        tr.gather_gradients();
        cuda_check(cudaMemcpyAsync(host, tr.model().grad_arena().data_ptr(),
                                   tr.model().parameter_count() * sizeof(float),
                                   cudaMemcpyDeviceToHost, cs()),
                   "veda_trainer_get_grads");
        cuda_check(cudaStreamSynchronize(cs()), "veda_trainer_get_grads");
    });
}

int veda_nccl_unique_id(void* out128)
{
    return guarded([&] {
        ncclUniqueId id;
        if (ncclGetUniqueId(&id) != ncclSuccess)
        {
            throw std::runtime_error("ncclGetUniqueId failed");
        }
        static_assert(sizeof(id) == 128, "NCCL unique id is 128 bytes");
        std::memcpy(out128, &id, sizeof(id));
    });
}

int veda_trainer_init_dp(veda_trainer* t, const void* unique_id128, int rank, int world,
                         size_t bucket_bytes)
{
    return guarded([&] { t->impl->init_data_parallel(unique_id128, rank, world, bucket_bytes); });
}

int veda_trainer_save_checkpoint(veda_trainer* t, const char* dir)
{
    return guarded([&] {
        if (dir == nullptr) throw std::invalid_argument("veda_trainer_save_checkpoint: null path");
        t->impl->save_checkpoint(dir);
    });
}

int veda_trainer_load_checkpoint(veda_trainer* t, const char* dir)
{
    return guarded([&] {
        if (dir == nullptr) throw std::invalid_argument("veda_trainer_load_checkpoint: null path");
        t->impl->load_checkpoint(dir);
    });
}

int veda_safetensors_write(const char* path, int64_t count, const char* const* names,
                           const char* const* dtypes, const int64_t* ranks, const int64_t* dims,
                           const void* const* data, int64_t meta_count, const char* const* meta_keys,
                           const char* const* meta_values)
{
    return guarded([&] {
        if (path == nullptr || count < 0 || meta_count < 0)
            throw std::invalid_argument("veda_safetensors_write: bad arguments");
        std::vector<veda::io::SafetensorsTensor> tensors;
        size_t d = 0;
        for (int64_t i = 0; i < count; ++i)
        {
            veda::io::SafetensorsTensor t;
            t.name = names[i];
            t.dtype = dtypes[i];
            size_t elems = 1;
            for (int64_t r = 0; r < ranks[i]; ++r)
            {
                t.shape.push_back(dims[d]);
                elems *= static_cast<size_t>(dims[d]);
                ++d;
            }
            const size_t bytes = elems * veda::io::dtype_bytes(t.dtype);
            const auto* p = static_cast<const uint8_t*>(data[i]);
            t.bytes.assign(p, p + bytes);
            tensors.push_back(std::move(t));
        }
        std::map<std::string, std::string> meta;
        for (int64_t i = 0; i < meta_count; ++i) meta[meta_keys[i]] = meta_values[i];
        veda::io::write_safetensors(path, tensors, meta);
    });
}

struct veda_corpus
{
    std::unique_ptr<veda::data::Corpus> impl;
};

int veda_corpus_create(const int64_t* ids, int64_t n, double validation_fraction, uint64_t seed,
                       veda_corpus** out)
{
    return guarded([&] {
        if (out == nullptr || n < 0 || (n > 0 && ids == nullptr))
            throw std::invalid_argument("veda_corpus_create: bad arguments");
        auto c = std::make_unique<veda_corpus>();
        c->impl = std::make_unique<veda::data::Corpus>(std::vector<int64_t>(ids, ids + n),
                                                       validation_fraction, seed);
        *out = c.release();
    });
}

int veda_corpus_destroy(veda_corpus* c)
{
    delete c;
    return 0;
}

int64_t veda_corpus_boundary(const veda_corpus* c)
{
    return c == nullptr ? -1 : static_cast<int64_t>(c->impl->boundary());
}

int veda_corpus_next_batch(veda_corpus* c, int64_t batch, int64_t length, int split,
                           int64_t* inputs, int64_t* targets)
{
    return guarded([&] {
        if (c == nullptr || batch < 0 || length < 0 || (split != 0 && split != 1))
            throw std::invalid_argument("veda_corpus_next_batch: bad arguments");
        c->impl->next_batch_into(static_cast<size_t>(batch), static_cast<size_t>(length),
                                 split ? veda::data::Split::Validation : veda::data::Split::Train,
                                 inputs, targets);
    });
}

int veda_trainer_set_step_graph(veda_trainer* t, int on)
{
    return guarded([&] { t->impl->set_step_graph(on != 0); });
}

int veda_trainer_generate(veda_trainer* t, const int32_t* prompt, int64_t n, int64_t max_new_tokens,
                          const int32_t* stop_tokens, int64_t n_stop, int cached, int32_t* out,
                          int64_t* out_count, int* stopped, int64_t* forward_passes)
{
    return guarded([&] {
        if (n < 0 || max_new_tokens < 0 || n_stop < 0 || (n > 0 && prompt == nullptr) ||
            (n_stop > 0 && stop_tokens == nullptr) || out_count == nullptr)
        {
            throw std::invalid_argument("veda_trainer_generate: bad arguments");
        }
        auto& tr = *t->impl;
        tr.sync();
        veda::generate::Options o;
        o.max_new_tokens = static_cast<size_t>(max_new_tokens);
        o.stop_tokens.assign(stop_tokens, stop_tokens + n_stop);
        const veda::generate::Generator g(tr.model());
        const std::vector<int32_t> p(prompt, prompt + n);
        const veda::generate::Result r = cached ? g.generate_cached(p, o) : g.generate(p, o);
        if (out != nullptr)
        {
            std::copy(r.generated.begin(), r.generated.end(), out);
        }
        *out_count = static_cast<int64_t>(r.generated.size());
        if (stopped) *stopped = r.stopped_on_token ? 1 : 0;
        if (forward_passes) *forward_passes = static_cast<int64_t>(r.forward_passes);
    });
}

int veda_trainer_last_logits(veda_trainer* t, const int32_t* ids, int64_t n, float* out)
{
    return guarded([&] {
        if (n <= 0 || ids == nullptr || out == nullptr)
        {
            throw std::invalid_argument("veda_trainer_last_logits: bad arguments");
        }
        auto& tr = *t->impl;
        tr.sync();
        const veda::generate::Generator g(tr.model());
        const std::vector<float> l = g.last_logits(std::vector<int32_t>(ids, ids + n));
        std::copy(l.begin(), l.end(), out);
    });
}

int veda_trainer_sync(veda_trainer* t)
{
    return guarded([&] { t->impl->sync(); });
}

int veda_trainer_init_dp_sharded(veda_trainer* t, const void* unique_id128, int rank, int world,
                                 size_t bucket_bytes)
{
    return guarded(
        [&] { t->impl->init_data_parallel(unique_id128, rank, world, bucket_bytes, true); });
}

int veda_trainer_step_host(veda_trainer* t, const int64_t* ids, const int64_t* targets,
                           float* loss, float* grad_norm)
{
    return guarded([&] {
        const auto s = t->impl->step_host(ids, targets);
        if (loss) *loss = s.loss;
        if (grad_norm) *grad_norm = s.grad_norm;
        t->last_skipped = s.skipped ? 1 : 0;
    });
}

int veda_trainer_step_device(veda_trainer* t, const int64_t* ids, const int64_t* targets)
{
    return guarded([&] {
        auto& tr = *t->impl;
        const size_t n = tr.batch() * tr.length();
        auto wrap = [&](const int64_t* p) {
            auto storage = std::make_shared<veda::core::Storage>(const_cast<int64_t*>(p),
                                                                 n * sizeof(int64_t));
            return veda::core::Tensor::view(storage, 0, veda::core::Shape({2 * n}),
                                            veda::core::DType::F32);
        };
        tr.step(wrap(ids), wrap(targets));
    });
}

int veda_trainer_last_stats(veda_trainer* t, float* loss, float* grad_norm)
{
    return guarded([&] {
        const auto s = t->impl->last_stats();
        if (loss) *loss = s.loss;
        if (grad_norm) *grad_norm = s.grad_norm;
        t->last_skipped = s.skipped ? 1 : 0;
    });
}

int veda_trainer_set_comm_timeout(veda_trainer* t, double seconds)
{
    return guarded([&] { t->impl->set_comm_timeout(seconds); });
}

int veda_trainer_abort_comm(veda_trainer* t)
{
    return guarded([&] { t->impl->abort_communication(); });
}

int veda_trainer_set_skip_nonfinite(veda_trainer* t, int on)
{
    return guarded([&] { t->impl->set_skip_nonfinite(on != 0); });
}

int veda_trainer_set_recompute_attention(veda_trainer* t, int on)
{
    return guarded([&] { t->impl->set_recompute_attention(on != 0); });
}

int veda_trainer_step_skipped(veda_trainer* t, int* skipped)
{
    return guarded([&] {
        if (skipped) *skipped = t->last_skipped;
    });
}

int veda_profile_enable(int on)
{
    veda::profile::enable(on != 0);
    return VEDA_OK;
}

int veda_profile_collect(char (*names)[32], double* ms, double* flops, double* bytes,
                         uint64_t* launches, int cap)
{
    int count = 0;
    const int rc = guarded([&] {
        const auto totals = veda::profile::collect(true);
        for (const auto& [name, t] : totals)
        {
            if (count < cap)
            {
                std::strncpy(names[count], name.c_str(), 31);
                names[count][31] = '\0';
                ms[count] = t.ms;
                flops[count] = t.flops;
                bytes[count] = t.bytes;
                launches[count] = t.launches;
            }
            ++count;
        }
    });
    return rc == VEDA_OK ? count : rc;
}

} // extern "C"
