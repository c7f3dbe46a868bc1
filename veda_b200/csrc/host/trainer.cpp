// The training step driver and the data-parallel gradient exchange.
//
// One step is the loop of the reference's tests (tests/TinyModelTest.cpp:290-299):
// zero_grad, forward, cross_entropy, backward, clip_gradient_norm, AdamW::step — here with the
// clip fused into the update, and, across GPUs, the flat fp32 gradient arena all-reduced by NCCL
// in buckets. A bucket is launched on a dedicated communication stream the moment the backward
// has produced the last gradient that falls into it (the tape reports each leaf as it becomes
// final), so the exchange of layer L's gradients overlaps the backward of layers L-1..0. The
// update waits for the last bucket; the 1/world average is folded into the AdamW kernel.
#include "veda/profile.hpp"
#include "veda/train.hpp"

#include "veda_cuda.h"

#include <cuda_runtime.h>
#include <nccl.h>

#include <cstdlib>
#include <cstring>
#include <stdexcept>
#include <unordered_map>

namespace veda::train
{

using autograd::Variable;
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

void nccl_check(ncclResult_t r, const char* what)
{
    if (r != ncclSuccess)
    {
        throw std::runtime_error(std::string(what) + ": " + ncclGetErrorString(r));
    }
}
} // namespace

class DataParallel
{
public:
    DataParallel(const void* unique_id, int rank, int world) : rank_(rank), world_(world)
    {
        ncclUniqueId id;
        std::memcpy(&id, unique_id, sizeof(id));
        nccl_check(ncclCommInitRank(&comm_, world, id, rank), "ncclCommInitRank");
        // Highest priority: the compute kernels hold every SM (one large block per SM), so the
        // all-reduce blocks must win each SM slot that frees up to overlap with the backward.
        int least = 0, greatest = 0;
        cuda_check(cudaDeviceGetStreamPriorityRange(&least, &greatest), "stream priorities");
        cuda_check(cudaStreamCreateWithPriority(&stream_, cudaStreamNonBlocking, greatest),
                   "comm stream");
        cuda_check(cudaEventCreateWithFlags(&done_, cudaEventDisableTiming), "comm event");
    }

    ~DataParallel()
    {
        for (Bucket& b : buckets_)
        {
            cudaEventDestroy(b.ready);
        }
        cudaEventDestroy(done_);
        if (comm_ != nullptr)
        {
            ncclCommDestroy(comm_);
        }
        cudaStreamDestroy(stream_);
    }

    // Buckets of `bucket_bytes` cut from the end of the arena (the backward produces the last
    // parameters first), each waiting for every graph leaf that overlaps it.
    void attach(TinyTransformer& model, size_t bucket_bytes)
    {
        arena_ = static_cast<float*>(model.grad_arena().data_ptr());
        const size_t total = model.parameter_count();
        const size_t per = std::max<size_t>(1, bucket_bytes / sizeof(float));
        for (size_t end = total; end > 0;)
        {
            const size_t begin = end > per ? end - per : 0;
            Bucket b{begin, end, 0, 0, false, nullptr};
            cuda_check(cudaEventCreateWithFlags(&b.ready, cudaEventDisableTiming), "bucket event");
            buckets_.push_back(b);
            end = begin;
        }
        for (const auto& leaf : model.graph_leaves())
        {
            const size_t lo = leaf.offset, hi = leaf.offset + leaf.count;
            std::vector<size_t>& list = leaf_buckets_[leaf.var.node().get()];
            for (size_t i = 0; i < buckets_.size(); ++i)
            {
                if (buckets_[i].begin < hi && lo < buckets_[i].end)
                {
                    list.push_back(i);
                    buckets_[i].waiting += 1;
                }
            }
        }
    }

    // From the start of the backward until every bucket is queued, the persistent kernels leave
    // reserved_sms_ SMs free so the all-reduce blocks run beside them instead of only in the gaps
    // between kernels (each compute block holds a whole SM).
    void begin_step()
    {
        for (Bucket& b : buckets_)
        {
            b.pending = b.waiting;
            b.launched = false;
        }
        veda_set_reserved_sms(reserved_sms_);
    }

    void leaf_ready(autograd::Node* node)
    {
        auto it = leaf_buckets_.find(node);
        if (it == leaf_buckets_.end())
        {
            return;
        }
        for (size_t i : it->second)
        {
            if (--buckets_[i].pending == 0)
            {
                launch(i);
            }
        }
    }

    void finish()
    {
        for (size_t i = 0; i < buckets_.size(); ++i)
        {
            if (!buckets_[i].launched)
            {
                launch(i);
            }
        }
        cuda_check(cudaEventRecord(done_, stream_), "comm done");
        cuda_check(cudaStreamWaitEvent(cs(), done_, 0), "comm wait");
        veda_set_reserved_sms(0);
    }

    int world() const noexcept { return world_; }

private:
    struct Bucket
    {
        size_t begin, end;
        int waiting, pending;
        bool launched;
        cudaEvent_t ready;
    };

    void launch(size_t i)
    {
        Bucket& b = buckets_[i];
        b.launched = true;
        cuda_check(cudaEventRecord(b.ready, cs()), "bucket ready");
        cuda_check(cudaStreamWaitEvent(stream_, b.ready, 0), "bucket wait");
        nccl_check(ncclAllReduce(arena_ + b.begin, arena_ + b.begin, b.end - b.begin, ncclFloat,
                                 ncclSum, comm_, stream_),
                   "ncclAllReduce");
    }

    // SMs left to NCCL during the backward (VEDA_DP_RESERVED_SMS, default 16)
    int reserved_sms_ = [] {
        const char* v = std::getenv("VEDA_DP_RESERVED_SMS");
        return v != nullptr ? std::atoi(v) : 16;
    }();
    ncclComm_t comm_ = nullptr;
    cudaStream_t stream_ = nullptr;
    cudaEvent_t done_ = nullptr;
    int rank_ = 0, world_ = 1;
    float* arena_ = nullptr;
    std::vector<Bucket> buckets_;
    std::unordered_map<autograd::Node*, std::vector<size_t>> leaf_buckets_;
};

Trainer::Trainer(ModelConfig config, optim::AdamWConfig adam, float max_norm, DType dtype,
                 size_t batch, size_t length, uint64_t seed)
    : max_norm_(max_norm), batch_(batch), length_(length)
{
    if (!(max_norm > 0.0f))
    {
        throw std::invalid_argument("Trainer: max_norm must be positive");
    }
    if (batch == 0 || length == 0)
    {
        throw std::invalid_argument("Trainer: empty batch");
    }
    model_ = std::make_unique<TinyTransformer>(std::move(config), seed, dtype);
    opt_ = std::make_unique<optim::AdamW>(model_->parameters(), adam);
    const size_t n = batch * length;
    ids_ = Tensor::empty(Shape({2 * n}), DType::F32);       // int64 payloads
    targets_ = Tensor::empty(Shape({2 * n}), DType::F32);
    loss_ = Tensor(Shape({1}), DType::F32);
}

Trainer::~Trainer() = default;

void Trainer::init_data_parallel(const void* nccl_unique_id, int rank, int world,
                                 size_t bucket_bytes)
{
    if (world < 1 || rank < 0 || rank >= world)
    {
        throw std::invalid_argument("Trainer: bad rank/world");
    }
    if (world == 1)
    {
        dp_.reset();
        return;
    }
    dp_ = std::make_unique<DataParallel>(nccl_unique_id, rank, world);
    dp_->attach(*model_, bucket_bytes);
}

int Trainer::world() const noexcept { return dp_ ? dp_->world() : 1; }

void Trainer::step(const Tensor& ids, const Tensor& targets)
{
    profile::HostScope whole("host:step");
    {
        // the backward overwrites each gradient on its first write, so no arena-wide memset
        profile::HostScope scope("host:zero_grad");
        model_->mark_grads_zero();
    }
    Variable logits = [&] {
        profile::HostScope scope("host:forward");
        return model_->forward_device(ids, batch_, length_);
    }();
    Variable loss = autograd::cross_entropy_device(logits, targets);
    autograd::BackwardOptions options;
    options.retain_intermediate_grads = false;
    if (dp_)
    {
        dp_->begin_step();
        options.on_leaf_ready = [this](autograd::Node* node) { dp_->leaf_ready(node); };
    }
    {
        profile::HostScope scope("host:backward");
        loss.backward(options);
    }
    model_->clear_untouched_grads();
    if (dp_)
    {
        dp_->finish();
    }
    {
        const double n = static_cast<double>(model_->parameter_count());
        profile::Scope scope("adamw", 0.0,
                             n * (4.0 + 16.0 + 12.0 + (model_->dtype() == DType::BF16 ? 2.0 : 0.0)));
        opt_->step_clipped(max_norm_, 1.0f / static_cast<float>(world()));
    }
    cuda_check(cudaMemcpyAsync(loss_.data_ptr(), loss.value().data_ptr(), sizeof(float),
                               cudaMemcpyDeviceToDevice, cs()),
               "loss copy");
}

StepStats Trainer::step_host(const int64_t* ids, const int64_t* targets)
{
    const size_t n = batch_ * length_;
    cuda_check(cudaMemcpyAsync(ids_.data_ptr(), ids, n * sizeof(int64_t), cudaMemcpyHostToDevice,
                               cs()),
               "ids upload");
    cuda_check(cudaMemcpyAsync(targets_.data_ptr(), targets, n * sizeof(int64_t),
                               cudaMemcpyHostToDevice, cs()),
               "targets upload");
    step(ids_, targets_);
    return last_stats();
}

StepStats Trainer::last_stats()
{
    StepStats s;
    cuda_check(cudaMemcpyAsync(&s.loss, loss_.data_ptr(), sizeof(float), cudaMemcpyDeviceToHost,
                               cs()),
               "loss read");
    s.grad_norm = opt_->last_grad_norm();   // synchronises
    autograd::detail::raise_device_flag();
    return s;
}

} // namespace veda::train
