// The training step driver and the data-parallel gradient exchange.
//
// One step is the loop of the reference's tests (tests/TinyModelTest.cpp:290-299):
// zero_grad, forward, cross_entropy, backward, clip_gradient_norm, AdamW::step — here with the
// clip fused into the update, and, across GPUs, the flat fp32 gradient arena all-reduced by NCCL
// in buckets. A bucket is launched on a dedicated communication stream the moment the backward
// has produced the last gradient that falls into it (the tape reports each leaf as it becomes
// final), so the exchange of layer L's gradients overlaps the backward of layers L-1..0. The
// update waits for the last bucket; the 1/world average is folded into the AdamW kernel.
#include "veda/checkpoint.hpp"
#include "veda/profile.hpp"
#include "veda/train.hpp"

#include "veda_cuda.h"

#include <cuda_runtime.h>
#include <nccl.h>

#include "watchdog.hpp"

#include <cmath>
#include <cstdlib>
#include <cstring>
#include <filesystem>
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

} // namespace

class DataParallel
{
public:
    // The communicator comes from ncclCommInitRankConfig: VEDA_NCCL_NONBLOCKING=1 makes it
    // non-blocking (every call is then settled by polling ncclCommGetAsyncError, bounded by the
    // communication timeout); VEDA_NCCL_MAX_CTAS / VEDA_NCCL_MIN_CTAS bound the blocks NCCL's
    // kernels take (the SMs they share with the backward's kernels).
    DataParallel(const void* unique_id, int rank, int world, bool sharded)
        : rank_(rank), world_(world), sharded_(sharded)
    {
        ncclUniqueId id;
        std::memcpy(&id, unique_id, sizeof(id));
        ncclConfig_t config = NCCL_CONFIG_INITIALIZER;
        if (const char* v = std::getenv("VEDA_NCCL_NONBLOCKING"); v != nullptr && std::atoi(v) != 0)
        {
            config.blocking = 0;
        }
        if (const char* v = std::getenv("VEDA_NCCL_MAX_CTAS"); v != nullptr && std::atoi(v) > 0)
        {
            config.maxCTAs = std::atoi(v);
        }
        if (const char* v = std::getenv("VEDA_NCCL_MIN_CTAS"); v != nullptr && std::atoi(v) > 0)
        {
            config.minCTAs = std::atoi(v);
        }
        if (const char* v = std::getenv("VEDA_DP_TIMEOUT_S"); v != nullptr && std::atof(v) > 0.0)
        {
            timeout_s_ = std::atof(v);
        }
        settle(ncclCommInitRankConfig(&comm_, world, id, rank, &config), "ncclCommInitRankConfig");
        // Highest priority: the compute kernels hold every SM (one large block per SM), so the
        // all-reduce blocks must win each SM slot that frees up to overlap with the backward.
        int least = 0, greatest = 0;
        cuda_check(cudaDeviceGetStreamPriorityRange(&least, &greatest), "stream priorities");
        cuda_check(cudaStreamCreateWithPriority(&stream_, cudaStreamNonBlocking, greatest),
                   "comm stream");
        cuda_check(cudaEventCreateWithFlags(&done_, cudaEventDisableTiming), "comm event");
        cuda_check(cudaEventCreateWithFlags(&main_ready_, cudaEventDisableTiming), "comm event");
    }

    ~DataParallel()
    {
        if (!aborted_)
        {
            cudaStreamSynchronize(stream_);
        }
        for (Bucket& b : buckets_)
        {
            cudaEventDestroy(b.ready);
            cudaEventDestroy(b.gathered);
        }
        cudaEventDestroy(done_);
        cudaEventDestroy(main_ready_);
        if (comm_ != nullptr)
        {
            ncclCommDestroy(comm_);
        }
        cudaStreamDestroy(stream_);
    }

    // Host wait for the work queued on `s` (which waits for the communication it depends on):
    // polls instead of blocking, so a collective stuck on a failed peer ends in an exception
    // (after ncclCommAbort) instead of a hang.
    void wait(cudaStream_t s)
    {
        ensure_alive();
        const detail::WaitOutcome o = detail::watch(
            [&] {
                const cudaError_t e = cudaStreamQuery(s);
                return e == cudaSuccess ? 0 : (e == cudaErrorNotReady ? 1 : -1);
            },
            [&] {
                ncclResult_t a = ncclSuccess;
                if (ncclCommGetAsyncError(comm_, &a) != ncclSuccess)
                {
                    return -1;
                }
                return a == ncclSuccess ? 0 : (a == ncclInProgress ? 1 : -1);
            },
            [&] { abort(); }, detail::monotonic_seconds, detail::short_pause, timeout_s_);
        if (o != detail::WaitOutcome::done)
        {
            throw std::runtime_error(std::string("data parallel (rank ") + std::to_string(rank_) +
                                     "): " + detail::describe(o));
        }
    }

    // Tears the communicator down without waiting for its peers (ncclCommAbort): for a caller
    // that has learned on the host that a peer is gone. Every later collective call throws.
    void abort()
    {
        if (comm_ != nullptr)
        {
            ncclCommAbort(comm_);
            comm_ = nullptr;
        }
        aborted_ = true;
    }

    void set_timeout(double seconds)
    {
        if (!(seconds > 0.0))
        {
            throw std::invalid_argument("data parallel: the communication timeout must be positive");
        }
        timeout_s_ = seconds;
    }

    // Buckets of `bucket_bytes` cut from the end of the arena (the backward produces the last
    // parameters first), each waiting for every graph leaf that overlaps it. Sharded, every
    // bucket is a whole number of 16-byte rows per rank, and rank r owns the r-th of the world
    // equal parts of each bucket; its parts, in arena order, make up its shard.
    //
    // The tied embedding table is one bucket of its own when its rows split evenly across the
    // ranks (rank r then owns the table rows [r V/world, (r+1) V/world)): its gradient holds only
    // the LM head's dW until the end of the backward, so it is reduced as soon as the head's
    // backward has run, and the rows the embedding lookup scatters (at most `tokens` per rank)
    // are exchanged separately at the end and added onto the reduced table in (rank, position)
    // order (embedding_rows).
    void attach(TinyTransformer& model, size_t bucket_bytes, const float* master, size_t steps,
                size_t tokens)
    {
        arena_ = static_cast<float*>(model.grad_arena().data_ptr());
        values_ = model.value_arena().data_ptr();
        bf16_ = model.dtype() == DType::BF16;
        params_ = model.parameter_count();
        total_ = sharded_ ? model.arena_length() : params_;
        const size_t unit = sharded_ ? 8 * static_cast<size_t>(world_) : 1;
        if (total_ % unit != 0)
        {
            throw std::invalid_argument("DataParallel: the arena does not split into " +
                                        std::to_string(world_) + " shards");
        }
        const auto [e0, e1] = model.embedding_range();
        vocab_ = model.config().vocab_size;
        dim_ = model.config().hidden_size;
        tokens_ = tokens;
        const char* rows_env = std::getenv("VEDA_DP_EMBEDDING_ROWS");
        rows_exchange_ = model.config().tie_word_embeddings && tokens > 0 && tokens <= 16384 &&
                         vocab_ % static_cast<size_t>(world_) == 0 && e0 % unit == 0 &&
                         e1 % unit == 0 && e1 - e0 == vocab_ * dim_ &&
                         (rows_env == nullptr || std::atoi(rows_env) != 0);
        const size_t per = std::max<size_t>(unit, bucket_bytes / sizeof(float) / unit * unit);
        auto cut = [&](size_t lo, size_t hi) {
            for (size_t end = hi; end > lo;)
            {
                const size_t begin = end - lo > per ? end - per : lo;
                add_bucket(begin, end);
                end = begin;
            }
        };
        if (rows_exchange_)
        {
            cut(e1, total_);
            rows_bucket_ = buckets_.size();
            add_bucket(e0, e1);
            cut(0, e0);
            const size_t n = tokens * static_cast<size_t>(world_);
            keys_ = Tensor::empty(Shape({2 * tokens}), DType::F32);   // uint64 payloads
            keys_all_ = Tensor::empty(Shape({2 * n}), DType::F32);
            rows_all_ = Tensor::empty(Shape({n, dim_}), model.dtype());
        }
        else
        {
            cut(0, total_);
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
        if (!sharded_)
        {
            return;
        }
        // shard offsets in arena order (buckets_ runs from the end of the arena)
        size_t at = 0;
        for (size_t i = buckets_.size(); i-- > 0;)
        {
            buckets_[i].shard_at = at;
            at += (buckets_[i].end - buckets_[i].begin) / world_;
        }
        shard_ = total_ / world_;
        const Shape sh({shard_});
        g_s_ = Tensor(sh, DType::F32);
        master_s_ = Tensor(sh, DType::F32);
        m_s_ = Tensor(sh, DType::F32);
        v_s_ = Tensor(sh, DType::F32);
        if (bf16_)
        {
            lowp_s_ = Tensor(Shape({shard_}), DType::BF16);
        }
        sumsq_ = Tensor(Shape({2}), DType::F32);   // one double
        bias_ = Tensor(Shape({4}), DType::F32);    // two doubles
        const size_t ws = veda_sumsq_workspace(static_cast<int64_t>(shard_));
        ws_ = Tensor::empty(Shape({(ws + 3) / 4 + 1}), DType::F32);
        steps_ = steps;
        load_master(master);
    }

    void load_master(const float* master) { load_shard(master, master_s_); }

    // This rank's parts of an arena-ordered fp32 vector (`params_` elements; the padding past
    // them stays zero) into one of its shards.
    void load_shard(const float* full, Tensor& shard)
    {
        const float* master = full;
        float* dst = static_cast<float*>(shard.data_ptr());
        for (const Bucket& b : buckets_)
        {
            const size_t len = (b.end - b.begin) / world_;
            const size_t lo = b.begin + static_cast<size_t>(rank_) * len;
            const size_t hi = std::min(lo + len, params_);
            if (hi > lo)
            {
                cuda_check(cudaMemcpyAsync(dst + b.shard_at, master + lo, (hi - lo) * sizeof(float),
                                           cudaMemcpyDeviceToDevice, cs()),
                           "shard master");
            }
        }
    }

    // From the start of the backward until every bucket is queued, the persistent kernels leave
    // reserved_sms_ SMs free so the all-reduce blocks run beside them instead of only in the gaps
    // between kernels (each compute block holds a whole SM).
    void begin_step()
    {
        ensure_alive();
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
        join_comm();
        rows_held_ = Tensor();   // the exchange has read them (ordered before later work)
        veda_set_reserved_sms(0);
    }

    bool rows_exchange() const noexcept { return rows_exchange_; }

    // The embedding lookup's backward (autograd::embedding_device_rows): this rank's (id,
    // position) keys sorted, every rank's keys and gradient rows all-gathered on the
    // communication stream after the table's own reduction, then each rank's rows added onto
    // this rank's reduced table rows (sharded: its own row range; replicated: the whole table),
    // rank after rank, each in its key order: deterministic, and the same sum on every rank.
    void embedding_rows(const Tensor& ids, size_t count, const Tensor& rows)
    {
        if (count != tokens_ || rows.numel() != count * dim_ || rows.dtype() != rows_all_.dtype())
        {
            throw std::logic_error("data parallel: the embedding rows do not match the batch");
        }
        const int d = static_cast<int>(rows.dtype());
        uint64_t* keys = static_cast<uint64_t*>(keys_.data_ptr());
        check(veda_embedding_sort(static_cast<const int64_t*>(ids.data_ptr()),
                                  static_cast<int64_t>(count), static_cast<int64_t>(vocab_), keys,
                                  current_stream()),
              "embedding rows: sort");
        Bucket& table = buckets_[rows_bucket_];
        if (!table.launched)
        {
            launch(rows_bucket_);
        }
        rows_held_ = rows;
        fork_comm();
        uint64_t* keys_all = static_cast<uint64_t*>(keys_all_.data_ptr());
        settle(ncclGroupStart(), "embedding rows all-gather");
        settle(ncclAllGather(keys, keys_all, count, ncclUint64, comm_, stream_),
               "embedding rows all-gather");
        settle(ncclAllGather(rows.data_ptr(), rows_all_.data_ptr(), count * dim_,
                             rows.dtype() == DType::BF16 ? ncclBfloat16 : ncclFloat, comm_, stream_),
               "embedding rows all-gather");
        settle(ncclGroupEnd(), "embedding rows all-gather");
        const size_t per_rank = vocab_ / static_cast<size_t>(world_);
        float* target = sharded_ ? static_cast<float*>(g_s_.data_ptr()) + table.shard_at
                                 : arena_ + table.begin;
        const size_t lo = sharded_ ? static_cast<size_t>(rank_) * per_rank : 0;
        const size_t hi = sharded_ ? lo + per_rank : vocab_;
        const size_t es = core::dtype_size(rows.dtype());
        for (int r = 0; r < world_; ++r)
        {
            check(veda_embedding_apply_sorted(
                      keys_all + static_cast<size_t>(r) * count, static_cast<int64_t>(count),
                      static_cast<const char*>(rows_all_.data_ptr()) + static_cast<size_t>(r) * count * dim_ * es,
                      static_cast<int64_t>(dim_), static_cast<int64_t>(dim_),
                      static_cast<int64_t>(lo), static_cast<int64_t>(hi), target, d, stream_),
                  "embedding rows: apply");
        }
    }

    // Sharded step: global norm of the averaged gradient (a sum over the shards), clip + AdamW on
    // this rank's shard (optim::AdamW's arithmetic, AdamW.cpp:38-93), then the updated weights
    // of every bucket all-gathered into the value arena.
    // Counts the step and leaves its bias corrections in device memory (outside any captured
    // graph: the update's kernel reads them when it runs).
    void advance(const optim::AdamWConfig& c)
    {
        ++steps_;
        bias_host_[0] = 1.0 - std::pow(static_cast<double>(c.beta1), static_cast<double>(steps_));
        bias_host_[1] = 1.0 - std::pow(static_cast<double>(c.beta2), static_cast<double>(steps_));
        cuda_check(cudaMemcpyAsync(bias_.data_ptr(), bias_host_, sizeof(bias_host_), cudaMemcpyHostToDevice, cs()),
                   "sharded bias corrections");
    }

    void update(const optim::AdamWConfig& c, float max_norm)
    {
        double* ss = static_cast<double*>(sumsq_.data_ptr());
        float* g = static_cast<float*>(g_s_.data_ptr());
        float* master = static_cast<float*>(master_s_.data_ptr());
        check(veda_sumsq(g, static_cast<int64_t>(shard_), ss, 0, ws_.data_ptr(), ws_.numel() * 4,
                         current_stream()),
              "sharded clip (norm)");
        fork_comm();
        settle(ncclAllReduce(ss, ss, 1, ncclFloat64, ncclSum, comm_, stream_), "norm all-reduce");
        join_comm();
        check(veda_adamw_step_dev(master, static_cast<float*>(m_s_.data_ptr()),
                                  static_cast<float*>(v_s_.data_ptr()), g,
                                  bf16_ ? lowp_s_.data_ptr() : nullptr, static_cast<int64_t>(shard_),
                                  c.learning_rate, c.beta1, c.beta2, c.eps, c.weight_decay,
                                  static_cast<const double*>(bias_.data_ptr()), ss, max_norm,
                                  1.0f / static_cast<float>(world_),
                                  skip_nonfinite_ ? VEDA_ADAMW_SKIP_NONFINITE : 0, current_stream()),
              "sharded AdamW");
        // the weights are gathered in arena order (the order the next forward reads them) and
        // not waited for here: the next forward waits for each bucket where it first needs it
        fork_comm();
        for (size_t i = buckets_.size(); i-- > 0;)
        {
            Bucket& b = buckets_[i];
            const size_t len = (b.end - b.begin) / world_;
            if (bf16_)
            {
                settle(ncclAllGather(static_cast<const uint16_t*>(lowp_s_.data_ptr()) + b.shard_at,
                                         static_cast<uint16_t*>(values_) + b.begin, len, ncclBfloat16,
                                         comm_, stream_),
                           "weight all-gather");
            }
            else
            {
                settle(ncclAllGather(master + b.shard_at, static_cast<float*>(values_) + b.begin, len,
                                         ncclFloat, comm_, stream_),
                           "weight all-gather");
            }
            cuda_check(cudaEventRecord(b.gathered, stream_), "bucket gathered");
            b.gate_open = false;
        }
        gathering_ = true;
        if (!overlap_gather_)
        {
            sync();
        }
    }

    // The current stream waits for the gathered weights of every bucket overlapping [lo, hi).
    // While the gather runs, kernels launched by the forward leave reserved_sms_ SMs to it; the
    // host launches about as far ahead as the device runs, so the reservation ends at the first
    // gate after the last bucket has arrived.
    void gate(size_t lo, size_t hi)
    {
        if (!gathering_)
        {
            return;
        }
        for (Bucket& b : buckets_)
        {
            if (!b.gate_open && b.begin < hi && lo < b.end)
            {
                cuda_check(cudaStreamWaitEvent(cs(), b.gathered, 0), "weight gate");
                b.gate_open = true;
            }
        }
        if (reserving_ && cudaEventQuery(buckets_.front().gathered) == cudaSuccess)
        {
            veda_set_reserved_sms(0);
            reserving_ = false;
        }
    }

    void begin_forward()
    {
        ensure_alive();
        if (gathering_ && forward_reserved_sms_ > 0)
        {
            veda_set_reserved_sms(forward_reserved_sms_);
            reserving_ = true;
        }
    }

    void end_forward()
    {
        if (gathering_)
        {
            sync();   // the forward has waited for every bucket but a padding-only one
        }
        if (reserving_)
        {
            veda_set_reserved_sms(0);
            reserving_ = false;
        }
    }

    // The current stream waits for everything queued on the communication stream.
    void sync()
    {
        join_comm();
        gathering_ = false;
        for (Bucket& b : buckets_)
        {
            b.gate_open = true;
        }
    }



    // Pre-clip norm of the averaged gradient of the last sharded step (synchronises).
    float grad_norm()
    {
        double ss = 0.0;
        cuda_check(cudaMemcpyAsync(&ss, sumsq_.data_ptr(), sizeof(double), cudaMemcpyDeviceToHost, cs()),
                   "norm read");
        cuda_check(cudaStreamSynchronize(cs()), "norm read");
        return static_cast<float>(std::sqrt(ss) / static_cast<double>(world_));
    }

    // Collective: every rank's reduced gradient parts into every rank's gradient arena (which
    // then holds the summed gradient, as after an all-reduce).
    void gather_gradients()
    {
        sync();
        fork_comm();
        settle(ncclGroupStart(), "gradient all-gather");
        for (const Bucket& b : buckets_)
        {
            settle(ncclAllGather(static_cast<const float*>(g_s_.data_ptr()) + b.shard_at, arena_ + b.begin,
                                     (b.end - b.begin) / world_, ncclFloat, comm_, stream_),
                       "gradient all-gather");
        }
        settle(ncclGroupEnd(), "gradient all-gather");
        join_comm();
    }

    // Collective: the full master weights, in arena order, into `master` (params_ elements).
    void gather_master(float* master) { gather_shard(master_s_, master); }

    // Collective: every rank's parts of a shard, in arena order, into `full` (params_ elements).
    void gather_shard(const Tensor& shard, float* full)
    {
        sync();
        Tensor whole = Tensor::empty(Shape({total_}), DType::F32);
        float* f = static_cast<float*>(whole.data_ptr());
        fork_comm();
        settle(ncclGroupStart(), "shard all-gather");
        for (const Bucket& b : buckets_)
        {
            settle(ncclAllGather(static_cast<const float*>(shard.data_ptr()) + b.shard_at, f + b.begin,
                                     (b.end - b.begin) / world_, ncclFloat, comm_, stream_),
                       "shard all-gather");
        }
        settle(ncclGroupEnd(), "shard all-gather");
        join_comm();
        cuda_check(cudaMemcpyAsync(full, f, params_ * sizeof(float), cudaMemcpyDeviceToDevice, cs()),
                   "shard copy");
        cuda_check(cudaStreamSynchronize(cs()), "shard copy");
    }

    // Moments and step count for a checkpoint (sharded; collective) and back.
    void gather_moments(float* m, float* v)
    {
        gather_shard(m_s_, m);
        gather_shard(v_s_, v);
    }
    void load_moments(const float* m, const float* v, size_t steps)
    {
        load_shard(m, m_s_);
        load_shard(v, v_s_);
        steps_ = steps;
    }
    size_t steps() const noexcept { return steps_; }
    // a skipped step (non-finite norm) is not counted: the next uses the same bias corrections
    void rewind_step() noexcept
    {
        if (steps_ > 0) --steps_;
    }
    void set_skip_nonfinite(bool on) noexcept { skip_nonfinite_ = on; }
    int rank() const noexcept { return rank_; }

    int world() const noexcept { return world_; }
    bool sharded() const noexcept { return sharded_; }
    // A step replayed from a CUDA graph ends with its weight gather (the next graph cannot wait
    // on a bucket event recorded by the previous one).
    void set_overlap_gather(bool on) noexcept { overlap_gather_ = on; }

private:
    struct Bucket
    {
        size_t begin, end;
        size_t shard_at;   // sharded: where this rank's part sits in its shard
        int waiting, pending;
        bool launched;
        bool gate_open;    // sharded: the current stream already waits for its gathered weights
        cudaEvent_t ready, gathered;
    };

    void add_bucket(size_t begin, size_t end)
    {
        Bucket b{begin, end, 0, 0, 0, false, true, nullptr, nullptr};
        cuda_check(cudaEventCreateWithFlags(&b.ready, cudaEventDisableTiming), "bucket event");
        cuda_check(cudaEventCreateWithFlags(&b.gathered, cudaEventDisableTiming), "bucket event");
        buckets_.push_back(b);
    }

    void launch(size_t i)
    {
        Bucket& b = buckets_[i];
        b.launched = true;
        cuda_check(cudaEventRecord(b.ready, cs()), "bucket ready");
        cuda_check(cudaStreamWaitEvent(stream_, b.ready, 0), "bucket wait");
        if (sharded_)
        {
            settle(ncclReduceScatter(arena_ + b.begin, static_cast<float*>(g_s_.data_ptr()) + b.shard_at,
                                         (b.end - b.begin) / world_, ncclFloat, ncclSum, comm_, stream_),
                       "ncclReduceScatter");
        }
        else
        {
            settle(ncclAllReduce(arena_ + b.begin, arena_ + b.begin, b.end - b.begin, ncclFloat,
                                     ncclSum, comm_, stream_),
                       "ncclAllReduce");
        }
    }

    void ensure_alive() const
    {
        if (aborted_)
        {
            throw std::runtime_error("data parallel: the communicator was aborted");
        }
    }

    // An NCCL call's result: on a non-blocking communicator ncclInProgress means the call is
    // still being queued, so poll until it has been (bounded by the communication timeout). Any
    // error aborts the communicator and throws.
    void settle(ncclResult_t r, const char* what)
    {
        ensure_alive();
        if (r == ncclInProgress && comm_ != nullptr)
        {
            const double start = detail::monotonic_seconds();
            while (r == ncclInProgress)
            {
                if (ncclCommGetAsyncError(comm_, &r) != ncclSuccess)
                {
                    r = ncclInternalError;
                    break;
                }
                if (r == ncclInProgress && detail::monotonic_seconds() - start > timeout_s_)
                {
                    abort();
                    throw std::runtime_error(std::string(what) + ": not queued within the "
                                             "communication timeout; the communicator was aborted");
                }
                if (r == ncclInProgress)
                {
                    detail::short_pause();
                }
            }
        }
        if (r != ncclSuccess)
        {
            abort();
            throw std::runtime_error(std::string(what) + ": " + ncclGetErrorString(r) +
                                     "; the communicator was aborted");
        }
    }

    // the communication stream waits for the work queued so far on the current stream
    void fork_comm()
    {
        cuda_check(cudaEventRecord(main_ready_, cs()), "comm fork");
        cuda_check(cudaStreamWaitEvent(stream_, main_ready_, 0), "comm fork");
    }

    // the current stream waits for the communication queued so far
    void join_comm()
    {
        cuda_check(cudaEventRecord(done_, stream_), "comm done");
        cuda_check(cudaStreamWaitEvent(cs(), done_, 0), "comm wait");
    }

    // SMs left to NCCL during the backward (VEDA_DP_RESERVED_SMS, default 16) and during a
    // forward that overlaps the weight all-gather (VEDA_DP_FORWARD_RESERVED_SMS, default 0)
    int reserved_sms_ = [] {
        const char* v = std::getenv("VEDA_DP_RESERVED_SMS");
        return v != nullptr ? std::atoi(v) : 16;
    }();
    // the weight all-gather runs into the next forward (VEDA_DP_GATHER_OVERLAP, default 1) or
    // is waited for at the end of the step
    bool overlap_gather_ = [] {
        const char* v = std::getenv("VEDA_DP_GATHER_OVERLAP");
        return v == nullptr || std::atoi(v) != 0;
    }();
    int forward_reserved_sms_ = [] {
        const char* v = std::getenv("VEDA_DP_FORWARD_RESERVED_SMS");
        return v != nullptr ? std::atoi(v) : 0;
    }();
    ncclComm_t comm_ = nullptr;
    bool aborted_ = false;
    bool skip_nonfinite_ = false;
    double timeout_s_ = 600.0;   // VEDA_DP_TIMEOUT_S or set_timeout
    cudaStream_t stream_ = nullptr;
    cudaEvent_t done_ = nullptr, main_ready_ = nullptr;
    int rank_ = 0, world_ = 1;
    bool sharded_ = false, bf16_ = false, gathering_ = false, reserving_ = false;
    float* arena_ = nullptr;
    void* values_ = nullptr;
    size_t params_ = 0, total_ = 0, shard_ = 0, steps_ = 0;
    std::vector<Bucket> buckets_;
    std::unordered_map<autograd::Node*, std::vector<size_t>> leaf_buckets_;
    // the embedding rows exchange (attach)
    bool rows_exchange_ = false;
    size_t rows_bucket_ = 0, vocab_ = 0, dim_ = 0, tokens_ = 0;
    Tensor keys_, keys_all_, rows_all_, rows_held_;
    Tensor g_s_, master_s_, m_s_, v_s_, lowp_s_, sumsq_, ws_, bias_;
    double bias_host_[2] = {1.0, 1.0};
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

Trainer::~Trainer()
{
    model_->set_embedding_rows_sink({});   // it points into dp_
    if (graph_exec_ != nullptr)
    {
        cudaGraphExecDestroy(graph_exec_);
    }
    if (capture_stream_ != nullptr)
    {
        cudaStreamDestroy(static_cast<cudaStream_t>(capture_stream_));
    }
}

void Trainer::init_data_parallel(const void* nccl_unique_id, int rank, int world,
                                 size_t bucket_bytes, bool sharded)
{
    if (world < 1 || rank < 0 || rank >= world)
    {
        throw std::invalid_argument("Trainer: bad rank/world");
    }
    if (world == 1)
    {
        model_->set_embedding_rows_sink({});
        model_->set_weight_gate({});
        dp_.reset();
        return;
    }
    dp_ = std::make_unique<DataParallel>(nccl_unique_id, rank, world, sharded);
    dp_->attach(*model_, bucket_bytes, master_weights(), opt_->steps(), batch_ * length_);
    dp_->set_skip_nonfinite(skip_nonfinite_);
    if (dp_->rows_exchange())
    {
        DataParallel* dp = dp_.get();
        model_->set_embedding_rows_sink([dp](const Tensor& ids, size_t count, const Tensor& rows) {
            dp->embedding_rows(ids, count, rows);
        });
    }
    else
    {
        model_->set_embedding_rows_sink({});
    }
    if (sharded)
    {
        DataParallel* dp = dp_.get();
        model_->set_weight_gate([dp](size_t lo, size_t hi) { dp->gate(lo, hi); });
    }
    else
    {
        model_->set_weight_gate({});
    }
}

void Trainer::sync()
{
    if (dp_)
    {
        dp_->sync();
        dp_->wait(cs());
    }
}

void Trainer::set_comm_timeout(double seconds)
{
    if (!dp_)
    {
        throw std::logic_error("set_comm_timeout: not data parallel");
    }
    dp_->set_timeout(seconds);
}

void Trainer::abort_communication()
{
    if (dp_)
    {
        dp_->abort();
    }
}

void Trainer::set_skip_nonfinite(bool on)
{
    skip_nonfinite_ = on;
    opt_->set_skip_nonfinite(on);
    if (dp_)
    {
        dp_->set_skip_nonfinite(on);
    }
}

void Trainer::set_recompute_attention(bool on)
{
    if (on == model_->recompute_attention())
    {
        return;
    }
    model_->set_recompute_attention(on);
    if (graph_exec_ != nullptr)
    {
        cuda_check(cudaStreamSynchronize(cs()), "recompute switch");
        cudaGraphExecDestroy(graph_exec_);
        graph_exec_ = nullptr;
    }
    eager_steps_ = 0;   // the next step runs eagerly before a capture of the new path
}

int Trainer::world() const noexcept { return dp_ ? dp_->world() : 1; }

bool Trainer::sharded() const noexcept { return dp_ && dp_->sharded(); }

float* Trainer::master_weights() noexcept
{
    return static_cast<float*>(model_->dtype() == DType::F32 ? model_->value_arena().data_ptr()
                                                             : opt_->master(0).data_ptr());
}

void Trainer::gather_master_weights()
{
    if (sharded() && model_->dtype() != DType::F32)
    {
        dp_->gather_master(master_weights());
    }
}

void Trainer::gather_gradients()
{
    if (sharded())
    {
        dp_->gather_gradients();
    }
}

void Trainer::master_weights_changed()
{
    if (sharded())
    {
        dp_->sync();
        dp_->load_master(master_weights());
    }
}

// One process on one GPU, no profiling: the step is captured once into a CUDA graph (after one
// eager step has created every persistent buffer) and replayed, so the ~850 launches of a step
// cost one graph launch on the host and the device runs them back to back. The graph reads its
// inputs from ids_ / targets_ and the optimizer's bias corrections from device memory, which are
// the only things that change between steps. VEDA_STEP_GRAPH=0 keeps every step eager.
bool Trainer::graph_eligible() const
{
    static const bool enabled = [] {
        const char* v = std::getenv("VEDA_STEP_GRAPH");
        return v == nullptr || std::atoi(v) != 0;
    }();
    // data-parallel steps too when VEDA_DP_GRAPH=1 (every rank captures the same step, NCCL
    // calls included)
    static const bool dp_graph = [] {
        const char* v = std::getenv("VEDA_DP_GRAPH");
        return v != nullptr && std::atoi(v) != 0;
    }();
    return enabled && use_graph_ && (!dp_ || dp_graph) && !profile::enabled();
}

void Trainer::set_step_graph(bool on)
{
    use_graph_ = on;
}

void Trainer::step(const Tensor& ids, const Tensor& targets)
{
    if (!graph_eligible())
    {
        if (sharded())
        {
            dp_->advance(opt_->config());
        }
        else
        {
            opt_->advance();
        }
        step_impl(ids, targets);
        return;
    }
    if (dp_)
    {
        dp_->set_overlap_gather(false);
        dp_->sync();
    }
    const size_t bytes = batch_ * length_ * sizeof(int64_t);
    if (ids.data_ptr() != ids_.data_ptr())
    {
        cuda_check(cudaMemcpyAsync(ids_.data_ptr(), ids.data_ptr(), bytes, cudaMemcpyDeviceToDevice, cs()),
                   "ids copy");
        cuda_check(cudaMemcpyAsync(targets_.data_ptr(), targets.data_ptr(), bytes,
                                   cudaMemcpyDeviceToDevice, cs()),
                   "targets copy");
    }
    if (sharded())
    {
        dp_->advance(opt_->config());
    }
    else
    {
        opt_->advance();
    }
    if (graph_exec_ == nullptr && eager_steps_ < 1)
    {
        step_impl(ids_, targets_);   // creates the persistent buffers outside any graph
        ++eager_steps_;
        return;
    }
    if (graph_exec_ == nullptr)
    {
        // recorded on a private stream (the caller's may be the legacy default stream, which
        // cannot be captured); nothing runs during the capture, the graph is launched below
        if (capture_stream_ == nullptr)
        {
            cudaStream_t st = nullptr;
            cuda_check(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking), "capture stream");
            capture_stream_ = st;
        }
        const veda_stream_t caller = current_stream();
        cudaStream_t cap = static_cast<cudaStream_t>(capture_stream_);
        const uint64_t before = veda_launch_count();
        cudaGraph_t graph = nullptr;
        cuda_check(cudaStreamBeginCapture(cap, cudaStreamCaptureModeThreadLocal), "step capture");
        set_current_stream(cap);
        try
        {
            step_impl(ids_, targets_);
        }
        catch (...)
        {
            set_current_stream(caller);
            cudaStreamEndCapture(cap, &graph);
            if (graph != nullptr) cudaGraphDestroy(graph);
            use_graph_ = false;   // later steps run eagerly
            throw;
        }
        set_current_stream(caller);
        cuda_check(cudaStreamEndCapture(cap, &graph), "step capture");
        const cudaError_t e = cudaGraphInstantiateWithFlags(&graph_exec_, graph,
                                                            cudaGraphInstantiateFlagAutoFreeOnLaunch);
        cudaGraphDestroy(graph);
        cuda_check(e, "step graph instantiate");
        graph_launches_ = static_cast<int64_t>(veda_launch_count() - before);
        veda_launch_count_add(-graph_launches_);   // captured, not launched
    }
    cuda_check(cudaGraphLaunch(graph_exec_, cs()), "step graph launch");
    veda_launch_count_add(graph_launches_);
}

namespace
{
// While a step is being captured: names the phase in which an operation that cannot be
// recorded invalidated the capture.
void capture_checkpoint(const char* phase)
{
    cudaStreamCaptureStatus status = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(cs(), &status) == cudaSuccess &&
        status == cudaStreamCaptureStatusInvalidated)
    {
        throw std::runtime_error(std::string("step capture invalidated during ") + phase + ": " +
                                 cudaGetErrorString(cudaGetLastError()));
    }
}
} // namespace

void Trainer::step_impl(const Tensor& ids, const Tensor& targets)
{
    profile::HostScope whole("host:step");
    {
        // the backward overwrites each gradient on its first write, so no arena-wide memset
        profile::HostScope scope("host:zero_grad");
        model_->mark_grads_zero();
    }
    if (dp_)
    {
        dp_->begin_forward();
    }
    Variable logits = [&] {
        profile::HostScope scope("host:forward");
        return model_->forward_device(ids, batch_, length_);
    }();
    capture_checkpoint("the forward");
    if (dp_)
    {
        dp_->end_forward();
    }
    Variable loss = autograd::cross_entropy_device(logits, targets);
    capture_checkpoint("the cross-entropy");
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
    capture_checkpoint("the backward");
    model_->clear_untouched_grads();
    if (dp_)
    {
        dp_->finish();
    }
    {
        const double n = static_cast<double>(model_->parameter_count()) /
                         static_cast<double>(sharded() ? world() : 1);
        profile::Scope scope("adamw", 0.0,
                             n * (4.0 + 16.0 + 12.0 + (model_->dtype() == DType::BF16 ? 2.0 : 0.0)));
        if (sharded())
        {
            dp_->update(opt_->config(), max_norm_);
        }
        else
        {
            opt_->launch_clipped(max_norm_, 1.0f / static_cast<float>(world()));
        }
    }
    cuda_check(cudaMemcpyAsync(loss_.data_ptr(), loss.value().data_ptr(), sizeof(float),
                               cudaMemcpyDeviceToDevice, cs()),
               "loss copy");
}

namespace
{
template <typename T>
std::vector<uint8_t> to_host_bytes(const void* device, size_t count)
{
    std::vector<uint8_t> out(count * sizeof(T));
    cuda_check(cudaMemcpyAsync(out.data(), device, out.size(), cudaMemcpyDeviceToHost, cs()), "checkpoint read");
    return out;
}
} // namespace

void Trainer::save_checkpoint(const std::string& dir)
{
    sync();
    const size_t n = model_->parameter_count();
    const bool bf16 = model_->dtype() == DType::BF16;
    float* master = master_weights();
    const float* m = static_cast<const float*>(opt_->first_moments().data_ptr());
    const float* v = static_cast<const float*>(opt_->second_moments().data_ptr());
    size_t steps = opt_->steps();
    Tensor m_full, v_full;
    if (sharded())
    {
        gather_master_weights();   // collective: the shards' master weights into master_weights()
        m_full = Tensor::empty(Shape({n}), DType::F32);
        v_full = Tensor::empty(Shape({n}), DType::F32);
        dp_->gather_moments(static_cast<float*>(m_full.data_ptr()), static_cast<float*>(v_full.data_ptr()));
        m = static_cast<const float*>(m_full.data_ptr());
        v = static_cast<const float*>(v_full.data_ptr());
        steps = dp_->steps();
    }
    if (dp_ && dp_->rank() != 0)
    {
        return;   // every rank holds the same state; rank 0 writes it
    }
    std::filesystem::create_directories(dir);
    std::vector<io::SafetensorsTensor> weights, state;
    size_t at = 0;
    for (const auto& [name, value] : model_->named_parameters())
    {
        const size_t count = value.numel();
        std::vector<int64_t> shape(value.shape().dims().begin(), value.shape().dims().end());
        weights.push_back({name, bf16 ? "BF16" : "F32", shape,
                           bf16 ? to_host_bytes<uint16_t>(value.data_ptr(), count)
                                : to_host_bytes<float>(value.data_ptr(), count)});
        state.push_back({name + ".master", "F32", shape, to_host_bytes<float>(master + at, count)});
        state.push_back({name + ".exp_avg", "F32", shape, to_host_bytes<float>(m + at, count)});
        state.push_back({name + ".exp_avg_sq", "F32", shape, to_host_bytes<float>(v + at, count)});
        at += count;
    }
    cuda_check(cudaStreamSynchronize(cs()), "checkpoint read");
    if (at != n)
    {
        throw std::logic_error("save_checkpoint: parameters do not tile the arena");
    }
    io::write_safetensors(dir + "/model.safetensors", weights, {{"format", "pt"}});
    io::write_safetensors(dir + "/optimizer.safetensors", state,
                          {{"format", "pt"}, {"step", std::to_string(steps)}});
}

void Trainer::load_checkpoint(const std::string& dir)
{
    sync();
    const io::SafetensorsFile weights = io::read_safetensors(dir + "/model.safetensors");
    const bool resume = std::filesystem::exists(dir + "/optimizer.safetensors");
    io::SafetensorsFile state;
    if (resume)
    {
        state = io::read_safetensors(dir + "/optimizer.safetensors");
    }
    const size_t n = model_->parameter_count();
    std::vector<float> master(n), m(n, 0.0f), v(n, 0.0f);
    size_t at = 0;
    auto take = [&](const io::SafetensorsTensor& t, const std::vector<int64_t>& shape, size_t count, float* dst) {
        if (t.shape != shape)
        {
            throw std::invalid_argument("load_checkpoint: " + t.name + " has the wrong shape");
        }
        if (t.dtype == "F32")
        {
            std::memcpy(dst, t.bytes.data(), count * sizeof(float));
        }
        else if (t.dtype == "BF16")
        {
            for (size_t i = 0; i < count; ++i)
            {
                uint16_t h;
                std::memcpy(&h, t.bytes.data() + 2 * i, 2);
                const uint32_t w = static_cast<uint32_t>(h) << 16;
                std::memcpy(dst + i, &w, 4);
            }
        }
        else
        {
            throw std::invalid_argument("load_checkpoint: " + t.name + " is " + t.dtype);
        }
    };
    for (const auto& [name, value] : model_->named_parameters())
    {
        const size_t count = value.numel();
        const std::vector<int64_t> shape(value.shape().dims().begin(), value.shape().dims().end());
        if (resume)
        {
            take(state.at(name + ".master"), shape, count, master.data() + at);
            take(state.at(name + ".exp_avg"), shape, count, m.data() + at);
            take(state.at(name + ".exp_avg_sq"), shape, count, v.data() + at);
        }
        else
        {
            take(weights.at(name), shape, count, master.data() + at);
        }
        at += count;
    }
    size_t steps = 0;
    if (resume)
    {
        auto it = state.metadata.find("step");
        if (it == state.metadata.end())
        {
            throw std::invalid_argument("load_checkpoint: optimizer.safetensors has no step");
        }
        steps = static_cast<size_t>(std::stoull(it->second));
    }
    float* dmaster = master_weights();
    cuda_check(cudaMemcpyAsync(dmaster, master.data(), n * sizeof(float), cudaMemcpyHostToDevice, cs()),
               "checkpoint write");
    if (model_->dtype() == DType::BF16)
    {
        check(veda_f32_to_bf16(dmaster, model_->value_arena().data_ptr(), static_cast<int64_t>(n), cs()),
              "checkpoint write");
    }
    cuda_check(cudaMemcpyAsync(opt_->first_moments().data_ptr(), m.data(), n * sizeof(float),
                               cudaMemcpyHostToDevice, cs()),
               "checkpoint write");
    cuda_check(cudaMemcpyAsync(opt_->second_moments().data_ptr(), v.data(), n * sizeof(float),
                               cudaMemcpyHostToDevice, cs()),
               "checkpoint write");
    opt_->set_steps(steps);
    if (sharded())
    {
        dp_->load_master(dmaster);
        dp_->load_moments(static_cast<const float*>(opt_->first_moments().data_ptr()),
                          static_cast<const float*>(opt_->second_moments().data_ptr()), steps);
    }
    cuda_check(cudaStreamSynchronize(cs()), "checkpoint write");
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
    if (dp_)
    {
        dp_->wait(cs());   // a peer that failed mid-step ends here in an exception, not a hang
    }
    cuda_check(cudaMemcpyAsync(&s.loss, loss_.data_ptr(), sizeof(float), cudaMemcpyDeviceToHost,
                               cs()),
               "loss read");
    s.grad_norm = sharded() ? dp_->grad_norm() : opt_->last_grad_norm();   // synchronises
    autograd::detail::raise_device_flag();
    if (skip_nonfinite_ && !std::isfinite(s.grad_norm))
    {
        // AdamW left every weight and moment as it was: take the step count back
        s.skipped = true;
        if (sharded())
        {
            dp_->rewind_step();
        }
        else if (opt_->steps() > 0)
        {
            opt_->set_steps(opt_->steps() - 1);
        }
    }
    return s;
}

} // namespace veda::train
