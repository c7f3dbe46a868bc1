// veda::optim — AdamW and global-norm clipping with the reference's API and arithmetic
// (src/libs/optim/AdamW.h:23-59, AdamW.cpp:15-109; Clip.h:34, Clip.cpp:12-61) on device
// gradients.
//
// AdamW keeps fp32 first and second moments in two flat arenas and, for bf16 parameters, an fp32
// master copy (the parameter's bf16 value is rewritten from it after every step). Parameters
// whose gradients, values and masters lie back to back in memory — every parameter of
// train::TinyTransformer does — are updated by one kernel launch. step_clipped() fuses the
// global-norm clip into the update (the norm is computed on the device and read by the update
// kernel, no host round trip).
#pragma once

#include "veda/autograd.hpp"

#include <vector>

namespace veda::optim
{

struct AdamWConfig
{
    float learning_rate = 1e-3f;
    float beta1 = 0.9f;
    float beta2 = 0.999f;
    float eps = 1e-8f;
    float weight_decay = 0.01f;
};

class AdamW
{
public:
    explicit AdamW(std::vector<autograd::Variable> parameters, AdamWConfig config = {});
    ~AdamW();
    AdamW(const AdamW&) = delete;
    AdamW& operator=(const AdamW&) = delete;

    // The reference step: m, v, bias correction in double, decoupled decay first. Does not clear
    // the gradients.
    void step();
    // Clip to max_norm (the global norm of grad_scale * g) and step, in two launches per run of
    // contiguous parameters; nothing is synchronised. grad_scale carries a data-parallel 1/world.
    void step_clipped(float max_norm, float grad_scale = 1.0f);
    // step_clipped split in two for a step replayed from a CUDA graph: advance() counts the step
    // and leaves its bias corrections in device memory (not capturable: call it before each
    // replay); launch_clipped() only launches kernels, which read them there.
    void advance();
    void launch_clipped(float max_norm, float grad_scale = 1.0f);
    // The pre-clip global norm of the last step_clipped() (synchronises the stream).
    float last_grad_norm();
    void zero_grad();

    size_t steps() const noexcept { return steps_; }
    const AdamWConfig& config() const noexcept { return config_; }
    // First and second moments of every parameter, fp32, back to back in parameter order.
    const core::Tensor& first_moments() const noexcept { return m_arena_; }
    const core::Tensor& second_moments() const noexcept { return v_arena_; }
    // Restores the step count (the bias corrections of the next step use steps + 1).
    void set_steps(size_t steps) noexcept { steps_ = steps; }
    // On: a clipped step whose global norm is not finite updates nothing (weights, moments and
    // gradients are left as they were); the caller, who reads the norm, then takes the step back
    // with set_steps(steps() - 1). Off (the default, the reference's behaviour): the step runs.
    void set_skip_nonfinite(bool on) noexcept { skip_nonfinite_ = on; }
    bool skip_nonfinite() const noexcept { return skip_nonfinite_; }
    const std::vector<autograd::Variable>& parameters() const noexcept { return parameters_; }
    // fp32 master weights of parameter i (the value itself for fp32 parameters).
    core::Tensor master(size_t i) const { return masters_[i]; }
    // Number of kernel launches one step issues (one per contiguous run).
    size_t runs() const noexcept { return runs_.size(); }

private:
    bool skip_nonfinite_ = false;
    struct Run
    {
        size_t first, count;
        int64_t n;
        float* grad;
        float* master;
        float* m;
        float* v;
        void* lowp;   // bf16 value copy, or null for fp32 parameters
    };
    void build_runs();
    void launch(const double* sumsq, float max_norm, float grad_scale);

    std::vector<autograd::Variable> parameters_;
    std::vector<core::Tensor> masters_;
    core::Tensor m_arena_, v_arena_, master_arena_;
    std::vector<Run> runs_;
    AdamWConfig config_;
    size_t steps_ = 0;
    core::Tensor sumsq_;     // device double
    core::Tensor bias_;      // device double [2]: 1 - beta1^t, 1 - beta2^t of the current step
    double bias_host_[2] = {1.0, 1.0};
    core::Tensor workspace_;
    float last_scale_ = 1.0f;
};

// Global-norm clip in place; returns the pre-clip norm (Clip.cpp semantics; synchronises).
float clip_gradient_norm(const std::vector<autograd::Variable>& parameters, float max_norm);

} // namespace veda::optim
