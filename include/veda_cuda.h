/*
 * veda_cuda.h — the C ABI of libveda_cuda.so: hand-written sm_100a kernels for the backward path
 * of Veda's training step (forward kernels included where the backward needs their saved state).
 *
 * Conventions
 *   - Every entry point returns an int status: VEDA_OK (0) or a negative VEDA_ERR_* code; the
 *     message of the last failure on the calling thread is veda_last_error().
 *   - Pointers are device pointers unless stated otherwise; sizes and leading dimensions are in
 *     ELEMENTS; matrices are row-major. `dtype` is VEDA_F32 or VEDA_BF16 and applies to every
 *     activation-like operand of the call; parameter gradients are always fp32.
 *   - `stream` is a cudaStream_t (NULL = legacy default stream). Nothing is synchronised: every
 *     call is an asynchronous launch on `stream`.
 *   - Token-major activations: element (b, t, h, d) of a [B, T, H, Dh] tensor lives at
 *     ptr[(b*T + t) * ld + h*Dh + d]; `ld` lets q, k and v be column slices of one fused buffer.
 *
 * The reference (pictaile/veda) has no C ABI: its boundary is the C++ autograd API of
 * src/libs/autograd/Variable.h:69-119. Each entry point names the reference function whose
 * arithmetic it carries. The C++ host library (include/veda/*.hpp) calls these and turns status
 * codes into the reference's exception types.
 */
#ifndef VEDA_CUDA_H
#define VEDA_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* veda_stream_t;

enum veda_status {
    VEDA_OK = 0,
    VEDA_ERR_INVALID_ARGUMENT = -1, /* reference: std::invalid_argument */
    VEDA_ERR_CUDA = -2,             /* a CUDA launch or runtime failure   */
    VEDA_ERR_TIMEOUT = -3,          /* a bounded device wait gave up      */
    VEDA_ERR_UNSUPPORTED = -4,      /* shape/alignment the library does not handle */
    VEDA_ERR_OUT_OF_RANGE = -5      /* reference: std::out_of_range (ids) */
};

enum veda_dtype { VEDA_F32 = 0, VEDA_BF16 = 1 };

/* ---------------------------------------------------------------------------------------- */
/* Library                                                                                    */
/* ---------------------------------------------------------------------------------------- */
const char* veda_last_error(void);
/* Number of SMs and compute capability of the current device. */
int veda_device_info(int* sm_count, int* cc_major, int* cc_minor);
/* Kernel launches issued by this library since load (all threads); a diagnostic counter. */
uint64_t veda_launch_count(void);
/* Adds n (may be negative) to that counter: a caller replaying a CUDA graph of this library's
 * kernels adds the graph's kernel count per replay. */
int veda_launch_count_add(int64_t n);
/* The current device's status word: 0, or VEDA_ERR_TIMEOUT if a kernel's bounded device-side
 * wait gave up since the last reset. Synchronises with the device; reset = 1 clears it. The word
 * is a device variable compiled into the library (one per GPU, never allocated); its address is
 * looked up once per device and cached, so after a cudaDeviceReset use a fresh process. */
int veda_kernel_status(int reset);
/* Diagnostic of the bounded waits: one CTA waits, through the same bounded mbarrier wait the
 * tensor-core and streaming kernels use, on a barrier nothing arrives on, giving up after
 * budget_cycles (at most 2^32, the kernels' own budget, about two seconds) with VEDA_ERR_TIMEOUT
 * in the status word; nothing else is in flight. No counterpart in the reference. */
int veda_wait_timeout_check(long long budget_cycles, veda_stream_t stream);
/* Number of SMs the persistent kernels (tensor-core GEMMs, streaming RMSNorm) leave free for
 * work running beside them, such as NCCL all-reduce blocks during a data-parallel backward;
 * 0 (the default) uses every SM. Process-wide; returns the previous value. No counterpart in
 * the reference (its kernels are CPU loops). */
int veda_set_reserved_sms(int n);

/* ---------------------------------------------------------------------------------------- */
/* GEMM — the Linear / LM-head matmuls and both of their backward products.                  */
/*   bf16 operands: tcgen05.mma (TMEM accumulator, TMA-fed shared memory), fp32 accumulate.   */
/*   fp32 operands: fp32 FFMA kernel (exact-precision path for fp32 parity).                 */
/* C[M,N] = alpha * op(A) op(B) + beta * C   (beta = 0: C is not read)                        */
/* ---------------------------------------------------------------------------------------- */
/* NT: A[M,K] (lda), B[N,K] (ldb). Linear forward y = x W^T: ops::matmul_nt
 *     (src/libs/ops/Matmul.cpp:259-262) via autograd::matmul_nt (src/libs/autograd/Variable.cpp:325-327). */
int veda_gemm_nt(int64_t M, int64_t N, int64_t K, const void* A, int64_t lda, const void* B,
                 int64_t ldb, void* C, int64_t ldc, int dtype_ab, int dtype_c, float alpha,
                 float beta, veda_stream_t stream);
/* NN: A[M,K] (lda), B[K,N] (ldb). Input gradient dX = dY W: ops::matmul(g, W)
 *     (src/libs/autograd/Variable.cpp:338). */
int veda_gemm_nn(int64_t M, int64_t N, int64_t K, const void* A, int64_t lda, const void* B,
                 int64_t ldb, void* C, int64_t ldc, int dtype_ab, int dtype_c, float alpha,
                 float beta, veda_stream_t stream);
/* TN: A[K,M] (lda), B[K,N] (ldb). Weight gradient dW = dY^T X summed over every token:
 *     ops::matmul(transpose(g), x) + unbroadcast (src/libs/autograd/Variable.cpp:342-343, 48-87). */
int veda_gemm_tn(int64_t M, int64_t N, int64_t K, const void* A, int64_t lda, const void* B,
                 int64_t ldb, void* C, int64_t ldc, int dtype_ab, int dtype_c, float alpha,
                 float beta, veda_stream_t stream);
/* Batched form of the three products above (op = 0 NT, 1 NN, 2 TN) with element strides between
 * batch entries; a stride of 0 broadcasts that operand (ops::matmul's batch broadcast,
 * src/libs/ops/Matmul.cpp:169-250). */
int veda_gemm_batched(int op, int64_t batch, int64_t M, int64_t N, int64_t K, const void* A,
                      int64_t lda, int64_t stride_a, const void* B, int64_t ldb, int64_t stride_b,
                      void* C, int64_t ldc, int64_t stride_c, int dtype_ab, int dtype_c,
                      float alpha, float beta, veda_stream_t stream);
/* The MLP's gate|up projection with SwiGLU fused into the GEMM (bf16): gate_up[rows, 2F] =
 * x[rows, D] w_gate_up[2F, D]^T (rows 0..F-1 of the weight the gate projection, F..2F-1 the up
 * projection) and h[rows, F] = silu(gate) * up (src/libs/train/Model.cpp:199-202). Bit for bit
 * veda_gemm_nt followed by veda_swiglu_fwd; VEDA_ERR_UNSUPPORTED (nothing runs) unless F is a
 * multiple of 128, rows >= 256 and D a multiple of 8, with 16-byte aligned rows. */
int veda_gemm_swiglu_fwd(int64_t rows, int64_t F, int64_t D, const void* x, int64_t ldx,
                         const void* w_gate_up, int64_t ldw, void* gate_up, int64_t ldgu, void* h,
                         int64_t ldh, veda_stream_t stream);
/* Its backward through the down projection (bf16): dh = dy[rows, D] w_down[D, F] is never
 * stored; with gate and up from gate_up[rows, 2F] the GEMM writes dgate_up[rows, 2F] =
 * (dgate | dup) (src/libs/autograd/Variable.cpp:338, NonLinear.cpp:47-63, Variable.cpp:218-239).
 * Bit for bit veda_gemm_nn into a bf16 dh followed by veda_swiglu_bwd; VEDA_ERR_UNSUPPORTED
 * (nothing runs) unless F is a multiple of 256, rows >= 256 and D a multiple of 8, with 16-byte
 * aligned rows. */
int veda_gemm_swiglu_bwd(int64_t rows, int64_t F, int64_t D, const void* dy, int64_t lddy,
                         const void* w_down, int64_t ldw, const void* gate_up, int64_t ldgu,
                         void* dgate_up, int64_t lddgu, veda_stream_t stream);

/* ---------------------------------------------------------------------------------------- */
/* RMSNorm with gain: y = gamma * x / sqrt(mean(x^2) + eps) over rows of n.                   */
/*   ops::rms_normalize (src/libs/ops/Normalize.cpp:18-70) + mul by gamma (Model.cpp:242-243).*/
/*   gamma == NULL means gain 1 (plain rms_normalize).                                       */
/* ---------------------------------------------------------------------------------------- */
int veda_rmsnorm_fwd(const void* x, int64_t ldx, const void* gamma, void* y, int64_t ldy,
                     int64_t rows, int64_t n, float eps, int dtype, veda_stream_t stream);
/* The residual add followed by the next norm (Model.cpp:244-249, the add of Variable.cpp:195-216
 * then the RMSNorm above), in one pass for bf16 rows of 256/512/1024/2048: sum = x + r (rounded
 * to the dtype, as the add stores it) and y = RMSNorm(sum) * gamma. */
int veda_add_rmsnorm_fwd(const void* x, int64_t ldx, const void* r, int64_t ldr,
                         const void* gamma, void* sum, int64_t lds, void* y, int64_t ldy,
                         int64_t rows, int64_t n, float eps, int dtype, veda_stream_t stream);
/* Backward (src/libs/autograd/NonLinear.cpp:153-201 and the gain's mul/unbroadcast,
 * Variable.cpp:218-239): dx = dresid + (G/r - x * sum(G x)/(n r^3)), G = dy * gamma;
 * dgamma (fp32 [n], may be NULL) += sum over rows of dy * x / r, in a fixed order. dresid may be
 * NULL. workspace: veda_rmsnorm_bwd_workspace(rows, n) bytes of device scratch (NULL if dgamma
 * NULL). */
int veda_rmsnorm_bwd(const void* x, int64_t ldx, const void* gamma, const void* dy, int64_t lddy,
                     const void* dresid, int64_t ldr, void* dx, int64_t lddx, float* dgamma,
                     void* workspace, size_t workspace_bytes, int64_t rows, int64_t n, float eps,
                     int dtype, veda_stream_t stream);
size_t veda_rmsnorm_bwd_workspace(int64_t rows, int64_t n);
/* veda_rmsnorm_bwd for callers that cannot allocate device memory. No counterpart in the
 * reference (its CPU loop needs no scratch); it exists because a workspace costs a cudaMalloc,
 * which synchronises the device and can fail under an engine that reserves its memory up front,
 * and because a caller binding this library through a plain C ABI may have no device allocator.
 * Its scratch (the per-block partial sums of dgamma) is a fixed 4 MiB array compiled into the
 * library: every GPU that loads the library holds it until the process exits. Limit: the
 * scratch needed, veda_rmsnorm_bwd_workspace(rows, n) bytes, must be at most 4 MiB (rows of up
 * to 3542 elements on a 148-SM B200); larger sizes are rejected with VEDA_ERR_INVALID_ARGUMENT.
 * The first call on a device looks up the array's device address (cudaGetSymbolAddress); make
 * that first call before any stream capture. The address is cached per device for the life of
 * the process, so after a cudaDeviceReset use a fresh process. All calls share the one array, so calls that
 * overlap on the GPU (on different streams without ordering) race; calls ordered on one stream
 * do not (each call overwrites the partials it reads). Allocates nothing. */
int veda_rmsnorm_bwd_noalloc(const void* x, int64_t ldx, const void* gamma, const void* dy,
                             int64_t lddy, const void* dresid, int64_t ldr, void* dx,
                             int64_t lddx, float* dgamma, int64_t rows, int64_t n, float eps,
                             int dtype, veda_stream_t stream);

/* ---------------------------------------------------------------------------------------- */
/* QK-norm + RoPE, per head over head_dim (Model.cpp:171-178): y = rope(gamma * x / r).       */
/*   x: tokens x heads x head_dim token-major (ld per token); token n sits at position        */
/*   n % seq_len. cos/sin: fp32 [seq_len, head_dim] tables of model::rope_tables              */
/*   (src/libs/model/Rope.cpp:17-63); rotation of autograd::rope (Views.cpp:78-134).           */
/* ---------------------------------------------------------------------------------------- */
int veda_qknorm_rope_fwd(const void* x, int64_t ldx, const void* gamma, const float* cos,
                         const float* sin, void* y, int64_t ldy, int64_t tokens, int64_t heads,
                         int64_t seq_len, int64_t head_dim, float eps, int dtype,
                         veda_stream_t stream);
/* veda_qknorm_rope_fwd for the q and the k heads of one attention layer in one launch: x rows xq
 * (heads) and xk (kv_heads) at stride ldx, their gains, outputs yq / yk at their strides; the
 * same arithmetic, bit for bit, as two veda_qknorm_rope_fwd calls. */
int veda_qknorm_rope_fwd_qk(const void* xq, const void* xk, int64_t ldx, const void* q_gamma,
                            const void* k_gamma, const float* cos, const float* sin, void* yq,
                            int64_t ldyq, void* yk, int64_t ldyk, int64_t tokens, int64_t heads,
                            int64_t kv_heads, int64_t seq_len, int64_t head_dim, float eps,
                            int dtype, veda_stream_t stream);
/* Backward: rotate dy by -theta (Views.cpp:136-171), then the gain and norm backward as above.
 * dgamma (fp32 [head_dim]) += sum over tokens and heads, in a fixed order. */
int veda_qknorm_rope_bwd(const void* x, int64_t ldx, const void* gamma, const float* cos,
                         const float* sin, const void* dy, int64_t lddy, void* dx, int64_t lddx,
                         float* dgamma, void* workspace, size_t workspace_bytes, int64_t tokens,
                         int64_t heads, int64_t seq_len, int64_t head_dim, float eps, int dtype,
                         veda_stream_t stream);
size_t veda_qknorm_rope_bwd_workspace(int64_t tokens, int64_t heads, int64_t head_dim);
/* veda_qknorm_rope_bwd for the q and the k heads of one attention layer (Model.cpp:171-178 applies
 * q_norm and k_norm to the same positions) in one launch, and one launch of the two gain
 * reductions: x rows xq (heads) and xk (kv_heads) at stride ldx, gradients dyq / dyk at their
 * strides, results dxq / dxk at stride lddx, dq_gamma / dk_gamma (either may be NULL) +=.
 * The same arithmetic as two veda_qknorm_rope_bwd calls; the gain gradients are summed over a
 * different number of blocks, so they agree with those calls to rounding. dyq_f32 = 1 (bf16,
 * head_dim 128 only): dyq holds fp32 rows (stride lddyq floats, 16-byte aligned), read as
 * bf16(dyq * dyq_scale) — the dQ accumulator veda_attention_bwd_dq_f32 leaves, with the rounding
 * veda_attention_bwd applies when it writes dq itself. workspace:
 * veda_qknorm_rope_bwd_qk_workspace() bytes. */
int veda_qknorm_rope_bwd_qk(const void* xq, const void* xk, int64_t ldx, const void* q_gamma,
                            const void* k_gamma, const float* cos, const float* sin,
                            const void* dyq, int64_t lddyq, int dyq_f32, float dyq_scale,
                            const void* dyk, int64_t lddyk, void* dxq, void* dxk, int64_t lddx,
                            float* dq_gamma, float* dk_gamma, void* workspace,
                            size_t workspace_bytes, int64_t tokens, int64_t heads,
                            int64_t kv_heads, int64_t seq_len, int64_t head_dim, float eps,
                            int dtype, veda_stream_t stream);
size_t veda_qknorm_rope_bwd_qk_workspace(int64_t tokens, int64_t heads, int64_t kv_heads,
                                         int64_t head_dim);

/* Plain RoPE on a contiguous [lanes, seq_len, head_dim] tensor (autograd::rope,
 * src/libs/autograd/Views.cpp:78-171); inverse = 1 rotates by -theta (the backward). */
int veda_rope(const void* x, void* y, const float* cos, const float* sin, int64_t lanes,
              int64_t seq_len, int64_t head_dim, int inverse, int dtype, veda_stream_t stream);

/* ---------------------------------------------------------------------------------------- */
/* SwiGLU: h = silu(gate) * up (Model.cpp:198-204; silu of Activations.cpp:13-16).            */
/* ---------------------------------------------------------------------------------------- */
int veda_swiglu_fwd(const void* gate, int64_t ldg, const void* up, int64_t ldu, void* h,
                    int64_t ldh, int64_t rows, int64_t n, int dtype, veda_stream_t stream);
/* dgate = dh * up * s(1 + g(1 - s)), dup = dh * silu(g)   (NonLinear.cpp:47-63, Variable.cpp:218-239) */
int veda_swiglu_bwd(const void* gate, int64_t ldg, const void* up, int64_t ldu, const void* dh,
                    int64_t lddh, void* dgate, int64_t lddg, void* dup, int64_t lddu,
                    int64_t rows, int64_t n, int dtype, veda_stream_t stream);

/* ---------------------------------------------------------------------------------------- */
/* Fused softmax cross-entropy (autograd::cross_entropy, src/libs/autograd/Loss.cpp:18-103).  */
/*   row_loss[r] = -(x_t - max - log sum exp(x - max)) in fp32;                                */
/*   dlogits = (softmax(x) - onehot(t)) * grad_scale (grad_scale = upstream / lanes), written  */
/*   in dtype; dlogits may alias logits (in place). dlogits == NULL: forward only.            */
/*   status (device int, may be NULL) receives VEDA_ERR_OUT_OF_RANGE if a target is outside  */
/*   [0, vocab); such a row is skipped.                                                        */
/* ---------------------------------------------------------------------------------------- */
int veda_cross_entropy(const void* logits, int64_t ldl, const int64_t* targets, float* row_loss,
                       void* dlogits, int64_t ldd, int64_t rows, int64_t vocab, float grad_scale,
                       int* status, int dtype, veda_stream_t stream);
/* out[0] = (float)(sum_i v[i] / n) with the sum in double, in a fixed order (Loss.cpp:52-60). */
int veda_mean_f64(const float* v, int64_t n, float* out, double* out_f64, veda_stream_t stream);

/* ---------------------------------------------------------------------------------------- */
/* Embedding (autograd::embedding, src/libs/autograd/NonLinear.cpp:203-254).                  */
/* ---------------------------------------------------------------------------------------- */
/* out[p] = table[ids[p]], bit-exact. An id outside [0, vocab) writes zeros and sets *status
 * (device int, may be NULL) to VEDA_ERR_OUT_OF_RANGE. */
int veda_embedding_fwd(const int64_t* ids, int64_t count, const void* table, int64_t vocab,
                       int64_t dim, void* out, int64_t ldo, int* status, int dtype,
                       veda_stream_t stream);
/* dtable (fp32 [vocab, dim]) += scatter of dout rows. deterministic = 1: each id's rows are
 * added in ascending position order onto the existing value, the loop order of
 * NonLinear.cpp:245-252, so the result equals the CPU's bit for bit given equal inputs.
 * deterministic = 0: fp32 atomics (order unspecified). */
int veda_embedding_bwd(const int64_t* ids, int64_t count, const void* dout, int64_t ldd,
                       int64_t vocab, int64_t dim, float* dtable, int deterministic,
                       void* workspace, size_t workspace_bytes, int dtype, veda_stream_t stream);
size_t veda_embedding_bwd_workspace(int64_t count);
/* The deterministic scatter of veda_embedding_bwd in two halves, for a caller that moves the rows
 * between them (the data-parallel exchange of the embedding's scattered rows). sort: keys[i] =
 * (id << 32 | position) of `count` <= 16384 positions, ascending (out-of-range ids last).
 * apply_sorted: for every id in [id_lo, id_hi), dtable[(id - id_lo) * dim ..] += its rows of
 * dout in key order; other ids are skipped. Applying the key lists of several senders one after
 * the other adds each id's rows in (sender, position) order. */
int veda_embedding_sort(const int64_t* ids, int64_t count, int64_t vocab, uint64_t* keys,
                        veda_stream_t stream);
int veda_embedding_apply_sorted(const uint64_t* keys, int64_t count, const void* dout, int64_t ldd,
                                int64_t dim, int64_t id_lo, int64_t id_hi, float* dtable,
                                int dtype, veda_stream_t stream);

/* ---------------------------------------------------------------------------------------- */
/* Global-norm clip + AdamW (optim::clip_gradient_norm, src/libs/optim/Clip.cpp:12-61;        */
/* optim::AdamW::step, src/libs/optim/AdamW.cpp:38-93).                                        */
/* ---------------------------------------------------------------------------------------- */
/* *sumsq (device double) = sum of g^2 over n floats, in double, deterministic order.
 * accumulate = 1 adds to the existing *sumsq (several tensors, one norm). */
int veda_sumsq(const float* g, int64_t n, double* sumsq, int accumulate, void* workspace,
               size_t workspace_bytes, veda_stream_t stream);
size_t veda_sumsq_workspace(int64_t n);
/* In place g *= clip scale, where total = sqrt(*sumsq) and the scale is float(max_norm/total)
 * only when total is finite and > max_norm (otherwise nothing is written). */
int veda_clip_apply(float* g, int64_t n, const double* sumsq, float max_norm,
                    veda_stream_t stream);
/* One AdamW step on fp32 master weights:
 *   g' = g * grad_scale (skipped when grad_scale == 1) * clip, where clip is computed as in
 *   veda_clip_apply from total = sqrt(*sumsq) * grad_scale (sumsq of the unscaled g; NULL = no
 *   clip) — grad_scale carries the 1/world average of data-parallel training
 *   m = b1 m + (1-b1) g';  v = b2 v + (1-b2) g'^2  (fp32, unfused roundings as the reference)
 *   w -= lr*wd*w;  w -= lr * float((m/bias1) / (sqrt(v/bias2) + eps))  (m_hat, v_hat in double)
 * bias1 = 1 - beta1^t, bias2 = 1 - beta2^t computed by the caller in double.
 * lowp (bf16 [n], may be NULL) receives the rounded copy the forward reads.
 * write_grad is a set of bits. Bit 0 (1) leaves g' in g (the clipped gradient, as Clip.cpp:52-58
 * leaves it); the store is skipped when g' == g (no clip and grad_scale 1). Bit 1
 * (VEDA_ADAMW_SKIP_NONFINITE) leaves master, m, v, g and lowp untouched when the norm
 * float(sqrt(*sumsq) * |grad_scale|) is not finite: the step is skipped (the reference has no
 * skip; its clip only declines to scale a non-finite norm, Clip.cpp:36-40). */
#define VEDA_ADAMW_SKIP_NONFINITE 2
int veda_adamw_step(float* master, float* m, float* v, float* g, void* lowp, int64_t n, float lr,
                    float beta1, float beta2, float eps, float weight_decay, double bias1,
                    double bias2, const double* sumsq, float max_norm, float grad_scale,
                    int write_grad, veda_stream_t stream);
/* The same with bias1, bias2 read from device memory (bias[0], bias[1], doubles) when the kernel
 * runs, so one launch recorded in a CUDA graph serves every step. */
int veda_adamw_step_dev(float* master, float* m, float* v, float* g, void* lowp, int64_t n,
                        float lr, float beta1, float beta2, float eps, float weight_decay,
                        const double* bias, const double* sumsq, float max_norm, float grad_scale,
                        int write_grad, veda_stream_t stream);

/* ---------------------------------------------------------------------------------------- */
/* Element-wise and per-lane ops of the fine-grained autograd API.                           */
/* ---------------------------------------------------------------------------------------- */
/* out = a (+|*) b with numpy broadcasting expressed by strides (0 = broadcast axis), rank <= 8.
 * op: 0 add (ops::add, src/libs/ops/Elementwise.cpp:24-49), 1 mul (ops::mul). */
int veda_binary(int op, const void* a, const int64_t* a_strides, const void* b,
                const int64_t* b_strides, void* out, const int64_t* shape, int rank, int dtype,
                veda_stream_t stream);
/* out = x * s (ops::mul by a scalar). */
int veda_scale(const void* x, float s, void* out, int64_t n, int dtype, veda_stream_t stream);
/* dst += src, element-wise over n (detail accumulate, Variable.cpp:27-38); dst in dtype_dst. */
int veda_accumulate(void* dst, int dtype_dst, const void* src, int dtype_src, int64_t n,
                    veda_stream_t stream);
/* Copy a strided view of rank <= 8 into a contiguous tensor (core::contiguous,
 * src/libs/tensor/Tensor.cpp:157-191); dtype conversion allowed. */
int veda_copy_strided(const void* src, int dtype_src, const int64_t* src_strides, int64_t offset,
                      void* dst, int dtype_dst, const int64_t* shape, int rank,
                      veda_stream_t stream);
/* Sum a contiguous gradient over broadcast axes down to `target` (detail::unbroadcast,
 * Variable.cpp:48-87). shape/target are aligned to `rank` (target axes of extent 1 or
 * leading axes absent from the target collapse). out is contiguous fp32 or dtype. */
int veda_unbroadcast(const void* g, const int64_t* shape, const int64_t* target, int rank,
                     void* out, int dtype, veda_stream_t stream);
/* out[0] = sum of x (autograd::sum, Variable.cpp:260-287), fp32 result, double accumulation. */
int veda_sum(const void* x, int64_t n, float* out, int dtype, veda_stream_t stream);
/* Fill n elements with a value. */
int veda_fill(void* x, float value, int64_t n, int dtype, veda_stream_t stream);
/* softmax over the last dim of [lanes, length] (ops::softmax, src/libs/ops/Softmax.cpp:20-80)
 * and its backward y * (g - sum(g y)) (NonLinear.cpp:89-151). */
int veda_softmax_fwd(const void* x, void* y, int64_t lanes, int64_t length, int dtype,
                     veda_stream_t stream);
int veda_softmax_bwd(const void* y, const void* g, void* dx, int64_t lanes, int64_t length,
                     int dtype, veda_stream_t stream);
/* log_softmax over the last dim of [lanes, length] (ops::log_softmax,
 * src/libs/ops/Softmax.cpp:82-151): x - m - log(sum exp(x - m)); an all -inf lane stays -inf. */
int veda_log_softmax_fwd(const void* x, void* y, int64_t lanes, int64_t length, int dtype,
                         veda_stream_t stream);
/* silu and its backward on n elements (Activations.cpp:13-16, NonLinear.cpp:47-63). */
int veda_silu_fwd(const void* x, void* y, int64_t n, int dtype, veda_stream_t stream);
int veda_silu_bwd(const void* x, const void* g, void* dx, int64_t n, int dtype,
                  veda_stream_t stream);
/* tanh-GELU and its backward on n elements (src/libs/ops/Activations.cpp:18-26,
 * src/libs/autograd/NonLinear.cpp:65-87). */
int veda_gelu_fwd(const void* x, void* y, int64_t n, int dtype, veda_stream_t stream);
int veda_gelu_bwd(const void* x, const void* g, void* dx, int64_t n, int dtype,
                  veda_stream_t stream);
/* Row argmax over [rows, n], ties to the lower index, NaN -> *status = VEDA_ERR_INVALID_ARGUMENT
 * (generate::greedy_of, src/libs/generate/Sampling.cpp:97-113). */
int veda_argmax(const void* x, int64_t ld, int64_t rows, int64_t n, int64_t* out, int* status,
                int dtype, veda_stream_t stream);
/* One query row per head against a KV cache (generation): out[h] = softmax(q[h] . k[j] * scale
 * over j < len) . v[j], k/v rows of len positions at stride ldkv holding kv_heads heads; query
 * head h reads KV head h / (heads / kv_heads) (ScaledDotProductAttention.cpp:138-191, one row). */
int veda_attention_decode(const void* q, const void* k, const void* v, int64_t ldkv, int64_t len,
                          int64_t heads, int64_t kv_heads, int64_t head_dim, float scale,
                          void* out, int dtype, veda_stream_t stream);
/* The same with the query's position read from device memory (len = *pos + 1), so a decode
 * step recorded once in a CUDA graph serves every position. */
int veda_attention_decode_at(const void* q, const void* k, const void* v, int64_t ldkv,
                             const int64_t* pos, int64_t heads, int64_t kv_heads, int64_t head_dim,
                             float scale, void* out, int dtype, veda_stream_t stream);
/* One decoded token's projections qkv [(H + 2 Hkv) Dh] at position *pos (device memory): QK-norm
 * and RoPE of the query heads into q_out and of the KV heads into row *pos of k_cache, the
 * values into row *pos of v_cache (rows of ldkv elements). Model.cpp:173-178, Views.cpp:78-134. */
int veda_decode_qkv_at(const void* qkv, const void* q_gain, const void* k_gain, const float* cos,
                       const float* sin, const int64_t* pos, void* q_out, void* k_cache,
                       void* v_cache, int64_t ldkv, int64_t heads, int64_t kv_heads,
                       int64_t head_dim, float eps, int dtype, veda_stream_t stream);
/* *pos += 1 on the device (the last node of a recorded decode step). */
int veda_decode_advance(int64_t* pos, veda_stream_t stream);
/* One activation row through a Linear layer (x . W^T of Variable.cpp:325, matmul_nt, at M = 1):
 * y[i] = sum_j x[j] * w[i, j] for i < n, j < k, rows of w at stride ldw; fp32 accumulation, each
 * output rounded once. HBM-bound: every weight byte is read once. k * element size <= 47 KB. */
int veda_gemv_nt(const void* x, const void* w, int64_t ldw, void* y, int64_t n, int64_t k, int dtype,
                 veda_stream_t stream);
/* The gate/up Linear and SwiGLU of one row in one pass: w_gate_up holds the gate rows [0, f) and
 * the up rows [f, 2f); h[i] = silu(g_i) * u_i on g and u rounded to the dtype, the arithmetic of
 * veda_gemv_nt followed by veda_swiglu_fwd (Model.cpp:198-204). */
int veda_gemv_swiglu(const void* x, const void* w_gate_up, int64_t ldw, void* h, int64_t f,
                     int64_t k, int dtype, veda_stream_t stream);
/* veda_gemv_nt / veda_gemv_swiglu on the pre-norm of a residual row (Model.cpp:242-249): the
 * activation is RMSNorm(s) * gamma with s = x + r (r may be NULL: s = x), s rounded to the dtype
 * and written to sum when sum is not NULL (sum must not alias x or r); 2 k * element size
 * <= 47 KB. */
int veda_gemv_rmsnorm(const void* x, const void* r, const void* gamma, float eps, void* sum,
                      const void* w, int64_t ldw, void* y, int64_t n, int64_t k, int dtype,
                      veda_stream_t stream);
int veda_gemv_rmsnorm_swiglu(const void* x, const void* r, const void* gamma, float eps, void* sum,
                             const void* w_gate_up, int64_t ldw, void* h, int64_t f, int64_t k,
                             int dtype, veda_stream_t stream);
/* veda_gemv_rmsnorm over the LM head with the greedy choice fused in: *token = argmax of the
 * rounded outputs y (ties to the lower index; a NaN anywhere: *token = -1 and *status =
 * VEDA_ERR_INVALID_ARGUMENT, as veda_argmax), merged by the last block to finish through
 * `workspace` (at least veda_gemv_argmax_workspace(n) bytes, 16-byte aligned, zero before its
 * first use, left ready for the next call; one call at a time per workspace). */
int64_t veda_gemv_argmax_workspace(int64_t n);
int veda_gemv_rmsnorm_argmax(const void* x, const void* r, const void* gamma, float eps, void* sum,
                             const void* w, int64_t ldw, void* y, int64_t n, int64_t k,
                             int64_t* token, int* status, void* workspace,
                             int64_t workspace_bytes, int dtype, veda_stream_t stream);
/* veda_decode_qkv_at followed by veda_attention_decode_at in one launch (head_dim 128, heads /
 * kv_heads in {1, 2, 4, 8}, 16-byte aligned cache rows, else VEDA_ERR_UNSUPPORTED): the token's
 * QK-norm + RoPE, its key and value written into cache row *pos, and out[h] = attention of query
 * head h over positions 0..*pos. The positions are split across CTAs by the cache's capacity (rows)
 * and the slices merged by the last CTA of each KV head to finish, through `workspace` (at least
 * veda_decode_attention_workspace bytes, 16-byte aligned, zero before its first use; every call
 * leaves it ready for the next; one call at a time per workspace). A *pos outside [0, capacity)
 * writes nothing. */
int64_t veda_decode_attention_workspace(int64_t heads, int64_t kv_heads, int64_t capacity);
int veda_decode_attention_at(const void* qkv, const void* q_gain, const void* k_gain,
                             const float* cos, const float* sin, const int64_t* pos, void* k_cache,
                             void* v_cache, int64_t ldkv, int64_t capacity, int64_t heads,
                             int64_t kv_heads, int64_t head_dim, float eps, float scale, void* out,
                             void* workspace, int64_t workspace_bytes, int dtype,
                             veda_stream_t stream);
/* Seeded N(0, std) fill (counter-based hash + Box-Muller) for synthetic weights. */
int veda_randn(void* x, int64_t n, float std, uint64_t seed, int dtype, veda_stream_t stream);
/* fp32 -> bf16 rounding copy (round to nearest even). */
int veda_f32_to_bf16(const float* src, void* dst, int64_t n, veda_stream_t stream);

/* ---------------------------------------------------------------------------------------- */
/* Corpus batches (data::Corpus::next_batch, src/libs/data/Corpus.cpp:64-107) from device ids. */
/* ---------------------------------------------------------------------------------------- */
/* Row k (0-based) of the batch starts at begin + splitmix64_mix(state + (k+1)*0x9E3779B97F4A7C15)
 * % (end - begin - length), the k-th draw of the reference's generator from `state`;
 * inputs[k*length + t] = ids[start + t], targets[...] = ids[start + t + 1]. The caller advances
 * its state by batch * 0x9E3779B97F4A7C15. Bit-identical to the reference's windows. */
int veda_corpus_gather(const int64_t* ids, int64_t begin, int64_t end, uint64_t state,
                       int64_t batch, int64_t length, int64_t* inputs, int64_t* targets,
                       veda_stream_t stream);

/* ---------------------------------------------------------------------------------------- */
/* Causal GQA attention (the composition of src/libs/train/Model.cpp:182-189:                 */
/* softmax(q k^T * scale + mask) v, KV head of query head h = h / (H/Hkv),                    */
/* src/libs/model/Attention.cpp:191).                                                          */
/*   q, o: [B, T, H, Dh] token-major; k, v: [B, T, Hkv, Dh]; lse: fp32 [B, H, T] saved for    */
/*   the backward (log-sum-exp of the scaled, masked scores).                                 */
/* ---------------------------------------------------------------------------------------- */
int veda_attention_fwd(const void* q, int64_t ldq, const void* k, int64_t ldk, const void* v,
                       int64_t ldv, void* o, int64_t ldo, float* lse, int64_t batch,
                       int64_t seq_len, int64_t heads, int64_t kv_heads, int64_t head_dim,
                       float scale, int causal, int dtype, veda_stream_t stream);
/* Recomputes P from lse; dq, dk, dv written (not accumulated) in dtype; dk/dv are summed over
 * the H/Hkv query heads of each group (the unbroadcast of the KV expansion).
 * workspace: veda_attention_bwd_workspace() bytes, sized for the mode set when it is asked
 * (bf16, head_dim 128: O(B*T*H*head_dim) fp32 for the fused kernel, O(B*H*T^2) bf16 in the
 * deterministic mode). The reference's backward of the composition is
 * src/libs/autograd/NonLinear.cpp:89-151 (softmax) with Variable.cpp:300-346 (the products). */
int veda_attention_bwd(const void* q, int64_t ldq, const void* k, int64_t ldk, const void* v,
                       int64_t ldv, const void* o, int64_t ldo, const void* dout, int64_t lddo,
                       const float* lse, void* dq, int64_t lddq, void* dk, int64_t lddk, void* dv,
                       int64_t lddv, void* workspace, size_t workspace_bytes, int64_t batch,
                       int64_t seq_len, int64_t heads, int64_t kv_heads, int64_t head_dim,
                       float scale, int causal, int dtype, veda_stream_t stream);
size_t veda_attention_bwd_workspace(int64_t batch, int64_t seq_len, int64_t heads,
                                    int64_t kv_heads, int64_t head_dim, int dtype);
/* veda_attention_bwd without its last pass: dQ is not written; it is left, unscaled, as fp32
 * [batch * seq_len, heads * 128] token-major rows (dQ = scale * row) at
 * workspace + veda_attention_bwd_dq_offset(), for a consumer that reads it directly
 * (veda_qknorm_rope_bwd_qk with dyq_f32). dK and dV are written as by veda_attention_bwd. Only the
 * fused tensor-core backward keeps dQ in fp32 (bf16, head_dim 128, 16-byte aligned operands, not
 * the deterministic mode); otherwise VEDA_ERR_UNSUPPORTED is returned and nothing runs. */
int veda_attention_bwd_dq_f32(const void* q, int64_t ldq, const void* k, int64_t ldk,
                              const void* v, int64_t ldv, const void* o, int64_t ldo,
                              const void* dout, int64_t lddo, const float* lse, void* dk,
                              int64_t lddk, void* dv, int64_t lddv, void* workspace,
                              size_t workspace_bytes, int64_t batch, int64_t seq_len, int64_t heads,
                              int64_t kv_heads, int64_t head_dim, float scale, int causal,
                              int dtype, veda_stream_t stream);
size_t veda_attention_bwd_dq_offset(int64_t batch, int64_t seq_len, int64_t heads);
/* on = 1: the bf16 backward runs its two-kernel form, whose dQ is bit-reproducible run to run
 * (dS^T through HBM, O(B*H*T^2) workspace); on = 0 (the default; VEDA_ATTENTION_DETERMINISTIC=1
 * in the environment starts at 1): the fused kernel, whose dQ sums key tiles in a varying order.
 * Process-wide; returns the previous setting. No counterpart in the reference (its CPU backward
 * is sequential). */
int veda_attention_set_deterministic(int on);

#ifdef __cplusplus
}
#endif

#endif /* VEDA_CUDA_H */
