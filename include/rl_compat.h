/*
 * rl_* entry points with the reference native library's names, argument lists and error
 * behaviour, exported by librl2.so beside the rl2_* ABI. A program that binds the
 * reference's ctypes tables (src/robolearn/cuda/_runtime.py:77-113, cuda/categorical.py:19-29,
 * cuda/flash.py:20-40, cuda/zero.py:17-22) can load librl2.so in place of the reference's
 * build of src/robolearn/cuda/kernels.cu and run unchanged.
 *
 * Conventions, as in the reference (src/robolearn/cuda/kernels.cu:4-49):
 *  - status 0 on success, -1 on a synchronous error with the message in rl_last_error();
 *  - run / step calls enqueue on the caller's stream, allocate nothing and do not
 *    synchronise; create / destroy calls may allocate and must run outside graph capture;
 *  - pointer tables and lengths are host arrays copied at create time; the device buffers
 *    they name stay caller-owned;
 *  - all floating-point buffers are fp32 unless a parameter says fp16.
 *
 * Differences that a caller can observe (everything else matches):
 *  - dense plans run on the library's tcgen05 kernels, not cuBLASLt: fp32 products use
 *    three tf32 tensor-core products per step (error ~1e-6 relative, fp32 storage), with
 *    or without allow_tf32; fp16 operands are read in place when lda and ldb are multiples
 *    of 8, else staged; rl_plan_workspace returns 0 (any staging is plan-owned);
 *    rl_plan_autotune validates its preconditions and freezes the single plan-chosen
 *    candidate, which rl_plan_tuning_metadata describes.
 *  - per-row categorical projections sum their contributions by runs of equal atom index in
 *    a fixed order (deterministic), where the reference adds them with shared-memory atomics;
 *    the categorical backward leaves intermediate sums in its scratch buffer.
 */
#ifndef RL_COMPAT_H
#define RL_COMPAT_H

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* kernels.cu:408. The same thread-local buffer as rl2_last_error. */
const char* rl_last_error(void);

/* Dense plans, column-major D = op(A) op(B) + beta C (+ bias[m] per row), kernels.cu:410-740.
 * transa / transb: 0 = N, 1 = T. input_dtype (mixed): 0 = fp32 A/B, 1 = fp16 A/B. */
void* rl_plan_create(int m, int n, int k, int transa, int transb, int lda, int ldb, int ldd,
                     int use_bias, int allow_tf32, size_t workspace_limit);           /* kernels.cu:528 */
void* rl_plan_create_mixed(int m, int n, int k, int transa, int transb, int lda, int ldb, int ldd,
                           int use_bias, int allow_tf32, int input_dtype,
                           size_t workspace_limit);                                    /* kernels.cu:534 */
int rl_plan_autotune(void* plan, float beta, void* stream);                           /* kernels.cu:540 */
const char* rl_plan_tuning_metadata(void* plan);                                      /* kernels.cu:654 */
size_t rl_plan_workspace(void* plan); /* SIZE_MAX on error */                         /* kernels.cu:689 */
int rl_plan_run(void* plan, const void* a, const void* b, const void* c, void* d, const void* bias,
                void* workspace, size_t workspace_bytes, float beta, void* stream);    /* kernels.cu:698 */
int rl_plan_destroy(void* plan);                                                      /* kernels.cu:733 */
int rl_cast_f32_f16(const void* source, void* destination, size_t count, void* stream); /* kernels.cu:663 */
/* db[c] += sum_rows dy[row * channels + c] (kernels.cu:742). */
int rl_bias_grad(const void* dy, void* db, int batch, int channels, void* stream);

/* Multi-tensor Adam with optional dynamic loss scaling (kernels.cu:760-916). */
void* rl_adam_create(size_t count, const void* const* parameters, const void* const* gradients,
                     const void* const* m1, const void* const* m2, const size_t* sizes, void* timestep,
                     void* learning_rate, double beta1, double beta2, double eps);
int rl_adam_set_scaler(void* plan, void* loss_scale, void* growth_tracker, void* found_inf,
                       void* step_skipped, void* attempted_steps, void* skipped_steps,
                       double growth_factor, double backoff_factor, int growth_interval);
int rl_adam_unscale(void* plan, void* stream);
int rl_adam_step(void* plan, void* stream);
int rl_adam_destroy(void* plan);

/* Weight-norm projection plans (flash_kernels.cuh:405-445). kinds: 0 = unit-linear row
 * (divided by max(||row||, 1e-8)), 1 = BN affine pair (joint norm sqrt(length)),
 * 2 = RMS scale vector (norm sqrt(length)). shadows: optional fp16 copies of kind-0 rows. */
void* rl_flash_projection_create(size_t count, const void* const* first, const void* const* second,
                                 const size_t* lengths, const int* kinds);
void* rl_flash_projection_create_with_shadows(size_t count, const void* const* first,
                                              const void* const* second, const size_t* lengths,
                                              const int* kinds, const void* const* shadows);
int rl_flash_projection_step(void* plan, void* stream);
int rl_flash_projection_destroy(void* plan);

/* Target EMA plans: target = (1 - tau) target + tau source (flash_kernels.cuh:447-497). */
void* rl_flash_ema_create(size_t count, const void* const* source, const void* const* target,
                          const size_t* lengths, float tau);
void* rl_flash_ema_create_with_shadows(size_t count, const void* const* source, const void* const* target,
                                       const size_t* lengths, float tau, const void* const* shadows);
int rl_flash_ema_step(void* plan, void* stream);
int rl_flash_ema_destroy(void* plan);

/* Batch norm over row-major [batch, channels] (flash_kernels.cuh:499-609). Scratch: partial
 * 2 * ceil(batch / 256) * channels floats, sums 2 * channels. Gradients accumulate into
 * dx / dw / db (dx overwritten when overwrite_dx); unused gradient pointers may be null. */
int rl_flash_bn_forward(const float* x, const float* w, const float* b, float* running_mean,
                        float* running_var, float* mean, float* var, float* partial, float* y, int batch,
                        int channels, float eps, float momentum, int training, int relu, void* stream);
int rl_flash_bn_forward_with_fp16(const float* x, const float* w, const float* b, float* running_mean,
                                  float* running_var, float* mean, float* var, float* partial, float* y,
                                  void* half_output, int batch, int channels, float eps, float momentum,
                                  int training, int relu, void* stream);
int rl_flash_bn_backward(const float* x, const float* dy, const float* y, const float* w, const float* mean,
                         const float* var, float* partial, float* sums, float* dx, float* dw, float* db,
                         int batch, int channels, float eps, int training, int relu, void* stream);
int rl_flash_bn_backward_with_fp16(const float* x, const float* dy, const float* y, const float* w,
                                   const float* mean, const float* var, float* partial, float* sums, float* dx,
                                   float* dw, float* db, void* half_dx, int batch, int channels, float eps,
                                   int training, int relu, void* stream);
int rl_flash_bn_backward_controlled(const float* x, const float* dy, const float* y, const float* w,
                                    const float* mean, const float* var, float* partial, float* sums,
                                    float* dx, float* dw, float* db, void* half_dx, int overwrite_dx, int batch,
                                    int channels, float eps, int training, int relu, void* stream);
/* RMS norm over rows (flash_kernels.cuh:611-634). var: batch floats; backward partial
 * ceil(batch / 256) * channels floats. */
int rl_flash_rms_forward(const float* x, const float* w, float* var, float* y, int batch, int channels,
                         float eps, void* stream);
int rl_flash_rms_backward(const float* x, const float* dy, const float* w, const float* var, float* partial,
                          float* dx, float* dw, int batch, int channels, float eps, void* stream);

/* Categorical heads (categorical_kernels.cuh:126-178). backward: scratch ([batch][bins], needed
 * with dbias) holds intermediate sums on return, not the per-row gradients. */
int rl_flash_categorical_forward(const void* raw, const void* bias, const void* support, void* log_probs,
                                 void* values, int batch, int bins, void* stream);
int rl_flash_categorical_backward(const void* log_probs, const void* support, const void* dlog_probs,
                                  const void* dvalues, void* scratch, void* draw, void* dbias, int batch,
                                  int bins, void* stream);
/* q: [2 twins][2 batch] expected values, log_probs: [2][2 batch][bins]; the next half
 * (rows batch..2 batch) of the twin with the smaller next value (ties: twin 0) is projected.
 * maximum_entropy is raised to max(alpha * next_log_probs) (not reset). */
int rl_flash_categorical_target(const void* q, const void* log_probs, const void* reward,
                                const void* terminated, const void* discount, const void* next_log_probs,
                                const void* alpha, void* target, void* maximum_entropy, int batch, int bins,
                                float min_v, float max_v, void* stream);

/* Grouped zeroing of sorted, disjoint fp32 spans (zero_kernels.cuh:53-116). */
void* rl_zero_create(size_t count, const void* const* pointers, const size_t* lengths);
int rl_zero_step(void* plan, void* stream);
int rl_zero_destroy(void* plan);

#ifdef __cplusplus
}
#endif

#endif /* RL_COMPAT_H */
