/*
 * librl2 — B200 (sm_100a) learner-update kernels behind a plain C ABI.
 *
 * Conventions (kept from the reference's native library, src/robolearn/cuda/kernels.cu:4-49):
 *  - every run entry point takes caller-owned device pointers and a cudaStream_t
 *    passed as void*, enqueues work on that stream, allocates nothing and does
 *    not synchronise;
 *  - status is 0 on success and -1 on a synchronous error; the message is read
 *    with rl2_last_error() (thread-local). Asynchronous device errors surface
 *    at the caller's synchronisation point;
 *  - plan create/destroy calls may allocate and must run outside CUDA graph
 *    capture; plans are tied to the current device and are not thread-safe;
 *  - device waits inside kernels are bounded: a wait that times out sets a bit
 *    in the caller's int "health" word (1 = timeout, 2 = non-finite value,
 *    4 = fp16 operand overflow) instead of hanging.
 *
 * All floating-point buffers are fp32 unless a parameter says fp16.
 */
#ifndef RL2_H
#define RL2_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------------------------------------------------------------------
 * library
 * ------------------------------------------------------------------------- */

/* Replaces rl_last_error (src/robolearn/cuda/kernels.cu:408). */
const char* rl2_last_error(void);

/* ABI version of this library (no reference counterpart; used by the loader). */
int rl2_abi_version(void);

/* ---------------------------------------------------------------------------
 * dense products (tcgen05 + TMA). Replaces the cuBLASLt dense plans
 * rl_plan_create / rl_plan_create_mixed / rl_plan_run / rl_plan_destroy
 * (src/robolearn/cuda/kernels.cu:410-731, driven by src/robolearn/cuda/linear.py:155-375)
 * and rl_bias_grad (kernels.cu:742-758; bias gradients come from the head kernels).
 *
 * D[z][m][n] = scale * sum_k A[z][m][k] B[z][n][k] (+ bias[z][n]) (+ residual[z][m][n]) (+ D[z][m][n] if accumulate)
 * a_major / b_major: 0 = K contiguous (row stride lda over m / ldb over n),
 *                    1 = M (or N) contiguous (row stride lda / ldb over k).
 * kind 0: fp16 operands; kind 1: fp32 operands given as tf32 hi/lo planes
 *         (a_lo, b_lo), three tensor-core products per step.
 * Batch strides are in elements; 0 shares the operand across the batch.
 * stat_mean / stat_m2 (optional): per-column moments of each 32-row group of
 *         the output, laid out [batch][ceil(m/32)][n] with stat_batch_stride.
 * k_splits > 1 writes independent partial products to d + s * d_split_stride
 *         (no bias / residual / accumulate / stats), reduced by rl2_split_reduce.
 * ------------------------------------------------------------------------- */
typedef struct rl2_gemm_desc {
    int kind;
    int m, n, k, batch;
    const void* a;
    const void* a_lo;
    int a_major;
    long long lda, a_batch_stride;
    const void* b;
    const void* b_lo;
    int b_major;
    long long ldb, b_batch_stride;
    float* d;
    long long ldd, d_batch_stride;
    int accumulate;
    const float* bias;
    long long bias_batch_stride;
    const float* residual;
    long long ldr, residual_batch_stride;
    float* stat_mean;
    float* stat_m2;
    long long stat_batch_stride;
    const float* scale;
    int k_splits;
    long long d_split_stride;
    int tile_n;
    int* health;
} rl2_gemm_desc;

void* rl2_gemm_create(const rl2_gemm_desc* desc);
int rl2_gemm_run(void* plan, void* stream);
int rl2_gemm_destroy(void* plan);
/* Tile width chosen by the plan (for tests and tuning reports). */
int rl2_gemm_tile_n(void* plan);

/* out[i] (+)= sum_s partial[s * split_stride + i], fixed order, i < count. */
int rl2_split_reduce(const float* partial, long long split_stride, int splits, float* out, long long count,
                     int accumulate, void* stream);

/* ---------------------------------------------------------------------------
 * fused categorical critic objective: min-Q twin selection + two-hot Bellman
 * projection onto the atom support + log-softmax cross-entropy + logits
 * gradient + head-bias gradient, one kernel. Replaces rl_flash_categorical_target
 * (src/robolearn/cuda/categorical_kernels.cuh:159-176) together with the
 * rl_flash_categorical_forward/backward pair (:126-157) on the critic-loss path
 * (reference semantics: src/robolearn/flashsac/updates.py:19-80,248-257).
 *
 * Rows: transition i reads target logits at row target_row_offset + i (the
 * next-observation half of the critic batch) and online logits at row i; both
 * carry the head bias already. Twin t lives at +t * *_twin_stride floats.
 * loss_weight multiplies every per-row CE and gradient (1 / (2B) for the mean).
 * min_v / max_v are the support bounds as the caller's doubles; the kernel
 * clamps with their float32 roundings and divides by float32((max-min)/(bins-1)),
 * the conversions Torch applies to the reference's Python scalars.
 * Outputs (each optional): dlogits fp32, d16 fp16 operand scaled by *d16_scale,
 * d_hi/d_lo tf32 operand planes, target_out [B][bins]. loss_out, max_entropy_out
 * (max of alpha * next_log_pi), bias_grad_out [2][bins] are reduced in a fixed
 * order. workspace holds rl2_categorical_workspace_floats(batch, bins) floats;
 * counter is one zero-initialised unsigned int that the kernel leaves at zero.
 * ------------------------------------------------------------------------- */
typedef struct rl2_critic_objective_args {
    const float* target_logits;
    long long target_row_stride, target_twin_stride;
    int target_row_offset;
    const float* online_logits;
    long long online_row_stride, online_twin_stride;
    const float* reward;
    const float* terminated;
    const float* discount;
    const float* next_log_pi;
    const float* alpha;
    const float* support;
    double min_v, max_v;
    int bins, batch;
    float loss_weight;
    float* dlogits;
    long long dlogits_row_stride, dlogits_twin_stride;
    void* d16;
    long long d16_row_stride, d16_twin_stride;
    const float* d16_scale;
    float* d_hi;
    float* d_lo;
    long long dplane_row_stride, dplane_twin_stride;
    float* target_out;
    long long target_out_row_stride;
    float* workspace;
    unsigned* counter;
    float* loss_out;
    float* max_entropy_out;
    float* bias_grad_out;
    int bias_grad_accumulate;
    int* health;
} rl2_critic_objective_args;

int rl2_categorical_workspace_floats(int batch, int bins);
int rl2_critic_objective(const rl2_critic_objective_args* args, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* RL2_H */
