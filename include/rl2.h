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

#ifdef __cplusplus
}
#endif

#endif /* RL2_H */
