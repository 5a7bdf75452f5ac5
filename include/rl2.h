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
 * operand planes: derived copies that feed the tensor-core products.
 * Either h16 (fp16, multiplied by *scale when scale is set, overflow -> *found_inf = 1)
 * or hi + lo (fp32 pair, hi exact in tf32, hi + lo = value). ld / twin_stride in elements.
 * A GEMM that also writes its fp32 output may take lo alone (hi null): kind::tf32 products
 * ignore the low 13 mantissa bits of their operands, so the fp32 output itself serves as
 * the hi operand of a later product (same layout as the lo plane).
 * ------------------------------------------------------------------------- */
typedef struct rl2_plane {
    void* h16;
    float* hi;
    float* lo;
    long long ld, twin_stride;
    const float* scale;
    int* found_inf;
} rl2_plane;

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
 *         the output, laid out [batch][ceil(m/32)][n] with stat_batch_stride;
 *         stat_m2 == null: stat_mean receives per-group column SUMS instead.
 * k_splits > 1 writes independent partial products to d + s * d_split_stride
 *         (no bias / residual / accumulate / stats), reduced by rl2_split_reduce.
 * out_plane (optional): operand plane copy of the final output (twin_stride per batch).
 * d may be null when out_plane is set (plane-only output).
 * activation (1 = ELU, 2 = tanh; 0 = none), applied last (after bias / residual /
 *         accumulate), before stats and outputs:
 *         act_aux == null: out = f(x)                        (layer forward)
 *         act_aux != null: out = x * f'(y), y = act_aux[z][m][n], the stored
 *                          f outputs (ELU: y > 0 ? 1 : y + 1; tanh: 1 - y^2)
 *         (activation layers of the PPO MLP, warp/ppo.py:313-350).
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
    rl2_plane out_plane;
    int activation;
    const float* act_aux;
    long long ld_aux, aux_batch_stride;
    /* evaluation-mode batch norm of the output columns (optional; transposed plans only,
     * i.e. n >= 128 and a plan-chosen tile): out = (x - mean) * invstd * gamma + beta,
     * then ReLU when bn_relu, then + residual (with bn the residual is added after the
     * normalisation). Per-column arrays [batch][n] at bn_twin_stride; replaces
     * rl_flash_bn_forward in evaluation mode (src/robolearn/cuda/flash_kernels.cuh:500-560). */
    const float* bn_mean;
    const float* bn_invstd;
    const float* bn_gamma;
    const float* bn_beta;
    long long bn_twin_stride;
    int bn_relu;
} rl2_gemm_desc;

void* rl2_gemm_create(const rl2_gemm_desc* desc);
int rl2_gemm_run(void* plan, void* stream);
int rl2_gemm_destroy(void* plan);
/* Tile width chosen by the plan (for tests and tuning reports). */
int rl2_gemm_tile_n(void* plan);
/* Epilogue form of a plan: 2 = transposed accumulator (n >= 128 and a plan-chosen tile
 * width: TMEM lane = output column, direct coalesced row-segment loads and stores);
 * 1 = outputs written by TMA stores (no activation / split-K, a residual only if it is D
 * itself, 16-byte aligned fp32 output and fp16 plane); 0 = register stores. */
int rl2_gemm_uses_tma_store(void* plan);
/* 1 if the plan runs on CTA pairs (fp16 products with at least 512 kernel rows, a
 * contraction of at least 16 k-blocks of 64 and a plan-chosen tile width: clusters of two
 * CTAs computing 256-row tiles with tcgen05 cta_group::2, each CTA staging half of the
 * operands). RL2_GEMM_PAIR=0 disables pairs, RL2_GEMM_PAIR=2 drops the length rule. */
int rl2_gemm_cta_pair(void* plan);

/* out[i] (+)= sum_s partial[s * split_stride + i], fixed order, i < count. */
int rl2_split_reduce(const float* partial, long long split_stride, int splits, float* out, long long count,
                     int accumulate, void* stream);
/* The same for batch independent reductions in one launch: reduction b reads
 * partial + b * in_batch_stride and writes out + b * out_batch_stride (strides in floats,
 * the output stride may be negative). */
int rl2_split_reduce_batched(const float* partial, long long split_stride, int splits, float* out, long long count,
                             int accumulate, int batch, long long in_batch_stride, long long out_batch_stride,
                             void* stream);

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
 * counter holds rl2_categorical_counter_words(batch, bins) zero-initialised unsigned
 * ints that the kernel leaves at zero.
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
int rl2_categorical_counter_words(int batch, int bins);
/* With 16-byte aligned logits and row / twin strides that are multiples of four floats the
 * logits rows are copied into shared memory whole, padding after the last atom included:
 * the full stride of every row read must be allocated. */
int rl2_critic_objective(const rl2_critic_objective_args* args, void* stream);

/* Allocation-free variant of rl2_critic_objective (no counterpart in the reference).
 * For callers that cannot allocate device memory where they run this objective, e.g. a
 * real-time control loop that must not stall in the driver's allocator, or a host whose
 * device memory is owned by another framework's pool. args->workspace and args->counter
 * are ignored: the kernel uses a file-scope device array (about 0.65 MB per GPU, held
 * until process exit). Limits: batch <= 65536, bins <= 128; larger sizes return -1.
 * Every call outside stream capture looks up that array's address in the current
 * driver context; a call during capture reuses the address found by the last such
 * call in the same context, so make one call per device (and again after a
 * cudaDeviceReset or in any other context the host makes current) before capturing.
 * The stream must belong to the current device, or -1 is returned. All calls share
 * the array: calls that overlap on the GPU race, so issue them in order on one
 * stream. Nothing is allocated or freed. */
int rl2_critic_objective_noalloc(const rl2_critic_objective_args* args, void* stream);

/* ---------------------------------------------------------------------------
 * batch norm over the rows of [twins][rows][cols] matrices, training or
 * evaluation mode. Replaces rl_flash_bn_forward / rl_flash_bn_backward and their
 * fp16 variants (src/robolearn/cuda/flash_kernels.cuh:500-609; semantics of
 * src/robolearn/flashsac/layers.py:32-64,189-222: biased variance normalises,
 * running variance uses rows/(rows-1), running buffers move by lerp(momentum)).
 * Column moments travel as per-32-row-group (mean, M2) partials [twins][G][cols],
 * G = ceil(rows / 32), merged in a fixed order (Chan et al.). A twin stride of 0
 * shares one matrix / one set of statistics across the twins.
 * ------------------------------------------------------------------------- */
int rl2_colstats(const float* x, long long ldx, long long x_twin_stride, int twins, int rows, int cols,
                 float* mean_part, float* m2_part, long long part_twin_stride, void* stream);

int rl2_bn_finalize(const float* mean_part, const float* m2_part, long long part_twin_stride, int twins, int rows,
                    int cols, float* mean, float* invstd, float* running_mean, float* running_var, float momentum,
                    float eps, int update_running, void* stream);
/* Partials gathered from several data-parallel ranks: group g of twin t lives at
 * t * part_twin_stride + (g / groups_per_rank) * rank_stride + (g % groups_per_rank) * cols
 * (rank-major blocks as an all-gather leaves them); rows = all ranks' rows. */
int rl2_bn_finalize_ranked(const float* mean_part, const float* m2_part, long long part_twin_stride,
                           int groups_per_rank, long long rank_stride, int twins, int rows, int cols, float* mean,
                           float* invstd, float* running_mean, float* running_var, float momentum, float eps,
                           int update_running, void* stream);

/* eval mode: mean = running_mean, invstd = 1 / sqrt(running_var + eps), count elements */
int rl2_bn_eval_prepare(const float* running_mean, const float* running_var, long long count, float eps,
                        float* mean, float* invstd, void* stream);

typedef struct rl2_bn_apply_args {
    const float* x;
    long long ldx, x_twin_stride;
    int twins, rows, cols;
    const float* mean;   /* [twins][cols] */
    const float* invstd; /* [twins][cols] */
    const float* gamma;  /* [twins][cols] */
    const float* beta;   /* [twins][cols] */
    int relu;
    const float* residual; /* optional, added after the activation */
    long long ldr, residual_twin_stride;
    float* y; /* optional fp32 output */
    long long ldy, y_twin_stride;
    rl2_plane plane; /* optional operand plane of the output */
} rl2_bn_apply_args;

int rl2_bn_apply(const rl2_bn_apply_args* args, void* stream);

typedef struct rl2_bn_backward_args {
    const float* dy; /* gradient w.r.t. the block output after the activation */
    long long lddy, dy_twin_stride;
    const float* x; /* pre-normalisation input */
    long long ldx, x_twin_stride;
    int twins, rows, cols;
    const float* mean;
    const float* invstd;
    const float* gamma;
    const float* beta;
    int relu, training;
    float* s1_part; /* [twins][G][cols] sums of dbn           */
    float* s2_part; /* [twins][G][cols] sums of dbn * xhat    */
    const float* coef1; /* [twins][cols] mean(dbn)   (apply)    */
    const float* coef2; /* [twins][cols] mean(dbn*xhat) (apply) */
    float* dx; /* optional fp32 input gradient */
    long long lddx, dx_twin_stride;
    int sum_twins; /* dx[r][c] = sum over twins (shared input) */
    rl2_plane plane; /* optional operand plane of dx */
} rl2_bn_backward_args;

int rl2_bn_backward_reduce(const rl2_bn_backward_args* args, void* stream);
int rl2_bn_backward_finalize(const float* s1_part, const float* s2_part, int twins, int rows, int cols,
                             float* dgamma, float* dbeta, long long grad_twin_stride, int accumulate, float* coef1,
                             float* coef2, void* stream);
/* Same with gathered partials (layout as rl2_bn_finalize_ranked; part_twin_stride explicit). */
int rl2_bn_backward_finalize_ranked(const float* s1_part, const float* s2_part, long long part_twin_stride,
                                    int groups_per_rank, long long rank_stride, int twins, int rows, int cols,
                                    float* dgamma, float* dbeta, long long dgamma_twin_stride, int accumulate,
                                    float* coef1, float* coef2, void* stream);
int rl2_bn_backward_apply(const rl2_bn_backward_args* args, void* stream);

/* ---------------------------------------------------------------------------
 * RMS post-norm u = h / sqrt(mean(h^2) + eps) * gamma per row. Replaces
 * rl_flash_rms_forward / rl_flash_rms_backward (flash_kernels.cuh:611-634;
 * src/robolearn/flashsac/layers.py:67-81,225-240).
 * ------------------------------------------------------------------------- */
int rl2_rms_forward(const float* h, long long ldh, long long h_twin_stride, int twins, int rows, int cols,
                    const float* gamma, float eps, float* r_out, float* u, long long ldu, long long u_twin_stride,
                    const rl2_plane* plane, void* stream);

/* dh = r * g*du - h * r^3 * sum(g*du*h) / cols; dgamma partials [twins][G][cols] of du*h*r */
int rl2_rms_backward(const float* du, long long lddu, long long du_twin_stride, const float* h, long long ldh,
                     long long h_twin_stride, const float* r, const float* gamma, int twins, int rows, int cols,
                     float* dh, long long lddh, long long dh_twin_stride, float* dgamma_part, void* stream);

/* out[t][c] (+)= sum_g part[t][g][c], fixed order */
int rl2_colsum_finalize(const float* part, int twins, int groups, int cols, float* out, long long out_twin_stride,
                        int accumulate, void* stream);

/* ---------------------------------------------------------------------------
 * tanh-Gaussian policy head (src/robolearn/flashsac/layers.py:116-166; Warp
 * restatement _sample_policy, src/robolearn/warp/flashsac.py:72-95).
 * head rows hold [mean (act) | pre-tanh log-std (act)], biases already added.
 * Sample: actions = tanh(mean + std * noise), log_pi = Gaussian log-density -
 * tanh Jacobian (deterministic: actions = tanh(mean)). Backward: from d_action
 * (rows < grad_rows) and d log pi (array, or one device scalar for rows <
 * grad_rows) to d_head (fp32 and/or operand plane) and per-32-row-group bias
 * partials [G][2*act]; optional behaviour-cloning term bc_alpha * q_abs *
 * mean((a - replay_action)^2) (updates.py:130-134).
 * ------------------------------------------------------------------------- */
typedef struct rl2_policy_args {
    const float* head;
    long long ld_head;
    const float* noise;
    long long ld_noise;
    int rows, act;
    float* actions;
    long long ld_actions;
    float* log_pi;
    /* backward */
    int grad_rows;
    const float* d_action;
    long long ld_d_action;
    const float* d_log_pi;
    const float* d_log_pi_value;
    float bc_alpha;
    const float* q_abs;
    const float* replay_action;
    long long ld_replay_action;
    float* d_head;
    long long ld_d_head;
    rl2_plane d_plane;
    float* bias_part;
} rl2_policy_args;

/* Replaces the actor-phase Warp kernels _sample_policy / _first_actions (warp/flashsac.py:72-102). */
int rl2_policy_sample(const rl2_policy_args* args, int deterministic, void* stream);
int rl2_policy_backward(const rl2_policy_args* args, void* stream);

/* ---------------------------------------------------------------------------
 * actor objective over the frozen critic (updates.py:117-137; Warp
 * _actor_objective / _actor_diagnostics, warp/flashsac.py:105-153): per row the
 * twins' log-softmax and expected value, q = min(q0, q1), loss = mean(alpha *
 * log_pi - q) (+ bc term), entropy = -mean(log_pi), mean_action, q_abs; the
 * logits gradient of -q/B goes to d_logits (plane, twin_stride per twin) and
 * d log pi = alpha / B to *d_log_pi_out.
 * ------------------------------------------------------------------------- */
typedef struct rl2_actor_objective_args {
    const float* logits;
    long long logits_row_stride, logits_twin_stride;
    const float* support;
    int bins, batch, act;
    const float* log_pi;
    const float* actions;
    long long actions_row_stride;
    const float* replay_action;
    long long replay_row_stride;
    float bc_alpha;
    const float* alpha;
    rl2_plane d_logits;
    float* workspace;
    unsigned* counter;
    float* loss_out;
    float* entropy_out;
    float* mean_action_out;
    float* q_abs_out;
    float* d_log_pi_out;
} rl2_actor_objective_args;

int rl2_actor_objective_workspace_floats(int batch);
int rl2_actor_objective(const rl2_actor_objective_args* args, void* stream);

/* ---------------------------------------------------------------------------
 * temperature (updates.py:297-326): loss = exp(log_temp) * (entropy - target),
 * one torch-formula Adam step on log_temp with the warmup-cosine schedule
 * (_utils/scheduler.py:43-65); adam_state = [step, m, v]. alpha_out receives
 * exp(log_temp) after the step (or without a step when update = 0).
 * ------------------------------------------------------------------------- */
typedef struct rl2_temperature_args {
    float* log_temp;
    const float* entropy;
    float target_entropy;
    float* adam_state;
    float beta1, beta2, eps;
    double lr_init, lr_peak, lr_end, warmup_steps, decay_steps;
    int update;
    float* value_out;
    float* loss_out;
    float* alpha_out;
} rl2_temperature_args;

int rl2_temperature_step(const rl2_temperature_args* args, void* stream);

/* ---------------------------------------------------------------------------
 * fused optimizer pass over one network's flat parameter arena: Adam (+ AMP
 * skip) -> weight-norm projection -> operand-plane refresh -> target EMA.
 * Replaces rl_adam_create / rl_adam_step / rl_adam_set_scaler / rl_adam_unscale
 * (src/robolearn/cuda/kernels.cu:760-907), rl_flash_projection_* and
 * rl_flash_ema_* (src/robolearn/cuda/flash_kernels.cuh:383-498) and the fp16
 * weight casts rl_cast_f32_f16 (kernels.cu:663-687).
 *
 * One segment = one projection unit, processed by one warp or one CTA (warp_segments):
 *   kind 0 plain vector (no projection: head / policy biases),
 *   kind 1 unit-linear weight row -> w / max(||w||, 1e-8),
 *   kind 2 BN (weight at offset, bias at offset2) -> both * sqrt(C)/sqrt(sum(w^2+b^2)+1e-8),
 *   kind 3 RMS scale -> w * sqrt(C)/sqrt(sum(w^2)+1e-8).
 * length <= rl2_segment_max_length() per vector (rl2_segment_warp_max_length() for the
 * leading warp_segments units). Units whose offsets and length are multiples of four
 * floats move in 16-byte vectors. plane_offset >= 0 refreshes the
 * row's operand copy in weight_plane (and target_plane for the EMA target).
 * formula 0 = torch Adam (lr/bc1 * m / (sqrt(v)/sqrt(bc2) + eps)),
 * formula 1 = Warp-NN Adam (lr * m c1 / (sqrt(v c2) + eps)).
 * ------------------------------------------------------------------------- */
typedef struct rl2_segment {
    long long offset;
    long long offset2;
    long long plane_offset;
    int length;
    int kind;
} rl2_segment;

/* state: 9 floats per optimizer [attempts, steps, step_size, bc2, lr, skip, scale, growth, skipped].
 * Schedules the learning rate (warmup-cosine over attempts or steps, or *lr_override),
 * advances the step unless *found_inf is set (then skip), updates the dynamic loss
 * scale when scaler = 1, and clears *found_inf. */
typedef struct rl2_adam_prepare_args {
    float* state;
    int* found_inf;
    int formula;
    float beta1, beta2;
    double lr_init, lr_peak, lr_end, warmup_steps, decay_steps;
    int schedule_on_attempts;
    const float* lr_override;
    int scaler;
    float growth, backoff;
    int growth_interval;
    float* scale_out;
    float* inv_scale_out;
} rl2_adam_prepare_args;

typedef struct rl2_adam_args {
    float* params;
    const float* grads; /* null: projection / EMA only */
    float* m;
    float* v;
    const rl2_segment* segments; /* device array */
    int count;
    const float* state;
    int formula;
    float beta1, beta2, eps;
    int project;
    rl2_plane weight_plane;
    float* target_params;
    float tau;
    rl2_plane target_plane;
    int warp_segments; /* the leading units, each <= rl2_segment_warp_max_length(), take one
                          warp each (eight per CTA); the rest one CTA each. 0: a CTA per unit */
} rl2_adam_args;

int rl2_adam_prepare(const rl2_adam_prepare_args* args, void* stream);
int rl2_adam_step(const rl2_adam_args* args, void* stream);
int rl2_segment_max_length(void);
int rl2_segment_warp_max_length(void);

/* ---------------------------------------------------------------------------
 * replay sampling and gather. Replaces the Warp kernels _sample_indices and
 * _gather_batch (src/robolearn/warp/_flash_replay.py:116-160) and the batch
 * assembly kernels _actor_observations / _critic_inputs (warp/flashsac.py:53-69,
 * 166-182); Torch counterpart TorchUniformBuffer.sample (flashsac/replay.py:179-194).
 *
 * rl2_replay_sample: indices[i] uniform in [0, n) by Warp's unbiased rejection
 * rule, n = *population (device int64) or fixed_population, random words from
 * Philox4x32-10 with key = seed and counter = (i, *epoch, round, stream).
 * rl2_counter_advance adds `by` to a device epoch counter (graph-capturable).
 * rl2_replay_gather copies rows bit-exactly into the network layouts and the
 * optional raw batch arrays; with g_var set, reward_out = r / max(sqrt(g_var +
 * norm_eps), g_r_max / g_max) (_utils/reward_normalization.py:28-38).
 * ------------------------------------------------------------------------- */
int rl2_replay_sample(unsigned long long seed, const unsigned long long* epoch, const long long* population,
                      long long fixed_population, int batch, int* indices, int* health, void* stream);
int rl2_counter_advance(unsigned long long* epoch, unsigned long long by, void* stream);

typedef struct rl2_replay_gather_args {
    const int* indices;
    int batch;
    const float* obs;
    const float* next_obs;
    long long ld_obs;
    const float* action;
    long long ld_action;
    const float* reward;
    const float* terminated;
    const float* truncated;
    const float* discount;
    int obs_dim, act_dim, actor_obs_dim;
    float* critic_x; /* [2B][ld_critic_x]: rows i = [obs | action], rows B+i = [next_obs | .] */
    long long ld_critic_x;
    float* actor_x; /* [2B][ld_actor_x]: rows i = obs prefix, rows B+i = next_obs prefix */
    long long ld_actor_x;
    float* reward_out;
    float* terminated_out;
    float* truncated_out;
    float* discount_out;
    const float* g_var;
    const float* g_r_max;
    float g_max, norm_eps;
    float* batch_obs;
    float* batch_next_obs;
    float* batch_action;
    float* batch_reward;
    float* critic_x_pi; /* [B][ld_critic_x_pi]: obs rows for the actor-phase critic input */
    long long ld_critic_x_pi;
} rl2_replay_gather_args;

int rl2_replay_gather(const rl2_replay_gather_args* args, void* stream);

/* Standard normal policy noise (Box-Muller over Philox4x32-10 words; replaces the Warp
 * _normal_noise kernel, src/robolearn/warp/flashsac.py:44-50): out[r][c], r < rows, c < cols. */
int rl2_normal_noise(unsigned long long seed, const unsigned long long* epoch, int rows, int cols, float* out,
                     long long ld, void* stream);
/* Rows row0 .. row0 + rows - 1 of the same stream (data-parallel ranks draw their slice of
 * the global noise array; bit-identical to the matching rows of one full launch). */
int rl2_normal_noise_rows(unsigned long long seed, const unsigned long long* epoch, long long row0, int rows,
                          int cols, float* out, long long ld, void* stream);

/* ---------------------------------------------------------------------------
 * replay ingest (one vector-environment step): stage the step in an n-step
 * ring, then commit the n-step transition that began n-1 steps ago into the
 * replay ring at (write position + env) % capacity. Replaces _copy_pending /
 * _commit_pending / _advance_replay (src/robolearn/warp/_flash_replay.py:26-113);
 * Torch semantics TorchUniformBuffer.add (src/robolearn/flashsac/replay.py:109-174):
 * a done (terminated or truncated) step ends the return, keeps its own next
 * observation and flags, discount = gamma^(steps included).
 * counters (device int64): [0] steps seen, [1] write position, [2] filled rows.
 * Done flags are fp32 (0/1) or uint8 (bool), whichever pointer is set.
 * ------------------------------------------------------------------------- */
typedef struct rl2_replay_ingest_args {
    const float* obs;
    const float* next_obs;
    long long ld_obs;
    const float* action;
    long long ld_action;
    const float* reward;
    const float* terminated;
    const float* truncated;
    const unsigned char* terminated_u8;
    const unsigned char* truncated_u8;
    long long num_envs;
    int obs_dim, act_dim, n_step;
    float gamma;
    float* pend_obs;      /* [n_step][num_envs][obs_dim] */
    float* pend_next_obs; /* [n_step][num_envs][obs_dim] */
    float* pend_act;      /* [n_step][num_envs][act_dim] */
    float* pend_reward;   /* [n_step][num_envs] */
    float* pend_term;
    float* pend_trunc;
    long long* counters;
    long long capacity;
    float* r_obs;
    float* r_next_obs;
    long long ld_replay_obs;
    float* r_act;
    long long ld_replay_act;
    float* r_reward;
    float* r_term;
    float* r_trunc;
    float* r_discount;
} rl2_replay_ingest_args;

int rl2_replay_ingest(const rl2_replay_ingest_args* args, void* stream);

/* Reward normaliser statistics for one environment step (replaces _update_returns /
 * _return_variance / _update_running_moments, src/robolearn/warp/_flash_replay.py:347-389;
 * Torch semantics src/robolearn/flashsac/_utils/reward_normalization.py:14-125):
 * g_r = gamma * (1 - done) * g_r + r per environment; state = [mean, var, count, G_r_max]
 * updated from the batch moments of g_r by Chan's rule with count epsilon. */
int rl2_reward_stats_update(const float* reward, const float* terminated, const float* truncated,
                            const unsigned char* terminated_u8, const unsigned char* truncated_u8, float* g_r,
                            int num_envs, float gamma, float* state, float epsilon, void* stream);

/* Host-side Philox4x32-10 block (for checking device streams against the published algorithm). */
void rl2_philox4x32(unsigned int c0, unsigned int c1, unsigned int c2, unsigned int c3, unsigned int k0,
                    unsigned int k1, unsigned int* out4);

/* ---------------------------------------------------------------------------
 * PPO learner update (replaces the Warp kernels of src/robolearn/warp/ppo.py).
 * Rollout index k = t * num_envs + i; flags are int32 (0 / nonzero).
 * ------------------------------------------------------------------------- */

/* GAE (_gae, ppo.py:101-133) as a warp-shuffle reverse scan: each environment's
 * horizon is split into up to 32 segments held by neighbouring lanes; every lane
 * composes its segment's affine map A -> delta + g A, the maps are combined by a
 * reverse shuffle scan, and each lane re-runs its segment from the exact carry-in. */
typedef struct rl2_ppo_gae_args {
    const float* rewards;
    const float* values;
    const float* next_values;
    const int* terminated;
    const int* truncated;
    int horizon, num_envs;
    float gamma, gae_lambda;
    int current_timeout_bootstrap; /* timeout_bootstrap == "current": V' = V(s_t) on truncation */
    float* advantages;
    float* returns;
} rl2_ppo_gae_args;

int rl2_ppo_gae(const rl2_ppo_gae_args* args, void* stream);

/* Advantage normalisation (_advantage_sum / _advantage_variance / _normalize,
 * ppo.py:136-159): two-pass mean and centred variance accumulated in double in a
 * fixed order; population (eps inside the sqrt) or sample (n - 1, eps outside).
 * stats: 2 doubles of workspace [sum, centred sum of squares]; counter: one int that
 * must start at zero (left at zero). */
int rl2_ppo_normalize_advantages(float* advantages, int n, int sample_std, double* stats, double* partials,
                                 int* counter, void* stream);
/* doubles of partials needed for n elements */
int rl2_ppo_partials(int n);

/* Minibatch permutation (replaces _shuffle_keys + radix_sort_pairs, ppo.py:162-169,
 * 603): indices[i] = pi(i) for a keyed Feistel bijection of [0, n) (cycle walking on
 * the enclosing power-of-four domain), keys from Philox4x32-10(seed, *epoch). */
int rl2_ppo_permutation(unsigned long long seed, const unsigned long long* epoch, int n, int* indices,
                        int* health, void* stream);

/* Minibatch gather (_gather_batch, ppo.py:172-204): row r of the batch is rollout row
 * indices[offset + r]; observations go straight into the first layer's operand plane.
 * Each batch_* output is optional (null: not copied). */
typedef struct rl2_ppo_gather_args {
    const int* indices; /* null: identity */
    int offset, rows, obs_dim, act_dim;
    const float* observations;
    const float* actions;
    const float* means;
    const float* stds;
    const float* log_probs;
    const float* values;
    const float* advantages;
    const float* returns;
    rl2_plane obs_plane;
    float* batch_actions;
    float* batch_means;
    float* batch_stds;
    float* batch_log_probs;
    float* batch_values;
    float* batch_advantages;
    float* batch_returns;
} rl2_ppo_gather_args;

int rl2_ppo_gather(const rl2_ppo_gather_args* args, void* stream);

/* Fused clipped-surrogate / value / entropy loss and its gradient (_make_ppo_loss,
 * ppo.py:255-310, with Warp's adjoint rules for min / max / clamp). head[0] holds the
 * actor means (columns 0..act-1), head[1] the critic value in column 0 (twin stride
 * head_twin_stride). Writes loss (1 float), metrics [policy, value, entropy] (means),
 * d_head (fp32 and/or operand plane; other columns of the critic twin zero), the
 * head bias gradients d_bias_actor [act] and d_bias_critic [1], and d_std_param [act].
 * std_type 0 = log std, 1 = scalar std clamped to [std_min, std_max]. Deterministic:
 * per-block partials reduced in a fixed order by the last block. */
typedef struct rl2_ppo_loss_args {
    const float* head;
    long long ld_head, head_twin_stride;
    const float* std_param;
    int rows, act;
    const float* actions;
    const float* old_log_probs;
    const float* old_values;
    const float* advantages;
    const float* returns;
    float clip_ratio, value_coefficient, entropy_coefficient, value_loss_scale;
    int clip_value, std_type;
    float std_min, std_max;
    float* loss;
    float* metrics;
    float* d_head;
    long long ld_d_head, d_head_twin_stride;
    rl2_plane d_plane;
    float* d_bias_actor;
    float* d_bias_critic;
    float* d_std_param;
    double* partials; /* rl2_ppo_loss_partials(rows, act) doubles */
    int* counter;    /* one int, zero on entry, left at zero */
} rl2_ppo_loss_args;

int rl2_ppo_loss(const rl2_ppo_loss_args* args, void* stream);
int rl2_ppo_loss_partials(int rows, int act);

/* KL(old || new) mean and adaptive learning rate (_make_kl_kernel / _adapt_learning_rate,
 * ppo.py:207-238): lr /= 1.5 (>= 1e-5) when kl > 2 desired_kl, lr *= 1.5 (<= 1e-2) when
 * 0 < kl < desired_kl / 2. partials: rl2_ppo_partials(rows) doubles. */
int rl2_ppo_kl(const float* mean, long long ld_mean, const float* std_param, const float* old_means,
               const float* old_stds, int rows, int act, int std_type, float std_min, float std_max,
               float desired_kl, float* kl, float* learning_rate, double* partials, int* counter, void* stream);

/* Gradient-norm clipping over the flat gradient arena laid out [actor | critic | std]
 * (ppo.py:241-252 and the optimizer's max_norm): separate = 0 clips all gradients by
 * one total norm, 1 clips (actor + std) and critic separately; coefficient =
 * min(1, max_norm / (sqrt(sum g^2) + 1e-6)). norms_out (5 floats) receives the sums of
 * squares [actor + std, critic, total] and the applied coefficients [actor + std, critic].
 * partials: 3 * rl2_ppo_partials(n) doubles. */
int rl2_ppo_clip_gradients(float* grads, long long actor_count, long long critic_count, long long std_count,
                           int separate, float max_norm, float* norms_out, double* partials, int* counter,
                           void* stream);

/* Rollout-side kernels (_sample / _store, ppo.py:26-98). head[0] = actor means,
 * head[1] column 0 = critic values (twin stride head_twin_stride). noise: standard
 * normal [rows][act] or null (deterministic). sampled_std receives the action std. */
typedef struct rl2_ppo_sample_args {
    const float* head;
    long long ld_head, head_twin_stride;
    const float* std_param;
    int std_type;
    float std_min, std_max;
    const float* noise;
    int rows, act;
    float* actions;
    float* log_probs;
    float* values;
    float* sampled_std;
} rl2_ppo_sample_args;

int rl2_ppo_sample(const rl2_ppo_sample_args* args, void* stream);

/* Store rollout step `step` (rows k = step * num_envs + i): observations, the last sampled
 * actions / log probs / values / means / std, rewards, flags and the next-state values
 * (critic column of next_head). */
typedef struct rl2_ppo_store_args {
    int step, num_envs, obs_dim, act;
    const float* observations;
    const float* actions;
    const float* log_probs;
    const float* values;
    const float* rewards;
    const int* terminated;
    const int* truncated;
    const float* mean;
    long long ld_mean;
    const float* next_values;
    long long next_values_stride;
    const float* sampled_std;
    float* r_observations;
    float* r_actions;
    float* r_log_probs;
    float* r_values;
    float* r_rewards;
    int* r_terminated;
    int* r_truncated;
    float* r_next_values;
    float* r_means;
    float* r_stds;
} rl2_ppo_store_args;

int rl2_ppo_store(const rl2_ppo_store_args* args, void* stream);

/* ---------------------------------------------------------------------------
 * Data-parallel batch-norm statistics over NVLink peer memory (one kernel per BN
 * layer, no collective library call). Replaces, for the data-parallel learner, the
 * all-gather + merge of per-group partials; the reference has no multi-GPU path
 * (its SyncBN design is the build's own, following the global-batch semantics of
 * src/robolearn/flashsac/layers.py:32-64 / updates.py:226-230).
 *
 * Every rank first merges its own per-32-row-group partials ([part_twins][G][cols],
 * twin stride part_twin_stride; part_twins = 1 shares one set across the twins) into one
 * entry per column, pushes the entry into every rank's exchange slot (plain stores
 * through peer pointers), raises a per-(column slab, rank) flag with the slot's epoch on
 * every rank, waits (bounded: timeout_s, then kHealthTimeout in *health) for all ranks'
 * flags of its slab and merges the ranks' entries in rank order: bit-identical results
 * on every rank. Epochs advance on the device (graph-capturable).
 *
 * Exchange slot layout (every rank): data [world][twins][2][cols] floats at
 * peer_data[r]; flags [twins * ceil(cols / 32)][world] u64 at peer_flags[r]; epoch[2]
 * (use counter, block ticket) local, zero-initialised. rows = this rank's rows.
 * ------------------------------------------------------------------------- */
typedef struct rl2_syncbn_exchange {
    float* const* peer_data;               /* device array [world] */
    unsigned long long* const* peer_flags; /* device array [world] */
    unsigned int* epoch;                   /* 2 words, this rank */
    int world, rank;
    int* health;
    float timeout_s;
} rl2_syncbn_exchange;

/* Forward: global mean / invstd (and running statistics, unbiased by world * rows). */
int rl2_syncbn_forward(const float* mean_part, const float* m2_part, long long part_twin_stride, int part_twins,
                       int twins, int rows, int cols, float* mean, float* invstd, float* running_mean,
                       float* running_var, float momentum, float eps, int update_running,
                       const rl2_syncbn_exchange* ex, void* stream);

/* Backward: dgamma / dbeta from this rank's rows (optional), coef1 / coef2 from the
 * global sums (sum over all ranks' rows / (world * rows)). */
int rl2_syncbn_backward(const float* s1_part, const float* s2_part, long long part_twin_stride, int twins, int rows,
                        int cols, float* dgamma, float* dbeta, long long dgamma_twin_stride, float* coef1,
                        float* coef2, const rl2_syncbn_exchange* ex, void* stream);

/* Bytes of one exchange slot's data and flag regions for (world, twins, cols). */
long long rl2_syncbn_slot_data_bytes(int world, int twins, int cols);
long long rl2_syncbn_slot_flag_bytes(int world, int twins, int cols);

/* Small all-reduce of the learner's scalars over the same peer slots (one warp; a slot
 * sized for twins = 1, cols = 32): mean[0 .. n_mean) averaged over the ranks (sum in
 * rank order / world), then max[0 .. n_max) and the flags max_int[0 .. n_max_int)
 * replaced by their maxima (max results written after the means, so max may point into
 * mean). n_mean + n_max + n_max_int <= 64. Replaces the entropy average before the
 * temperature step (src/robolearn/flashsac/updates.py), the overflow-flag maximum before
 * each optimizer step and the reported-metrics reductions of data-parallel updates. */
typedef struct rl2_peer_reduce_args {
    float* mean;
    int n_mean;
    float* max;
    int n_max;
    int* max_int;
    int n_max_int;
} rl2_peer_reduce_args;

int rl2_peer_reduce(const rl2_peer_reduce_args* args, const rl2_syncbn_exchange* ex, void* stream);

/* Mean over the ranks of a float arena held in symmetric memory, in place on every rank
 * (the data-parallel gradient average before each optimizer step: every rank then steps
 * on the global batch's gradient, src/robolearn/flashsac/updates.py). ex->peer_data[q] =
 * rank q's arena (16-byte aligned, the same count on every rank), ex->peer_flags[q] =
 * rank q's flag region of this call site (rl2_peer_mean_flag_bytes(world) bytes, zeroed
 * once), ex->epoch = this call site's two-word counter. One kernel of 148 blocks that must
 * all be resident: launch it on a stream with no other waiting kernel beside it. Each rank
 * averages 1/world of the arena (sum in rank order / world) and stores it into every
 * rank's arena, so the ranks hold bit-identical results. A wait on a peer that runs out
 * (ex->timeout_s) records the timeout in ex->health and leaves the arena partly averaged.
 * count: floats, a multiple of 4. Replaces an NCCL all-reduce (AVG) of the arena. */
long long rl2_peer_mean_flag_bytes(int world);
int rl2_peer_mean(long long count, const rl2_syncbn_exchange* ex, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* RL2_H */
