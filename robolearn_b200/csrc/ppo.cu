// PPO learner kernels: GAE, advantage normalisation, minibatch permutation and gather,
// the fused clipped-surrogate / value / entropy loss with its gradient, the KL learning-
// rate schedule and gradient-norm clipping (src/robolearn/warp/ppo.py). The MLP layers
// run on the tcgen05 GEMM (with fused activations) and Adam on the segment optimizer.
//
// Every reduction is deterministic: blocks write partials that the last block to
// finish (atomic ticket) combines in a fixed order, then resets the ticket.

#include "philox.cuh"
#include "planes.cuh"

#include <cmath>

namespace rl2 {
namespace ppo {

constexpr int kT = 256;

// ---------------------------------------------------------------------------
// GAE: segmented warp-shuffle reverse scan over time
// ---------------------------------------------------------------------------
struct Step {
    float delta, g;
};

__device__ __forceinline__ Step gae_step(const rl2_ppo_gae_args& a, long long k, float gl) {
    const bool te = a.terminated[k] != 0;
    const bool tr = a.truncated[k] != 0;
    float boot = te ? 0.0f : 1.0f;
    const float cont = (te || tr) ? 0.0f : 1.0f;
    float nxt = a.next_values[k];
    const float v = a.values[k];
    if (a.current_timeout_bootstrap && tr) {
        nxt = v;
        boot = 1.0f;
    }
    // delta = (r + (gamma * boot) * V') - V; no contraction, as the reference restatement
    const float delta = __fsub_rn(__fadd_rn(a.rewards[k], __fmul_rn(__fmul_rn(a.gamma, boot), nxt)), v);
    return {delta, __fmul_rn(gl, cont)};
}

// Lane layout: S consecutive lanes per environment (S | 32), lane c of a group owns
// times [c L, min((c + 1) L, T)).
__global__ void gae_kernel(const rl2_ppo_gae_args a, int S, int L) {
    const long long tid = static_cast<long long>(blockIdx.x) * kT + threadIdx.x;
    const int lane = threadIdx.x & 31;
    const int c = lane % S;
    const long long env = tid / S;
    const bool live = env < a.num_envs;
    const int N = a.num_envs, T = a.horizon;
    const int t0 = min(c * L, T), t1 = min(t0 + L, T);
    const float gl = __fmul_rn(a.gamma, a.gae_lambda);
    // pass 1: this segment's map A_start = P + Q * A_end
    float P = 0.0f, Q = 1.0f;
    if (live) {
        for (int t = t1 - 1; t >= t0; --t) {
            const Step s = gae_step(a, static_cast<long long>(t) * N + env, gl);
            P = __fadd_rn(s.delta, __fmul_rn(s.g, P));
            Q = __fmul_rn(s.g, Q);
        }
    }
    // inclusive suffix scan of the maps over the group: lane c -> segments c..S-1
    for (int off = 1; off < S; off <<= 1) {
        const float Pn = __shfl_down_sync(0xffffffffu, P, off);
        const float Qn = __shfl_down_sync(0xffffffffu, Q, off);
        if (c + off < S) {
            P = __fadd_rn(P, __fmul_rn(Q, Pn));
            Q = __fmul_rn(Q, Qn);
        }
    }
    // carry-in = A at the start of the next segment (0 past the horizon)
    const float next_start = __shfl_down_sync(0xffffffffu, P, 1);
    float A = (c + 1 < S) ? next_start : 0.0f;
    if (!live) return;
    for (int t = t1 - 1; t >= t0; --t) {
        const long long k = static_cast<long long>(t) * N + env;
        const Step s = gae_step(a, k, gl);
        A = __fadd_rn(s.delta, __fmul_rn(s.g, A));
        a.advantages[k] = A;
        a.returns[k] = __fadd_rn(A, a.values[k]);
    }
}

// ---------------------------------------------------------------------------
// deterministic double sums: per-block partials + last-block combine
// ---------------------------------------------------------------------------
__device__ __forceinline__ double block_sum_d(double v) {
    __shared__ double sh[kT / 32];
    v = warp_sum_d(v);
    const int w = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) sh[w] = v;
    __syncthreads();
    double r = 0.0;
    if (threadIdx.x < 32) {
        r = threadIdx.x < kT / 32 ? sh[threadIdx.x] : 0.0;
        r = warp_sum_d(r);
    }
    __syncthreads();
    return r;  // valid in thread 0
}

// True in every thread of the last block to finish (all partials are then written);
// the ticket is reset for the next launch.
__device__ __forceinline__ bool last_block(int* counter) {
    __shared__ bool is_last;
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        const int ticket = atomicAdd(counter, 1);
        is_last = ticket == static_cast<int>(gridDim.x) - 1;
        if (is_last) *counter = 0;
    }
    __syncthreads();
    return is_last;
}

__device__ __forceinline__ double fixed_order_sum(const double* partials, int count) {
    // thread-strided then tree: a fixed order for a given count; L1 is bypassed because
    // the partials were written by other SMs
    double v = 0.0;
    for (int i = threadIdx.x; i < count; i += kT) v += __ldcg(partials + i);
    return block_sum_d(v);
}

inline int sum_blocks(long long n) {
    const long long b = (n + kT - 1) / kT;
    return static_cast<int>(b < 1024 ? (b < 1 ? 1 : b) : 1024);
}

// mode 0: stats[0] = sum x; mode 1: stats[1] = sum (x - mean)^2 with mean = stats[0] / n
__global__ void adv_moment_kernel(const float* __restrict__ x, int n, int mode, double* stats, double* partials,
                                  int* counter) {
    const double mean = mode ? __ldcg(stats) / n : 0.0;
    double v = 0.0;
    for (long long i = static_cast<long long>(blockIdx.x) * kT + threadIdx.x; i < n;
         i += static_cast<long long>(gridDim.x) * kT) {
        const double d = static_cast<double>(x[i]) - mean;
        v += mode ? d * d : d;
    }
    v = block_sum_d(v);
    if (threadIdx.x == 0) partials[blockIdx.x] = v;
    if (last_block(counter)) {
        const double s = fixed_order_sum(partials, gridDim.x);
        if (threadIdx.x == 0) stats[mode] = s;
    }
}

__global__ void adv_normalize_kernel(float* __restrict__ x, int n, int sample_std, const double* stats) {
    const double nn = static_cast<double>(n);
    const double mean = stats[0] / nn;
    const double denom = sample_std ? sqrt(stats[1] / (nn - 1.0 > 1.0 ? nn - 1.0 : 1.0)) + 1.0e-8
                                    : sqrt(stats[1] / nn + 1.0e-8);
    for (long long i = static_cast<long long>(blockIdx.x) * kT + threadIdx.x; i < n;
         i += static_cast<long long>(gridDim.x) * kT)
        x[i] = static_cast<float>((static_cast<double>(x[i]) - mean) / denom);
}

// ---------------------------------------------------------------------------
// minibatch permutation: keyed Feistel network + cycle walking
// ---------------------------------------------------------------------------
// 32-bit integer mix "lowbias32" (C. Wellons, hash-prospector, public domain).
__device__ __forceinline__ uint32_t mix32(uint32_t x) {
    x ^= x >> 16;
    x *= 0x7feb352du;
    x ^= x >> 15;
    x *= 0x846ca68bu;
    x ^= x >> 16;
    return x;
}

// Four-round balanced Feistel permutation of [0, 4^half).
__device__ __forceinline__ uint32_t feistel(uint32_t x, int half, const uint32_t (&key)[4]) {
    const uint32_t mask = (1u << half) - 1u;
    uint32_t l = x >> half, r = x & mask;
#pragma unroll
    for (int round = 0; round < 4; ++round) {
        const uint32_t f = mix32(r ^ key[round]) & mask;
        const uint32_t nl = r;
        r = l ^ f;
        l = nl;
    }
    return (l << half) | r;
}

__global__ void permutation_kernel(uint64_t seed, const unsigned long long* epoch, int n, int half, int* out,
                                   int* fail) {
    const int i = blockIdx.x * kT + threadIdx.x;
    if (i >= n) return;
    const unsigned long long e = epoch ? *epoch : 0ull;
    const U4 k = philox(U4{static_cast<uint32_t>(e), static_cast<uint32_t>(e >> 32), 0x50504Fu, 0x5EEDu},
                        static_cast<uint32_t>(seed), static_cast<uint32_t>(seed >> 32));
    const uint32_t key[4] = {k.x, k.y, k.z, k.w};
    const uint32_t domain = 1u << (2 * half);
    uint32_t x = static_cast<uint32_t>(i);
    // cycle walking: the first image below n along i's cycle; the cycle through i holds
    // at most `domain` points, so the walk is bounded.
    for (uint32_t step = 0; step < domain; ++step) {
        x = feistel(x, half, key);
        if (x < static_cast<uint32_t>(n)) {
            out[i] = static_cast<int>(x);
            return;
        }
    }
    out[i] = i;  // unreachable for a bijection; reported instead of looping further
    atomicOr(fail, 1);
}

// ---------------------------------------------------------------------------
// minibatch gather (one warp per row)
// ---------------------------------------------------------------------------
__global__ void gather_kernel(const rl2_ppo_gather_args a, const Plane obs_plane) {
    const int warp = (blockIdx.x * kT + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (warp >= a.rows) return;
    const int r = warp;
    const long long src = a.indices ? a.indices[a.offset + r] : a.offset + r;
    PlaneWriter pw(obs_plane);
    for (int j = lane; j < a.obs_dim; j += 32) pw.store(0, r, j, a.observations[src * a.obs_dim + j]);
    for (int j = lane; j < a.act_dim; j += 32) {
        const long long s = src * a.act_dim + j, d = static_cast<long long>(r) * a.act_dim + j;
        if (a.batch_actions) a.batch_actions[d] = a.actions[s];
        if (a.batch_means) a.batch_means[d] = a.means[s];
        if (a.batch_stds) a.batch_stds[d] = a.stds[s];
    }
    if (lane == 0) {
        if (a.batch_log_probs) a.batch_log_probs[r] = a.log_probs[src];
        if (a.batch_values) a.batch_values[r] = a.values[src];
        if (a.batch_advantages) a.batch_advantages[r] = a.advantages[src];
        if (a.batch_returns) a.batch_returns[r] = a.returns[src];
    }
    pw.flush();
}

// ---------------------------------------------------------------------------
// fused PPO loss + gradient (one thread per minibatch row)
// ---------------------------------------------------------------------------
constexpr int kMaxAct = 64;
constexpr float kLog2Pi = 1.8378770664093453f;
constexpr float kHalfLog2PiE = 1.4189385332046727f;

// partial slots per block: [loss, policy, value, entropy, d_bias_critic, d_s[act], d_bias_actor[act]]
__host__ __device__ constexpr int loss_slots(int act) { return 5 + 2 * act; }

__device__ __forceinline__ float action_log_std(const rl2_ppo_loss_args& a, int j) {
    const float p = a.std_param[j];
    return a.std_type ? logf(fminf(fmaxf(p, a.std_min), a.std_max)) : p;
}

// MAXA: compile-time bound on the action count (16, or kMaxAct), so the per-action arrays
// are indexed statically and stay in registers; the arithmetic and its order do not
// depend on it.
template <int MAXA>
__global__ void loss_kernel(const rl2_ppo_loss_args a, const Plane dplane) {
    __shared__ double sh[kT / 32][loss_slots(kMaxAct)];
    const int row = blockIdx.x * kT + threadIdx.x;
    const int A = a.act;
    const int nslot = loss_slots(A);
    const bool live = row < a.rows;
    const float sc = 1.0f / static_cast<float>(a.rows);
    const float eps = a.clip_ratio;
    float vals[5] = {0.f, 0.f, 0.f, 0.f, 0.f};
    float ds[MAXA], dm[MAXA];
#pragma unroll
    for (int j = 0; j < MAXA; ++j) ds[j] = dm[j] = 0.0f;
    PlaneWriter pw(dplane);
    if (live) {
        const float* mean = a.head + static_cast<long long>(row) * a.ld_head;
        const float value = a.head[a.head_twin_stride + static_cast<long long>(row) * a.ld_head];
        const float* act = a.actions + static_cast<long long>(row) * A;
        float logp = 0.0f, entropy = 0.0f;
        float r[MAXA];
#pragma unroll
        for (int j = 0; j < MAXA; ++j) {
            r[j] = 0.0f;
            if (j < A) {
                const float s = action_log_std(a, j);
                r[j] = (act[j] - mean[j]) * expf(-s);
                logp = logp - 0.5f * (r[j] * r[j] + 2.0f * s + kLog2Pi);
                entropy = entropy + s + kHalfLog2PiE;
            }
        }
        const float adv = a.advantages[row];
        const float ratio = expf(logp - a.old_log_probs[row]);
        const float ua = ratio * adv;
        const float ca = fminf(fmaxf(ratio, 1.0f - eps), 1.0f + eps) * adv;
        const bool first = ua < ca;  // min(a, b): the first argument only when strictly smaller
        const float policy = -(first ? ua : ca);
        const float ret = a.returns[row];
        const float err = value - ret;
        float vloss = err * err;
        float dv = 2.0f * err;
        if (a.clip_value) {
            const float dvo = value - a.old_values[row];
            const float cv = a.old_values[row] + fminf(fmaxf(dvo, -eps), eps);
            const float ce = cv - ret;
            const bool unclipped = vloss > ce * ce;  // max(a, b): the first only when strictly larger
            const bool vin = dvo >= -eps && dvo <= eps;
            dv = unclipped ? 2.0f * err : (vin ? 2.0f * ce : 0.0f);
            vloss = unclipped ? vloss : ce * ce;
        }
        vloss = a.value_loss_scale * vloss;
        vals[0] = sc * (policy + a.value_coefficient * vloss - a.entropy_coefficient * entropy);
        vals[1] = sc * policy;
        vals[2] = sc * vloss;
        vals[3] = sc * entropy;
        const bool inside = ratio >= 1.0f - eps && ratio <= 1.0f + eps;
        const float d_logp = ((first || inside) ? -adv * sc : 0.0f) * ratio;
#pragma unroll
        for (int j = 0; j < MAXA; ++j) {
            if (j < A) {
                const float s = action_log_std(a, j);
                dm[j] = d_logp * r[j] * expf(-s);
                ds[j] = d_logp * (r[j] * r[j] - 1.0f);
            }
        }
        const float dval = dv * a.value_loss_scale * a.value_coefficient * sc;
        vals[4] = dval;
        // d_head: actor twin = d mean (padding columns zero), critic twin = [dV, 0, ...]
        const long long ld = a.ld_d_head;
        // tf32 planes with 16-byte rows: four columns per store (one 16-byte piece per
        // plane instead of one scalar store per column and plane)
        const bool vec4 = pw.active() && !pw.p.h16 && ld % 4 == 0 && pw.p.ld % 4 == 0 && pw.p.tstride % 4 == 0 &&
                          (reinterpret_cast<uintptr_t>(pw.p.lo) & 15u) == 0 &&
                          (reinterpret_cast<uintptr_t>(pw.p.hi) & 15u) == 0;
        auto put = [&](int j, float g0, float g1) {
            if (a.d_head) {
                a.d_head[static_cast<long long>(row) * ld + j] = g0;
                a.d_head[a.d_head_twin_stride + static_cast<long long>(row) * ld + j] = g1;
            }
            if (pw.active() && !vec4) {
                pw.store(0, row, j, g0);
                pw.store(1, row, j, g1);
            }
        };
#pragma unroll
        for (int j = 0; j < MAXA; ++j)
            if (j < ld) put(j, j < A ? dm[j] : 0.0f, j == 0 ? dval : 0.0f);
        for (int j = MAXA; j < ld; ++j) put(j, 0.0f, 0.0f);
        if (vec4) {
#pragma unroll
            for (int j = 0; j < MAXA; j += 4) {
                if (j < ld) {
                    pw.store4(0, row, j, make_float4(j < A ? dm[j] : 0.0f, j + 1 < A ? dm[j + 1] : 0.0f,
                                                     j + 2 < A ? dm[j + 2] : 0.0f, j + 3 < A ? dm[j + 3] : 0.0f));
                    pw.store4(1, row, j, make_float4(j == 0 ? dval : 0.0f, 0.0f, 0.0f, 0.0f));
                }
            }
            for (int j = MAXA; j < ld; j += 4) {
                pw.store4(0, row, j, make_float4(0.0f, 0.0f, 0.0f, 0.0f));
                pw.store4(1, row, j, make_float4(0.0f, 0.0f, 0.0f, 0.0f));
            }
        }
    }
    pw.flush();
    // block partials: warp sums then a fixed-order combine of the warps (slots in the order
    // loss, policy, value, entropy, d bias critic, d s[0 .. A), d bias actor[0 .. A))
    const int warp = threadIdx.x >> 5;
    auto push = [&](int v, double x) {
        x = warp_sum_d(x);
        if ((threadIdx.x & 31) == 0) sh[warp][v] = x;
    };
#pragma unroll
    for (int v = 0; v < 5; ++v) push(v, vals[v]);
#pragma unroll
    for (int j = 0; j < MAXA; ++j)
        if (j < A) push(5 + j, ds[j]);
#pragma unroll
    for (int j = 0; j < MAXA; ++j)
        if (j < A) push(5 + A + j, dm[j]);
    __syncthreads();
    for (int v = threadIdx.x; v < nslot; v += kT) {
        double s = 0.0;
        for (int w = 0; w < kT / 32; ++w) s += sh[w][v];
        a.partials[static_cast<long long>(blockIdx.x) * nslot + v] = s;
    }
    if (last_block(a.counter)) {
        // warp w sums slots w, w + 8, ...: lane l the blocks l, l + 32, ... in order, then a
        // fixed shuffle tree (the partials were written by other SMs: L1 bypassed)
        const int lane = threadIdx.x & 31;
        for (int v = warp; v < nslot; v += kT / 32) {
            double s = 0.0;
            for (int b = lane; b < static_cast<int>(gridDim.x); b += 32)
                s += __ldcg(a.partials + static_cast<long long>(b) * nslot + v);
            s = warp_sum_d(s);
            if (lane != 0) continue;
            if (v == 0) {
                *a.loss = static_cast<float>(s);
            } else if (v < 4) {
                a.metrics[v - 1] = static_cast<float>(s);
            } else if (v == 4) {
                if (a.d_bias_critic) a.d_bias_critic[0] = static_cast<float>(s);
            } else if (v < 5 + A) {
                const int j = v - 5;
                // d/ds adds the entropy bonus -c_H (mean over rows of a per-row constant)
                double g = s - static_cast<double>(a.entropy_coefficient);
                if (a.std_type) {
                    const float p = a.std_param[j];
                    g = (p >= a.std_min && p <= a.std_max) ? g / static_cast<double>(p) : 0.0;
                }
                a.d_std_param[j] = static_cast<float>(g);
            } else if (a.d_bias_actor) {
                a.d_bias_actor[v - 5 - A] = static_cast<float>(s);
            }
        }
    }
}

// ---------------------------------------------------------------------------
// KL(old || new) and the adaptive learning rate
// ---------------------------------------------------------------------------
__global__ void kl_kernel(const float* mean, long long ld_mean, const float* std_param, const float* old_means,
                          const float* old_stds, int rows, int act, int std_type, float std_min, float std_max,
                          float desired_kl, float* kl, float* learning_rate, double* partials, int* counter) {
    const int row = blockIdx.x * kT + threadIdx.x;
    double v = 0.0;
    if (row < rows) {
        float acc = 0.0f;
        for (int j = 0; j < act; ++j) {
            const float p = std_param[j];
            const float sd = std_type ? fminf(fmaxf(p, std_min), std_max) : expf(p);
            const float vr = old_stds[static_cast<long long>(row) * act + j] / sd;
            const float md = (old_means[static_cast<long long>(row) * act + j] - mean[static_cast<long long>(row) * ld_mean + j]) / sd;
            acc = acc + 0.5f * (vr * vr + md * md - 1.0f);
            acc = acc - logf(vr);
        }
        v = acc;
    }
    v = block_sum_d(v);
    if (threadIdx.x == 0) partials[blockIdx.x] = v;
    if (last_block(counter)) {
        const double s = fixed_order_sum(partials, gridDim.x);
        if (threadIdx.x == 0) {
            const float k = static_cast<float>(s / rows);
            *kl = k;
            if (learning_rate) {
                float lr = *learning_rate;
                if (k > desired_kl * 2.0f) lr = fmaxf(1.0e-5f, lr / 1.5f);
                else if (k < desired_kl / 2.0f && k > 0.0f) lr = fminf(1.0e-2f, lr * 1.5f);
                *learning_rate = lr;
            }
        }
    }
}

// ---------------------------------------------------------------------------
// gradient-norm clipping
// ---------------------------------------------------------------------------
__global__ void sumsq_kernel(const float* __restrict__ g, long long na, long long nc, long long n, int separate,
                             float max_norm, float* norms, double* partials, int* counter) {
    double s[3] = {0.0, 0.0, 0.0};  // actor, critic, std
    for (long long i = static_cast<long long>(blockIdx.x) * kT + threadIdx.x; i < n;
         i += static_cast<long long>(gridDim.x) * kT) {
        const double x = g[i];
        s[i < na ? 0 : (i < na + nc ? 1 : 2)] += x * x;
    }
    for (int q = 0; q < 3; ++q) {
        const double b = block_sum_d(s[q]);
        if (threadIdx.x == 0) partials[static_cast<long long>(q) * gridDim.x + blockIdx.x] = b;
    }
    if (last_block(counter)) {
        double t[3];
        for (int q = 0; q < 3; ++q) t[q] = fixed_order_sum(partials + static_cast<long long>(q) * gridDim.x, gridDim.x);
        if (threadIdx.x == 0) {
            const double group_a = t[0] + t[2], group_c = t[1], total = t[0] + t[1] + t[2];
            auto coef = [&](double ss) { return fmin(1.0, static_cast<double>(max_norm) / (sqrt(ss) + 1.0e-6)); };
            norms[0] = static_cast<float>(group_a);
            norms[1] = static_cast<float>(group_c);
            norms[2] = static_cast<float>(total);
            norms[3] = static_cast<float>(separate ? coef(group_a) : coef(total));
            norms[4] = static_cast<float>(separate ? coef(group_c) : coef(total));
        }
    }
}

__global__ void scale_kernel(float* __restrict__ g, long long na, long long nc, long long n, const float* norms) {
    const float ca = norms[3], cc = norms[4];
    for (long long i = static_cast<long long>(blockIdx.x) * kT + threadIdx.x; i < n;
         i += static_cast<long long>(gridDim.x) * kT)
        g[i] *= (i >= na && i < na + nc) ? cc : ca;
}

// ---------------------------------------------------------------------------
// rollout side: sample actions, store one step
// ---------------------------------------------------------------------------
__global__ void sample_kernel(const rl2_ppo_sample_args a) {
    const int i = blockIdx.x * kT + threadIdx.x;
    if (i >= a.rows) return;
    float log_prob = 0.0f;
    for (int j = 0; j < a.act; ++j) {
        float sd = expf(a.std_param[j]);
        float action_log_std = a.std_param[j];
        if (a.std_type) {
            sd = fminf(fmaxf(a.std_param[j], a.std_min), a.std_max);
            action_log_std = logf(sd);
        }
        if (i == 0 && a.sampled_std) a.sampled_std[j] = sd;
        const float noise = a.noise ? a.noise[static_cast<long long>(i) * a.act + j] : 0.0f;
        a.actions[static_cast<long long>(i) * a.act + j] = a.head[static_cast<long long>(i) * a.ld_head + j] + sd * noise;
        log_prob = log_prob - 0.5f * (noise * noise + 2.0f * action_log_std + kLog2Pi);
    }
    if (a.log_probs) a.log_probs[i] = log_prob;
    if (a.values) a.values[i] = a.head[a.head_twin_stride + static_cast<long long>(i) * a.ld_head];
}

__global__ void store_kernel(const rl2_ppo_store_args a) {
    const int i = blockIdx.x * kT + threadIdx.x;
    if (i >= a.num_envs) return;
    const long long k = static_cast<long long>(a.step) * a.num_envs + i;
    for (int j = 0; j < a.obs_dim; ++j)
        a.r_observations[k * a.obs_dim + j] = a.observations[static_cast<long long>(i) * a.obs_dim + j];
    for (int j = 0; j < a.act; ++j) {
        a.r_actions[k * a.act + j] = a.actions[static_cast<long long>(i) * a.act + j];
        a.r_means[k * a.act + j] = a.mean[static_cast<long long>(i) * a.ld_mean + j];
        a.r_stds[k * a.act + j] = a.sampled_std[j];
    }
    a.r_log_probs[k] = a.log_probs[i];
    a.r_values[k] = a.values[i];
    a.r_rewards[k] = a.rewards[i];
    a.r_terminated[k] = a.terminated[i];
    a.r_truncated[k] = a.truncated[i];
    a.r_next_values[k] = a.next_values[static_cast<long long>(i) * a.next_values_stride];
}

}  // namespace ppo
}  // namespace rl2

// ===========================================================================
// C ABI
// ===========================================================================
using namespace rl2;

extern "C" int rl2_ppo_partials(int n) { return ppo::sum_blocks(n < 1 ? 1 : n); }

extern "C" int rl2_ppo_loss_partials(int rows, int act) {
    return ppo::sum_blocks(rows < 1 ? 1 : rows) * ppo::loss_slots(act < 1 ? 1 : act);
}

extern "C" int rl2_ppo_gae(const rl2_ppo_gae_args* a, void* stream) {
    clear_error();
    if (!a || !a->rewards || !a->values || !a->next_values || !a->terminated || !a->truncated || !a->advantages ||
        !a->returns || a->horizon < 1 || a->num_envs < 1) {
        set_error("rl2_ppo_gae: null array or non-positive horizon / num_envs");
        return -1;
    }
    int S = 1;
    while ((a->horizon + S - 1) / S > 8 && S < 32) S *= 2;
    const int L = (a->horizon + S - 1) / S;
    const long long threads = static_cast<long long>(a->num_envs) * S;
    const long long blocks = (threads + ppo::kT - 1) / ppo::kT;
    if (blocks > 0x7FFFFFFF) {
        set_error("rl2_ppo_gae: too many environments");
        return -1;
    }
    ppo::gae_kernel<<<static_cast<unsigned>(blocks), ppo::kT, 0, as_stream(stream)>>>(*a, S, L);
    return launch_status("rl2_ppo_gae");
}

extern "C" int rl2_ppo_normalize_advantages(float* adv, int n, int sample_std, double* stats, double* partials,
                                            int* counter, void* stream) {
    clear_error();
    if (!adv || !stats || !partials || !counter || n < 1) {
        set_error("rl2_ppo_normalize_advantages: null workspace or n < 1");
        return -1;
    }
    const int blocks = ppo::sum_blocks(n);
    cudaStream_t s = as_stream(stream);
    ppo::adv_moment_kernel<<<blocks, ppo::kT, 0, s>>>(adv, n, 0, stats, partials, counter);
    ppo::adv_moment_kernel<<<blocks, ppo::kT, 0, s>>>(adv, n, 1, stats, partials, counter);
    ppo::adv_normalize_kernel<<<blocks, ppo::kT, 0, s>>>(adv, n, sample_std, stats);
    return launch_status("rl2_ppo_normalize_advantages");
}

extern "C" int rl2_ppo_permutation(unsigned long long seed, const unsigned long long* epoch, int n, int* indices,
                                   int* health, void* stream) {
    clear_error();
    if (!indices || !health || n < 1) {
        set_error("rl2_ppo_permutation: null output / health or n < 1");
        return -1;
    }
    int half = 1;
    while ((1LL << (2 * half)) < n) ++half;
    if (half > 15) {
        set_error("rl2_ppo_permutation: n must be below 2^30");
        return -1;
    }
    ppo::permutation_kernel<<<(n + ppo::kT - 1) / ppo::kT, ppo::kT, 0, as_stream(stream)>>>(seed, epoch, n, half,
                                                                                           indices, health);
    return launch_status("rl2_ppo_permutation");
}

extern "C" int rl2_ppo_gather(const rl2_ppo_gather_args* a, void* stream) {
    clear_error();
    if (!a || a->rows < 1 || a->obs_dim < 1 || a->act_dim < 0 || !a->observations || !plane_used(&a->obs_plane) ||
        !plane_valid(&a->obs_plane) || (a->batch_actions && !a->actions) || (a->batch_means && !a->means) ||
        (a->batch_stds && !a->stds) || (a->batch_log_probs && !a->log_probs) || (a->batch_values && !a->values) ||
        (a->batch_advantages && !a->advantages) || (a->batch_returns && !a->returns)) {
        set_error("rl2_ppo_gather: invalid arguments");
        return -1;
    }
    const long long threads = static_cast<long long>(a->rows) * 32;
    ppo::gather_kernel<<<static_cast<unsigned>((threads + ppo::kT - 1) / ppo::kT), ppo::kT, 0, as_stream(stream)>>>(
        *a, to_plane(&a->obs_plane));
    return launch_status("rl2_ppo_gather");
}

extern "C" int rl2_ppo_loss(const rl2_ppo_loss_args* a, void* stream) {
    clear_error();
    if (!a || !a->head || !a->std_param || a->rows < 1 || a->act < 1 || a->act > ppo::kMaxAct || !a->actions ||
        !a->old_log_probs || !a->old_values || !a->advantages || !a->returns || !a->loss || !a->metrics ||
        !a->d_std_param || !a->partials || !a->counter || (!a->d_head && !plane_used(&a->d_plane)) ||
        !plane_valid(&a->d_plane) || a->ld_d_head < a->act || a->ld_head < a->act) {
        set_error("rl2_ppo_loss: invalid arguments (act must be in [1, %d])", ppo::kMaxAct);
        return -1;
    }
    const int blocks = (a->rows + ppo::kT - 1) / ppo::kT;
    if (a->act <= 16)
        ppo::loss_kernel<16><<<blocks, ppo::kT, 0, as_stream(stream)>>>(*a, to_plane(&a->d_plane));
    else
        ppo::loss_kernel<ppo::kMaxAct><<<blocks, ppo::kT, 0, as_stream(stream)>>>(*a, to_plane(&a->d_plane));
    return launch_status("rl2_ppo_loss");
}

extern "C" int rl2_ppo_kl(const float* mean, long long ld_mean, const float* std_param, const float* old_means,
                          const float* old_stds, int rows, int act, int std_type, float std_min, float std_max,
                          float desired_kl, float* kl, float* learning_rate, double* partials, int* counter,
                          void* stream) {
    clear_error();
    if (!mean || !std_param || !old_means || !old_stds || !kl || !partials || !counter || rows < 1 || act < 1) {
        set_error("rl2_ppo_kl: invalid arguments");
        return -1;
    }
    const int blocks = (rows + ppo::kT - 1) / ppo::kT;
    ppo::kl_kernel<<<blocks, ppo::kT, 0, as_stream(stream)>>>(mean, ld_mean, std_param, old_means, old_stds, rows, act,
                                                             std_type, std_min, std_max, desired_kl, kl,
                                                             learning_rate, partials, counter);
    return launch_status("rl2_ppo_kl");
}

extern "C" int rl2_ppo_clip_gradients(float* grads, long long actor_count, long long critic_count,
                                      long long std_count, int separate, float max_norm, float* norms_out,
                                      double* partials, int* counter, void* stream) {
    clear_error();
    const long long n = actor_count + critic_count + std_count;
    if (!grads || !norms_out || !partials || !counter || n < 1 || actor_count < 0 || critic_count < 0 ||
        std_count < 0) {
        set_error("rl2_ppo_clip_gradients: invalid arguments");
        return -1;
    }
    const int blocks = ppo::sum_blocks(n);
    // the sums: two CTAs per SM at most (fewer partials for the last block's fixed-order merge)
    const int sum_grid = blocks < 296 ? blocks : 296;
    cudaStream_t s = as_stream(stream);
    ppo::sumsq_kernel<<<sum_grid, ppo::kT, 0, s>>>(grads, actor_count, critic_count, n, separate, max_norm, norms_out,
                                                   partials, counter);
    ppo::scale_kernel<<<blocks, ppo::kT, 0, s>>>(grads, actor_count, critic_count, n, norms_out);
    return launch_status("rl2_ppo_clip_gradients");
}

extern "C" int rl2_ppo_sample(const rl2_ppo_sample_args* a, void* stream) {
    clear_error();
    if (!a || !a->head || !a->std_param || !a->actions || a->rows < 1 || a->act < 1) {
        set_error("rl2_ppo_sample: invalid arguments");
        return -1;
    }
    ppo::sample_kernel<<<(a->rows + ppo::kT - 1) / ppo::kT, ppo::kT, 0, as_stream(stream)>>>(*a);
    return launch_status("rl2_ppo_sample");
}

extern "C" int rl2_ppo_store(const rl2_ppo_store_args* a, void* stream) {
    clear_error();
    if (!a || a->num_envs < 1 || a->obs_dim < 1 || a->act < 1 || a->step < 0 || !a->observations || !a->actions ||
        !a->log_probs || !a->values || !a->rewards || !a->terminated || !a->truncated || !a->mean ||
        !a->next_values || !a->sampled_std || !a->r_observations || !a->r_actions || !a->r_log_probs ||
        !a->r_values || !a->r_rewards || !a->r_terminated || !a->r_truncated || !a->r_next_values || !a->r_means ||
        !a->r_stds) {
        set_error("rl2_ppo_store: invalid arguments");
        return -1;
    }
    ppo::store_kernel<<<(a->num_envs + ppo::kT - 1) / ppo::kT, ppo::kT, 0, as_stream(stream)>>>(*a);
    return launch_status("rl2_ppo_store");
}
