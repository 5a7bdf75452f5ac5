// Tanh-Gaussian policy head, the actor objective and the temperature step.
//
// Reference semantics (paths inside the reference project):
//   policy head + rsample   src/robolearn/flashsac/layers.py:116-166, _utils/distribution.py:12-19
//   actor objective         src/robolearn/flashsac/updates.py:83-166 (min over twins, torch.minimum
//                           splits the derivative equally at a tie, warp/flashsac.py:140-145)
//   temperature             src/robolearn/flashsac/updates.py:297-326, networks.py:113-119
//
// The head GEMM writes [mean | pre-tanh log-std] per row (2A columns, biases
// fused). Sampling keeps no intermediates: the backward recomputes them from
// the head output and the noise, so the only stored per-row state is log pi.

#include "planes.cuh"

#include <algorithm>

namespace rl2 {
namespace policy {

constexpr int kT = 256;
constexpr int kWarps = kT / 32;
constexpr float kLogStdMin = -10.0f;
constexpr float kLogStdMax = 2.0f;
constexpr float kLog2 = 0.69314718055994530942f;
constexpr float kHalfLog2Pi = 0.91893853320467274178f;

__device__ __forceinline__ float softplus(float x) { return x > 20.0f ? x : log1pf(expf(x)); }

struct Sample {
    float std, log_std, raw, action, ts;
};

__device__ __forceinline__ Sample sample(float mean, float s, float eps) {
    Sample o;
    o.ts = tanhf(s);
    o.log_std = kLogStdMin + (kLogStdMax - kLogStdMin) * 0.5f * (1.0f + o.ts);
    o.std = expf(o.log_std);
    o.raw = mean + eps * o.std;
    o.action = tanhf(o.raw);
    return o;
}

// one warp per row
__global__ void sample_kernel(const rl2_policy_args a) {
    const int lane = threadIdx.x & 31;
    for (long long row = blockIdx.x * static_cast<long long>(kWarps) + (threadIdx.x >> 5); row < a.rows;
         row += static_cast<long long>(gridDim.x) * kWarps) {
        const float* h = a.head + row * a.ld_head;
        const float* n = a.noise + row * a.ld_noise;
        float lp = 0.0f;
        for (int j = lane; j < a.act; j += 32) {
            const Sample s = sample(h[j], h[a.act + j], n[j]);
            const float var = s.std * s.std;
            const float diff = s.raw - h[j];
            const float gauss = -(diff * diff) / (2.0f * var) - logf(s.std) - kHalfLog2Pi;
            const float jac = 2.0f * (kLog2 - s.raw - softplus(-2.0f * s.raw));
            lp += gauss - jac;
            if (a.actions) a.actions[row * a.ld_actions + j] = s.action;
        }
        lp = warp_sum(lp);
        if (lane == 0 && a.log_pi) a.log_pi[row] = lp;
    }
}

__global__ void deterministic_kernel(const rl2_policy_args a) {
    const long long total = static_cast<long long>(a.rows) * a.act;
    for (long long i = blockIdx.x * static_cast<long long>(kT) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * kT) {
        const long long r = i / a.act;
        const int j = static_cast<int>(i % a.act);
        a.actions[r * a.ld_actions + j] = tanhf(a.head[r * a.ld_head + j]);
    }
}

// one warp per row; dgrad columns [0,A) = d mean, [A,2A) = d pre-tanh log-std
// One CTA per 32-row column-sum group: the group's 32 x A elements are computed by all
// threads at once (each element's arithmetic as in a per-row loop), their d(mean) and
// d(log-std pre-activation) kept in shared memory, then thread c < 2A adds column c over
// the group's rows in row order (the same sequential sum per group as one warp walking
// the rows), so the bias-gradient partials do not depend on the thread layout.
__global__ void __launch_bounds__(kT) backward_kernel(const rl2_policy_args a, const Plane plane) {
    PlaneWriter pw(plane);
    __shared__ float dmean_s[32][64];
    __shared__ float ds_s[32][64];
    const float dlp_val = a.d_log_pi_value ? *a.d_log_pi_value : 0.0f;
    const float bc = (a.bc_alpha > 0.0f && a.q_abs) ? a.bc_alpha * *a.q_abs : 0.0f;
    const int groups = (a.rows + 31) / 32;
    const int A = a.act;
    for (int g = blockIdx.x; g < groups; g += gridDim.x) {
        const long long r0 = static_cast<long long>(g) * 32;
        const int nrows = static_cast<int>(min(32LL, static_cast<long long>(a.rows) - r0));
        for (int e = threadIdx.x; e < nrows * A; e += kT) {
            const int rr = e / A, j = e - rr * A;
            const long long row = r0 + rr;
            const float* h = a.head + row * a.ld_head;
            const float* n = a.noise + row * a.ld_noise;
            const float dlp = row < a.grad_rows ? (a.d_log_pi ? a.d_log_pi[row] : dlp_val) : 0.0f;
            const Sample smp = sample(h[j], h[A + j], n[j]);
            float da = 0.0f;
            if (row < a.grad_rows && a.d_action) da = a.d_action[row * a.ld_d_action + j];
            if (bc != 0.0f && row < a.grad_rows)
                da += bc * 2.0f * (smp.action - a.replay_action[row * a.ld_replay_action + j]) /
                      (static_cast<float>(a.grad_rows) * A);
            const float draw = da * (1.0f - smp.action * smp.action) + dlp * 2.0f * smp.action;
            const float dmean = draw;
            const float dlogstd = draw * smp.std * n[j] - dlp;
            const float ds = dlogstd * (kLogStdMax - kLogStdMin) * 0.5f * (1.0f - smp.ts * smp.ts);
            if (a.d_head) {
                a.d_head[row * a.ld_d_head + j] = dmean;
                a.d_head[row * a.ld_d_head + A + j] = ds;
            }
            if (pw.active()) {
                pw.store(0, row, j, dmean);
                pw.store(0, row, A + j, ds);
            }
            dmean_s[rr][j] = dmean;
            ds_s[rr][j] = ds;
        }
        __syncthreads();
        if (a.bias_part && threadIdx.x < 2 * A) {
            const int c = threadIdx.x < A ? threadIdx.x : threadIdx.x - A;
            const float(*src)[64] = threadIdx.x < A ? dmean_s : ds_s;
            float acc = 0.0f;
            for (int rr = 0; rr < nrows; ++rr) acc += src[rr][c];
            a.bias_part[static_cast<long long>(g) * 2 * A + threadIdx.x] = acc;
        }
        __syncthreads();  // the next group reuses the shared rows
    }
    pw.flush();
}

}  // namespace policy

// ---------------------------------------------------------------------------
// actor objective over the frozen critic's twin logits
// ---------------------------------------------------------------------------
namespace actor_obj {

constexpr int kWarps = 8;
constexpr int kT = kWarps * 32;

__global__ void __launch_bounds__(kT) kernel(const rl2_actor_objective_args a, const Plane plane) {
    PlaneWriter pw(plane);
    __shared__ float z_s[128];
    __shared__ float red[kWarps][5];
    __shared__ bool last_block;
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int bins = a.bins;
    for (int k = threadIdx.x; k < 128; k += kT) z_s[k] = k < bins ? a.support[k] : 0.0f;
    __syncthreads();
    const float alpha = a.alpha[0];
    const float inv_b = 1.0f / static_cast<float>(a.batch);
    float s_obj = 0.0f, s_lp = 0.0f, s_act = 0.0f, s_qabs = 0.0f, s_bc = 0.0f;
    for (int row = blockIdx.x * kWarps + warp; row < a.batch; row += gridDim.x * kWarps) {
        float p[2][4];
        float q[2];
#pragma unroll
        for (int t = 0; t < 2; ++t) {
            const float* src = a.logits + t * a.logits_twin_stride + static_cast<long long>(row) * a.logits_row_stride;
            float x[4];
            float mx = -INFINITY;
#pragma unroll
            for (int s = 0; s < 4; ++s) {
                const int k = lane + 32 * s;
                x[s] = k < bins ? src[k] : -INFINITY;
                mx = fmaxf(mx, x[s]);
            }
            mx = warp_max(mx);
            float se = 0.0f;
#pragma unroll
            for (int s = 0; s < 4; ++s) se += (lane + 32 * s < bins) ? expf(x[s] - mx) : 0.0f;
            const float lse = mx + logf(warp_sum(se));
            float qq = 0.0f;
#pragma unroll
            for (int s = 0; s < 4; ++s) {
                const int k = lane + 32 * s;
                p[t][s] = k < bins ? expf(x[s] - lse) : 0.0f;
                qq += p[t][s] * z_s[k];
            }
            q[t] = warp_sum(qq);
        }
        // torch.minimum: the smaller twin gets the whole derivative, a tie splits it
        float dq0 = q[0] < q[1] ? -inv_b : (q[0] == q[1] ? -0.5f * inv_b : 0.0f);
        float dq1 = q[1] < q[0] ? -inv_b : (q[0] == q[1] ? -0.5f * inv_b : 0.0f);
        const float qmin = fminf(q[0], q[1]);
#pragma unroll
        for (int t = 0; t < 2; ++t) {
            const float dq = t == 0 ? dq0 : dq1;
#pragma unroll
            for (int s = 0; s < 4; ++s) {
                const int k = lane + 32 * s;
                if (k < bins) pw.store(t, row, k, dq * p[t][s] * (z_s[k] - q[t]));
            }
        }
        float asum = 0.0f, bcs = 0.0f;
        for (int j = lane; j < a.act; j += 32) {
            const float av = a.actions[static_cast<long long>(row) * a.actions_row_stride + j];
            asum += av;
            if (a.replay_action) {
                const float d = av - a.replay_action[static_cast<long long>(row) * a.replay_row_stride + j];
                bcs += d * d;
            }
        }
        asum = warp_sum(asum);
        bcs = warp_sum(bcs);
        const float lp = a.log_pi[row];
        s_obj += lp * alpha - qmin;
        s_lp += lp;
        s_act += asum;
        s_qabs += fabsf(qmin);
        s_bc += bcs;
    }
    if (lane == 0) {
        red[warp][0] = s_obj;
        red[warp][1] = s_lp;
        red[warp][2] = s_act;
        red[warp][3] = s_qabs;
        red[warp][4] = s_bc;
    }
    __syncthreads();
    if (threadIdx.x < 5) {
        float v = 0.0f;
        for (int w = 0; w < kWarps; ++w) v += red[w][threadIdx.x];
        a.workspace[static_cast<long long>(blockIdx.x) * 5 + threadIdx.x] = v;
    }
    pw.flush();
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) last_block = atomicAdd(a.counter, 1u) == gridDim.x - 1;
    __syncthreads();
    if (!last_block) return;
    __threadfence();
    // all block rows summed by the last block's threads: thread i takes rows i, i + kT, ...
    // in order, then a fixed pairwise tree over the threads (deterministic)
    __shared__ float tree[5][kT];
    {
        float s[5] = {0, 0, 0, 0, 0};
        for (unsigned b = threadIdx.x; b < gridDim.x; b += kT)
            for (int i = 0; i < 5; ++i) s[i] += __ldcg(a.workspace + static_cast<long long>(b) * 5 + i);
        for (int i = 0; i < 5; ++i) tree[i][threadIdx.x] = s[i];
    }
    __syncthreads();
    for (int w = kT / 2; w >= 1; w >>= 1) {
        if (threadIdx.x < w)
            for (int i = 0; i < 5; ++i) tree[i][threadIdx.x] += tree[i][threadIdx.x + w];
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        float v[5];
        for (int i = 0; i < 5; ++i) v[i] = tree[i][0];
        const float B = static_cast<float>(a.batch);
        const float q_abs = v[3] / B;
        float loss = v[0] / B;
        if (a.bc_alpha > 0.0f) loss += a.bc_alpha * q_abs * (v[4] / (B * a.act));
        a.loss_out[0] = loss;
        a.entropy_out[0] = -v[1] / B;
        a.mean_action_out[0] = v[2] / (B * a.act);
        if (a.q_abs_out) a.q_abs_out[0] = q_abs;
        if (a.d_log_pi_out) a.d_log_pi_out[0] = alpha / B;
        *a.counter = 0u;
    }
}

}  // namespace actor_obj

// ---------------------------------------------------------------------------
// temperature: one scalar Adam step (torch formula) plus alpha for the critic phase
// ---------------------------------------------------------------------------
namespace temp {
__global__ void kernel(const rl2_temperature_args a) {
    const float log_t = a.log_temp[0];
    const float value = expf(log_t);
    if (a.update) {
        const float ent = a.entropy[0];
        const float diff = ent - a.target_entropy;
        a.value_out[0] = value;
        a.loss_out[0] = value * diff;
        const float g = value * diff;
        // schedule index = completed steps (LambdaLR steps after optimizer.step)
        float* st = a.adam_state;  // [step, m, v]
        const double step = static_cast<double>(st[0]) + 1.0;
        const double k = step - 1.0;
        double lr;
        if (k < a.warmup_steps)
            lr = a.lr_init + (a.lr_peak - a.lr_init) * (k / a.warmup_steps);
        else if (k < a.decay_steps)
            lr = a.lr_end + (a.lr_peak - a.lr_end) * 0.5 *
                                (1.0 + cos(3.14159265358979323846 * (k - a.warmup_steps) / (a.decay_steps - a.warmup_steps)));
        else
            lr = a.lr_end;
        float m = st[1], v = st[2];
        m = m + (1.0f - a.beta1) * (g - m);
        v = v * a.beta2 + (1.0f - a.beta2) * g * g;
        const double bc1 = 1.0 - pow(static_cast<double>(a.beta1), step);
        const double bc2 = 1.0 - pow(static_cast<double>(a.beta2), step);
        const float step_size = static_cast<float>(lr / bc1);
        const float denom = sqrtf(v) / static_cast<float>(sqrt(bc2)) + a.eps;
        const float nt = log_t - step_size * (m / denom);
        st[0] = static_cast<float>(step);
        st[1] = m;
        st[2] = v;
        a.log_temp[0] = nt;
        if (a.alpha_out) a.alpha_out[0] = expf(nt);
    } else if (a.alpha_out) {
        a.alpha_out[0] = value;
    }
}
}  // namespace temp

}  // namespace rl2

using namespace rl2;

extern "C" int rl2_policy_sample(const rl2_policy_args* a, int deterministic, void* stream) {
    clear_error();
    if (!a || !a->head || a->rows < 1 || a->act < 1 || a->act > 64 || (!deterministic && !a->noise) ||
        (deterministic && !a->actions)) {
        set_error("policy sample: invalid arguments (1..64 action dimensions)");
        return -1;
    }
    if (deterministic) {
        const long long work = static_cast<long long>(a->rows) * a->act;
        const int blocks = static_cast<int>(std::min<long long>((work + policy::kT - 1) / policy::kT, 148 * 16));
        policy::deterministic_kernel<<<blocks, policy::kT, 0, as_stream(stream)>>>(*a);
    } else {
        const int blocks = std::min((a->rows + policy::kWarps - 1) / policy::kWarps, 148 * 16);
        policy::sample_kernel<<<blocks, policy::kT, 0, as_stream(stream)>>>(*a);
    }
    return launch_status("policy sample");
}

extern "C" int rl2_policy_backward(const rl2_policy_args* a, void* stream) {
    clear_error();
    if (!a || !a->head || !a->noise || a->rows < 1 || a->act < 1 || a->act > 64 || !plane_valid(&a->d_plane) ||
        (!a->d_head && !plane_used(&a->d_plane)) || (a->bc_alpha > 0.0f && (!a->replay_action || !a->q_abs))) {
        set_error("policy backward: invalid arguments");
        return -1;
    }
    const int groups = (a->rows + 31) / 32;
    const int blocks = std::min(groups, 148 * 8);
    policy::backward_kernel<<<blocks, policy::kT, 0, as_stream(stream)>>>(*a, to_plane(&a->d_plane));
    return launch_status("policy backward");
}

extern "C" int rl2_actor_objective_workspace_floats(int batch) {
    return std::min((batch + actor_obj::kWarps - 1) / actor_obj::kWarps, 148 * 8) * 5;
}

extern "C" int rl2_actor_objective(const rl2_actor_objective_args* a, void* stream) {
    clear_error();
    if (!a || !a->logits || !a->support || !a->log_pi || !a->actions || !a->alpha || !a->workspace || !a->counter ||
        !a->loss_out || !a->entropy_out || !a->mean_action_out || a->bins < 2 || a->bins > 128 || a->batch < 1 ||
        !plane_valid(&a->d_logits) || (a->bc_alpha > 0.0f && !a->replay_action)) {
        set_error("actor objective: invalid arguments");
        return -1;
    }
    const int blocks = std::min((a->batch + actor_obj::kWarps - 1) / actor_obj::kWarps, 148 * 8);
    actor_obj::kernel<<<blocks, actor_obj::kT, 0, as_stream(stream)>>>(*a, to_plane(&a->d_logits));
    return launch_status("actor objective");
}

extern "C" int rl2_temperature_step(const rl2_temperature_args* a, void* stream) {
    clear_error();
    if (!a || !a->log_temp || (a->update && (!a->entropy || !a->adam_state || !a->value_out || !a->loss_out))) {
        set_error("temperature step: invalid arguments");
        return -1;
    }
    temp::kernel<<<1, 1, 0, as_stream(stream)>>>(*a);
    return launch_status("temperature step");
}
