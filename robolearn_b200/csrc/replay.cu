// Replay index sampling and batch gather for the FlashSAC learner.
//
// Reference semantics (paths inside the reference project):
//   unbiased bounded index   src/robolearn/warp/_flash_replay.py:116-128 (threshold = (-n) % n,
//                            reject v < threshold, index = v % n)
//   batch gather             src/robolearn/warp/_flash_replay.py:131-160, flashsac/replay.py:179-194
//   batch assembly           src/robolearn/warp/flashsac.py:53-69,166-182 (actor rows, critic rows)
//   reward normalisation     src/robolearn/flashsac/_utils/reward_normalization.py:28-38
//
// The random stream is Philox4x32-10 (Salmon, Moraes, Dror, Shaw, "Parallel
// random numbers: as easy as 1, 2, 3", SC'11), counter = (row, draw epoch,
// rejection round, stream) and key = seed. Warp's own generator is not
// reproduced; parity is anchored on explicit indices, which this gather takes too.
// The gather writes straight into the concatenated layouts the networks read:
// critic rows [obs | action] for i and [next_obs | (next action later)] for B+i,
// actor rows obs_prefix for i and next_obs_prefix for B+i. Copies are bit-exact.

#include "common.cuh"
#include "../../include/rl2.h"

#include <algorithm>

#include "philox.cuh"

namespace rl2 {
namespace replay {

constexpr int kT = 256;

using rl2::U4;
using rl2::mulhilo;
using rl2::philox;

__global__ void sample_kernel(uint64_t seed, const unsigned long long* epoch, const long long* population,
                              long long fixed_population, int batch, int* out, int* health) {
    const int i = blockIdx.x * kT + threadIdx.x;
    if (i >= batch) return;
    const uint32_t n = static_cast<uint32_t>(population ? *population : fixed_population);
    if (n == 0) {
        out[i] = 0;
        return;
    }
    const uint32_t threshold = (0u - n) % n;
    const unsigned long long e = epoch ? *epoch : 0ull;
    const uint32_t k0 = static_cast<uint32_t>(seed), k1 = static_cast<uint32_t>(seed >> 32);
    for (uint32_t round = 0; round < 64; ++round) {
        const U4 r = philox(U4{static_cast<uint32_t>(i), static_cast<uint32_t>(e), static_cast<uint32_t>(e >> 32) ^ round, 0x5A11u},
                            k0, k1);
        const uint32_t vals[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            if (vals[j] >= threshold) {
                out[i] = static_cast<int>(vals[j] % n);
                return;
            }
        }
    }
    out[i] = 0;  // unreachable in practice (probability < 2^-256); reported, never silent
    if (health) atomicOr(health, kHealthTimeout);
}

__global__ void advance_kernel(unsigned long long* epoch, unsigned long long by) { *epoch += by; }

// Standard normal samples by the Box-Muller transform of two Philox uniforms per pair.
// Elements e0 .. e0 + rows * cols - 1 of the row-major [*, cols] stream (element i comes
// from Philox counter quad i / 4), written as rows 0.. of out: any row range of the
// global array reproduces exactly the values a single launch over all rows would give.
__global__ void normal_kernel(uint64_t seed, const unsigned long long* epoch, long long e0, int rows, int cols,
                              float* out, long long ld) {
    const long long total = static_cast<long long>(rows) * cols;
    const unsigned long long e = epoch ? *epoch : 0ull;
    const uint32_t k0 = static_cast<uint32_t>(seed), k1 = static_cast<uint32_t>(seed >> 32);
    const long long q_first = e0 / 4, q_end = (e0 + total + 3) / 4;
    for (long long q = q_first + blockIdx.x * static_cast<long long>(kT) + threadIdx.x; q < q_end;
         q += static_cast<long long>(gridDim.x) * kT) {
        const U4 r = philox(U4{static_cast<uint32_t>(q), static_cast<uint32_t>(q >> 32), static_cast<uint32_t>(e),
                               static_cast<uint32_t>(e >> 32) ^ 0x0A0Fu},
                            k0, k1);
        const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
        for (int p = 0; p < 2; ++p) {
            // uniforms in (0, 1]: (u + 1) * 2^-32 with u in [0, 2^32)
            const float u1 = (static_cast<float>(w[2 * p]) + 1.0f) * 2.3283064365386963e-10f;
            const float u2 = static_cast<float>(w[2 * p + 1]) * 2.3283064365386963e-10f;
            const float rad = sqrtf(-2.0f * logf(u1));
            float sn, cs;
            sincospif(2.0f * u2, &sn, &cs);
            const float z[2] = {rad * cs, rad * sn};
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const long long i = q * 4 + 2 * p + h - e0;
                if (i >= 0 && i < total) out[(i / cols) * ld + (i % cols)] = z[h];
            }
        }
    }
}

// one warp per sampled row
__global__ void gather_kernel(const rl2_replay_gather_args a) {
    const int lane = threadIdx.x & 31;
    const int B = a.batch;
    float rscale = 1.0f;
    if (a.g_var) {
        // r / max(sqrt(var + eps), G_r_max / G_max)
        const float den = fmaxf(sqrtf(a.g_var[0] + a.norm_eps), a.g_r_max[0] / a.g_max);
        rscale = den;
    }
    for (long long w = blockIdx.x * static_cast<long long>(kT / 32) + (threadIdx.x >> 5); w < B;
         w += static_cast<long long>(gridDim.x) * (kT / 32)) {
        const int i = static_cast<int>(w);
        const long long src = a.indices[i];
        const float* o = a.obs + src * a.ld_obs;
        const float* no = a.next_obs + src * a.ld_obs;
        const float* ac = a.action + src * a.ld_action;
        for (int c = lane; c < a.obs_dim; c += 32) {
            const float ov = o[c], nv = no[c];
            if (a.critic_x_pi) a.critic_x_pi[static_cast<long long>(i) * a.ld_critic_x_pi + c] = ov;
            if (a.critic_x) {
                a.critic_x[static_cast<long long>(i) * a.ld_critic_x + c] = ov;
                a.critic_x[static_cast<long long>(B + i) * a.ld_critic_x + c] = nv;
            }
            if (a.actor_x && c < a.actor_obs_dim) {
                a.actor_x[static_cast<long long>(i) * a.ld_actor_x + c] = ov;
                a.actor_x[static_cast<long long>(B + i) * a.ld_actor_x + c] = nv;
            }
            if (a.batch_obs) a.batch_obs[static_cast<long long>(i) * a.obs_dim + c] = ov;
            if (a.batch_next_obs) a.batch_next_obs[static_cast<long long>(i) * a.obs_dim + c] = nv;
        }
        for (int c = lane; c < a.act_dim; c += 32) {
            const float av = ac[c];
            if (a.critic_x) a.critic_x[static_cast<long long>(i) * a.ld_critic_x + a.obs_dim + c] = av;
            if (a.batch_action) a.batch_action[static_cast<long long>(i) * a.act_dim + c] = av;
        }
        if (lane == 0) {
            const float r = a.reward[src];
            if (a.reward_out) a.reward_out[i] = a.g_var ? r / rscale : r;
            if (a.batch_reward) a.batch_reward[i] = r;
            if (a.terminated_out) a.terminated_out[i] = a.terminated[src];
            if (a.truncated_out && a.truncated) a.truncated_out[i] = a.truncated[src];
            if (a.discount_out) a.discount_out[i] = a.discount[src];
        }
    }
}

}  // namespace replay
}  // namespace rl2

using namespace rl2;

extern "C" int rl2_replay_sample(unsigned long long seed, const unsigned long long* epoch, const long long* population,
                                 long long fixed_population, int batch, int* indices, int* health, void* stream) {
    clear_error();
    if (!indices || batch < 1 || (!population && (fixed_population < 1 || fixed_population > 0x7FFFFFFFLL))) {
        set_error("replay sample: invalid arguments");
        return -1;
    }
    replay::sample_kernel<<<(batch + replay::kT - 1) / replay::kT, replay::kT, 0, as_stream(stream)>>>(
        seed, epoch, population, fixed_population, batch, indices, health);
    return launch_status("replay sample");
}

extern "C" int rl2_counter_advance(unsigned long long* epoch, unsigned long long by, void* stream) {
    clear_error();
    if (!epoch) {
        set_error("counter advance: null counter");
        return -1;
    }
    replay::advance_kernel<<<1, 1, 0, as_stream(stream)>>>(epoch, by);
    return launch_status("counter advance");
}

extern "C" int rl2_normal_noise_rows(unsigned long long seed, const unsigned long long* epoch, long long row0,
                                     int rows, int cols, float* out, long long ld, void* stream) {
    clear_error();
    if (!out || rows < 1 || cols < 1 || ld < cols || row0 < 0) {
        set_error("normal noise: invalid arguments");
        return -1;
    }
    const long long e0 = row0 * cols;
    const long long quads = (e0 + static_cast<long long>(rows) * cols + 3) / 4 - e0 / 4;
    const int blocks = static_cast<int>(std::min<long long>((quads + replay::kT - 1) / replay::kT, 148 * 8));
    replay::normal_kernel<<<blocks, replay::kT, 0, as_stream(stream)>>>(seed, epoch, e0, rows, cols, out, ld);
    return launch_status("normal noise");
}

extern "C" int rl2_normal_noise(unsigned long long seed, const unsigned long long* epoch, int rows, int cols,
                                float* out, long long ld, void* stream) {
    return rl2_normal_noise_rows(seed, epoch, 0, rows, cols, out, ld, stream);
}

extern "C" int rl2_replay_gather(const rl2_replay_gather_args* a, void* stream) {
    clear_error();
    if (!a || !a->indices || !a->obs || !a->next_obs || !a->action || !a->reward || !a->terminated ||
        !a->discount || a->batch < 1 || a->obs_dim < 1 || a->act_dim < 1 || (a->g_var && !a->g_r_max)) {
        set_error("replay gather: invalid arguments");
        return -1;
    }
    const int blocks = std::min((a->batch + 7) / 8, 148 * 16);
    replay::gather_kernel<<<blocks, replay::kT, 0, as_stream(stream)>>>(*a);
    return launch_status("replay gather");
}

extern "C" void rl2_philox4x32(unsigned int c0, unsigned int c1, unsigned int c2, unsigned int c3, unsigned int k0,
                               unsigned int k1, unsigned int* out4) {
    const replay::U4 r = replay::philox(replay::U4{c0, c1, c2, c3}, k0, k1);
    out4[0] = r.x;
    out4[1] = r.y;
    out4[2] = r.z;
    out4[3] = r.w;
}

// ===========================================================================
// replay ingest: n-step staging ring + commit, and the reward normaliser
// ===========================================================================
//
// Semantics (paths inside the reference project): n-step return, done handling and
// timeout bootstrap of src/robolearn/flashsac/replay.py:109-174 and the Warp
// restatement _copy_pending / _commit_pending / _advance_replay
// (src/robolearn/warp/_flash_replay.py:26-113); reward statistics of
// src/robolearn/flashsac/_utils/reward_normalization.py:14-125.
// counters (int64): [0] steps seen, [1] write position, [2] filled rows.
namespace rl2 {
namespace ingest {

constexpr int kT = 256;

// one warp per environment: stage this step, then (from step n-1 on) commit the
// n-step transition that starts n-1 steps ago into the replay ring
__global__ void stage_commit_kernel(const rl2_replay_ingest_args a) {
    const int lane = threadIdx.x & 31;
    const long long step = a.counters[0];
    const int n = a.n_step;
    const int latest = static_cast<int>(step % n);
    const long long E = a.num_envs;
    for (long long i = blockIdx.x * static_cast<long long>(kT / 32) + (threadIdx.x >> 5); i < E;
         i += static_cast<long long>(gridDim.x) * (kT / 32)) {
        const long long ps = static_cast<long long>(latest) * E + i;  // pending row of this step
        for (int c = lane; c < a.obs_dim; c += 32) {
            a.pend_obs[ps * a.obs_dim + c] = a.obs[i * a.ld_obs + c];
            a.pend_next_obs[ps * a.obs_dim + c] = a.next_obs[i * a.ld_obs + c];
        }
        for (int c = lane; c < a.act_dim; c += 32) a.pend_act[ps * a.act_dim + c] = a.action[i * a.ld_action + c];
        if (lane == 0) {
            a.pend_reward[ps] = a.reward[i];
            a.pend_term[ps] = a.terminated_u8 ? static_cast<float>(a.terminated_u8[i] != 0) : a.terminated[i];
            a.pend_trunc[ps] = a.truncated_u8 ? static_cast<float>(a.truncated_u8[i] != 0) : a.truncated[i];
        }
        __syncwarp();
        if (step < n - 1) continue;
        const int oldest = (latest + 1) % n;
        int next_slot = latest;
        float total = a.pend_reward[ps];
        float term = a.pend_term[ps];
        float trunc = a.pend_trunc[ps];
        float factor = a.gamma;
        for (int off = 1; off < n; ++off) {
            const int slot = (latest - off + n) % n;
            const long long q = static_cast<long long>(slot) * E + i;
            const bool done = a.pend_term[q] != 0.0f || a.pend_trunc[q] != 0.0f;
            if (done) {
                total = a.pend_reward[q];
                factor = a.gamma;
                term = a.pend_term[q];
                trunc = a.pend_trunc[q];
                next_slot = slot;
            } else {
                total = a.pend_reward[q] + a.gamma * total;
                factor = a.gamma * factor;
            }
        }
        const long long dst = (a.counters[1] + i) % a.capacity;
        const long long po = static_cast<long long>(oldest) * E + i;
        const long long pn = static_cast<long long>(next_slot) * E + i;
        for (int c = lane; c < a.obs_dim; c += 32) {
            a.r_obs[dst * a.ld_replay_obs + c] = a.pend_obs[po * a.obs_dim + c];
            a.r_next_obs[dst * a.ld_replay_obs + c] = a.pend_next_obs[pn * a.obs_dim + c];
        }
        for (int c = lane; c < a.act_dim; c += 32) a.r_act[dst * a.ld_replay_act + c] = a.pend_act[po * a.act_dim + c];
        if (lane == 0) {
            a.r_reward[dst] = total;
            a.r_term[dst] = term;
            a.r_trunc[dst] = trunc;
            a.r_discount[dst] = factor;
        }
    }
}

__global__ void advance_kernel(long long* counters, int n_step, long long num_envs, long long capacity) {
    if (counters[0] >= n_step - 1) {
        counters[1] = (counters[1] + num_envs) % capacity;
        counters[2] = counters[2] + num_envs < capacity ? counters[2] + num_envs : capacity;
    }
    counters[0] += 1;
}

// One block: per-environment discounted return, running max |G|, and the running
// mean / variance of G by Chan's parallel update (reward_normalization.py:14-38,
// :64-91). state = [mean, var, count, G_r_max].
__global__ void reward_stats_kernel(const float* reward, const float* term, const float* trunc,
                                    const unsigned char* term_u8, const unsigned char* trunc_u8, float* g_r,
                                    int num_envs, float gamma, float* state, float epsilon) {
    __shared__ double red[3][kT];
    double s = 0.0, mx = 0.0;
    for (int i = threadIdx.x; i < num_envs; i += kT) {
        const bool done = (term_u8 ? term_u8[i] != 0 : term[i] != 0.0f) || (trunc_u8 ? trunc_u8[i] != 0 : trunc[i] != 0.0f);
        const float g = gamma * (done ? 0.0f : 1.0f) * g_r[i] + reward[i];
        g_r[i] = g;
        s += g;
        mx = fmax(mx, fabs(static_cast<double>(g)));
    }
    red[0][threadIdx.x] = s;
    red[2][threadIdx.x] = mx;
    __syncthreads();
    for (int o = kT / 2; o > 0; o >>= 1) {
        if (threadIdx.x < o) {
            red[0][threadIdx.x] += red[0][threadIdx.x + o];
            red[2][threadIdx.x] = fmax(red[2][threadIdx.x], red[2][threadIdx.x + o]);
        }
        __syncthreads();
    }
    const double mean_b = red[0][0] / num_envs;
    double q = 0.0;
    for (int i = threadIdx.x; i < num_envs; i += kT) {
        const double d = g_r[i] - mean_b;
        q += d * d;
    }
    red[1][threadIdx.x] = q;
    __syncthreads();
    for (int o = kT / 2; o > 0; o >>= 1) {
        if (threadIdx.x < o) red[1][threadIdx.x] += red[1][threadIdx.x + o];
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        const float batch_mean = static_cast<float>(mean_b);
        const float batch_var = static_cast<float>(red[1][0] / num_envs);
        const float batch_count = static_cast<float>(num_envs);
        const float mean = state[0], var = state[1], count = state[2];
        const float delta = batch_mean - mean;
        const float total = count + batch_count;
        const float ratio = batch_count / total;
        const float m_a = var * (count + epsilon);
        const float m_b = batch_var * batch_count;
        const float m2 = m_a + m_b + delta * delta * count * ratio;
        state[0] = mean + delta * ratio;
        state[1] = m2 / total;
        state[2] = total;
        state[3] = fmaxf(state[3], static_cast<float>(red[2][0]));
    }
}

}  // namespace ingest
}  // namespace rl2

extern "C" int rl2_replay_ingest(const rl2_replay_ingest_args* a, void* stream) {
    using namespace rl2;
    clear_error();
    if (!a || !a->counters || !a->obs || !a->next_obs || !a->action || !a->reward ||
        (!a->terminated && !a->terminated_u8) || (!a->truncated && !a->truncated_u8) || a->n_step < 1 ||
        a->num_envs < 1 || a->capacity < a->num_envs || !a->pend_obs || !a->r_obs) {
        set_error("replay ingest: invalid arguments");
        return -1;
    }
    const int blocks = static_cast<int>(std::min<long long>((a->num_envs + 7) / 8, 148 * 16));
    ingest::stage_commit_kernel<<<blocks, ingest::kT, 0, as_stream(stream)>>>(*a);
    if (launch_status("replay ingest")) return -1;
    ingest::advance_kernel<<<1, 1, 0, as_stream(stream)>>>(a->counters, a->n_step, a->num_envs, a->capacity);
    return launch_status("replay advance");
}

extern "C" int rl2_reward_stats_update(const float* reward, const float* terminated, const float* truncated,
                                       const unsigned char* terminated_u8, const unsigned char* truncated_u8,
                                       float* g_r, int num_envs, float gamma, float* state, float epsilon,
                                       void* stream) {
    using namespace rl2;
    clear_error();
    if (!reward || (!terminated && !terminated_u8) || (!truncated && !truncated_u8) || !g_r || !state ||
        num_envs < 1) {
        set_error("reward stats: invalid arguments");
        return -1;
    }
    ingest::reward_stats_kernel<<<1, ingest::kT, 0, as_stream(stream)>>>(
        reward, terminated, truncated, terminated_u8, truncated_u8, g_r, num_envs, gamma, state, epsilon);
    return launch_status("reward statistics");
}
