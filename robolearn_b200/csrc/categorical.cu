// Fused categorical critic objective: two-hot Bellman target projection onto the
// fixed atom support + log-softmax cross-entropy + logits gradient, one pass.
//
// Reference semantics (all paths inside the reference project):
//   target selection  src/robolearn/flashsac/updates.py:19-31  (argmin over twins, tie -> twin 0)
//   projection        src/robolearn/flashsac/updates.py:34-80  (lower/upper split, scatter_add)
//   CE + gradient     src/robolearn/flashsac/updates.py:248-257 (mean over [2, B]; autograd)
//   native version    src/robolearn/cuda/categorical_kernels.cuh:87-114 (shared-memory atomics)
//
// Design: eight lanes per transition row, four rows per warp. A lane holds E = ceil(bins /
// 8) atoms of its row, strided (atom k = sub + 8 s) for the elementwise work, so every
// load and store instruction covers whole 32-byte row segments and every row reduction is
// three shuffles inside the lane's group of eight; each atom's exp(x - max) serves both the
// softmax sum and the probabilities (one exponential per atom and twin, the __expf
// intrinsic). The projection runs on the blocked
// layout (atom j = E sub + s, exchanged through shared memory): the shifted atom values are
// monotone in the source atom j, so every target atom receives a contiguous run of j, and a
// segmented scan (sequential inside a lane, three shuffle steps across the group) produces
// each run's sum in a fixed order: deterministic without atomics. The float arithmetic of
// the bin location uses round-to-nearest intrinsics (no FMA contraction) in the reference's
// operation order, so lower/upper/fraction agree with Torch's float32 evaluation.
//
// Cross-block reduction of the head-bias gradient, loss and entropy maximum: each block
// writes one partial row; the last block of each group of 16 (by ticket) sums its group's
// rows in block order, and the last group to finish sums the group rows in group order.

#include "common.cuh"
#include "../../include/rl2.h"

#include <algorithm>
#include <climits>

namespace rl2 {
namespace cat {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kRowsPerWarp = 4;  // eight lanes per row
constexpr int kRowsPerBlock = kWarps * kRowsPerWarp;
constexpr int kMaxBins = 128;
constexpr int kGroup = 16;  // blocks per first-level reduction group
constexpr int kMaxGrid = 148 * 4;

struct Args {
    const float* target_logits;
    long long t_row, t_twin;
    int t_row0;
    const float* online_logits;
    long long o_row, o_twin;
    const float* reward;
    const float* terminated;
    const float* discount;
    const float* next_log_pi;
    const float* alpha;
    const float* support;
    float min_v, max_v, width;
    int bins, batch;
    float loss_weight;
    float* dlogits;
    long long d_row, d_twin;
    __half* d16;
    long long d16_row, d16_twin;
    const float* d16_scale;
    float* d_hi;
    float* d_lo;
    long long dp_row, dp_twin;
    float* target_out;
    long long target_row;
    float* partial;  // [grid][2*bins + 2] block rows, then [groups][2*bins + 2] group rows
    unsigned* counter;  // [0]: group tickets; [1 + g]: block tickets of group g
    float* loss_out;
    float* max_entropy_out;
    float* bias_grad_out;
    int bias_accumulate;
    int* health;
};

inline int grid_for(int batch) { return std::max(1, std::min((batch + kRowsPerBlock - 1) / kRowsPerBlock, kMaxGrid)); }
inline int groups_for(int grid) { return (grid + kGroup - 1) / kGroup; }

// Row pitch of the per-row shared arrays: >= G E and = G (mod 32), so that the strided
// (k = sub + G s) and blocked (j = E sub + s) accesses of the rows of a warp spread over
// the banks.
template <int G, int E>
__host__ __device__ constexpr int pitch() {
    return G * E + ((G - (G * E) % 32) + 32) % 32;
}

// Sum / maximum over the G lanes of a row.
template <int G>
__device__ __forceinline__ float gsum(float v) {
#pragma unroll
    for (int d = 1; d < G; d <<= 1) v += __shfl_xor_sync(0xffffffffu, v, d);
    return v;
}

template <int G>
__device__ __forceinline__ float gmax(float v) {
#pragma unroll
    for (int d = 1; d < G; d <<= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, d));
    return v;
}

// Segmented inclusive scan over the blocked elements of a row (lane sub holds j = E sub + s)
// with monotone non-decreasing keys: each run's total goes to out[key] at the run's last
// element (out[key] += total when add). Keys outside [0, bins) are never written.
template <int G, int E>
__device__ __forceinline__ void scatter_runs(const int (&key)[E], const float (&val)[E], float* out, int bins,
                                             bool add) {
    const int sub = threadIdx.x & (G - 1);
    float acc[E];
    acc[0] = val[0];
#pragma unroll
    for (int s = 1; s < E; ++s) acc[s] = (key[s] == key[s - 1]) ? acc[s - 1] + val[s] : val[s];
    const int tail = key[E - 1];
    float run = acc[E - 1];
    bool open = key[0] == key[E - 1];
#pragma unroll
    for (int d = 1; d < G; d <<= 1) {
        const int ok = __shfl_up_sync(0xffffffffu, tail, d, G);
        const float os = __shfl_up_sync(0xffffffffu, run, d, G);
        const int oo = __shfl_up_sync(0xffffffffu, static_cast<int>(open), d, G);
        if (sub >= d && open && ok == tail) {
            run = os + run;
            open = oo != 0;
        }
    }
    const int prev_tail = __shfl_up_sync(0xffffffffu, tail, 1, G);
    const float prev_run = __shfl_up_sync(0xffffffffu, run, 1, G);
    const float carry = (sub > 0 && prev_tail == key[0]) ? prev_run : 0.0f;
#pragma unroll
    for (int s = 0; s < E; ++s)
        if (key[s] == key[0]) acc[s] = carry + acc[s];
    const int next_head = __shfl_down_sync(0xffffffffu, key[0], 1, G);
#pragma unroll
    for (int s = 0; s < E; ++s) {
        const int nk = s < E - 1 ? key[s + 1] : (sub < G - 1 ? next_head : INT_MAX - 1);
        if (key[s] != nk && key[s] >= 0 && key[s] < bins) out[key[s]] = add ? out[key[s]] + acc[s] : acc[s];
    }
}

// One row per group of G lanes (lane group rg of a warp): target-twin selection,
// projection, cross-entropy and logits gradient. t0 / t1 and o0 / o1 point at the row's
// next-observation target logits and current-observation online logits of twins 0 / 1, in
// global memory or in a shared-memory stage; they are read only when rv.
template <int G, int E>
__device__ __forceinline__ void row_work(const Args& a, const float* t0, const float* t1, const float* o0,
                                         const float* o1, int row, bool rv, const float* z_s, float* pw, float* tw, float alpha,
                                         float scale16, float (&bias_acc)[2][E], float& loss_acc, float& ent_max,
                                         bool& overflow) {
    const int sub = threadIdx.x & (G - 1);
    const int bins = a.bins;
    const float width = a.width;
    // ---- target twins at the next-observation row: softmax and expected value; twin 0's
    // probabilities go to shared memory and twin 1's replace them when its value is lower
    float q0 = 0.0f;
#pragma unroll
    for (int t = 0; t < 2; ++t) {
        const float* src = t == 0 ? t0 : t1;
        float e[E];
        float mx = -INFINITY;
#pragma unroll
        for (int s = 0; s < E; ++s) {
            const int k = sub + G * s;
            e[s] = (rv && k < bins) ? src[k] : -INFINITY;
            mx = fmaxf(mx, e[s]);
        }
        mx = gmax<G>(mx);
        float se = 0.0f;
#pragma unroll
        for (int s = 0; s < E; ++s) {
            e[s] = (sub + G * s < bins) ? __expf(e[s] - mx) : 0.0f;
            se += e[s];
        }
        const float inv = 1.0f / gsum<G>(se);
        float qq = 0.0f;
#pragma unroll
        for (int s = 0; s < E; ++s) {
            e[s] = e[s] * inv;  // probabilities
            qq += e[s] * z_s[sub + G * s];
        }
        qq = gsum<G>(qq);
        if (t == 0) {
            q0 = qq;
#pragma unroll
            for (int s = 0; s < E; ++s) {
                pw[sub + G * s] = e[s];
                tw[sub + G * s] = 0.0f;
            }
        } else if (qq < q0) {  // min-Q twin, ties keep twin 0
#pragma unroll
            for (int s = 0; s < E; ++s) pw[sub + G * s] = e[s];
        }
    }
    __syncwarp();

    // ---- projection of the selected distribution (blocked layout j = E sub + s)
    const float r = rv ? a.reward[row] : 0.0f;
    const float done = rv ? a.terminated[row] : 0.0f;
    const float g = rv ? a.discount[row] : 0.0f;
    const float ent = rv ? __fmul_rn(alpha, a.next_log_pi[row]) : -INFINITY;
    ent_max = fmaxf(ent_max, ent);
    const float cont = __fsub_rn(1.0f, done);
    int kl[E], ku[E];
    float ml[E], mu[E];
#pragma unroll
    for (int s = 0; s < E; ++s) {
        const int j = E * sub + s;
        if (rv && j < bins) {
            float v = __fadd_rn(r, __fmul_rn(__fmul_rn(g, __fsub_rn(z_s[j], ent)), cont));
            v = fminf(fmaxf(v, a.min_v), a.max_v);
            const float b = __fdiv_rn(__fsub_rn(v, a.min_v), width);
            const int lower = static_cast<int>(floorf(b));
            const int upper = min(max(lower + 1, 0), bins - 1);
            const float frac = __fsub_rn(b, static_cast<float>(lower));
            const float p = pw[j];
            kl[s] = lower;
            ku[s] = upper;
            ml[s] = __fmul_rn(p, __fsub_rn(1.0f, frac));
            mu[s] = __fmul_rn(p, frac);
        } else {
            kl[s] = INT_MAX;
            ku[s] = INT_MAX;
            ml[s] = 0.0f;
            mu[s] = 0.0f;
        }
    }
    scatter_runs<G, E>(kl, ml, tw, bins, false);
    __syncwarp();
    scatter_runs<G, E>(ku, mu, tw, bins, true);
    __syncwarp();
    float tgt[E];
    float tsum = 0.0f;
#pragma unroll
    for (int s = 0; s < E; ++s) {
        const int k = sub + G * s;
        tgt[s] = k < bins ? tw[k] : 0.0f;
        tsum += tgt[s];
        if (a.target_out && rv && k < bins) a.target_out[static_cast<long long>(row) * a.target_row + k] = tgt[s];
    }
    tsum = gsum<G>(tsum);

    // ---- online twins at the current-observation row: CE and logits gradient
#pragma unroll
    for (int t = 0; t < 2; ++t) {
        const float* src = t == 0 ? o0 : o1;
        float x[E];
        float mx = -INFINITY;
#pragma unroll
        for (int s = 0; s < E; ++s) {
            const int k = sub + G * s;
            x[s] = (rv && k < bins) ? src[k] : -INFINITY;
            mx = fmaxf(mx, x[s]);
        }
        mx = gmax<G>(mx);
        float ex[E];
        float se = 0.0f;
#pragma unroll
        for (int s = 0; s < E; ++s) {
            ex[s] = (sub + G * s < bins) ? __expf(x[s] - mx) : 0.0f;
            se += ex[s];
        }
        se = gsum<G>(se);
        const float lse = mx + logf(se);
        const float inv = 1.0f / se;
        if (!rv) continue;
        float ce = 0.0f;
#pragma unroll
        for (int s = 0; s < E; ++s) {
            const int k = sub + G * s;
            if (k >= bins) continue;
            const float lp = x[s] - lse;
            ce -= tgt[s] * lp;
            const float grad = (ex[s] * inv * tsum - tgt[s]) * a.loss_weight;
            bias_acc[t][s] += grad;
            if (a.dlogits) a.dlogits[t * a.d_twin + static_cast<long long>(row) * a.d_row + k] = grad;
            if (a.d16) {
                const float sv = grad * scale16;
                overflow |= !(fabsf(sv) <= 65504.0f);
                a.d16[t * a.d16_twin + static_cast<long long>(row) * a.d16_row + k] = __float2half_rn(sv);
            }
            if (a.d_hi) {
                const float hi = __uint_as_float(__float_as_uint(grad) & 0xFFFFE000u);
                const long long o = t * a.dp_twin + static_cast<long long>(row) * a.dp_row + k;
                a.d_hi[o] = hi;
                a.d_lo[o] = grad - hi;
            }
        }
        loss_acc += ce;
    }
}

// Block partial row of the head-bias gradient [2][bins], loss and entropy maximum, then the
// two-level fixed-order cross-block reduction (groups of kGroup blocks by ticket).
template <int G, int E>
__device__ __forceinline__ void finish(const Args& a, float (&bias_acc)[2][E], float loss_acc, float ent_max,
                                       bool overflow, float (*red_s)[2 * G * E + 2], bool& last_s) {
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int sub = lane & (G - 1);
    const int rg = lane / G;
    const int bins = a.bins;
    if (overflow && a.health) atomicOr(a.health, kHealthOverflow);

    // ---- block partial row: bias gradient [2][bins], loss, max entropy
    // (the row groups of a warp hold the same atoms: xor G .. 16 combine them)
#pragma unroll
    for (int t = 0; t < 2; ++t)
#pragma unroll
        for (int s = 0; s < E; ++s) {
            float v = bias_acc[t][s];
#pragma unroll
            for (int d = G; d < 32; d <<= 1) v += __shfl_xor_sync(0xffffffffu, v, d);
            if (rg == 0) red_s[warp][t * G * E + sub + G * s] = v;
        }
    {
        const float l = warp_sum(loss_acc) * a.loss_weight;
        const float e = warp_max(ent_max);
        if (lane == 0) {
            red_s[warp][2 * G * E] = l;
            red_s[warp][2 * G * E + 1] = e;
        }
    }
    __syncthreads();
    const int W = 2 * bins + 2;
    float* rows = a.partial;
    const int grid = static_cast<int>(gridDim.x);
    const int groups = (grid + kGroup - 1) / kGroup;
    float* group_rows = a.partial + static_cast<long long>(grid) * W;
    for (int i = threadIdx.x; i < W; i += kThreads) {
        float s;
        if (i < 2 * bins) {
            const int t = i / bins, k = i % bins;
            s = 0.0f;
            for (int w = 0; w < kWarps; ++w) s += red_s[w][t * G * E + k];
        } else if (i == 2 * bins) {
            s = 0.0f;
            for (int w = 0; w < kWarps; ++w) s += red_s[w][2 * G * E];
        } else {
            s = -INFINITY;
            for (int w = 0; w < kWarps; ++w) s = fmaxf(s, red_s[w][2 * G * E + 1]);
        }
        rows[static_cast<long long>(blockIdx.x) * W + i] = s;
    }
    // ---- first level: the last block of the group sums the group's rows in block order
    const int grp = blockIdx.x / kGroup;
    const int first = grp * kGroup;
    const int members = min(kGroup, grid - first);
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) last_s = atomicAdd(a.counter + 1 + grp, 1u) == static_cast<unsigned>(members - 1);
    __syncthreads();
    if (!last_s) return;
    __threadfence();
    for (int i = threadIdx.x; i < W; i += kThreads) {
        const bool is_max = i == 2 * bins + 1;
        float v[kGroup];
#pragma unroll
        for (int b = 0; b < kGroup; ++b) v[b] = b < members ? __ldcg(rows + static_cast<long long>(first + b) * W + i) : 0.0f;
        float s = is_max ? -INFINITY : 0.0f;
#pragma unroll
        for (int b = 0; b < kGroup; ++b)
            if (b < members) s = is_max ? fmaxf(s, v[b]) : s + v[b];
        group_rows[static_cast<long long>(grp) * W + i] = s;
    }
    if (threadIdx.x == 0) a.counter[1 + grp] = 0u;
    // ---- second level: the last group sums the group rows in group order
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) last_s = atomicAdd(a.counter, 1u) == static_cast<unsigned>(groups - 1);
    __syncthreads();
    if (!last_s) return;
    __threadfence();
    for (int i = threadIdx.x; i < W; i += kThreads) {
        const bool is_max = i == 2 * bins + 1;
        float s = is_max ? -INFINITY : 0.0f;
        for (int g0 = 0; g0 < groups; g0 += 8) {
            float v[8];
#pragma unroll
            for (int u = 0; u < 8; ++u)
                v[u] = g0 + u < groups ? __ldcg(group_rows + static_cast<long long>(g0 + u) * W + i) : 0.0f;
#pragma unroll
            for (int u = 0; u < 8; ++u)
                if (g0 + u < groups) s = is_max ? fmaxf(s, v[u]) : s + v[u];
        }
        if (i < 2 * bins) {
            if (a.bias_grad_out) a.bias_grad_out[i] = a.bias_accumulate ? a.bias_grad_out[i] + s : s;
        } else if (i == 2 * bins) {
            if (a.loss_out) a.loss_out[0] = s;
        } else {
            if (a.max_entropy_out) a.max_entropy_out[0] = s;
        }
    }
    if (threadIdx.x == 0) a.counter[0] = 0u;
}

template <int G, int E>
__global__ void __launch_bounds__(kThreads) critic_objective_kernel(const Args a) {
    constexpr int P = pitch<G, E>();
    constexpr int R = 32 / G;  // rows per warp
    __shared__ float z_s[G * E];
    __shared__ float p_s[kWarps][R][P];  // selected target distribution (strided write, blocked read)
    __shared__ float t_s[kWarps][R][P];  // projected target
    __shared__ float red_s[kWarps][2 * G * E + 2];
    __shared__ bool last_s;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int rg = lane / G;
    const int bins = a.bins;
    for (int k = threadIdx.x; k < G * E; k += kThreads) z_s[k] = k < bins ? a.support[k] : 0.0f;
    __syncthreads();
    float* pw = p_s[warp][rg];
    float* tw = t_s[warp][rg];
    const float alpha = a.alpha[0];
    const float scale16 = a.d16 ? a.d16_scale[0] : 1.0f;
    float bias_acc[2][E];
#pragma unroll
    for (int t = 0; t < 2; ++t)
#pragma unroll
        for (int s = 0; s < E; ++s) bias_acc[t][s] = 0.0f;
    float loss_acc = 0.0f;
    float ent_max = -INFINITY;
    bool overflow = false;
    for (int base = (blockIdx.x * kWarps + warp) * R; base < a.batch; base += gridDim.x * kWarps * R) {
        const int row = base + rg;
        const float* tr = a.target_logits + static_cast<long long>(a.t_row0 + row) * a.t_row;
        const float* orow = a.online_logits + static_cast<long long>(row) * a.o_row;
        row_work<G, E>(a, tr, tr + a.t_twin, orow, orow + a.o_twin, row, row < a.batch, z_s, pw, tw, alpha, scale16,
                       bias_acc, loss_acc, ent_max, overflow);
        __syncwarp();  // the next rows overwrite this warp's shared rows
    }
    finish<G, E>(a, bias_acc, loss_acc, ent_max, overflow, red_s, last_s);
}

// Staged variant: persistent CTAs (three per SM) walk 16-row tiles; one thread copies each tile's four
// logits blocks (target twins 0 / 1 at the next-observation rows, online twins 0 / 1 at
// the current rows: contiguous row ranges) into a shared-memory stage with 1-D bulk
// asynchronous copies completing on the stage's mbarrier, kStages tiles ahead, so HBM
// reads stay in flight while the warps compute on an earlier stage. Row work and
// reduction are those of critic_objective_kernel (the same per-row results; the block
// sums visit rows in another fixed order, so they are deterministic but not bit-identical
// to that kernel's). Needs 16-byte aligned logits bases and row / twin strides that are
// multiples of four floats, and reads every row with its full stride (padding included);
// rl2_critic_objective falls back to critic_objective_kernel otherwise. Every mbarrier
// wait is bounded: on a timeout the health word records it, the block waits (bounded
// again) for its copies in flight, contributes what it has and returns.
constexpr int kStages = 2;
constexpr int kStageRows = 16;
constexpr int kStagedBlocksPerSm = 3;  // 16-row stages keep three CTAs (24 warps) on an SM

inline size_t staged_smem_bytes(long long t_row, long long o_row) {
    return static_cast<size_t>(kStages) * kStageRows * 2 * static_cast<size_t>(t_row + o_row) * sizeof(float);
}

template <int G, int E>
__global__ void __launch_bounds__(kThreads, kStagedBlocksPerSm) critic_objective_staged_kernel(const Args a, int tiles) {
    constexpr int P = pitch<G, E>();
    constexpr int R = 32 / G;
    constexpr int kPasses = kStageRows / (kWarps * R) > 0 ? kStageRows / (kWarps * R) : 1;
    static_assert(kPasses * kWarps * R >= kStageRows, "every row of a stage is processed");
    extern __shared__ __align__(128) float stage_s[];  // [kStages][target twin 0 | 1 | online twin 0 | 1][kStageRows]
    __shared__ float z_s[G * E];
    __shared__ float p_s[kWarps][R][P];
    __shared__ float t_s[kWarps][R][P];
    __shared__ float red_s[kWarps][2 * G * E + 2];
    __shared__ __align__(8) uint64_t full_s[kStages];
    __shared__ bool last_s;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int rg = lane / G;
    const int bins = a.bins;
    const int tr = static_cast<int>(a.t_row), orr = static_cast<int>(a.o_row);
    const int stage_floats = kStageRows * 2 * (tr + orr);
    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) ptx::mbar_init(&full_s[s], 1);
        ptx::fence_barrier_init();
    }
    for (int k = threadIdx.x; k < G * E; k += kThreads) z_s[k] = k < bins ? a.support[k] : 0.0f;
    __syncthreads();

    // thread 0: arm stage i % kStages and copy local tile i into it
    auto issue = [&](int i) {
        const int r0 = (blockIdx.x + i * static_cast<int>(gridDim.x)) * kStageRows;
        const int rows = min(kStageRows, a.batch - r0);
        float* st = stage_s + (i % kStages) * stage_floats;
        const uint32_t tb = static_cast<uint32_t>(rows * tr) * 4u, ob = static_cast<uint32_t>(rows * orr) * 4u;
        uint64_t* bar = &full_s[i % kStages];
        ptx::mbar_arrive_expect_tx(bar, 2u * (tb + ob));
        const float* t = a.target_logits + static_cast<long long>(a.t_row0 + r0) * tr;
        const float* o = a.online_logits + static_cast<long long>(r0) * orr;
        ptx::bulk_load(st, t, tb, bar);
        ptx::bulk_load(st + kStageRows * tr, t + a.t_twin, tb, bar);
        ptx::bulk_load(st + 2 * kStageRows * tr, o, ob, bar);
        ptx::bulk_load(st + 2 * kStageRows * tr + kStageRows * orr, o + a.o_twin, ob, bar);
    };
    const int mine = blockIdx.x < tiles ? (tiles - 1 - static_cast<int>(blockIdx.x)) / static_cast<int>(gridDim.x) + 1
                                        : 0;
    int issued = 0;
    if (threadIdx.x == 0)
        for (; issued < min(kStages, mine); ++issued) issue(issued);

    float* pw = p_s[warp][rg];
    float* tw = t_s[warp][rg];
    const float alpha = a.alpha[0];
    const float scale16 = a.d16 ? a.d16_scale[0] : 1.0f;
    float bias_acc[2][E];
#pragma unroll
    for (int t = 0; t < 2; ++t)
#pragma unroll
        for (int s = 0; s < E; ++s) bias_acc[t][s] = 0.0f;
    float loss_acc = 0.0f;
    float ent_max = -INFINITY;
    bool overflow = false;
    int done = 0;
    for (int i = 0; i < mine; ++i) {
        const int s = i % kStages;
        const bool got = ptx::mbar_wait(&full_s[s], static_cast<uint32_t>((i / kStages) & 1), a.health);
        if (!__syncthreads_and(got)) break;
        const float* st = stage_s + s * stage_floats;
#pragma unroll 1
        for (int pass = 0; pass < kPasses; ++pass) {
            const int lr = (pass * kWarps + warp) * R + rg;
            const int row = lr < kStageRows ? (blockIdx.x + i * static_cast<int>(gridDim.x)) * kStageRows + lr : a.batch;
            const float* t0 = st + lr * tr;
            const float* o0 = st + 2 * kStageRows * tr + lr * orr;
            row_work<G, E>(a, t0, t0 + kStageRows * tr, o0, o0 + kStageRows * orr, row, row < a.batch, z_s, pw, tw,
                           alpha, scale16, bias_acc, loss_acc, ent_max, overflow);
            __syncwarp();  // the next pass overwrites this warp's shared rows
        }
        done = i + 1;
        __syncthreads();  // every warp is done with stage s
        if (threadIdx.x == 0 && issued < mine) {
            ptx::fence_proxy_async_smem();
            issue(issued++);
        }
    }
    // copies armed but not consumed (only after a timeout) land before the block exits
    if (threadIdx.x == 0)
        for (int i = done; i < issued; ++i)
            ptx::mbar_wait(&full_s[i % kStages], static_cast<uint32_t>((i / kStages) & 1), nullptr);
    __syncthreads();
    finish<G, E>(a, bias_acc, loss_acc, ent_max, overflow, red_s, last_s);
}

constexpr size_t kSmemPerBlock = 232448;  // opt-in dynamic + static shared memory one CTA may use

inline int sm_count() {
    int dev = 0, n = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n > 0 ? n : 148;
}

// The staged kernel reads whole row ranges with bulk copies: 16-byte aligned bases and
// strides that are multiples of four floats, and stages that fit next to the static arrays.
inline bool staged_ok(const rl2_critic_objective_args* g) {
    const auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
    if (!a16(g->target_logits) || !a16(g->online_logits)) return false;
    if (g->target_row_stride % 4 || g->online_row_stride % 4 || g->target_twin_stride % 4 ||
        g->online_twin_stride % 4 || g->target_row_stride < g->bins || g->online_row_stride < g->bins)
        return false;
    return staged_smem_bytes(g->target_row_stride, g->online_row_stride) + 48 * 1024 <= kSmemPerBlock;
}

template <int G, int E>
inline int launch(const Args& a, const rl2_critic_objective_args* g, int grid, cudaStream_t s) {
    if (staged_ok(g)) {
        const int tiles = (g->batch + kStageRows - 1) / kStageRows;
        // the caller's workspace holds grid_for(batch) partial rows
        const int sg = std::min({tiles, kStagedBlocksPerSm * sm_count(), grid});
        const size_t smem = staged_smem_bytes(g->target_row_stride, g->online_row_stride);
        if (cudaFuncSetAttribute(critic_objective_staged_kernel<G, E>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(smem)) != cudaSuccess) {
            set_error("critic objective: cannot reserve %zu bytes of shared memory", smem);
            return -1;
        }
        critic_objective_staged_kernel<G, E><<<sg, kThreads, smem, s>>>(a, tiles);
        return launch_status("critic objective (staged)");
    }
    critic_objective_kernel<G, E><<<grid, kThreads, 0, s>>>(a);
    return launch_status("critic objective");
}

// Lanes per transition row: 16 (E = ceil(bins / 16) atoms per lane, fewer registers per
// thread, so more warps per SM to hide the latency of the row's reductions and scans).
constexpr int kLanes = 16;

inline int dispatch(const Args& a, const rl2_critic_objective_args* g, int grid, cudaStream_t s) {
    if (kLanes == 16) {
        const int e = (g->bins + 15) / 16;
        if (e <= 2) return launch<16, 2>(a, g, grid, s);
        if (e <= 4) return launch<16, 4>(a, g, grid, s);
        if (e <= 7) return launch<16, 7>(a, g, grid, s);
        return launch<16, 8>(a, g, grid, s);
    }
    const int e = (g->bins + 7) / 8;
    if (e <= 4) return launch<8, 4>(a, g, grid, s);
    if (e <= 8) return launch<8, 8>(a, g, grid, s);
    if (e <= 13) return launch<8, 13>(a, g, grid, s);
    return launch<8, 16>(a, g, grid, s);
}

}  // namespace cat
}  // namespace rl2

extern "C" int rl2_categorical_workspace_floats(int batch, int bins) {
    const int grid = rl2::cat::grid_for(batch);
    return (grid + rl2::cat::groups_for(grid)) * (2 * bins + 2);
}

extern "C" int rl2_categorical_counter_words(int batch, int bins) {
    (void)bins;
    return 1 + rl2::cat::groups_for(rl2::cat::grid_for(batch));
}

extern "C" int rl2_critic_objective(const rl2_critic_objective_args* g, void* stream) {
    using namespace rl2;
    clear_error();
    if (!g || !g->target_logits || !g->online_logits || !g->reward || !g->terminated || !g->discount ||
        !g->next_log_pi || !g->alpha || !g->support || !g->workspace || !g->counter) {
        set_error("critic objective: null input or workspace");
        return -1;
    }
    if (g->bins < 2 || g->bins > cat::kMaxBins || g->batch < 1 || !(g->min_v < g->max_v)) {
        set_error("critic objective supports 2..%d atoms, batch >= 1 and min_v < max_v", cat::kMaxBins);
        return -1;
    }
    if ((g->d_hi == nullptr) != (g->d_lo == nullptr) || (g->d16 && !g->d16_scale)) {
        set_error("critic objective: tf32 planes need both hi and lo; fp16 output needs a scale");
        return -1;
    }
    cat::Args a{};
    a.target_logits = g->target_logits;
    a.t_row = g->target_row_stride;
    a.t_twin = g->target_twin_stride;
    a.t_row0 = g->target_row_offset;
    a.online_logits = g->online_logits;
    a.o_row = g->online_row_stride;
    a.o_twin = g->online_twin_stride;
    a.reward = g->reward;
    a.terminated = g->terminated;
    a.discount = g->discount;
    a.next_log_pi = g->next_log_pi;
    a.alpha = g->alpha;
    a.support = g->support;
    a.min_v = static_cast<float>(g->min_v);
    a.max_v = static_cast<float>(g->max_v);
    a.width = static_cast<float>((g->max_v - g->min_v) / static_cast<double>(g->bins - 1));
    a.bins = g->bins;
    a.batch = g->batch;
    a.loss_weight = g->loss_weight;
    a.dlogits = g->dlogits;
    a.d_row = g->dlogits_row_stride;
    a.d_twin = g->dlogits_twin_stride;
    a.d16 = reinterpret_cast<__half*>(g->d16);
    a.d16_row = g->d16_row_stride;
    a.d16_twin = g->d16_twin_stride;
    a.d16_scale = g->d16_scale;
    a.d_hi = g->d_hi;
    a.d_lo = g->d_lo;
    a.dp_row = g->dplane_row_stride;
    a.dp_twin = g->dplane_twin_stride;
    a.target_out = g->target_out;
    a.target_row = g->target_out_row_stride;
    a.partial = g->workspace;
    a.counter = g->counter;
    a.loss_out = g->loss_out;
    a.max_entropy_out = g->max_entropy_out;
    a.bias_grad_out = g->bias_grad_out;
    a.bias_accumulate = g->bias_grad_accumulate;
    a.health = g->health;
    return cat::dispatch(a, g, cat::grid_for(g->batch), as_stream(stream));
}

// ===========================================================================
// Allocation-free variant of rl2_critic_objective.
//
// Some callers cannot allocate device memory where they need this objective: a
// robot controller's real-time loop must not stall in the driver's allocator, and
// a host that embeds this library inside another framework may own all device
// memory through that framework's pool with no hook to hand out a workspace. This
// entry point needs no workspace from them: its block partials and completion
// counter live in the file-scope array below, which every GPU that loads the
// library holds until the process exits (about 0.65 MB).
//
// Limits: batch <= kNoAllocMaxBatch rows and bins <= 128 atoms; larger sizes are
// rejected with an error. The array's device address is looked up
// (cudaGetSymbolAddress) with the caller's device current on every call made outside
// stream capture, and remembered per driver context; a call made while its stream is
// being captured uses the address remembered for the current context, so make one
// call on each device (and again after a cudaDeviceReset, or in any other context
// the host makes current) before capturing a stream. The stream must belong to the
// current device; a stream of another device is rejected. All calls share the one
// array and it keeps the last call's contents: the counters are cleared at the start
// of every call (the partials are fully rewritten before they are read), and calls
// that overlap on the GPU (concurrent streams, or concurrent host threads) race on
// it, so issue them in order on one stream.
// ===========================================================================
#include <mutex>

namespace rl2 {
namespace cat {

constexpr int kNoAllocMaxBatch = 65536;
constexpr int kNoAllocGroups = (kMaxGrid + kGroup - 1) / kGroup;  // same grid rule as rl2_critic_objective
// partial rows (162,282 floats), rounded up to 64 floats so the counter words that
// follow start on a 256-byte boundary like the array itself
constexpr int kNoAllocFloats = ((kMaxGrid + kNoAllocGroups) * (2 * kMaxBins + 2) + 63) / 64 * 64;
constexpr int kNoAllocCounterPad = 64;  // counter words (1 + groups <= 64)
static_assert(kNoAllocFloats % 64 == 0, "counter words must start 256-byte aligned");
static_assert(1 + kNoAllocGroups <= kNoAllocCounterPad, "counter pad too small");

static __device__ __align__(256) float g_noalloc_scratch[kNoAllocFloats + kNoAllocCounterPad];

namespace {
using CtxGetCurrent = int (*)(void**);  // CUresult cuCtxGetCurrent(CUcontext*)

std::mutex g_noalloc_mutex;
struct NoAllocEntry {
    void* context;
    void* address;
};
NoAllocEntry g_noalloc_cache[64] = {};
int g_noalloc_next = 0;

CtxGetCurrent ctx_get_current() {
    static CtxGetCurrent fn = [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return static_cast<CtxGetCurrent>(nullptr);
        return reinterpret_cast<CtxGetCurrent>(p);
    }();
    return fn;
}
}  // namespace

// Device address of the scratch array in the current driver context. Outside capture
// the address is looked up afresh (so a reset device or another context never gets a
// stale address) and remembered for the context; during capture the remembered one is
// used, as no lookup may run then.
static float* noalloc_scratch(bool capturing) {
    void* ctx = nullptr;
    const CtxGetCurrent get = ctx_get_current();
    if (!get || get(&ctx) != 0 || !ctx) {
        set_error("critic objective (no-alloc): no current CUDA context");
        return nullptr;
    }
    std::lock_guard<std::mutex> lock(g_noalloc_mutex);
    NoAllocEntry* slot = nullptr;
    for (auto& e : g_noalloc_cache)
        if (e.context == ctx) slot = &e;
    if (capturing) {
        if (!slot) {
            set_error("critic objective (no-alloc): the first call in this CUDA context was made during stream "
                      "capture; make one call outside capture first");
            return nullptr;
        }
        return static_cast<float*>(slot->address);
    }
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p) {
        set_error("critic objective (no-alloc): cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
        return nullptr;
    }
    if (!slot) {
        slot = &g_noalloc_cache[g_noalloc_next];
        g_noalloc_next = (g_noalloc_next + 1) % 64;
    }
    slot->context = ctx;
    slot->address = p;
    return static_cast<float*>(p);
}

}  // namespace cat
}  // namespace rl2

extern "C" int rl2_critic_objective_noalloc(const rl2_critic_objective_args* g, void* stream) {
    using namespace rl2;
    clear_error();
    if (!g) {
        set_error("critic objective (no-alloc): null arguments");
        return -1;
    }
    if (g->batch < 1 || g->batch > cat::kNoAllocMaxBatch || g->bins < 2 || g->bins > cat::kMaxBins) {
        set_error("critic objective (no-alloc): batch must be in [1, %d] and bins in [2, %d] (got batch %d, bins %d)",
                  cat::kNoAllocMaxBatch, cat::kMaxBins, g->batch, g->bins);
        return -1;
    }
    int device = -1, stream_device = -1;
    if (cudaGetDevice(&device) != cudaSuccess || device < 0) {
        set_error("critic objective (no-alloc): no current CUDA device");
        return -1;
    }
    if (cudaStreamGetDevice(as_stream(stream), &stream_device) != cudaSuccess || stream_device != device) {
        cudaGetLastError();
        set_error("critic objective (no-alloc): the stream belongs to device %d, not to the current device %d",
                  stream_device, device);
        return -1;
    }
    cudaStreamCaptureStatus capture = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(as_stream(stream), &capture) != cudaSuccess) {
        set_error("critic objective (no-alloc): cannot query the stream's capture status");
        return -1;
    }
    float* scratch = cat::noalloc_scratch(capture != cudaStreamCaptureStatusNone);
    if (!scratch) return -1;
    unsigned* counter = reinterpret_cast<unsigned*>(scratch + cat::kNoAllocFloats);
    if (cudaMemsetAsync(counter, 0, sizeof(unsigned) * (1 + cat::kNoAllocGroups), as_stream(stream)) != cudaSuccess) {
        set_error("critic objective (no-alloc): clearing the completion counters failed");
        return -1;
    }
    rl2_critic_objective_args a = *g;
    a.workspace = scratch;
    a.counter = counter;
    return rl2_critic_objective(&a, stream);
}
