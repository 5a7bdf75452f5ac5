// Fused categorical critic objective: two-hot Bellman target projection onto the
// fixed atom support + log-softmax cross-entropy + logits gradient, one pass.
//
// Reference semantics (all paths inside the reference project):
//   target selection  src/robolearn/flashsac/updates.py:19-31  (argmin over twins, tie -> twin 0)
//   projection        src/robolearn/flashsac/updates.py:34-80  (lower/upper split, scatter_add)
//   CE + gradient     src/robolearn/flashsac/updates.py:248-257 (mean over [2, B]; autograd)
//   native version    src/robolearn/cuda/categorical_kernels.cuh:87-114 (shared-memory atomics)
//
// Design: one warp per transition row. The target twin's log-softmax and
// expected value, the min-Q selection, the projection and the online twins'
// cross-entropy all stay in registers / per-warp shared memory; the only global
// traffic is the two logits reads and the gradient write. The projection is
// deterministic without atomics: the shifted atom values are monotone in the
// source atom index j, so every target atom receives a contiguous run of j and a
// warp segmented scan produces each run's sum in a fixed order.
// The float arithmetic of the bin location uses round-to-nearest intrinsics (no
// FMA contraction) in the reference's operation order, so lower/upper/fraction
// agree with Torch's float32 evaluation.

#include "common.cuh"
#include "../../include/rl2.h"

#include <algorithm>
#include <climits>

namespace rl2 {
namespace cat {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kMaxBins = 128;  // 4 atoms per lane

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
    float* partial;  // [grid][2*bins + 2]
    unsigned* counter;
    float* loss_out;
    float* max_entropy_out;
    float* bias_grad_out;
    int bias_accumulate;
    int* health;
};

// Warp segmented inclusive scan over 4 blocked elements per lane (element j = 4*lane + s)
// with monotone non-decreasing keys; writes each run's total to out[key] at the run's end.
__device__ __forceinline__ void scatter_runs(const int (&key)[4], const float (&val)[4], float* out, int bins) {
    const int lane = threadIdx.x & 31;
    float acc[4];
    acc[0] = val[0];
#pragma unroll
    for (int s = 1; s < 4; ++s) acc[s] = (key[s] == key[s - 1]) ? acc[s - 1] + val[s] : val[s];
    const int tail = key[3];
    float run = acc[3];
    bool open = key[0] == key[3];
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
        const int ok = __shfl_up_sync(0xffffffffu, tail, d);
        const float os = __shfl_up_sync(0xffffffffu, run, d);
        const int oo = __shfl_up_sync(0xffffffffu, static_cast<int>(open), d);
        if (lane >= d && open && ok == tail) {
            run = os + run;
            open = oo != 0;
        }
    }
    const int prev_tail = __shfl_up_sync(0xffffffffu, tail, 1);
    const float prev_run = __shfl_up_sync(0xffffffffu, run, 1);
    const float carry = (lane > 0 && prev_tail == key[0]) ? prev_run : 0.0f;
#pragma unroll
    for (int s = 0; s < 4; ++s)
        if (key[s] == key[0]) acc[s] = carry + acc[s];
    const int next_head = __shfl_down_sync(0xffffffffu, key[0], 1);
#pragma unroll
    for (int s = 0; s < 4; ++s) {
        const int nk = s < 3 ? key[s + 1] : (lane < 31 ? next_head : INT_MAX - 1);
        if (key[s] != nk && key[s] >= 0 && key[s] < bins) out[key[s]] = acc[s];
    }
}

__global__ void __launch_bounds__(kThreads) critic_objective_kernel(const Args a) {
    __shared__ float z_s[kMaxBins];
    __shared__ float p_s[kWarps][kMaxBins];
    __shared__ float lo_s[kWarps][kMaxBins];
    __shared__ float up_s[kWarps][kMaxBins];
    __shared__ float red_s[kWarps][2 * kMaxBins + 2];
    __shared__ bool last_block;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int bins = a.bins;
    for (int k = threadIdx.x; k < kMaxBins; k += kThreads) z_s[k] = k < bins ? a.support[k] : 0.0f;
    __syncthreads();

    const float alpha = a.alpha[0];
    const float scale16 = a.d16 ? a.d16_scale[0] : 1.0f;
    const float width = a.width;
    float bias_acc[2][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}};
    float loss_acc = 0.0f;
    float ent_max = -INFINITY;
    bool overflow = false;

    for (int row = blockIdx.x * kWarps + warp; row < a.batch; row += gridDim.x * kWarps) {
        // ---- target twins at the next-observation row: log-softmax and expected value
        float tl[2][4];
        float q[2];
#pragma unroll
        for (int t = 0; t < 2; ++t) {
            const float* src = a.target_logits + t * a.t_twin + static_cast<long long>(a.t_row0 + row) * a.t_row;
            float mx = -INFINITY;
#pragma unroll
            for (int s = 0; s < 4; ++s) {
                const int k = lane + 32 * s;
                tl[t][s] = k < bins ? src[k] : -INFINITY;
                mx = fmaxf(mx, tl[t][s]);
            }
            mx = warp_max(mx);
            float se = 0.0f;
#pragma unroll
            for (int s = 0; s < 4; ++s) se += (lane + 32 * s < bins) ? expf(tl[t][s] - mx) : 0.0f;
            const float lse = mx + logf(warp_sum(se));
            float qq = 0.0f;
#pragma unroll
            for (int s = 0; s < 4; ++s) {
                const int k = lane + 32 * s;
                const float lp = tl[t][s] - lse;
                tl[t][s] = k < bins ? expf(lp) : 0.0f;  // now probabilities
                qq += tl[t][s] * z_s[k];
            }
            q[t] = warp_sum(qq);
        }
        const int sel = q[1] < q[0] ? 1 : 0;
#pragma unroll
        for (int s = 0; s < 4; ++s) p_s[warp][lane + 32 * s] = sel ? tl[1][s] : tl[0][s];
#pragma unroll
        for (int s = 0; s < 4; ++s) {
            lo_s[warp][lane + 32 * s] = 0.0f;
            up_s[warp][lane + 32 * s] = 0.0f;
        }
        __syncwarp();

        // ---- projection of the selected distribution (blocked layout j = 4*lane + s)
        const float r = a.reward[row];
        const float done = a.terminated[row];
        const float g = a.discount[row];
        const float ent = __fmul_rn(alpha, a.next_log_pi[row]);
        ent_max = fmaxf(ent_max, ent);
        const float cont = __fsub_rn(1.0f, done);
        int kl[4], ku[4];
        float ml[4], mu[4];
#pragma unroll
        for (int s = 0; s < 4; ++s) {
            const int j = 4 * lane + s;
            if (j < bins) {
                float v = __fadd_rn(r, __fmul_rn(__fmul_rn(g, __fsub_rn(z_s[j], ent)), cont));
                v = fminf(fmaxf(v, a.min_v), a.max_v);
                const float b = __fdiv_rn(__fsub_rn(v, a.min_v), width);
                const int lower = static_cast<int>(floorf(b));
                const int upper = min(max(lower + 1, 0), bins - 1);
                const float frac = __fsub_rn(b, static_cast<float>(lower));
                const float p = p_s[warp][j];
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
        scatter_runs(kl, ml, lo_s[warp], bins);
        scatter_runs(ku, mu, up_s[warp], bins);
        __syncwarp();
        float tgt[4];
        float tsum = 0.0f;
#pragma unroll
        for (int s = 0; s < 4; ++s) {
            const int k = lane + 32 * s;
            tgt[s] = k < bins ? lo_s[warp][k] + up_s[warp][k] : 0.0f;
            tsum += tgt[s];
            if (a.target_out && k < bins) a.target_out[static_cast<long long>(row) * a.target_row + k] = tgt[s];
        }
        tsum = warp_sum(tsum);
        __syncwarp();

        // ---- online twins at the current-observation row: CE and logits gradient
#pragma unroll
        for (int t = 0; t < 2; ++t) {
            const float* src = a.online_logits + t * a.o_twin + static_cast<long long>(row) * a.o_row;
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
            float ce = 0.0f;
#pragma unroll
            for (int s = 0; s < 4; ++s) {
                const int k = lane + 32 * s;
                if (k >= bins) continue;
                const float lp = x[s] - lse;
                ce -= tgt[s] * lp;
                const float grad = (expf(lp) * tsum - tgt[s]) * a.loss_weight;
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
            loss_acc += warp_sum(ce) * a.loss_weight;
        }
    }
    if (overflow && a.health) atomicOr(a.health, kHealthOverflow);

    // ---- block partials: bias gradient [2][bins], loss, max entropy
#pragma unroll
    for (int t = 0; t < 2; ++t)
#pragma unroll
        for (int s = 0; s < 4; ++s) red_s[warp][t * kMaxBins + lane + 32 * s] = bias_acc[t][s];
    if (lane == 0) {
        red_s[warp][2 * kMaxBins] = loss_acc;
        red_s[warp][2 * kMaxBins + 1] = warp_max(ent_max);
    } else {
        (void)warp_max(ent_max);
    }
    __syncthreads();
    const int width_p = 2 * bins + 2;
    float* part = a.partial + static_cast<long long>(blockIdx.x) * width_p;
    for (int i = threadIdx.x; i < 2 * bins; i += kThreads) {
        const int t = i / bins, k = i % bins;
        float s = 0.0f;
        for (int w = 0; w < kWarps; ++w) s += red_s[w][t * kMaxBins + k];
        part[i] = s;
    }
    if (threadIdx.x == 0) {
        float l = 0.0f, e = -INFINITY;
        for (int w = 0; w < kWarps; ++w) {
            l += red_s[w][2 * kMaxBins];
            e = fmaxf(e, red_s[w][2 * kMaxBins + 1]);
        }
        part[2 * bins] = l;
        part[2 * bins + 1] = e;
    }
    // ---- last block reduces all block partials in a fixed order
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) last_block = atomicAdd(a.counter, 1u) == gridDim.x - 1;
    __syncthreads();
    if (!last_block) return;
    __threadfence();
    for (int i = threadIdx.x; i < width_p; i += kThreads) {
        float s = i == 2 * bins + 1 ? -INFINITY : 0.0f;
        for (unsigned b = 0; b < gridDim.x; ++b) {
            const float v = a.partial[static_cast<long long>(b) * width_p + i];
            s = (i == 2 * bins + 1) ? fmaxf(s, v) : s + v;
        }
        if (i < 2 * bins) {
            if (a.bias_grad_out) a.bias_grad_out[i] = a.bias_accumulate ? a.bias_grad_out[i] + s : s;
        } else if (i == 2 * bins) {
            if (a.loss_out) a.loss_out[0] = s;
        } else {
            if (a.max_entropy_out) a.max_entropy_out[0] = s;
        }
    }
    if (threadIdx.x == 0) *a.counter = 0u;
}

}  // namespace cat
}  // namespace rl2

extern "C" int rl2_categorical_workspace_floats(int batch, int bins) {
    const int grid = std::min((batch + rl2::cat::kWarps - 1) / rl2::cat::kWarps, 148 * 8);
    return grid * (2 * bins + 2);
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
    const int grid = std::min((g->batch + cat::kWarps - 1) / cat::kWarps, 148 * 8);
    cat::critic_objective_kernel<<<grid, cat::kThreads, 0, as_stream(stream)>>>(a);
    return launch_status("critic objective");
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
// library holds until the process exits (about 1.2 MB).
//
// Limits: batch <= kNoAllocMaxBatch rows and bins <= 128 atoms; larger sizes are
// rejected with an error. The first call on a device looks up the array's device
// address (cudaGetSymbolAddress) with that device current; make that first call
// before any stream capture. All calls share the one array and it keeps the last
// call's contents: the counter is cleared at the start of every call (the partials
// are fully rewritten before they are read), and calls that overlap on the GPU
// (concurrent streams, or concurrent host threads) race on it, so issue them in
// order on one stream.
// ===========================================================================
#include <mutex>

namespace rl2 {
namespace cat {

constexpr int kNoAllocMaxBatch = 65536;
constexpr int kNoAllocMaxGrid = 148 * 8;                        // same grid rule as rl2_critic_objective
constexpr int kNoAllocFloats = kNoAllocMaxGrid * (2 * kMaxBins + 2);  // 305,472 floats of block partials
constexpr int kNoAllocCounterPad = 64;                          // counter word kept 256-byte aligned

static __device__ __align__(256) float g_noalloc_scratch[kNoAllocFloats + kNoAllocCounterPad];

namespace {
std::mutex g_noalloc_mutex;
void* g_noalloc_addr[256] = {};
}  // namespace

// Device address of the scratch array for the current device (looked up once per device).
static float* noalloc_scratch(int device) {
    std::lock_guard<std::mutex> lock(g_noalloc_mutex);
    if (!g_noalloc_addr[device]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p) {
            set_error("critic objective (no-alloc): cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
            return nullptr;
        }
        g_noalloc_addr[device] = p;
    }
    return static_cast<float*>(g_noalloc_addr[device]);
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
    int device = -1;
    if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= 256) {
        set_error("critic objective (no-alloc): no current CUDA device");
        return -1;
    }
    float* scratch = cat::noalloc_scratch(device);
    if (!scratch) return -1;
    unsigned* counter = reinterpret_cast<unsigned*>(scratch + cat::kNoAllocFloats);
    if (cudaMemsetAsync(counter, 0, sizeof(unsigned), as_stream(stream)) != cudaSuccess) {
        set_error("critic objective (no-alloc): clearing the completion counter failed");
        return -1;
    }
    rl2_critic_objective_args a = *g;
    a.workspace = scratch;
    a.counter = counter;
    return rl2_critic_objective(&a, stream);
}
