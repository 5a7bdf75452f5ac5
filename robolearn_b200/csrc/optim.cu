// Fused optimizer pass for one network: Adam -> weight-norm projection ->
// operand-plane refresh -> target EMA (+ target operand plane), one CTA per
// projection unit (a weight row, a BN (weight, bias) pair, an RMS scale, or a
// plain vector such as a head bias).
//
// Reference semantics (paths inside the reference project):
//   Adam (torch single-tensor)   torch.optim.Adam as used by src/robolearn/flashsac/agent.py:64-65,92-96
//   Adam (Warp-NN formula)       src/robolearn/cuda/kernels.cu:310-337
//   schedule                     src/robolearn/flashsac/_utils/scheduler.py:43-65 (LambdaLR, agent.py:66-69)
//   projection                   src/robolearn/flashsac/layers.py:24-29,57-64,76-81,186,217-240
//   target EMA                   src/robolearn/flashsac/_utils/network.py:66-80 (foreach lerp)
//   AMP skip / scale update      src/robolearn/cuda/kernels.cu:378-404 (GradScaler semantics)
// The reference runs these as separate passes (Adam, projection, EMA, fp16 casts);
// here each parameter element is read and written once per update.

#include "planes.cuh"

#include <algorithm>
#include <cmath>

namespace rl2 {
namespace optim {

constexpr int kT = 256;
constexpr int kPer = 16;  // elements per thread kept in registers -> rows up to 4096 (x2 for BN pairs)

// state layout (floats): [0] attempts, [1] successful steps, [2] step_size, [3] bc2_sqrt,
// [4] lr, [5] skip flag, [6] loss scale, [7] growth tracker, [8] attempts skipped
__global__ void prepare_kernel(const rl2_adam_prepare_args a) {
    float* st = a.state;
    const bool skip = a.found_inf && *a.found_inf != 0;
    const double attempts = static_cast<double>(st[0]);
    const double k = a.schedule_on_attempts ? attempts : static_cast<double>(st[1]);
    double lr;
    if (k < a.warmup_steps)
        lr = a.lr_init + (a.lr_peak - a.lr_init) * (k / a.warmup_steps);
    else if (k < a.decay_steps)
        lr = a.lr_end + (a.lr_peak - a.lr_end) * 0.5 *
                            (1.0 + cos(3.14159265358979323846 * (k - a.warmup_steps) / (a.decay_steps - a.warmup_steps)));
    else
        lr = a.lr_end;
    if (a.lr_override) lr = static_cast<double>(*a.lr_override);
    st[0] = static_cast<float>(attempts + 1.0);
    st[5] = skip ? 1.0f : 0.0f;
    if (!skip) {
        const double t = static_cast<double>(st[1]) + 1.0;
        st[1] = static_cast<float>(t);
        const double bc1 = 1.0 - pow(static_cast<double>(a.beta1), t);
        const double bc2 = 1.0 - pow(static_cast<double>(a.beta2), t);
        if (a.formula == 0) {
            st[2] = static_cast<float>(lr / bc1);
            st[3] = static_cast<float>(sqrt(bc2));
        } else {
            st[2] = static_cast<float>(1.0 / bc1);  // Warp-NN: c1, c2 multiply the moments
            st[3] = static_cast<float>(1.0 / bc2);
        }
    }
    st[4] = static_cast<float>(lr);
    if (a.scaler) {
        // dynamic loss scale: back off on overflow, grow after growth_interval clean steps
        float scale = st[6];
        float growth = st[7];
        if (skip) {
            scale = fmaxf(scale * a.backoff, 1.1754944e-38f);
            growth = 0.0f;
            st[8] = st[8] + 1.0f;
        } else {
            growth += 1.0f;
            if (growth >= static_cast<float>(a.growth_interval)) {
                const float grown = scale * a.growth;
                if (isfinite(grown)) scale = grown;
                growth = 0.0f;
            }
        }
        st[7] = growth;
        // the scale used by the next backward; inverse kept beside it for the products
        if (a.scale_out) a.scale_out[0] = scale;
        if (a.inv_scale_out) a.inv_scale_out[0] = 1.0f / scale;
        st[6] = scale;
    }
    if (a.found_inf) *a.found_inf = 0;
}

__device__ __forceinline__ float block_sum(float v, float* sh) {
    v = warp_sum(v);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) sh[w] = v;
    __syncthreads();
    float t = 0.0f;
    if (threadIdx.x < 32) {
        t = threadIdx.x < (kT / 32) ? sh[threadIdx.x] : 0.0f;
        t = warp_sum(t);
        if (threadIdx.x == 0) sh[0] = t;
    }
    __syncthreads();
    return sh[0];
}

__device__ __forceinline__ void plane_write(const Plane& p, long long off, float v) {
    if (p.h16) {
        p.h16[off] = __float2half_rn(v);
    } else if (p.hi) {
        const float h = tf32_hi(v);
        p.hi[off] = h;
        p.lo[off] = v - h;
    }
}

__global__ void __launch_bounds__(kT) step_kernel(const rl2_adam_args a, const Plane wp, const Plane tp) {
    __shared__ float sh[32];
    const rl2_segment seg = a.segments[blockIdx.x];
    const float* st = a.state;
    const bool update = a.state == nullptr || st[5] == 0.0f;
    const float step_size = a.state ? st[2] : 0.0f;
    const float bc2 = a.state ? st[3] : 1.0f;
    const int n = seg.length;
    const int vecs = seg.kind == 2 ? 2 : 1;
    float pv[2][kPer];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        if (h >= vecs) break;
        const long long base = h == 0 ? seg.offset : seg.offset2;
#pragma unroll
        for (int s = 0; s < kPer; ++s) {
            const int i = threadIdx.x + s * kT;
            if (i >= n) break;
            const long long o = base + i;
            float p = a.params[o];
            if (update && a.grads) {
                const float g = a.grads[o];
                float m = a.m[o], v = a.v[o];
                if (a.formula == 0) {
                    m = m + (1.0f - a.beta1) * (g - m);
                    v = v * a.beta2 + (1.0f - a.beta2) * g * g;
                    const float denom = sqrtf(v) / bc2 + a.eps;
                    p = p - step_size * (m / denom);
                } else {
                    m = a.beta1 * m + (1.0f - a.beta1) * g;
                    v = a.beta2 * v + (1.0f - a.beta2) * (g * g);
                    p = p - st[4] * ((m * step_size) / (sqrtf(v * bc2) + a.eps));
                }
                a.m[o] = m;
                a.v[o] = v;
            }
            pv[h][s] = p;
        }
    }
    // projection factor
    float factor = 1.0f;
    if (seg.kind != 0 && a.project) {
        float ss = 0.0f;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            if (h >= vecs) break;
#pragma unroll
            for (int s = 0; s < kPer; ++s) {
                const int i = threadIdx.x + s * kT;
                if (i < n) ss += pv[h][s] * pv[h][s];
            }
        }
        const float total = block_sum(ss, sh);
        if (seg.kind == 1) {
            factor = fmaxf(sqrtf(total), 1e-8f);  // divide (F.normalize, eps 1e-8)
        } else {
            factor = sqrtf(static_cast<float>(n)) * (1.0f / sqrtf(total + 1e-8f));
        }
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        if (h >= vecs) break;
        const long long base = h == 0 ? seg.offset : seg.offset2;
#pragma unroll
        for (int s = 0; s < kPer; ++s) {
            const int i = threadIdx.x + s * kT;
            if (i >= n) break;
            float p = pv[h][s];
            if (seg.kind == 1 && a.project)
                p = p / factor;
            else if (seg.kind != 0 && a.project)
                p = p * factor;
            a.params[base + i] = p;
            if (seg.plane_offset >= 0 && h == 0) plane_write(wp, seg.plane_offset + i, p);
            if (a.target_params) {
                const float t = a.target_params[base + i];
                const float nt = t + a.tau * (p - t);
                a.target_params[base + i] = nt;
                if (seg.plane_offset >= 0 && h == 0) plane_write(tp, seg.plane_offset + i, nt);
            }
        }
    }
}

}  // namespace optim
}  // namespace rl2

using namespace rl2;

extern "C" int rl2_adam_prepare(const rl2_adam_prepare_args* a, void* stream) {
    clear_error();
    if (!a || !a->state || !(a->decay_steps > 0) || a->warmup_steps < 0 || a->formula < 0 || a->formula > 1) {
        set_error("adam prepare: invalid arguments");
        return -1;
    }
    optim::prepare_kernel<<<1, 1, 0, as_stream(stream)>>>(*a);
    return launch_status("adam prepare");
}

extern "C" int rl2_adam_step(const rl2_adam_args* a, void* stream) {
    clear_error();
    if (!a || !a->params || !a->segments || a->count < 1 || (a->grads && (!a->m || !a->v)) ||
        !plane_valid(&a->weight_plane) || !plane_valid(&a->target_plane) || a->formula < 0 || a->formula > 1) {
        set_error("adam step: invalid arguments");
        return -1;
    }
    optim::step_kernel<<<a->count, optim::kT, 0, as_stream(stream)>>>(*a, to_plane(&a->weight_plane),
                                                                       to_plane(&a->target_plane));
    return launch_status("fused adam / projection / EMA");
}

extern "C" int rl2_segment_max_length(void) { return optim::kT * optim::kPer; }
