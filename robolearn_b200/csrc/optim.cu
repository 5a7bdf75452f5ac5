// Fused optimizer pass for one network: Adam -> weight-norm projection ->
// operand-plane refresh -> target EMA (+ target operand plane) per projection unit
// (a weight row, a BN (weight, bias) pair, an RMS scale, or a plain vector such as a
// head bias). Short units take one warp each, eight to a CTA; long ones a CTA each.
// Accesses are 16-byte vectors where the unit's rows allow (8-byte fp16 plane stores).
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
constexpr int kWarps = kT / 32;
constexpr int kSlots = 4;  // float4 slots per thread and vector: units up to 16 x 256 = 4096 elements per CTA,
                           // 16 x 32 = 512 per warp (x2 for BN pairs)

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

// Launch-wide scalars of one optimizer step.
struct StepScalars {
    bool update;
    float step_size, bc2, inv_bc2, lr, c1, c2;
};

// Square root and quotient on the special-function unit (sqrt.approx: about 1 ulp;
// __fdividef: 2 ulp for divisors in [2^-126, 2^126], which eps keeps the denominators in).
// The update is otherwise the reference's arithmetic, in the same order.
__device__ __forceinline__ float sqrt_approx(float x) {
    float r;
    asm("sqrt.approx.f32 %0, %1;" : "=f"(r) : "f"(x));
    return r;
}

__device__ __forceinline__ float adam(const rl2_adam_args& a, const StepScalars& s, float p, float g, float& m,
                                      float& v) {
    if (a.formula == 0) {
        m = m + s.c1 * (g - m);
        v = v * a.beta2 + s.c2 * g * g;
        const float denom = sqrt_approx(v) * s.inv_bc2 + a.eps;
        return p - s.step_size * __fdividef(m, denom);
    }
    m = a.beta1 * m + s.c1 * g;
    v = a.beta2 * v + s.c2 * (g * g);
    return p - s.lr * __fdividef(m * s.step_size, sqrt_approx(v * s.bc2) + a.eps);
}

// Slot (j, c) of thread t in a segment handled by G threads: on the vector path the
// thread owns the float4 at element 4 (t + j G) (c its component), on the scalar path
// element t + (4 j + c) G. Both cover 16 G elements per vector.
template <bool VEC, int G>
__device__ __forceinline__ int slot_index(int t, int j, int c) {
    return VEC ? 4 * (t + j * G) + c : t + (4 * j + c) * G;
}

template <bool VEC, int G>
__device__ __forceinline__ void load_slots(const float* __restrict__ src, int t, int j, int n, float* out) {
    if (VEC) {
        const int e = slot_index<true, G>(t, j, 0);
        if (e < n) {
            const float4 x = *reinterpret_cast<const float4*>(src + e);
            out[0] = x.x, out[1] = x.y, out[2] = x.z, out[3] = x.w;
        }
    } else {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const int e = slot_index<false, G>(t, j, c);
            if (e < n) out[c] = src[e];
        }
    }
}

template <bool VEC, int G>
__device__ __forceinline__ void store_slots(float* __restrict__ dst, int t, int j, int n, const float* in) {
    if (VEC) {
        const int e = slot_index<true, G>(t, j, 0);
        if (e < n) *reinterpret_cast<float4*>(dst + e) = make_float4(in[0], in[1], in[2], in[3]);
    } else {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const int e = slot_index<false, G>(t, j, c);
            if (e < n) dst[e] = in[c];
        }
    }
}

// Pulls the lines of a thread's slots into L2 (read later in the same pass).
template <bool VEC, int G>
__device__ __forceinline__ void prefetch_slots(const float* src, int t, int j, int n) {
    const int e = slot_index<VEC, G>(t, j, 0);
    if (e < n) asm volatile("prefetch.global.L2 [%0];" ::"l"(src + e));
}

// Operand-plane copy of four slots: fp16 (8-byte stores on the vector path) or tf32 hi + lo.
template <bool VEC, int G>
__device__ __forceinline__ void plane_slots(const Plane& p, long long off, int t, int j, int n, const float* in) {
    if (!p.h16 && !p.hi) return;
    if (VEC) {
        const int e = slot_index<true, G>(t, j, 0);
        if (e >= n) return;
        if (p.h16) {
            const __half2 a = __floats2half2_rn(in[0], in[1]), b = __floats2half2_rn(in[2], in[3]);
            uint2 u;
            u.x = *reinterpret_cast<const unsigned*>(&a);
            u.y = *reinterpret_cast<const unsigned*>(&b);
            *reinterpret_cast<uint2*>(p.h16 + off + e) = u;
        } else {
            float h[4], l[4];
#pragma unroll
            for (int c = 0; c < 4; ++c) h[c] = tf32_hi(in[c]), l[c] = in[c] - h[c];
            *reinterpret_cast<float4*>(p.hi + off + e) = make_float4(h[0], h[1], h[2], h[3]);
            *reinterpret_cast<float4*>(p.lo + off + e) = make_float4(l[0], l[1], l[2], l[3]);
        }
    } else {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const int e = slot_index<false, G>(t, j, c);
            if (e >= n) continue;
            if (p.h16) {
                p.h16[off + e] = __float2half_rn(in[c]);
            } else {
                const float h = tf32_hi(in[c]);
                p.hi[off + e] = h;
                p.lo[off + e] = in[c] - h;
            }
        }
    }
}

// One projection unit handled by G threads (a warp, or the whole CTA); PAIRED: a BN
// (weight, bias) pair of two vectors. Every element is read once (parameter, gradient,
// moments, target) and written once; the loads of a thread's slots are issued before any
// of them is used, and slots past the unit's end (the same for the whole group) are skipped.
template <bool VEC, int G, bool PAIRED>
__device__ __forceinline__ void run_segment(const rl2_adam_args& a, const Plane& wp, const Plane& tp,
                                            const rl2_segment& seg, const StepScalars& s, int t, float* sh) {
    constexpr int S = kSlots;
    constexpr int V = PAIRED ? 2 : 1;
    const int n = seg.length;
    const int used = (n + 4 * G - 1) / (4 * G);  // slots holding any element of the unit
    const bool adam_on = s.update && a.grads != nullptr;
    const bool ema = a.target_params != nullptr;
    float pv[V][4 * S];
    float ss = 0.0f;
#pragma unroll
    for (int h = 0; h < V; ++h) {
        const long long base = h == 0 ? seg.offset : seg.offset2;
        float gv[4 * S], mv[4 * S], vv[4 * S];
#pragma unroll
        for (int k = 0; k < 4 * S; ++k) pv[h][k] = 0.0f, gv[k] = 0.0f, mv[k] = 0.0f, vv[k] = 0.0f;
#pragma unroll
        for (int j = 0; j < S; ++j) {
            if (j >= used) break;
            load_slots<VEC, G>(a.params + base, t, j, n, &pv[h][4 * j]);
            if (adam_on) {
                load_slots<VEC, G>(a.grads + base, t, j, n, &gv[4 * j]);
                load_slots<VEC, G>(a.m + base, t, j, n, &mv[4 * j]);
                load_slots<VEC, G>(a.v + base, t, j, n, &vv[4 * j]);
            }
            if (ema) prefetch_slots<VEC, G>(a.target_params + base, t, j, n);
        }
        if (adam_on) {
#pragma unroll
            for (int j = 0; j < S; ++j) {
                if (j >= used) break;
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    const int k = 4 * j + c;
                    pv[h][k] = adam(a, s, pv[h][k], gv[k], mv[k], vv[k]);  // zeros stay zero
                }
                store_slots<VEC, G>(a.m + base, t, j, n, &mv[4 * j]);
                store_slots<VEC, G>(a.v + base, t, j, n, &vv[4 * j]);
            }
        }
#pragma unroll
        for (int j = 0; j < S; ++j) {
            if (j >= used) break;
#pragma unroll
            for (int c = 0; c < 4; ++c) ss += pv[h][4 * j + c] * pv[h][4 * j + c];  // unused slots hold zero
        }
    }
    // projection factor over the unit (both vectors of a BN pair): a multiplier
    float factor = 1.0f;
    if (seg.kind != 0 && a.project) {
        const float total = G == 32 ? warp_sum(ss) : block_sum(ss, sh);
        if (seg.kind == 1)
            factor = 1.0f / fmaxf(sqrtf(total), 1e-8f);  // F.normalize, eps 1e-8
        else
            factor = sqrtf(static_cast<float>(n)) * (1.0f / sqrtf(total + 1e-8f));
    }
#pragma unroll
    for (int h = 0; h < V; ++h) {
        const long long base = h == 0 ? seg.offset : seg.offset2;
        float tv[4 * S];
        if (ema) {  // every target slot requested before the first is used (lines already in L2)
#pragma unroll
            for (int j = 0; j < S; ++j) {
                if (j >= used) break;
                load_slots<VEC, G>(a.target_params + base, t, j, n, &tv[4 * j]);
            }
        }
#pragma unroll
        for (int j = 0; j < S; ++j) {
            if (j >= used) break;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const int k = 4 * j + c;
                pv[h][k] *= factor;
                if (ema) tv[k] = tv[k] + a.tau * (pv[h][k] - tv[k]);
            }
            store_slots<VEC, G>(a.params + base, t, j, n, &pv[h][4 * j]);
            if (ema) store_slots<VEC, G>(a.target_params + base, t, j, n, &tv[4 * j]);
            if (h == 0 && seg.plane_offset >= 0) {
                plane_slots<VEC, G>(wp, seg.plane_offset, t, j, n, &pv[h][4 * j]);
                if (ema) plane_slots<VEC, G>(tp, seg.plane_offset, t, j, n, &tv[4 * j]);
            }
        }
    }
}

__device__ __forceinline__ bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// The vector path needs every row start 16-byte aligned: length and offsets multiples of
// four floats on 16-byte aligned arrays (the fp16 plane then gets 8-byte aligned stores).
__device__ __forceinline__ bool vector_ok(const rl2_adam_args& a, const Plane& wp, const Plane& tp,
                                          const rl2_segment& seg) {
    bool ok = (seg.length & 3) == 0 && (seg.offset & 3) == 0 && (seg.kind != 2 || (seg.offset2 & 3) == 0);
    ok = ok && aligned16(a.params) && (a.grads == nullptr || (aligned16(a.grads) && aligned16(a.m) && aligned16(a.v)));
    ok = ok && (a.target_params == nullptr || aligned16(a.target_params));
    if (seg.plane_offset >= 0) {
        ok = ok && (seg.plane_offset & 3) == 0;
        ok = ok && (wp.h16 == nullptr || (reinterpret_cast<uintptr_t>(wp.h16) & 7u) == 0);
        ok = ok && (wp.hi == nullptr || (aligned16(wp.hi) && aligned16(wp.lo)));
        ok = ok && (tp.h16 == nullptr || (reinterpret_cast<uintptr_t>(tp.h16) & 7u) == 0);
        ok = ok && (tp.hi == nullptr || (aligned16(tp.hi) && aligned16(tp.lo)));
    }
    return ok;
}

// Grid: ceil(warp_segments / 8) CTAs whose warps take one of the leading warp_segments
// units each (lengths <= 16 x 32), then one CTA per remaining unit (lengths <= 16 x 256).
__global__ void __launch_bounds__(kT, 2) step_kernel(const rl2_adam_args a, const Plane wp, const Plane tp) {
    __shared__ float sh[32];
    StepScalars s;
    s.update = a.state == nullptr || a.state[5] == 0.0f;
    s.step_size = a.state ? a.state[2] : 0.0f;
    s.bc2 = a.state ? a.state[3] : 1.0f;
    s.inv_bc2 = 1.0f / s.bc2;
    s.lr = a.state ? a.state[4] : 0.0f;
    s.c1 = 1.0f - a.beta1;
    s.c2 = 1.0f - a.beta2;
    const int warp_blocks = (a.warp_segments + kWarps - 1) / kWarps;
    if (static_cast<int>(blockIdx.x) < warp_blocks) {
        const int idx = blockIdx.x * kWarps + (threadIdx.x >> 5);
        if (idx >= a.warp_segments) return;  // whole warp; the warp path has no block barrier
        const rl2_segment seg = a.segments[idx];
        if (seg.length > kSlots * 4 * 32) return;  // outside the warp path's contract (checked on the host)
        const int lane = threadIdx.x & 31;
        const bool vec = vector_ok(a, wp, tp, seg);
        if (seg.kind == 2)
            vec ? run_segment<true, 32, true>(a, wp, tp, seg, s, lane, nullptr)
                : run_segment<false, 32, true>(a, wp, tp, seg, s, lane, nullptr);
        else
            vec ? run_segment<true, 32, false>(a, wp, tp, seg, s, lane, nullptr)
                : run_segment<false, 32, false>(a, wp, tp, seg, s, lane, nullptr);
        return;
    }
    const rl2_segment seg = a.segments[a.warp_segments + (blockIdx.x - warp_blocks)];
    if (seg.length > kSlots * 4 * kT) return;  // block-uniform
    const bool vec = vector_ok(a, wp, tp, seg);
    if (seg.kind == 2)
        vec ? run_segment<true, kT, true>(a, wp, tp, seg, s, threadIdx.x, sh)
            : run_segment<false, kT, true>(a, wp, tp, seg, s, threadIdx.x, sh);
    else
        vec ? run_segment<true, kT, false>(a, wp, tp, seg, s, threadIdx.x, sh)
            : run_segment<false, kT, false>(a, wp, tp, seg, s, threadIdx.x, sh);
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
        !plane_valid(&a->weight_plane) || !plane_valid(&a->target_plane) || a->formula < 0 || a->formula > 1 ||
        a->warp_segments < 0 || a->warp_segments > a->count) {
        set_error("adam step: invalid arguments");
        return -1;
    }
    const int warp_blocks = (a->warp_segments + optim::kWarps - 1) / optim::kWarps;
    const int grid = warp_blocks + (a->count - a->warp_segments);
    optim::step_kernel<<<grid, optim::kT, 0, as_stream(stream)>>>(*a, to_plane(&a->weight_plane),
                                                                 to_plane(&a->target_plane));
    return launch_status("fused adam / projection / EMA");
}

extern "C" int rl2_segment_max_length(void) { return optim::kT * optim::kSlots * 4; }

extern "C" int rl2_segment_warp_max_length(void) { return 32 * optim::kSlots * 4; }
