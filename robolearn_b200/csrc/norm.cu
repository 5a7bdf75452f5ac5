// Batch norm (training / evaluation), RMS post-norm and column-sum helpers for
// the residual MLPs. Reference semantics: src/robolearn/flashsac/layers.py:32-81
// and :189-240; reference native kernels: src/robolearn/cuda/flash_kernels.cuh:142-379.
//
// Column statistics travel as per-32-row-group partials (the same layout the
// GEMM epilogue writes), merged in a fixed order, so every reduction is
// deterministic run to run and needs no atomics. The element-wise passes are
// plain HBM-streaming kernels: one thread per (row, column) with consecutive
// threads on consecutive columns (coalesced), grid-stride over rows.

#include "planes.cuh"

#include <algorithm>

namespace rl2 {
namespace norm {

constexpr int kT = 256;
constexpr int kRowRegs = 16;  // row values a lane keeps in registers (rows up to 512 columns)

__device__ __forceinline__ void chan_merge(float& n_a, float& mean_a, float& m2_a, float n_b, float mean_b,
                                           float m2_b) {
    if (n_b <= 0.0f) return;
    const float n = n_a + n_b;
    const float delta = mean_b - mean_a;
    mean_a = mean_a + delta * (n_b / n);
    m2_a = m2_a + m2_b + delta * delta * (n_a * n_b / n);
    n_a = n;
}

// grid (ceil(cols/kT), G, twins)
__global__ void colstats_kernel(const float* __restrict__ x, long long ldx, long long xt, int rows, int cols,
                                float* __restrict__ mean_p, float* __restrict__ m2_p, long long pt) {
    const int c = blockIdx.x * kT + threadIdx.x;
    const int g = blockIdx.y;
    const int t = blockIdx.z;
    if (c >= cols) return;
    const int r0 = g * 32;
    const int n = min(32, rows - r0);
    const float* src = x + t * xt + static_cast<long long>(r0) * ldx + c;
    float s = 0.0f;
    for (int i = 0; i < n; ++i) s += src[i * ldx];
    const float mean = s / static_cast<float>(n);
    float m2 = 0.0f;
    for (int i = 0; i < n; ++i) {
        const float d = src[i * ldx] - mean;
        m2 += d * d;
    }
    const long long o = t * pt + static_cast<long long>(g) * cols + c;
    mean_p[o] = mean;
    m2_p[o] = m2;
}

// grid (ceil(cols/32), twins), 8 warps: lane = column, warp w merges a contiguous
// range of groups in order, then warp 0 merges the 8 results in order (deterministic).
// Group g of the partials lives at (g / gpr) * rs + (g % gpr) * cols: gpr groups per rank,
// rank blocks rs floats apart (one rank: gpr = groups, rs = 0).
// Warps merge contiguous group ranges (eight groups loaded ahead of the merge), then a
// fixed pairwise tree over the warps: with NT = 1024 a 256-group column takes 8 sequential
// merges and 5 tree levels.
template <int NT>
__global__ void __launch_bounds__(NT) finalize_kernel(const float* __restrict__ mean_p, const float* __restrict__ m2_p,
                                                      long long pt, int gpr, long long rs, int twins, int rows,
                                                      int cols, float* mean, float* invstd, float* rm, float* rv,
                                                      float momentum, float eps, int update) {
    constexpr int NW = NT / 32;
    __shared__ float sh[3][NW][32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int c = blockIdx.x * 32 + lane;
    const int t = blockIdx.y;
    const int groups = (rows + 31) / 32;
    const int per = (groups + NW - 1) / NW;
    const int g0 = warp * per, g1 = min(groups, g0 + per);
    float n = 0.0f, mu = 0.0f, m2 = 0.0f;
    if (c < cols) {
        const float* mp = mean_p + t * pt + c;
        const float* qp = m2_p + t * pt + c;
        // eight groups' partials are loaded before they are merged (same merge order)
        for (int g = g0; g < g1; g += 8) {
            float pm[8], pq[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int gg = g + j;
                const long long o = static_cast<long long>(gg / gpr) * rs + static_cast<long long>(gg % gpr) * cols;
                pm[j] = gg < g1 ? mp[o] : 0.0f;
                pq[j] = gg < g1 ? qp[o] : 0.0f;
            }
#pragma unroll
            for (int j = 0; j < 8; ++j)
                if (g + j < g1) chan_merge(n, mu, m2, static_cast<float>(min(32, rows - (g + j) * 32)), pm[j], pq[j]);
        }
    }
    sh[0][warp][lane] = n;
    sh[1][warp][lane] = mu;
    sh[2][warp][lane] = m2;
#pragma unroll
    for (int w = NW / 2; w >= 1; w >>= 1) {
        __syncthreads();
        if (warp < w) {
            chan_merge(n, mu, m2, sh[0][warp + w][lane], sh[1][warp + w][lane], sh[2][warp + w][lane]);
            sh[0][warp][lane] = n;
            sh[1][warp][lane] = mu;
            sh[2][warp][lane] = m2;
        }
    }
    if (warp != 0 || c >= cols) return;
    const int i = t * cols + c;
    const float var = m2 / static_cast<float>(rows);
    mean[i] = mu;
    invstd[i] = 1.0f / sqrtf(var + eps);
    if (update) {
        const float unbiased = var * (static_cast<float>(rows) / static_cast<float>(rows - 1));
        rm[i] = rm[i] + momentum * (mu - rm[i]);
        rv[i] = rv[i] + momentum * (unbiased - rv[i]);
    }
}

__global__ void eval_prepare_kernel(const float* rm, const float* rv, long long count, float eps, float* mean,
                                    float* invstd) {
    const long long i = blockIdx.x * static_cast<long long>(kT) + threadIdx.x;
    if (i >= count) return;
    mean[i] = rm[i];
    invstd[i] = 1.0f / sqrtf(rv[i] + eps);
}

__global__ void apply_kernel(const rl2_bn_apply_args a, const Plane plane) {
    PlaneWriter pw(plane);
    const long long per_twin = static_cast<long long>(a.rows) * a.cols;
    const long long total = per_twin * a.twins;
    for (long long i = blockIdx.x * static_cast<long long>(kT) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * kT) {
        const int t = static_cast<int>(i / per_twin);
        const long long rc = i % per_twin;
        const long long r = rc / a.cols;
        const int c = static_cast<int>(rc % a.cols);
        const int tc = t * a.cols + c;
        const float xv = a.x[t * a.x_twin_stride + r * a.ldx + c];
        float y = (xv - a.mean[tc]) * a.invstd[tc] * a.gamma[tc] + a.beta[tc];
        if (a.relu) y = fmaxf(y, 0.0f);
        if (a.residual) y += a.residual[t * a.residual_twin_stride + r * a.ldr + c];
        if (a.y) a.y[t * a.y_twin_stride + r * a.ldy + c] = y;
        if (pw.active()) pw.store(t, r, c, y);
    }
    pw.flush();
}

__device__ __forceinline__ float4 ld4(const float* p) { return *reinterpret_cast<const float4*>(p); }

// Vectorised apply: four columns per thread, 32-bit index math, grid.y = twin.
__global__ void __launch_bounds__(kT) apply_vec4_kernel(const rl2_bn_apply_args a, const Plane plane) {
    PlaneWriter pw(plane);
    const int t = blockIdx.y;
    const int c4n = a.cols >> 2;
    const int total = a.rows * c4n;
    const float* x = a.x + t * a.x_twin_stride;
    const float* res = a.residual ? a.residual + t * a.residual_twin_stride : nullptr;
    float* y = a.y ? a.y + t * a.y_twin_stride : nullptr;
    const int tc0 = t * a.cols;
    for (int i = blockIdx.x * kT + threadIdx.x; i < total; i += gridDim.x * kT) {
        const int r = i / c4n;
        const int c = (i - r * c4n) << 2;
        const float4 xv = ld4(x + static_cast<long long>(r) * a.ldx + c);
        const float4 mu = ld4(a.mean + tc0 + c), is = ld4(a.invstd + tc0 + c);
        const float4 g = ld4(a.gamma + tc0 + c), b = ld4(a.beta + tc0 + c);
        float4 o = make_float4((xv.x - mu.x) * is.x * g.x + b.x, (xv.y - mu.y) * is.y * g.y + b.y,
                               (xv.z - mu.z) * is.z * g.z + b.z, (xv.w - mu.w) * is.w * g.w + b.w);
        if (a.relu) o = make_float4(fmaxf(o.x, 0.f), fmaxf(o.y, 0.f), fmaxf(o.z, 0.f), fmaxf(o.w, 0.f));
        if (res) {
            const float4 rv = ld4(res + static_cast<long long>(r) * a.ldr + c);
            o = make_float4(o.x + rv.x, o.y + rv.y, o.z + rv.z, o.w + rv.w);
        }
        if (y) *reinterpret_cast<float4*>(y + static_cast<long long>(r) * a.ldy + c) = o;
        if (pw.active()) pw.store4(t, r, c, o);
    }
    pw.flush();
}

// Vectorised backward apply (twins kept separate, or summed into one output when sum_twins).
__global__ void __launch_bounds__(kT) bwd_apply_vec4_kernel(const rl2_bn_backward_args a, const Plane plane) {
    PlaneWriter pw(plane);
    const int to = blockIdx.y;
    const int c4n = a.cols >> 2;
    const int total = a.rows * c4n;
    const int t_begin = a.sum_twins ? 0 : to, t_end = a.sum_twins ? a.twins : to + 1;
    for (int i = blockIdx.x * kT + threadIdx.x; i < total; i += gridDim.x * kT) {
        const int r = i / c4n;
        const int c = (i - r * c4n) << 2;
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        for (int t = t_begin; t < t_end; ++t) {
            const int tc = t * a.cols + c;
            const float4 xv = ld4(a.x + t * a.x_twin_stride + static_cast<long long>(r) * a.ldx + c);
            const float4 dv = ld4(a.dy + t * a.dy_twin_stride + static_cast<long long>(r) * a.lddy + c);
            const float4 mu = ld4(a.mean + tc), is = ld4(a.invstd + tc), g = ld4(a.gamma + tc), b = ld4(a.beta + tc);
            const float xs[4] = {xv.x, xv.y, xv.z, xv.w}, ds[4] = {dv.x, dv.y, dv.z, dv.w};
            const float ms[4] = {mu.x, mu.y, mu.z, mu.w}, iv[4] = {is.x, is.y, is.z, is.w};
            const float gs[4] = {g.x, g.y, g.z, g.w}, bs[4] = {b.x, b.y, b.z, b.w};
            float c1[4] = {0.f, 0.f, 0.f, 0.f}, c2[4] = {0.f, 0.f, 0.f, 0.f};
            if (a.training) {
                const float4 p1 = ld4(a.coef1 + tc), p2 = ld4(a.coef2 + tc);
                c1[0] = p1.x; c1[1] = p1.y; c1[2] = p1.z; c1[3] = p1.w;
                c2[0] = p2.x; c2[1] = p2.y; c2[2] = p2.z; c2[3] = p2.w;
            }
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float xhat = (xs[j] - ms[j]) * iv[j];
                float d = ds[j];
                if (a.relu && !(xhat * gs[j] + bs[j] > 0.0f)) d = 0.0f;
                acc[j] += a.training ? gs[j] * iv[j] * (d - c1[j] - xhat * c2[j]) : gs[j] * iv[j] * d;
            }
        }
        const float4 o = make_float4(acc[0], acc[1], acc[2], acc[3]);
        if (a.dx) *reinterpret_cast<float4*>(a.dx + to * a.dx_twin_stride + static_cast<long long>(r) * a.lddx + c) = o;
        if (pw.active()) pw.store4(to, r, c, o);
    }
    pw.flush();
}

// d(normalised output) for one element: dy masked by the ReLU of the recomputed output
__device__ __forceinline__ float masked_dbn(const rl2_bn_backward_args& a, int t, long long r, int c, float& xhat) {
    const int tc = t * a.cols + c;
    const float xv = a.x[t * a.x_twin_stride + r * a.ldx + c];
    xhat = (xv - a.mean[tc]) * a.invstd[tc];
    float d = a.dy[t * a.dy_twin_stride + r * a.lddy + c];
    if (a.relu && !(xhat * a.gamma[tc] + a.beta[tc] > 0.0f)) d = 0.0f;
    return d;
}

// grid (ceil(cols/kT), G, twins)
__global__ void bwd_reduce_kernel(const rl2_bn_backward_args a) {
    const int c = blockIdx.x * kT + threadIdx.x;
    const int g = blockIdx.y;
    const int t = blockIdx.z;
    if (c >= a.cols) return;
    const int r0 = g * 32;
    const int n = min(32, a.rows - r0);
    float s1 = 0.0f, s2 = 0.0f;
    int i = 0;
    {  // eight rows' loads in flight before they are used (same per-row arithmetic and order)
        const int tc = t * a.cols + c;
        const float mu = a.mean[tc], is = a.invstd[tc], ga = a.gamma[tc], be = a.beta[tc];
        for (; i + 8 <= n; i += 8) {
            float xv[8], dv[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const long long r = r0 + i + k;
                xv[k] = a.x[t * a.x_twin_stride + r * a.ldx + c];
                dv[k] = a.dy[t * a.dy_twin_stride + r * a.lddy + c];
            }
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const float xhat = (xv[k] - mu) * is;
                float d = dv[k];
                if (a.relu && !(xhat * ga + be > 0.0f)) d = 0.0f;
                s1 += d;
                s2 += d * xhat;
            }
        }
    }
    for (; i < n; ++i) {
        float xhat;
        const float d = masked_dbn(a, t, r0 + i, c, xhat);
        s1 += d;
        s2 += d * xhat;
    }
    const int groups = (a.rows + 31) / 32;
    const long long o = (static_cast<long long>(t) * groups + g) * a.cols + c;
    a.s1_part[o] = s1;
    a.s2_part[o] = s2;
}

// grid (ceil(cols/32), twins), 8 warps over contiguous group ranges, fixed-order combine.
template <int NT>
__global__ void __launch_bounds__(NT) bwd_finalize_kernel(const float* s1p, const float* s2p, long long pt, int gpr,
                                                          long long rs, int twins, int rows, int cols, float* dgamma,
                                                          float* dbeta, long long gts, int accumulate, float* coef1,
                                                          float* coef2) {
    constexpr int NW = NT / 32;
    __shared__ float sh[2][NW][32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int c = blockIdx.x * 32 + lane;
    const int t = blockIdx.y;
    const int groups = (rows + 31) / 32;
    const int per = (groups + NW - 1) / NW;
    const int g0 = warp * per, g1 = min(groups, g0 + per);
    float s1 = 0.0f, s2 = 0.0f;
    if (c < cols) {
        for (int g = g0; g < g1; g += 8) {
            float a[8], b[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int gg = g + j;
                const long long o = static_cast<long long>(t) * pt + static_cast<long long>(gg / gpr) * rs +
                                    static_cast<long long>(gg % gpr) * cols + c;
                a[j] = gg < g1 ? s1p[o] : 0.0f;
                b[j] = gg < g1 ? s2p[o] : 0.0f;
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                if (g + j < g1) {
                    s1 += a[j];
                    s2 += b[j];
                }
            }
        }
    }
    sh[0][warp][lane] = s1;
    sh[1][warp][lane] = s2;
#pragma unroll
    for (int w = NW / 2; w >= 1; w >>= 1) {
        __syncthreads();
        if (warp < w) {
            s1 += sh[0][warp + w][lane];
            s2 += sh[1][warp + w][lane];
            sh[0][warp][lane] = s1;
            sh[1][warp][lane] = s2;
        }
    }
    if (warp != 0 || c >= cols) return;
    const int i = t * cols + c;
    if (dgamma) dgamma[t * gts + c] = accumulate ? dgamma[t * gts + c] + s2 : s2;
    if (dbeta) dbeta[t * gts + c] = accumulate ? dbeta[t * gts + c] + s1 : s1;
    if (coef1) coef1[i] = s1 / static_cast<float>(rows);
    if (coef2) coef2[i] = s2 / static_cast<float>(rows);
}

__global__ void bwd_apply_kernel(const rl2_bn_backward_args a, const Plane plane) {
    PlaneWriter pw(plane);
    const int twins_out = a.sum_twins ? 1 : a.twins;
    const long long per_twin = static_cast<long long>(a.rows) * a.cols;
    const long long total = per_twin * twins_out;
    for (long long i = blockIdx.x * static_cast<long long>(kT) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * kT) {
        const int to = static_cast<int>(i / per_twin);
        const long long rc = i % per_twin;
        const long long r = rc / a.cols;
        const int c = static_cast<int>(rc % a.cols);
        float acc = 0.0f;
        const int t_begin = a.sum_twins ? 0 : to;
        const int t_end = a.sum_twins ? a.twins : to + 1;
        for (int t = t_begin; t < t_end; ++t) {
            const int tc = t * a.cols + c;
            float xhat;
            const float d = masked_dbn(a, t, r, c, xhat);
            float dx;
            if (a.training)
                dx = a.gamma[tc] * a.invstd[tc] * (d - a.coef1[tc] - xhat * a.coef2[tc]);
            else
                dx = a.gamma[tc] * a.invstd[tc] * d;
            acc += dx;
        }
        if (a.dx) a.dx[to * a.dx_twin_stride + r * a.lddx + c] = acc;
        if (pw.active()) pw.store(to, r, c, acc);
    }
    pw.flush();
}

// one warp per row
__global__ void rms_forward_kernel(const float* __restrict__ h, long long ldh, long long ht, int twins, int rows,
                                   int cols, const float* __restrict__ gamma, float eps, float* __restrict__ r_out,
                                   float* __restrict__ u, long long ldu, long long ut, const Plane plane) {
    PlaneWriter pw(plane);
    const int lane = threadIdx.x & 31;
    const long long warps = static_cast<long long>(gridDim.x) * (kT / 32);
    for (long long w = blockIdx.x * static_cast<long long>(kT / 32) + (threadIdx.x >> 5); w < static_cast<long long>(twins) * rows;
         w += warps) {
        const int t = static_cast<int>(w / rows);
        const long long r = w % rows;
        const float* src = h + t * ht + r * ldh;
        float ss = 0.0f;
        for (int c = lane; c < cols; c += 32) ss += src[c] * src[c];
        ss = warp_sum(ss);
        const float rr = 1.0f / sqrtf(ss / static_cast<float>(cols) + eps);
        if (lane == 0) r_out[w] = rr;
        for (int c = lane; c < cols; c += 32) {
            const float v = src[c] * rr * gamma[t * cols + c];
            if (u) u[t * ut + r * ldu + c] = v;
            if (pw.active()) pw.store(t, r, c, v);
        }
    }
    pw.flush();
}

__global__ void rms_backward_kernel(const float* __restrict__ du, long long lddu, long long dut,
                                    const float* __restrict__ h, long long ldh, long long ht,
                                    const float* __restrict__ rv, const float* __restrict__ gamma, int twins, int rows,
                                    int cols, float* __restrict__ dh, long long lddh, long long dht) {
    const int lane = threadIdx.x & 31;
    const long long warps = static_cast<long long>(gridDim.x) * (kT / 32);
    for (long long w = blockIdx.x * static_cast<long long>(kT / 32) + (threadIdx.x >> 5); w < static_cast<long long>(twins) * rows;
         w += warps) {
        const int t = static_cast<int>(w / rows);
        const long long r = w % rows;
        const float* d = du + t * dut + r * lddu;
        const float* x = h + t * ht + r * ldh;
        const float* g = gamma + t * cols;
        float s = 0.0f;
        float* o = dh + t * dht + r * lddh;
        if (cols <= 32 * kRowRegs) {
            // the row's values loaded once, all in flight before the (sequential) sum
            float gv[kRowRegs], dv[kRowRegs], xv[kRowRegs];
#pragma unroll
            for (int q = 0; q < kRowRegs; ++q) {
                const int c = lane + 32 * q;
                if (c < cols) gv[q] = g[c], dv[q] = d[c], xv[q] = x[c];
            }
#pragma unroll
            for (int q = 0; q < kRowRegs; ++q)
                if (lane + 32 * q < cols) s += gv[q] * dv[q] * xv[q];
            s = warp_sum(s);
            const float rr = rv[w];
            const float k = rr * rr * rr * s / static_cast<float>(cols);
#pragma unroll
            for (int q = 0; q < kRowRegs; ++q) {
                const int c = lane + 32 * q;
                if (c < cols) o[c] = rr * gv[q] * dv[q] - xv[q] * k;
            }
            continue;
        }
        for (int c = lane; c < cols; c += 32) s += g[c] * d[c] * x[c];
        s = warp_sum(s);
        const float rr = rv[w];
        const float k = rr * rr * rr * s / static_cast<float>(cols);
        for (int c = lane; c < cols; c += 32) o[c] = rr * g[c] * d[c] - x[c] * k;
    }
}

// grid (ceil(cols/kT), G, twins): per-group column sums of du * h * r
__global__ void rms_dgamma_kernel(const float* __restrict__ du, long long lddu, long long dut,
                                  const float* __restrict__ h, long long ldh, long long ht,
                                  const float* __restrict__ rv, int rows, int cols, float* __restrict__ part) {
    const int c = blockIdx.x * kT + threadIdx.x;
    const int g = blockIdx.y;
    const int t = blockIdx.z;
    if (c >= cols) return;
    const int r0 = g * 32;
    const int n = min(32, rows - r0);
    float s = 0.0f;
    int i = 0;
    for (; i + 8 <= n; i += 8) {  // eight rows' loads in flight before they are added in order
        float a[8], b[8], q[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const long long r = r0 + i + k;
            a[k] = du[t * dut + r * lddu + c];
            b[k] = h[t * ht + r * ldh + c];
            q[k] = rv[static_cast<long long>(t) * rows + r];
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) s += a[k] * b[k] * q[k];
    }
    for (; i < n; ++i) {
        const long long r = r0 + i;
        s += du[t * dut + r * lddu + c] * h[t * ht + r * ldh + c] * rv[static_cast<long long>(t) * rows + r];
    }
    const int groups = (rows + 31) / 32;
    part[(static_cast<long long>(t) * groups + g) * cols + c] = s;
}

// out[t][c] (+)= sum_g part[t][g][c]. Block (32 columns, twin t); warp w sums the contiguous
// group range w of 32 (lane = column, coalesced rows), then warp 0 adds the partial sums
// in warp order: a fixed order for given (groups, cols).
constexpr int kColsumThreads = 1024;

__global__ void __launch_bounds__(kColsumThreads) colsum_finalize_kernel(const float* part, int twins, int groups,
                                                                        int cols, float* out, long long ots,
                                                                        int accumulate) {
    constexpr int kW = kColsumThreads / 32;
    __shared__ float sh[kW][32];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t = blockIdx.y;
    const int c = blockIdx.x * 32 + lane;
    const int per = (groups + kW - 1) / kW;
    const int g0 = min(warp * per, groups), g1 = min(g0 + per, groups);
    float s = 0.0f;
    if (c < cols) {
        const float* src = part + static_cast<long long>(t) * groups * cols + c;
        // eight groups' loads in flight before they are added (the sum stays sequential in g)
        int g = g0;
        for (; g + 8 <= g1; g += 8) {
            float x[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) x[k] = src[static_cast<long long>(g + k) * cols];
#pragma unroll
            for (int k = 0; k < 8; ++k) s = s + x[k];
        }
        for (; g < g1; ++g) s += src[static_cast<long long>(g) * cols];
    }
    sh[warp][lane] = s;
    __syncthreads();
    if (warp == 0 && c < cols) {
        float r = 0.0f;
#pragma unroll
        for (int w = 0; w < kW; ++w) r += sh[w][lane];
        float* o = out + t * ots + c;
        *o = accumulate ? *o + r : r;
    }
}

inline bool a16(const void* p) { return p == nullptr || aligned(p, 16); }
inline bool m4(long long v) { return (v & 3) == 0; }

// Whether a plane can take 4-column stores (fp16: 8-byte pairs; tf32: float4 pairs).
inline bool plane_vec4(const rl2_plane& p) {
    if (!plane_used(&p)) return true;
    if (!m4(p.ld) || !m4(p.twin_stride)) return false;
    return p.h16 ? aligned(p.h16, 8) : (aligned(p.hi, 16) && aligned(p.lo, 16));
}

inline bool apply_vec4(const rl2_bn_apply_args& a) {
    return m4(a.cols) && m4(a.ldx) && m4(a.x_twin_stride) && m4(a.ldr) && m4(a.residual_twin_stride) && m4(a.ldy) &&
           m4(a.y_twin_stride) && a16(a.x) && a16(a.residual) && a16(a.y) && a16(a.mean) && a16(a.invstd) &&
           a16(a.gamma) && a16(a.beta) && plane_vec4(a.plane) &&
           static_cast<long long>(a.rows) * a.cols < (1LL << 31);
}

inline bool backward_vec4(const rl2_bn_backward_args& a) {
    return m4(a.cols) && m4(a.ldx) && m4(a.x_twin_stride) && m4(a.lddy) && m4(a.dy_twin_stride) && m4(a.lddx) &&
           m4(a.dx_twin_stride) && a16(a.x) && a16(a.dy) && a16(a.dx) && a16(a.mean) && a16(a.invstd) &&
           a16(a.gamma) && a16(a.beta) && a16(a.coef1) && a16(a.coef2) && plane_vec4(a.plane) &&
           static_cast<long long>(a.rows) * a.cols < (1LL << 31);
}

inline int stream_blocks(long long work) {
    return static_cast<int>(std::max<long long>(1, std::min<long long>((work + kT - 1) / kT, 148LL * 16)));
}

}  // namespace norm
}  // namespace rl2

using namespace rl2;

extern "C" int rl2_colstats(const float* x, long long ldx, long long xt, int twins, int rows, int cols, float* mean_p,
                            float* m2_p, long long pt, void* stream) {
    clear_error();
    if (!x || !mean_p || !m2_p || twins < 1 || rows < 1 || cols < 1) {
        set_error("colstats: null buffer or empty shape");
        return -1;
    }
    const dim3 grid((cols + norm::kT - 1) / norm::kT, (rows + 31) / 32, twins);
    norm::colstats_kernel<<<grid, norm::kT, 0, as_stream(stream)>>>(x, ldx, xt, rows, cols, mean_p, m2_p, pt);
    return launch_status("column statistics");
}

extern "C" int rl2_bn_finalize_ranked(const float* mean_p, const float* m2_p, long long pt, int groups_per_rank,
                                      long long rank_stride, int twins, int rows, int cols, float* mean,
                                      float* invstd, float* rm, float* rv, float momentum, float eps, int update,
                                      void* stream) {
    clear_error();
    if (!mean_p || !m2_p || !mean || !invstd || twins < 1 || rows < 1 || cols < 1 || !(eps > 0.0f) ||
        groups_per_rank < 1 || rank_stride < 0 || (update && (!rm || !rv || rows < 2))) {
        set_error("bn finalize: invalid buffers or shape (running update needs rows >= 2)");
        return -1;
    }
    const dim3 grid((cols + 31) / 32, twins);
    if ((rows + 31) / 32 >= 128)
        norm::finalize_kernel<1024><<<grid, 1024, 0, as_stream(stream)>>>(
            mean_p, m2_p, pt, groups_per_rank, rank_stride, twins, rows, cols, mean, invstd, rm, rv, momentum, eps,
            update);
    else
        norm::finalize_kernel<norm::kT><<<grid, norm::kT, 0, as_stream(stream)>>>(
            mean_p, m2_p, pt, groups_per_rank, rank_stride, twins, rows, cols, mean, invstd, rm, rv, momentum, eps,
            update);
    return launch_status("batch-norm statistics");
}

extern "C" int rl2_bn_finalize(const float* mean_p, const float* m2_p, long long pt, int twins, int rows, int cols,
                               float* mean, float* invstd, float* rm, float* rv, float momentum, float eps,
                               int update, void* stream) {
    return rl2_bn_finalize_ranked(mean_p, m2_p, pt, (rows + 31) / 32, 0, twins, rows, cols, mean, invstd, rm, rv,
                                  momentum, eps, update, stream);
}

extern "C" int rl2_bn_eval_prepare(const float* rm, const float* rv, long long count, float eps, float* mean,
                                   float* invstd, void* stream) {
    clear_error();
    if (!rm || !rv || !mean || !invstd || count < 1) {
        set_error("bn eval prepare: invalid buffers");
        return -1;
    }
    norm::eval_prepare_kernel<<<static_cast<int>((count + norm::kT - 1) / norm::kT), norm::kT, 0,
                                as_stream(stream)>>>(rm, rv, count, eps, mean, invstd);
    return launch_status("batch-norm eval statistics");
}

extern "C" int rl2_bn_apply(const rl2_bn_apply_args* a, void* stream) {
    clear_error();
    if (!a || !a->x || !a->mean || !a->invstd || !a->gamma || !a->beta || a->twins < 1 || a->rows < 1 ||
        a->cols < 1 || !plane_valid(&a->plane) || (!a->y && !plane_used(&a->plane))) {
        set_error("bn apply: invalid arguments");
        return -1;
    }
    const long long work = static_cast<long long>(a->twins) * a->rows * a->cols;
    if (norm::apply_vec4(*a)) {
        const long long per_twin = static_cast<long long>(a->rows) * (a->cols / 4);
        const int blocks = std::max(1, norm::stream_blocks(per_twin) / a->twins);
        norm::apply_vec4_kernel<<<dim3(blocks, a->twins), norm::kT, 0, as_stream(stream)>>>(*a, to_plane(&a->plane));
        return launch_status("batch-norm apply");
    }
    norm::apply_kernel<<<norm::stream_blocks(work), norm::kT, 0, as_stream(stream)>>>(*a, to_plane(&a->plane));
    return launch_status("batch-norm apply");
}

extern "C" int rl2_bn_backward_reduce(const rl2_bn_backward_args* a, void* stream) {
    clear_error();
    if (!a || !a->dy || !a->x || !a->mean || !a->invstd || !a->gamma || !a->beta || !a->s1_part || !a->s2_part ||
        a->twins < 1 || a->rows < 1 || a->cols < 1) {
        set_error("bn backward reduce: invalid arguments");
        return -1;
    }
    const dim3 grid((a->cols + norm::kT - 1) / norm::kT, (a->rows + 31) / 32, a->twins);
    norm::bwd_reduce_kernel<<<grid, norm::kT, 0, as_stream(stream)>>>(*a);
    return launch_status("batch-norm backward reduce");
}

extern "C" int rl2_bn_backward_finalize_ranked(const float* s1p, const float* s2p, long long pt, int groups_per_rank,
                                               long long rank_stride, int twins, int rows, int cols, float* dgamma,
                                               float* dbeta, long long gts, int accumulate, float* coef1, float* coef2,
                                               void* stream) {
    clear_error();
    if (!s1p || !s2p || twins < 1 || rows < 1 || cols < 1 || groups_per_rank < 1 || rank_stride < 0) {
        set_error("bn backward finalize: invalid arguments");
        return -1;
    }
    const dim3 grid((cols + 31) / 32, twins);
    if ((rows + 31) / 32 >= 128)
        norm::bwd_finalize_kernel<1024><<<grid, 1024, 0, as_stream(stream)>>>(
            s1p, s2p, pt, groups_per_rank, rank_stride, twins, rows, cols, dgamma, dbeta, gts, accumulate, coef1, coef2);
    else
        norm::bwd_finalize_kernel<norm::kT><<<grid, norm::kT, 0, as_stream(stream)>>>(
            s1p, s2p, pt, groups_per_rank, rank_stride, twins, rows, cols, dgamma, dbeta, gts, accumulate, coef1, coef2);
    return launch_status("batch-norm backward finalize");
}

extern "C" int rl2_bn_backward_finalize(const float* s1p, const float* s2p, int twins, int rows, int cols,
                                        float* dgamma, float* dbeta, long long gts, int accumulate, float* coef1,
                                        float* coef2, void* stream) {
    const int groups = (rows + 31) / 32;
    return rl2_bn_backward_finalize_ranked(s1p, s2p, static_cast<long long>(groups) * cols, groups, 0, twins, rows,
                                           cols, dgamma, dbeta, gts, accumulate, coef1, coef2, stream);
}

extern "C" int rl2_bn_backward_apply(const rl2_bn_backward_args* a, void* stream) {
    clear_error();
    if (!a || !a->dy || !a->x || !a->mean || !a->invstd || !a->gamma || !a->beta || a->twins < 1 || a->rows < 1 ||
        a->cols < 1 || (a->training && (!a->coef1 || !a->coef2)) || !plane_valid(&a->plane) ||
        (!a->dx && !plane_used(&a->plane))) {
        set_error("bn backward apply: invalid arguments");
        return -1;
    }
    const long long work = static_cast<long long>(a->sum_twins ? 1 : a->twins) * a->rows * a->cols;
    if (norm::backward_vec4(*a)) {
        const int outs = a->sum_twins ? 1 : a->twins;
        const long long per_twin = static_cast<long long>(a->rows) * (a->cols / 4);
        const int blocks = std::max(1, norm::stream_blocks(per_twin) / outs);
        norm::bwd_apply_vec4_kernel<<<dim3(blocks, outs), norm::kT, 0, as_stream(stream)>>>(*a, to_plane(&a->plane));
        return launch_status("batch-norm backward apply");
    }
    norm::bwd_apply_kernel<<<norm::stream_blocks(work), norm::kT, 0, as_stream(stream)>>>(*a, to_plane(&a->plane));
    return launch_status("batch-norm backward apply");
}

extern "C" int rl2_rms_forward(const float* h, long long ldh, long long ht, int twins, int rows, int cols,
                               const float* gamma, float eps, float* r_out, float* u, long long ldu, long long ut,
                               const rl2_plane* plane, void* stream) {
    clear_error();
    if (!h || !gamma || !r_out || twins < 1 || rows < 1 || cols < 1 || !plane_valid(plane) ||
        (!u && !plane_used(plane))) {
        set_error("rms forward: invalid arguments");
        return -1;
    }
    const long long warps = static_cast<long long>(twins) * rows;
    norm::rms_forward_kernel<<<norm::stream_blocks(warps * 32), norm::kT, 0, as_stream(stream)>>>(
        h, ldh, ht, twins, rows, cols, gamma, eps, r_out, u, ldu, ut, to_plane(plane));
    return launch_status("rms forward");
}

extern "C" int rl2_rms_backward(const float* du, long long lddu, long long dut, const float* h, long long ldh,
                                long long ht, const float* r, const float* gamma, int twins, int rows, int cols,
                                float* dh, long long lddh, long long dht, float* dgamma_part, void* stream) {
    clear_error();
    if (!du || !h || !r || !gamma || !dh || twins < 1 || rows < 1 || cols < 1) {
        set_error("rms backward: invalid arguments");
        return -1;
    }
    const long long warps = static_cast<long long>(twins) * rows;
    norm::rms_backward_kernel<<<norm::stream_blocks(warps * 32), norm::kT, 0, as_stream(stream)>>>(
        du, lddu, dut, h, ldh, ht, r, gamma, twins, rows, cols, dh, lddh, dht);
    if (launch_status("rms backward")) return -1;
    if (dgamma_part) {
        const dim3 grid((cols + norm::kT - 1) / norm::kT, (rows + 31) / 32, twins);
        norm::rms_dgamma_kernel<<<grid, norm::kT, 0, as_stream(stream)>>>(du, lddu, dut, h, ldh, ht, r, rows, cols,
                                                                        dgamma_part);
    }
    return launch_status("rms weight gradient");
}

extern "C" int rl2_colsum_finalize(const float* part, int twins, int groups, int cols, float* out, long long ots,
                                   int accumulate, void* stream) {
    clear_error();
    if (!part || !out || twins < 1 || groups < 1 || cols < 1) {
        set_error("colsum finalize: invalid arguments");
        return -1;
    }
    norm::colsum_finalize_kernel<<<dim3((cols + 31) / 32, twins), norm::kColsumThreads, 0, as_stream(stream)>>>(
        part, twins, groups, cols, out, ots, accumulate);
    return launch_status("column-sum finalize");
}
