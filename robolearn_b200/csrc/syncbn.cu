// Data-parallel batch-norm statistics exchanged through NVLink peer memory.
//
// One kernel per BN layer and direction. Block (slab of 32 columns, twin t), 8 warps:
// the warps merge this rank's per-32-row-group partials (contiguous group ranges,
// fixed order); warp 0 pushes the per-column entry into every rank's exchange slot
// with plain peer stores, raises one epoch flag per rank for its slab (system-scope release
// after a warp barrier), then polls its own slot's flags (acquire loads, bounded by wall-clock time)
// and merges the ranks' entries in rank order. Blocks never wait on one another, and a
// wait that runs out records kHealthTimeout and returns.

#include "common.cuh"
#include "../../include/rl2.h"

namespace rl2 {
namespace syncbn {

constexpr int kT = 256;
constexpr int kW = kT / 32;

__device__ __forceinline__ void chan_merge(float& n_a, float& mean_a, float& m2_a, float n_b, float mean_b,
                                           float m2_b) {
    if (n_b <= 0.0f) return;
    const float n = n_a + n_b;
    const float delta = mean_b - mean_a;
    mean_a = mean_a + delta * (n_b / n);
    m2_a = m2_a + m2_b + delta * delta * (n_a * n_b / n);
    n_a = n;
}

__device__ __forceinline__ unsigned long long load_acquire(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void store_release(unsigned long long* p, unsigned long long v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ uint64_t now_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Warp 0: push two per-column values of this rank to every rank, flag the slab, wait for
// every rank's flag of the slab. Returns false on a timeout (recorded in *health).
__device__ bool exchange(const rl2_syncbn_exchange& ex, int twins, int t, int cols, int c, float a, float b,
                         unsigned long long epoch) {
    const int lane = threadIdx.x & 31;
    const int W = ex.world;
    const int slabs = (cols + 31) / 32;
    const long long flag_index = (static_cast<long long>(t) * slabs + blockIdx.x) * W;
    if (c < cols) {
        for (int p = 0; p < W; ++p) {
            float* dst = ex.peer_data[p] + (static_cast<long long>(ex.rank) * twins + t) * 2 * cols;
            dst[c] = a;
            dst[cols + c] = b;
        }
    }
    // The warp barrier orders every lane's pushes before the flag stores; each flag store is
    // a system-scope release (cumulative over those pushes), so a peer that acquires the
    // flag sees this rank's entries without a full system fence here.
    __syncwarp();
    if (lane < W) store_release(ex.peer_flags[lane] + flag_index + ex.rank, epoch);
    bool ok = true;
    if (lane < W) {
        const unsigned long long* f = ex.peer_flags[ex.rank] + flag_index + lane;
        if (load_acquire(f) < epoch) {
            const uint64_t start = now_ns();
            const uint64_t limit = static_cast<uint64_t>(ex.timeout_s * 1e9f);
            for (uint32_t i = 1;; ++i) {
                if (load_acquire(f) >= epoch) break;
                if ((i & 255u) == 0 && now_ns() - start > limit) {
                    ok = false;
                    if (ex.health) atomicOr(ex.health, kHealthTimeout);
                    break;
                }
            }
        }
    }
    ok = __all_sync(0xffffffffu, ok);
    __syncwarp();  // every lane's reads of the entries follow the acquiring lanes' loads
    return ok;
}

// Epoch of this launch (read by every block before it takes its ticket) and advance by
// the last block to finish.
__device__ __forceinline__ unsigned long long launch_epoch(const rl2_syncbn_exchange& ex) {
    return static_cast<unsigned long long>(*reinterpret_cast<volatile unsigned int*>(ex.epoch)) + 1ull;
}

__device__ __forceinline__ void finish_launch(const rl2_syncbn_exchange& ex, unsigned long long epoch) {
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        const unsigned int blocks = gridDim.x * gridDim.y;
        const unsigned int ticket = atomicAdd(ex.epoch + 1, 1u);
        if (ticket == blocks - 1) {
            ex.epoch[1] = 0u;
            ex.epoch[0] = static_cast<unsigned int>(epoch);
        }
    }
}

__global__ void __launch_bounds__(kT) forward_kernel(const float* __restrict__ mean_p, const float* __restrict__ m2_p,
                                                     long long pt, int twins, int rows, int cols, float* mean,
                                                     float* invstd, float* rm, float* rv, float momentum, float eps,
                                                     int update, const rl2_syncbn_exchange ex) {
    __shared__ float sh[3][kW][32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int t = blockIdx.y;
    const int c = blockIdx.x * 32 + lane;
    const unsigned long long epoch = launch_epoch(ex);
    // this rank's groups, eight loaded ahead of the fixed-order merge
    const int groups = (rows + 31) / 32;
    const int per = (groups + kW - 1) / kW;
    const int g0 = min(warp * per, groups), g1 = min(g0 + per, groups);
    float n = 0.0f, mu = 0.0f, m2 = 0.0f;
    if (c < cols) {
        const float* mp = mean_p + t * pt + c;
        const float* qp = m2_p + t * pt + c;
        for (int g = g0; g < g1; g += 8) {
            float a[8], b[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                a[j] = g + j < g1 ? mp[static_cast<long long>(g + j) * cols] : 0.0f;
                b[j] = g + j < g1 ? qp[static_cast<long long>(g + j) * cols] : 0.0f;
            }
#pragma unroll
            for (int j = 0; j < 8; ++j)
                if (g + j < g1) chan_merge(n, mu, m2, static_cast<float>(min(32, rows - (g + j) * 32)), a[j], b[j]);
        }
    }
    sh[0][warp][lane] = n;
    sh[1][warp][lane] = mu;
    sh[2][warp][lane] = m2;
    __syncthreads();
    if (warp == 0) {
        n = sh[0][0][lane];
        mu = sh[1][0][lane];
        m2 = sh[2][0][lane];
        for (int w = 1; w < kW; ++w) chan_merge(n, mu, m2, sh[0][w][lane], sh[1][w][lane], sh[2][w][lane]);
        exchange(ex, twins, t, cols, c, mu, m2, epoch);
        if (c < cols) {
            // all ranks' entries, rank order (each rank holds `rows` rows)
            float gn = 0.0f, gmu = 0.0f, gm2 = 0.0f;
            const float* base = ex.peer_data[ex.rank];
            for (int r = 0; r < ex.world; ++r) {
                const float* src = base + (static_cast<long long>(r) * twins + t) * 2 * cols;
                chan_merge(gn, gmu, gm2, static_cast<float>(rows), __ldcv(src + c), __ldcv(src + cols + c));
            }
            const int i = t * cols + c;
            const float total = static_cast<float>(rows) * ex.world;
            const float var = gm2 / total;
            mean[i] = gmu;
            invstd[i] = 1.0f / sqrtf(var + eps);
            if (update) {
                const float unbiased = var * (total / (total - 1.0f));
                rm[i] = rm[i] + momentum * (gmu - rm[i]);
                rv[i] = rv[i] + momentum * (unbiased - rv[i]);
            }
        }
    }
    finish_launch(ex, epoch);
}

__global__ void __launch_bounds__(kT) backward_kernel(const float* __restrict__ s1p, const float* __restrict__ s2p,
                                                      long long pt, int twins, int rows, int cols, float* dgamma,
                                                      float* dbeta, long long gts, float* coef1, float* coef2,
                                                      const rl2_syncbn_exchange ex) {
    __shared__ float sh[2][kW][32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int t = blockIdx.y;
    const int c = blockIdx.x * 32 + lane;
    const unsigned long long epoch = launch_epoch(ex);
    const int groups = (rows + 31) / 32;
    const int per = (groups + kW - 1) / kW;
    const int g0 = min(warp * per, groups), g1 = min(g0 + per, groups);
    float s1 = 0.0f, s2 = 0.0f;
    if (c < cols) {
        const float* a = s1p + t * pt + c;
        const float* b = s2p + t * pt + c;
        for (int g = g0; g < g1; g += 8) {
            float x[8], y[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                x[j] = g + j < g1 ? a[static_cast<long long>(g + j) * cols] : 0.0f;
                y[j] = g + j < g1 ? b[static_cast<long long>(g + j) * cols] : 0.0f;
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                if (g + j < g1) {
                    s1 += x[j];
                    s2 += y[j];
                }
            }
        }
    }
    sh[0][warp][lane] = s1;
    sh[1][warp][lane] = s2;
    __syncthreads();
    if (warp == 0) {
        s1 = 0.0f;
        s2 = 0.0f;
        for (int w = 0; w < kW; ++w) {
            s1 += sh[0][w][lane];
            s2 += sh[1][w][lane];
        }
        // gamma / beta gradients of this rank's rows (averaged with the other gradients later)
        if (c < cols) {
            if (dgamma) dgamma[t * gts + c] = s2;
            if (dbeta) dbeta[t * gts + c] = s1;
        }
        exchange(ex, twins, t, cols, c, s1, s2, epoch);
        if (c < cols) {
            float g1s = 0.0f, g2s = 0.0f;
            const float* base = ex.peer_data[ex.rank];
            for (int r = 0; r < ex.world; ++r) {
                const float* src = base + (static_cast<long long>(r) * twins + t) * 2 * cols;
                g1s += __ldcv(src + c);
                g2s += __ldcv(src + cols + c);
            }
            const float total = static_cast<float>(rows) * ex.world;
            coef1[t * cols + c] = g1s / total;
            coef2[t * cols + c] = g2s / total;
        }
    }
    finish_launch(ex, epoch);
}

// One warp: value v (0 .. 63) of this rank travels as entry v of the slot (lanes carry
// v = lane and v = 32 + lane); every rank reduces all ranks' entries in rank order.
__global__ void __launch_bounds__(32) small_reduce_kernel(const rl2_peer_reduce_args a, const rl2_syncbn_exchange ex) {
    const int lane = threadIdx.x;
    const unsigned long long epoch = launch_epoch(ex);
    const int n1 = a.n_mean, n2 = n1 + a.n_max, n3 = n2 + a.n_max_int;
    auto own = [&](int v) -> float {
        if (v < n1) return a.mean[v];
        if (v < n2) return a.max[v - n1];
        if (v < n3) return __int_as_float(a.max_int[v - n2]);
        return 0.0f;
    };
    const float x0 = own(lane), x1 = own(32 + lane);
    const bool ok = exchange(ex, 1, 0, 32, lane, x0, x1, epoch);
    float r[2];
    const float* base = ex.peer_data[ex.rank];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int v = lane + 32 * h;
        float acc = 0.0f;
        int iacc = 0;
        for (int q = 0; q < ex.world; ++q) {
            const float e = ok ? __ldcv(base + static_cast<long long>(q) * 64 + v) : (h == 0 ? x0 : x1);
            if (v < n1)
                acc = q == 0 ? e : acc + e;
            else if (v < n2)
                acc = q == 0 ? e : fmaxf(acc, e);
            else
                iacc = q == 0 ? __float_as_int(e) : max(iacc, __float_as_int(e));
            if (!ok) break;  // a timed-out exchange keeps this rank's own values
        }
        r[h] = v < n1 ? (ok ? acc / static_cast<float>(ex.world) : acc) : v < n2 ? acc : __int_as_float(iacc);
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int v = lane + 32 * h;
        if (v < n1) a.mean[v] = r[h];
    }
    __syncwarp();  // max results after the means (max may alias an entry of mean)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int v = lane + 32 * h;
        if (v >= n1 && v < n2) a.max[v - n1] = r[h];
        if (v >= n2 && v < n3) a.max_int[v - n2] = __float_as_int(r[h]);
    }
    finish_launch(ex, epoch);
}

// ---- gradient arena mean over the ranks ------------------------------------------------
//
// One launch per optimizer step. Every rank's arena lives in symmetric memory. Rank r owns
// the float4 range [n4 * r / W, n4 * (r + 1) / W), split evenly over the blocks. Block b
// of rank r: (1) entry barrier with block b of every rank (each rank's block b has started,
// so that rank's backward kernels have finished writing its arena); (2) for each float4 of
// its share, loads the W ranks' values, sums them in rank order, divides by W and stores
// the mean into every rank's arena (this rank's share of the reduce-scatter and of the
// all-gather in one pass, one copy of each value crossing each link per direction);
// (3) exit barrier with block b of every rank (every rank's share is in this rank's arena
// before the kernel ends). Flags of a call site: [2 (entry, exit)][blocks][W] u64 per rank.
// Every value is computed by one rank only, so all ranks hold bit-identical means.

constexpr int kGradT = 512;
constexpr int kGradU = 2;         // float4 per thread and rank per iteration
constexpr int kGradBlocks = 148;  // all resident on a B200 (one 512-thread block per SM)

__device__ bool wait_epoch(const unsigned long long* f, unsigned long long epoch, const rl2_syncbn_exchange& ex) {
    if (load_acquire(f) >= epoch) return true;
    const uint64_t start = now_ns();
    const uint64_t limit = static_cast<uint64_t>(ex.timeout_s * 1e9f);
    for (uint32_t i = 1;; ++i) {
        if (load_acquire(f) >= epoch) return true;
        if ((i & 255u) == 0 && now_ns() - start > limit) {
            if (ex.health) atomicOr(ex.health, kHealthTimeout);
            return false;
        }
    }
}

// Block-wide barrier with block b of every rank on flag row `phase`; false on a timeout.
__device__ bool rank_barrier(const rl2_syncbn_exchange& ex, int phase, unsigned long long epoch, int* s_ok) {
    const int W = ex.world, t = threadIdx.x;
    const long long row = (static_cast<long long>(phase) * gridDim.x + blockIdx.x) * W;
    __syncthreads();  // every thread's earlier stores precede the release below
    if (t == 0) *s_ok = 1;
    if (t < W) store_release(ex.peer_flags[t] + row + ex.rank, epoch);
    __syncthreads();
    if (t < W && !wait_epoch(ex.peer_flags[ex.rank] + row + t, epoch, ex)) *s_ok = 0;
    __syncthreads();
    return *s_ok != 0;
}

__device__ __forceinline__ float4 ld_peer(const float4* p) { return __ldcv(p); }

__device__ __forceinline__ void add4(float4& a, const float4& b) {
    a.x += b.x;
    a.y += b.y;
    a.z += b.z;
    a.w += b.w;
}

template <int W>  // W > 0: compile-time world; W == 0: runtime world
__global__ void __launch_bounds__(kGradT) grad_mean_kernel(long long n4, const rl2_syncbn_exchange ex) {
    __shared__ int s_ok;
    __shared__ float4* s_ptr[32];
    const int world = W > 0 ? W : ex.world;
    const unsigned long long epoch = launch_epoch(ex);
    if (threadIdx.x < world) s_ptr[threadIdx.x] = reinterpret_cast<float4*>(ex.peer_data[threadIdx.x]);
    bool ok = rank_barrier(ex, 0, epoch, &s_ok);
    if (ok) {
        const long long lo = n4 * ex.rank / world, len = n4 * (ex.rank + 1) / world - lo;
        const long long c0 = lo + len * blockIdx.x / gridDim.x, c1 = lo + len * (blockIdx.x + 1) / gridDim.x;
        const float wf = static_cast<float>(world);
        for (long long i = c0 + threadIdx.x; i < c1; i += static_cast<long long>(kGradT) * kGradU) {
            float4 acc[kGradU];
            if constexpr (W > 0) {
                float4 x[W][kGradU];
#pragma unroll
                for (int q = 0; q < W; ++q)
#pragma unroll
                    for (int u = 0; u < kGradU; ++u) {
                        const long long e = i + static_cast<long long>(u) * kGradT;
                        if (e < c1) x[q][u] = ld_peer(s_ptr[q] + e);
                    }
#pragma unroll
                for (int u = 0; u < kGradU; ++u) {
                    acc[u] = x[0][u];
#pragma unroll
                    for (int q = 1; q < W; ++q) add4(acc[u], x[q][u]);
                }
            } else {
#pragma unroll
                for (int u = 0; u < kGradU; ++u) {
                    const long long e = i + static_cast<long long>(u) * kGradT;
                    if (e < c1) acc[u] = ld_peer(s_ptr[0] + e);
                }
                for (int q = 1; q < world; ++q)
#pragma unroll
                    for (int u = 0; u < kGradU; ++u) {
                        const long long e = i + static_cast<long long>(u) * kGradT;
                        if (e < c1) add4(acc[u], ld_peer(s_ptr[q] + e));
                    }
            }
#pragma unroll
            for (int u = 0; u < kGradU; ++u) {
                acc[u].x = acc[u].x / wf;
                acc[u].y = acc[u].y / wf;
                acc[u].z = acc[u].z / wf;
                acc[u].w = acc[u].w / wf;
            }
#pragma unroll 4
            for (int q = 0; q < world; ++q)
#pragma unroll
                for (int u = 0; u < kGradU; ++u) {
                    const long long e = i + static_cast<long long>(u) * kGradT;
                    if (e < c1) s_ptr[q][e] = acc[u];
                }
        }
    }
    // a rank whose entry wait ran out skips the exit wait (its peers then time out too)
    if (ok) rank_barrier(ex, 1, epoch, &s_ok);
    finish_launch(ex, epoch);
}

}  // namespace syncbn
}  // namespace rl2

using namespace rl2;

namespace {
bool exchange_valid(const rl2_syncbn_exchange* ex) {
    return ex && ex->peer_data && ex->peer_flags && ex->epoch && ex->world >= 1 && ex->world <= 32 && ex->rank >= 0 &&
           ex->rank < ex->world && ex->timeout_s > 0.0f;
}

// Every block of a launch must be resident while peers wait on its flags: keep the grid
// within a few blocks per SM.
bool grid_resident(int twins, int cols) { return static_cast<long long>(twins) * ((cols + 31) / 32) <= 148LL * 4; }
}  // namespace

extern "C" long long rl2_syncbn_slot_data_bytes(int world, int twins, int cols) {
    return static_cast<long long>(world) * twins * 2 * cols * 4;
}

extern "C" long long rl2_syncbn_slot_flag_bytes(int world, int twins, int cols) {
    return static_cast<long long>(twins) * ((cols + 31) / 32) * world * 8;
}

extern "C" int rl2_syncbn_forward(const float* mean_p, const float* m2_p, long long pt, int part_twins, int twins,
                                  int rows, int cols, float* mean, float* invstd, float* rm, float* rv, float momentum,
                                  float eps, int update, const rl2_syncbn_exchange* ex, void* stream) {
    clear_error();
    if (!mean_p || !m2_p || !mean || !invstd || twins < 1 || rows < 1 || cols < 1 || !(eps > 0.0f) ||
        (part_twins != 1 && part_twins != twins) || (update && (!rm || !rv)) || !exchange_valid(ex) ||
        !grid_resident(twins, cols)) {
        set_error("syncbn forward: invalid arguments");
        return -1;
    }
    syncbn::forward_kernel<<<dim3((cols + 31) / 32, twins), syncbn::kT, 0, as_stream(stream)>>>(
        mean_p, m2_p, part_twins == 1 ? 0 : pt, twins, rows, cols, mean, invstd, rm, rv, momentum, eps, update, *ex);
    return launch_status("data-parallel batch-norm statistics");
}

extern "C" int rl2_syncbn_backward(const float* s1p, const float* s2p, long long pt, int twins, int rows, int cols,
                                   float* dgamma, float* dbeta, long long gts, float* coef1, float* coef2,
                                   const rl2_syncbn_exchange* ex, void* stream) {
    clear_error();
    if (!s1p || !s2p || !coef1 || !coef2 || twins < 1 || rows < 1 || cols < 1 || !exchange_valid(ex) ||
        !grid_resident(twins, cols)) {
        set_error("syncbn backward: invalid arguments");
        return -1;
    }
    syncbn::backward_kernel<<<dim3((cols + 31) / 32, twins), syncbn::kT, 0, as_stream(stream)>>>(
        s1p, s2p, pt, twins, rows, cols, dgamma, dbeta, gts, coef1, coef2, *ex);
    return launch_status("data-parallel batch-norm backward sums");
}

extern "C" int rl2_peer_reduce(const rl2_peer_reduce_args* a, const rl2_syncbn_exchange* ex, void* stream) {
    clear_error();
    if (!a || a->n_mean < 0 || a->n_max < 0 || a->n_max_int < 0 || a->n_mean + a->n_max + a->n_max_int > 64 ||
        (a->n_mean && !a->mean) || (a->n_max && !a->max) || (a->n_max_int && !a->max_int) || !exchange_valid(ex)) {
        set_error("peer reduce: invalid arguments");
        return -1;
    }
    syncbn::small_reduce_kernel<<<1, 32, 0, as_stream(stream)>>>(*a, *ex);
    return launch_status("data-parallel scalar reduction");
}

extern "C" long long rl2_peer_mean_flag_bytes(int world) {
    return 2LL * syncbn::kGradBlocks * world * 8;
}

extern "C" int rl2_peer_mean(long long count, const rl2_syncbn_exchange* ex, void* stream) {
    clear_error();
    if (count < 0 || count % 4 != 0 || !exchange_valid(ex)) {
        set_error("peer mean: invalid arguments (count a multiple of 4 floats)");
        return -1;
    }
    const long long n4 = count / 4;
    const dim3 grid(syncbn::kGradBlocks), block(syncbn::kGradT);
    cudaStream_t s = as_stream(stream);
    switch (ex->world) {
        case 2: syncbn::grad_mean_kernel<2><<<grid, block, 0, s>>>(n4, *ex); break;
        case 4: syncbn::grad_mean_kernel<4><<<grid, block, 0, s>>>(n4, *ex); break;
        case 8: syncbn::grad_mean_kernel<8><<<grid, block, 0, s>>>(n4, *ex); break;
        default: syncbn::grad_mean_kernel<0><<<grid, block, 0, s>>>(n4, *ex); break;
    }
    return launch_status("data-parallel gradient mean");
}
