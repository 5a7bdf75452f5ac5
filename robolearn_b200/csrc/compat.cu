// rl_* entry points with the reference native library's names, argument lists and error
// behaviour (src/robolearn/cuda/kernels.cu, flash_kernels.cuh, categorical_kernels.cuh,
// zero_kernels.cuh), implemented on this library's kernels so that the reference's ctypes
// callers can bind librl2.so unchanged. Declared in include/rl_compat.h, which lists the
// differences a caller can observe.
//
// Dense plans run on the tcgen05 GEMM: the column-major D = op(A) op(B) is the row-major
// product D^T[n][m] = op(B)^T op(A)^T, so both operands are staged K-contiguous (fp16
// copies, or tf32 hi / lo planes for fp32) into plan-owned buffers and the plan's output,
// bias and residual pointers are bound at every launch.
#include "common.cuh"
#include "planes.cuh"
#include "../../include/rl2.h"
#include "../../include/rl_compat.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <limits>
#include <new>
#include <string>
#include <vector>

namespace rl2 {
const char* last_error() noexcept;
namespace gemm {
void* create_rebindable(const rl2_gemm_desc* g);
int run_rebound(void* plan, float* d, const float* bias, const float* residual, int accumulate,
                cudaStream_t stream);
int run_rebound_ab(void* plan, const void* a, const void* b, float* d, const float* bias, const float* residual,
                   int accumulate, cudaStream_t stream);
}  // namespace gemm
}  // namespace rl2

namespace rl2 {
namespace compat {

constexpr int kT = 256;

// ---------------------------------------------------------------------------
// dense plans
// ---------------------------------------------------------------------------

// dst[r][kk] (row pitch kp) = src[r * rs + kk * ks] for r < rows, kk < k; one of rs / ks is 1.
// 32 x 32 tiles through shared memory so that both the read (along the source's contiguous
// index) and the write (along kk) are coalesced. fp32 sources become tf32 hi / lo planes.
template <bool kHalf>
__global__ void __launch_bounds__(kT) pack_kernel(const void* __restrict__ src, long long rs, long long ks, int rows,
                                                  int k, long long kp, float* __restrict__ hi,
                                                  float* __restrict__ lo, __half* __restrict__ h16) {
    __shared__ float tile[32][33];
    const int r0 = blockIdx.x * 32, k0 = blockIdx.y * 32;
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
    const bool k_fast = ks == 1;
    for (int j = ty; j < 32; j += kT / 32) {
        const int r = r0 + (k_fast ? j : tx), kk = k0 + (k_fast ? tx : j);
        float v = 0.0f;
        if (r < rows && kk < k) {
            const long long o = static_cast<long long>(r) * rs + static_cast<long long>(kk) * ks;
            v = kHalf ? __half2float(static_cast<const __half*>(src)[o]) : static_cast<const float*>(src)[o];
        }
        if (k_fast)
            tile[j][tx] = v;
        else
            tile[tx][j] = v;
    }
    __syncthreads();
    for (int j = ty; j < 32; j += kT / 32) {
        const int r = r0 + j, kk = k0 + tx;
        if (r >= rows || kk >= k) continue;
        const long long o = static_cast<long long>(r) * kp + kk;
        const float v = tile[j][tx];
        if (kHalf) {
            h16[o] = __float2half_rn(v);  // exact: the source is fp16
        } else {
            const float h = tf32_hi(v);
            hi[o] = h;
            lo[o] = v - h;
        }
    }
}

// d[i + j * ldd] = beta * c[i + j * ldd] (column-major m x n), for beta other than 0 and 1.
__global__ void __launch_bounds__(kT) scale_c_kernel(const float* __restrict__ c, float* d, int m, int n, int ldd,
                                                     float beta) {
    const long long total = static_cast<long long>(m) * n;
    for (long long t = blockIdx.x * static_cast<long long>(kT) + threadIdx.x; t < total;
         t += static_cast<long long>(gridDim.x) * kT) {
        const long long j = t / m, i = t - j * m;
        const long long o = i + j * ldd;
        d[o] = beta * c[o];
    }
}

struct DensePlan {
    int m = 0, n = 0, k = 0, transa = 0, transb = 0, lda = 0, ldb = 0, ldd = 0;
    bool bias = false;
    int dtype = 0;  // 0: fp32 operands (tf32 hi / lo planes), 1: fp16 operands
    long long kp = 0;
    void* stage = nullptr;
    float *a_hi = nullptr, *a_lo = nullptr, *b_hi = nullptr, *b_lo = nullptr;  // kernel view: A' = op(B)^T, B' = op(A)
    __half *a16 = nullptr, *b16 = nullptr;
    void* gemm = nullptr;
    bool direct = false;  // fp16 operands read in place by TMA (no staging): leading dimensions multiples of 8
    bool tuned = false, used = false;
    std::string metadata;

    ~DensePlan() {
        if (gemm) rl2_gemm_destroy(gemm);
        if (stage) cudaFree(stage);
    }
};

void describe(DensePlan& p, float beta) {
    char buf[768];
    const char* beta_s = "null";
    char beta_buf[32];
    if (p.tuned) {
        std::snprintf(beta_buf, sizeof(beta_buf), "%.9g", beta);
        beta_s = beta_buf;
    }
    std::snprintf(buf, sizeof(buf),
                  "{\"enabled\":%s,\"tuned_beta\":%s,\"backend\":\"tcgen05\",\"operands\":\"%s\","
                  "\"default_candidate_index\":0,\"selected_candidate_index\":0,\"selected_workspace_bytes\":0,"
                  "\"candidates\":[{\"heuristic_index\":0,\"tile_n\":%d,\"epilogue_form\":%d,\"workspace_bytes\":0,"
                  "\"status\":0,\"samples_ms\":[],\"median_ms\":null}]}",
                  p.tuned ? "true" : "false", beta_s,
                  p.dtype == 1 ? (p.direct ? "fp16 in place" : "fp16 staged") : "tf32x3 staged", rl2_gemm_tile_n(p.gemm),
                  rl2_gemm_uses_tma_store(p.gemm));
    p.metadata = buf;
}

void* create_dense(int m, int n, int k, int transa, int transb, int lda, int ldb, int ldd, int use_bias,
                   int allow_tf32, int input_dtype) {
    clear_error();
    if (m <= 0 || n <= 0 || k <= 0) {
        set_error("Dense dimensions must be positive.");
        return nullptr;
    }
    if ((transa != 0 && transa != 1) || (transb != 0 && transb != 1)) {
        set_error("Transpose flags must be 0 or 1.");
        return nullptr;
    }
    if ((use_bias != 0 && use_bias != 1) || (allow_tf32 != 0 && allow_tf32 != 1)) {
        set_error("Bias and TF32 flags must be 0 or 1.");
        return nullptr;
    }
    if (input_dtype != 0 && input_dtype != 1) {
        set_error("Dense input dtype must be 0=FP32 or 1=FP16.");
        return nullptr;
    }
    if (input_dtype == 1 && allow_tf32) {
        set_error("TF32 applies only to FP32 inputs.");
        return nullptr;
    }
    const int a_rows = transa ? k : m, b_rows = transb ? n : k;
    if (lda < a_rows || ldb < b_rows || ldd < m) {
        set_error("Invalid column-major leading dimension.");
        return nullptr;
    }
    DensePlan* p = new (std::nothrow) DensePlan();
    if (!p) {
        set_error("out of host memory");
        return nullptr;
    }
    p->m = m, p->n = n, p->k = k, p->transa = transa, p->transb = transb, p->lda = lda, p->ldb = ldb, p->ldd = ldd;
    p->bias = use_bias != 0;
    p->dtype = input_dtype;
    rl2_gemm_desc g;
    std::memset(&g, 0, sizeof(g));
    p->direct = input_dtype == 1 && lda % 8 == 0 && ldb % 8 == 0;
    if (!p->direct && (k + 31) / 32 > 65535) {  // the staging kernel's grid.y covers K in 32-wide tiles
        set_error("Dense K above 2097120 needs fp16 operands with leading dimensions that are multiples of 8.");
        delete p;
        return nullptr;
    }
    if (p->direct) {
        // kernel view read in place: A'[j][kk] = op(B)(kk, j), B'[i][kk] = op(A)(i, kk); the
        // operand addresses are bound at every launch (a 256-byte placeholder until then)
        if (cudaMalloc(&p->stage, 256) != cudaSuccess) {
            cudaGetLastError();
            set_error("Allocate dense plan placeholder");
            delete p;
            return nullptr;
        }
        g.kind = 0;
        g.a = g.b = p->stage;
        g.a_major = transb ? 1 : 0;
        g.lda = ldb;
        g.b_major = transa ? 0 : 1;
        g.ldb = lda;
    } else {
        // staged rows are K-contiguous with a 16-byte row pitch (TMA stride rule)
        p->kp = input_dtype == 1 ? (k + 7) / 8 * 8 : (k + 3) / 4 * 4;
        const size_t elem = input_dtype == 1 ? 2 : 4;
        auto region = [&](long long rows) { return (static_cast<size_t>(rows) * p->kp * elem + 255) / 256 * 256; };
        const size_t ra = region(n), rb = region(m);
        const size_t total = input_dtype == 1 ? ra + rb : 2 * (ra + rb);
        if (cudaMalloc(&p->stage, total) != cudaSuccess) {
            cudaGetLastError();
            set_error("Allocate dense operand staging (%zu bytes)", total);
            delete p;
            return nullptr;
        }
        char* base = static_cast<char*>(p->stage);
        if (input_dtype == 1) {
            p->a16 = reinterpret_cast<__half*>(base);
            p->b16 = reinterpret_cast<__half*>(base + ra);
            g.kind = 0;
            g.a = p->a16;
            g.b = p->b16;
        } else {
            p->a_hi = reinterpret_cast<float*>(base);
            p->a_lo = reinterpret_cast<float*>(base + ra);
            p->b_hi = reinterpret_cast<float*>(base + 2 * ra);
            p->b_lo = reinterpret_cast<float*>(base + 2 * ra + rb);
            g.kind = 1;
            g.a = p->a_hi;
            g.a_lo = p->a_lo;
            g.b = p->b_hi;
            g.b_lo = p->b_lo;
        }
        g.a_major = 0;
        g.lda = p->kp;
        g.b_major = 0;
        g.ldb = p->kp;
    }
    g.m = n;
    g.n = m;
    g.k = k;
    g.batch = 1;
    g.d = static_cast<float*>(p->stage);  // placeholder: the output is bound at every launch
    g.ldd = ldd;
    g.ldr = ldd;
    g.k_splits = 1;
    p->gemm = rl2::gemm::create_rebindable(&g);
    if (!p->gemm) {
        delete p;
        return nullptr;
    }
    describe(*p, 0.0f);
    return p;
}

int pack(const DensePlan& p, const void* src, bool contiguous_rows, int ld, int rows, float* hi, float* lo,
         __half* h16, cudaStream_t s) {
    // contiguous_rows: element (r, kk) at src[r + kk * ld]; else at src[kk + r * ld]
    const long long rs = contiguous_rows ? 1 : ld, ks = contiguous_rows ? ld : 1;
    const dim3 grid(static_cast<unsigned>((rows + 31) / 32), static_cast<unsigned>((p.k + 31) / 32));
    if (p.dtype == 1)
        pack_kernel<true><<<grid, kT, 0, s>>>(src, rs, ks, rows, p.k, p.kp, nullptr, nullptr, h16);
    else
        pack_kernel<false><<<grid, kT, 0, s>>>(src, rs, ks, rows, p.k, p.kp, hi, lo, nullptr);
    return launch_status("Stage dense operand");
}

// ---------------------------------------------------------------------------
// fp16 cast and bias gradient
// ---------------------------------------------------------------------------

__global__ void __launch_bounds__(kT) cast_kernel(const float* __restrict__ src, __half* __restrict__ dst, size_t count,
                                                  bool vec) {
    const size_t stride = static_cast<size_t>(gridDim.x) * kT;
    size_t t = static_cast<size_t>(blockIdx.x) * kT + threadIdx.x;
    if (vec) {  // 16-byte source and 8-byte destination alignment
        const size_t quads = count / 4;
        for (size_t q = t; q < quads; q += stride) {
            const float4 v = reinterpret_cast<const float4*>(src)[q];
            __half2* o = reinterpret_cast<__half2*>(dst + 4 * q);
            o[0] = __floats2half2_rn(v.x, v.y);
            o[1] = __floats2half2_rn(v.z, v.w);
        }
        for (size_t i = quads * 4 + t; i < count; i += stride) dst[i] = __float2half_rn(src[i]);
    } else {
        for (size_t i = t; i < count; i += stride) dst[i] = __float2half_rn(src[i]);
    }
}

int grid_for(size_t work, int per_block) {
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const size_t blocks = (work + per_block - 1) / per_block;
    const size_t cap = static_cast<size_t>(sms) * 8;
    return static_cast<int>(blocks < 1 ? 1 : blocks > cap ? cap : blocks);
}

// db[c] += sum over rows of dy[row][c]: 32 channels per block (coalesced row segments),
// 32 row lanes per channel (one warp each, four independent partial sums for memory-level
// parallelism), then a fixed-order combine of the 32 lane sums.
constexpr int kColT = 1024;

__global__ void __launch_bounds__(kColT) column_sum_kernel(const float* __restrict__ dy, float* db, int batch,
                                                           int channels, long long ld) {
    __shared__ float part[kColT / 32][33];
    const int lane = threadIdx.x & 31, grp = threadIdx.x >> 5;
    const int c = blockIdx.x * 32 + lane;
    constexpr int G = kColT / 32;
    float s0 = 0.0f, s1 = 0.0f, s2 = 0.0f, s3 = 0.0f;
    if (c < channels) {
        const float* col = dy + c;
        int r = grp;
        for (; r + 3 * G < batch; r += 4 * G) {
            s0 += col[static_cast<long long>(r) * ld];
            s1 += col[static_cast<long long>(r + G) * ld];
            s2 += col[static_cast<long long>(r + 2 * G) * ld];
            s3 += col[static_cast<long long>(r + 3 * G) * ld];
        }
        for (; r < batch; r += G) s0 += col[static_cast<long long>(r) * ld];
    }
    part[grp][lane] = (s0 + s1) + (s2 + s3);
    __syncthreads();
    if (grp == 0 && c < channels) {
        float t = part[0][lane];
#pragma unroll
        for (int g = 1; g < G; ++g) t += part[g][lane];
        db[c] += t;
    }
}

// First pass of a column sum over many rows whose source may be overwritten: block
// (channel tile, row slab) sums its slab's rows (8 row lanes per channel, fixed-order
// combine) and stores the sum over the slab's FIRST row, which no other block reads. The
// slab sums are then added by column_sum_kernel over rows strided by the slab height.
__global__ void __launch_bounds__(kT) slab_sum_kernel(float* src, int batch, int channels, int rows) {
    __shared__ float part[kT / 32][33];
    const int lane = threadIdx.x & 31, grp = threadIdx.x >> 5;
    const int c = blockIdx.x * 32 + lane;
    const int r0 = blockIdx.y * rows, r1 = min(batch, r0 + rows);
    float s = 0.0f;
    if (c < channels)
        for (int r = r0 + grp; r < r1; r += kT / 32) s += src[static_cast<long long>(r) * channels + c];
    part[grp][lane] = s;
    __syncthreads();
    if (grp == 0 && c < channels) {
        float t = part[0][lane];
#pragma unroll
        for (int g = 1; g < kT / 32; ++g) t += part[g][lane];
        src[static_cast<long long>(r0) * channels + c] = t;
    }
}

}  // namespace compat
}  // namespace rl2

using rl2::compat::DensePlan;

extern "C" const char* rl_last_error(void) { return rl2::last_error(); }

extern "C" void* rl_plan_create(int m, int n, int k, int transa, int transb, int lda, int ldb, int ldd, int use_bias,
                                int allow_tf32, size_t workspace_limit) {
    (void)workspace_limit;  // staging is plan-owned: every plan fits any limit
    return rl2::compat::create_dense(m, n, k, transa, transb, lda, ldb, ldd, use_bias, allow_tf32, 0);
}

extern "C" void* rl_plan_create_mixed(int m, int n, int k, int transa, int transb, int lda, int ldb, int ldd,
                                      int use_bias, int allow_tf32, int input_dtype, size_t workspace_limit) {
    (void)workspace_limit;
    return rl2::compat::create_dense(m, n, k, transa, transb, lda, ldb, ldd, use_bias, allow_tf32, input_dtype);
}

extern "C" int rl_plan_autotune(void* opaque, float beta, void* stream) {
    rl2::clear_error();
    if (!opaque || !(beta == 0.0f || beta == 1.0f)) {
        rl2::set_error("Autotuning requires a plan and beta=0 or beta=1.");
        return -1;
    }
    DensePlan* p = static_cast<DensePlan*>(opaque);
    if (p->tuned || p->used) {
        rl2::set_error("Dense plans may be autotuned only once, before use/capture.");
        return -1;
    }
    cudaStreamCaptureStatus capture = cudaStreamCaptureStatusNone;
    const cudaError_t e = cudaStreamIsCapturing(rl2::as_stream(stream), &capture);
    if (e != cudaSuccess) {
        rl2::set_error("Inspect autotuning stream capture: %s", cudaGetErrorString(e));
        return -1;
    }
    if (capture != cudaStreamCaptureStatusNone) {
        rl2::set_error("Autotuning cannot run inside graph capture.");
        return -1;
    }
    p->tuned = true;  // one candidate: the plan-chosen tile
    rl2::compat::describe(*p, beta);
    return 0;
}

extern "C" const char* rl_plan_tuning_metadata(void* opaque) {
    rl2::clear_error();
    if (!opaque) {
        rl2::set_error("Dense plan is null.");
        return nullptr;
    }
    return static_cast<DensePlan*>(opaque)->metadata.c_str();
}

extern "C" size_t rl_plan_workspace(void* opaque) {
    rl2::clear_error();
    if (!opaque) {
        rl2::set_error("Dense plan is null.");
        return std::numeric_limits<size_t>::max();
    }
    return 0;
}

extern "C" int rl_plan_run(void* opaque, const void* a, const void* b, const void* c, void* d, const void* bias,
                           void* workspace, size_t workspace_bytes, float beta, void* stream) {
    using namespace rl2;
    clear_error();
    (void)workspace;
    (void)workspace_bytes;
    if (!opaque || !a || !b || !d) {
        set_error("Dense plan, A, B and D must be nonnull.");
        return -1;
    }
    DensePlan* p = static_cast<DensePlan*>(opaque);
    if (!std::isfinite(beta) || (beta != 0.0f && !c)) {
        set_error("Nonzero beta requires C; beta must be finite.");
        return -1;
    }
    const size_t in_align = p->dtype == 1 ? 16 : 4;
    if (!aligned(a, in_align) || !aligned(b, in_align) || !aligned(d, 4) || (c && !aligned(c, 4))) {
        set_error("Dense input/output alignment does not meet the plan's requirements.");
        return -1;
    }
    if (p->bias && (!bias || !aligned(bias, 4))) {
        set_error("Dense bias must be a nonnull FP32-aligned device buffer.");
        return -1;
    }
    const cudaStream_t s = as_stream(stream);
    p->used = true;
    // kernel view: A'[j][kk] = op(B)(kk, j), B'[i][kk] = op(A)(i, kk)
    if (!p->direct && (compat::pack(*p, b, p->transb == 1, p->ldb, p->n, p->a_hi, p->a_lo, p->a16, s) ||
                       compat::pack(*p, a, p->transa == 0, p->lda, p->m, p->b_hi, p->b_lo, p->b16, s)))
        return -1;
    float* dst = static_cast<float*>(d);
    const float* cc = static_cast<const float*>(c);
    const float* residual = nullptr;
    int accumulate = 0;
    if (beta == 1.0f) {
        if (cc == dst)
            accumulate = 1;
        else
            residual = cc;
    } else if (beta != 0.0f) {
        compat::scale_c_kernel<<<compat::grid_for(static_cast<size_t>(p->m) * p->n, compat::kT * 4), compat::kT, 0,
                                 s>>>(cc, dst, p->m, p->n, p->ldd, beta);
        if (launch_status("Scale dense C")) return -1;
        accumulate = 1;
    }
    const float* bv = p->bias ? static_cast<const float*>(bias) : nullptr;
    if (p->direct) return gemm::run_rebound_ab(p->gemm, b, a, dst, bv, residual, accumulate, s);
    return gemm::run_rebound(p->gemm, dst, bv, residual, accumulate, s);
}

extern "C" int rl_plan_destroy(void* opaque) {
    rl2::clear_error();
    delete static_cast<DensePlan*>(opaque);
    return 0;
}

extern "C" int rl_cast_f32_f16(const void* source, void* destination, size_t count, void* stream) {
    using namespace rl2;
    clear_error();
    if (!source || !destination || !count || !aligned(source, 4) || !aligned(destination, 2)) {
        set_error("FP16 conversion requires nonempty aligned buffers within CUDA grid limits.");
        return -1;
    }
    const bool vec = aligned(source, 16) && aligned(destination, 8);
    compat::cast_kernel<<<compat::grid_for(count, compat::kT * 8), compat::kT, 0, as_stream(stream)>>>(
        static_cast<const float*>(source), static_cast<__half*>(destination), count, vec);
    return launch_status("Convert FP32 to FP16");
}

extern "C" int rl_bias_grad(const void* dy, void* db, int batch, int channels, void* stream) {
    using namespace rl2;
    clear_error();
    if (!dy || !db || batch <= 0 || channels <= 0 || !aligned(dy, 4) || !aligned(db, 4)) {
        set_error("Bias gradient requires FP32 buffers and positive batch/channels.");
        return -1;
    }
    compat::column_sum_kernel<<<(channels + 31) / 32, compat::kColT, 0, as_stream(stream)>>>(
        static_cast<const float*>(dy), static_cast<float*>(db), batch, channels, channels);
    return launch_status("Run bias gradient");
}

// ---------------------------------------------------------------------------
// multi-tensor Adam, projection, EMA and grouped zeroing
// ---------------------------------------------------------------------------

namespace rl2 {
namespace compat {

constexpr unsigned kAdamChunk = 4096;  // elements per block

struct AdamTensor {
    float* p;
    float* g;
    float* m1;
    float* m2;
    size_t n;
    int vec;  // all four arrays 16-byte aligned: float4 accesses (chunks start at multiples of 4096)
};

// block b works on tensor i with first[i] <= b < first[i + 1] (first[count] = blocks)
__device__ __forceinline__ int tensor_of(const unsigned* first, int count, unsigned b) {
    int lo = 0, hi = count - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (first[mid] <= b)
            lo = mid;
        else
            hi = mid - 1;
    }
    return lo;
}

struct AdamState {
    float* timestep;
    const float* lr;
    float* corr;  // 1 / (1 - beta1^t), 1 / (1 - beta2^t)
    float* loss_scale;
    int* growth_tracker;
    int* found_inf;
    int* step_skipped;
    long long* attempted;
    long long* skipped;
    float growth_factor, backoff_factor;
    int growth_interval;
};

// the step's scalar prologue: count the attempt, skip on a non-finite scaled gradient
// (back the scale off, floor 2^-126), else advance the timestep, the bias corrections and
// the growth schedule (kernels.cu:332-404)
__global__ void adam_prologue_kernel(AdamState s, float beta1, float beta2) {
    if (s.loss_scale) {
        s.attempted[0] += 1;
        const int skip = s.found_inf[0] != 0;
        s.step_skipped[0] = skip;
        if (skip) {
            s.skipped[0] += 1;
            s.growth_tracker[0] = 0;
            s.loss_scale[0] = fmaxf(s.loss_scale[0] * s.backoff_factor, 1.17549435e-38f);
            return;
        }
        const int grown = s.growth_tracker[0] + 1;
        if (grown >= s.growth_interval) {
            const float up = s.loss_scale[0] * s.growth_factor;
            if (isfinite(up)) s.loss_scale[0] = up;
            s.growth_tracker[0] = 0;
        } else {
            s.growth_tracker[0] = grown;
        }
    }
    const float t = s.timestep[0] + 1.0f;
    s.timestep[0] = t;
    s.corr[0] = 1.0f / (1.0f - powf(beta1, t));
    s.corr[1] = 1.0f / (1.0f - powf(beta2, t));
}

__global__ void __launch_bounds__(kT) adam_kernel(const AdamTensor* __restrict__ tensors,
                                                  const unsigned* __restrict__ first, int count, AdamState s,
                                                  float beta1, float beta2, float omb1, float omb2, float eps) {
    if (s.step_skipped && s.step_skipped[0]) return;
    const int i = tensor_of(first, count, blockIdx.x);
    const AdamTensor t = tensors[i];
    const size_t off = static_cast<size_t>(blockIdx.x - first[i]) * kAdamChunk;
    const size_t len = t.n - off < kAdamChunk ? t.n - off : kAdamChunk;
    const float c1 = s.corr[0], c2 = s.corr[1], lr = s.lr[0];
    auto one = [&](float g, float& m1, float& m2, float& p) {
        m1 = beta1 * m1 + omb1 * g;
        m2 = beta2 * m2 + omb2 * (g * g);
        p -= lr * ((m1 * c1) / (sqrtf(m2 * c2) + eps));
    };
    size_t j0 = 0;
    if (t.vec) {
        const size_t quads = len / 4;
        float4* p4 = reinterpret_cast<float4*>(t.p + off);
        const float4* g4 = reinterpret_cast<const float4*>(t.g + off);
        float4* a4 = reinterpret_cast<float4*>(t.m1 + off);
        float4* b4 = reinterpret_cast<float4*>(t.m2 + off);
        for (size_t q = threadIdx.x; q < quads; q += kT) {
            const float4 g = g4[q];
            float4 a = a4[q], b = b4[q], pv = p4[q];
            one(g.x, a.x, b.x, pv.x);
            one(g.y, a.y, b.y, pv.y);
            one(g.z, a.z, b.z, pv.z);
            one(g.w, a.w, b.w, pv.w);
            a4[q] = a;
            b4[q] = b;
            p4[q] = pv;
        }
        j0 = quads * 4;
    }
    for (size_t j = j0 + threadIdx.x; j < len; j += kT) {
        const size_t o = off + j;
        float a = t.m1[o], b = t.m2[o], pv = t.p[o];
        one(t.g[o], a, b, pv);
        t.m1[o] = a;
        t.m2[o] = b;
        t.p[o] = pv;
    }
}

// gradients *= 1 / scale; *found_inf = 1 when a gradient, its unscaled value or the scale
// is not finite (or the scale is not positive)
__global__ void __launch_bounds__(kT) unscale_kernel(const AdamTensor* __restrict__ tensors,
                                                     const unsigned* __restrict__ first, int count,
                                                     const float* loss_scale, int* found_inf) {
    const int i = tensor_of(first, count, blockIdx.x);
    const AdamTensor t = tensors[i];
    const size_t off = static_cast<size_t>(blockIdx.x - first[i]) * kAdamChunk;
    const size_t len = t.n - off < kAdamChunk ? t.n - off : kAdamChunk;
    const float scale = loss_scale[0];
    const float inv = 1.0f / scale;
    const bool scale_bad = !isfinite(scale) || !(scale > 0.0f);
    int bad = 0;
    for (size_t j = threadIdx.x; j < len; j += kT) {
        const float g = t.g[off + j];
        const float u = g * inv;
        bad |= !isfinite(g) || !isfinite(u);
        t.g[off + j] = u;
    }
    if (__syncthreads_or(bad || scale_bad) && threadIdx.x == 0) atomicExch(found_inf, 1);
}

struct AdamPlan {
    AdamTensor* tensors = nullptr;  // device
    unsigned* first = nullptr;      // device, count + 1 entries
    float* corr = nullptr;          // device, 2 floats
    int count = 0;
    unsigned blocks = 0;
    float beta1 = 0, beta2 = 0, omb1 = 0, omb2 = 0, eps = 0;
    AdamState s{};

    ~AdamPlan() {
        if (tensors) cudaFree(tensors);
        if (first) cudaFree(first);
        if (corr) cudaFree(corr);
    }
};

// Row projections (kind 0: divide by max(||row||, 1e-8); 1: joint norm of the pair set to
// sqrt(length); 2: norm set to sqrt(length)), flash_kernels.cuh:112-131.
struct ProjRow {
    float* first;
    float* second;
    size_t len;
    int kind;
    __half* shadow;
};

__device__ __forceinline__ float block_total(float v, float* sh) {
    v = warp_sum(v);
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    if (lane == 0) sh[w] = v;
    __syncthreads();
    if (w == 0) {
        float x = lane < kT / 32 ? sh[lane] : 0.0f;
        x = warp_sum(x);
        if (lane == 0) sh[kT / 32] = x;
    }
    __syncthreads();
    return sh[kT / 32];
}

__global__ void __launch_bounds__(kT) project_kernel(const ProjRow* __restrict__ rows) {
    __shared__ float sh[kT / 32 + 1];
    const ProjRow r = rows[blockIdx.x];
    float ss = 0.0f;
    for (size_t i = threadIdx.x; i < r.len; i += kT) {
        const float a = r.first[i];
        ss += a * a;
        if (r.kind == 1) {
            const float b = r.second[i];
            ss += b * b;
        }
    }
    const float total = block_total(ss, sh);
    if (r.kind == 0) {
        const float norm = fmaxf(sqrtf(total), 1e-8f);
        for (size_t i = threadIdx.x; i < r.len; i += kT) {
            const float v = r.first[i] / norm;
            r.first[i] = v;
            if (r.shadow) r.shadow[i] = __float2half_rn(v);
        }
    } else {
        const float f = sqrtf(static_cast<float>(r.len)) / sqrtf(total + 1e-8f);
        for (size_t i = threadIdx.x; i < r.len; i += kT) {
            r.first[i] *= f;
            if (r.kind == 1) r.second[i] *= f;
        }
    }
}

constexpr unsigned kSpan = 8192;  // elements per block (EMA and zero spans)

struct EmaSpan {
    const float* src;
    float* dst;
    unsigned len;
    __half* shadow;
};

__global__ void __launch_bounds__(kT) ema_kernel(const EmaSpan* __restrict__ spans, float tau) {
    const EmaSpan e = spans[blockIdx.x];
    const float keep = 1.0f - tau;
    unsigned i0 = 0;
    const bool vec = ptx::aligned16(e.src) && ptx::aligned16(e.dst) && (!e.shadow || (reinterpret_cast<uintptr_t>(e.shadow) & 7u) == 0);
    if (vec) {
        const unsigned quads = e.len / 4;
        const float4* s4 = reinterpret_cast<const float4*>(e.src);
        float4* d4 = reinterpret_cast<float4*>(e.dst);
        for (unsigned q = threadIdx.x; q < quads; q += kT) {
            const float4 a = s4[q];
            float4 d = d4[q];
            d.x = keep * d.x + tau * a.x;
            d.y = keep * d.y + tau * a.y;
            d.z = keep * d.z + tau * a.z;
            d.w = keep * d.w + tau * a.w;
            d4[q] = d;
            if (e.shadow) {
                __half2* h = reinterpret_cast<__half2*>(e.shadow + 4 * q);
                h[0] = __floats2half2_rn(d.x, d.y);
                h[1] = __floats2half2_rn(d.z, d.w);
            }
        }
        i0 = quads * 4;
    }
    for (unsigned i = i0 + threadIdx.x; i < e.len; i += kT) {
        const float v = keep * e.dst[i] + tau * e.src[i];
        e.dst[i] = v;
        if (e.shadow) e.shadow[i] = __float2half_rn(v);
    }
}

struct ZeroSpan {
    float* p;
    unsigned len;
};

__global__ void __launch_bounds__(kT) zero_kernel(const ZeroSpan* __restrict__ spans) {
    const ZeroSpan z = spans[blockIdx.x];
    // scalar head up to a 16-byte boundary, float4 body, scalar tail
    const unsigned head = static_cast<unsigned>(((16u - (reinterpret_cast<uintptr_t>(z.p) & 15u)) & 15u) / 4u);
    const unsigned h = head < z.len ? head : z.len;
    if (threadIdx.x < h) z.p[threadIdx.x] = 0.0f;
    const unsigned quads = (z.len - h) / 4;
    float4* body = reinterpret_cast<float4*>(z.p + h);
    for (unsigned i = threadIdx.x; i < quads; i += kT) body[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    for (unsigned i = h + quads * 4 + threadIdx.x; i < z.len; i += kT) z.p[i] = 0.0f;
}

template <class T>
struct Table {
    T* dev = nullptr;
    unsigned count = 0;
    float tau = 0.0f;
    ~Table() {
        if (dev) cudaFree(dev);
    }
};

template <class T>
Table<T>* upload(const std::vector<T>& rows, const char* what) {
    if (rows.empty() || rows.size() > static_cast<size_t>(std::numeric_limits<int>::max())) {
        set_error("%s: descriptor count must fit a nonempty CUDA grid.", what);
        return nullptr;
    }
    Table<T>* t = new (std::nothrow) Table<T>();
    if (!t) {
        set_error("out of host memory");
        return nullptr;
    }
    if (cudaMalloc(&t->dev, rows.size() * sizeof(T)) != cudaSuccess ||
        cudaMemcpy(t->dev, rows.data(), rows.size() * sizeof(T), cudaMemcpyHostToDevice) != cudaSuccess) {
        set_error("%s: %s", what, cudaGetErrorString(cudaGetLastError()));
        delete t;
        return nullptr;
    }
    t->count = static_cast<unsigned>(rows.size());
    return t;
}

void* create_projection(size_t count, const void* const* first, const void* const* second, const size_t* lengths,
                        const int* kinds, const void* const* shadows) {
    clear_error();
    if (!count || !first || !second || !lengths || !kinds) {
        set_error("Invalid projection metadata.");
        return nullptr;
    }
    std::vector<ProjRow> rows;
    rows.reserve(count);
    for (size_t i = 0; i < count; ++i) {
        if (!first[i] || !lengths[i] || kinds[i] < 0 || kinds[i] > 2 || (kinds[i] == 1 && !second[i])) {
            set_error("Invalid projection row/vector.");
            return nullptr;
        }
        const void* sh = shadows ? shadows[i] : nullptr;
        if (sh && (kinds[i] != 0 || !aligned(sh, 2))) {
            set_error("Projection shadows require aligned FP16 unit-linear row destinations.");
            return nullptr;
        }
        rows.push_back({static_cast<float*>(const_cast<void*>(first[i])), static_cast<float*>(const_cast<void*>(second[i])),
                        lengths[i], kinds[i], static_cast<__half*>(const_cast<void*>(sh))});
    }
    return upload(rows, "Create projection plan");
}

void* create_ema(size_t count, const void* const* source, const void* const* target, const size_t* lengths,
                 float tau, const void* const* shadows) {
    clear_error();
    if (!count || !source || !target || !lengths || !std::isfinite(tau) || tau < 0.0f || tau > 1.0f) {
        set_error("Invalid EMA metadata/tau.");
        return nullptr;
    }
    std::vector<EmaSpan> spans;
    for (size_t i = 0; i < count; ++i) {
        if (!source[i] || !target[i] || !lengths[i]) {
            set_error("Invalid EMA tensor.");
            return nullptr;
        }
        const void* sh = shadows ? shadows[i] : nullptr;
        if (sh && !aligned(sh, 2)) {
            set_error("EMA shadows require aligned FP16 destinations.");
            return nullptr;
        }
        for (size_t o = 0; o < lengths[i]; o += kSpan) {
            const size_t len = lengths[i] - o < kSpan ? lengths[i] - o : kSpan;
            spans.push_back({static_cast<const float*>(source[i]) + o, static_cast<float*>(const_cast<void*>(target[i])) + o,
                             static_cast<unsigned>(len),
                             sh ? static_cast<__half*>(const_cast<void*>(sh)) + o : nullptr});
        }
    }
    Table<EmaSpan>* t = upload(spans, "Create EMA plan");
    if (t) t->tau = tau;
    return t;
}

}  // namespace compat
}  // namespace rl2

extern "C" void* rl_adam_create(size_t count, const void* const* parameters, const void* const* gradients,
                                const void* const* m1, const void* const* m2, const size_t* sizes, void* timestep,
                                void* learning_rate, double beta1, double beta2, double eps) {
    using namespace rl2;
    using namespace rl2::compat;
    clear_error();
    if (!count || !parameters || !gradients || !m1 || !m2 || !sizes || !timestep || !learning_rate) {
        set_error("Adam requires nonempty host pointer tables and device step/lr buffers.");
        return nullptr;
    }
    if (!std::isfinite(beta1) || !std::isfinite(beta2) || !std::isfinite(eps) || beta1 < 0.0 || beta1 >= 1.0 ||
        beta2 < 0.0 || beta2 >= 1.0 || !(eps > 0.0)) {
        set_error("Adam betas must lie in [0,1) and epsilon must be positive.");
        return nullptr;
    }
    if (!aligned(timestep, 4) || !aligned(learning_rate, 4)) {
        set_error("Adam step/lr buffers must be FP32-aligned.");
        return nullptr;
    }
    std::vector<AdamTensor> tensors;
    std::vector<unsigned> first;
    unsigned long long blocks = 0;
    for (size_t i = 0; i < count; ++i) {
        if (!parameters[i] || !gradients[i] || !m1[i] || !m2[i] || !sizes[i]) {
            set_error("Adam tensors must be nonnull and nonempty.");
            return nullptr;
        }
        if (!aligned(parameters[i], 4) || !aligned(gradients[i], 4) || !aligned(m1[i], 4) || !aligned(m2[i], 4)) {
            set_error("Adam tensors must be FP32-aligned.");
            return nullptr;
        }
        first.push_back(static_cast<unsigned>(blocks));
        blocks += (sizes[i] + kAdamChunk - 1) / kAdamChunk;
        if (blocks > static_cast<unsigned long long>(std::numeric_limits<int>::max())) {
            set_error("Adam tensor block count exceeds CUDA grid limits.");
            return nullptr;
        }
        tensors.push_back({static_cast<float*>(const_cast<void*>(parameters[i])),
                           static_cast<float*>(const_cast<void*>(gradients[i])),
                           static_cast<float*>(const_cast<void*>(m1[i])), static_cast<float*>(const_cast<void*>(m2[i])),
                           sizes[i],
                           aligned(parameters[i], 16) && aligned(gradients[i], 16) && aligned(m1[i], 16) &&
                               aligned(m2[i], 16)});
    }
    first.push_back(static_cast<unsigned>(blocks));
    AdamPlan* p = new (std::nothrow) AdamPlan();
    if (!p) {
        set_error("out of host memory");
        return nullptr;
    }
    if (cudaMalloc(&p->tensors, tensors.size() * sizeof(AdamTensor)) != cudaSuccess ||
        cudaMalloc(&p->first, first.size() * sizeof(unsigned)) != cudaSuccess ||
        cudaMalloc(&p->corr, 2 * sizeof(float)) != cudaSuccess ||
        cudaMemcpy(p->tensors, tensors.data(), tensors.size() * sizeof(AdamTensor), cudaMemcpyHostToDevice) !=
            cudaSuccess ||
        cudaMemcpy(p->first, first.data(), first.size() * sizeof(unsigned), cudaMemcpyHostToDevice) != cudaSuccess) {
        set_error("Create Adam plan: %s", cudaGetErrorString(cudaGetLastError()));
        delete p;
        return nullptr;
    }
    p->count = static_cast<int>(count);
    p->blocks = static_cast<unsigned>(blocks);
    p->beta1 = static_cast<float>(beta1);
    p->beta2 = static_cast<float>(beta2);
    p->omb1 = static_cast<float>(1.0 - beta1);
    p->omb2 = static_cast<float>(1.0 - beta2);
    p->eps = static_cast<float>(eps);
    p->s.timestep = static_cast<float*>(timestep);
    p->s.lr = static_cast<const float*>(learning_rate);
    p->s.corr = p->corr;
    return p;
}

extern "C" int rl_adam_set_scaler(void* opaque, void* loss_scale, void* growth_tracker, void* found_inf,
                                  void* step_skipped, void* attempted_steps, void* skipped_steps, double growth_factor,
                                  double backoff_factor, int growth_interval) {
    using namespace rl2;
    clear_error();
    if (!opaque || !loss_scale || !growth_tracker || !found_inf || !step_skipped || !attempted_steps ||
        !skipped_steps) {
        set_error("Dynamic loss scaling requires persistent device state.");
        return -1;
    }
    if (!aligned(loss_scale, 4) || !aligned(growth_tracker, 4) || !aligned(found_inf, 4) ||
        !aligned(step_skipped, 4) || !aligned(attempted_steps, 8) || !aligned(skipped_steps, 8)) {
        set_error("Dynamic loss scaling state has invalid alignment.");
        return -1;
    }
    if (!std::isfinite(growth_factor) || !(growth_factor > 1.0) || !std::isfinite(backoff_factor) ||
        !(backoff_factor > 0.0) || !(backoff_factor < 1.0) || growth_interval <= 0) {
        set_error("Dynamic scale growth/backoff/interval are invalid.");
        return -1;
    }
    compat::AdamState& s = static_cast<compat::AdamPlan*>(opaque)->s;
    s.loss_scale = static_cast<float*>(loss_scale);
    s.growth_tracker = static_cast<int*>(growth_tracker);
    s.found_inf = static_cast<int*>(found_inf);
    s.step_skipped = static_cast<int*>(step_skipped);
    s.attempted = static_cast<long long*>(attempted_steps);
    s.skipped = static_cast<long long*>(skipped_steps);
    s.growth_factor = static_cast<float>(growth_factor);
    s.backoff_factor = static_cast<float>(backoff_factor);
    s.growth_interval = growth_interval;
    return 0;
}

extern "C" int rl_adam_unscale(void* opaque, void* stream) {
    using namespace rl2;
    clear_error();
    compat::AdamPlan* p = static_cast<compat::AdamPlan*>(opaque);
    if (!p || !p->s.loss_scale) {
        set_error("Unscale requires an Adam plan with dynamic loss scaling.");
        return -1;
    }
    const cudaStream_t s = as_stream(stream);
    const cudaError_t e = cudaMemsetAsync(p->s.found_inf, 0, sizeof(int), s);
    if (e != cudaSuccess) {
        set_error("Unscale/check Adam gradients: %s", cudaGetErrorString(e));
        return -1;
    }
    compat::unscale_kernel<<<p->blocks, compat::kT, 0, s>>>(p->tensors, p->first, p->count, p->s.loss_scale,
                                                            p->s.found_inf);
    return launch_status("Unscale/check Adam gradients");
}

extern "C" int rl_adam_step(void* opaque, void* stream) {
    using namespace rl2;
    clear_error();
    compat::AdamPlan* p = static_cast<compat::AdamPlan*>(opaque);
    if (!p) {
        set_error("Adam plan is null.");
        return -1;
    }
    const cudaStream_t s = as_stream(stream);
    compat::adam_prologue_kernel<<<1, 1, 0, s>>>(p->s, p->beta1, p->beta2);
    if (launch_status("Run Adam")) return -1;
    compat::adam_kernel<<<p->blocks, compat::kT, 0, s>>>(p->tensors, p->first, p->count, p->s, p->beta1, p->beta2,
                                                         p->omb1, p->omb2, p->eps);
    return launch_status("Run Adam");
}

extern "C" int rl_adam_destroy(void* opaque) {
    rl2::clear_error();
    delete static_cast<rl2::compat::AdamPlan*>(opaque);
    return 0;
}

extern "C" void* rl_flash_projection_create(size_t count, const void* const* first, const void* const* second,
                                            const size_t* lengths, const int* kinds) {
    return rl2::compat::create_projection(count, first, second, lengths, kinds, nullptr);
}

extern "C" void* rl_flash_projection_create_with_shadows(size_t count, const void* const* first,
                                                         const void* const* second, const size_t* lengths,
                                                         const int* kinds, const void* const* shadows) {
    return rl2::compat::create_projection(count, first, second, lengths, kinds, shadows);
}

extern "C" int rl_flash_projection_step(void* opaque, void* stream) {
    using namespace rl2;
    clear_error();
    auto* t = static_cast<compat::Table<compat::ProjRow>*>(opaque);
    if (!t) {
        set_error("Projection plan is null.");
        return -1;
    }
    compat::project_kernel<<<t->count, compat::kT, 0, as_stream(stream)>>>(t->dev);
    return launch_status("Run FlashSAC projections");
}

extern "C" int rl_flash_projection_destroy(void* opaque) {
    rl2::clear_error();
    delete static_cast<rl2::compat::Table<rl2::compat::ProjRow>*>(opaque);
    return 0;
}

extern "C" void* rl_flash_ema_create(size_t count, const void* const* source, const void* const* target,
                                     const size_t* lengths, float tau) {
    return rl2::compat::create_ema(count, source, target, lengths, tau, nullptr);
}

extern "C" void* rl_flash_ema_create_with_shadows(size_t count, const void* const* source, const void* const* target,
                                                  const size_t* lengths, float tau, const void* const* shadows) {
    return rl2::compat::create_ema(count, source, target, lengths, tau, shadows);
}

extern "C" int rl_flash_ema_step(void* opaque, void* stream) {
    using namespace rl2;
    clear_error();
    auto* t = static_cast<compat::Table<compat::EmaSpan>*>(opaque);
    if (!t) {
        set_error("EMA plan is null.");
        return -1;
    }
    compat::ema_kernel<<<t->count, compat::kT, 0, as_stream(stream)>>>(t->dev, t->tau);
    return launch_status("Run FlashSAC target EMA");
}

extern "C" int rl_flash_ema_destroy(void* opaque) {
    rl2::clear_error();
    delete static_cast<rl2::compat::Table<rl2::compat::EmaSpan>*>(opaque);
    return 0;
}

extern "C" void* rl_zero_create(size_t count, const void* const* pointers, const size_t* lengths) {
    using namespace rl2;
    using namespace rl2::compat;
    clear_error();
    if (!count || !pointers || !lengths) {
        set_error("Zero plan requires nonempty host pointer/length tables.");
        return nullptr;
    }
    std::vector<ZeroSpan> spans;
    uintptr_t end = 0;
    for (size_t i = 0; i < count; ++i) {
        const uintptr_t start = reinterpret_cast<uintptr_t>(pointers[i]);
        if (!start || !aligned(pointers[i], 4) || !lengths[i]) {
            set_error("Zero plan requires aligned, nonempty FP32 spans.");
            return nullptr;
        }
        if (lengths[i] > (std::numeric_limits<uintptr_t>::max() - start) / sizeof(float)) {
            set_error("Zero span pointer arithmetic overflows.");
            return nullptr;
        }
        if (start < end) {
            set_error("Zero spans must be sorted and nonoverlapping.");
            return nullptr;
        }
        end = start + lengths[i] * sizeof(float);
        float* base = static_cast<float*>(const_cast<void*>(pointers[i]));
        for (size_t o = 0; o < lengths[i]; o += kSpan)
            spans.push_back({base + o, static_cast<unsigned>(lengths[i] - o < kSpan ? lengths[i] - o : kSpan)});
    }
    return upload(spans, "Create zero plan");
}

extern "C" int rl_zero_step(void* opaque, void* stream) {
    using namespace rl2;
    clear_error();
    auto* t = static_cast<compat::Table<compat::ZeroSpan>*>(opaque);
    if (!t) {
        set_error("Zero plan is null.");
        return -1;
    }
    compat::zero_kernel<<<t->count, compat::kT, 0, as_stream(stream)>>>(t->dev);
    return launch_status("Grouped zero launch");
}

extern "C" int rl_zero_destroy(void* opaque) {
    rl2::clear_error();
    delete static_cast<rl2::compat::Table<rl2::compat::ZeroSpan>*>(opaque);
    return 0;
}

// ---------------------------------------------------------------------------
// batch norm, RMS norm and categorical heads
// ---------------------------------------------------------------------------

namespace rl2 {
namespace compat {

constexpr int kRowsPerChunk = 256;  // statistics chunk: the scratch contract sizes partials per 256 rows

// Per (32-channel tile, 256-row chunk): the chunk mean and its centred sum of squares,
// exact two-pass over the chunk (the second pass re-reads 32 KB that the first left in L1).
__global__ void __launch_bounds__(kT) bn_chunk_moments_kernel(const float* __restrict__ x, float* partial, int batch,
                                                              int channels, int chunks) {
    __shared__ float red[kT / 32][33];
    const int lane = threadIdx.x & 31, grp = threadIdx.x >> 5;
    const int c = blockIdx.x * 32 + lane;
    const int r0 = blockIdx.y * kRowsPerChunk;
    const int r1 = min(batch, r0 + kRowsPerChunk);
    const bool ok = c < channels;
    float s = 0.0f;
    if (ok)
        for (int r = r0 + grp; r < r1; r += kT / 32) s += x[static_cast<long long>(r) * channels + c];
    red[grp][lane] = s;
    __syncthreads();
    float tot = 0.0f;
#pragma unroll
    for (int g = 0; g < kT / 32; ++g) tot += red[g][lane];
    const float mean = tot / static_cast<float>(r1 - r0);
    __syncthreads();
    float q = 0.0f;
    if (ok)
        for (int r = r0 + grp; r < r1; r += kT / 32) {
            const float d = x[static_cast<long long>(r) * channels + c] - mean;
            q += d * d;
        }
    red[grp][lane] = q;
    __syncthreads();
    if (grp == 0 && ok) {
        float m2 = 0.0f;
#pragma unroll
        for (int g = 0; g < kT / 32; ++g) m2 += red[g][lane];
        partial[static_cast<long long>(blockIdx.y) * channels + c] = mean;
        partial[static_cast<long long>(chunks + blockIdx.y) * channels + c] = m2;
    }
}

// Chan's parallel merge of the chunk moments in chunk order; biased variance for the
// normalisation, unbiased (x B / (B - 1)) for the running estimate (momentum lerp).
__global__ void __launch_bounds__(kT) bn_merge_kernel(const float* __restrict__ partial, float* mean, float* var,
                                                      float* running_mean, float* running_var, int batch,
                                                      int channels, int chunks, float momentum) {
    const int c = blockIdx.x * kT + threadIdx.x;
    if (c >= channels) return;
    float mu = 0.0f, m2 = 0.0f, n = 0.0f;
    for (int k = 0; k < chunks; ++k) {
        const float nk = static_cast<float>(min(kRowsPerChunk, batch - k * kRowsPerChunk));
        const float mk = partial[static_cast<long long>(k) * channels + c];
        const float qk = partial[static_cast<long long>(chunks + k) * channels + c];
        const float nt = n + nk;
        const float delta = mk - mu;
        mu += delta * (nk / nt);
        m2 += qk + delta * delta * (n * nk / nt);
        n = nt;
    }
    const float v = m2 / static_cast<float>(batch);
    mean[c] = mu;
    var[c] = v;
    if (running_mean && running_var) {
        const float unbiased = v * static_cast<float>(batch) / static_cast<float>(batch - 1);
        running_mean[c] = (1.0f - momentum) * running_mean[c] + momentum * mu;
        running_var[c] = (1.0f - momentum) * running_var[c] + momentum * unbiased;
    }
}

// Channel-parallel row loops for the element-wise passes: a thread owns V consecutive
// channels (V = 4 when rows start 16-byte aligned), keeps their constants in registers and
// walks a slab of rows, so no per-element index division or constant reload is needed.
template <int V>
__device__ __forceinline__ void ld_v(const float* p, float (&o)[V]) {
    if constexpr (V == 4) {
        const float4 t = *reinterpret_cast<const float4*>(p);
        o[0] = t.x, o[1] = t.y, o[2] = t.z, o[3] = t.w;
    } else {
        o[0] = *p;
    }
}

template <int V>
__device__ __forceinline__ void st_v(float* p, const float (&o)[V]) {
    if constexpr (V == 4)
        *reinterpret_cast<float4*>(p) = make_float4(o[0], o[1], o[2], o[3]);
    else
        *p = o[0];
}

template <int V>
__device__ __forceinline__ void st_h(__half* p, const float (&o)[V]) {
    if constexpr (V == 4) {
        reinterpret_cast<__half2*>(p)[0] = __floats2half2_rn(o[0], o[1]);
        reinterpret_cast<__half2*>(p)[1] = __floats2half2_rn(o[2], o[3]);
    } else {
        *p = __float2half_rn(o[0]);
    }
}

struct Slab {
    dim3 grid;
    int rows;  // rows per block
};

Slab slab(int batch, int channels, int v) {
    const int gx = (channels + kT * v - 1) / (kT * v);
    int gy = std::max(1, std::min(batch, 592 / gx));
    const int rows = (batch + gy - 1) / gy;
    gy = (batch + rows - 1) / rows;
    return {dim3(static_cast<unsigned>(gx), static_cast<unsigned>(gy)), rows};
}

// y = (x - mean) / sqrt(var + eps) * w + b (w, b optional), ReLU optional, optional fp16 copy.
template <int V>
__global__ void __launch_bounds__(kT) bn_apply_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                                      const float* __restrict__ b, const float* __restrict__ mean,
                                                      const float* __restrict__ var, float* __restrict__ y,
                                                      __half* __restrict__ y16, int batch, int channels, float eps,
                                                      bool relu, int rows) {
    const int c0 = (blockIdx.x * kT + threadIdx.x) * V;
    if (c0 >= channels) return;
    float mu[V], sd[V], wv[V], bv[V];
#pragma unroll
    for (int v = 0; v < V; ++v) {
        mu[v] = mean[c0 + v];
        sd[v] = sqrtf(var[c0 + v] + eps);
        wv[v] = w ? w[c0 + v] : 1.0f;
        bv[v] = b ? b[c0 + v] : 0.0f;
    }
    const int r1 = min(batch, static_cast<int>(blockIdx.y + 1) * rows);
    for (int r = blockIdx.y * rows; r < r1; ++r) {
        const long long o = static_cast<long long>(r) * channels + c0;
        float t[V];
        ld_v<V>(x + o, t);
#pragma unroll
        for (int v = 0; v < V; ++v) {
            float q = (t[v] - mu[v]) / sd[v];
            if (w) q *= wv[v];
            if (b) q += bv[v];
            t[v] = relu && q <= 0.0f ? 0.0f : q;
        }
        st_v<V>(y + o, t);
        if (y16) st_h<V>(y16 + o, t);
    }
}

// Per (channel tile, 256-row chunk): sum g and sum g * xhat, g = dy masked by the ReLU output.
__global__ void __launch_bounds__(kT) bn_chunk_grads_kernel(const float* __restrict__ x, const float* __restrict__ dy,
                                                            const float* __restrict__ y, const float* __restrict__ mean,
                                                            const float* __restrict__ var, float* partial, int batch,
                                                            int channels, int chunks, float eps, bool relu) {
    __shared__ float r_g[kT / 32][33], r_gx[kT / 32][33];
    const int lane = threadIdx.x & 31, grp = threadIdx.x >> 5;
    const int c = blockIdx.x * 32 + lane;
    const int r0 = blockIdx.y * kRowsPerChunk;
    const int r1 = min(batch, r0 + kRowsPerChunk);
    float sg = 0.0f, sgx = 0.0f;
    if (c < channels) {
        const float mu = mean[c], inv = 1.0f / sqrtf(var[c] + eps);
        for (int r = r0 + grp; r < r1; r += kT / 32) {
            const long long o = static_cast<long long>(r) * channels + c;
            const float g = relu && y[o] <= 0.0f ? 0.0f : dy[o];
            sg += g;
            sgx += g * ((x[o] - mu) * inv);
        }
    }
    r_g[grp][lane] = sg;
    r_gx[grp][lane] = sgx;
    __syncthreads();
    if (grp == 0 && c < channels) {
        float a = 0.0f, bsum = 0.0f;
#pragma unroll
        for (int g = 0; g < kT / 32; ++g) {
            a += r_g[g][lane];
            bsum += r_gx[g][lane];
        }
        partial[static_cast<long long>(blockIdx.y) * channels + c] = a;
        partial[static_cast<long long>(chunks + blockIdx.y) * channels + c] = bsum;
    }
}

__global__ void __launch_bounds__(kT) bn_grad_merge_kernel(const float* __restrict__ partial, float* sums, float* dw,
                                                           float* db, int batch, int channels, int chunks) {
    const int c = blockIdx.x * kT + threadIdx.x;
    if (c >= channels) return;
    float sg = 0.0f, sgx = 0.0f;
    for (int k = 0; k < chunks; ++k) {
        sg += partial[static_cast<long long>(k) * channels + c];
        sgx += partial[static_cast<long long>(chunks + k) * channels + c];
    }
    sums[c] = sg / static_cast<float>(batch);
    sums[channels + c] = sgx / static_cast<float>(batch);
    if (dw) dw[c] += sgx;
    if (db) db[c] += sg;
}

// dx (+)= w / sqrt(var + eps) * (g - [training] (mean(g) + xhat * mean(g xhat)))
template <int V, bool kOverwrite>
__global__ void __launch_bounds__(kT) bn_dx_kernel(const float* __restrict__ x, const float* __restrict__ dy,
                                                   const float* __restrict__ y, const float* __restrict__ w,
                                                   const float* __restrict__ mean, const float* __restrict__ var,
                                                   const float* __restrict__ sums, float* dx, __half* dx16, int batch,
                                                   int channels, float eps, bool training, bool relu, int rows) {
    const int c0 = (blockIdx.x * kT + threadIdx.x) * V;
    if (c0 >= channels) return;
    float mu[V], inv[V], wi[V], mg[V], mgx[V];
#pragma unroll
    for (int v = 0; v < V; ++v) {
        inv[v] = 1.0f / sqrtf(var[c0 + v] + eps);
        wi[v] = (w ? w[c0 + v] : 1.0f) * inv[v];
        mu[v] = training ? mean[c0 + v] : 0.0f;
        mg[v] = training ? sums[c0 + v] : 0.0f;
        mgx[v] = training ? sums[channels + c0 + v] : 0.0f;
    }
    const int r1 = min(batch, static_cast<int>(blockIdx.y + 1) * rows);
    for (int r = blockIdx.y * rows; r < r1; ++r) {
        const long long o = static_cast<long long>(r) * channels + c0;
        float g[V], old[V], xv[V], yv[V];
        ld_v<V>(dy + o, g);
        if (relu) ld_v<V>(y + o, yv);
        if (training) ld_v<V>(x + o, xv);
        if (!kOverwrite) ld_v<V>(dx + o, old);
#pragma unroll
        for (int v = 0; v < V; ++v) {
            float q = relu && yv[v] <= 0.0f ? 0.0f : g[v];
            if (training) q = q - mg[v] - (xv[v] - mu[v]) * inv[v] * mgx[v];
            const float c = wi[v] * q;
            g[v] = kOverwrite ? c : old[v] + c;
        }
        st_v<V>(dx + o, g);
        if (dx16) st_h<V>(dx16 + o, g);
    }
}

// One warp per row: var[row] = mean(x^2), y = x / sqrt(var + eps) * w.
__global__ void __launch_bounds__(kT) rms_forward_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                                         float* var, float* y, int batch, int channels, float eps) {
    const int row = blockIdx.x * (kT / 32) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (row >= batch) return;
    const float* xr = x + static_cast<long long>(row) * channels;
    float ss = 0.0f;
    for (int c = lane; c < channels; c += 32) ss += xr[c] * xr[c];
    const float v = warp_sum(ss) / static_cast<float>(channels);
    if (lane == 0) var[row] = v;
    const float rs = sqrtf(v + eps);
    float* yr = y + static_cast<long long>(row) * channels;
    for (int c = lane; c < channels; c += 32) yr[c] = (xr[c] / rs) * (w ? w[c] : 1.0f);
}

// Per (channel tile, 256-row chunk): sum of dy * x / sqrt(var[row] + eps).
__global__ void __launch_bounds__(kT) rms_chunk_dw_kernel(const float* __restrict__ x, const float* __restrict__ dy,
                                                          const float* __restrict__ var, float* partial, int batch,
                                                          int channels, float eps) {
    __shared__ float red[kT / 32][33];
    const int lane = threadIdx.x & 31, grp = threadIdx.x >> 5;
    const int c = blockIdx.x * 32 + lane;
    const int r0 = blockIdx.y * kRowsPerChunk;
    const int r1 = min(batch, r0 + kRowsPerChunk);
    float s = 0.0f;
    if (c < channels)
        for (int r = r0 + grp; r < r1; r += kT / 32) {
            const long long o = static_cast<long long>(r) * channels + c;
            s += dy[o] * (x[o] / sqrtf(var[r] + eps));
        }
    red[grp][lane] = s;
    __syncthreads();
    if (grp == 0 && c < channels) {
        float t = 0.0f;
#pragma unroll
        for (int g = 0; g < kT / 32; ++g) t += red[g][lane];
        partial[static_cast<long long>(blockIdx.y) * channels + c] = t;
    }
}

__global__ void __launch_bounds__(kT) chunk_sum_kernel(const float* __restrict__ partial, float* out, int channels,
                                                       int chunks) {
    const int c = blockIdx.x * kT + threadIdx.x;
    if (c >= channels) return;
    float s = 0.0f;
    for (int k = 0; k < chunks; ++k) s += partial[static_cast<long long>(k) * channels + c];
    out[c] += s;
}

// One warp per row: dx += inv * (dy w - x inv^2 mean_c(dy w x)), inv = 1 / sqrt(var + eps).
__global__ void __launch_bounds__(kT) rms_dx_kernel(const float* __restrict__ x, const float* __restrict__ dy,
                                                    const float* __restrict__ w, const float* __restrict__ var,
                                                    float* dx, int batch, int channels, float eps) {
    const int row = blockIdx.x * (kT / 32) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (row >= batch) return;
    const long long base = static_cast<long long>(row) * channels;
    float s = 0.0f;
    for (int c = lane; c < channels; c += 32) s += dy[base + c] * (w ? w[c] : 1.0f) * x[base + c];
    const float mean = warp_sum(s) / static_cast<float>(channels);
    const float inv = 1.0f / sqrtf(var[row] + eps);
    for (int c = lane; c < channels; c += 32) {
        const float g = dy[base + c] * (w ? w[c] : 1.0f) - x[base + c] * inv * inv * mean;
        dx[base + c] += inv * g;
    }
}

// One warp per row: log_probs = log_softmax(raw + bias), values = sum exp(log_probs) * support.
__global__ void __launch_bounds__(kT) cat_forward_kernel(const float* __restrict__ raw, const float* __restrict__ bias,
                                                         const float* __restrict__ support, float* log_probs,
                                                         float* values, int batch, int bins) {
    const int row = blockIdx.x * (kT / 32) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (row >= batch) return;
    const long long base = static_cast<long long>(row) * bins;
    float mx = -INFINITY;
    for (int j = lane; j < bins; j += 32) mx = fmaxf(mx, raw[base + j] + bias[j]);
    mx = warp_max(mx);
    float se = 0.0f;
    for (int j = lane; j < bins; j += 32) se += expf(raw[base + j] + bias[j] - mx);
    const float lse = logf(warp_sum(se));
    float ev = 0.0f;
    for (int j = lane; j < bins; j += 32) {
        const float lp = raw[base + j] + bias[j] - mx - lse;
        log_probs[base + j] = lp;
        ev += expf(lp) * support[j];
    }
    ev = warp_sum(ev);
    if (lane == 0) values[row] = ev;
}

// One warp per row: g_j = dlp_j + p_j (dq s_j - sum_k (dlp_k + dq p_k s_k)); draw += g, scratch = g.
__global__ void __launch_bounds__(kT) cat_backward_kernel(const float* __restrict__ log_probs,
                                                          const float* __restrict__ support,
                                                          const float* __restrict__ dlog_probs,
                                                          const float* __restrict__ dvalues, float* scratch,
                                                          float* draw, int batch, int bins) {
    const int row = blockIdx.x * (kT / 32) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (row >= batch) return;
    const long long base = static_cast<long long>(row) * bins;
    const float dq = dvalues ? dvalues[row] : 0.0f;
    float t = 0.0f;
    for (int j = lane; j < bins; j += 32)
        t += (dlog_probs ? dlog_probs[base + j] : 0.0f) + dq * expf(log_probs[base + j]) * support[j];
    t = warp_sum(t);
    for (int j = lane; j < bins; j += 32) {
        const float p = expf(log_probs[base + j]);
        const float g = (dlog_probs ? dlog_probs[base + j] : 0.0f) + p * (dq * support[j] - t);
        if (draw) draw[base + j] += g;
        if (scratch) scratch[base + j] = g;
    }
}

__device__ __forceinline__ void atomic_max_float(float* addr, float v) {
    int* a = reinterpret_cast<int*>(addr);
    int seen = *reinterpret_cast<volatile int*>(a);
    while (__int_as_float(seen) < v) {
        const int prev = atomicCAS(a, seen, __float_as_int(v));
        if (prev == seen) break;
        seen = prev;
    }
}

// Adds v into t[key] for every run of equal keys across the warp's lanes: a segmented
// inclusive scan (runs found from lane-order key changes, so any key sequence is handled)
// leaves each run's sum in its last lane, which commits it. The keys of one row are monotone
// in the atom index (the two-hot location is a monotone function of the support value), so
// every key has at most one run per call and the sums do not depend on scheduling.
__device__ __forceinline__ void run_commit(float* t, int key, float v, int lane) {
    const int kprev = __shfl_up_sync(0xffffffffu, key, 1);
    const bool head = lane == 0 || kprev != key;
    const unsigned heads = __ballot_sync(0xffffffffu, head);
    const int run = __popc(heads & (lane == 31 ? 0xffffffffu : ((2u << lane) - 1u)));
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const float vo = __shfl_up_sync(0xffffffffu, v, o);
        const int ro = __shfl_up_sync(0xffffffffu, run, o);
        if (lane >= o && ro == run) v += vo;
    }
    const int rnext = __shfl_down_sync(0xffffffffu, run, 1);
    if ((lane == 31 || rnext != run) && key >= 0) atomicAdd(t + key, v);
}

// One warp per row, the row's target in shared memory: lanes compute the two-hot split of
// 32 atoms at a time, then the lower and the upper contributions are committed by runs.
__global__ void __launch_bounds__(kT) cat_target_kernel(const float* __restrict__ q, const float* __restrict__ log_probs,
                                                        const float* __restrict__ reward,
                                                        const float* __restrict__ terminated,
                                                        const float* __restrict__ discount,
                                                        const float* __restrict__ next_log_probs,
                                                        const float* __restrict__ alpha, float* target,
                                                        float* maximum_entropy, int batch, int bins, float min_v,
                                                        float max_v) {
    extern __shared__ float rows_s[];
    const int wpb = blockDim.x >> 5;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row = blockIdx.x * wpb + warp;
    if (row >= batch) return;  // warp-uniform
    float* t = rows_s + static_cast<long long>(warp) * bins;
    for (int j = lane; j < bins; j += 32) t[j] = 0.0f;
    __syncwarp();
    const float ent = alpha[0] * next_log_probs[row];
    const int twin = q[3LL * batch + row] < q[static_cast<long long>(batch) + row] ? 1 : 0;
    const float* lp = log_probs + (static_cast<long long>(twin) * 2 * batch + batch + row) * bins;
    const float width = (max_v - min_v) / static_cast<float>(bins - 1);
    const float r = reward[row], disc = discount[row], live = 1.0f - terminated[row];
    for (int j0 = 0; j0 < bins; j0 += 32) {
        const int j = j0 + lane;
        int lo = -1, up = -1;
        float wl = 0.0f, wu = 0.0f;
        if (j < bins) {
            const float z = min_v + static_cast<float>(j) * width;
            const float v = r + disc * (z - ent) * live;
            const float loc = (fminf(fmaxf(v, min_v), max_v) - min_v) / width;
            lo = min(max(static_cast<int>(floorf(loc)), 0), bins - 1);
            up = min(lo + 1, bins - 1);
            const float frac = loc - static_cast<float>(lo);
            const float p = expf(lp[j]);
            wl = p * (1.0f - frac);
            wu = p * frac;
        }
        run_commit(t, lo, wl, lane);
        __syncwarp();
        run_commit(t, up, wu, lane);
        __syncwarp();
    }
    float* out = target + static_cast<long long>(row) * bins;
    for (int j = lane; j < bins; j += 32) out[j] = t[j];
    if (lane == 0) atomic_max_float(maximum_entropy, ent);
}

bool norm_dims(int batch, int channels, float eps) {
    if (batch > 0 && channels > 0 && std::isfinite(eps) && eps > 0.0f &&
        static_cast<long long>(batch) * channels <= std::numeric_limits<int>::max())
        return true;
    set_error("FlashSAC normalization requires positive finite epsilon and B*C fitting signed int.");
    return false;
}

int bn_forward(const float* x, const float* w, const float* b, float* running_mean, float* running_var, float* mean,
               float* var, float* partial, float* y, __half* y16, int batch, int channels, float eps, float momentum,
               int training, int relu, void* stream) {
    clear_error();
    if (!norm_dims(batch, channels, eps)) return -1;
    if (!x || !y || !mean || !var || !partial || (!training && (!running_mean || !running_var)) ||
        (training && running_mean && batch < 2)) {
        set_error("Invalid BN forward arrays/count.");
        return -1;
    }
    if (y16 && !aligned(y16, 2)) {
        set_error("Invalid FP16 BN output alignment.");
        return -1;
    }
    const cudaStream_t s = as_stream(stream);
    const int chunks = (batch + kRowsPerChunk - 1) / kRowsPerChunk;
    if (training) {
        bn_chunk_moments_kernel<<<dim3((channels + 31) / 32, chunks), kT, 0, s>>>(x, partial, batch, channels, chunks);
        bn_merge_kernel<<<(channels + kT - 1) / kT, kT, 0, s>>>(partial, mean, var, running_mean, running_var, batch,
                                                               channels, chunks, momentum);
    }
    const bool v4 = channels % 4 == 0 && aligned(x, 16) && aligned(y, 16) && (!y16 || aligned(y16, 8));
    const Slab sl = slab(batch, channels, v4 ? 4 : 1);
    const float* mu = training ? mean : running_mean;
    const float* va = training ? var : running_var;
    if (v4)
        bn_apply_kernel<4><<<sl.grid, kT, 0, s>>>(x, w, b, mu, va, y, y16, batch, channels, eps, relu != 0, sl.rows);
    else
        bn_apply_kernel<1><<<sl.grid, kT, 0, s>>>(x, w, b, mu, va, y, y16, batch, channels, eps, relu != 0, sl.rows);
    return launch_status("Run FlashSAC BatchNorm forward");
}

int bn_backward(const float* x, const float* dy, const float* y, const float* w, const float* mean, const float* var,
                float* partial, float* sums, float* dx, float* dw, float* db, __half* dx16, int batch, int channels,
                float eps, int training, int relu, void* stream, bool overwrite) {
    clear_error();
    if (!norm_dims(batch, channels, eps)) return -1;
    if (!x || !dy || !y || !mean || !var || !partial || !sums) {
        set_error("Invalid BN backward arrays.");
        return -1;
    }
    if (dx16 && (!dx || !aligned(dx16, 2))) {
        set_error("FP16 BN input adjoint requires aligned storage and a FP32 input adjoint.");
        return -1;
    }
    const cudaStream_t s = as_stream(stream);
    const int chunks = (batch + kRowsPerChunk - 1) / kRowsPerChunk;
    if ((training && dx) || dw || db) {
        bn_chunk_grads_kernel<<<dim3((channels + 31) / 32, chunks), kT, 0, s>>>(x, dy, y, mean, var, partial, batch,
                                                                               channels, chunks, eps, relu != 0);
        bn_grad_merge_kernel<<<(channels + kT - 1) / kT, kT, 0, s>>>(partial, sums, dw, db, batch, channels, chunks);
    }
    if (dx) {
        const bool v4 = channels % 4 == 0 && aligned(x, 16) && aligned(dy, 16) && aligned(y, 16) && aligned(dx, 16) &&
                        (!dx16 || aligned(dx16, 8));
        const Slab sl = slab(batch, channels, v4 ? 4 : 1);
        const bool tr = training != 0, rl = relu != 0;
        if (v4 && overwrite)
            bn_dx_kernel<4, true><<<sl.grid, kT, 0, s>>>(x, dy, y, w, mean, var, sums, dx, dx16, batch, channels, eps,
                                                         tr, rl, sl.rows);
        else if (v4)
            bn_dx_kernel<4, false><<<sl.grid, kT, 0, s>>>(x, dy, y, w, mean, var, sums, dx, dx16, batch, channels, eps,
                                                          tr, rl, sl.rows);
        else if (overwrite)
            bn_dx_kernel<1, true><<<sl.grid, kT, 0, s>>>(x, dy, y, w, mean, var, sums, dx, dx16, batch, channels, eps,
                                                         tr, rl, sl.rows);
        else
            bn_dx_kernel<1, false><<<sl.grid, kT, 0, s>>>(x, dy, y, w, mean, var, sums, dx, dx16, batch, channels,
                                                          eps, tr, rl, sl.rows);
    }
    return launch_status("Run FlashSAC BatchNorm backward");
}

}  // namespace compat
}  // namespace rl2

extern "C" int rl_flash_bn_forward(const float* x, const float* w, const float* b, float* running_mean,
                                   float* running_var, float* mean, float* var, float* partial, float* y, int batch,
                                   int channels, float eps, float momentum, int training, int relu, void* stream) {
    return rl2::compat::bn_forward(x, w, b, running_mean, running_var, mean, var, partial, y, nullptr, batch,
                                   channels, eps, momentum, training, relu, stream);
}

extern "C" int rl_flash_bn_forward_with_fp16(const float* x, const float* w, const float* b, float* running_mean,
                                             float* running_var, float* mean, float* var, float* partial, float* y,
                                             void* half_output, int batch, int channels, float eps, float momentum,
                                             int training, int relu, void* stream) {
    if (!half_output) {
        rl2::set_error("FP16 BN output must be nonnull.");
        return -1;
    }
    return rl2::compat::bn_forward(x, w, b, running_mean, running_var, mean, var, partial, y,
                                   static_cast<__half*>(half_output), batch, channels, eps, momentum, training, relu,
                                   stream);
}

extern "C" int rl_flash_bn_backward(const float* x, const float* dy, const float* y, const float* w, const float* mean,
                                    const float* var, float* partial, float* sums, float* dx, float* dw, float* db,
                                    int batch, int channels, float eps, int training, int relu, void* stream) {
    return rl2::compat::bn_backward(x, dy, y, w, mean, var, partial, sums, dx, dw, db, nullptr, batch, channels, eps,
                                    training, relu, stream, false);
}

extern "C" int rl_flash_bn_backward_with_fp16(const float* x, const float* dy, const float* y, const float* w,
                                              const float* mean, const float* var, float* partial, float* sums,
                                              float* dx, float* dw, float* db, void* half_dx, int batch, int channels,
                                              float eps, int training, int relu, void* stream) {
    if (!half_dx) {
        rl2::set_error("FP16 BN input adjoint must be nonnull.");
        return -1;
    }
    return rl2::compat::bn_backward(x, dy, y, w, mean, var, partial, sums, dx, dw, db, static_cast<__half*>(half_dx),
                                    batch, channels, eps, training, relu, stream, false);
}

extern "C" int rl_flash_bn_backward_controlled(const float* x, const float* dy, const float* y, const float* w,
                                               const float* mean, const float* var, float* partial, float* sums,
                                               float* dx, float* dw, float* db, void* half_dx, int overwrite_dx,
                                               int batch, int channels, float eps, int training, int relu,
                                               void* stream) {
    if (!dx || (overwrite_dx != 0 && overwrite_dx != 1)) {
        rl2::set_error("Controlled BN backward requires dx and a Boolean overwrite flag.");
        return -1;
    }
    return rl2::compat::bn_backward(x, dy, y, w, mean, var, partial, sums, dx, dw, db, static_cast<__half*>(half_dx),
                                    batch, channels, eps, training, relu, stream, overwrite_dx != 0);
}

extern "C" int rl_flash_rms_forward(const float* x, const float* w, float* var, float* y, int batch, int channels,
                                    float eps, void* stream) {
    using namespace rl2;
    clear_error();
    if (!compat::norm_dims(batch, channels, eps)) return -1;
    if (!x || !var || !y) {
        set_error("Invalid RMSNorm forward arrays.");
        return -1;
    }
    compat::rms_forward_kernel<<<(batch + 7) / 8, compat::kT, 0, as_stream(stream)>>>(x, w, var, y, batch, channels,
                                                                                       eps);
    return launch_status("Run FlashSAC RMSNorm forward");
}

extern "C" int rl_flash_rms_backward(const float* x, const float* dy, const float* w, const float* var, float* partial,
                                     float* dx, float* dw, int batch, int channels, float eps, void* stream) {
    using namespace rl2;
    clear_error();
    if (!compat::norm_dims(batch, channels, eps)) return -1;
    if (!x || !dy || !var || !partial) {
        set_error("Invalid RMSNorm backward arrays.");
        return -1;
    }
    const cudaStream_t s = as_stream(stream);
    const int chunks = (batch + compat::kRowsPerChunk - 1) / compat::kRowsPerChunk;
    if (dw) {
        compat::rms_chunk_dw_kernel<<<dim3((channels + 31) / 32, chunks), compat::kT, 0, s>>>(x, dy, var, partial,
                                                                                              batch, channels, eps);
        compat::chunk_sum_kernel<<<(channels + compat::kT - 1) / compat::kT, compat::kT, 0, s>>>(partial, dw, channels,
                                                                                                 chunks);
    }
    if (dx)
        compat::rms_dx_kernel<<<(batch + 7) / 8, compat::kT, 0, s>>>(x, dy, w, var, dx, batch, channels, eps);
    return launch_status("Run FlashSAC RMSNorm backward");
}

extern "C" int rl_flash_categorical_forward(const void* raw, const void* bias, const void* support, void* log_probs,
                                            void* values, int batch, int bins, void* stream) {
    using namespace rl2;
    clear_error();
    if (!raw || !bias || !support || !log_probs || !values || batch < 1 || bins < 2) {
        set_error("Categorical forward requires nonempty FP32 buffers and at least two bins.");
        return -1;
    }
    compat::cat_forward_kernel<<<(batch + 7) / 8, compat::kT, 0, as_stream(stream)>>>(
        static_cast<const float*>(raw), static_cast<const float*>(bias), static_cast<const float*>(support),
        static_cast<float*>(log_probs), static_cast<float*>(values), batch, bins);
    return launch_status("Categorical forward");
}

extern "C" int rl_flash_categorical_backward(const void* log_probs, const void* support, const void* dlog_probs,
                                             const void* dvalues, void* scratch, void* draw, void* dbias, int batch,
                                             int bins, void* stream) {
    using namespace rl2;
    clear_error();
    if (!log_probs || !support || (!draw && !dbias) || (dbias && !scratch) || batch < 1 || bins < 2) {
        set_error("Categorical backward requires FP32 buffers, gradients and valid dimensions.");
        return -1;
    }
    const cudaStream_t s = as_stream(stream);
    compat::cat_backward_kernel<<<(batch + 7) / 8, compat::kT, 0, s>>>(
        static_cast<const float*>(log_probs), static_cast<const float*>(support),
        static_cast<const float*>(dlog_probs), static_cast<const float*>(dvalues),
        dbias ? static_cast<float*>(scratch) : nullptr, static_cast<float*>(draw), batch, bins);
    if (launch_status("Categorical backward")) return -1;
    if (dbias) {  // the per-row gradients in scratch are summed in two fixed-order passes
        const int tiles = (bins + 31) / 32;
        const int slabs = std::max(1, std::min((batch + 31) / 32, 600 / tiles));
        const int rows = (batch + slabs - 1) / slabs;
        const int used = (batch + rows - 1) / rows;
        float* sc = static_cast<float*>(scratch);
        compat::slab_sum_kernel<<<dim3(tiles, used), compat::kT, 0, s>>>(sc, batch, bins, rows);
        compat::column_sum_kernel<<<tiles, compat::kColT, 0, s>>>(sc, static_cast<float*>(dbias), used, bins,
                                                                 static_cast<long long>(rows) * bins);
    }
    return launch_status("Categorical bias backward");
}

extern "C" int rl_flash_categorical_target(const void* q, const void* log_probs, const void* reward,
                                           const void* terminated, const void* discount, const void* next_log_probs,
                                           const void* alpha, void* target, void* maximum_entropy, int batch, int bins,
                                           float min_v, float max_v, void* stream) {
    using namespace rl2;
    clear_error();
    if (!q || !log_probs || !reward || !terminated || !discount || !next_log_probs || !alpha || !target ||
        !maximum_entropy || batch < 1 || bins < 2 || bins > 4096 || !(min_v < max_v)) {
        set_error("Categorical target requires FP32 buffers, valid support and 2..4096 bins.");
        return -1;
    }
    // warps per block: as many rows as fit 48 KB of shared memory, at most 8
    const int wpb = std::max(1, std::min(8, static_cast<int>((48 * 1024) / (static_cast<size_t>(bins) * 4))));
    compat::cat_target_kernel<<<(batch + wpb - 1) / wpb, 32 * wpb, static_cast<size_t>(wpb) * bins * 4,
                                as_stream(stream)>>>(
        static_cast<const float*>(q), static_cast<const float*>(log_probs), static_cast<const float*>(reward),
        static_cast<const float*>(terminated), static_cast<const float*>(discount),
        static_cast<const float*>(next_log_probs), static_cast<const float*>(alpha), static_cast<float*>(target),
        static_cast<float*>(maximum_entropy), batch, bins, min_v, max_v);
    return launch_status("Categorical target");
}
