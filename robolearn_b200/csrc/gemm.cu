// tcgen05 / TMEM / TMA GEMM for the residual-MLP forward and backward products.
//
// One kernel computes, for each batch z (twin critic index),
//     D[z][m][n] = scale * sum_k A[z][m][k] * B[z][n][k]   (+ bias[n]) (+ residual[m][n]) (+ D_old)
// with A and B each either K-contiguous ("K-major") or M/N-contiguous
// ("MN-major") in global memory. That covers the three products of a linear
// layer y = x W^T that the reference issues as cuBLASLt plans
// (src/robolearn/cuda/linear.py:179-185): forward (A=x K-major, B=W K-major),
// input gradient dx = dy W (A=dy K-major, B=W MN-major) and weight gradient
// dW = dy^T x (A=dy MN-major, B=x MN-major, contraction over the batch rows).
//
// Two operand kinds:
//   kind 0: fp16 operands, fp32 accumulation (tcgen05.mma kind::f16);
//   kind 1: fp32 operands through a three-product tf32 split, A = A_hi + A_lo,
//           D = A_hi B_hi + A_hi B_lo + A_lo B_hi (tcgen05.mma kind::tf32), which
//           keeps the products within ~1e-6 relative of fp32 (the reference's
//           FP32 recipe uses pedantic fp32 GEMMs, kernels.cu:436-444).
//
// Layout: persistent kernel, one CTA per SM walking 128 x BN output tiles (BN a
// multiple of 16, <= 256). K is staged 128 bytes at a time through a multi-stage
// TMA -> smem ring with 128-byte swizzle; the accumulator lives in TMEM, double
// buffered (2 x BN columns) so that the epilogue of tile i overlaps the main loop of
// tile i + 1 and the producer runs ahead across tile boundaries. Warp roles: warp 0 =
// TMA producer, warp 1 = TMEM allocation + MMA issue (one elected thread), warps 2..9
// = epilogue (two per TMEM lane quarter). Every mbarrier wait is bounded by
// wall-clock time, reports through the caller's health word and stops the other
// roles through a shared abort word.
//
// The epilogue stages each 32 x 16 accumulator slice in shared memory and walks it
// 8 rows x 16 columns per warp step, so every global access of a warp covers whole
// row segments (bias, residual, fp32 output, fp16 or tf32 hi/lo operand plane).
// Extras: per-column partial moments over each 32-row group (mean and sum of squared
// deviations) feed training-mode batch norm without another read of the output.

#include "planes.cuh"

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <new>

namespace rl2 {
namespace gemm {

constexpr int kBM = 128;
constexpr int kEpiWarps = 8;                  // two per TMEM lane quarter (register- and TMA-store epilogues)
constexpr int kEpiWarpsWide = 16;             // four per quarter: transposed-accumulator plans
constexpr int kThreads = 64 + 32 * kEpiWarps;  // producer warp, MMA warp, epilogue warps
__host__ __device__ constexpr int threads_for(int epi) { return 64 + 32 * epi; }
constexpr int kMaxSmem = 232448;           // dynamic shared memory one CTA may use
// k-blocks per tensor-core accumulation chain of a 3xTF32 product (32 k each: 256 products,
// about 2e-6 relative from the accumulation), folded with round-to-nearest fp32 additions
// by the epilogue
constexpr int kChainBlocks = 8;
// k-blocks per tile (64 each for fp16) from which a product runs on CTA pairs
constexpr int kPairMinKBlocks = 16;

struct Params {
    int M, N, K;
    int batch, splits, kblocks_total, kblocks_per_split;
    int BN, a_batched, b_batched;
    float* d;
    long long ldd, d_bstride, d_split_stride;
    int accumulate;
    const float* bias;
    long long bias_bstride;
    const float* residual;
    long long ldr, r_bstride;
    float* stat_mean;
    float* stat_m2;
    long long stat_bstride;
    const float* scale;
    int* health;
    Plane out_plane;
    int tiles_n, tiles_m, tiles_total;  // persistent work list (n fastest)
    uint32_t buf_cols;                  // TMEM columns per accumulator buffer (power of two >= 32, >= BN)
    bool vec_d, vec_res, vec_bias, vec_plane, vec_stat;  // 16-byte (plane: 8-byte) column-group access allowed
    int activation;  // 0 none, 1 ELU, 2 tanh
    const float* aux;  // stored activation outputs: multiply by the derivative instead of applying f
    long long ld_aux, aux_bstride;
    bool vec_aux;
    // store-engine epilogue: output boxes written by TMA stores (tma_d: fp32 output map,
    // tma_plane: fp16 plane map)
    bool tma_epi, tma_d, tma_plane;
    bool tma_reduce;   // store-engine epilogue adds into D in L2 (D += result: in-place residual / accumulate)
    const float* bn_mean;  // evaluation-mode batch norm of the output columns (transposed plans)
    const float* bn_invstd;
    const float* bn_gamma;
    const float* bn_beta;
    long long bn_tstride;
    int bn_relu;
    bool swap;         // accumulator holds D^T: kernel M = output columns, kernel N = output rows
    int out_m, out_n;  // output rows / columns (the kernel's N / M when swapped)
    int epi_bufs;      // staging boxes per warp and output (store-engine epilogue: 1 or 2)
    int stage_floats;  // per-warp staging floats (multiple of 256: 1 KB-aligned regions)
    int kc_blocks;     // k-blocks per tensor-core accumulation chunk (0: one chain per tile)
    int epi_warps;     // epilogue warps of the launch (kEpiWarps, or kEpiWarpsWide for transposed plans)
    bool pair;         // CTA pairs: 256-row tiles over two SMs (tcgen05 cta_group::2), tiles_m counts pairs
    int bn_cta;        // rows of the B tile each CTA stages (BN, or BN / 2 in a pair)
};

// Epilogue activations. ELU (alpha 1) and tanh; derivatives from the stored outputs y.
__device__ __forceinline__ float act_fwd(int a, float x) { return a == 1 ? (x > 0.f ? x : expf(x) - 1.0f) : tanhf(x); }
__device__ __forceinline__ float act_grad(int a, float y) { return a == 1 ? (y > 0.f ? 1.0f : y + 1.0f) : 1.0f - y * y; }
__device__ __forceinline__ float4 act4(int a, const float* aux_row, float4 x, float4 y) {
    if (aux_row) return make_float4(x.x * act_grad(a, y.x), x.y * act_grad(a, y.y), x.z * act_grad(a, y.z), x.w * act_grad(a, y.w));
    return make_float4(act_fwd(a, x.x), act_fwd(a, x.y), act_fwd(a, x.z), act_fwd(a, x.w));
}

// Shared-memory matrix descriptor. layout 2 = 128-byte swizzle (16-byte granules,
// 8-row atoms); layout 1 = 128-byte swizzle with 32-byte granules (4-row atoms),
// the only form tcgen05 accepts for MN-major 32-bit (tf32) operands.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo, uint32_t layout = 2) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((addr >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
    d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
    d |= static_cast<uint64_t>(1) << 46;  // descriptor version (sm_100)
    d |= static_cast<uint64_t>(layout) << 61;
    return d;
}

// Wall-clock bounded mbarrier wait (4 s) that also gives up as soon as another role of
// the CTA has raised the shared abort word, so a lost arrival cannot hang the GPU.
__device__ __forceinline__ bool wait_bar(uint64_t* bar, uint32_t phase, int* health, volatile int* abort_flag) {
    if (ptx::mbar_try_wait(bar, phase)) return true;
    uint64_t start;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(start));
    for (uint32_t i = 1;; ++i) {
        if (ptx::mbar_try_wait(bar, phase)) return true;
        if ((i & 1023u) == 0) {
            if (*abort_flag) return false;
            uint64_t now;
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(now));
            if (now - start > 4000000000ull) {
                if (health) atomicOr(health, kHealthTimeout);
                *abort_flag = 1;
                return false;
            }
        }
    }
}

// Output tile of a linear work index: n fastest (consecutive CTAs share the A rows),
// then m, then (batch, split).
struct Tile {
    int n_tile, m_tile, z, split, kb_begin, kb_end;
};

// Persistent walk over the work list: CTA b takes tiles b, b + gridDim.x, ...; in pair mode
// the two CTAs of cluster c (blocks 2c, 2c + 1) take pair tiles c, c + gridDim.x / 2, ...
__device__ __forceinline__ int tile_first(const Params& p) { return p.pair ? static_cast<int>(blockIdx.x >> 1) : blockIdx.x; }
__device__ __forceinline__ int tile_step(const Params& p) { return p.pair ? static_cast<int>(gridDim.x >> 1) : gridDim.x; }

// A pair tile covers kernel rows [256 m, 256 m + 256): each CTA of the pair owns the 128-row
// half of its rank (its TMEM holds those rows of the accumulator), so decode() returns that
// half as a 128-row m_tile and the epilogues are the same as for one CTA.
__device__ __forceinline__ Tile decode(const Params& p, int t) {
    Tile w;
    w.n_tile = t % p.tiles_n;
    t /= p.tiles_n;
    w.m_tile = t % p.tiles_m;
    if (p.pair) w.m_tile = 2 * w.m_tile + static_cast<int>(blockIdx.x & 1);
    t /= p.tiles_m;
    w.z = t / p.splits;
    w.split = t % p.splits;
    w.kb_begin = w.split * p.kblocks_per_split;
    w.kb_end = min(p.kblocks_total, w.kb_begin + p.kblocks_per_split);
    return w;
}

// An epilogue warp is done with an accumulator buffer: arrive on the MMA issuer's barrier
// (in a pair, the leader CTA's, which counts the warps of both CTAs).
__device__ __forceinline__ void release_acc(const Params& p, uint64_t* bar) {
    if (p.pair)
        ptx::mbar_arrive_cluster(ptx::cluster_addr(bar, 0));
    else
        ptx::mbar_arrive(bar);
}

template <int KIND, int A_MN, int B_MN, bool PAIR>
__device__ __forceinline__ void produce(const CUtensorMap* tma_a, const CUtensorMap* tma_b, const CUtensorMap* tma_a_lo,
                                        const CUtensorMap* tma_b_lo, const Params& p, int stages, uint8_t* smem,
                                        uint32_t stage_bytes, uint64_t* full, uint64_t* empty, volatile int* abort_flag) {
    constexpr int kElem = KIND == 0 ? 2 : 4;
    constexpr int kBK = 128 / kElem;
    constexpr int kChunk = 128 / kElem;
    constexpr int kPlanes = KIND == 0 ? 1 : 2;
    const int BNC = p.bn_cta;  // B rows this CTA stages
    const uint32_t a_bytes = kBM * 128;
    const uint32_t b_bytes = static_cast<uint32_t>(BNC) * 128;
    // In a pair, both CTAs' loads complete on the leader's full barrier, which the leader
    // alone arms with the pair's bytes; each CTA waits on its own empty barrier (the MMA
    // issuer commits to both).
    const uint32_t rank = PAIR ? (blockIdx.x & 1u) : 0u;
    const bool arms = !PAIR || rank == 0;
    ptx::prefetch_tensormap(tma_a);
    ptx::prefetch_tensormap(tma_b);
    int s = 0;
    uint32_t phase = 0;
    long long issued = 0;
    bool ok = true;
    for (int t = tile_first(p); t < p.tiles_total && ok; t += tile_step(p)) {
        const Tile w = decode(p, t);
        const int za = p.a_batched ? w.z : 0;
        const int zb = p.b_batched ? w.z : 0;
        const int m0 = w.m_tile * kBM;
        const int n0 = w.n_tile * p.BN + static_cast<int>(rank) * BNC;
        for (int kb = w.kb_begin; kb < w.kb_end; ++kb) {
            if (!wait_bar(&empty[s], phase ^ 1, p.health, abort_flag)) {
                ok = false;
                break;
            }
            if (arms) ptx::mbar_arrive_expect_tx(&full[s], PAIR ? 2 * stage_bytes : stage_bytes);
            ++issued;
            const uint32_t bar = PAIR ? ptx::cluster_addr(&full[s], 0) : 0u;
            uint8_t* sa = smem + s * stage_bytes;
            uint8_t* sb = sa + a_bytes * kPlanes;
            const int k0 = kb * kBK;
            for (int plane = 0; plane < kPlanes; ++plane) {
                const CUtensorMap* ma = plane == 0 ? tma_a : tma_a_lo;
                const CUtensorMap* mb = plane == 0 ? tma_b : tma_b_lo;
                uint8_t* da = sa + plane * a_bytes;
                uint8_t* db = sb + plane * b_bytes;
                auto load = [&](uint8_t* dst, const CUtensorMap* map, int x, int y, int z) {
                    if (PAIR)
                        ptx::tma_load_3d_pair(dst, map, bar, x, y, z);
                    else
                        ptx::tma_load_3d(dst, map, &full[s], x, y, z);
                };
                if (A_MN) {
                    for (int c = 0; c < kBM / kChunk; ++c) load(da + c * (kBK * 128), ma, m0 + c * kChunk, k0, za);
                } else {
                    load(da, ma, k0, m0, za);
                }
                if (B_MN) {
                    for (int c = 0; c < BNC / kChunk; ++c) load(db + c * (kBK * 128), mb, n0 + c * kChunk, k0, zb);
                } else {
                    load(db, mb, k0, n0, zb);
                }
            }
            if (++s == stages) {
                s = 0;
                phase ^= 1;
            }
        }
    }
    // Before the CTA may exit (and free its shared memory), every armed stage must have
    // landed, including loads nobody consumed after an abort (bounded waits). In a pair the
    // leader's barriers also count the follower's loads, and the follower leaves only
    // after the leader (cluster barrier at the end of the kernel).
    if (!arms) return;
    for (int st = 0; st < stages; ++st) {
        const long long armed = issued > st ? (issued - 1 - st) / stages + 1 : 0;
        if (armed > 0) {
            volatile int no_abort = 0;
            wait_bar(&full[st], static_cast<uint32_t>((armed - 1) & 1), p.health, &no_abort);
        }
    }
}

// One elected thread issues every tcgen05.mma of the CTA (of the pair: the leader's).
// Local tile i accumulates into TMEM buffer i & 1 once the epilogue has drained that
// buffer's previous tile. In a pair the MMA spans both CTAs (M = 256: A rows 128 per CTA,
// B rows BN / 2 per CTA at the same shared-memory offsets, accumulator rows in each CTA's
// TMEM), and its completions are committed to the barriers of both CTAs.
template <int KIND, int A_MN, int B_MN, bool PAIR>
__device__ __forceinline__ void issue(const Params& p, int stages, uint8_t* smem, uint32_t stage_bytes, uint64_t* full,
                                      uint64_t* empty, uint64_t* acc_full, uint64_t* acc_empty, uint32_t tmem,
                                      uint32_t buf_cols, volatile int* abort_flag) {
    static_assert(!PAIR || KIND == 0, "CTA pairs run fp16 products");
    constexpr int kElem = KIND == 0 ? 2 : 4;
    constexpr int kBK = 128 / kElem;
    constexpr int kUK = 32 / kElem;
    constexpr int kPlanes = KIND == 0 ? 1 : 2;
    const int BN = p.BN;
    const uint32_t a_bytes = kBM * 128;
    const uint32_t b_bytes = static_cast<uint32_t>(p.bn_cta) * 128;
    const uint32_t fmt = KIND == 0 ? 0u : 2u;
    const uint32_t mma_m = PAIR ? 2 * kBM : kBM;
    const uint32_t idesc = (1u << 4) | (fmt << 7) | (fmt << 10) | (static_cast<uint32_t>(A_MN) << 15) |
                           (static_cast<uint32_t>(B_MN) << 16) | (static_cast<uint32_t>(BN >> 3) << 17) |
                           ((mma_m >> 4) << 24);
    // MN-major: LBO = distance between 128-byte MN chunks (one box), SBO = one swizzle
    // atom of K rows (8 rows = 1024 B for fp16; 4 rows = 512 B for the tf32 32-byte-granule
    // swizzle). K-major: SBO = 8 rows of 128 bytes, LBO unused (encoded as 16 bytes).
    const uint32_t lbo_mn = kBK * 128;
    const uint32_t sbo_mn = KIND == 0 ? 1024u : 512u;
    const uint32_t lay_mn = KIND == 0 ? 2u : 1u;
    auto commit = [&](uint64_t* bar) {
        if (PAIR) {
            ptx::mma_commit_pair(ptx::cluster_addr(bar, 0));
            ptx::mma_commit_pair(ptx::cluster_addr(bar, 1));
        } else {
            ptx::mma_commit(bar);
        }
    };
    int s = 0;
    uint32_t phase = 0;
    int i = 0;  // accumulation chain counter: one per tile, or one per chunk of kc_blocks k-blocks
    for (int t = tile_first(p); t < p.tiles_total; t += tile_step(p)) {
        const Tile w = decode(p, t);
        const int span = p.kc_blocks > 0 ? p.kc_blocks : w.kb_end - w.kb_begin;
        for (int c0 = w.kb_begin; c0 < w.kb_end; c0 += span, ++i) {
            const int c1 = min(c0 + span, w.kb_end);
            const int buf = i & 1;
            if (!wait_bar(&acc_empty[buf], ((i >> 1) & 1) ^ 1, p.health, abort_flag)) return;
            ptx::tc_fence_after();
            const uint32_t d_tmem = tmem + static_cast<uint32_t>(buf) * buf_cols;
            for (int kb = c0; kb < c1; ++kb) {
                if (!wait_bar(&full[s], phase, p.health, abort_flag)) return;
                ptx::tc_fence_after();
                const uint32_t sa = ptx::smem_u32(smem + s * stage_bytes);
                const uint32_t sb = sa + a_bytes * kPlanes;
                const bool first = kb == c0;
#pragma unroll
                for (int j = 0; j < kBK / kUK; ++j) {
                    const uint32_t a_off = A_MN ? j * kUK * 128 : j * 32;
                    const uint32_t b_off = B_MN ? j * kUK * 128 : j * 32;
                    const uint64_t da =
                        A_MN ? smem_desc(sa + a_off, lbo_mn, sbo_mn, lay_mn) : smem_desc(sa + a_off, 16, 1024);
                    const uint64_t db =
                        B_MN ? smem_desc(sb + b_off, lbo_mn, sbo_mn, lay_mn) : smem_desc(sb + b_off, 16, 1024);
                    const uint32_t acc = (!first || j > 0) ? 1u : 0u;
                    if (PAIR) {
                        ptx::mma_f16_pair(d_tmem, da, db, idesc, acc);
                    } else if (KIND == 0) {
                        ptx::mma_f16(d_tmem, da, db, idesc, acc);
                    } else {
                        const uint64_t da_lo = A_MN ? smem_desc(sa + a_bytes + a_off, lbo_mn, sbo_mn, lay_mn)
                                                    : smem_desc(sa + a_bytes + a_off, 16, 1024);
                        const uint64_t db_lo = B_MN ? smem_desc(sb + b_bytes + b_off, lbo_mn, sbo_mn, lay_mn)
                                                    : smem_desc(sb + b_bytes + b_off, 16, 1024);
                        ptx::mma_tf32(d_tmem, da_lo, db, idesc, acc);
                        ptx::mma_tf32(d_tmem, da, db_lo, idesc, 1u);
                        ptx::mma_tf32(d_tmem, da, db, idesc, 1u);
                    }
                }
                commit(&empty[s]);
                if (++s == stages) {
                    s = 0;
                    phase ^= 1;
                }
            }
            commit(&acc_full[buf]);
        }
    }
}

// Chunked accumulation (p.kc_blocks > 0): the MMA issuer accumulates every kc_blocks
// k-blocks of a tile into a fresh chain in TMEM buffer i & 1 (i counting chains). The
// tensor cores add into an fp32 accumulator with an error that grows with the chain's
// length (about 7e-9 K relative, measured), so chains stay short and the epilogue warps
// add them with ordinary round-to-nearest fp32 additions: chains 0 .. n-2 into a running
// sum in TMEM columns [2 buf_cols, 3 buf_cols), and the running sum into the last chain's
// buffer, which the epilogue then reads as the tile's accumulator. Each warp folds its own
// TMEM lane quarter and every other 16-column group (the two warps of a quarter); the
// warps then meet on an mbarrier (bounded wait) before any of them reads the total. On
// return, i indexes the tile's last chain.
__device__ __forceinline__ bool fold_chunks(const Params& p, const Tile& w, uint64_t* acc_full, uint64_t* acc_empty,
                                            uint64_t* epi_sync, uint32_t& epi_phase, uint32_t tmem, int& i,
                                            volatile int* abort_flag) {
    const int chains = (w.kb_end - w.kb_begin + p.kc_blocks - 1) / p.kc_blocks;
    if (chains <= 1) return true;
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int q = warp & 3;
    const int slot = (warp - 2) >> 2;
    const uint32_t lanes = static_cast<uint32_t>(q * 32) << 16;
    const uint32_t run = tmem + 2u * p.buf_cols + lanes;
    const int groups = (p.BN + 15) / 16;
    for (int c = 0; c < chains; ++c, ++i) {
        const int buf = i & 1;
        if (!wait_bar(&acc_full[buf], (i >> 1) & 1, p.health, abort_flag)) return false;
        ptx::tc_fence_after();
        const uint32_t src = tmem + static_cast<uint32_t>(buf) * p.buf_cols + lanes;
        const bool last = c == chains - 1;
        for (int g = slot; g < groups; g += p.epi_warps / 4) {
            float v[16];
            ptx::tmem_ld16(src + 16u * g, v);
            if (c > 0) {
                float r[16];
                ptx::tmem_ld16(run + 16u * g, r);
#pragma unroll
                for (int e = 0; e < 16; ++e) v[e] = __fadd_rn(r[e], v[e]);
            }
            ptx::tmem_st16(last ? src + 16u * g : run + 16u * g, v);
        }
        ptx::tmem_st_wait();
        ptx::tc_fence_before();
        __syncwarp();
        if (!last) {
            if (lane == 0) release_acc(p, &acc_empty[buf]);  // this chain's buffer is free again
        } else {
            if (lane == 0) ptx::mbar_arrive(epi_sync);
            if (!wait_bar(epi_sync, epi_phase, p.health, abort_flag)) return false;
            epi_phase ^= 1u;
            ptx::tc_fence_after();
        }
    }
    --i;
    return true;
}

// Staged 32 x 16 slice: rows of 16 floats, 16-byte chunk j of row r stored at chunk
// j ^ ((r >> 1) & 3), which keeps both the row-per-lane writes and the 8-row x 16-column
// reads free of bank conflicts.
constexpr int kStagePitch = 16;
// Per-warp staging region (Params::stage_floats floats, a multiple of 256 so every region
// starts on a 1 KB boundary): the register-store epilogue uses one 32 x 16 fp32 slice;
// the store-engine epilogue uses epi_bufs fp32 boxes (2 KB each) then epi_bufs fp16 plane
// boxes (1 KB each), every box on a 1 KB boundary (beyond the swizzle repeats).

__device__ __forceinline__ float4 load_cols(const float* src, int n, bool vec) {
    if (vec && n == 4) return *reinterpret_cast<const float4*>(src);
    float4 r = make_float4(0.f, 0.f, 0.f, 0.f);
    if (n > 0) r.x = src[0];
    if (n > 1) r.y = src[1];
    if (n > 2) r.z = src[2];
    if (n > 3) r.w = src[3];
    return r;
}

__device__ __forceinline__ void store_cols(float* dst, float4 v, int n, bool vec) {
    if (vec && n == 4) {
        *reinterpret_cast<float4*>(dst) = v;
        return;
    }
    if (n > 0) dst[0] = v.x;
    if (n > 1) dst[1] = v.y;
    if (n > 2) dst[2] = v.z;
    if (n > 3) dst[3] = v.w;
}

__device__ __forceinline__ float4 add4(float4 a, float4 b) { return make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w); }

__device__ __forceinline__ float4 xor_sum4(float4 v, int mask) {
    v.x += __shfl_xor_sync(0xffffffffu, v.x, mask);
    v.y += __shfl_xor_sync(0xffffffffu, v.y, mask);
    v.z += __shfl_xor_sync(0xffffffffu, v.z, mask);
    v.w += __shfl_xor_sync(0xffffffffu, v.w, mask);
    return v;
}

// Epilogue warps 2 .. 2 + kEpiWarps - 1, kEpiWarps / 4 per TMEM lane quarter: warp w may
// only read TMEM lanes (tile rows) 32*(w % 4) .. +31, and the warps of a quarter take
// every (kEpiWarps / 4)-th 16-column chunk. A 32 x 16 accumulator slice is read with
// lane = row, staged in shared memory and walked 8 rows x 16 columns per step (lane = 4
// consecutive columns of one row), so every global access covers whole row segments.
// Interior chunks (32 valid rows, 16 valid columns, vector-aligned operands) take a
// branch-free path; edge chunks take a guarded path. The bias of all of a warp's chunks
// is fetched once per tile before the accumulator wait, and a chunk's residual / old
// output rows are fetched before its TMEM read. After its last TMEM read of a tile each
// warp releases the accumulator buffer to the MMA issuer.
constexpr int kEpiSlots = kEpiWarps / 4;        // warps per TMEM lane quarter
constexpr int kMaxChunks = (256 / 16 + kEpiSlots - 1) / kEpiSlots;  // chunks per warp and tile (BN <= 256)

__device__ __forceinline__ float4 pick4(const float4 (&v)[kMaxChunks], int k) {
    float4 r = v[0];
#pragma unroll
    for (int j = 1; j < kMaxChunks; ++j)
        if (k == j) r = v[j];
    return r;
}

__device__ __forceinline__ void drain(const Params& p, uint64_t* acc_full, uint64_t* acc_empty, uint64_t* epi_sync,
                                      uint32_t tmem, float* staging, volatile int* abort_flag) {
    uint32_t epi_phase = 0;
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int q = warp & 3;
    const int slot = (warp - 2) >> 2;
    float* sq = staging + (warp - 2) * p.stage_floats;
    const int cg = lane & 3;
    const int rsub = lane >> 2;
    const float scale = p.scale ? *p.scale : 1.0f;
    const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
    PlaneWriter pw(p.out_plane);
    const bool plane_on = pw.active();
    const bool fast_ok = (!p.d || p.vec_d) && (!p.residual || p.vec_res) && (!p.bias || p.vec_bias) &&
                         (!plane_on || p.vec_plane) && (!p.stat_mean || p.vec_stat) && (!p.aux || p.vec_aux);
    const int actv = p.activation;
    const int BN = p.BN;
    int i = 0;
    for (int t = tile_first(p); t < p.tiles_total; t += tile_step(p), ++i) {
        const Tile w = decode(p, t);
        if (p.kc_blocks > 0 && !fold_chunks(p, w, acc_full, acc_empty, epi_sync, epi_phase, tmem, i, abort_flag))
            break;
        const int buf = i & 1;
        const int r0 = w.m_tile * kBM + q * 32;
        const int valid = min(max(p.M - r0, 0), 32);
        const float inv_valid = 1.0f / static_cast<float>(max(valid, 1));  // exact for full 32-row groups
        float* d = p.d ? p.d + static_cast<long long>(w.z) * p.d_bstride + static_cast<long long>(w.split) * p.d_split_stride
                       : nullptr;
        const float* bias = p.bias ? p.bias + static_cast<long long>(w.z) * p.bias_bstride : nullptr;
        const float* res = p.residual ? p.residual + static_cast<long long>(w.z) * p.r_bstride : nullptr;
        const float* aux = p.aux ? p.aux + static_cast<long long>(w.z) * p.aux_bstride : nullptr;
        const long long group = static_cast<long long>(w.m_tile * kBM) / 32 + q;
        float4 bias_k[kMaxChunks];
#pragma unroll
        for (int k = 0; k < kMaxChunks; ++k) {
            const int c0 = 16 * slot + 16 * kEpiSlots * k;
            const int col = w.n_tile * BN + c0 + 4 * cg;
            const int nc = c0 < BN ? max(0, min(4, p.N - col)) : 0;
            bias_k[k] = (bias && nc > 0) ? load_cols(bias + col, nc, p.vec_bias) : zero;
        }
        if (!wait_bar(&acc_full[buf], (i >> 1) & 1, p.health, abort_flag)) break;
        ptx::tc_fence_after();
        const uint32_t t_base = tmem + static_cast<uint32_t>(buf) * p.buf_cols + (static_cast<uint32_t>(q * 32) << 16);
        for (int k = 0; k < kMaxChunks; ++k) {
            const int c0 = 16 * slot + 16 * kEpiSlots * k;
            const int col0 = w.n_tile * BN + c0;
            if (c0 >= BN || col0 >= p.N) break;  // warp-uniform
            const int col = col0 + 4 * cg;
            // interior chunks add at most one of residual / old output (both: guarded path)
            const float* add_src = res ? res : ((d && p.accumulate) ? d : nullptr);
            const long long add_ld = res ? p.ldr : p.ldd;
            const bool fast = fast_ok && valid == 32 && col0 + 16 <= p.N && !(res && d && p.accumulate);
            float4 rv[4], av[4];
            if (fast && add_src) {
#pragma unroll
                for (int it = 0; it < 4; ++it)
                    rv[it] = *reinterpret_cast<const float4*>(add_src + static_cast<long long>(r0 + 8 * it + rsub) * add_ld + col);
            }
            if (fast && aux) {
#pragma unroll
                for (int it = 0; it < 4; ++it)
                    av[it] = *reinterpret_cast<const float4*>(aux + static_cast<long long>(r0 + 8 * it + rsub) * p.ld_aux + col);
            }
            {
                float v[16];
                ptx::tmem_ld16(t_base + static_cast<uint32_t>(c0), v);
                float4* mine = reinterpret_cast<float4*>(sq + lane * kStagePitch);
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    mine[j ^ ((lane >> 1) & 3)] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
            }
            __syncwarp();
            float4 x[4];
#pragma unroll
            for (int it = 0; it < 4; ++it) {
                const float4 a = *reinterpret_cast<const float4*>(sq + (8 * it + rsub) * kStagePitch + 4 * (cg ^ ((rsub >> 1) & 3)));
                x[it] = make_float4(a.x * scale, a.y * scale, a.z * scale, a.w * scale);
            }
            const float4 b4 = pick4(bias_k, k);
            if (fast) {
                // ---- interior chunk: no per-row or per-lane guards ----
#pragma unroll
                for (int it = 0; it < 4; ++it) {
                    if (bias) x[it] = add4(x[it], b4);
                    if (add_src) x[it] = add4(x[it], rv[it]);
                    if (actv) x[it] = act4(actv, aux, x[it], aux ? av[it] : x[it]);
                }
                if (d) {
#pragma unroll
                    for (int it = 0; it < 4; ++it)
                        *reinterpret_cast<float4*>(d + static_cast<long long>(r0 + 8 * it + rsub) * p.ldd + col) = x[it];
                }
                if (plane_on) {
#pragma unroll
                    for (int it = 0; it < 4; ++it) pw.store4(w.z, r0 + 8 * it + rsub, col, x[it]);
                }
            } else {
                // ---- edge chunk: guarded per row and per column ----
                const int nc = max(0, min(4, p.N - col));
#pragma unroll
                for (int it = 0; it < 4; ++it) {
                    const int r = 8 * it + rsub;
                    const long long row = r0 + r;
                    if (bias) x[it] = add4(x[it], b4);
                    if (r < valid && nc > 0) {
                        if (res) x[it] = add4(x[it], load_cols(res + row * p.ldr + col, nc, p.vec_res));
                        float* dp = d ? d + row * p.ldd + col : nullptr;
                        if (dp && p.accumulate) x[it] = add4(x[it], load_cols(dp, nc, p.vec_d));
                        if (actv) {
                            const float* arow = aux ? aux + row * p.ld_aux + col : nullptr;
                            x[it] = act4(actv, arow, x[it], arow ? load_cols(arow, nc, p.vec_aux) : x[it]);
                        }
                        if (dp) store_cols(dp, x[it], nc, p.vec_d);
                        if (plane_on) {
                            if (nc == 4 && p.vec_plane) {
                                pw.store4(w.z, row, col, x[it]);
                            } else {
                                if (nc > 0) pw.store(w.z, row, col, x[it].x);
                                if (nc > 1) pw.store(w.z, row, col + 1, x[it].y);
                                if (nc > 2) pw.store(w.z, row, col + 2, x[it].z);
                                if (nc > 3) pw.store(w.z, row, col + 3, x[it].w);
                            }
                        }
                    }
                    if (r >= valid) x[it] = zero;
                }
            }
            if (p.stat_mean && valid > 0) {
                // rows >= valid hold zeros here (interior chunks have none)
                float4 sum = add4(add4(x[0], x[1]), add4(x[2], x[3]));
                sum = xor_sum4(xor_sum4(xor_sum4(sum, 4), 8), 16);
                if (!p.stat_m2) {  // sums mode: per-group column sums only
                    const int nc = max(0, min(4, p.N - col));
                    if (rsub == 0 && nc > 0)
                        store_cols(p.stat_mean + static_cast<long long>(w.z) * p.stat_bstride + group * p.N + col, sum,
                                   nc, p.vec_stat);
                    __syncwarp();
                    continue;
                }
                const float4 mean = make_float4(sum.x * inv_valid, sum.y * inv_valid, sum.z * inv_valid, sum.w * inv_valid);
                float4 m2 = zero;
#pragma unroll
                for (int it = 0; it < 4; ++it) {
                    if (8 * it + rsub < valid) {
                        const float4 dv = make_float4(x[it].x - mean.x, x[it].y - mean.y, x[it].z - mean.z,
                                                      x[it].w - mean.w);
                        m2 = make_float4(m2.x + dv.x * dv.x, m2.y + dv.y * dv.y, m2.z + dv.z * dv.z, m2.w + dv.w * dv.w);
                    }
                }
                m2 = xor_sum4(xor_sum4(xor_sum4(m2, 4), 8), 16);
                const int nc = max(0, min(4, p.N - col));
                if (rsub == 0 && nc > 0) {
                    const long long idx = static_cast<long long>(w.z) * p.stat_bstride + group * p.N + col;
                    store_cols(p.stat_mean + idx, mean, nc, p.vec_stat);
                    store_cols(p.stat_m2 + idx, m2, nc, p.vec_stat);
                }
            }
            __syncwarp();
        }
        ptx::tc_fence_before();
        __syncwarp();
        if (lane == 0) release_acc(p, &acc_empty[buf]);
    }
    pw.flush();
}

// Store-engine epilogue, for products without activation or split-K whose residual, if
// any, is the output itself (D += result then goes out as TMA reduce-add stores).
// A warp reads its 32 x 16 accumulator slices with lane = row (the next slice's TMEM read
// is in flight while the current one is processed), applies scale and bias in registers
// and writes each slice once into a staging box in the TMA layout (fp32 box: 64-byte
// rows, 16-byte chunk j of row r at slot j ^ ((r >> 1) & 3), the 64-byte swizzle; fp16
// plane box: 32-byte rows, chunk j at slot j ^ ((r >> 2) & 1), the 32-byte swizzle). One
// lane hands the boxes to the TMA store engine, which writes whole lines and leaves out
// rows and columns beyond the output; with two boxes per warp the engine reads one while
// the warp fills the other. Column moments are then read back from the fp32 box with
// lane = (column c, row half h): lane (c, h) visits rows 16h + (e ^ h), so the 32 lanes of
// every load hit 32 different banks.
struct TmaEpi {
    const CUtensorMap* tma_d;
    const CUtensorMap* tma_p;
    float* region;  // this warp's staging: [fp32 box][fp32 box][fp16 box][fp16 box]
    int nbuf;
    int lane, sc, sh, cq, dsw, psw;
    bool scaled, plane16;
    float scale;
    PlaneWriter pw;
    uint32_t count;  // slices handed to the store engine so far

    __device__ __forceinline__ TmaEpi(const CUtensorMap* d, const CUtensorMap* pm, const Params& p, float* r, int nb)
        : tma_d(d), tma_p(pm), region(r), nbuf(nb), pw(p.out_plane), count(0) {
        lane = threadIdx.x & 31;
        sc = lane & 15;
        sh = lane >> 4;
        cq = sc >> 2;
        dsw = (lane >> 1) & 3;
        psw = (lane >> 2) & 1;
        scaled = p.scale != nullptr;
        scale = scaled ? *p.scale : 1.0f;
        plane16 = p.tma_plane;
    }

    // One 32 x 16 slice: rows r0 .. r0 + 31 (valid of them inside the output), columns
    // col0 .. col0 + 15 (ncols inside), accumulator values v (lane = row).
    __device__ __forceinline__ void slice(const Params& p, const float* bias, float (&v)[16], int col0, int ncols,
                                          int r0, int valid, float inv_valid, int z, long long stat_row) {
        if (bias) {
            if (ncols == 16 && p.vec_bias) {
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const float4 b4 = __ldg(reinterpret_cast<const float4*>(bias + col0) + j);
                    v[4 * j] = (scaled ? v[4 * j] * scale : v[4 * j]) + b4.x;
                    v[4 * j + 1] = (scaled ? v[4 * j + 1] * scale : v[4 * j + 1]) + b4.y;
                    v[4 * j + 2] = (scaled ? v[4 * j + 2] * scale : v[4 * j + 2]) + b4.z;
                    v[4 * j + 3] = (scaled ? v[4 * j + 3] * scale : v[4 * j + 3]) + b4.w;
                }
            } else {
#pragma unroll
                for (int j = 0; j < 16; ++j)
                    v[j] = (scaled ? v[j] * scale : v[j]) + (j < ncols ? __ldg(bias + col0 + j) : 0.0f);
            }
        } else if (scaled) {
#pragma unroll
            for (int j = 0; j < 16; ++j) v[j] = v[j] * scale;
        }
        const int b = nbuf == 2 ? static_cast<int>(count & 1u) : 0;
        float* sd = region + b * 512;
        __half* sp = reinterpret_cast<__half*>(region + nbuf * 512 + b * 256);
        // the box this slice uses has been read by the store engine
        if (lane == 0) {
            if (nbuf == 2)
                ptx::bulk_wait_read1();
            else
                ptx::bulk_wait_read0();
        }
        __syncwarp();
        float4* drow = reinterpret_cast<float4*>(sd + lane * 16);
#pragma unroll
        for (int j = 0; j < 4; ++j) drow[j ^ dsw] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
        if (plane16) {
            uint32_t h[8];
            bool over = false;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const float s0 = v[2 * j] * pw.scale, s1 = v[2 * j + 1] * pw.scale;
                over |= (2 * j < ncols && !(fabsf(s0) <= 65504.0f)) || (2 * j + 1 < ncols && !(fabsf(s1) <= 65504.0f));
                const __half2 hh = __floats2half2_rn(s0, s1);
                h[j] = *reinterpret_cast<const uint32_t*>(&hh);
            }
            pw.overflow |= over && lane < valid;
            uint4* prow = reinterpret_cast<uint4*>(sp + lane * 16);
            prow[psw] = make_uint4(h[0], h[1], h[2], h[3]);
            prow[1 ^ psw] = make_uint4(h[4], h[5], h[6], h[7]);
        }
        ptx::fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
            if (p.tma_reduce)
                ptx::tma_reduce_add_3d(tma_d, sd, col0, r0, z);
            else if (p.tma_d)
                ptx::tma_store_3d(tma_d, sd, col0, r0, z);
            if (plane16) ptx::tma_store_3d(tma_p, sp, col0, r0, z);
            ptx::bulk_commit();
        }
        ++count;
        if (!p.stat_mean) return;
        // rows 16h + (e ^ h): e = 2m -> 16h + h + 2m, e = 2m + 1 -> 16h + 1 - h + 2m; swizzle term m & 3
        const float* col_even = sd + (16 * sh + sh) * 16 + (sc & 3);
        const float* col_odd = sd + (16 * sh + 1 - sh) * 16 + (sc & 3);
        float y[16];
        float sum = 0.0f;
#pragma unroll
        for (int e = 0; e < 16; ++e) {
            const int m = e >> 1;
            y[e] = ((e & 1) ? col_odd : col_even)[32 * m + 4 * (cq ^ (m & 3))];
            if (valid < 32 && 16 * sh + (e ^ sh) >= valid) y[e] = 0.0f;
            sum += y[e];
        }
        sum += __shfl_xor_sync(0xffffffffu, sum, 16);
        const long long idx = static_cast<long long>(z) * p.stat_bstride + stat_row * p.N + col0 + sc;
        if (!p.stat_m2) {  // sums mode: per-group column sums only
            if (sh == 0 && sc < ncols) p.stat_mean[idx] = sum;
            return;
        }
        const float mean = sum * inv_valid;
        float m2 = 0.0f;
#pragma unroll
        for (int e = 0; e < 16; ++e) {
            const float dv = y[e] - mean;
            if (valid == 32 || 16 * sh + (e ^ sh) < valid) m2 = fmaf(dv, dv, m2);
        }
        m2 += __shfl_xor_sync(0xffffffffu, m2, 16);
        if (sh == 0 && sc < ncols) {
            p.stat_mean[idx] = mean;
            p.stat_m2[idx] = m2;
        }
    }
};

__device__ __forceinline__ void drain_tma(const CUtensorMap* tma_d, const CUtensorMap* tma_p, const Params& p,
                                          uint64_t* acc_full, uint64_t* acc_empty, uint64_t* epi_sync, uint32_t tmem,
                                          float* staging, volatile int* abort_flag) {
    uint32_t epi_phase = 0;
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int q = warp & 3;
    const int slot = (warp - 2) >> 2;
    TmaEpi epi(tma_d, tma_p, p, staging + (warp - 2) * p.stage_floats, p.epi_bufs);
    const int BN = p.BN;
    int i = 0;
    for (int t = tile_first(p); t < p.tiles_total; t += tile_step(p), ++i) {
        const Tile w = decode(p, t);
        if (p.kc_blocks > 0 && !fold_chunks(p, w, acc_full, acc_empty, epi_sync, epi_phase, tmem, i, abort_flag))
            break;
        const int buf = i & 1;
        const int r0 = w.m_tile * kBM + q * 32;
        const int valid = min(max(p.M - r0, 0), 32);
        const float inv_valid = 1.0f / static_cast<float>(max(valid, 1));
        const float* bias = p.bias ? p.bias + static_cast<long long>(w.z) * p.bias_bstride : nullptr;
        const long long stat_row = static_cast<long long>(w.m_tile * kBM) / 32 + q;
        // this warp's slices of the tile: c0 = 16 * slot + 16 * kEpiSlots * k
        const int col_base = w.n_tile * BN + 16 * slot;
        int nk = 0;
        while (nk < kMaxChunks && 16 * slot + 16 * kEpiSlots * nk < BN && col_base + 16 * kEpiSlots * nk < p.N) ++nk;
        if (valid == 0) nk = 0;
        if (!wait_bar(&acc_full[buf], (i >> 1) & 1, p.health, abort_flag)) break;
        ptx::tc_fence_after();
        const uint32_t t_base = tmem + static_cast<uint32_t>(buf) * p.buf_cols + (static_cast<uint32_t>(q * 32) << 16) +
                                static_cast<uint32_t>(16 * slot);
        // the next slice's TMEM read is in flight while this one is processed
        uint32_t cur[16];
        if (nk > 0) {
            ptx::tmem_ld16_issue(t_base, cur);
            ptx::tmem_ld_wait(cur);
        }
#pragma unroll 1
        for (int k = 0; k < nk; ++k) {
            uint32_t nxt[16];
            const bool more = k + 1 < nk;
            if (more) ptx::tmem_ld16_issue(t_base + static_cast<uint32_t>(16 * kEpiSlots * (k + 1)), nxt);
            float v[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) v[j] = __uint_as_float(cur[j]);
            const int col0 = col_base + 16 * kEpiSlots * k;
            epi.slice(p, bias, v, col0, min(16, p.N - col0), r0, valid, inv_valid, w.z, stat_row);
            if (more) {
                ptx::tmem_ld_wait(nxt);
#pragma unroll
                for (int j = 0; j < 16; ++j) cur[j] = nxt[j];
            }
        }
        ptx::tc_fence_before();
        __syncwarp();
        if (lane == 0) release_acc(p, &acc_empty[buf]);
    }
    if (lane == 0) ptx::bulk_wait0();
    __syncwarp();
    epi.pw.flush();
}

// Transposed-accumulator epilogue (swapped plans: every product whose output has at least
// 128 columns and whose tile width is chosen by the plan). TMEM lane = output column, TMEM
// column = output row, so one 32x32b.x32 read gives every lane 32 consecutive rows of its
// own column. Everything after that is per-lane register work plus global accesses in
// which, for each row, the 32 lanes touch 32 consecutive columns (whole 128-byte lines):
// residual / old-output / stored-activation rows are loaded that way, the output and the
// operand plane are stored that way, and the 32-row column moments are pairwise sums in
// registers (no shared memory and no shuffles). The two warps of a TMEM lane quarter take
// alternate 32-row groups of the tile.
__device__ __forceinline__ float sum32(const float (&x)[32]) {
    float s[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) s[j] = x[j] + x[j + 16];
#pragma unroll
    for (int w = 8; w >= 1; w >>= 1)
#pragma unroll
        for (int j = 0; j < w; ++j) s[j] = s[j] + s[j + w];
    return s[0];
}

// kLoads: the product adds rows of another array (residual / old output) or scales by stored
// activation outputs; the instance without them keeps the add / aux registers out of the
// common path.
template <bool kLoads>
__device__ __forceinline__ void drain_swap(const Params& p, uint64_t* acc_full, uint64_t* acc_empty,
                                           uint64_t* epi_sync, uint32_t tmem, volatile int* abort_flag) {
    uint32_t epi_phase = 0;
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int q = warp & 3;
    const int slot = (warp - 2) >> 2;
    const bool scaled = p.scale != nullptr;
    const float scale = scaled ? *p.scale : 1.0f;
    PlaneWriter pw(p.out_plane);
    const bool plane_on = pw.active();
    const int actv = p.activation;
    const int BN = p.BN;  // output rows per tile (a multiple of 32)
    int i = 0;
    for (int t = tile_first(p); t < p.tiles_total; t += tile_step(p), ++i) {
        const Tile w = decode(p, t);
        if (p.kc_blocks > 0 && !fold_chunks(p, w, acc_full, acc_empty, epi_sync, epi_phase, tmem, i, abort_flag))
            break;
        const int buf = i & 1;
        const int col0 = w.m_tile * kBM + q * 32;  // this warp's 32 output columns
        const int n = col0 + lane;
        const bool col_ok = n < p.out_n;
        const float bv = (p.bias && col_ok) ? __ldg(p.bias + static_cast<long long>(w.z) * p.bias_bstride + n) : 0.0f;
        float bn_mu = 0.0f, bn_is = 1.0f, bn_g = 1.0f, bn_b = 0.0f;
        if (p.bn_mean && col_ok) {
            const long long o = static_cast<long long>(w.z) * p.bn_tstride + n;
            bn_mu = __ldg(p.bn_mean + o);
            bn_is = __ldg(p.bn_invstd + o);
            bn_g = __ldg(p.bn_gamma + o);
            bn_b = __ldg(p.bn_beta + o);
        }
        float* dcol = p.d ? p.d + static_cast<long long>(w.z) * p.d_bstride +
                                static_cast<long long>(w.split) * p.d_split_stride + n
                          : nullptr;
        const float* rcol = kLoads && p.residual ? p.residual + static_cast<long long>(w.z) * p.r_bstride + n : nullptr;
        const float* acol = kLoads && p.aux ? p.aux + static_cast<long long>(w.z) * p.aux_bstride + n : nullptr;
        if (!wait_bar(&acc_full[buf], (i >> 1) & 1, p.health, abort_flag)) break;
        ptx::tc_fence_after();
        const uint32_t t_base = tmem + static_cast<uint32_t>(buf) * p.buf_cols + (static_cast<uint32_t>(q * 32) << 16);
        for (int gl = slot; gl < BN / 32 && col0 < p.out_n; gl += p.epi_warps / 4) {
            const int m0 = w.n_tile * BN + 32 * gl;  // first output row of the group
            const int vr = min(32, p.out_m - m0);
            if (vr <= 0) break;  // warp-uniform
            const bool full = vr == 32;
            // rows added to the product (residual, else the old output) and stored activation
            // outputs: loaded before the TMEM read so their latency overlaps it
            const float* add_src = !kLoads ? nullptr
                                   : rcol ? rcol + static_cast<long long>(m0) * p.ldr
                                          : (dcol && p.accumulate ? dcol + static_cast<long long>(m0) * p.ldd : nullptr);
            const long long add_ld = rcol ? p.ldr : p.ldd;
            float add[32], aux[32];
            if (add_src && col_ok) {
#pragma unroll
                for (int r = 0; r < 32; ++r) add[r] = (full || r < vr) ? add_src[static_cast<long long>(r) * add_ld] : 0.0f;
            }
            if (actv && acol && col_ok) {
                const float* src = acol + static_cast<long long>(m0) * p.ld_aux;
#pragma unroll
                for (int r = 0; r < 32; ++r) aux[r] = (full || r < vr) ? src[static_cast<long long>(r) * p.ld_aux] : 0.0f;
            }
            float v[32];
            ptx::tmem_ld32(t_base + static_cast<uint32_t>(32 * gl), v);
#pragma unroll
            for (int r = 0; r < 32; ++r) {
                if (scaled) v[r] = v[r] * scale;
                if (p.bias) v[r] = v[r] + bv;
            }
            if (p.bn_mean) {  // evaluation-mode batch norm (+ ReLU); a residual is added after it
#pragma unroll
                for (int r = 0; r < 32; ++r) {
                    const float o = (v[r] - bn_mu) * bn_is * bn_g + bn_b;
                    v[r] = p.bn_relu ? fmaxf(o, 0.0f) : o;
                }
            }
            if (col_ok) {
                if (add_src) {
#pragma unroll
                    for (int r = 0; r < 32; ++r) v[r] = v[r] + add[r];
                }
                if (kLoads && rcol && dcol && p.accumulate) {  // both: the old output after the residual
                    const float* src = dcol + static_cast<long long>(m0) * p.ldd;
#pragma unroll
                    for (int r = 0; r < 32; ++r)
                        if (full || r < vr) v[r] = v[r] + src[static_cast<long long>(r) * p.ldd];
                }
                // the activation kind is uniform: one specialised loop each (no per-element
                // selection between the ELU and tanh code)
                if (actv == 1) {
                    if (acol) {
#pragma unroll
                        for (int r = 0; r < 32; ++r) v[r] = v[r] * (aux[r] > 0.f ? 1.0f : aux[r] + 1.0f);
                    } else {
#pragma unroll
                        for (int r = 0; r < 32; ++r) v[r] = v[r] > 0.f ? v[r] : expf(v[r]) - 1.0f;
                    }
                } else if (actv == 2) {
                    if (acol) {
#pragma unroll
                        for (int r = 0; r < 32; ++r) v[r] = v[r] * (1.0f - aux[r] * aux[r]);
                    } else {
#pragma unroll
                        for (int r = 0; r < 32; ++r) v[r] = tanhf(v[r]);
                    }
                }
            }
            // (whole 32-row groups take unpredicated copies of the same arithmetic)
            if (p.stat_mean) {
                float x[32];
                float sum;
                if (full) {
                    sum = sum32(v);
                } else {
#pragma unroll
                    for (int r = 0; r < 32; ++r) x[r] = r < vr ? v[r] : 0.0f;
                    sum = sum32(x);
                }
                const long long idx =
                    static_cast<long long>(w.z) * p.stat_bstride + static_cast<long long>(m0 / 32) * p.out_n + n;
                if (!p.stat_m2) {
                    if (col_ok) p.stat_mean[idx] = sum;
                } else {
                    const float mean = sum * (full ? 0.03125f : 1.0f / static_cast<float>(vr));
                    if (full) {
#pragma unroll
                        for (int r = 0; r < 32; ++r) {
                            const float dv = v[r] - mean;
                            x[r] = dv * dv;
                        }
                    } else {
#pragma unroll
                        for (int r = 0; r < 32; ++r) {
                            const float dv = v[r] - mean;
                            x[r] = r < vr ? dv * dv : 0.0f;
                        }
                    }
                    const float m2 = sum32(x);
                    if (col_ok) {
                        p.stat_mean[idx] = mean;
                        p.stat_m2[idx] = m2;
                    }
                }
            }
            if (col_ok) {
                if (dcol) {
                    float* dst = dcol + static_cast<long long>(m0) * p.ldd;
                    const long long ld = p.ldd;
                    if (full) {
#pragma unroll
                        for (int r = 0; r < 32; ++r) dst[r * ld] = v[r];
                    } else {
#pragma unroll
                        for (int r = 0; r < 32; ++r)
                            if (r < vr) dst[r * ld] = v[r];
                    }
                }
                if (plane_on) {
                    const long long o = static_cast<long long>(w.z) * pw.p.tstride + static_cast<long long>(m0) * pw.p.ld + n;
                    if (pw.p.h16) {
                        bool over = false;
                        __half* dst = pw.p.h16 + o;
                        const long long ld = pw.p.ld;
                        if (full) {
#pragma unroll
                            for (int r = 0; r < 32; ++r) {
                                const float s = v[r] * pw.scale;
                                over |= !(fabsf(s) <= 65504.0f);
                                dst[r * ld] = __float2half_rn(s);
                            }
                        } else {
#pragma unroll
                            for (int r = 0; r < 32; ++r) {
                                if (r < vr) {
                                    const float s = v[r] * pw.scale;
                                    over |= !(fabsf(s) <= 65504.0f);
                                    dst[r * ld] = __float2half_rn(s);
                                }
                            }
                        }
                        pw.overflow |= over;
                    } else {
#pragma unroll
                        for (int r = 0; r < 32; ++r) {
                            if (full || r < vr) {
                                const float h = tf32_hi(v[r]);
                                if (pw.p.hi) pw.p.hi[o + static_cast<long long>(r) * pw.p.ld] = h;
                                pw.p.lo[o + static_cast<long long>(r) * pw.p.ld] = v[r] - h;
                            }
                        }
                    }
                }
            }
        }
        ptx::tc_fence_before();
        __syncwarp();
        if (lane == 0) release_acc(p, &acc_empty[buf]);
    }
    pw.flush();
}

// Persistent kernel: one CTA per SM walks the output tiles blockIdx.x, +gridDim.x, ...
// (PAIR: clusters of two CTAs walk 256-row pair tiles, the leader issuing the MMAs).
// Shared memory: [stage ring][epilogue staging kEpiWarps x 32 x 16 floats][barriers].
template <int KIND, int A_MN, int B_MN, bool PAIR, int EPI>
__global__ void __launch_bounds__(threads_for(EPI), 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
                const __grid_constant__ CUtensorMap tma_a_lo, const __grid_constant__ CUtensorMap tma_b_lo,
                const __grid_constant__ CUtensorMap tma_d, const __grid_constant__ CUtensorMap tma_p, const Params p,
                const int stages) {
    constexpr int kPlanes = KIND == 0 ? 1 : 2;
    const uint32_t stage_bytes = (kBM * 128 + static_cast<uint32_t>(p.bn_cta) * 128) * kPlanes;

    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    float* staging = reinterpret_cast<float*>(smem + stages * stage_bytes);
    uint64_t* full = reinterpret_cast<uint64_t*>(staging + EPI * p.stage_floats);
    uint64_t* empty = full + stages;
    uint64_t* acc_full = empty + stages;
    uint64_t* acc_empty = acc_full + 2;
    uint64_t* mma_done = acc_empty + 2;
    uint64_t* epi_sync = mma_done + 1;  // epilogue warps meet here after folding a tile's chains
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(epi_sync + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const bool leader = !PAIR || (blockIdx.x & 1u) == 0;
    // two accumulator buffers, plus a running-sum region when chains are folded (power of two)
    const uint32_t tmem_cols = (p.kc_blocks > 0 ? 4 : 2) * p.buf_cols;

    if (threadIdx.x == 0) {
        for (int s = 0; s < stages; ++s) {
            ptx::mbar_init(&full[s], 1);
            ptx::mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            ptx::mbar_init(&acc_full[b], 1);
            ptx::mbar_init(&acc_empty[b], (PAIR ? 2 : 1) * EPI);  // one arrival per epilogue warp (of the pair)
        }
        ptx::mbar_init(mma_done, 1);
        ptx::mbar_init(epi_sync, EPI);
        *abort_flag = 0;
        ptx::fence_barrier_init();
    }
    if (warp == 1) {
        if (PAIR) {
            ptx::tmem_alloc_pair(tmem_slot, tmem_cols);
            ptx::tmem_relinquish_pair();
        } else {
            ptx::tmem_alloc(tmem_slot, tmem_cols);
            ptx::tmem_relinquish();
        }
    }
    ptx::tc_fence_before();
    __syncthreads();
    if (PAIR) ptx::cluster_sync();  // the peer's barriers are initialised before any remote use
    ptx::tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (ptx::elect_one())
            produce<KIND, A_MN, B_MN, PAIR>(&tma_a, &tma_b, &tma_a_lo, &tma_b_lo, p, stages, smem, stage_bytes, full,
                                            empty, abort_flag);
    } else if (warp == 1) {
        if (ptx::elect_one()) {
            if (leader) {
                issue<KIND, A_MN, B_MN, PAIR>(p, stages, smem, stage_bytes, full, empty, acc_full, acc_empty, tmem,
                                              p.buf_cols, abort_flag);
                // every issued MMA has completed before TMEM is released (also after an abort)
                if (PAIR) {
                    ptx::mma_commit_pair(ptx::cluster_addr(mma_done, 0));
                    ptx::mma_commit_pair(ptx::cluster_addr(mma_done, 1));
                } else {
                    ptx::mma_commit(mma_done);
                }
            }
            volatile int no_abort = 0;
            wait_bar(mma_done, 0, p.health, &no_abort);
        }
    } else if (EPI != kEpiWarps) {  // the wide instances serve transposed plans without row loads
        drain_swap<false>(p, acc_full, acc_empty, epi_sync, tmem, abort_flag);
    } else if (p.swap) {
        if (p.residual || p.accumulate || p.aux)
            drain_swap<true>(p, acc_full, acc_empty, epi_sync, tmem, abort_flag);
        else
            drain_swap<false>(p, acc_full, acc_empty, epi_sync, tmem, abort_flag);
    } else if (p.tma_epi) {
        drain_tma(&tma_d, &tma_p, p, acc_full, acc_empty, epi_sync, tmem, staging, abort_flag);
    } else {
        drain(p, acc_full, acc_empty, epi_sync, tmem, staging, abort_flag);
    }
    ptx::tc_fence_before();
    __syncthreads();
    __syncwarp();
    if (PAIR) ptx::cluster_sync();  // neither CTA leaves while the peer may still address its memory
    if (warp == 1) {
        ptx::tc_fence_after();
        if (PAIR)
            ptx::tmem_dealloc_pair(tmem, tmem_cols);
        else
            ptx::tmem_dealloc(tmem, tmem_cols);
    }
}

}  // namespace gemm
}  // namespace rl2

// ===========================================================================
// host side: tensor maps, plans, dispatch
// ===========================================================================
namespace rl2 {
namespace gemm {
namespace {

typedef CUresult (*EncodeTiled)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encoder() {
    static EncodeTiled fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiled>(p);
    }
    return fn;
}

// 3D map {inner, outer, batch} with a 128-byte-swizzled box {box_inner, box_outer, 1}.
bool make_map(CUtensorMap* map, const void* base, int elem, long long inner, long long outer, long long batch,
              long long ld_elems, long long batch_stride_elems, int box_inner, int box_outer,
              CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
    EncodeTiled enc = encoder();
    if (!enc) {
        set_error("cuTensorMapEncodeTiled is unavailable from the driver");
        return false;
    }
    if (!aligned(base, 16)) {
        set_error("GEMM operand base address must be 16-byte aligned");
        return false;
    }
    const long long ld_bytes = ld_elems * elem;
    if (ld_bytes % 16 != 0 || ld_bytes <= 0) {
        set_error("GEMM operand row stride must be a positive multiple of 16 bytes (got %lld)", ld_bytes);
        return false;
    }
    long long bs_bytes = batch_stride_elems * elem;
    if (batch <= 1) {
        batch = 1;
        bs_bytes = ld_bytes * outer;
        bs_bytes = (bs_bytes + 15) / 16 * 16;
    }
    if (bs_bytes % 16 != 0 || bs_bytes <= 0) {
        set_error("GEMM operand batch stride must be a positive multiple of 16 bytes");
        return false;
    }
    const cuuint64_t dims[3] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(outer),
                                static_cast<cuuint64_t>(batch)};
    const cuuint64_t strides[2] = {static_cast<cuuint64_t>(ld_bytes), static_cast<cuuint64_t>(bs_bytes)};
    const cuuint32_t box[3] = {static_cast<cuuint32_t>(box_inner), static_cast<cuuint32_t>(box_outer), 1};
    const cuuint32_t estr[3] = {1, 1, 1};
    const CUresult r = enc(map, elem == 2 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3,
                           const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                           swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_error("cuTensorMapEncodeTiled failed (%d) for extents %lld x %lld x %lld", static_cast<int>(r), inner,
                  outer, batch);
        return false;
    }
    return true;
}

// RL2_GEMM_SWAP=0 keeps the caller's orientation (no transposed accumulator) for every product.
bool swap_enabled() {
    static const bool on = [] {
        const char* e = std::getenv("RL2_GEMM_SWAP");
        return !(e && e[0] == '0');
    }();
    return on;
}

// RL2_GEMM_TMA_STORE=0 keeps the register-store epilogue for every product.
bool tma_store_enabled() {
    static const bool on = [] {
        const char* e = std::getenv("RL2_GEMM_TMA_STORE");
        return !(e && e[0] == '0');
    }();
    return on;
}

// The fp32 output and the fp16 plane (if any) satisfy the TMA store rules: 16-byte aligned
// bases, row and batch strides in multiples of 16 bytes, rows at least n wide.
bool outputs_tma_ok(const rl2_gemm_desc* g) {
    const bool batched = g->batch > 1;
    const bool d_ok = !g->d || (aligned(g->d, 16) && (g->ldd * 4) % 16 == 0 && g->ldd >= g->n &&
                                 (!batched || (g->d_batch_stride > 0 && (g->d_batch_stride * 4) % 16 == 0)));
    if (!plane_used(&g->out_plane)) return d_ok;
    const rl2_plane& q = g->out_plane;
    return d_ok && q.h16 && aligned(q.h16, 16) && (q.ld * 2) % 16 == 0 && q.ld >= g->n &&
           (!batched || (q.twin_stride > 0 && (q.twin_stride * 2) % 16 == 0));
}

struct Plan {
    CUtensorMap ta, tb, ta_lo, tb_lo, td, tp;
    Params p;
    int kind, a_mn, b_mn, stages, smem;
    dim3 grid;
};

typedef void (*KernelFn)(const CUtensorMap, const CUtensorMap, const CUtensorMap, const CUtensorMap, const CUtensorMap,
                         const CUtensorMap, const Params, const int);

template <int EPI>
KernelFn pick_for(int kind, int a_mn, int b_mn, bool pair) {
    const int key = kind * 4 + a_mn * 2 + b_mn;
    if (pair) {  // fp16 products only
        switch (key & 3) {
            case 0: return gemm_kernel<0, 0, 0, true, EPI>;
            case 1: return gemm_kernel<0, 0, 1, true, EPI>;
            case 2: return gemm_kernel<0, 1, 0, true, EPI>;
            default: return gemm_kernel<0, 1, 1, true, EPI>;
        }
    }
    switch (key) {
        case 0: return gemm_kernel<0, 0, 0, false, EPI>;
        case 1: return gemm_kernel<0, 0, 1, false, EPI>;
        case 2: return gemm_kernel<0, 1, 0, false, EPI>;
        case 3: return gemm_kernel<0, 1, 1, false, EPI>;
        case 4: return gemm_kernel<1, 0, 0, false, EPI>;
        case 5: return gemm_kernel<1, 0, 1, false, EPI>;
        case 6: return gemm_kernel<1, 1, 0, false, EPI>;
        default: return gemm_kernel<1, 1, 1, false, EPI>;
    }
}

KernelFn pick(const Plan* plan) {
    return plan->p.epi_warps == kEpiWarpsWide ? pick_for<kEpiWarpsWide>(plan->kind, plan->a_mn, plan->b_mn, plan->p.pair)
                                              : pick_for<kEpiWarps>(plan->kind, plan->a_mn, plan->b_mn, plan->p.pair);
}

// RL2_GEMM_EPI_WARPS=8 keeps every plan on eight epilogue warps (default: sixteen for
// transposed plans without row loads).
int swap_epi_warps() {
    static const int w = [] {
        const char* e = std::getenv("RL2_GEMM_EPI_WARPS");
        return e && std::atoi(e) == kEpiWarps ? kEpiWarps : kEpiWarpsWide;
    }();
    return w;
}

// RL2_GEMM_PAIR=0 keeps every product on single-CTA tiles; 2 puts every eligible fp16
// product on CTA pairs whatever its contraction length; unset or 1: long contractions.
int pair_mode() {
    static const int mode = [] {
        const char* e = std::getenv("RL2_GEMM_PAIR");
        return e && (e[0] == '0' || e[0] == '2') ? e[0] - '0' : 1;
    }();
    return mode;
}

// Launch of a plan's kernel: CTA-pair plans as clusters of two.
cudaError_t launch(KernelFn fn, const Plan* plan, const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& ta_lo,
                   const CUtensorMap& tb_lo, const Params& p, cudaStream_t stream) {
    const int threads = threads_for(p.epi_warps);
    if (!p.pair) {
        fn<<<plan->grid, threads, plan->smem, stream>>>(ta, tb, ta_lo, tb_lo, plan->td, plan->tp, p, plan->stages);
        return cudaSuccess;
    }
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.gridDim = plan->grid;
    cfg.blockDim = dim3(threads, 1, 1);
    cfg.dynamicSmemBytes = static_cast<size_t>(plan->smem);
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, fn, ta, tb, ta_lo, tb_lo, plan->td, plan->tp, p, plan->stages);
}

int auto_tile_n(int n, int kind, int b_mn) {
    const int chunk = kind == 0 ? 64 : 32;
    const int quantum = b_mn ? chunk : 16;
    if (n <= 256) return (n + quantum - 1) / quantum * quantum;
    return 256;
}

}  // namespace
}  // namespace gemm
}  // namespace rl2

using rl2::gemm::Plan;

// rebindable: the plan's output, bias and residual pointers are replaced at every launch
// (rl2::gemm::run_rebound), so no epilogue form may bake them into a tensor map.
static void* create_plan(const rl2_gemm_desc* g, bool rebindable) {
    using namespace rl2;
    using namespace rl2::gemm;
    clear_error();
    if (!g) {
        set_error("null GEMM descriptor");
        return nullptr;
    }
    if ((g->kind != 0 && g->kind != 1) || g->m < 1 || g->n < 1 || g->k < 1 || g->batch < 1) {
        set_error("GEMM requires kind 0/1 and positive m, n, k, batch");
        return nullptr;
    }
    if (!g->a || !g->b || (!g->d && !plane_used(&g->out_plane) && !g->stat_mean) ||
        (g->kind == 1 && (!g->a_lo || !g->b_lo))) {
        set_error("GEMM operands / output must be non-null (kind 1 also needs a_lo and b_lo)");
        return nullptr;
    }
    if ((!plane_valid(&g->out_plane) && !(plane_lo_only(&g->out_plane) && g->d)) ||
        (plane_used(&g->out_plane) && (g->k_splits > 1 || g->accumulate))) {
        set_error("GEMM output plane must be a valid fp16 or hi/lo plane (lo alone only beside an fp32 output), "
                  "without split-K or accumulate");
        return nullptr;
    }
    if ((g->a_major != 0 && g->a_major != 1) || (g->b_major != 0 && g->b_major != 1)) {
        set_error("GEMM majors must be 0 (K contiguous) or 1 (M/N contiguous)");
        return nullptr;
    }
    const int splits = g->k_splits < 1 ? 1 : g->k_splits;
    if (splits > 1 && (g->bias || g->residual || g->accumulate || g->stat_mean || g->activation ||
                       g->d_split_stride <= 0)) {
        set_error("split-K GEMMs write plain partials: no bias/residual/accumulate/stats/activation, positive split stride");
        return nullptr;
    }
    if (g->bn_mean && (!g->bn_invstd || !g->bn_gamma || !g->bn_beta || g->stat_mean || g->activation ||
                       g->accumulate || g->k_splits > 1)) {
        set_error("GEMM batch-norm epilogue needs mean, invstd, gamma and beta, and no statistics, "
                  "activation, accumulate or split-K");
        return nullptr;
    }
    if (!g->stat_mean && g->stat_m2) {
        set_error("GEMM column statistics: stat_m2 needs stat_mean");
        return nullptr;
    }
    const int elem = g->kind == 0 ? 2 : 4;
    const int bk = 128 / elem;
    const int chunk = 128 / elem;
    // Products with at least 128 output columns (and a plan-chosen tile width) run with the
    // operands swapped: the accumulator tile is D^T (TMEM lane = output column), so a
    // thread holds 32 rows of its column, the 32-row moments stay in registers and every
    // global access of the epilogue covers whole 128-byte row segments (drain_swap).
    // Kernel view of a swapped plan: M' = n, N' = m, A' = B, B' = A. RL2_GEMM_SWAP=0 keeps
    // the caller's orientation for every product.
    // D += result with nothing else reading the final values (no plane, no statistics, no
    // activation) is faster as TMA reduce-add stores in the caller's orientation.
    const bool in_place = g->d && (g->accumulate || (g->residual == g->d && g->ldr == g->ldd &&
                                                      g->residual_batch_stride == g->d_batch_stride)) &&
                          !(g->accumulate && g->residual);
    const bool reduce_ok = in_place && !plane_used(&g->out_plane) && !g->stat_mean;
    const bool reduce_path = !rebindable && tma_store_enabled() && splits == 1 && reduce_ok && !g->activation && !g->act_aux &&
                             !g->bn_mean && outputs_tma_ok(g);
    const bool swap = swap_enabled() && g->tile_n <= 0 && g->n >= 128 && !reduce_path;
    if (g->bn_mean && !swap) {
        set_error("GEMM batch-norm epilogue needs a transposed plan (n >= 128, plan-chosen tile width)");
        return nullptr;
    }
    rl2_gemm_desc sw = *g;
    if (swap) {
        sw.m = g->n;
        sw.n = g->m;
        sw.a = g->b;
        sw.a_lo = g->b_lo;
        sw.a_major = g->b_major;
        sw.lda = g->ldb;
        sw.a_batch_stride = g->b_batch_stride;
        sw.b = g->a;
        sw.b_lo = g->a_lo;
        sw.b_major = g->a_major;
        sw.ldb = g->lda;
        sw.b_batch_stride = g->a_batch_stride;
    }
    const rl2_gemm_desc& o = sw;  // operands and tiles (the caller's view unless swapped)
    int bn = o.tile_n > 0 ? o.tile_n : auto_tile_n(o.n, o.kind, o.b_major);
    if (swap) {  // whole 32-row groups per tile (and whole 128-byte chunks of an M-contiguous A)
        const int q = o.b_major ? chunk : 32;
        bn = std::min(256, (bn + q - 1) / q * q);
    }
    // 3xTF32 products longer than one chain accumulate in chains of kChainBlocks k-blocks
    // folded by the epilogue (fold_chunks); the running sum takes a third TMEM region, so
    // such plans use tiles of at most 128 columns (four 128-column regions fill TMEM).
    const int kblocks_tile = ((g->k + bk - 1) / bk + std::max(splits, 1) - 1) / std::max(splits, 1);
    const bool chained = g->kind == 1 && kblocks_tile > kChainBlocks;
    // fp16 products with at least 256 kernel rows run on CTA pairs: 256 x BN tiles whose
    // operands each SM stages half of (A: its 128 rows, B: BN / 2 rows), so a pair reads
    // (256 + BN) K operand rows from L2 where two single-CTA tiles read 2 (128 + BN).
    // Pairs pay where the main loop dominates (long K) over at least two pair rows; a pair's
    // MMAs also wait for the slower of its two epilogues, which costs more than the saved
    // operand traffic on short-K products with wide fp32 outputs (measured: K = 512 slower,
    // K >= 2048 faster, 256 kernel rows slower).
    bool pair = pair_mode() > 0 && !rebindable && g->kind == 0 && g->tile_n <= 0 &&
                (pair_mode() == 2 ? o.m >= 2 * kBM : o.m >= 4 * kBM && kblocks_tile >= kPairMinKBlocks);
    // Fewer tiles than SMs: narrower tiles (down to 128) until the grid covers the SMs (a
    // pair tile occupies two); with at most one tile per CTA a CTA's tile is all of its
    // serial work. (64-wide tiles re-read the A tile from shared memory per 64 columns:
    // slower on long-K products.)
    int nsm = 0;
    if (g->tile_n <= 0) {
        int dev = 0;
        if (cudaGetDevice(&dev) != cudaSuccess ||
            cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
            nsm = 0;
    }
    auto narrowed = [&](int w, bool in_pairs) {
        if (nsm <= 0) return w;
        const int q = o.b_major ? chunk : (swap ? 32 : 16);
        const int rows = in_pairs ? 2 * kBM : kBM;
        const int units = in_pairs ? nsm / 2 : nsm;
        auto tiles_for = [&](int x) {
            return static_cast<long long>((o.n + x - 1) / x) * ((o.m + rows - 1) / rows) * o.batch * splits;
        };
        while (w / 2 >= 128 && (w / 2) % q == 0 && tiles_for(w) < units) w /= 2;
        return w;
    };
    if (pair) {
        // a pair stages BN / 2 rows of B per CTA: whole 16-row groups (whole 128-byte chunks
        // of an N-contiguous B)
        const int w = narrowed(bn, true);
        if (w % 32 == 0 && (o.b_major == 0 || (w / 2) % chunk == 0))
            bn = w;
        else
            pair = false;
    }
    if (!pair) bn = narrowed(bn, false);
    if (chained) bn = std::min(bn, 128);
    if (bn % 16 != 0 || bn < 16 || bn > 256 || (o.b_major == 1 && bn % chunk != 0)) {
        set_error("GEMM tile_n must be a multiple of 16 in [16, 256] (and of %d for an N-contiguous B)", chunk);
        return nullptr;
    }
    Plan* plan = new (std::nothrow) Plan();
    if (!plan) {
        set_error("out of host memory");
        return nullptr;
    }
    std::memset(plan, 0, sizeof(Plan));
    plan->kind = g->kind;
    plan->a_mn = o.a_major;
    plan->b_mn = o.b_major;
    const long long a_batch = o.a_batch_stride ? o.batch : 1;
    const long long b_batch = o.b_batch_stride ? o.batch : 1;
    bool ok = true;
    for (int plane = 0; plane < (g->kind == 0 ? 1 : 2) && ok; ++plane) {
        const void* a = plane == 0 ? o.a : o.a_lo;
        const void* b = plane == 0 ? o.b : o.b_lo;
        CUtensorMap* ma = plane == 0 ? &plan->ta : &plan->ta_lo;
        CUtensorMap* mb = plane == 0 ? &plan->tb : &plan->tb_lo;
        // MN-major tf32 tiles use the 32-byte-granule 128-byte swizzle (see smem_desc).
        const CUtensorMapSwizzle mn_swz = g->kind == 0 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B;
        if (o.a_major == 0)
            ok = ok && make_map(ma, a, elem, o.k, o.m, a_batch, o.lda, o.a_batch_stride, bk, kBM);
        else
            ok = ok && make_map(ma, a, elem, o.m, o.k, a_batch, o.lda, o.a_batch_stride, chunk, bk, mn_swz);
        if (o.b_major == 0)
            ok = ok && make_map(mb, b, elem, o.k, o.n, b_batch, o.ldb, o.b_batch_stride, bk, pair ? bn / 2 : bn);
        else
            ok = ok && make_map(mb, b, elem, o.n, o.k, b_batch, o.ldb, o.b_batch_stride, chunk, bk, mn_swz);
    }
    if (!ok) {
        delete plan;
        return nullptr;
    }
    if (g->kind == 0) {
        plan->ta_lo = plan->ta;
        plan->tb_lo = plan->tb;
    }
    Params& p = plan->p;
    p.M = o.m;
    p.N = o.n;
    p.K = o.k;
    p.swap = swap;
    p.out_m = g->m;
    p.out_n = g->n;
    p.bn_mean = g->bn_mean;
    p.bn_invstd = g->bn_invstd;
    p.bn_gamma = g->bn_gamma;
    p.bn_beta = g->bn_beta;
    p.bn_tstride = g->bn_twin_stride;
    p.bn_relu = g->bn_relu;
    p.batch = g->batch;
    p.kblocks_total = (g->k + bk - 1) / bk;
    p.splits = std::min(splits, p.kblocks_total);
    p.kblocks_per_split = (p.kblocks_total + p.splits - 1) / p.splits;
    p.splits = (p.kblocks_total + p.kblocks_per_split - 1) / p.kblocks_per_split;  // every split non-empty
    p.BN = bn;
    // sixteen epilogue warps (four per TMEM lane quarter) for transposed plans that read no
    // rows besides the accumulator: twice the warps to hide the epilogue's dependent
    // latency (its register work per 32-row group) within the 113 registers a thread gets
    // (rebindable plans may gain a residual or an accumulate at launch: eight warps)
    p.epi_warps = swap && !rebindable && !g->residual && !g->accumulate && !g->act_aux ? swap_epi_warps() : kEpiWarps;
    p.pair = pair;
    p.bn_cta = pair ? bn / 2 : bn;
    p.kc_blocks = chained ? kChainBlocks : 0;
    p.a_batched = o.a_batch_stride != 0;
    p.b_batched = o.b_batch_stride != 0;
    p.d = g->d;
    p.ldd = g->ldd;
    p.d_bstride = g->d_batch_stride;
    p.d_split_stride = g->d_split_stride;
    p.accumulate = g->accumulate;
    p.bias = g->bias;
    p.bias_bstride = g->bias_batch_stride;
    p.residual = g->residual;
    p.ldr = g->ldr;
    p.r_bstride = g->residual_batch_stride;
    p.stat_mean = g->stat_mean;
    p.stat_m2 = g->stat_m2;
    p.stat_bstride = g->stat_batch_stride;
    p.scale = g->scale;
    p.health = g->health;
    p.out_plane = to_plane(&g->out_plane);
    const long long tiles_n = (o.n + bn - 1) / bn;
    const long long tiles_m = (o.m + (pair ? 2 * kBM : kBM) - 1) / (pair ? 2 * kBM : kBM);  // pair tiles in a pair plan
    const long long tiles = tiles_n * tiles_m * g->batch * p.splits;
    if (tiles > 0x7FFFFFFFLL) {
        set_error("GEMM has too many output tiles");
        delete plan;
        return nullptr;
    }
    p.tiles_n = static_cast<int>(tiles_n);
    p.tiles_m = static_cast<int>(tiles_m);
    p.tiles_total = static_cast<int>(tiles);
    p.buf_cols = bn <= 32 ? 32 : bn <= 64 ? 64 : bn <= 128 ? 128 : 256;
    auto a16 = [](const void* q) { return aligned(q, 16); };
    p.vec_d = g->d && a16(g->d) && g->ldd % 4 == 0 && g->d_batch_stride % 4 == 0 && g->d_split_stride % 4 == 0;
    p.vec_res = g->residual && a16(g->residual) && g->ldr % 4 == 0 && g->residual_batch_stride % 4 == 0;
    p.vec_bias = g->bias && a16(g->bias) && g->bias_batch_stride % 4 == 0;
    p.vec_stat = g->stat_mean && a16(g->stat_mean) && (!g->stat_m2 || a16(g->stat_m2)) && g->n % 4 == 0 &&
                 g->stat_batch_stride % 4 == 0;
    if (g->activation < 0 || g->activation > 2 || (g->act_aux && !g->activation)) {
        set_error("GEMM activation must be 0 (none), 1 (ELU) or 2 (tanh); act_aux needs an activation");
        delete plan;
        return nullptr;
    }
    p.activation = g->activation;
    p.aux = g->act_aux;
    p.ld_aux = g->ld_aux;
    p.aux_bstride = g->aux_batch_stride;
    p.vec_aux = g->act_aux && a16(g->act_aux) && g->ld_aux % 4 == 0 && g->aux_batch_stride % 4 == 0;
    p.vec_plane = plane_used(&g->out_plane) && g->out_plane.ld % 4 == 0 && g->out_plane.twin_stride % 4 == 0 &&
                  (g->out_plane.h16 ? aligned(g->out_plane.h16, 8)
                                    : a16(g->out_plane.hi) && a16(g->out_plane.lo));
    // store-engine epilogue (plans that keep the caller's orientation): outputs written by
    // TMA stores of 32-row x 16-column boxes (fp32: 64-byte swizzle; fp16: 32-byte swizzle)
    // when the product has no activation / split-K and the outputs satisfy the TMA rules.
    // D += result (accumulate, or a residual that is D itself) goes through TMA reduce-add
    // stores when nothing else needs the final values (reduce_ok).
    if (!rebindable && !swap && tma_store_enabled() && p.splits == 1 && (!(g->residual || g->accumulate) || reduce_ok) &&
        !g->activation && !g->act_aux && outputs_tma_ok(g)) {
        const bool plane_on = plane_used(&g->out_plane);
        bool mok = true;
        if (g->d)
            mok = make_map(&plan->td, g->d, 4, g->n, g->m, g->batch, g->ldd, g->d_batch_stride, 16, 32,
                           CU_TENSOR_MAP_SWIZZLE_64B);
        if (mok && plane_on)
            mok = make_map(&plan->tp, g->out_plane.h16, 2, g->n, g->m, g->batch, g->out_plane.ld,
                           g->out_plane.twin_stride, 16, 32, CU_TENSOR_MAP_SWIZZLE_32B);
        if (mok) {
            p.tma_epi = true;
            p.tma_d = g->d != nullptr;
            p.tma_plane = plane_on;
            p.tma_reduce = reduce_ok;
        } else {
            clear_error();  // fall back to the register-store epilogue
        }
    }
    // shared memory: ring + epilogue staging + barriers (2 x stages + 5 words, TMEM slot,
    // abort word) + alignment slack. The store-engine epilogue double-buffers its boxes
    // unless that costs the operand ring its fourth stage (RL2_GEMM_EPI_BUFS=1 or 2 forces).
    {
        const int planes = g->kind == 0 ? 1 : 2;
        const int stage_bytes = (kBM * 128 + p.bn_cta * 128) * planes;
        auto stages_for = [&](int stage_floats) {
            return std::min(8, (kMaxSmem - (1024 + p.epi_warps * stage_floats * 4 + 256)) / stage_bytes);
        };
        auto tma_floats = [&](int nbuf) { return nbuf * (512 + (p.tma_plane ? 256 : 0)); };
        p.epi_bufs = 1;
        p.stage_floats = swap ? 0 : 512;  // the transposed epilogue stages nothing
        if (p.tma_epi) {
            static const int forced = [] {
                const char* e = std::getenv("RL2_GEMM_EPI_BUFS");
                return e ? std::atoi(e) : 0;
            }();
            const int s1 = stages_for(tma_floats(1)), s2 = stages_for(tma_floats(2));
            p.epi_bufs = forced == 1 || forced == 2 ? forced : (s2 >= std::min(s1, 4) ? 2 : 1);
            p.stage_floats = tma_floats(p.epi_bufs);
        }
        plan->stages = stages_for(p.stage_floats);
        if (plan->stages < 2) {
            set_error("GEMM tile does not fit shared memory");
            delete plan;
            return nullptr;
        }
        plan->smem = plan->stages * stage_bytes + 1024 + p.epi_warps * p.stage_floats * 4 + 256;
    }
    int device = 0, sms = 0;
    if (cudaGetDevice(&device) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || sms < 1) {
        set_error("cannot query the SM count of the current device");
        delete plan;
        return nullptr;
    }
    // The limit is an attribute of the kernel function shared by every plan that uses
    // it, so it is always raised to the device maximum (never lowered by a small plan).
    KernelFn fn = pick(plan);
    if (cudaFuncSetAttribute(reinterpret_cast<const void*>(fn), cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kMaxSmem) != cudaSuccess) {
        set_error("cudaFuncSetAttribute(max dynamic smem %d) failed", kMaxSmem);
        delete plan;
        return nullptr;
    }
    if (!p.pair) {
        plan->grid = dim3(static_cast<unsigned>(std::min<long long>(tiles, sms)), 1, 1);
        return plan;
    }
    // one cluster of two CTAs per pair of SMs that can hold one at once
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3(static_cast<unsigned>(2 * std::max(1, sms / 2)), 1, 1);
    cfg.blockDim = dim3(threads_for(p.epi_warps), 1, 1);
    cfg.dynamicSmemBytes = static_cast<size_t>(plan->smem);
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, reinterpret_cast<const void*>(fn), &cfg) != cudaSuccess ||
        clusters < 1) {
        set_error("no cluster of two GEMM CTAs fits the device");
        delete plan;
        return nullptr;
    }
    plan->grid = dim3(static_cast<unsigned>(2 * std::min<long long>(tiles, clusters)), 1, 1);
    return plan;
}

extern "C" void* rl2_gemm_create(const rl2_gemm_desc* g) { return create_plan(g, false); }

namespace rl2 {
namespace gemm {

void* create_rebindable(const rl2_gemm_desc* g) { return create_plan(g, true); }

namespace {

typedef CUresult (*ReplaceAddress)(CUtensorMap*, void*);

ReplaceAddress replacer() {
    static ReplaceAddress fn = [] {
        void* q = nullptr;
        cudaDriverEntryPointQueryResult r;
        return cudaGetDriverEntryPoint("cuTensorMapReplaceAddress", &q, cudaEnableDefault, &r) == cudaSuccess &&
                       r == cudaDriverEntryPointSuccess
                   ? reinterpret_cast<ReplaceAddress>(q)
                   : nullptr;
    }();
    return fn;
}

int launch_rebound(const Plan* plan, const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& ta_lo,
                   const CUtensorMap& tb_lo, float* d, const float* bias, const float* residual, int accumulate,
                   cudaStream_t stream) {
    Params p = plan->p;
    p.d = d;
    p.bias = bias;
    p.residual = residual;
    p.accumulate = accumulate;
    p.vec_d = aligned(d, 16) && p.ldd % 4 == 0 && p.d_bstride % 4 == 0 && p.d_split_stride % 4 == 0;
    p.vec_res = residual && aligned(residual, 16) && p.ldr % 4 == 0 && p.r_bstride % 4 == 0;
    p.vec_bias = bias && aligned(bias, 16) && p.bias_bstride % 4 == 0;
    KernelFn fn = pick(plan);
    const cudaError_t e = launch(fn, plan, ta, tb, ta_lo, tb_lo, p, stream);
    if (e != cudaSuccess) {
        set_error("tcgen05 GEMM (rebound) launch: %s", cudaGetErrorString(e));
        return -1;
    }
    return launch_status("tcgen05 GEMM (rebound)");
}

}  // namespace

int run_rebound(void* opaque, float* d, const float* bias, const float* residual, int accumulate,
                cudaStream_t stream) {
    clear_error();
    const Plan* plan = static_cast<const Plan*>(opaque);
    if (!plan || plan->p.tma_epi || !d) {
        set_error("rebound GEMM launch needs a rebindable plan and an output");
        return -1;
    }
    return launch_rebound(plan, plan->ta, plan->tb, plan->ta_lo, plan->tb_lo, d, bias, residual, accumulate, stream);
}

// The same with the operands rebound too (fp16 plans): a and b in the descriptor's view, their
// layouts (majors, leading dimensions, extents) those the plan was created with; the plan's
// tensor maps are copied and given the new base addresses (cuTensorMapReplaceAddress).
int run_rebound_ab(void* opaque, const void* a, const void* b, float* d, const float* bias, const float* residual,
                   int accumulate, cudaStream_t stream) {
    clear_error();
    const Plan* plan = static_cast<const Plan*>(opaque);
    if (!plan || plan->p.tma_epi || !d || plan->kind != 0) {
        set_error("operand-rebound GEMM launch needs a rebindable fp16 plan and an output");
        return -1;
    }
    const ReplaceAddress rep = replacer();
    if (!rep) {
        set_error("cuTensorMapReplaceAddress is unavailable from the driver");
        return -1;
    }
    if (!a || !b || !aligned(a, 16) || !aligned(b, 16)) {
        set_error("GEMM operand base addresses must be 16-byte aligned");
        return -1;
    }
    CUtensorMap ta = plan->ta, tb = plan->tb;
    const void* ka = plan->p.swap ? b : a;  // kernel view of a swapped plan: A' = B, B' = A
    const void* kb = plan->p.swap ? a : b;
    if (rep(&ta, const_cast<void*>(ka)) != CUDA_SUCCESS || rep(&tb, const_cast<void*>(kb)) != CUDA_SUCCESS) {
        set_error("cuTensorMapReplaceAddress failed");
        return -1;
    }
    return launch_rebound(plan, ta, tb, ta, tb, d, bias, residual, accumulate, stream);
}

}  // namespace gemm
}  // namespace rl2

extern "C" int rl2_gemm_run(void* opaque, void* stream) {
    using namespace rl2;
    using namespace rl2::gemm;
    clear_error();
    if (!opaque) {
        set_error("null GEMM plan");
        return -1;
    }
    Plan* plan = static_cast<Plan*>(opaque);
    KernelFn fn = pick(plan);
    const cudaError_t e = launch(fn, plan, plan->ta, plan->tb, plan->ta_lo, plan->tb_lo, plan->p, as_stream(stream));
    if (e != cudaSuccess) {
        set_error("tcgen05 GEMM launch: %s", cudaGetErrorString(e));
        return -1;
    }
    return launch_status("tcgen05 GEMM");
}

extern "C" int rl2_gemm_destroy(void* opaque) {
    rl2::clear_error();
    delete static_cast<Plan*>(opaque);
    return 0;
}

extern "C" int rl2_gemm_tile_n(void* opaque) {
    return opaque ? static_cast<Plan*>(opaque)->p.BN : -1;
}

extern "C" int rl2_gemm_cta_pair(void* opaque) { return opaque && static_cast<Plan*>(opaque)->p.pair ? 1 : 0; }

extern "C" int rl2_gemm_uses_tma_store(void* opaque) {
    if (!opaque) return 0;
    const rl2::gemm::Params& p = static_cast<Plan*>(opaque)->p;
    return p.swap ? 2 : p.tma_epi ? 1 : 0;
}

// ---------------------------------------------------------------------------
// split-K reduction (fixed summation order -> run-to-run bitwise determinism)
// ---------------------------------------------------------------------------
namespace rl2 {
namespace gemm {
__global__ void split_reduce_kernel(const float* __restrict__ part, long long stride, int splits,
                                    float* __restrict__ out, long long count, int accumulate, int allow_vec,
                                    long long in_bstride, long long out_bstride) {
    part += blockIdx.y * in_bstride;  // grid.y: independent reductions of the same shape
    out += blockIdx.y * out_bstride;
    const long long n4 = count / 4;
    const bool vec = allow_vec && (stride % 4 == 0) && ptx::aligned16(part) && ptx::aligned16(out);
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < (vec ? n4 : count);
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        if (vec) {
            float4 acc = accumulate ? reinterpret_cast<const float4*>(out)[i] : make_float4(0.f, 0.f, 0.f, 0.f);
            // unrolled so that eight partial rows are in flight; the sum keeps split order
#pragma unroll 8
            for (int s = 0; s < splits; ++s) {
                const float4 v = reinterpret_cast<const float4*>(part + s * stride)[i];
                acc.x += v.x;
                acc.y += v.y;
                acc.z += v.z;
                acc.w += v.w;
            }
            reinterpret_cast<float4*>(out)[i] = acc;
        } else {
            float acc = accumulate ? out[i] : 0.0f;
#pragma unroll 8
            for (int s = 0; s < splits; ++s) acc += part[s * stride + i];
            out[i] = acc;
        }
    }
    if (vec && blockIdx.x == 0) {
        for (long long i = n4 * 4 + threadIdx.x; i < count; i += blockDim.x) {
            float acc = accumulate ? out[i] : 0.0f;
#pragma unroll 8
            for (int s = 0; s < splits; ++s) acc += part[s * stride + i];
            out[i] = acc;
        }
    }
}
}  // namespace gemm
}  // namespace rl2

extern "C" int rl2_split_reduce_batched(const float* partial, long long split_stride, int splits, float* out,
                                        long long count, int accumulate, int batch, long long in_batch_stride,
                                        long long out_batch_stride, void* stream) {
    using namespace rl2;
    clear_error();
    if (!partial || !out || splits < 1 || count < 1 || split_stride < count || batch < 1 || batch > 65535) {
        set_error("split reduce needs non-null buffers, splits >= 1, split_stride >= count and 1..65535 batches");
        return -1;
    }
    // small outputs: one thread per element (more loads in flight than float4 threads);
    // large outputs: float4 per thread
    const int vec = count > (1LL << 22) ? 1 : 0;
    const long long work = vec ? count / 4 + 1 : count;
    const int blocks = static_cast<int>(std::min<long long>((work + 255) / 256, 148LL * 16));
    gemm::split_reduce_kernel<<<dim3(blocks, batch), 256, 0, as_stream(stream)>>>(
        partial, split_stride, splits, out, count, accumulate, vec, in_batch_stride, out_batch_stride);
    return launch_status("split-K reduce");
}

extern "C" int rl2_split_reduce(const float* partial, long long split_stride, int splits, float* out,
                                long long count, int accumulate, void* stream) {
    return rl2_split_reduce_batched(partial, split_stride, splits, out, count, accumulate, 1, 0, 0, stream);
}
