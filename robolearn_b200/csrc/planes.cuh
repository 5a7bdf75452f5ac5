// Operand planes: the derived copies of activations / gradients / weights that
// feed the tensor-core products. Kind 0 is one fp16 plane (optionally multiplied
// by a device loss scale, overflow recorded in *found_inf); kind 1 is a pair of
// fp32 planes hi + lo with hi exactly representable in tf32 (the 3xTF32 split).
// Rows have their own stride (16-byte aligned for TMA) and an optional twin stride.
#pragma once

#include "common.cuh"
#include "../../include/rl2.h"

namespace rl2 {

struct Plane {
    __half* h16;
    float* hi;
    float* lo;
    long long ld, tstride;
    const float* scale;
    int* found_inf;
};

inline Plane to_plane(const rl2_plane* p) {
    Plane q{};
    if (!p) return q;
    q.h16 = reinterpret_cast<__half*>(p->h16);
    q.hi = p->hi;
    q.lo = p->lo;
    q.ld = p->ld;
    q.tstride = p->twin_stride;
    q.scale = p->scale;
    q.found_inf = p->found_inf;
    return q;
}

inline bool plane_valid(const rl2_plane* p) {
    if (!p) return true;
    if (p->h16 && (p->hi || p->lo)) return false;
    if ((p->hi == nullptr) != (p->lo == nullptr)) return false;
    return true;
}

inline bool plane_used(const rl2_plane* p) { return p && (p->h16 || p->hi || p->lo); }

// A tf32 plane given as lo alone: the caller reads the operand's hi part from fp32 values
// stored elsewhere in the same layout (the tensor cores ignore the low 13 mantissa bits of
// a kind::tf32 operand, so raw fp32 serves as hi). Only GEMM outputs that also write the
// fp32 result accept it.
inline bool plane_lo_only(const rl2_plane* p) { return p && !p->h16 && !p->hi && p->lo; }

#if defined(__CUDACC__)
__device__ __forceinline__ float tf32_hi(float v) { return __uint_as_float(__float_as_uint(v) & 0xFFFFE000u); }

// Per-thread cache of the plane's scale (read once).
struct PlaneWriter {
    Plane p;
    float scale;
    bool overflow;
    __device__ __forceinline__ explicit PlaneWriter(const Plane& q) : p(q), scale(1.0f), overflow(false) {
        if (p.h16 && p.scale) scale = *p.scale;
    }
    __device__ __forceinline__ bool active() const { return p.h16 != nullptr || p.lo != nullptr; }
    __device__ __forceinline__ void store(int t, long long row, int col, float v) {
        const long long o = static_cast<long long>(t) * p.tstride + row * p.ld + col;
        if (p.h16) {
            const float s = v * scale;
            overflow |= !(fabsf(s) <= 65504.0f);
            p.h16[o] = __float2half_rn(s);
        } else if (p.lo) {
            const float h = tf32_hi(v);
            if (p.hi) p.hi[o] = h;
            p.lo[o] = v - h;
        }
    }
    // four consecutive columns (col % 4 == 0, row and twin strides % 4 == 0; base 8-byte
    // aligned for fp16, 16-byte aligned for hi/lo)
    __device__ __forceinline__ void store4(int t, long long row, int col, float4 v) {
        const long long o = static_cast<long long>(t) * p.tstride + row * p.ld + col;
        if (p.h16) {
            const float4 s = make_float4(v.x * scale, v.y * scale, v.z * scale, v.w * scale);
            overflow |= !(fabsf(s.x) <= 65504.0f && fabsf(s.y) <= 65504.0f && fabsf(s.z) <= 65504.0f &&
                          fabsf(s.w) <= 65504.0f);
            const __half2 lo2 = __floats2half2_rn(s.x, s.y);
            const __half2 hi2 = __floats2half2_rn(s.z, s.w);
            uint2 packed;
            packed.x = *reinterpret_cast<const uint32_t*>(&lo2);
            packed.y = *reinterpret_cast<const uint32_t*>(&hi2);
            *reinterpret_cast<uint2*>(p.h16 + o) = packed;
        } else if (p.lo) {
            const float4 h = make_float4(tf32_hi(v.x), tf32_hi(v.y), tf32_hi(v.z), tf32_hi(v.w));
            if (p.hi) *reinterpret_cast<float4*>(p.hi + o) = h;
            *reinterpret_cast<float4*>(p.lo + o) = make_float4(v.x - h.x, v.y - h.y, v.z - h.z, v.w - h.w);
        }
    }
    __device__ __forceinline__ void flush() {
        if (p.found_inf && overflow) atomicOr(p.found_inf, 1);
    }
};
#endif

}  // namespace rl2
