// Philox4x32-10 counter-based generator (Salmon et al., SC'11), shared by the replay
// sampler, the policy noise and the PPO minibatch permutation.
#pragma once

#include <cstdint>

namespace rl2 {

struct U4 {
    uint32_t x, y, z, w;
};

__host__ __device__ __forceinline__ void mulhilo(uint32_t a, uint32_t b, uint32_t& hi, uint32_t& lo) {
    const uint64_t p = static_cast<uint64_t>(a) * static_cast<uint64_t>(b);
    hi = static_cast<uint32_t>(p >> 32);
    lo = static_cast<uint32_t>(p);
}

// Philox4x32 with 10 rounds: multipliers 0xD2511F53 / 0xCD9E8D57, Weyl key
// increments 0x9E3779B9 / 0xBB67AE85 (constants from the published algorithm).
__host__ __device__ __forceinline__ U4 philox(U4 c, uint32_t k0, uint32_t k1) {
#pragma unroll
    for (int r = 0; r < 10; ++r) {
        uint32_t hi0, lo0, hi1, lo1;
        mulhilo(0xD2511F53u, c.x, hi0, lo0);
        mulhilo(0xCD9E8D57u, c.z, hi1, lo1);
        c = U4{hi1 ^ c.y ^ k0, lo1, hi0 ^ c.w ^ k1, lo0};
        k0 += 0x9E3779B9u;
        k1 += 0xBB67AE85u;
    }
    return c;
}

}  // namespace rl2
