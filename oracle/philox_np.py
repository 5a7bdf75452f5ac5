"""Philox4x32-10 counter-based generator in numpy (test infrastructure only).

Published algorithm: Salmon, Moraes, Dror, Shaw, "Parallel random numbers: as easy as
1, 2, 3" (SC'11): per round (hi0, lo0) = mulhilo(0xD2511F53, c0), (hi1, lo1) =
mulhilo(0xCD9E8D57, c2), c = (hi1 ^ c1 ^ k0, lo1, hi0 ^ c3 ^ k1, lo0), then the key
is bumped by (0x9E3779B9, 0xBB67AE85); ten rounds. Also restates the device replay
sampler's use of it (the reference's Warp stream itself is not reproduced): Warp's
unbiased bounded rule threshold = (-n) % n, reject v < threshold, index = v % n
(``src/robolearn/warp/_flash_replay.py:116-128``).
"""

from __future__ import annotations

M0, M1, W0, W1 = 0xD2511F53, 0xCD9E8D57, 0x9E3779B9, 0xBB67AE85
MASK = 0xFFFFFFFF


def philox4x32(c, k0, k1, rounds=10):
    c0, c1, c2, c3 = (int(x) & MASK for x in c)
    k0, k1 = int(k0) & MASK, int(k1) & MASK
    for _ in range(rounds):
        p0, p1 = M0 * c0, M1 * c2
        hi0, lo0, hi1, lo1 = p0 >> 32, p0 & MASK, p1 >> 32, p1 & MASK
        c0, c1, c2, c3 = (hi1 ^ c1 ^ k0) & MASK, lo1, (hi0 ^ c3 ^ k1) & MASK, lo0
        k0, k1 = (k0 + W0) & MASK, (k1 + W1) & MASK
    return c0, c1, c2, c3


def replay_indices(seed: int, epoch: int, n: int, batch: int) -> list[int]:
    """Indices the device sampler draws: counter = (row, epoch lo, epoch hi ^ round, 0x5A11)."""
    k0, k1 = seed & MASK, (seed >> 32) & MASK
    threshold = ((1 << 32) - n) % n
    out = []
    for i in range(batch):
        value = None
        for rnd in range(64):
            words = philox4x32((i, epoch & MASK, ((epoch >> 32) ^ rnd) & MASK, 0x5A11), k0, k1)
            for w in words:
                if w >= threshold:
                    value = w % n
                    break
            if value is not None:
                break
        out.append(value)
    return out
