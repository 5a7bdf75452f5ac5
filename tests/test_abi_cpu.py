"""CPU-side checks of the native boundary: the library loads, every entry point that
``include/rl2.h`` declares is exported and has a ctypes declaration, and the host
Philox block matches the published algorithm (no GPU needed)."""

import ctypes
import re
from pathlib import Path

from oracle import philox_np

ROOT = Path(__file__).resolve().parents[1]


def _declared() -> set[str]:
    text = (ROOT / "include" / "rl2.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return set(re.findall(r"\b(rl2_[a-z0-9_]+)\s*\(", text))


def test_library_exports_every_declared_symbol():
    from robolearn_b200 import _native as N

    lib = N.load()
    declared = _declared()
    assert len(declared) > 30
    for name in sorted(declared):
        assert hasattr(lib, name), name
        assert name in N.SIGNATURES, f"{name} lacks a ctypes declaration"
    assert lib.rl2_abi_version() == 1


def test_host_philox_block_matches_published_algorithm():
    from robolearn_b200 import _native as N

    lib = N.load()
    out = (ctypes.c_uint * 4)()
    lib.rl2_philox4x32(0, 0, 0, 0, 0, 0, out)
    assert [hex(x) for x in out] == ["0x6627e8d5", "0xe169c58d", "0xbc57ac4c", "0x9b00dbd8"]
    for c, k in (((1, 2, 3, 4), (5, 6)), ((0xFFFFFFFF,) * 4, (0xFFFFFFFF, 0xFFFFFFFF)), ((7, 0, 9, 0x5A11), (11, 0))):
        lib.rl2_philox4x32(*c, *k, out)
        assert tuple(out) == philox_np.philox4x32(c, *k)


def test_unbiased_bounded_rule_stays_in_range():
    idx = philox_np.replay_indices(seed=11, epoch=3, n=65536 - 17, batch=64)
    assert all(0 <= i < 65536 - 17 for i in idx)


def test_host_sizing_rules():
    """Host-side sizing rules of the native calls (no GPU): weight-gradient splits and the
    categorical objective's workspace / counter sizes."""
    from robolearn_b200 import _native as N
    from robolearn_b200.dense import FP16, TF32X3, dw_splits

    # critic weight gradients at cfg3 (2048 x 512, twins, 8192 rows): 128 x 128 tiles fill the SMs
    assert dw_splits(2048, 512, 8192, 2, FP16) == 1
    # actor (1024 x 256, one network): splits of >= 40 k-blocks of 64 rows
    assert dw_splits(1024, 256, 8192, 1, FP16) == 3
    # long K over few tiles: bounded by 32 and by the SM count over the tiles
    assert dw_splits(512, 48, 24576, 2, TF32X3) == 19
    assert dw_splits(12, 128, 100000, 1, TF32X3) == 32
    assert dw_splits(64, 64, 64, 1, FP16) == 1  # too short to split
    lib = N.load()
    for batch, bins in ((4096, 101), (65536, 101), (1, 2), (777, 51)):
        grid = min(-(-batch // 32), 148 * 4)
        groups = -(-grid // 16)
        assert lib.rl2_categorical_workspace_floats(batch, bins) == (grid + groups) * (2 * bins + 2)
        assert lib.rl2_categorical_counter_words(batch, bins) == 1 + groups
