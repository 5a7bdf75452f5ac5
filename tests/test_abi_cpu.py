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
