"""Record the reference's ctypes declarations of its native ABI into ``rl_abi.json``.

The reference declares argtypes / restype of its ``rl_*`` entry points in
``src/robolearn/cuda/_runtime.py:77-113`` (``_declare``), ``cuda/flash.py:12-40``,
``cuda/categorical.py:13-29`` and ``cuda/zero.py:13-24`` (each ``_library``). This script
runs that declaration code unchanged against a recording stand-in for the loaded library
(Warp and Warp-NN, which the modules import but the declarations do not use, are replaced
by inert stubs) and writes, per entry point, the argument and result kinds.

Usage: ``python tests/golden/make_rl_abi.py <reference src directory>``
"""

from __future__ import annotations

import ctypes
import json
import sys
import types
from pathlib import Path
from unittest import mock

KINDS = [
    (ctypes.c_void_p, "ptr"),
    (ctypes.c_int, "int"),
    (ctypes.c_size_t, "size"),
    (ctypes.c_float, "float"),
    (ctypes.c_double, "double"),
    (ctypes.c_char_p, "str"),
    (ctypes.POINTER(ctypes.c_void_p), "ptr*"),
    (ctypes.POINTER(ctypes.c_size_t), "size*"),
    (ctypes.POINTER(ctypes.c_int), "int*"),
]


def kind(t) -> str:
    for c, name in KINDS:
        if t is c:
            return name
    raise TypeError(f"unexpected ctypes type {t!r}")


class _Function:
    def __init__(self):
        self.argtypes = None
        self.restype = None


class _Recorder:
    def __init__(self):
        object.__setattr__(self, "functions", {})

    def __getattr__(self, name):
        if name.startswith("rl_"):
            return self.functions.setdefault(name, _Function())
        raise AttributeError(name)


def _stub_warp() -> None:
    warp = mock.MagicMock(name="warp")
    nn = types.SimpleNamespace(Module=type("Module", (), {}))
    warp_nn = types.ModuleType("warp_nn")
    warp_nn.nn = nn
    sys.modules.setdefault("warp", warp)
    sys.modules.setdefault("warp_nn", warp_nn)


def record(reference_src: Path) -> dict:
    _stub_warp()
    sys.path.insert(0, str(reference_src))
    from robolearn.cuda import _runtime, categorical, flash, zero  # noqa: E402

    lib = _Recorder()
    _runtime._declare(lib)
    device = types.SimpleNamespace(alias="cuda:0", is_cuda=True, is_capturing=False)
    for module in (flash, categorical, zero):
        module.library_for = lambda _device, _lib=lib: _lib
        module._library(device)
    return {
        name: {"argtypes": [kind(t) for t in f.argtypes], "restype": kind(f.restype)}
        for name, f in sorted(lib.functions.items())
    }


def main() -> None:
    if len(sys.argv) != 2:
        raise SystemExit(__doc__)
    table = record(Path(sys.argv[1]))
    out = Path(__file__).with_name("rl_abi.json")
    out.write_text(json.dumps(table, indent=1, sort_keys=True) + "\n")
    print(f"{len(table)} entry points -> {out}")


if __name__ == "__main__":
    main()
