"""Bind librl2's ``rl_*`` entry points with the reference's own ctypes declarations.

``tests/golden/rl_abi.json`` is recorded from the reference's declaration code by
``tests/golden/make_rl_abi.py``; binding through it is what a reference caller does.
"""

from __future__ import annotations

import ctypes
import json
from pathlib import Path

TABLE = json.loads((Path(__file__).resolve().parent / "golden" / "rl_abi.json").read_text())

CTYPES = {
    "ptr": ctypes.c_void_p,
    "int": ctypes.c_int,
    "size": ctypes.c_size_t,
    "float": ctypes.c_float,
    "double": ctypes.c_double,
    "str": ctypes.c_char_p,
    "ptr*": ctypes.POINTER(ctypes.c_void_p),
    "size*": ctypes.POINTER(ctypes.c_size_t),
    "int*": ctypes.POINTER(ctypes.c_int),
}


def bound_library() -> ctypes.CDLL:
    """librl2 loaded afresh (its own handle, so the rl2_* declarations stay untouched)."""
    from robolearn_b200 import _native as N

    N.load()
    lib = ctypes.CDLL(str(N.library_path()))
    for name, sig in TABLE.items():
        fn = getattr(lib, name)
        fn.argtypes = [CTYPES[k] for k in sig["argtypes"]]
        fn.restype = CTYPES[sig["restype"]]
    return lib


def pointers(values) -> ctypes.Array:
    arr = (ctypes.c_void_p * len(values))()
    for i, v in enumerate(values):
        arr[i] = v
    return arr


def sizes(values) -> ctypes.Array:
    return (ctypes.c_size_t * len(values))(*values)


def ints(values) -> ctypes.Array:
    return (ctypes.c_int * len(values))(*values)
