"""ctypes binding of ``librl2.so`` (the C ABI declared in ``include/rl2.h``).

Mirrors the reference's loader contract (``src/robolearn/cuda/_runtime.py:77-135``):
explicit ``argtypes``/``restype`` per entry point and ``check()`` that turns a -1
status into ``RuntimeError`` with the library's thread-local message. There is no
CPU or library fallback: if the shared library cannot be found or built, loading
raises.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

from . import build as _build

_LOCK = threading.Lock()
_LIB: ctypes.CDLL | None = None

P = ctypes.c_void_p
I = ctypes.c_int  # noqa: E741
LL = ctypes.c_longlong
F = ctypes.c_float
D = ctypes.c_double
SZ = ctypes.c_size_t
U64 = ctypes.c_uint64


class GemmDesc(ctypes.Structure):
    """``rl2_gemm_desc`` (include/rl2.h)."""

    _fields_ = [
        ("kind", I), ("m", I), ("n", I), ("k", I), ("batch", I),
        ("a", P), ("a_lo", P), ("a_major", I), ("lda", LL), ("a_batch_stride", LL),
        ("b", P), ("b_lo", P), ("b_major", I), ("ldb", LL), ("b_batch_stride", LL),
        ("d", P), ("ldd", LL), ("d_batch_stride", LL), ("accumulate", I),
        ("bias", P), ("bias_batch_stride", LL),
        ("residual", P), ("ldr", LL), ("residual_batch_stride", LL),
        ("stat_mean", P), ("stat_m2", P), ("stat_batch_stride", LL),
        ("scale", P), ("k_splits", I), ("d_split_stride", LL), ("tile_n", I), ("health", P),
    ]


class CriticObjectiveArgs(ctypes.Structure):
    """``rl2_critic_objective_args`` (include/rl2.h)."""

    _fields_ = [
        ("target_logits", P), ("target_row_stride", LL), ("target_twin_stride", LL), ("target_row_offset", I),
        ("online_logits", P), ("online_row_stride", LL), ("online_twin_stride", LL),
        ("reward", P), ("terminated", P), ("discount", P), ("next_log_pi", P), ("alpha", P), ("support", P),
        ("min_v", D), ("max_v", D), ("bins", I), ("batch", I), ("loss_weight", F),
        ("dlogits", P), ("dlogits_row_stride", LL), ("dlogits_twin_stride", LL),
        ("d16", P), ("d16_row_stride", LL), ("d16_twin_stride", LL), ("d16_scale", P),
        ("d_hi", P), ("d_lo", P), ("dplane_row_stride", LL), ("dplane_twin_stride", LL),
        ("target_out", P), ("target_out_row_stride", LL),
        ("workspace", P), ("counter", P), ("loss_out", P), ("max_entropy_out", P), ("bias_grad_out", P),
        ("bias_grad_accumulate", I), ("health", P),
    ]


# name -> (argtypes, restype); every symbol here is declared in include/rl2.h
SIGNATURES: dict[str, tuple[list, object]] = {
    "rl2_last_error": ([], ctypes.c_char_p),
    "rl2_abi_version": ([], I),
    "rl2_gemm_create": ([ctypes.POINTER(GemmDesc)], P),
    "rl2_gemm_run": ([P, P], I),
    "rl2_gemm_destroy": ([P], I),
    "rl2_gemm_tile_n": ([P], I),
    "rl2_split_reduce": ([P, LL, I, P, LL, I, P], I),
    "rl2_categorical_workspace_floats": ([I, I], I),
    "rl2_critic_objective": ([ctypes.POINTER(CriticObjectiveArgs), P], I),
}


def library_path() -> Path:
    return _build.LIBRARY


def load(build_if_missing: bool = True) -> ctypes.CDLL:
    """Load (building first if needed and possible) and declare the library."""
    global _LIB
    with _LOCK:
        if _LIB is not None:
            return _LIB
        path = library_path()
        if build_if_missing:
            try:
                path = _build.build()
            except RuntimeError:
                if not path.exists():
                    raise
        if not path.exists():
            raise RuntimeError(f"librl2.so not found at {path}; run robolearn_b200/build.py (needs nvcc)")
        lib = ctypes.CDLL(str(path))
        for name, (args, res) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.argtypes, fn.restype = args, res
        _LIB = lib
        return lib


def check(status: int, what: str) -> None:
    if status:
        message = load().rl2_last_error()
        detail = message.decode("utf-8", errors="replace") if message else "no native error message"
        raise RuntimeError(f"{what}: {detail}")


def created(handle, what: str):
    if not handle:
        message = load().rl2_last_error()
        raise RuntimeError(f"{what}: {message.decode('utf-8', errors='replace') if message else 'creation failed'}")
    return handle


def ptr(t) -> int | None:
    """Device address of a torch tensor (None passes a null pointer)."""
    return None if t is None else t.data_ptr()


def stream_ptr(stream=None) -> int:
    import torch

    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream
