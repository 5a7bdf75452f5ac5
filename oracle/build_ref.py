"""Test infrastructure: compile the reference's own native CUDA library into ``oracle/_ref``.

The reference's native backend is one translation unit, ``src/robolearn/cuda/kernels.cu``
(which includes ``flash_kernels.cuh``, ``categorical_kernels.cuh`` and ``zero_kernels.cuh``)
linked against cuBLASLt. It is compiled here from the sources where they lie, with the
reference's own flags (``src/robolearn/cuda/_runtime.py:41,64``: ``-std=c++17 -O3 --shared
-Xcompiler=-fPIC --fmad=false``, architecture 100), into ``oracle/_ref/librobolearn_cuda.so``.

Only the tests use the result: ``tests/test_compat_ref_gpu.py`` runs the same inputs
through the reference's library and through librl2's ``rl_*`` entry points. Nothing in the
product loads it. The reference tree is given by ``--root``, else ``RL2_REFERENCE_ROOT``,
else a checkout named ``reference`` beside this repository's directory; where it is absent
the build is skipped and the comparison tests skip.

Usage: ``python oracle/build_ref.py [--root PATH]`` (also run by ``__graft_entry__.build()``).
"""

from __future__ import annotations

import hashlib
import os
import shutil
import subprocess
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref" / "librobolearn_cuda.so"
FLAGS = ["-std=c++17", "-O3", "--shared", "-Xcompiler=-fPIC", "--fmad=false", "-gencode",
         "arch=compute_100,code=sm_100"]


def reference_root(root: str | Path | None = None) -> Path:
    """The reference project's root: ``root`` when given, else ``RL2_REFERENCE_ROOT``, else a
    checkout named ``reference`` beside this repository's directory."""
    if root is not None:
        return Path(root)
    env = os.environ.get("RL2_REFERENCE_ROOT")
    return Path(env) if env else HERE.parents[1] / "reference"


def _sources(root: Path) -> list[Path]:
    cuda = root / "src" / "robolearn" / "cuda"
    return [cuda / "kernels.cu", *sorted(cuda.glob("*.cuh"))]


def build(verbose: bool = False, root: str | Path | None = None) -> Path | None:
    """Compile the reference library when its sources are present; returns the path or None."""
    root = reference_root(root)
    srcs = _sources(root)
    if not srcs[0].is_file():
        return None
    nvcc = os.environ.get("RL2_NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    h = hashlib.sha256(" ".join(FLAGS).encode())
    for p in srcs:
        h.update(p.name.encode())
        h.update(p.read_bytes())
    stamp = OUT.with_suffix(".sha256")
    if OUT.is_file() and stamp.is_file() and stamp.read_text() == h.hexdigest():
        return OUT
    OUT.parent.mkdir(parents=True, exist_ok=True)
    tmp = OUT.with_suffix(".tmp.so")
    cmd = [nvcc, *FLAGS, str(srcs[0]), "-lcublasLt", "-o", str(tmp)]
    done = subprocess.run(cmd, capture_output=True, text=True)
    if done.returncode:
        raise RuntimeError(f"reference library build failed:\n{done.stdout}{done.stderr}")
    os.replace(tmp, OUT)
    stamp.write_text(h.hexdigest())
    if verbose:
        print(f"built {OUT}")
    return OUT


if __name__ == "__main__":
    import argparse

    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--root", default=None, help="the reference project's root directory")
    path = build(verbose=True, root=parser.parse_args().root)
    if path is None:
        print("reference sources absent: nothing built")
