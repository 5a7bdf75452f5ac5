"""Build ``librl2.so`` (all CUDA sources under ``csrc/``) for sm_100a, in-tree.

The library is compiled with ``nvcc -gencode arch=compute_100a,code=sm_100a`` and
placed at ``robolearn_b200/_lib/librl2.so`` so it travels with the source tree.
A content hash of the sources, headers and flags skips rebuilding an up-to-date
library. There is no fallback: a failed build raises.
"""

from __future__ import annotations

import concurrent.futures as cf
import hashlib
import os
import shutil
import subprocess
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
CSRC = PACKAGE / "csrc"
INCLUDE = PACKAGE.parent / "include"
OUT_DIR = PACKAGE / "_lib"
LIBRARY = OUT_DIR / "librl2.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-std=c++17", "-O3", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-O3", "--expt-relaxed-constexpr"]


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _identity(nvcc: str) -> str:
    h = hashlib.sha256()
    for path in sorted(list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h"))):
        h.update(path.name.encode())
        h.update(path.read_bytes())
    h.update(" ".join(ARCH + FLAGS).encode())
    h.update(subprocess.run([nvcc, "--version"], capture_output=True, text=True).stdout.encode())
    return h.hexdigest()


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile every ``csrc/*.cu`` and link ``librl2.so``; returns its path."""
    nvcc = os.environ.get("RL2_NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(nvcc).exists() and shutil.which(nvcc) is None:
        raise RuntimeError("nvcc not found: the sm_100a kernels cannot be built")
    identity = _identity(nvcc)
    stamp = OUT_DIR / "librl2.sha256"
    if not force and LIBRARY.exists() and stamp.exists() and stamp.read_text().strip() == identity:
        return LIBRARY
    OUT_DIR.mkdir(parents=True, exist_ok=True)
    objects_dir = OUT_DIR / "obj"
    objects_dir.mkdir(exist_ok=True)

    def compile_one(src: Path) -> Path:
        obj = objects_dir / (src.stem + ".o")
        cmd = [nvcc, *ARCH, *FLAGS, "-I", str(INCLUDE), "-c", str(src), "-o", str(obj)]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
        done = subprocess.run(cmd, capture_output=True, text=True)
        if done.returncode:
            raise RuntimeError(f"nvcc failed for {src.name}:\n{done.stdout}\n{done.stderr}")
        if verbose and done.stderr:
            print(done.stderr)
        return obj

    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as pool:
        objects = list(pool.map(compile_one, _sources()))
    tmp = OUT_DIR / "librl2.so.tmp"
    link = [nvcc, *ARCH, "-shared", "-o", str(tmp), *map(str, objects), "-lcuda"]
    done = subprocess.run(link, capture_output=True, text=True)
    if done.returncode:
        # the driver stub is only needed if a source links a driver symbol directly
        link = [nvcc, *ARCH, "-shared", "-o", str(tmp), *map(str, objects)]
        done = subprocess.run(link, capture_output=True, text=True)
        if done.returncode:
            raise RuntimeError(f"link failed:\n{done.stdout}\n{done.stderr}")
    os.replace(tmp, LIBRARY)
    stamp.write_text(identity + "\n")
    return LIBRARY


if __name__ == "__main__":
    import sys

    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
