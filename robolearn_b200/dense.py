"""Host wrapper of the tcgen05 dense-product plans (``rl2_gemm_*``).

A plan binds persistent device buffers once (their TMA descriptors are encoded
at creation) and then enqueues the product on a stream with no allocation, so
it can be captured in a CUDA graph. This replaces the reference's
``CudaLinear`` cuBLASLt plans (``src/robolearn/cuda/linear.py:155-375``).
"""

from __future__ import annotations

import ctypes

import torch

from . import _native as N

FP16 = 0
TF32X3 = 1
# epilogue activations (rl2_gemm_desc.activation)
ELU = 1
TANH = 2


def operand_ld(cols: int, kind: int) -> int:
    """Row stride (elements) giving 16-byte aligned rows for an operand plane."""
    q = 8 if kind == FP16 else 4
    return (cols + q - 1) // q * q


def dw_splits(m: int, n: int, rows: int, batch: int, kind: int, sms: int = 148) -> int:
    """K splits of a weight-gradient product dW[m][n] = sum over ``rows``: none when the
    128 x 128 tiles already fill most SMs, else enough splits to approach one wave while
    every split keeps at least 40 k-blocks (each split adds a partial output that the
    fixed-order reduce reads back; short splits pay the pipeline fill for little work)."""
    tiles = -(-m // 128) * -(-n // 128) * batch
    if tiles * 3 >= 2 * sms:
        return 1
    kblocks = -(-rows // (64 if kind == FP16 else 32))
    return max(1, min(32, kblocks // 40, -(-sms // tiles)))


def tf32_split(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Exact split ``x = hi + lo`` with ``hi`` representable in tf32 (low 13 mantissa bits cleared)."""
    hi = (x.contiguous().view(torch.int32) & -8192).view(torch.float32)
    return hi, x - hi


class DensePlan:
    """One ``D = scale * A B^T (+ bias) (+ residual) (+ D)`` product over fixed buffers."""

    def __init__(
        self,
        *,
        kind: int,
        m: int,
        n: int,
        k: int,
        a: torch.Tensor,
        b: torch.Tensor,
        d: torch.Tensor,
        lda: int,
        ldb: int,
        ldd: int,
        a_major: int = 0,
        b_major: int = 0,
        batch: int = 1,
        a_batch_stride: int = 0,
        b_batch_stride: int = 0,
        d_batch_stride: int = 0,
        a_lo: torch.Tensor | None = None,
        b_lo: torch.Tensor | None = None,
        accumulate: bool = False,
        bias: torch.Tensor | None = None,
        bias_batch_stride: int = 0,
        residual: torch.Tensor | None = None,
        ldr: int = 0,
        residual_batch_stride: int = 0,
        stat_mean: torch.Tensor | None = None,
        stat_m2: torch.Tensor | None = None,
        stat_batch_stride: int = 0,
        scale: torch.Tensor | None = None,
        k_splits: int = 1,
        d_split_stride: int = 0,
        tile_n: int = 0,
        health: torch.Tensor | None = None,
        out_plane=None,
        activation: int = 0,
        act_aux=None,
        ld_aux: int = 0,
        aux_batch_stride: int = 0,
        bn=None,
    ):
        """``bn``: optional evaluation-mode batch norm of the output columns, a tuple
        (mean, invstd, gamma, beta, twin_stride, relu) of device addresses / ints; the
        residual is then added after the normalisation (transposed plans only)."""
        self._keep = [a, b, d, a_lo, b_lo, bias, residual, stat_mean, stat_m2, scale, health, out_plane, act_aux]
        A = N.addr
        desc = N.GemmDesc(
            kind=kind, m=m, n=n, k=k, batch=batch,
            a=A(a), a_lo=A(a_lo), a_major=a_major, lda=lda, a_batch_stride=a_batch_stride,
            b=A(b), b_lo=A(b_lo), b_major=b_major, ldb=ldb, b_batch_stride=b_batch_stride,
            d=A(d), ldd=ldd, d_batch_stride=d_batch_stride, accumulate=int(accumulate),
            bias=A(bias), bias_batch_stride=bias_batch_stride,
            residual=A(residual), ldr=ldr, residual_batch_stride=residual_batch_stride,
            stat_mean=A(stat_mean), stat_m2=A(stat_m2), stat_batch_stride=stat_batch_stride,
            scale=A(scale), k_splits=k_splits, d_split_stride=d_split_stride, tile_n=tile_n,
            health=A(health), out_plane=out_plane if out_plane is not None else N.Plane(),
            activation=activation, act_aux=A(act_aux), ld_aux=ld_aux, aux_batch_stride=aux_batch_stride,
        )
        if bn is not None:
            desc.bn_mean, desc.bn_invstd, desc.bn_gamma, desc.bn_beta = (A(v) for v in bn[:4])
            desc.bn_twin_stride, desc.bn_relu = int(bn[4]), int(bn[5])
        self._lib = N.load()
        self.handle = N.created(self._lib.rl2_gemm_create(ctypes.byref(desc)), "create tcgen05 GEMM plan")
        self.tile_n = self._lib.rl2_gemm_tile_n(self.handle)
        mode = self._lib.rl2_gemm_uses_tma_store(self.handle)
        self.tma_store = mode == 1
        self.transposed = mode == 2
        self.cta_pair = bool(self._lib.rl2_gemm_cta_pair(self.handle))
        self.flops = 2 * m * n * k * batch * (3 if kind == TF32X3 else 1)
        self.recompute = False  # set by callers that compute the same product twice
        # algorithmic bytes of one launch (operands read once, outputs written once)
        el = 2 if kind == 0 else 8  # fp16, or the tf32 hi + lo planes
        plane = out_plane is not None and (out_plane.h16 or out_plane.hi or out_plane.lo)
        self.bytes = batch * (m * k * el + n * k * el + (m * n * 4 * max(k_splits, 1) if d is not None else 0)
                              + (m * n * el if plane else 0) + (m * n * 4 if residual is not None else 0)
                              + (m * n * 4 if accumulate else 0)
                              + ((m + 31) // 32 * n * 8 if stat_mean is not None else 0))
        self.shape = dict(m=m, n=n, k=k, batch=batch, kind=kind, a_major=a_major, b_major=b_major, splits=k_splits,
                          stats=stat_mean is not None, plane=bool(plane), residual=residual is not None,
                          tile_n=self.tile_n, pair=self.cta_pair, form="transposed" if self.transposed else
                          ("tma-store" if self.tma_store else "register-store"))

    def run(self, stream=None) -> None:
        N.check(self._lib.rl2_gemm_run(self.handle, N.stream_ptr(stream)), "tcgen05 GEMM")

    def __call__(self) -> None:
        self.run()

    def close(self) -> None:
        if self.handle:
            self._lib.rl2_gemm_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def split_reduce(partial: torch.Tensor, split_stride: int, splits: int, out: torch.Tensor, count: int,
                 accumulate: bool = False, stream=None) -> None:
    lib = N.load()
    N.check(lib.rl2_split_reduce(N.ptr(partial), split_stride, splits, N.ptr(out), count, int(accumulate),
                                 N.stream_ptr(stream)), "split-K reduce")
