"""Single-kernel timing of the tcgen05 GEMM on one product shape of the update.

    python -m robolearn_b200.microbench --m 8192 --n 2048 --k 512 --batch 2 --stats --plane

Runs the product ``D[z] = A[z] B[z]^T`` (fp16 operands unless ``--kind 1``) with the
forward epilogue the update uses (bias, optional residual, 32-row column moments,
fp16 / tf32 operand-plane copy of the output), times ``--iters`` launches with CUDA
events on the launching stream after ``--warmup`` launches and prints one JSON line
with the duration, TFLOP/s and the algorithmic bytes per launch. Intended as the
small, self-contained case for ``ncu`` captures of the GEMM.
"""

from __future__ import annotations

import argparse
import json

import torch

from . import _native as N
from . import dense


def main() -> None:
    p = argparse.ArgumentParser()
    p.add_argument("--m", type=int, default=8192)
    p.add_argument("--n", type=int, default=2048)
    p.add_argument("--k", type=int, default=512)
    p.add_argument("--batch", type=int, default=2)
    p.add_argument("--kind", type=int, choices=(0, 1), default=0)
    p.add_argument("--a-major", type=int, choices=(0, 1), default=0)
    p.add_argument("--b-major", type=int, choices=(0, 1), default=0)
    p.add_argument("--tile-n", type=int, default=0)
    p.add_argument("--splits", type=int, default=1)
    p.add_argument("--stats", action="store_true")
    p.add_argument("--plane", action="store_true")
    p.add_argument("--residual", action="store_true")
    p.add_argument("--in-place", action="store_true", help="residual = the output itself")
    p.add_argument("--act", type=int, choices=(0, 1, 2), default=0, help="epilogue activation: 1 ELU, 2 tanh")
    p.add_argument("--lo-only", action="store_true", help="tf32 plane as lo alone beside the fp32 output")
    p.add_argument("--no-d", action="store_true", help="write only the operand plane")
    p.add_argument("--iters", type=int, default=20)
    p.add_argument("--warmup", type=int, default=3)
    a = p.parse_args()
    if not torch.cuda.is_available():
        raise SystemExit("microbench needs a CUDA device")
    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    m, n, k, z, kind = a.m, a.n, a.k, a.batch, a.kind
    dt = torch.float16 if kind == 0 else torch.float32
    g = torch.Generator(device=dev).manual_seed(0)

    def operand(rows: int, major: int) -> tuple[torch.Tensor, int]:
        inner, outer = (k, rows) if major == 0 else (rows, k)
        ld = dense.operand_ld(inner, kind)
        t = torch.zeros(z, outer, ld, device=dev, dtype=dt)
        t[:, :, :inner] = (torch.randn(z, outer, inner, device=dev, generator=g) / k**0.5).to(dt)
        return t, ld

    A, lda = operand(m, a.a_major)
    B, ldb = operand(n, a.b_major)
    kw = {}
    if kind == 1:
        A, a_lo = dense.tf32_split(A)
        B, b_lo = dense.tf32_split(B)
        kw.update(a_lo=a_lo, b_lo=b_lo)
    ldd = dense.operand_ld(n, 1)
    splits = max(1, a.splits)
    D = None if a.no_d else torch.zeros(splits, z, m, ldd, device=dev)
    kw.update(d=None, ldd=0)
    if D is not None:
        kw.update(d=D, ldd=ldd, d_batch_stride=m * ldd)
        if splits > 1:
            kw.update(k_splits=splits, d_split_stride=z * m * ldd)
    if splits == 1:
        kw.update(bias=torch.randn(z, n, device=dev, generator=g), bias_batch_stride=n)
    if a.in_place and splits == 1 and D is not None:
        kw.update(residual=D[0], ldr=ldd, residual_batch_stride=m * ldd)
    elif a.residual and splits == 1:
        kw.update(residual=torch.randn(z, m, n, device=dev, generator=g), ldr=n, residual_batch_stride=m * n)
    groups = (m + 31) // 32
    if a.stats and splits == 1:
        kw.update(stat_mean=torch.zeros(z, groups, n, device=dev), stat_m2=torch.zeros(z, groups, n, device=dev),
                  stat_batch_stride=groups * n)
    keep = []
    if a.plane and splits == 1:
        pld = dense.operand_ld(n, kind)
        if kind == 0:
            h = torch.zeros(z, m, pld, device=dev, dtype=torch.float16)
            keep.append(h)
            kw["out_plane"] = N.Plane(h16=h.data_ptr(), ld=pld, twin_stride=m * pld)
        else:
            lo = torch.zeros(z, m, ldd if a.lo_only else pld, device=dev)
            keep.append(lo)
            if a.lo_only:
                kw["out_plane"] = N.Plane(lo=lo.data_ptr(), ld=ldd, twin_stride=m * ldd)
            else:
                hi = torch.zeros(z, m, pld, device=dev)
                keep.append(hi)
                kw["out_plane"] = N.Plane(hi=hi.data_ptr(), lo=lo.data_ptr(), ld=pld, twin_stride=m * pld)
    if a.act:
        kw["activation"] = a.act
    plan = dense.DensePlan(kind=kind, m=m, n=n, k=k, a=A, b=B, lda=lda, ldb=ldb, a_major=a.a_major,
                           b_major=a.b_major, batch=z, a_batch_stride=A[0].numel(), b_batch_stride=B[0].numel(),
                           tile_n=a.tile_n, **kw)
    stream = torch.cuda.current_stream()
    for _ in range(max(a.warmup, 0)):
        plan.run()
    torch.cuda.synchronize()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for _ in range(a.iters):
        plan.run()
    t1.record(stream)
    torch.cuda.synchronize()
    us = t0.elapsed_time(t1) * 1000.0 / max(a.iters, 1)
    el = 2 if kind == 0 else 8
    out_bytes = (0 if D is None else z * m * n * 4 * splits) + (z * m * n * el if a.plane and splits == 1 else 0)
    in_bytes = z * (m + n) * k * el + (z * m * n * 4 if a.residual and splits == 1 else 0)
    flops = 2.0 * z * m * n * k
    print(json.dumps({
        "kernel": "rl2 tcgen05 GEMM", "m": m, "n": n, "k": k, "batch": z, "kind": kind, "a_major": a.a_major,
        "b_major": a.b_major, "tile_n": plan.tile_n, "splits": splits, "stats": a.stats, "plane": a.plane,
        "residual": a.residual, "us_per_launch": round(us, 2), "tflops": round(flops / us / 1e6, 1),
        "algorithmic_bytes": in_bytes + out_bytes, "gbs": round((in_bytes + out_bytes) / us / 1e3, 1),
    }))
    del keep


if __name__ == "__main__":
    main()
