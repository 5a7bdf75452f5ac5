"""FlashSAC residual-MLP networks on flat device arenas, run as explicit launch programs.

Layout in HBM (one ``Net`` per actor / critic / target critic):

* ``params``, ``grads``, ``m``, ``v``: flat fp32 arenas with identical offsets;
  each tensor keeps the reference's ``state_dict`` key and shape
  (``src/robolearn/flashsac/layers.py``, ``networks.py``), twin critics stacked
  on a leading axis of 2 exactly as ``EnsembleUnitLinear`` stores them;
* ``buffers``: BatchNorm running mean / variance, ``[twins][C]`` per layer;
* ``planes``: operand copies of every linear weight, ``[twins][rows][K_pad]``
  (fp16, or tf32 hi + lo for the FP32 recipe), refreshed by the optimizer pass.

A backbone run (``Run``) binds one row count and mode (training / evaluation)
to activation buffers and builds two lists of launches: the forward
(embedder BN -> linear -> residual blocks -> RMS -> head) and the analytic
backward. Every launch is a ctypes call of ``librl2.so`` on the current torch
stream; the learner captures whole updates in CUDA graphs.
"""

from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass, field

import numpy as np
import torch

from .. import _native as N
from ..dense import FP16, TF32X3, DensePlan, dw_splits, operand_ld, split_reduce

BN_EPS = 1e-5
BN_MOMENTUM = 0.01
RMS_EPS = 1e-6
SM_COUNT = 148


def _a4(n: int) -> int:
    return (n + 3) // 4 * 4


def _lib():
    return N.load()


def _call(fn, args, what):
    """Launch closure for an entry point taking (struct*, stream)."""
    ref = ctypes.byref(args)

    def launch():
        N.check(fn(ref, N.stream_ptr()), what)

    launch.args = args  # keep the struct alive
    return launch


# ---------------------------------------------------------------------------
# operand planes
# ---------------------------------------------------------------------------


class PlaneBuf:
    """``[twins][rows][ld]`` operand plane(s): fp16, or tf32 hi + lo."""

    def __init__(self, kind: int, twins: int, rows: int, cols: int, device):
        self.kind, self.twins, self.rows, self.cols = kind, twins, rows, cols
        self.ld = operand_ld(cols, kind)
        self.tstride = rows * self.ld
        n = twins * rows * self.ld
        if kind == FP16:
            self.main = torch.zeros(n, dtype=torch.float16, device=device)
            self.lo = None
        else:
            self.main = torch.zeros(n, dtype=torch.float32, device=device)
            self.lo = torch.zeros(n, dtype=torch.float32, device=device)

    def c(self, scale=None, found_inf=None) -> N.Plane:
        if self.kind == FP16:
            return N.Plane(h16=N.addr(self.main), hi=None, lo=None, ld=self.ld, twin_stride=self.tstride,
                           scale=N.addr(scale), found_inf=N.addr(found_inf))
        return N.Plane(h16=None, hi=N.addr(self.main), lo=N.addr(self.lo), ld=self.ld, twin_stride=self.tstride,
                       scale=None, found_inf=None)

    def value(self) -> torch.Tensor:
        """fp32 view ``[twins, rows, cols]`` of the represented values (tests)."""
        m = self.main.view(self.twins, self.rows, self.ld)[:, :, : self.cols].float()
        if self.lo is not None:
            m = m + self.lo.view(self.twins, self.rows, self.ld)[:, :, : self.cols]
        return m


# ---------------------------------------------------------------------------
# network parameter layout
# ---------------------------------------------------------------------------


@dataclass
class Linear:
    key: str          # state-dict key of the weight (first of a stacked group)
    out: int          # rows per twin (stacked heads: both heads)
    inp: int
    plane_off: int = 0


@dataclass
class Spec:
    """Backbone description: ``twins`` 1 (actor) or 2 (double critic)."""

    twins: int
    in_dim: int
    hidden: int
    blocks: int
    head_out: int                  # critic: bins; actor: 2 * act
    actor_act: int = 0             # actor: action dimension (heads stacked)
    expansion: int = 4

    @property
    def critic(self) -> bool:
        return self.twins == 2


class Net:
    """Parameters, gradients, Adam moments, BN buffers and weight planes of one network."""

    def __init__(self, spec: Spec, kind: int, device, with_optimizer: bool = True):
        self.spec, self.kind, self.device = spec, kind, device
        T, H, E = spec.twins, spec.hidden, spec.hidden * spec.expansion
        crit = spec.critic
        tw = (T,) if crit else ()
        wsuf = ".weight" if crit else ".w.weight"
        # ---- parameter table in nn.Module.parameters() order
        entries: list[tuple[str, tuple, bool]] = []  # (key, shape, starts_aligned_group)
        entries += [("embedder.norm.weight", tw + (spec.in_dim,), True), ("embedder.norm.bias", tw + (spec.in_dim,), True)]
        entries += [(f"embedder.w{wsuf}", tw + (H, spec.in_dim), True)]
        for i in range(spec.blocks):
            entries += [
                (f"encoder.{i}.w1{wsuf}", tw + (E, H), True),
                (f"encoder.{i}.w2{wsuf}", tw + (H, E), True),
                (f"encoder.{i}.norm1.weight", tw + (E,), True),
                (f"encoder.{i}.norm1.bias", tw + (E,), True),
                (f"encoder.{i}.norm2.weight", tw + (H,), True),
                (f"encoder.{i}.norm2.bias", tw + (H,), True),
            ]
        entries += [("post_norm.weight", tw + (H,), True)]
        if crit:
            entries += [("predictor.bias", (T, spec.head_out), True), ("predictor.w.weight", (T, spec.head_out, H), True)]
        else:
            A = spec.actor_act
            # mean/std biases and mean/std weights stay adjacent so each pair reads as one [2A] / [2A][H] tensor
            entries += [("predictor.mean_bias", (A,), True), ("predictor.std_bias", (A,), False),
                        ("predictor.mean_w.w.weight", (A, H), True), ("predictor.std_w.w.weight", (A, H), False)]
        self.param_names = [e[0] for e in entries]
        self.shapes = {k: s for k, s, _ in entries}
        self.offsets = {}
        off = 0
        for key, shape, aligned in entries:
            if aligned:
                off = _a4(off)
            self.offsets[key] = off
            off += int(np.prod(shape))
        self.size = _a4(off)
        # ---- BN buffers
        self.bn_layers = [("embedder.norm", spec.in_dim)]
        for i in range(spec.blocks):
            self.bn_layers += [(f"encoder.{i}.norm1", E), (f"encoder.{i}.norm2", H)]
        # all running means first, then all running variances at the same relative offsets,
        # so one launch turns the whole arena into evaluation (mean, invstd)
        self.buf_offsets = {}
        boff = 0
        for pre, C in self.bn_layers:
            self.buf_offsets[pre + ".running_mean"] = boff
            boff += T * C
        self.means_size = boff
        for pre, C in self.bn_layers:
            self.buf_offsets[pre + ".running_var"] = self.buf_offsets[pre + ".running_mean"] + self.means_size
        self.buf_size = 2 * boff
        # ---- linear layers and their operand planes
        self.linears = {"embed": Linear(f"embedder.w{wsuf}", H, spec.in_dim)}
        for i in range(spec.blocks):
            self.linears[f"w1.{i}"] = Linear(f"encoder.{i}.w1{wsuf}", E, H)
            self.linears[f"w2.{i}"] = Linear(f"encoder.{i}.w2{wsuf}", H, E)
        head_key = "predictor.w.weight" if crit else "predictor.mean_w.w.weight"
        self.linears["head"] = Linear(head_key, spec.head_out, H)
        poff = 0
        q = 8 if kind == FP16 else 4
        for lin in self.linears.values():
            poff = (poff + 63) // 64 * 64
            lin.plane_off = poff
            poff += T * lin.out * operand_ld(lin.inp, kind)
        self.plane_size = (poff + q - 1) // q * q
        # ---- storage
        f32 = dict(dtype=torch.float32, device=device)
        self.params = torch.zeros(self.size, **f32)
        self.buffers = torch.zeros(max(self.buf_size, 4), **f32)
        self.eval_mean = torch.zeros(max(self.means_size, 4), **f32)
        self.eval_invstd = torch.zeros(max(self.means_size, 4), **f32)
        for pre, C in self.bn_layers:
            self.buffer(pre + ".running_var").fill_(1.0)
        if kind == FP16:
            self.plane_main = torch.zeros(self.plane_size, dtype=torch.float16, device=device)
            self.plane_lo = None
        else:
            self.plane_main = torch.zeros(self.plane_size, **f32)
            self.plane_lo = torch.zeros(self.plane_size, **f32)
        self.with_optimizer = with_optimizer
        if with_optimizer:
            self.grads = torch.zeros(self.size, **f32)
            self.m = torch.zeros(self.size, **f32)
            self.v = torch.zeros(self.size, **f32)
            # [attempts, steps, step_size, bc2, lr, skip, scale, growth, skipped]
            self.opt_state = torch.zeros(9, **f32)
        self.segments = self._segments()

    # ---- views
    def param(self, key: str) -> torch.Tensor:
        shape = self.shapes[key]
        o = self.offsets[key]
        return self.params[o:o + int(np.prod(shape))].view(shape)

    def grad(self, key: str) -> torch.Tensor:
        shape = self.shapes[key]
        o = self.offsets[key]
        return self.grads[o:o + int(np.prod(shape))].view(shape)

    def moment(self, which: str, key: str) -> torch.Tensor:
        shape = self.shapes[key]
        o = self.offsets[key]
        arena = self.m if which == "m" else self.v
        return arena[o:o + int(np.prod(shape))].view(shape)

    def buffer(self, key: str) -> torch.Tensor:
        pre = key.rsplit(".", 1)[0]
        C = dict(self.bn_layers)[pre]
        o = self.buf_offsets[key]
        t = self.buffers[o:o + self.spec.twins * C]
        return t.view(self.spec.twins, C) if self.spec.critic else t.view(C)

    def eval_stats(self, pre: str) -> tuple[int, int]:
        """Addresses of the evaluation-mode (mean, invstd) for BN layer ``pre``."""
        o = self.buf_offsets[pre + ".running_mean"]
        return (self.eval_mean.data_ptr() + 4 * o, self.eval_invstd.data_ptr() + 4 * o)

    def eval_prepare(self) -> None:
        """mean = running_mean, invstd = 1/sqrt(running_var + eps) for every BN layer, one launch."""
        n = self.means_size
        N.check(_lib().rl2_bn_eval_prepare(self.buffers.data_ptr(), self.buffers.data_ptr() + 4 * n, n, BN_EPS,
                                           self.eval_mean.data_ptr(), self.eval_invstd.data_ptr(), N.stream_ptr()),
                "bn eval prepare")

    def addr(self, key: str, arena: str = "params") -> int:
        t = self.params if arena == "params" else self.grads
        return t.data_ptr() + 4 * self.offsets[key]

    def plane_addr(self, lin: Linear) -> tuple[int, int | None]:
        es = 2 if self.kind == FP16 else 4
        main = self.plane_main.data_ptr() + es * lin.plane_off
        lo = None if self.plane_lo is None else self.plane_lo.data_ptr() + 4 * lin.plane_off
        return main, lo

    def plane_c(self) -> N.Plane:
        if self.kind == FP16:
            return N.Plane(h16=N.addr(self.plane_main), ld=0, twin_stride=0)
        return N.Plane(hi=N.addr(self.plane_main), lo=N.addr(self.plane_lo), ld=0, twin_stride=0)

    def state_dict(self) -> dict[str, torch.Tensor]:
        out = {k: self.param(k).clone() for k in self.param_names}
        for pre, _ in self.bn_layers:
            out[pre + ".running_mean"] = self.buffer(pre + ".running_mean").clone()
            out[pre + ".running_var"] = self.buffer(pre + ".running_var").clone()
        return out

    def load_state_dict(self, state: dict, strict: bool = True) -> None:
        for k in self.param_names:
            if k in state:
                self.param(k).copy_(torch.as_tensor(state[k]).reshape(self.shapes[k]))
            elif strict:
                raise KeyError(k)
        for pre, _ in self.bn_layers:
            for suf in (".running_mean", ".running_var"):
                if pre + suf in state:
                    self.buffer(pre + suf).copy_(torch.as_tensor(state[pre + suf]).reshape(self.buffer(pre + suf).shape))
        self.refresh_planes()

    # ---- optimizer segments (projection units)
    def _segments(self) -> torch.Tensor:
        spec = self.spec
        T = spec.twins
        rows: list[tuple[int, int, int, int, int]] = []  # offset, offset2, plane_offset, length, kind
        lin_by_key = {lin.key: lin for lin in self.linears.values()}
        for key in self.param_names:
            shape = self.shapes[key]
            o = self.offsets[key]
            if key in lin_by_key or key == "predictor.std_w.w.weight":
                if key == "predictor.std_w.w.weight":
                    lin = self.linears["head"]
                    row_shift = spec.actor_act
                else:
                    lin = lin_by_key[key]
                    row_shift = 0
                n_out, k_in = shape[-2], shape[-1]
                kp = operand_ld(k_in, self.kind)
                for t in range(T):
                    for r in range(n_out):
                        rows.append((o + (t * n_out + r) * k_in, -1,
                                     lin.plane_off + (t * lin.out + row_shift + r) * kp, k_in, 1))
            elif key == "post_norm.weight":
                C = shape[-1]
                for t in range(T):
                    rows.append((o + t * C, -1, -1, C, 3))
            elif key.endswith("norm.weight") or key.endswith("norm1.weight") or key.endswith("norm2.weight"):
                C = shape[-1]
                ob = self.offsets[key[: -len("weight")] + "bias"]
                for t in range(T):
                    rows.append((o + t * C, ob + t * C, -1, C, 2))
            elif key.endswith(".bias") and "norm" in key:
                continue
            else:  # plain biases
                C = shape[-1]
                for t in range(T if len(shape) == 2 else 1):
                    rows.append((o + t * C, -1, -1, C, 0))
        table, self.segment_count, self.warp_segment_count = N.segment_table(rows, self.device)
        return table

    def refresh_planes(self, project: bool = False) -> None:
        """Rewrite every weight operand plane from the fp32 parameters (and optionally project)."""
        a = N.AdamArgs(params=N.addr(self.params), grads=None, m=None, v=None, segments=N.addr(self.segments),
                       count=self.segment_count, state=None, formula=0, beta1=0.9, beta2=0.999, eps=1e-8,
                       project=int(project), weight_plane=self.plane_c(), target_params=None, tau=0.0,
                       target_plane=N.Plane(), warp_segments=self.warp_segment_count)
        N.check(_lib().rl2_adam_step(ctypes.byref(a), N.stream_ptr()), "refresh weight planes")


# ---------------------------------------------------------------------------
# one backbone run: forward and backward launch programs
# ---------------------------------------------------------------------------


@dataclass
class Scaler:
    """Loss-scale device scalars of the fp16 recipe (None in the FP32 recipe)."""

    scale: torch.Tensor | None = None
    inv_scale: torch.Tensor | None = None
    found_inf: torch.Tensor | None = None


class Run:
    """Forward / backward programs of one ``Net`` over ``rows`` input rows.

    ``x`` is the fp32 input ``[rows][ldx]`` (shared by both twins). ``pool`` lets
    several runs of the same shape share activation buffers (runs that never
    overlap in time, e.g. target and online critic forwards).
    """

    def __init__(self, net: Net, rows: int, training: bool, x_addr: int, ldx: int, *, update_running: bool,
                 need_param_grads: bool, need_input_grad: bool, scaler: Scaler | None = None,
                 pool: dict | None = None, head_ld: int | None = None, out_plane_rows: int | None = None,
                 dp=None):
        self.net, self.rows, self.training = net, rows, training
        # data parallel: batch-norm statistics over the global batch of all ranks
        self.dp = dp if (dp is not None and dp.world > 1 and training) else None
        self.x_addr, self.ldx = x_addr, ldx
        self.update_running = update_running and training
        self.need_param_grads = need_param_grads
        self.need_input_grad = need_input_grad
        self.backward_needed = need_param_grads or need_input_grad
        self.scaler = scaler or Scaler()
        spec = net.spec
        self.T, self.H, self.E = spec.twins, spec.hidden, spec.hidden * spec.expansion
        self.G = (rows + 31) // 32
        if spec.blocks < 1:
            raise NotImplementedError("backbones need at least one residual block")
        if training and rows < 2:
            raise ValueError("training-mode batch norm needs at least two rows")
        dev = net.device
        self.pool = pool if pool is not None else {}
        T, H, E, R, kind = self.T, self.H, self.E, rows, net.kind
        f32 = lambda *shape: torch.zeros(*shape, dtype=torch.float32, device=dev)  # noqa: E731

        def buf(name, maker):
            if name not in self.pool:
                self.pool[name] = maker()
            return self.pool[name]

        self.e = buf("e", lambda: PlaneBuf(kind, T, R, spec.in_dim, dev))
        self.h = [buf(f"h{i}", lambda: f32(T, R, H)) for i in range(spec.blocks + 1)]
        self.hp = [buf(f"hp{i}", lambda: PlaneBuf(kind, T, R, H, dev)) for i in range(spec.blocks + 1)]
        self.t1 = [buf(f"t1.{i}", lambda: f32(T, R, E)) for i in range(spec.blocks)]
        self.t2 = [buf(f"t2.{i}", lambda: f32(T, R, H)) for i in range(spec.blocks)]
        self.a1 = [buf(f"a1.{i}", lambda: PlaneBuf(kind, T, R, E, dev)) for i in range(spec.blocks)]
        self.u = buf("u", lambda: PlaneBuf(kind, T, R, H, dev))
        self.r = buf("r", lambda: f32(T, R))
        self.head_ld = head_ld or _a4(spec.head_out)
        self.out = buf("out", lambda: f32(T, R, self.head_ld))
        # batch statistics of this run (per BN layer): partials + mean / invstd
        Cmax = max(spec.in_dim, E)
        # per-group column moments of the current BN layer, packed [mean: T][G][C] | [M2: T][G][C]
        self.pmq = buf("pmq", lambda: f32(2 * T * self.G * Cmax))
        if self.dp is not None:
            if rows % 32:
                raise ValueError("data-parallel batch norm needs a per-rank batch that is a multiple of 32")
            W = self.dp.world
            self.gpmq = buf("gpmq", lambda: f32(W * 2 * T * self.G * Cmax))
        self.stats = {}
        for pre, C in net.bn_layers:
            self.stats[pre] = (buf(f"mean.{pre}", lambda C=C: f32(T, C)), buf(f"inv.{pre}", lambda C=C: f32(T, C)))
        # backward buffers
        if need_param_grads or need_input_grad:
            self.dhead = buf("dhead", lambda: PlaneBuf(kind, T, out_plane_rows or R, spec.head_out, dev))
            self.du = buf("du", lambda: f32(T, R, H))
            self.dh = buf("dh", lambda: f32(T, R, H))
            self.dh_plane = buf("dhp", lambda: PlaneBuf(kind, T, R, H, dev))
            self.da1 = buf("da1", lambda: f32(T, R, E))
            self.dt2 = buf("dt2", lambda: PlaneBuf(kind, T, R, H, dev))
            self.dt1 = buf("dt1", lambda: PlaneBuf(kind, T, R, E, dev))
            self.de = buf("de", lambda: f32(T, R, spec.in_dim))
            # backward per-group sums of the current BN layer, packed [s1: T][G][C] | [s2: T][G][C]
            self.s12 = buf("s12", lambda: f32(2 * T * self.G * Cmax))
            self.coef1 = buf("c1", lambda: f32(T, Cmax))
            self.coef2 = buf("c2", lambda: f32(T, Cmax))
            self.rms_part = buf("rmsp", lambda: f32(T, self.G, H))
            if self.dp is not None:
                W = self.dp.world
                self.gs12 = buf("gs12", lambda: f32(W * 2 * T * self.G * Cmax))
                self.coef_local = buf("cl", lambda: f32(2, T, Cmax))
            if need_input_grad:
                self.dx = buf("dx", lambda: f32(R, _a4(spec.in_dim)))
        self.split_ws = None
        self.forward_program = self._forward()
        self.backward_program = self._backward() if (need_param_grads or need_input_grad) else []

    # ---- GEMM plan helpers ------------------------------------------------
    def _fwd_gemm(self, lin: Linear, a: PlaneBuf, d: torch.Tensor, ldd: int, stats: bool, bias_addr=None,
                  out_plane: PlaneBuf | None = None):
        net = self.net
        bm, bl = net.plane_addr(lin)
        kp = operand_ld(lin.inp, net.kind)
        kw = {}
        if stats:
            base = self.pmq.data_ptr()
            kw = dict(stat_mean=base, stat_m2=base + 4 * self.T * self.G * lin.out, stat_batch_stride=self.G * lin.out)
        return DensePlan(kind=net.kind, m=self.rows, n=lin.out, k=lin.inp, batch=self.T,
                         a=a.main, a_lo=a.lo, a_major=0, lda=a.ld, a_batch_stride=a.tstride,
                         b=bm, b_lo=bl, b_major=0, ldb=kp, b_batch_stride=lin.out * kp,
                         d=d, ldd=ldd, d_batch_stride=self.rows * ldd if d is not None else 0, bias=bias_addr,
                         bias_batch_stride=lin.out if bias_addr else 0,
                         out_plane=out_plane.c() if out_plane is not None else None, **kw)

    def _fwd_gemm_bn(self, lin: Linear, a: PlaneBuf, pre: str, out_plane: PlaneBuf, d=None, ldd: int = 0,
                     residual=None):
        """Evaluation-mode product with the following batch norm + ReLU (+ residual) fused into
        its epilogue: out = residual + relu(BN_eval(a W^T)); no pre-normalisation output."""
        net = self.net
        bm, bl = net.plane_addr(lin)
        kp = operand_ld(lin.inp, net.kind)
        mean, inv = self._stats_ptrs(pre)
        bn = (mean, inv, net.addr(pre + ".weight"), net.addr(pre + ".bias"), lin.out, 1)
        return DensePlan(kind=net.kind, m=self.rows, n=lin.out, k=lin.inp, batch=self.T,
                         a=a.main, a_lo=a.lo, a_major=0, lda=a.ld, a_batch_stride=a.tstride,
                         b=bm, b_lo=bl, b_major=0, ldb=kp, b_batch_stride=lin.out * kp,
                         d=d, ldd=ldd, d_batch_stride=self.rows * ldd if d is not None else 0,
                         residual=residual, ldr=ldd, residual_batch_stride=self.rows * ldd if residual is not None else 0,
                         out_plane=out_plane.c(), bn=bn)

    def _dx_gemm(self, lin: Linear, dplane: PlaneBuf, d_addr, ldd: int, residual=None, out_plane=None):
        net = self.net
        bm, bl = net.plane_addr(lin)
        kp = operand_ld(lin.inp, net.kind)
        return DensePlan(kind=net.kind, m=self.rows, n=lin.inp, k=lin.out, batch=self.T,
                         a=dplane.main, a_lo=dplane.lo, a_major=0, lda=dplane.ld, a_batch_stride=dplane.tstride,
                         b=bm, b_lo=bl, b_major=1, ldb=kp, b_batch_stride=lin.out * kp,
                         d=d_addr, ldd=ldd, d_batch_stride=self.rows * ldd,
                         residual=residual, ldr=ldd, residual_batch_stride=self.rows * ldd if residual is not None else 0,
                         scale=self.scaler.inv_scale, out_plane=out_plane)

    def _dw_gemm(self, lin: Linear, dplane: PlaneBuf, xplane: PlaneBuf, grad_key: str):
        """dW[t] = dY[t]^T X[t] into the gradient arena, split over rows when the grid is small."""
        net = self.net
        n_out, k_in = lin.out, lin.inp
        splits = dw_splits(n_out, k_in, self.rows, self.T, net.kind, SM_COUNT)
        d_addr = net.addr(grad_key, "grads")
        count = self.T * n_out * k_in
        common = dict(kind=net.kind, m=n_out, n=k_in, k=self.rows, batch=self.T,
                      a=dplane.main, a_lo=dplane.lo, a_major=1, lda=dplane.ld, a_batch_stride=dplane.tstride,
                      b=xplane.main, b_lo=xplane.lo, b_major=1, ldb=xplane.ld, b_batch_stride=xplane.tstride,
                      ldd=k_in, d_batch_stride=n_out * k_in, scale=self.scaler.inv_scale)
        if splits == 1:
            return [DensePlan(d=d_addr, **common)]
        ws = self._workspace(splits * count)
        plan = DensePlan(d=ws, k_splits=splits, d_split_stride=count, **common)
        lib = _lib()

        def reduce_launch():
            N.check(lib.rl2_split_reduce(ws.data_ptr(), count, splits, d_addr, count, 0, N.stream_ptr()),
                    "split-K reduce")

        return [plan, reduce_launch]

    def _workspace(self, floats: int) -> torch.Tensor:
        key = "splitws"
        have = self.pool.get(key)
        if have is None or have.numel() < floats:
            self.pool[key] = torch.zeros(floats, dtype=torch.float32, device=self.net.device)
        return self.pool[key]

    # ---- forward ----------------------------------------------------------
    def _bn_stats(self, pre: str, C: int, src_part_shared: bool):
        """finalize launch for BN layer ``pre`` from the per-group partials in pm/pq."""
        lib = _lib()
        mean, inv = self.stats[pre]
        rm = self.net.buffer(pre + ".running_mean")
        rv = self.net.buffer(pre + ".running_var")
        pt = 0 if src_part_shared else self.G * C
        T, R, upd = self.T, self.rows, int(self.update_running)
        tw = 1 if src_part_shared else T  # twins holding partials (the shared input has one set)
        n = tw * self.G * C
        pmq = self.pmq
        dp = self.dp
        if dp is not None and dp.peer is not None:  # one kernel: local merge, peer exchange, global merge
            ex = dp.peer.slot(C, T)

            def launch():
                base = pmq.data_ptr()
                N.check(lib.rl2_syncbn_forward(base, base + 4 * n, pt, tw, T, R, C, mean.data_ptr(), inv.data_ptr(),
                                               rm.data_ptr(), rv.data_ptr(), BN_MOMENTUM, BN_EPS, upd,
                                               ctypes.byref(ex), N.stream_ptr()), "bn statistics (peer exchange)")

            return launch
        if dp is not None:  # one all-gather of every rank's packed partials, then a global merge
            gpmq, W, G = self.gpmq, dp.world, self.G

            def launch():
                dp.all_gather(pmq[:2 * n], gpmq[:W * 2 * n])
                base = gpmq.data_ptr()
                N.check(lib.rl2_bn_finalize_ranked(base, base + 4 * n, pt, G, 2 * n, T, W * R, C, mean.data_ptr(),
                                                   inv.data_ptr(), rm.data_ptr(), rv.data_ptr(), BN_MOMENTUM, BN_EPS,
                                                   upd, N.stream_ptr()), "bn finalize (global)")

            launch.launches = 1
            return launch

        def launch():
            base = pmq.data_ptr()
            N.check(lib.rl2_bn_finalize(base, base + 4 * n, pt, T, R, C, mean.data_ptr(), inv.data_ptr(),
                                        rm.data_ptr(), rv.data_ptr(), BN_MOMENTUM, BN_EPS, upd, N.stream_ptr()),
                    "bn finalize")

        return launch

    def _stats_ptrs(self, pre: str):
        if self.training:
            m, i = self.stats[pre]
            return m.data_ptr(), i.data_ptr()
        return self.net.eval_stats(pre)

    def _apply(self, pre: str, C: int, x_addr: int, ldx: int, xts: int, relu: bool, residual=None,
               y: torch.Tensor | None = None, plane: PlaneBuf | None = None):
        lib = _lib()
        mean, inv = self._stats_ptrs(pre)
        a = N.BnApplyArgs(x=x_addr, ldx=ldx, x_twin_stride=xts, twins=self.T, rows=self.rows, cols=C,
                          mean=mean, invstd=inv, gamma=self.net.addr(pre + ".weight"),
                          beta=self.net.addr(pre + ".bias"), relu=int(relu),
                          residual=N.addr(residual), ldr=C, residual_twin_stride=self.rows * C if residual is not None else 0,
                          y=N.addr(y), ldy=C, y_twin_stride=self.rows * C,
                          plane=plane.c() if plane is not None else N.Plane())
        return _call(lib.rl2_bn_apply, a, "bn apply")

    def _forward(self):
        net, spec, lib = self.net, self.net.spec, _lib()
        T, H, E, R = self.T, self.H, self.E, self.rows
        prog = []
        if not self.training:
            prog.append(net.eval_prepare)
        # embedder BN on the shared fp32 input
        Cin = spec.in_dim
        if self.training:
            x_addr, ldx, pmq, G = self.x_addr, self.ldx, self.pmq, self.G

            def colstats():
                base = pmq.data_ptr()  # one shared set: [mean: G][Cin] | [M2: G][Cin]
                N.check(lib.rl2_colstats(x_addr, ldx, 0, 1, R, Cin, base, base + 4 * G * Cin, G * Cin,
                                         N.stream_ptr()), "input column statistics")

            prog += [colstats, self._bn_stats("embedder.norm", Cin, src_part_shared=True)]
        prog.append(self._apply("embedder.norm", Cin, self.x_addr, self.ldx, 0, relu=False, plane=self.e))
        prog.append(self._fwd_gemm(net.linears["embed"], self.e, self.h[0], H, stats=False, out_plane=self.hp[0]))
        # evaluation-mode BN + ReLU (+ residual) in the product epilogue (transposed plans, so
        # both widths >= 128); the pre-normalisation outputs t1 / t2 are then not stored, so a
        # run whose backward needs them (the frozen critic's action gradient rebuilds its ReLU
        # masks from them) keeps the separate products and apply passes
        fused_eval = not self.training and not self.backward_needed and min(E, H) >= 128
        # training without a backward pass (the target critic): the wide pre-normalisation
        # output is never stored; a statistics-only product, then the product again with the
        # batch norm fused into its epilogue
        # (only where the product is cheap next to the bytes it saves: fp16 operands, K <= 512;
        # a 3xTF32 product or a long K costs more than the stored output and the apply pass)
        recompute_wide = (self.training and not self.backward_needed and E >= 128 and net.kind == FP16
                          and H <= 512)
        for i in range(spec.blocks):
            if recompute_wide:
                w1, pre1 = net.linears[f"w1.{i}"], f"encoder.{i}.norm1"
                stats_pass = self._fwd_gemm(w1, self.hp[i], None, 0, stats=True)
                stats_pass.recompute = True  # the product is computed twice: one counts as work
                prog.append(stats_pass)
                prog.append(self._bn_stats(pre1, E, src_part_shared=False))
                prog.append(self._fwd_gemm_bn(w1, self.hp[i], pre1, self.a1[i]))
                prog.append(self._fwd_gemm(net.linears[f"w2.{i}"], self.a1[i], self.t2[i], H, stats=True))
                prog.append(self._bn_stats(f"encoder.{i}.norm2", H, src_part_shared=False))
                prog.append(self._apply(f"encoder.{i}.norm2", H, self.t2[i].data_ptr(), H, R * H, relu=True,
                                        residual=self.h[i], y=self.h[i + 1], plane=self.hp[i + 1]))
                continue
            if fused_eval:
                prog.append(self._fwd_gemm_bn(net.linears[f"w1.{i}"], self.hp[i], f"encoder.{i}.norm1", self.a1[i]))
                prog.append(self._fwd_gemm_bn(net.linears[f"w2.{i}"], self.a1[i], f"encoder.{i}.norm2", self.hp[i + 1],
                                              d=self.h[i + 1], ldd=H, residual=self.h[i]))
                continue
            prog.append(self._fwd_gemm(net.linears[f"w1.{i}"], self.hp[i], self.t1[i], E, stats=self.training))
            if self.training:
                prog.append(self._bn_stats(f"encoder.{i}.norm1", E, src_part_shared=False))
            prog.append(self._apply(f"encoder.{i}.norm1", E, self.t1[i].data_ptr(), E, R * E, relu=True,
                                    plane=self.a1[i]))
            prog.append(self._fwd_gemm(net.linears[f"w2.{i}"], self.a1[i], self.t2[i], H, stats=self.training))
            if self.training:
                prog.append(self._bn_stats(f"encoder.{i}.norm2", H, src_part_shared=False))
            prog.append(self._apply(f"encoder.{i}.norm2", H, self.t2[i].data_ptr(), H, R * H, relu=True,
                                    residual=self.h[i], y=self.h[i + 1], plane=self.hp[i + 1]))
        hL, r, u = self.h[spec.blocks], self.r, self.u
        gamma = net.addr("post_norm.weight")
        uplane = u.c()

        def rms():
            N.check(lib.rl2_rms_forward(hL.data_ptr(), H, R * H, T, R, H, gamma, RMS_EPS, r.data_ptr(), None, 0, 0,
                                        ctypes.byref(uplane), N.stream_ptr()), "rms forward")

        prog.append(rms)
        bias_key = "predictor.bias" if spec.critic else "predictor.mean_bias"
        prog.append(self._fwd_gemm(net.linears["head"], self.u, self.out, self.head_ld, stats=False,
                                   bias_addr=net.addr(bias_key)))
        return prog

    # ---- backward ---------------------------------------------------------
    def _bn_backward(self, pre: str, C: int, dy: torch.Tensor, x_addr: int, ldx: int, xts: int, relu: bool,
                     plane: PlaneBuf | None, dx=None, lddx=0, dxts=0, sum_twins=False):
        lib, net = _lib(), self.net
        mean, inv = self._stats_ptrs(pre)
        sc = self.scaler
        n12 = self.T * self.G * C  # packed [s1 | s2] of this layer
        s1p = self.s12.data_ptr() if self.training else None
        s2p = s1p + 4 * n12 if self.training else None
        a = N.BnBackwardArgs(dy=dy.data_ptr(), lddy=C, dy_twin_stride=self.rows * C, x=x_addr, ldx=ldx,
                             x_twin_stride=xts, twins=self.T, rows=self.rows, cols=C, mean=mean, invstd=inv,
                             gamma=net.addr(pre + ".weight"), beta=net.addr(pre + ".bias"), relu=int(relu),
                             training=int(self.training), s1_part=N.addr(s1p), s2_part=N.addr(s2p),
                             coef1=N.addr(self.coef1), coef2=N.addr(self.coef2), dx=N.addr(dx), lddx=lddx,
                             dx_twin_stride=dxts, sum_twins=int(sum_twins),
                             plane=plane.c(sc.scale, sc.found_inf) if plane is not None else N.Plane())
        prog = []
        if self.training:
            prog.append(_call(lib.rl2_bn_backward_reduce, a, "bn backward reduce"))
            T, R = self.T, self.rows
            s12, c1, c2 = self.s12, self.coef1, self.coef2
            gw = net.addr(pre + ".weight", "grads") if self.need_param_grads else None
            gb = net.addr(pre + ".bias", "grads") if self.need_param_grads else None
            gts = C if self.T == 2 else 0

            dp = self.dp
            if dp is not None and dp.peer is not None:
                # gamma / beta gradients from this rank's rows, dx coefficients from the
                # global sums, exchanged over peer memory inside the kernel
                ex = dp.peer.slot(C, T)

                def fin():
                    N.check(lib.rl2_syncbn_backward(s1p, s2p, self.G * C, T, R, C, gw, gb, gts, c1.data_ptr(),
                                                    c2.data_ptr(), ctypes.byref(ex), N.stream_ptr()),
                            "bn backward sums (peer exchange)")
            elif dp is None:
                def fin():
                    N.check(lib.rl2_bn_backward_finalize(s1p, s2p, T, R, C, gw, gb, gts, 0, c1.data_ptr(),
                                                         c2.data_ptr(), N.stream_ptr()), "bn backward finalize")
            else:
                # gamma / beta gradients from this rank's rows (averaged with the other
                # gradients later); dx coefficients from the global sums of all ranks
                gs12, cl, W, G = self.gs12, self.coef_local, dp.world, self.G

                def fin():
                    s = N.stream_ptr()
                    if gw is not None:
                        N.check(lib.rl2_bn_backward_finalize(s1p, s2p, T, R, C, gw, gb, gts, 0, cl[0].data_ptr(),
                                                             cl[1].data_ptr(), s), "bn backward finalize (local)")
                    dp.all_gather(s12[:2 * n12], gs12[:W * 2 * n12])
                    base = gs12.data_ptr()
                    N.check(lib.rl2_bn_backward_finalize_ranked(base, base + 4 * n12, G * C, G, 2 * n12, T, W * R, C,
                                                                None, None, 0, 0, c1.data_ptr(), c2.data_ptr(),
                                                                N.stream_ptr()), "bn backward finalize (global)")

                fin.launches = 2 if gw is not None else 1

            prog.append(fin)
        if plane is not None or dx is not None:
            prog.append(_call(lib.rl2_bn_backward_apply, a, "bn backward apply"))
        return prog

    def _backward(self):
        """Backward launch list; ``grad_marks`` records (position, arena offset) pairs: after
        the launch at that position every parameter gradient from the offset on is final."""
        self.grad_marks = []
        net, spec, lib = self.net, self.net.spec, _lib()
        T, H, E, R = self.T, self.H, self.E, self.rows
        pg = self.need_param_grads
        prog = []
        head = net.linears["head"]
        head_key = "predictor.w.weight" if spec.critic else "predictor.mean_w.w.weight"
        if pg:
            prog += self._dw_gemm(head, self.dhead, self.u, head_key)
        prog.append(self._dx_gemm(head, self.dhead, self.du, H))
        du, dh, hL, r = self.du, self.dh, self.h[spec.blocks], self.r
        gamma = net.addr("post_norm.weight")
        rp = self.rms_part if pg else None
        g_rms = net.addr("post_norm.weight", "grads") if pg else None
        G = self.G

        def rms_b():
            N.check(lib.rl2_rms_backward(du.data_ptr(), H, R * H, hL.data_ptr(), H, R * H, r.data_ptr(), gamma, T, R,
                                         H, dh.data_ptr(), H, R * H, N.addr(rp), N.stream_ptr()), "rms backward")
            if rp is not None:
                N.check(lib.rl2_colsum_finalize(rp.data_ptr(), T, G, H, g_rms, H if T == 2 else 0, 0,
                                                N.stream_ptr()), "rms weight gradient")

        prog.append(rms_b)
        wsuf = ".weight" if spec.critic else ".w.weight"
        for i in reversed(range(spec.blocks)):
            prog += self._bn_backward(f"encoder.{i}.norm2", H, self.dh, self.t2[i].data_ptr(), H, R * H, True,
                                      self.dt2)
            if pg:
                prog += self._dw_gemm(net.linears[f"w2.{i}"], self.dt2, self.a1[i], f"encoder.{i}.w2{wsuf}")
            prog.append(self._dx_gemm(net.linears[f"w2.{i}"], self.dt2, self.da1, E))
            prog += self._bn_backward(f"encoder.{i}.norm1", E, self.da1, self.t1[i].data_ptr(), E, R * E, True,
                                      self.dt1)
            if pg:
                prog += self._dw_gemm(net.linears[f"w1.{i}"], self.dt1, self.hp[i], f"encoder.{i}.w1{wsuf}")
                # every gradient from this block's first parameter to the end of the arena is
                # final here (blocks, post-norm and head come after it in the arena)
                self.grad_marks.append((len(prog), net.offsets[f"encoder.{i}.w1{wsuf}"]))
            # block 0's input gradient dh0 also feeds the embedder products as an operand plane
            emit = self.dh_plane.c(self.scaler.scale, self.scaler.found_inf) if i == 0 else None
            prog.append(self._dx_gemm(net.linears[f"w1.{i}"], self.dt1, self.dh, H, residual=self.dh, out_plane=emit))
        embed = net.linears["embed"]
        if pg:
            prog += self._dw_gemm(embed, self.dh_plane, self.e, f"embedder.w{wsuf}")
        Cin = spec.in_dim
        # d(BN_e output) = dh0 W_e, then the embedder BN backward (parameter and/or input gradient)
        prog.append(self._dx_gemm(embed, self.dh_plane, self.de, Cin))
        prog += self._bn_backward("embedder.norm", Cin, self.de, self.x_addr, self.ldx, 0, False, None,
                                  dx=self.dx if self.need_input_grad else None, lddx=_a4(Cin), dxts=0,
                                  sum_twins=True)
        return prog

    # ---- execution --------------------------------------------------------
    def forward(self):
        for f in self.forward_program:
            f()

    def backward(self):
        for f in self.backward_program:
            f()
