"""Host wrapper of the fused categorical critic objective (``rl2_critic_objective``)."""

from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import _native as N


def support(bins: int, min_v: float, max_v: float) -> np.ndarray:
    """Atom values with Torch's float32 ``linspace`` rule (``src/robolearn/flashsac/layers.py:289-292``).

    Torch evaluates ``start + step * i`` for the first half and ``end - step * (n - 1 - i)``
    for the second, each fused (one rounding), with ``step`` rounded to float32.
    """
    start, end = float(np.float32(min_v)), float(np.float32(max_v))
    step = float(np.float32(np.float32(end - start) / np.float32(bins - 1)))
    half = bins // 2
    vals = [start + step * i if i < half else end - step * (bins - 1 - i) for i in range(bins)]
    return np.asarray(vals, dtype=np.float64).astype(np.float32)


class CriticObjective:
    """Persistent workspace for one (batch, bins) critic objective launch."""

    def __init__(self, batch: int, bins: int, min_v: float, max_v: float, device="cuda"):
        self.batch, self.bins, self.min_v, self.max_v = batch, bins, float(min_v), float(max_v)
        lib = N.load()
        self._lib = lib
        self.workspace = torch.zeros(lib.rl2_categorical_workspace_floats(batch, bins), device=device)
        self.counter = torch.zeros(lib.rl2_categorical_counter_words(batch, bins), dtype=torch.int32, device=device)
        self.support = torch.from_numpy(support(bins, min_v, max_v)).to(device)

    def run(self, *, target_logits, target_row_stride, target_twin_stride, target_row_offset, online_logits,
            online_row_stride, online_twin_stride, reward, terminated, discount, next_log_pi, alpha,
            loss_weight, loss_out, max_entropy_out, bias_grad_out=None, bias_grad_accumulate=False,
            dlogits=None, dlogits_row_stride=0, dlogits_twin_stride=0, d16=None, d16_row_stride=0,
            d16_twin_stride=0, d16_scale=None, d_hi=None, d_lo=None, dplane_row_stride=0, dplane_twin_stride=0,
            target_out=None, target_out_row_stride=0, health=None, stream=None) -> None:
        a = N.CriticObjectiveArgs(
            target_logits=N.ptr(target_logits), target_row_stride=target_row_stride,
            target_twin_stride=target_twin_stride, target_row_offset=target_row_offset,
            online_logits=N.ptr(online_logits), online_row_stride=online_row_stride,
            online_twin_stride=online_twin_stride, reward=N.ptr(reward), terminated=N.ptr(terminated),
            discount=N.ptr(discount), next_log_pi=N.ptr(next_log_pi), alpha=N.ptr(alpha),
            support=N.ptr(self.support), min_v=self.min_v, max_v=self.max_v, bins=self.bins, batch=self.batch,
            loss_weight=loss_weight, dlogits=N.ptr(dlogits), dlogits_row_stride=dlogits_row_stride,
            dlogits_twin_stride=dlogits_twin_stride, d16=N.ptr(d16), d16_row_stride=d16_row_stride,
            d16_twin_stride=d16_twin_stride, d16_scale=N.ptr(d16_scale), d_hi=N.ptr(d_hi), d_lo=N.ptr(d_lo),
            dplane_row_stride=dplane_row_stride, dplane_twin_stride=dplane_twin_stride,
            target_out=N.ptr(target_out), target_out_row_stride=target_out_row_stride,
            workspace=N.ptr(self.workspace), counter=N.ptr(self.counter), loss_out=N.ptr(loss_out),
            max_entropy_out=N.ptr(max_entropy_out), bias_grad_out=N.ptr(bias_grad_out),
            bias_grad_accumulate=int(bias_grad_accumulate), health=N.ptr(health),
        )
        N.check(self._lib.rl2_critic_objective(ctypes.byref(a), N.stream_ptr(stream)), "critic objective")
