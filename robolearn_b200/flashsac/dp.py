"""Data-parallel collectives of the FlashSAC learner (one process per GPU).

The global minibatch is split into contiguous per-rank slices: every rank draws the
same global replay indices and policy noise (same seeds) and processes its slice, so
the N-GPU update works on exactly the batch a 1-GPU update at the global size would.
Three exchanges keep the update equal to the global-batch one (reference semantics:
src/robolearn/flashsac/updates.py):

* batch-norm statistics over the global batch (training-mode forward and backward):
  each rank's packed per-32-row-group partials of a layer are all-gathered in one call
  and merged in a fixed rank-major group order by the same kernels as on one GPU, so
  every rank computes bit-identical statistics;
* the gradient arena of each optimised network is averaged (``all_reduce`` AVG) before
  Adam; the fp16 recipe's overflow flags are combined with MAX so every rank skips the
  same steps;
* the actor entropy feeding the temperature step is averaged, and the reported metrics
  are averaged (``critic/max_entropy_bonus``: maximum).

Each rank back-propagates its local loss (mean over its rows), so local gradients are
``world`` times their share of the global gradient; batch-norm backward coefficients
use global means of those local-scaled sums (consistent), and the weight / bias
gradients of batch norm are reduced from LOCAL partials so that the final average is
the global gradient.

Collectives go through ``torch.distributed`` (NCCL on GPUs: AVG / MAX reductions and
all-gather are recorded into the learner's CUDA graphs; gloo on CPU for tests).
"""

from __future__ import annotations

import torch


class DataParallel:
    """Rank / world of the learner's process group and the collectives it issues."""

    def __init__(self, group=None):
        import torch.distributed as dist

        if not dist.is_initialized():
            raise RuntimeError("data-parallel FlashSAC needs an initialised torch.distributed process group")
        self.dist = dist
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.nccl = dist.get_backend(group) == "nccl"

    # ---- reductions -------------------------------------------------------
    def all_reduce_mean(self, t: torch.Tensor) -> None:
        if self.world == 1:
            return
        if self.nccl:
            self.dist.all_reduce(t, op=self.dist.ReduceOp.AVG, group=self.group)
        else:
            self.dist.all_reduce(t, op=self.dist.ReduceOp.SUM, group=self.group)
            t.div_(self.world)

    def all_reduce_max(self, t: torch.Tensor) -> None:
        if self.world > 1:
            self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX, group=self.group)

    # ---- batch-norm partials --------------------------------------------
    def all_gather(self, local: torch.Tensor, out: torch.Tensor) -> None:
        """out = [rank 0's local | rank 1's local | ...] (flat, contiguous). Batch-norm layers
        gather their packed per-group partials in one call; the merge kernels address the
        rank-major result directly."""
        self.dist.all_gather_into_tensor(out.view(-1), local.view(-1), group=self.group)

    def gather_groups(self, local: torch.Tensor, out: torch.Tensor, twins: int, groups: int, cols: int) -> None:
        """local [twins][groups][cols] (flat prefix) -> out [twins][world * groups][cols] (flat prefix)."""
        n = groups * cols
        lo = local.view(-1)
        go = out.view(-1)
        for t in range(twins):
            self.dist.all_gather_into_tensor(go[t * self.world * n:(t + 1) * self.world * n], lo[t * n:(t + 1) * n],
                                             group=self.group)

    def row_slice(self, global_rows: int) -> tuple[int, int]:
        """(first row, rows) of this rank's contiguous slice of a global batch."""
        if global_rows % self.world:
            raise ValueError("the global batch must split evenly over the ranks")
        per = global_rows // self.world
        return self.rank * per, per
