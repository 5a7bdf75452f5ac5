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
* the gradient arena of each optimised network is averaged before Adam: on NVLink by one
  peer-memory kernel per optimizer step over arenas held in symmetric memory
  (``PeerGradients``: each rank sums its share of the arena over the ranks in rank order
  and stores the mean into every rank's arena), otherwise by ``all_reduce`` AVG; the fp16
  recipe's overflow flags are combined with MAX so every rank skips the same steps;
* the actor entropy feeding the temperature step is averaged, and the reported metrics
  are averaged (``critic/max_entropy_bonus``: maximum); on NVLink these scalars and the
  overflow flags travel through one peer-memory kernel per sync point
  (``scalar_reducer``) instead of NCCL calls.

Each rank back-propagates its local loss (mean over its rows), so local gradients are
``world`` times their share of the global gradient; batch-norm backward coefficients
use global means of those local-scaled sums (consistent), and the weight / bias
gradients of batch norm are reduced from LOCAL partials so that the final average is
the global gradient.

Collectives go through ``torch.distributed`` (NCCL on GPUs: AVG / MAX reductions and
all-gather are recorded into the learner's CUDA graphs; gloo on CPU for tests). On
NVLink-connected GPUs the batch-norm exchanges instead run inside one kernel per sync
point over peer memory (``PeerExchange``): the all-gather's launch and protocol latency
was most of the exchange time for these kilobyte-sized partials.
"""

from __future__ import annotations

import ctypes

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
        self.peer: PeerExchange | None = None
        self.peer_grads: PeerGradients | None = None

    def enable_peer(self, device, slots: int, max_cols: int, health_ptr: int, timeout_s: float = 10.0) -> bool:
        """Exchange batch-norm statistics through NVLink peer memory instead of NCCL all-gathers
        (one kernel per sync point). Collective; needs NCCL ranks on GPUs of one node with
        symmetric memory. ``RL2_DP_PEER=0`` keeps the all-gather path. Returns whether it is on."""
        import os

        if self.world == 1 or not self.nccl or os.environ.get("RL2_DP_PEER", "1") == "0":
            return False
        self.peer = PeerExchange(self, slots, max_cols, device, health_ptr=health_ptr, timeout_s=timeout_s)
        return True

    def enable_peer_gradients(self, nets, device, health_ptr: int, timeout_s: float = 10.0) -> bool:
        """Move the gradient arenas of ``nets`` into NVLink symmetric memory and average them
        with one peer-memory kernel per optimizer step (``gradient_mean``) instead of NCCL
        all-reduces. Collective; call before any launch list takes the arenas' addresses.
        Needs the peer exchange; ``RL2_DP_PEER_GRAD=0`` keeps NCCL. Returns whether it is on."""
        import os

        if self.peer is None or os.environ.get("RL2_DP_PEER_GRAD", "1") == "0":
            return False
        self.peer_grads = PeerGradients(self, nets, device, health_ptr=health_ptr, timeout_s=timeout_s)
        return True

    def gradient_mean(self, net):
        """A launch (callable, graph-capturable) that replaces ``net.grads`` by its mean over
        the ranks: one peer-memory kernel (``rl2_peer_mean``) when the arenas are in symmetric
        memory, else an NCCL / gloo all-reduce. ``launch.launches`` counts this library's kernels."""
        pg = self.peer_grads
        if pg is not None and pg.holds(net):
            return pg.reducer(net)

        def launch():
            self.all_reduce_mean(net.grads)

        launch.launches = 0
        return launch

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

    def scalar_reducer(self, mean: torch.Tensor | None = None, max: torch.Tensor | None = None,
                       max_int: torch.Tensor | None = None):
        """A launch (callable, graph-capturable) that averages ``mean`` over the ranks and
        replaces ``max`` (float) and ``max_int`` (int32 flags) by their maxima, the maxima
        last (``max`` may be a view into ``mean``). One peer-memory kernel (``rl2_peer_reduce``)
        when the peer exchange is on and a slot is left, else the same through collectives."""
        views = [v for v in (mean, max, max_int) if v is not None]
        if self.peer is not None and sum(v.numel() for v in views) <= 64:
            ex = self.peer.try_slot(32, 1)
            if ex is not None:
                from .. import _native as N

                lib = N.load()
                args = N.PeerReduceArgs(mean=N.addr(mean), n_mean=mean.numel() if mean is not None else 0,
                                        max=N.addr(max), n_max=max.numel() if max is not None else 0,
                                        max_int=N.addr(max_int), n_max_int=max_int.numel() if max_int is not None else 0)

                def launch():
                    N.check(lib.rl2_peer_reduce(ctypes.byref(args), ctypes.byref(ex), N.stream_ptr()),
                            "data-parallel scalar reduction")

                launch.keep = (args, ex, views)
                launch.launches = 1
                return launch

        def launch():
            for v in (max, max_int):
                if v is not None:
                    self.all_reduce_max(v)
            if mean is not None:
                self.all_reduce_mean(mean)

        launch.launches = 0
        return launch

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


class PeerExchange:
    """NVLink peer-memory slots for the data-parallel batch-norm kernels.

    One symmetric buffer per rank (``torch.distributed._symmetric_memory``: every rank
    maps every other rank's buffer), split into ``slots`` equal slots, one per batch-norm
    sync point of the learner's programs (assigned in program-construction order, the
    same on every rank). A slot holds the ranks' per-column entries and per-(column
    slab, rank) epoch flags; epochs live in a local device counter per slot.
    """

    def __init__(self, dp: DataParallel, slots: int, max_cols: int, device, twins: int = 2, health_ptr: int = 0,
                 timeout_s: float = 10.0):
        import torch.distributed._symmetric_memory as symm

        from .. import _native as N

        lib = N.load()
        W = dp.world
        align = lambda b: (int(b) + 255) // 256 * 256  # noqa: E731
        self.data_bytes = align(lib.rl2_syncbn_slot_data_bytes(W, twins, max_cols))
        self.flag_bytes = align(lib.rl2_syncbn_slot_flag_bytes(W, twins, max_cols))
        self.slot_bytes = self.data_bytes + self.flag_bytes
        self.slots, self.max_cols, self.twins, self.timeout_s = slots, max_cols, twins, timeout_s
        self.buf = symm.empty(slots * self.slot_bytes // 4, dtype=torch.float32, device=device)
        self.buf.zero_()
        group = dp.group if dp.group is not None else dp.dist.group.WORLD
        self.handle = symm.rendezvous(self.buf, group)
        torch.cuda.synchronize(device)
        dp.dist.barrier(group=dp.group)
        self.ptrs = list(self.handle.buffer_ptrs)
        self.world, self.rank = W, dp.rank
        self.device = device
        self.epochs = torch.zeros(2 * slots, dtype=torch.int32, device=device)
        self.health_ptr = health_ptr or None
        self.next = 0
        self._keep: list = []

    def try_slot(self, cols: int, twins: int):
        """``slot`` or None when every slot is taken or the slots are narrower."""
        if self.next >= self.slots or cols > self.max_cols or twins > self.twins:
            return None
        return self.slot(cols, twins)

    def slot(self, cols: int, twins: int):
        """Exchange arguments of the next free slot (host struct; keep it alive while in use)."""
        from .. import _native as N

        if self.next >= self.slots:
            raise RuntimeError("peer exchange: all batch-norm slots are in use")
        if cols > self.max_cols or twins > self.twins:
            raise ValueError("peer exchange: a batch-norm layer is wider than the slots")
        s = self.next
        self.next += 1
        base = s * self.slot_bytes
        data = torch.tensor([p + base for p in self.ptrs], dtype=torch.int64, device=self.device)
        flags = torch.tensor([p + base + self.data_bytes for p in self.ptrs], dtype=torch.int64, device=self.device)
        ex = N.SyncBNExchange(peer_data=data.data_ptr(), peer_flags=flags.data_ptr(),
                              epoch=self.epochs.data_ptr() + 8 * s, world=self.world, rank=self.rank,
                              health=self.health_ptr, timeout_s=self.timeout_s)
        self._keep += [data, flags, ex]
        return ex


class PeerGradients:
    """Gradient arenas of the optimised networks in one NVLink symmetric buffer.

    Layout of every rank's buffer: the networks' arenas (each padded to 64 floats), then
    ``sites`` flag regions of ``rl2_peer_mean_flag_bytes(world)`` bytes, one per call site
    of ``reducer`` (assigned in program-construction order, the same on every rank), each
    with its own two-word epoch counter on this rank. ``net.grads`` becomes a view of the
    buffer, so every launch list built afterwards addresses the shared arena.
    """

    def __init__(self, dp: DataParallel, nets, device, health_ptr: int = 0, timeout_s: float = 10.0,
                 sites: int = 16):
        import torch.distributed._symmetric_memory as symm

        from .. import _native as N

        lib = N.load()
        W = dp.world
        self.flag_bytes = (int(lib.rl2_peer_mean_flag_bytes(W)) + 255) // 256 * 256
        self.offsets = {}
        off = 0
        for net in nets:
            self.offsets[id(net)] = (off, net.size)
            off += (net.size + 63) // 64 * 64
        self.flag_base = 4 * off
        self.sites = sites
        self.buf = symm.empty(off + sites * self.flag_bytes // 4, dtype=torch.float32, device=device)
        self.buf.zero_()
        group = dp.group if dp.group is not None else dp.dist.group.WORLD
        self.handle = symm.rendezvous(self.buf, group)
        for net in nets:
            o, n = self.offsets[id(net)]
            self.buf[o:o + n].copy_(net.grads)
            net.grads = self.buf[o:o + n]
        torch.cuda.synchronize(device)
        dp.dist.barrier(group=dp.group)
        self.ptrs = list(self.handle.buffer_ptrs)
        self.world, self.rank, self.device = W, dp.rank, device
        self.epochs = torch.zeros(2 * sites, dtype=torch.int32, device=device)
        self.health_ptr = health_ptr or None
        self.timeout_s = timeout_s
        self.next = 0
        self._keep: list = []

    def holds(self, net) -> bool:
        return id(net) in self.offsets and net.grads.data_ptr() == self.buf.data_ptr() + 4 * self.offsets[id(net)][0]

    def reducer(self, net):
        """Launch averaging ``net.grads`` over the ranks (one ``rl2_peer_mean`` kernel)."""
        from .. import _native as N

        if self.next >= self.sites:
            raise RuntimeError("peer gradients: all call sites are in use")
        s = self.next
        self.next += 1
        o, n = self.offsets[id(net)]
        data = torch.tensor([p + 4 * o for p in self.ptrs], dtype=torch.int64, device=self.device)
        flags = torch.tensor([p + self.flag_base + s * self.flag_bytes for p in self.ptrs], dtype=torch.int64,
                             device=self.device)
        ex = N.SyncBNExchange(peer_data=data.data_ptr(), peer_flags=flags.data_ptr(),
                              epoch=self.epochs.data_ptr() + 8 * s, world=self.world, rank=self.rank,
                              health=self.health_ptr, timeout_s=self.timeout_s)
        lib = N.load()
        ref = ctypes.byref(ex)

        def launch():
            N.check(lib.rl2_peer_mean(n, ref, N.stream_ptr()), "data-parallel gradient mean")

        launch.keep = (data, flags, ex)
        launch.launches = 1
        return launch
