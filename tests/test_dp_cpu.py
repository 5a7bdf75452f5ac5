"""Host-side logic of data-parallel FlashSAC on CPU ranks (gloo, world size 2): the
batch-norm partial all-gather layout, mean / max reductions, the collective forms of the
scalar reducer and of the gradient mean (the peer-memory kernels' fallbacks) and row
slicing."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from robolearn_b200.flashsac.dp import DataParallel

        dp = DataParallel()
        T, G, C = 2, 3, 5
        local = torch.arange(T * G * C, dtype=torch.float32).view(T, G, C) + 1000 * rank
        big = torch.zeros(T, world * G, C + 2)  # wider buffer: only the [T][W*G][C] prefix is used
        dp.gather_groups(local, big, T, G, C)
        flat = big.view(-1)[: T * world * G * C].view(T, world * G, C)
        ok = True
        for t in range(T):
            for r in range(world):
                ok &= torch.equal(flat[t, r * G:(r + 1) * G], torch.arange(T * G * C).view(T, G, C)[t] + 1000 * r)
        x = torch.tensor([float(rank + 1), 10.0 * rank])
        dp.all_reduce_mean(x)
        ok &= torch.allclose(x, torch.tensor([1.5, 5.0]))
        y = torch.tensor([float(rank)])
        dp.all_reduce_max(y)
        ok &= y.item() == world - 1
        ok &= dp.row_slice(8) == (4 * rank, 4)
        # scalar reducer (collective form): means, then maxima over an aliasing view, flags
        metrics = torch.tensor([float(rank), 2.0 * rank, 5.0 + rank])
        flag = torch.tensor([rank], dtype=torch.int32)
        dp.scalar_reducer(mean=metrics, max=metrics[2:3])()
        dp.scalar_reducer(max_int=flag)()
        ok &= torch.allclose(metrics, torch.tensor([0.5, 1.0, 6.0]))
        ok &= flag.item() == world - 1
        # gradient mean without peer memory: the collective form, and no peer arenas on gloo

        class Net:
            grads = torch.tensor([1.0 + rank, -2.0 * rank, 4.0, 8.0 * rank])

        net = Net()
        ok &= dp.enable_peer_gradients([net], "cpu", 0) is False and dp.peer_grads is None
        launch = dp.gradient_mean(net)
        ok &= launch.launches == 0
        launch()
        ok &= torch.allclose(net.grads, torch.tensor([1.5, -1.0, 4.0, 4.0]))
        out[rank] = bool(ok)
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(120)
def test_data_parallel_collectives_gloo():
    world = 2
    ctx = mp.get_context("spawn")
    with ctx.Manager() as m:
        out = m.dict()
        port = _free_port()
        procs = [ctx.Process(target=_worker, args=(r, world, port, out)) for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(90)
            assert p.exitcode == 0
        assert dict(out) == {0: True, 1: True}
