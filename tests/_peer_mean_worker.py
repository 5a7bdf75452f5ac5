"""Worker of tests/test_dp_gpu.py::test_peer_mean_bit_exact (torch.distributed.run, one
process per GPU).

Arenas of several sizes (a single float4, sizes that leave most blocks without work,
ragged splits over the ranks and blocks, a few million floats) live in one symmetric
buffer (``PeerGradients``). Each is filled with rank-dependent values, averaged by
``rl2_peer_mean`` (eagerly, then twice from a captured CUDA graph with fresh inputs
between the replays) and compared bit for bit with the mean that every rank computes
from an all-gather of the inputs: the sum in rank order divided by the world size.
Writes {"ok": ..., "health": ...} to the JSON path given.
"""

import datetime
import json
import os
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from robolearn_b200.flashsac.dp import DataParallel  # noqa: E402

SIZES = [4, 12, 148 * 4 * 2 + 8, 40004, 3 * 1024 * 1024 + 36]


class Arena:
    def __init__(self, size, device):
        self.size = size
        self.grads = torch.zeros(size, dtype=torch.float32, device=device)


def fill(arenas, rank, salt):
    for i, a in enumerate(arenas):
        g = torch.Generator(device=a.grads.device).manual_seed(1000 * salt + 10 * i + rank)
        x = torch.randn(a.size, device=a.grads.device, generator=g)
        # wide magnitudes so that the order of the sum matters at the last bit
        x *= torch.exp2(torch.randint(-20, 20, (a.size,), device=a.grads.device, generator=g).float())
        a.grads.copy_(x)


def expected(arenas, world):
    out = []
    for a in arenas:
        parts = [torch.empty_like(a.grads) for _ in range(world)]
        dist.all_gather(parts, a.grads)
        acc = parts[0].clone()
        for q in range(1, world):
            acc = acc + parts[q]
        out.append(acc / float(world))
    return out


def main():
    out_path = sys.argv[1]
    local = int(os.environ["LOCAL_RANK"])
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)
    dp = DataParallel()
    health = torch.zeros(1, dtype=torch.int32, device=device)
    assert dp.enable_peer(device, 4, 32, health.data_ptr())
    arenas = [Arena(n, device) for n in SIZES]
    assert dp.enable_peer_gradients(arenas, device, health.data_ptr())
    launches = [dp.gradient_mean(a) for a in arenas]
    ok = True
    # eager
    fill(arenas, dp.rank, 0)
    want = expected(arenas, dp.world)
    for f in launches:
        f()
    torch.cuda.synchronize()
    for a, w in zip(arenas, want):
        ok &= bool(torch.equal(a.grads.view(torch.int32), w.view(torch.int32)))
    # captured, replayed twice with fresh inputs
    graph = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream(device)
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.graph(graph, stream=s):
        for f in launches:
            f()
    for salt in (1, 2):
        fill(arenas, dp.rank, salt)
        want = expected(arenas, dp.world)
        torch.cuda.synchronize()
        dist.barrier()
        graph.replay()
        torch.cuda.synchronize()
        for a, w in zip(arenas, want):
            ok &= bool(torch.equal(a.grads.view(torch.int32), w.view(torch.int32)))
    flag = torch.tensor([0 if ok else 1], device=device)
    dist.all_reduce(flag, op=dist.ReduceOp.MAX)
    h = torch.tensor([int(health.item())], device=device)
    dist.all_reduce(h, op=dist.ReduceOp.MAX)
    del graph
    if dp.rank == 0:
        Path(out_path).write_text(json.dumps({"ok": int(flag.item()) == 0, "health": int(h.item())}))
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
