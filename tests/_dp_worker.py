"""Worker of tests/test_dp_gpu.py (run under torch.distributed.run, one process per GPU).

Every rank runs data-parallel FlashSAC updates with a per-rank batch of B; rank 0 also
runs a single-GPU learner with the global batch world * B on the same replay, indices
and noise, and writes the largest relative differences (per tensor) to a JSON file.
The third update replays a CUDA graph that contains the NCCL collectives (and, with the
peer exchange on, the batch-norm kernels that exchange statistics over NVLink). With
config 5's widths ("wide") the first two phases stop at the gradients, which are
compared (averaged over the ranks) with the global batch's.
"""

import datetime
import json
import os
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from robolearn_b200.flashsac.config import FlashSACConfig  # noqa: E402
from robolearn_b200.flashsac.dp import DataParallel  # noqa: E402
from robolearn_b200.flashsac.learner import Learner  # noqa: E402
from robolearn_b200.flashsac.replay import DeviceReplay  # noqa: E402
from robolearn_b200.flashsac.sampling import sampling_program  # noqa: E402

OBS, ACT, B, CAP = 17, 5, 64, 4096


# network widths: "small" (critic 64 x 1, actor 32 x 1) or "wide" (config 5's critic
# 1024 x 3 and actor 128 x 2)
WIDTHS = {"small": dict(critic_hidden_dim=64, critic_num_blocks=1, actor_hidden_dim=32, actor_num_blocks=1),
          "wide": dict(critic_hidden_dim=1024, critic_num_blocks=3, actor_hidden_dim=128, actor_num_blocks=2)}


def make(batch: int, dp, device, precision: str, widths: str = "small"):
    cfg = FlashSACConfig(device=str(device), sample_batch_size=batch, critic_num_bins=51, critic_min_v=-10.0,
                         critic_max_v=10.0, n_step=1, buffer_max_length=CAP, buffer_min_length=256,
                         dense_precision=precision, seed=0, learning_rate_decay_step=1000, **WIDTHS[widths])
    L = Learner(OBS, OBS, ACT, cfg, device, dp=dp)
    R = DeviceReplay(OBS, ACT, 256, CAP, 1, 0.99, 256, device, seed=0)
    g = torch.Generator(device=device).manual_seed(7)
    R.observation.copy_(torch.randn(CAP, OBS, device=device, generator=g))
    R.next_observation.copy_(torch.randn(CAP, OBS, device=device, generator=g))
    R.action.uniform_(-1, 1, generator=g)
    R.reward.copy_(torch.randn(CAP, device=device, generator=g))
    R.terminated.copy_((torch.rand(CAP, device=device, generator=g) < 0.05).float())
    R.discount.fill_(0.99)
    R.counters.copy_(torch.tensor([0, 0, CAP], device=device))
    R._host_count = CAP
    return L, R, sampling_program(L, R, seed=0)


def state(L) -> dict:
    out = {}
    for tag, net in (("actor", L.actor), ("critic", L.critic), ("target", L.target)):
        for k, v in net.state_dict().items():
            out[f"{tag}.{k}"] = v.detach().cpu().numpy().astype(np.float64)
    out["log_temp"] = L.log_temp.cpu().numpy().astype(np.float64)
    return out


def grads(L) -> dict:
    out = {}
    for tag, net in (("actor", L.actor), ("critic", L.critic)):
        for k in net.param_names:
            off, shape = net.offsets[k], net.shapes[k]
            n = int(np.prod(shape))
            out[f"{tag}.{k}"] = net.grads[off:off + n].detach().cpu().numpy().astype(np.float64)
    return out


def compare(a: dict, b: dict) -> dict:
    """Per tensor: [max |a - b| / max |b| (buffers floored at 1e-3), ||a - b|| / ||b||]."""
    res = {}
    for k in a:
        floor = 1e-3 if k.endswith(("running_mean", "running_var")) else 1e-12
        rel_max = float(np.abs(a[k] - b[k]).max() / max(np.abs(b[k]).max(), floor))
        rel_l2 = float(np.linalg.norm(a[k] - b[k]) / max(np.linalg.norm(b[k]), floor))
        res[k] = [rel_max, rel_l2]
    return res


def main():
    out_path = sys.argv[1]
    precision = sys.argv[2] if len(sys.argv) > 2 else "fp32"
    widths = sys.argv[3] if len(sys.argv) > 3 else "small"
    rows = B if widths == "small" else 8 * B  # per rank
    local = int(os.environ["LOCAL_RANK"])
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)
    dp = DataParallel()
    L, R, feed = make(rows, dp, device, precision, widths)
    single = make(rows * dp.world, None, device, precision, widths) if dp.rank == 0 else None
    torch.cuda.synchronize()
    dist.barrier()  # rank 0 built a second learner: start the updates together
    report = {"world": dp.world, "precision": precision, "peer": dp.peer is not None,
              "peer_grads": dp.peer_grads is not None, "updates": []}
    phases = (True, False)
    wide = widths == "wide"
    for phase in phases:
        for f in feed:
            f()
        # wide networks: gradients of the phase (ranks' local gradients averaged here) against
        # the global batch's, since Adam's first steps turn rounding-level differences of
        # near-zero gradients into full learning-rate steps
        L.run(phase, apply_optimizer=not wide)
        if single:
            for f in single[2]:
                f()
            single[0].run(phase, apply_optimizer=not wide)
        torch.cuda.synchronize()
        if wide:
            for net in (L.actor, L.critic):
                dist.all_reduce(net.grads, op=dist.ReduceOp.AVG)
            torch.cuda.synchronize()
        if single:
            got, want = (grads(L), grads(single[0])) if wide else (state(L), state(single[0]))
            report["updates"].append({"phase": phase, "errors": compare(got, want),
                                      "metrics_dp": L.metrics.cpu().tolist(),
                                      "metrics_single": single[0].metrics.cpu().tolist()})
    # captured update with the collectives inside the graph
    graph = L.capture(True, pre=feed)
    g_single = single[0].capture(True, pre=single[2]) if single else None
    graph.replay()
    if g_single is not None:
        g_single.replay()
    torch.cuda.synchronize()
    if single and not wide:
        report["updates"].append({"phase": "captured", "errors": compare(state(L), state(single[0]))})
    # every rank holds the same parameters
    flat = torch.cat([L.actor.params, L.critic.params, L.target.params, L.log_temp])
    ref = flat.clone()
    dist.broadcast(ref, 0)
    same = torch.equal(flat, ref)
    ok = torch.tensor([1 if same else 0], device=device)
    dist.all_reduce(ok, op=dist.ReduceOp.MIN)
    report["ranks_identical"] = bool(ok.item())
    health = L.health.clone()
    dist.all_reduce(health, op=dist.ReduceOp.MAX)
    report["health"] = int(health.item())
    del graph, g_single
    torch.cuda.synchronize()
    dist.barrier()
    dist.destroy_process_group()
    if single:
        Path(out_path).write_text(json.dumps(report))


if __name__ == "__main__":
    main()
