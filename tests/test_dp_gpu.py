"""Data-parallel FlashSAC on 2 GPUs against one GPU with the global batch.

Launches tests/_dp_worker.py under torch.distributed.run (one process per GPU, NCCL,
127.0.0.1 rendezvous). After each of two eager updates and one CUDA-graph update whose
graph holds the NCCL collectives, every parameter, batch-norm buffer and the
temperature of the 2-rank learner must match the single-GPU learner at the global
batch: FP32 recipe within 1e-4 relative to each tensor's largest magnitude (batch-norm
buffers with a 1e-3 floor); FP16-operand recipe within 1e-2 in relative L2 norm (the
two runs sum weight gradients in different orders and Adam's first steps amplify that
for near-zero gradients). At config 5's widths (critic 1024 x 3, actor 128 x 2, 512 rows
per rank, FP32 recipe) the gradients of both phases, averaged over the ranks, match the
global batch's within 5e-3 relative L2 per tensor: the two runs sum batch statistics in
different orders, and every ReLU decision that rounding-level differences take the other
way at a pre-activation within rounding of zero moves a 1024-wide layer's gradients by
about 1e-3 (measured: 5.9e-4 relative L2 and 1.1e-2 of the largest element on
encoder.0.w2 after one phase). Parameters are not the measure there: Adam's first steps
turn such differences of near-zero gradients into whole learning-rate steps. Both ranks must hold
bit-identical parameters and report no health flag. Batch-norm statistics and the gradient
means go through the NVLink peer-memory kernels (``RL2_DP_PEER=1``, the default) and, in
one FP32 case, through NCCL all-gathers and all-reduces. ``test_peer_mean_bit_exact``
checks the gradient-mean kernel alone, bit for bit.
Skipped with fewer than two GPUs.
"""

import json
import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("precision,measure,tol,peer,widths", [("fp32", 0, 1e-4, "1", "small"),
                                                               ("fp16", 1, 1e-2, "1", "small"),
                                                               ("fp32", 0, 1e-4, "0", "small"),
                                                               ("fp32", 1, 5e-3, "1", "wide")])
def test_two_rank_update_matches_global_batch(tmp_path, precision, measure, tol, peer, widths):
    out = tmp_path / "dp.json"
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr", "127.0.0.1", "--master-port", str(_free_port()), str(ROOT / "tests" / "_dp_worker.py"),
           str(out), precision, widths]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", RL2_DP_PEER=peer)
    done = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)
    assert done.returncode == 0, done.stdout[-4000:] + done.stderr[-4000:]
    report = json.loads(out.read_text())
    assert report["ranks_identical"]
    assert report["peer"] == (peer == "1")
    assert report["peer_grads"] == (peer == "1")
    assert report["health"] == 0
    for upd in report["updates"]:
        worst = max(upd["errors"].items(), key=lambda kv: kv[1][measure])
        assert worst[1][measure] < tol, (upd["phase"], worst)
        if "metrics_dp" in upd:  # reported metrics reduced over the ranks (scalar reducer)
            for got, want in zip(upd["metrics_dp"], upd["metrics_single"]):
                assert abs(got - want) <= 1e-2 * max(abs(want), 1e-2), (upd["phase"], upd["metrics_dp"],
                                                                         upd["metrics_single"])


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_peer_mean_bit_exact(tmp_path):
    """rl2_peer_mean over 2 ranks: bit-identical to the rank-order sum / world, eager and
    from a captured graph, for arenas from one float4 to a few million floats."""
    out = tmp_path / "mean.json"
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           str(ROOT / "tests" / "_peer_mean_worker.py"), str(out)]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    done = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=300)
    assert done.returncode == 0, done.stdout[-4000:] + done.stderr[-4000:]
    report = json.loads(out.read_text())
    assert report["health"] == 0
    assert report["ok"]
