"""The allocation-free critic objective (``rl2_critic_objective_noalloc``) through the C ABI.

It exists for callers that cannot allocate device memory where they run the objective
(a real-time control loop that must not stall in the driver's allocator, or a host
whose device memory belongs to another framework's pool): its partials and counter
live in a library-owned device array instead of a caller workspace. Checked here: two
calls in a row give the same loss, max entropy bonus, head-bias gradient, projected
target and logits gradient as ``rl2_critic_objective`` with a caller workspace, and
oversized requests are rejected. This file is collected last so that a failure here
does not hide the rest of the suite.
"""

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

from robolearn_b200 import _native as N  # noqa: E402
from robolearn_b200.categorical import support  # noqa: E402


def _args(B, bins, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    dev = "cuda"
    t = {
        "tl": torch.log_softmax(torch.randn(2, 2 * B, bins, device=dev, generator=g), -1).contiguous(),
        "ol": torch.randn(2, 2 * B, bins, device=dev, generator=g),
        "r": torch.randn(B, device=dev, generator=g),
        "d": (torch.rand(B, device=dev, generator=g) < 0.05).float(),
        "disc": torch.full((B,), 0.99, device=dev),
        "nlp": torch.randn(B, device=dev, generator=g),
        "alpha": torch.tensor([0.01], device=dev),
        "z": torch.from_numpy(support(bins, -10.0, 10.0)).to(dev),
        "loss": torch.zeros(1, device=dev), "ent": torch.zeros(1, device=dev),
        "bias": torch.zeros(2, bins, device=dev), "target": torch.zeros(B, bins, device=dev),
        "dl": torch.zeros(2, 2 * B, bins, device=dev),
    }
    a = N.CriticObjectiveArgs(
        target_logits=t["tl"].data_ptr(), target_row_stride=bins, target_twin_stride=2 * B * bins,
        target_row_offset=B, online_logits=t["ol"].data_ptr(), online_row_stride=bins,
        online_twin_stride=2 * B * bins, reward=t["r"].data_ptr(), terminated=t["d"].data_ptr(),
        discount=t["disc"].data_ptr(), next_log_pi=t["nlp"].data_ptr(), alpha=t["alpha"].data_ptr(),
        support=t["z"].data_ptr(), min_v=-10.0, max_v=10.0, bins=bins, batch=B, loss_weight=1.0 / (2 * B),
        dlogits=t["dl"].data_ptr(), dlogits_row_stride=bins, dlogits_twin_stride=2 * B * bins,
        target_out=t["target"].data_ptr(), target_out_row_stride=bins, loss_out=t["loss"].data_ptr(),
        max_entropy_out=t["ent"].data_ptr(), bias_grad_out=t["bias"].data_ptr())
    return a, t


def _outputs(t):
    return {k: t[k].cpu().numpy().copy() for k in ("loss", "ent", "bias", "target", "dl")}


@pytest.mark.parametrize("B,bins", [(4096, 101), (777, 51)])
def test_no_alloc_matches_workspace_entry_point_twice(B, bins):
    lib = N.load()
    stream = torch.cuda.current_stream().cuda_stream
    # reference: the existing entry point with a caller-provided workspace and counter
    a, t = _args(B, bins, seed=B)
    ws = torch.zeros(lib.rl2_categorical_workspace_floats(B, bins), device="cuda")
    counter = torch.zeros(lib.rl2_categorical_counter_words(B, bins), dtype=torch.int32, device="cuda")
    a.workspace, a.counter = ws.data_ptr(), counter.data_ptr()
    assert lib.rl2_critic_objective(ctypes.byref(a), stream) == 0
    torch.cuda.synchronize()
    expected = _outputs(t)
    for call in range(2):
        b, u = _args(B, bins, seed=B)
        b.workspace, b.counter = None, None
        assert lib.rl2_critic_objective_noalloc(ctypes.byref(b), stream) == 0, lib.rl2_last_error()
        torch.cuda.synchronize()
        got = _outputs(u)
        for k, v in expected.items():
            np.testing.assert_allclose(got[k], v, rtol=1e-6, atol=1e-9, err_msg=f"call {call} {k}")


def test_no_alloc_rejects_sizes_beyond_its_limit():
    lib = N.load()
    a, _ = _args(16, 11, seed=1)
    a.batch = 65537
    assert lib.rl2_critic_objective_noalloc(ctypes.byref(a), torch.cuda.current_stream().cuda_stream) == -1
    assert b"batch must be in [1, 65536]" in lib.rl2_last_error()


def test_no_alloc_rejects_a_stream_of_another_device():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    lib = N.load()
    a, _ = _args(16, 11, seed=1)
    with torch.cuda.device(1):
        other = torch.cuda.Stream()
    assert lib.rl2_critic_objective_noalloc(ctypes.byref(a), other.cuda_stream) == -1
    assert b"belongs to device 1" in lib.rl2_last_error()
