"""Replay row of the hot path: bit-exact index sampling (against the numpy Philox
restatement of the device sampler), bit-exact fused gather, reward normalisation,
and the n-step ingest against the reference's known-answer timeline
(``tests/test_flashsac.py:197-231`` in the reference, fixture ``replay_nstep.npz``)."""

import ctypes

import numpy as np
import pytest
import torch

from oracle import philox_np
from tests import _golden as G

pytestmark = pytest.mark.gpu

from robolearn_b200 import _native as N  # noqa: E402
from robolearn_b200.flashsac.replay import DeviceReplay  # noqa: E402


@pytest.mark.parametrize("n,batch,epoch", [(65536, 4096, 0), (1000003, 257, 5), (3, 17, 2**33 + 7)])
def test_indices_bit_exact(n, batch, epoch):
    lib = N.load()
    idx = torch.zeros(batch, dtype=torch.int32, device="cuda")
    ep = torch.tensor([epoch], dtype=torch.int64, device="cuda")
    seed = 0x1234_5678_9ABC_DEF0
    assert lib.rl2_replay_sample(seed, ep.data_ptr(), None, n, batch, idx.data_ptr(), None,
                                 torch.cuda.current_stream().cuda_stream) == 0
    expect = philox_np.replay_indices(seed, epoch, n, batch)
    assert idx.cpu().tolist() == expect


def test_gather_bit_exact_and_reward_normalisation():
    from robolearn_b200.flashsac.config import FlashSACConfig
    from robolearn_b200.flashsac.learner import Learner
    from robolearn_b200.flashsac.sampling import replay_indices, sampling_program

    cfg = FlashSACConfig(device="cuda", sample_batch_size=64, actor_hidden_dim=16, critic_hidden_dim=16,
                         actor_num_blocks=1, critic_num_blocks=1, critic_num_bins=11, buffer_max_length=512,
                         buffer_min_length=64, n_step=1)
    L = Learner(7, 9, 3, cfg, "cuda")
    R = DeviceReplay(9, 3, 8, 512, 1, 0.99, 64, "cuda")
    g = torch.Generator(device="cuda").manual_seed(3)
    for t in (R.observation, R.next_observation, R.action, R.reward, R.terminated, R.discount):
        t.copy_(torch.randn(t.shape, device="cuda", generator=g))
    R.counters.copy_(torch.tensor([0, 0, 300], device="cuda"))
    state = torch.tensor([0.0, 2.5, 10.0, 30.0], device="cuda")  # mean, var, count, G_r_max
    for f in sampling_program(L, R, reward_state=state, g_max=5.0, noise=False):
        f()
    torch.cuda.synchronize()
    idx = replay_indices(L).long()
    assert int(idx.max()) < 300
    B = 64
    assert torch.equal(L.critic_x[:B, :9], R.observation[idx])
    assert torch.equal(L.critic_x[:B, 9:12], R.action[idx])
    assert torch.equal(L.critic_x[B:, :9], R.next_observation[idx])
    assert torch.equal(L.critic_x_pi[:B, :9], R.observation[idx])
    assert torch.equal(L.actor_x[:B, :7], R.observation[idx][:, :7])
    assert torch.equal(L.actor_x[B:, :7], R.next_observation[idx][:, :7])
    assert torch.equal(L.terminated, R.terminated[idx])
    assert torch.equal(L.discount, R.discount[idx])
    den = max(np.sqrt(np.float32(2.5) + np.float32(1e-8)), np.float32(30.0) / np.float32(5.0))
    np.testing.assert_allclose(L.reward.cpu().numpy(), R.reward[idx].cpu().numpy() / den, rtol=1e-6)


def test_n_step_ingest_matches_reference_timeline():
    g = G.load("replay_nstep.npz")
    R = DeviceReplay(1, 1, 3, 16, 3, 0.5, 3, "cuda")
    for step in range(3):
        s = {k[len(f"step{step}."):]: v for k, v in g.items() if k.startswith(f"step{step}.")}
        R.add(*(torch.as_tensor(s[k], device="cuda") for k in
                ("observation", "action", "reward", "terminated", "truncated", "next_observation")))
    torch.cuda.synchronize()
    assert len(R) == 3
    for key, buf in (("reward", R.reward), ("terminated", R.terminated), ("truncated", R.truncated),
                     ("discount", R.discount)):
        np.testing.assert_array_equal(buf[:3].cpu().numpy(), g[f"sample.{key}"].reshape(-1))
    np.testing.assert_array_equal(R.next_observation[:3].cpu().numpy(), g["sample.next_observation"])
    np.testing.assert_array_equal(R.observation[:3].cpu().numpy(), g["sample.observation"])
