"""The reference-facing ``FlashSAC`` agent on the GPU.

* ``act`` (eval-mode actor forward + fused policy kernel) against the CPU oracle's
  actor forward from the same weights: deterministic actions = tanh(mean), training
  actions = tanh(mean + std * cached noise), within the FP32 recipe tolerance 1e-4.
* observe -> ready -> update: both phases return the reference's metric keys with
  finite values; ``tensor_metrics=True`` returns device scalars.
* save -> load into a fresh agent restores parameters, BN buffers, Adam moments, step
  counters, temperature and reward statistics; replay save/load round trips.
"""

import numpy as np
import pytest
import torch

from oracle import flashsac_np as fs

pytestmark = pytest.mark.gpu

from robolearn_b200.flashsac.agent import FlashSAC  # noqa: E402
from robolearn_b200.flashsac.config import FlashSACConfig  # noqa: E402

OBS, ACT, ENVS = 11, 3, 32


def _cfg(**kw):
    base = dict(device="cuda:0", buffer_max_length=512, buffer_min_length=96, sample_batch_size=64,
                actor_hidden_dim=32, actor_num_blocks=1, critic_hidden_dim=32, critic_num_blocks=1,
                critic_num_bins=21, n_step=2, dense_precision="fp32", seed=3)
    base.update(kw)
    return FlashSACConfig(**base)


def _dims(agent) -> fs.Dims:
    c = agent._cfg
    return fs.Dims(obs=OBS, act=ACT, actor_hidden=c.actor_hidden_dim, actor_blocks=c.actor_num_blocks,
                   critic_hidden=c.critic_hidden_dim, critic_blocks=c.critic_num_blocks, bins=c.critic_num_bins,
                   min_v=c.critic_min_v, max_v=c.critic_max_v)


def _fill(agent, steps: int, seed: int = 0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    obs = torch.randn(ENVS, OBS, device="cuda", generator=g)
    for _ in range(steps):
        act = agent.act(obs)
        nxt = torch.randn(ENVS, OBS, device="cuda", generator=g)
        rew = torch.randn(ENVS, device="cuda", generator=g)
        term = (torch.rand(ENVS, device="cuda", generator=g) < 0.05).float()
        agent.observe(obs, act, rew, term, torch.zeros(ENVS, device="cuda"), nxt)
        obs = nxt


def _oracle_actions(agent, obs: torch.Tensor, noise: np.ndarray) -> np.ndarray:
    p = {k: v.cpu().numpy() for k, v in agent.learner.actor.state_dict().items()}
    a, _, _, _ = fs.actor_forward(p, _dims(agent), obs.cpu().numpy(), noise, training=False)
    return a


def test_act_matches_oracle_eval_forward():
    agent = FlashSAC(OBS, ACT, ENVS, _cfg())
    _fill(agent, 4)  # moves nothing in the actor, but exercises act between ingests
    obs = torch.randn(ENVS, OBS, device="cuda")
    det = agent.act(obs, training=False)
    ref = _oracle_actions(agent, obs, np.zeros((ENVS, ACT)))
    assert np.abs(det.cpu().numpy() - ref).max() < 1e-4
    trn = agent.act(obs, training=True)
    ref_t = _oracle_actions(agent, obs, agent._cached_noise.cpu().numpy())
    assert np.abs(trn.cpu().numpy() - ref_t).max() < 1e-4
    assert (trn.abs() <= 1).all() and not torch.allclose(trn, det)


def test_observe_update_metrics_and_actions_after_training():
    agent = FlashSAC(OBS, ACT, ENVS, _cfg())
    assert not agent.ready
    _fill(agent, 6)
    assert agent.ready and agent.can_start_training()
    first = agent.update()
    assert set(first) == {"actor/loss", "actor/entropy", "actor/mean_action", "critic/loss",
                          "critic/max_entropy_bonus", "temperature/value", "temperature/loss"}
    second = agent.update()
    assert set(second) == {"critic/loss", "critic/max_entropy_bonus"}
    for _ in range(4):
        m = agent.update(tensor_metrics=True)
        assert all(isinstance(v, torch.Tensor) and v.is_cuda for v in m.values())
    assert all(np.isfinite(v) for v in {**first, **second}.values())
    # the actor moved: eval-mode actions still match the oracle from the updated weights and BN buffers
    obs = torch.randn(ENVS, OBS, device="cuda")
    det = agent.act(obs, training=False)
    ref = _oracle_actions(agent, obs, np.zeros((ENVS, ACT)))
    assert np.abs(det.cpu().numpy() - ref).max() < 1e-4


@pytest.mark.parametrize("precision", ["fp32", "fp16"])
def test_save_load_round_trip(tmp_path, precision):
    a = FlashSAC(OBS, ACT, ENVS, _cfg(dense_precision=precision))
    _fill(a, 6)
    for _ in range(3):
        a.update()
    a.save(str(tmp_path))
    a.save_replay_buffer(str(tmp_path))
    b = FlashSAC(OBS, ACT, ENVS, _cfg(dense_precision=precision, seed=9))
    b.load(str(tmp_path))
    b.load_replay_buffer(str(tmp_path))
    La, Lb = a.learner, b.learner
    for na, nb in ((La.actor, Lb.actor), (La.critic, Lb.critic), (La.target, Lb.target)):
        sa, sb = na.state_dict(), nb.state_dict()
        assert set(sa) == set(sb)
        for k in sa:
            assert torch.equal(sa[k], sb[k]), k
    for na, nb in ((La.actor, Lb.actor), (La.critic, Lb.critic)):
        assert torch.equal(na.m, nb.m) and torch.equal(na.v, nb.v)
        assert na.opt_state[1] == nb.opt_state[1]  # Adam steps
    assert torch.equal(La.log_temp, Lb.log_temp)
    assert torch.equal(a._reward_state, b._reward_state)
    assert b._update_step == a._update_step
    assert len(b.replay) == len(a.replay)
    m = b.update()
    assert all(np.isfinite(v) for v in m.values())


def test_constructor_validation():
    with pytest.raises(ValueError):
        FlashSAC(0, ACT, ENVS, _cfg())
    with pytest.raises(ValueError):
        FlashSAC(OBS, ACT, ENVS, _cfg(), critic_observation_dim=OBS - 1)
    with pytest.raises(RuntimeError):
        FlashSAC(OBS, ACT, ENVS, _cfg(device="cpu"))
