"""``WarpFlashSAC`` (reference Warp-class interface, Warp-NN Adam) on the GPU.

* ``update_from_batch`` with the reference's tiny golden batch and injected noise: metrics
  and parameters against the oracle with the Warp-NN Adam formula, within 1e-4 (FP32).
* ``apply_optimizer=False`` leaves parameters and optimizer counters unchanged.
* ``prepare(capture=True)`` + ``update()`` replays graphs; ``state_dict`` / ``save`` /
  ``load`` round trip in place (graphs keep working).
"""

import warnings

import numpy as np
import pytest
import torch

from oracle import flashsac_np as fs
from tests import _golden as G

pytestmark = pytest.mark.gpu

from robolearn_b200.flashsac.config import FlashSACConfig  # noqa: E402
from robolearn_b200.flashsac.warp_agent import WarpFlashSAC  # noqa: E402


def _golden_agent(g, precision="fp32"):
    s = lambda k: g[f"spec.{k}"].item()  # noqa: E731
    d = G.dims(g)
    cfg = FlashSACConfig(
        device="cuda:0", sample_batch_size=int(s("batch")), actor_hidden_dim=int(s("actor_hidden")),
        actor_num_blocks=int(s("actor_blocks")), critic_hidden_dim=int(s("critic_hidden")),
        critic_num_blocks=int(s("critic_blocks")), critic_num_bins=int(s("bins")), critic_min_v=float(s("min_v")),
        critic_max_v=float(s("max_v")), critic_target_update_tau=0.005, learning_rate_init=3e-4,
        learning_rate_peak=3e-4, learning_rate_end=1.5e-4, learning_rate_warmup_step=0, learning_rate_decay_step=10,
        n_step=1, buffer_max_length=256, buffer_min_length=8, dense_precision=precision, normalize_reward=False,
        temp_target_sigma=0.15)
    with pytest.warns(RuntimeWarning):
        a = WarpFlashSAC(d.obs, d.act, 8, cfg, critic_observation_dim=d.critic_obs)
    L = a.learner
    L.actor.load_state_dict(G.network(g, "before", "actor"))
    L.critic.load_state_dict(G.network(g, "before", "critic"))
    L.target.load_state_dict(G.network(g, "before", "target"))
    L.log_temp.fill_(float(g["before.temp.log_temp"][0]))
    return a, d


def test_update_from_batch_matches_oracle_with_warp_adam():
    g = G.load("flashsac_update_tiny.npz")
    agent, d = _golden_agent(g)
    batch = G.batch(g, 0)
    a_noise, n_noise = G.noise(g, 0)
    h = G.hyper(g)
    h.target_entropy = agent._cfg.temp_target_entropy
    h.adam = "warp"
    state, ref = fs.update_networks(G.initial_state(g), batch, a_noise, n_noise, d, h, do_actor=True)
    got = agent.update_from_batch(batch, actor_noise=a_noise, next_noise=n_noise, do_actor_update=True,
                                  tensor_metrics=False)
    for k, v in ref.items():
        assert abs(got[k] - float(v)) <= 1e-4 * max(1.0, abs(float(v))), (k, got[k], float(v))
    for tag, net in (("actor", agent.learner.actor), ("critic", agent.learner.critic)):
        for k, v in state[tag].items():
            if k.endswith(("running_mean", "running_var")) or k == "predictor.bin_values":
                continue
            ours = net.param(k).cpu().numpy().astype(np.float64)
            err = np.abs(ours - v).max() / max(np.abs(v).max(), 1e-12)
            assert err < 1e-4, (tag, k, err)


def test_apply_optimizer_false_keeps_parameters():
    g = G.load("flashsac_update_tiny.npz")
    agent, _ = _golden_agent(g)
    before = [p.clone() for p in agent.parameters()]
    a_noise, n_noise = G.noise(g, 0)
    agent.update_from_batch(G.batch(g, 0), actor_noise=a_noise, next_noise=n_noise, do_actor_update=True,
                            apply_optimizer=False)
    torch.cuda.synchronize()
    for b, p in zip(before, agent.parameters()):
        assert torch.equal(b, p)
    assert agent._update_step == 0
    assert float(agent.learner.critic.grads.abs().sum()) > 0


def test_prepare_capture_update_and_checkpoint_round_trip(tmp_path):
    cfg = FlashSACConfig(device="cuda:0", sample_batch_size=64, actor_hidden_dim=32, actor_num_blocks=1,
                         critic_hidden_dim=32, critic_num_blocks=1, critic_num_bins=21, n_step=1,
                         buffer_max_length=512, buffer_min_length=96, dense_precision="fp32", seed=2)
    with warnings.catch_warnings():
        warnings.simplefilter("ignore", RuntimeWarning)
        a = WarpFlashSAC(9, 3, 32, cfg)
        b = WarpFlashSAC(9, 3, 32, cfg)
    gen = torch.Generator(device="cuda").manual_seed(0)
    obs = torch.randn(32, 9, device="cuda", generator=gen)
    for _ in range(4):
        act = a.act(obs)
        nxt = torch.randn(32, 9, device="cuda", generator=gen)
        a.observe(obs, act, torch.randn(32, device="cuda", generator=gen), torch.zeros(32, device="cuda"),
                  torch.zeros(32, device="cuda"), nxt)
        obs = nxt
    a.prepare(capture=True)
    for _ in range(3):
        m = a.update()
        assert all(np.isfinite(v) for v in m.values())
    a.save(tmp_path, include_replay=True)
    b.load(tmp_path)
    sa, sb = a.state_dict(), b.state_dict()
    assert set(sa) == set(sb)
    for k in sa:
        np.testing.assert_array_equal(sa[k], sb[k], err_msg=k)
    m_a = a.update(capture=True)
    m_b = b.update(capture=True)
    assert m_a.keys() == m_b.keys()
    for k in m_a:
        assert m_a[k] == m_b[k], k  # same state, same counters: identical update
    info = a.get_metrics()
    assert info["critic_optimizer_steps"] == 4.0


def test_constructor_validation():
    with pytest.raises(ValueError):
        WarpFlashSAC(4, 2, 8, FlashSACConfig(device="cuda:0", use_amp=True))
    with pytest.raises(ValueError):
        WarpFlashSAC(4, 2, 8, FlashSACConfig(device="cuda:0"), dense_backend="tiles")
