"""WarpPPO on the GPU against the PPO oracle and the reference's known answers.

Tolerances: GAE 1e-6 relative (the reference's own GAE test; relative to the largest
magnitude when the horizon spans several scan segments), bit-exact for horizons that
fit one segment; advantages 1e-5; the fused loss and its gradients 1e-5
relative; a full update (tf32x3 GEMMs, fp32 everywhere else) 1e-4 relative per
parameter tensor after every Adam step of 2 epochs x 4 minibatches. Captured and
eager updates are bitwise equal; checkpoints restore bitwise.
"""

import ctypes

import numpy as np
import pytest
import torch

from oracle import ppo_np as P

pytestmark = pytest.mark.gpu

from robolearn_b200 import _native as N  # noqa: E402
from robolearn_b200.ppo import PPOConfig, WarpPPO  # noqa: E402


def _hyper(cfg: PPOConfig) -> P.PPOHyper:
    fields = P.PPOHyper.__dataclass_fields__
    return P.PPOHyper(**{k: getattr(cfg, k) for k in fields})


def test_gae_known_answer():
    agent = WarpPPO(1, 1, 2, 3, PPOConfig(hidden_dims=(), normalize_advantages=False))
    reward = np.array([[1, 2], [3, 4], [5, 6]], dtype=np.float32)
    value = np.array([[0.1, 0.2], [0.3, 0.4], [0.5, 0.6]], dtype=np.float32)
    next_value = np.array([[0.3, 0.4], [9, 10], [11, 12]], dtype=np.float32)
    terminated = np.array([[0, 0], [1, 0], [0, 0]], dtype=np.int32)
    truncated = np.array([[0, 0], [0, 1], [0, 0]], dtype=np.int32)
    for name, data in (("rewards", reward), ("values", value), ("next_values", next_value),
                       ("terminated", terminated), ("truncated", truncated)):
        getattr(agent, name).copy_(torch.from_numpy(data.ravel()))
    expected = np.zeros_like(reward)
    tail = np.zeros(2, dtype=np.float32)
    for t in range(2, -1, -1):
        delta = reward[t] + 0.99 * (1 - terminated[t]) * next_value[t] - value[t]
        tail = delta + 0.99 * 0.95 * (1 - np.maximum(terminated[t], truncated[t])) * tail
        expected[t] = tail
    agent.compute_returns()
    np.testing.assert_allclose(agent.advantages.cpu().numpy().reshape(3, 2), expected, rtol=1e-6)
    np.testing.assert_allclose(agent.returns.cpu().numpy().reshape(3, 2), expected + value, rtol=1e-6)
    adv, ret = P.gae(reward.ravel(), value.ravel(), next_value.ravel(), terminated.ravel(), truncated.ravel(), 3, 2,
                     0.99, 0.95)
    assert np.array_equal(agent.advantages.cpu().numpy(), adv)  # one scan segment: same operation order
    assert np.array_equal(agent.returns.cpu().numpy(), ret)


@pytest.mark.parametrize("horizon,bootstrap", [(24, "next"), (100, "current"), (7, "current")])
def test_gae_segmented_scan_matches_oracle(horizon, bootstrap):
    n = 300
    agent = WarpPPO(1, 1, n, horizon, PPOConfig(hidden_dims=(), normalize_advantages=False,
                                                  timeout_bootstrap=bootstrap))
    rng = np.random.default_rng(horizon)
    B = n * horizon
    data = dict(rewards=rng.normal(size=B).astype(np.float32), values=rng.normal(size=B).astype(np.float32),
                next_values=rng.normal(size=B).astype(np.float32),
                terminated=(rng.random(B) < 0.05).astype(np.int32), truncated=(rng.random(B) < 0.05).astype(np.int32))
    for k, v in data.items():
        getattr(agent, k).copy_(torch.from_numpy(v))
    agent.compute_returns()
    adv, ret = P.gae(data["rewards"], data["values"], data["next_values"], data["terminated"], data["truncated"],
                     horizon, n, 0.99, 0.95, bootstrap == "current")
    got = agent.advantages.cpu().numpy()
    # segments compose their maps in another rounding order: 1e-6 relative to the largest magnitude
    assert np.abs(got - adv).max() <= 1e-6 * np.abs(adv).max()
    assert np.abs(agent.returns.cpu().numpy() - ret).max() <= 1e-6 * np.abs(ret).max()
    if horizon <= 8:
        assert np.array_equal(got, adv)


@pytest.mark.parametrize("sample_std", [False, True])
def test_advantage_normalization(sample_std):
    agent = WarpPPO(1, 1, 2, 1, PPOConfig(hidden_dims=(), gamma=0.0, advantage_sample_std=sample_std))
    rewards = torch.tensor([10000.0, 10001.0])
    agent.rewards.copy_(rewards)
    agent.compute_returns()
    expect = P.normalize_advantages(np.array([10000.0, 10001.0]), sample_std)
    np.testing.assert_allclose(agent.advantages.cpu().numpy(), expect, rtol=1e-6)
    assert torch.equal(agent.returns.cpu(), rewards)
    # larger batch: two-pass double statistics against the oracle
    big = WarpPPO(1, 1, 4096, 24, PPOConfig(hidden_dims=(), advantage_sample_std=sample_std))
    rng = np.random.default_rng(1)
    for k in ("rewards", "values", "next_values"):
        getattr(big, k).copy_(torch.from_numpy(rng.normal(50.0, 3.0, size=big.batch_size).astype(np.float32)))
    big.compute_returns()
    adv, _ = P.gae(big.rewards.cpu().numpy(), big.values.cpu().numpy(), big.next_values.cpu().numpy(),
                   np.zeros(big.batch_size), np.zeros(big.batch_size), 24, 4096, 0.99, 0.95)
    np.testing.assert_allclose(big.advantages.cpu().numpy(), P.normalize_advantages(adv, sample_std), rtol=1e-5,
                               atol=2e-5)


def test_loss_kernel_known_answer():
    lib = N.load()
    dev = "cuda"
    mean_np = np.array([[0.4, 0.1], [-0.3, 0.2], [0.2, -0.2]], dtype=np.float32)
    action_np = np.array([[0.0, 0.5], [0.6, 0.1], [-0.5, 0.4]], dtype=np.float32)
    old_lp = np.array([-2.4, -1.8, -2.0], dtype=np.float32)
    adv = np.array([1.0, -0.8, 0.4], dtype=np.float32)
    value = np.array([0.8, 1.0, -0.5], dtype=np.float32)
    old_value = np.array([0.2, 1.3, -0.4], dtype=np.float32)
    ret = np.array([0.7, -0.2, 1.0], dtype=np.float32)
    log_std = np.array([-0.2, 0.1], dtype=np.float32)
    M, A, ld = 3, 2, 4
    head = torch.zeros(2, M, ld, device=dev)
    head[0, :, :A] = torch.from_numpy(mean_np)
    head[1, :, 0] = torch.from_numpy(value)
    t = lambda x: torch.from_numpy(np.ascontiguousarray(x)).to(dev)  # noqa: E731
    ins = dict(std=t(log_std), act=t(action_np), olp=t(old_lp), ov=t(old_value), adv=t(adv), ret=t(ret))
    d_head = torch.full((2, M, ld), 7.0, device=dev)
    out = dict(loss=torch.zeros(1, device=dev), metrics=torch.zeros(3, device=dev), dba=torch.zeros(A, device=dev),
               dbc=torch.zeros(1, device=dev), dstd=torch.zeros(A, device=dev),
               part=torch.zeros(lib.rl2_ppo_loss_partials(M, A), dtype=torch.float64, device=dev),
               ctr=torch.zeros(1, dtype=torch.int32, device=dev))
    args = N.PPOLossArgs(head=head.data_ptr(), ld_head=ld, head_twin_stride=M * ld, std_param=ins["std"].data_ptr(),
                         rows=M, act=A, actions=ins["act"].data_ptr(), old_log_probs=ins["olp"].data_ptr(),
                         old_values=ins["ov"].data_ptr(), advantages=ins["adv"].data_ptr(),
                         returns=ins["ret"].data_ptr(), clip_ratio=0.2, value_coefficient=0.5,
                         entropy_coefficient=0.01, value_loss_scale=0.5, clip_value=1, std_type=0, std_min=1e-6,
                         std_max=1e6, loss=out["loss"].data_ptr(), metrics=out["metrics"].data_ptr(),
                         d_head=d_head.data_ptr(), ld_d_head=ld, d_head_twin_stride=M * ld,
                         d_bias_actor=out["dba"].data_ptr(), d_bias_critic=out["dbc"].data_ptr(),
                         d_std_param=out["dstd"].data_ptr(), partials=out["part"].data_ptr(),
                         counter=out["ctr"].data_ptr())
    for _ in range(2):  # the ticket must be reset: a second launch gives the same answer
        N.check(lib.rl2_ppo_loss(ctypes.byref(args), N.stream_ptr()), "loss")
    torch.cuda.synchronize()
    h = P.PPOHyper(clip_ratio=0.2, value_coefficient=0.5, entropy_coefficient=0.01, clip_value=True)
    loss, metrics, d_mean, d_value, d_std = P.ppo_loss(mean_np, value, log_std, action_np, old_lp, old_value, adv,
                                                       ret, h)
    assert abs(out["loss"].item() - loss) < 1e-5 * max(1.0, abs(loss))
    np.testing.assert_allclose(out["metrics"].cpu().numpy(), metrics, rtol=1e-5, atol=1e-7)
    dh = d_head.cpu().numpy()
    np.testing.assert_allclose(dh[0, :, :A], d_mean, rtol=1e-5, atol=1e-7)
    np.testing.assert_allclose(dh[1, :, 0], d_value, rtol=1e-5, atol=1e-7)
    assert (dh[0, :, A:] == 0).all() and (dh[1, :, 1:] == 0).all()
    np.testing.assert_allclose(out["dstd"].cpu().numpy(), d_std, rtol=1e-5, atol=1e-7)
    np.testing.assert_allclose(out["dba"].cpu().numpy(), d_mean.sum(0), rtol=1e-5, atol=1e-7)
    np.testing.assert_allclose(out["dbc"].cpu().numpy(), [d_value.sum()], rtol=1e-5, atol=1e-7)
    assert out["ctr"].item() == 0


@pytest.mark.parametrize("n", [5, 16, 98304, 24577])
def test_permutation_is_a_bijection(n):
    lib = N.load()
    idx = torch.zeros(n, dtype=torch.int32, device="cuda")
    epoch = torch.tensor([3], dtype=torch.int64, device="cuda")
    health = torch.zeros(1, dtype=torch.int32, device="cuda")
    N.check(lib.rl2_ppo_permutation(12345, epoch.data_ptr(), n, idx.data_ptr(), health.data_ptr(), N.stream_ptr()),
            "perm")
    got = idx.cpu().numpy()
    assert np.array_equal(np.sort(got), np.arange(n)) and health.item() == 0
    if n > 16:
        assert not np.array_equal(got, np.arange(n))


def _fill_rollout(agent: WarpPPO, seed: int = 29):
    """Synthetic fixed rollout in the style of the reference's controlled update check."""
    rng = np.random.default_rng(seed)
    B, O, A = agent.batch_size, agent.observation_dim, agent.action_dim
    cfg = agent.config
    obs = rng.normal(size=(B, O)).astype(np.float32)
    params = [p.cpu().numpy() for p in agent.parameters]
    actor, critic, _ = P.split(params, cfg.hidden_dims)
    means, _ = P.mlp_forward(actor, obs, cfg.activation)
    values, _ = P.mlp_forward(critic, obs, cfg.activation)
    actions = (means + rng.normal(size=means.shape)).astype(np.float32)
    data = dict(observations=obs, actions=actions, means=means.astype(np.float32), stds=np.ones((B, A), np.float32),
                values=values[:, 0].astype(np.float32),
                log_probs=(-0.5 * ((actions - means) ** 2 + np.log(2 * np.pi))).sum(1).astype(np.float32),
                rewards=rng.normal(0.2, 0.05, size=B).astype(np.float32),
                next_values=rng.normal(0.0, 0.2, size=B).astype(np.float32),
                terminated=np.zeros(B, np.int32), truncated=np.zeros(B, np.int32))
    data["terminated"][min(18, B - 1)] = 1
    data["truncated"][min(39, B - 1)] = 1
    for k, v in data.items():
        getattr(agent, k).copy_(torch.from_numpy(v))
    return data


CONFIGS = {
    "rsl_adaptive": PPOConfig(hidden_dims=(16, 8), activation="elu", std_type="scalar", epochs=2, num_mini_batches=4,
                              learning_rate=1.0e-3, schedule="adaptive", desired_kl=0.01, value_coefficient=1.0,
                              value_loss_scale=1.0, entropy_coefficient=0.008, advantage_sample_std=True,
                              timeout_bootstrap="current", separate_grad_clipping=True),
    "fixed_tanh": PPOConfig(hidden_dims=(32, 16), epochs=2, num_mini_batches=2, learning_rate=3e-4,
                            entropy_coefficient=0.01),
}


@pytest.mark.parametrize("name", list(CONFIGS))
def test_full_update_matches_oracle(name):
    cfg = CONFIGS[name]
    agent = WarpPPO(7, 3, 16, 4, cfg)
    initial = [p.detach().cpu().numpy().copy() for p in agent.parameters]
    data = _fill_rollout(agent)
    agent.update(capture=False)
    torch.cuda.synchronize()
    perm = agent._perm.cpu().numpy()
    assert np.array_equal(np.sort(perm), np.arange(agent.batch_size))
    h = _hyper(cfg)
    state = P.PPOState.fresh(initial, cfg.learning_rate)
    out = P.update(state, data, agent.horizon, agent.num_envs, h, permutation=perm)
    np.testing.assert_allclose(agent.advantages.cpu().numpy(), out["advantages"], rtol=1e-5, atol=1e-5)
    for i, (got, ref) in enumerate(zip(agent.parameters, state.params)):
        g = got.detach().cpu().numpy().astype(np.float64).reshape(ref.shape)
        err = np.abs(g - ref).max() / max(np.abs(ref).max(), 1e-6)
        assert err < 1e-4, (i, err)
    sd = agent.state_dict()
    for i, ref in enumerate(state.m1):
        np.testing.assert_allclose(sd[f"adam_m1_{i}"].reshape(ref.shape), ref, rtol=2e-3, atol=1e-7)
    hm = agent.health_metrics()
    assert hm["optimizer_updates"] == cfg.epochs * cfg.num_mini_batches
    assert abs(hm["learning_rate"] - state.lr) < 1e-7
    np.testing.assert_allclose([hm["policy_loss"], hm["value_loss"], hm["entropy"]], out["last"]["metrics"],
                               rtol=1e-4, atol=1e-6)


def test_captured_update_matches_eager_and_checkpoint_preserves_graph(tmp_path):
    config = PPOConfig(hidden_dims=(16,), epochs=2)
    eager = WarpPPO(3, 2, 8, 4, config)
    captured = WarpPPO(3, 2, 8, 4, config)
    captured.load_state_dict(eager.state_dict())
    rng = np.random.default_rng(7)
    for name, shape in (("observations", (32, 3)), ("actions", (32, 2)), ("rewards", (32,))):
        samples = torch.from_numpy(rng.normal(size=shape).astype(np.float32))
        getattr(eager, name).copy_(samples)
        getattr(captured, name).copy_(samples)
    for _ in range(2):
        eager.update(capture=False)
        captured.update()
    for e, c in zip(eager.parameters, captured.parameters):
        assert torch.equal(e, c)
    ckpt = tmp_path / "ppo.npz"
    captured.save(ckpt)
    saved = captured.state_dict()
    captured.update()
    captured.load(ckpt)
    for k, v in saved.items():
        np.testing.assert_array_equal(captured.state_dict()[k], v)
    captured.update()
    eager.update(capture=False)
    for e, c in zip(eager.parameters, captured.parameters):
        assert torch.equal(e, c)


def test_act_and_store():
    cfg = PPOConfig(hidden_dims=(16, 8), activation="elu")
    agent = WarpPPO(5, 2, 8, 3, cfg)
    rng = np.random.default_rng(3)
    obs = torch.from_numpy(rng.normal(size=(8, 5)).astype(np.float32)).cuda()
    det = agent.act(obs, deterministic=True).clone()
    params = [p.cpu().numpy() for p in agent.parameters]
    actor, critic, _ = P.split(params, cfg.hidden_dims)
    mean, _ = P.mlp_forward(actor, obs.cpu().numpy(), "elu")
    np.testing.assert_allclose(det.cpu().numpy(), mean, rtol=1e-5, atol=1e-6)
    sto = agent.act(obs).clone()
    assert not torch.allclose(sto, det)
    nxt = torch.from_numpy(rng.normal(size=(8, 5)).astype(np.float32)).cuda()
    agent.store(1, obs, torch.ones(8), torch.zeros(8, dtype=torch.int32), torch.ones(8, dtype=torch.int32), nxt)
    rows = slice(8, 16)
    assert torch.equal(agent.observations[rows], obs)
    assert torch.equal(agent.actions[rows], sto)
    assert torch.equal(agent.truncated[rows].cpu(), torch.ones(8, dtype=torch.int32))
    nv, _ = P.mlp_forward(critic, nxt.cpu().numpy(), "elu")
    np.testing.assert_allclose(agent.next_values[rows].cpu().numpy(), nv[:, 0], rtol=1e-5, atol=1e-6)
    v, _ = P.mlp_forward(critic, obs.cpu().numpy(), "elu")
    np.testing.assert_allclose(agent.values[rows].cpu().numpy(), v[:, 0], rtol=1e-5, atol=1e-6)
    with pytest.raises(ValueError):
        agent.store(3, obs, torch.ones(8), torch.zeros(8), torch.zeros(8), nxt)


def test_cfg2_update_matches_oracle_at_the_reference_protocol_tolerances():
    """Config 2 at full size: WarpPPO(48, 12, 4096 envs, 24 steps), actor / critic 512-256-128
    ELU, 5 epochs x 4 minibatches of 24576 rows (split-K weight gradients, the large
    minibatch gathers), clip 0.2, value coefficient 1.0, entropy 0.01, lr 1e-3, through the
    captured update graph. Rollout with the config-2 distributions (obs ~N(0,1), actions =
    initial means + N(0,1), rewards ~N(0,1), terminated ~Bernoulli(0.005), next values from
    the critic on next observations ~N(0,1)). The float64 oracle runs the same update with
    the device's own permutation; the thresholds are those of the reference's controlled
    update check (examples/diagnose_ppo_update.py:197-206, maximum absolute errors): returns
    and advantages 1e-5, every parameter and Adam moment 2e-4."""
    cfg = PPOConfig(hidden_dims=(512, 256, 128), activation="elu", epochs=5, num_mini_batches=4, clip_ratio=0.2,
                    value_coefficient=1.0, entropy_coefficient=0.01, learning_rate=1e-3, gamma=0.99, gae_lambda=0.95)
    agent = WarpPPO(48, 12, 4096, 24, cfg)
    initial = [p.detach().cpu().numpy().copy() for p in agent.parameters]
    rng = np.random.default_rng(2026)
    B, O, A = agent.batch_size, 48, 12
    actor, critic, _ = P.split(initial, cfg.hidden_dims)
    obs = rng.standard_normal((B, O)).astype(np.float32)
    means, _ = P.mlp_forward(actor, obs, "elu")
    values, _ = P.mlp_forward(critic, obs, "elu")
    next_values, _ = P.mlp_forward(critic, rng.standard_normal((B, O)).astype(np.float32), "elu")
    actions = (means + rng.standard_normal(means.shape)).astype(np.float32)
    data = dict(observations=obs, actions=actions, means=means.astype(np.float32), stds=np.ones((B, A), np.float32),
                values=values[:, 0].astype(np.float32), next_values=next_values[:, 0].astype(np.float32),
                log_probs=(-0.5 * ((actions - means) ** 2 + np.log(2 * np.pi))).sum(1).astype(np.float32),
                rewards=rng.standard_normal(B).astype(np.float32),
                terminated=(rng.random(B) < 0.005).astype(np.int32), truncated=np.zeros(B, np.int32))
    for k, v in data.items():
        getattr(agent, k).copy_(torch.from_numpy(v))
    agent.update()  # captured graph (first call: eager warm pass, capture, replay)
    torch.cuda.synchronize()
    perm = agent._perm.cpu().numpy()
    assert np.array_equal(np.sort(perm), np.arange(B))
    state = P.PPOState.fresh(initial, cfg.learning_rate)
    out = P.update(state, data, agent.horizon, agent.num_envs, _hyper(cfg), permutation=perm)
    assert np.abs(agent.advantages.cpu().numpy() - out["advantages"]).max() < 1e-5
    assert np.abs(agent.returns.cpu().numpy() - out["returns"]).max() < 1e-5
    sd = agent.state_dict()
    for i, (got, ref) in enumerate(zip(agent.parameters, state.params)):
        err = np.abs(got.detach().cpu().numpy().astype(np.float64).reshape(ref.shape) - ref).max()
        assert err < 2e-4, ("parameter", i, err)
        for name, moments in (("adam_m1", state.m1), ("adam_m2", state.m2)):
            m_err = np.abs(sd[f"{name}_{i}"].reshape(ref.shape).astype(np.float64) - moments[i]).max()
            assert m_err < 2e-4, (name, i, m_err)
    assert agent.health_metrics()["optimizer_updates"] == 20
