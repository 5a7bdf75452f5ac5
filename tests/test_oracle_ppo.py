"""The PPO oracle against the reference's known-answer tests (CPU).

tests/test_warp_ppo.py of the reference pins: the GAE trace across termination,
timeout and the rollout boundary (:23-46), advantage normalisation of a small variance
at a large offset (:49-56), and the clipped Gaussian loss value plus finite-difference
gradients (:59-119). The same checks run here on the restatement; the MLP / loss
adjoints are also checked against torch autograd in float64.
"""

import math

import numpy as np
import torch

from oracle import ppo_np as P


def test_gae_termination_timeout_and_rollout_boundary():
    reward = np.array([[1, 2], [3, 4], [5, 6]], dtype=np.float32)
    value = np.array([[0.1, 0.2], [0.3, 0.4], [0.5, 0.6]], dtype=np.float32)
    next_value = np.array([[0.3, 0.4], [9, 10], [11, 12]], dtype=np.float32)
    terminated = np.array([[0, 0], [1, 0], [0, 0]], dtype=np.int32)
    truncated = np.array([[0, 0], [0, 1], [0, 0]], dtype=np.int32)
    expected = np.zeros_like(reward)
    tail = np.zeros(2, dtype=np.float32)
    for t in range(2, -1, -1):
        delta = reward[t] + 0.99 * (1 - terminated[t]) * next_value[t] - value[t]
        tail = delta + 0.99 * 0.95 * (1 - np.maximum(terminated[t], truncated[t])) * tail
        expected[t] = tail
    adv, ret = P.gae(reward.ravel(), value.ravel(), next_value.ravel(), terminated.ravel(), truncated.ravel(), 3, 2,
                     0.99, 0.95)
    np.testing.assert_allclose(adv.reshape(3, 2), expected, rtol=1e-6)
    np.testing.assert_allclose(ret.reshape(3, 2), expected + value, rtol=1e-6)


def test_gae_current_timeout_bootstrap_uses_own_value():
    adv, _ = P.gae([1.0], [0.5], [9.0], [0], [1], 1, 1, 0.99, 0.95, current_timeout_bootstrap=True)
    assert adv[0] == np.float32(np.float32(1.0 + np.float32(0.99) * np.float32(0.5)) - np.float32(0.5))


def test_advantage_normalization_small_variance_at_large_offset():
    h = P.PPOHyper(hidden_dims=(), gamma=0.0)
    data = dict(rewards=np.array([10000.0, 10001.0], np.float32), values=np.zeros(2, np.float32),
                next_values=np.zeros(2, np.float32), terminated=np.zeros(2, np.int32), truncated=np.zeros(2, np.int32))
    adv, ret = P.returns_and_advantages(data, 1, 2, h)
    np.testing.assert_allclose(adv, [-1.0, 1.0], rtol=1e-6)
    np.testing.assert_array_equal(ret, data["rewards"])


def test_clipped_gaussian_loss_and_gradient_known_answer():
    mean_np = np.array([[0.4, 0.1], [-0.3, 0.2], [0.2, -0.2]], dtype=np.float32)
    action_np = np.array([[0.0, 0.5], [0.6, 0.1], [-0.5, 0.4]], dtype=np.float32)
    old_lp_np = np.array([-2.4, -1.8, -2.0], dtype=np.float32)
    advantage_np = np.array([1.0, -0.8, 0.4], dtype=np.float32)
    value_np = np.array([[0.8], [1.0], [-0.5]], dtype=np.float32)
    old_value_np = np.array([0.2, 1.3, -0.4], dtype=np.float32)
    return_np = np.array([0.7, -0.2, 1.0], dtype=np.float32)
    log_std_np = np.array([-0.2, 0.1], dtype=np.float32)
    h = P.PPOHyper(clip_ratio=0.2, value_coefficient=0.5, entropy_coefficient=0.01, clip_value=True)

    def reference(mean_values=mean_np, value_values=value_np, std_values=log_std_np):
        lp = (-0.5 * (((action_np - mean_values) * np.exp(-std_values)) ** 2 + 2 * std_values
                      + np.log(2 * np.pi))).sum(axis=1)
        ratio = np.exp(lp - old_lp_np)
        policy = -np.minimum(ratio * advantage_np, np.clip(ratio, 0.8, 1.2) * advantage_np).mean()
        clipped_value = old_value_np + np.clip(value_values[:, 0] - old_value_np, -0.2, 0.2)
        value_loss = 0.5 * np.maximum((value_values[:, 0] - return_np) ** 2, (clipped_value - return_np) ** 2).mean()
        entropy = (std_values + 0.5 * np.log(2 * np.pi * np.e)).sum()
        return policy + 0.5 * value_loss - 0.01 * entropy

    loss, metrics, d_mean, d_value, d_std = P.ppo_loss(mean_np, value_np[:, 0], log_std_np, action_np, old_lp_np,
                                                       old_value_np, advantage_np, return_np, h)
    np.testing.assert_allclose(loss, reference(), rtol=1e-5, atol=1e-7)
    for argument, data, gradient in (("mean_values", mean_np, d_mean), ("value_values", value_np, d_value[:, None]),
                                     ("std_values", log_std_np, d_std)):
        numerical = np.zeros_like(data, dtype=np.float64)
        for index in np.ndindex(data.shape):
            plus, minus = data.astype(np.float64), data.astype(np.float64)
            plus[index] += 1e-3
            minus[index] -= 1e-3
            numerical[index] = (reference(**{argument: plus}) - reference(**{argument: minus})) / 2e-3
        np.testing.assert_allclose(gradient, numerical, atol=2e-4, rtol=2e-3)


def _torch_minibatch_grads(params, batch, h):
    t = [torch.tensor(np.asarray(p, np.float64), requires_grad=True) for p in params]
    nl = 2 * (len(h.hidden_dims) + 1)
    actor, critic, std_p = t[:nl], t[nl:2 * nl], t[-1]

    def forward(x, net):
        for i in range(0, len(net), 2):
            x = torch.nn.functional.linear(x, net[i], net[i + 1].reshape(-1))
            if i < len(net) - 2:
                x = torch.nn.functional.elu(x) if h.activation == "elu" else torch.tanh(x)
        return x

    obs = torch.tensor(batch["observations"], dtype=torch.float64)
    mean = forward(obs, actor)
    value = forward(obs, critic)[:, 0]
    std = std_p.clamp(*h.std_range) if h.std_type == "scalar" else std_p.exp()
    dist = torch.distributions.Normal(mean, std)
    ratio = (dist.log_prob(torch.tensor(batch["actions"], dtype=torch.float64)).sum(-1)
             - torch.tensor(batch["log_probs"], dtype=torch.float64)).exp()
    adv = torch.tensor(batch["advantages"], dtype=torch.float64)
    policy = torch.maximum(-ratio * adv, -ratio.clamp(1 - h.clip_ratio, 1 + h.clip_ratio) * adv).mean()
    ov = torch.tensor(batch["values"], dtype=torch.float64)
    ret = torch.tensor(batch["returns"], dtype=torch.float64)
    clipped = ov + (value - ov).clamp(-h.clip_ratio, h.clip_ratio)
    vloss = h.value_loss_scale * torch.maximum((value - ret) ** 2, (clipped - ret) ** 2).mean()
    loss = policy + h.value_coefficient * vloss - h.entropy_coefficient * dist.entropy().sum(-1).mean()
    loss.backward()
    return float(loss.detach()), [p.grad.numpy() for p in t]


def test_mlp_and_loss_adjoints_match_torch_autograd():
    for activation, std_type in (("elu", "log"), ("tanh", "scalar")):
        h = P.PPOHyper(hidden_dims=(16, 8), activation=activation, std_type=std_type, entropy_coefficient=0.01,
                       value_coefficient=1.0, clip_value=True, max_grad_norm=1e9)
        params = P.init_params(7, 3, h, seed=5)
        rng = np.random.default_rng(11)
        M = 40
        obs = rng.normal(size=(M, 7))
        actor, critic, std_p = P.split(params, h.hidden_dims)
        mean, _ = P.mlp_forward(actor, obs, activation)
        value, _ = P.mlp_forward(critic, obs, activation)
        batch = dict(observations=obs, actions=mean + rng.normal(size=mean.shape), means=mean,
                     stds=np.ones_like(mean), log_probs=rng.normal(-4, 0.3, size=M),
                     values=value[:, 0] + rng.normal(0, 0.3, size=M), advantages=rng.normal(size=M),
                     returns=rng.normal(size=M))
        ref_loss, ref_grads = _torch_minibatch_grads(params, batch, h)
        state = P.PPOState.fresh(params, 1e-3)
        out = P.minibatch_step(state, batch, h)
        assert abs(out["loss"] - ref_loss) < 1e-12 * max(1.0, abs(ref_loss))
        for g, r in zip(out["grads"], ref_grads):
            np.testing.assert_allclose(np.asarray(g).reshape(r.shape), r, rtol=1e-9, atol=1e-12)


def test_clip_coefficient_and_adam_formula():
    g = [np.array([3.0, 4.0])]
    assert abs(P.clip_coefficient(g, 1.0) - 1.0 / (5.0 + 1e-6)) < 1e-15
    assert P.clip_coefficient(g, 10.0) == 1.0
    p, m1, m2 = P.adam_warp(np.array([1.0]), np.array([0.5]), np.zeros(1), np.zeros(1), 1, 0.1)
    # first step: m1 c1 = g, m2 c2 = g^2 -> p - lr * g / (|g| + eps)
    assert abs(p[0] - (1.0 - 0.1 * 0.5 / (0.5 + 1e-8))) < 1e-12
    assert math.isclose(m1[0], 0.05) and math.isclose(m2[0], 0.001 * 0.25)


def test_oracle_matches_reference_torch_controlled_update():
    """The reference's controlled PPO update check (examples/diagnose_ppo_update.py, run by
    tests/golden/make_ppo_golden.py with the oracle standing in for Warp PPO): its Torch half's
    final parameters, Adam moments and adaptive learning rate after 5 epochs x 4 minibatches
    (adaptive KL, scalar std, separate clipping, timeout bootstrap 'current', sample-std
    advantages) are matched by the oracle within that check's thresholds (maximum absolute
    error 2e-4 for parameters and moments, 1e-7 for the learning rate)."""
    import numpy as np

    from oracle import ppo_np as P
    from robolearn_b200.ppo.config import PPOConfig
    from tests import _golden as G

    g = G.load("ppo_controlled_update.npz")
    cfg = PPOConfig(hidden_dims=(16, 8), activation="elu", std_type="scalar", epochs=5, num_mini_batches=4,
                    learning_rate=1.0e-3, schedule="adaptive", desired_kl=0.01, value_coefficient=1.0,
                    value_loss_scale=1.0, entropy_coefficient=0.008, advantage_sample_std=True,
                    timeout_bootstrap="current", separate_grad_clipping=True)
    h = P.PPOHyper(**{k: getattr(cfg, k) for k in P.PPOHyper.__dataclass_fields__})
    n = len([k for k in g if k.startswith("initial.")])
    initial = [g[f"initial.{i}"] for i in range(n)]
    np.testing.assert_array_equal(np.concatenate([x.ravel() for x in initial]),
                                  np.concatenate([x.ravel() for x in P.init_params(7, 3, h, seed=cfg.seed)]))
    data = {k[len("data."):]: v for k, v in g.items() if k.startswith("data.")}
    state = P.PPOState.fresh(initial, cfg.learning_rate)
    P.update(state, data, 4, 16, h, permutation=g["permutation"])
    assert abs(state.lr - float(g["torch.learning_rate"])) < 1e-7
    for i in range(n):
        ref = g[f"torch.parameter.{i}"].reshape(-1)
        assert np.abs(state.params[i].reshape(-1) - ref).max() < 2e-4, i
        assert np.abs(state.m1[i].reshape(-1) - g[f"torch.exp_avg.{i}"].reshape(-1)).max() < 2e-4, i
        assert np.abs(state.m2[i].reshape(-1) - g[f"torch.exp_avg_sq.{i}"].reshape(-1)).max() < 2e-4, i
    # the reference's own check passed on the oracle when the fixture was made
    assert float(g["report.torch_warp_parameters_max_abs_error"]) < 2e-4
    assert float(g["report.returns_max_abs_error"]) < 1e-5 and float(g["report.advantages_max_abs_error"]) < 1e-5
