"""CPU restatement of the WarpPPO learner update -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU baseline may use
this module, as the checker; the product path never imports it.

Follows ``src/robolearn/warp/ppo.py`` of the reference:
  * ``gae``                 -> ``_gae`` (ppo.py:101-133), float32 with the kernel's
                               operation order (no fused multiply-add);
  * ``normalize_advantages``-> ``_advantage_sum/_variance/_normalize`` (ppo.py:136-159),
                               two-pass mean and centred variance;
  * ``init_params``         -> ``_mlp`` init (ppo.py:313-350) and ``WarpPPO.__init__``
                               parameter order actor + critic + std parameter
                               (ppo.py:405-433); Warp-NN ``Linear`` stores W as [out, in]
                               and b as [out, 1] (warp/_linear.py:57-79);
  * ``mlp_forward/backward``-> the ELU / tanh MLP (ELU alpha 1);
  * ``ppo_loss``            -> ``_make_ppo_loss`` (ppo.py:255-310) and its adjoint, with
                               Warp's adjoint rules: min -> first argument only if
                               strictly smaller, max -> first argument only if strictly
                               larger, clamp -> passes at and inside the bounds;
  * ``kl_mean`` / ``adapt_learning_rate`` -> ppo.py:207-238 (the KL in float32, as its
                               comparisons with zero and the thresholds depend on it);
  * ``clip_coefficient``    -> ``_clip_gradients`` (ppo.py:248-252): min(1, max_norm /
                               (sqrt(sum g^2) + 1e-6)). The combined-norm clip of
                               Warp-NN's Adam (``max_norm``) is not vendored; the same
                               formula is used for it (parity unpinned for that epsilon);
  * ``adam_warp``           -> Warp-NN Adam as restated in src/robolearn/cuda/kernels.cu:310-337;
  * ``update``              -> ``launch_update`` (ppo.py:586-695) with the minibatch
                               permutation given explicitly (the Warp RNG stream is not
                               reproduced).

Pinned by the reference's known-answer tests (tests/test_warp_ppo.py:23-119): the GAE
trace with termination / timeout / rollout boundary, advantages of +/-1 at an offset of
1e4, and the clipped Gaussian loss value with finite-difference gradients.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np

LOG_2PI = 1.8378770664093453
HALF_LOG_2PI_E = 1.4189385332046727


@dataclass
class PPOHyper:
    """The PPOConfig fields the update uses (src/robolearn/warp/config.py:9-34)."""

    hidden_dims: tuple = (64, 64)
    learning_rate: float = 3e-4
    gamma: float = 0.99
    gae_lambda: float = 0.95
    clip_ratio: float = 0.2
    value_coefficient: float = 0.5
    entropy_coefficient: float = 0.0
    epochs: int = 4
    max_grad_norm: float = 1.0
    initial_std: float = 1.0
    normalize_advantages: bool = True
    clip_value: bool = True
    activation: str = "tanh"
    std_type: str = "log"
    std_range: tuple = (1.0e-6, 1.0e6)
    num_mini_batches: int = 1
    schedule: str = "fixed"
    desired_kl: float = 0.01
    value_loss_scale: float = 0.5
    advantage_sample_std: bool = False
    timeout_bootstrap: str = "next"
    separate_grad_clipping: bool = False


# ---------------------------------------------------------------------------
# returns
# ---------------------------------------------------------------------------
def gae(rewards, values, next_values, terminated, truncated, horizon: int, num_envs: int, gamma: float,
        gae_lambda: float, current_timeout_bootstrap: bool = False):
    """Reverse-time GAE per environment; index k = t * num_envs + i. float32 throughout."""
    f = np.float32
    r = np.asarray(rewards, f)
    v = np.asarray(values, f)
    nv = np.asarray(next_values, f)
    te = np.asarray(terminated) != 0
    tr = np.asarray(truncated) != 0
    g, gl = f(gamma), f(f(gamma) * f(gae_lambda))
    adv = np.zeros(horizon * num_envs, f)
    ret = np.zeros(horizon * num_envs, f)
    for i in range(num_envs):
        a = f(0.0)
        for s in range(horizon):
            k = (horizon - s - 1) * num_envs + i
            boot = f(0.0) if te[k] else f(1.0)
            cont = f(0.0) if (te[k] or tr[k]) else f(1.0)
            nxt = nv[k]
            if current_timeout_bootstrap and tr[k]:
                nxt, boot = v[k], f(1.0)
            delta = f(f(r[k] + f(f(g * boot) * nxt)) - v[k])
            a = f(delta + f(f(gl * cont) * a))
            adv[k] = a
            ret[k] = f(a + v[k])
    return adv, ret


def normalize_advantages(adv, sample_std: bool = False) -> np.ndarray:
    x = np.asarray(adv, np.float64)
    n = x.size
    mean = x.sum() / n
    c = ((x - mean) ** 2).sum()
    if sample_std:
        out = (x - mean) / (math.sqrt(c / max(n - 1.0, 1.0)) + 1e-8)
    else:
        out = (x - mean) / math.sqrt(c / n + 1e-8)
    return out


# ---------------------------------------------------------------------------
# parameters and MLP
# ---------------------------------------------------------------------------
# Working floating-point type of the MLP, loss and optimiser arithmetic: float64 for the
# parity checks (default), float32 for timing the update as the reference's Torch
# restatement computes it. GAE keeps its own float32 operation order either way.
_WORK = {"dtype": np.float64}


def set_dtype(dtype) -> None:
    _WORK["dtype"] = np.dtype(dtype).type


def _FT():
    return _WORK["dtype"]


def init_mlp(in_dim: int, out_dim: int, hidden: tuple, rng: np.random.Generator) -> list[np.ndarray]:
    widths = (in_dim, *hidden, out_dim)
    params = []
    for i, o in zip(widths[:-1], widths[1:]):
        bound = 1.0 / math.sqrt(i)
        params.append(rng.uniform(-bound, bound, (o, i)).astype(np.float32))
        params.append(rng.uniform(-bound, bound, (o, 1)).astype(np.float32))
    return params


def init_params(obs: int, act: int, h: PPOHyper, seed: int) -> list[np.ndarray]:
    rng = np.random.default_rng(seed)
    actor = init_mlp(obs, act, tuple(h.hidden_dims), rng)
    critic = init_mlp(obs, 1, tuple(h.hidden_dims), rng)
    s0 = math.log(h.initial_std) if h.std_type == "log" else h.initial_std
    return actor + critic + [np.full(act, s0, np.float32)]


def split(params: list, hidden: tuple) -> tuple[list, list, np.ndarray]:
    n = 2 * (len(hidden) + 1)
    return params[:n], params[n:2 * n], params[-1]


def _act(x, kind):
    return np.where(x > 0, x, np.expm1(np.minimum(x, 0.0))) if kind == "elu" else np.tanh(x)


def _act_grad(y, kind):
    return np.where(y > 0, 1.0, y + 1.0) if kind == "elu" else 1.0 - y * y


def mlp_forward(net: list, x, activation: str):
    h = np.asarray(x, _FT())
    acts = [h]
    layers = len(net) // 2
    for li in range(layers):
        w = net[2 * li].astype(_FT())
        b = net[2 * li + 1].astype(_FT()).reshape(-1)
        h = h @ w.T + b
        if li < layers - 1:
            h = _act(h, activation)
        acts.append(h)
    return h, acts


def mlp_backward(net: list, acts: list, dout, activation: str) -> list[np.ndarray]:
    layers = len(net) // 2
    grads = [None] * len(net)
    d = np.asarray(dout, _FT())
    for li in range(layers - 1, -1, -1):
        x = acts[li]
        grads[2 * li] = d.T @ x
        grads[2 * li + 1] = d.sum(0).reshape(-1, 1)
        if li > 0:
            d = (d @ net[2 * li].astype(_FT())) * _act_grad(acts[li], activation)
    return grads


# ---------------------------------------------------------------------------
# loss and its adjoint
# ---------------------------------------------------------------------------
def _action_log_std(param, h: PPOHyper):
    p = np.asarray(param, _FT())
    if h.std_type == "scalar":
        lo, hi = h.std_range
        inside = (p >= lo) & (p <= hi)
        return np.log(np.clip(p, lo, hi)), np.where(inside, 1.0 / np.clip(p, lo, hi), 0.0)
    return p, np.ones_like(p)


def ppo_loss(mean, value, std_param, actions, old_log_probs, old_values, advantages, returns, h: PPOHyper):
    """Returns (loss, metrics[policy, value, entropy], d_mean, d_value, d_std_param)."""
    mean = np.asarray(mean, _FT())
    value = np.asarray(value, _FT()).reshape(-1)
    a = np.asarray(actions, _FT())
    olp = np.asarray(old_log_probs, _FT())
    ov = np.asarray(old_values, _FT())
    adv = np.asarray(advantages, _FT())
    ret = np.asarray(returns, _FT())
    M = mean.shape[0]
    s, ds_dp = _action_log_std(std_param, h)
    r = (a - mean) * np.exp(-s)
    logp = (-0.5 * (r * r + 2.0 * s + LOG_2PI)).sum(1)
    entropy = (s + HALF_LOG_2PI_E).sum() * np.ones(M)
    ratio = np.exp(logp - olp)
    eps = h.clip_ratio
    cl = np.clip(ratio, 1.0 - eps, 1.0 + eps)
    ua, ca = ratio * adv, cl * adv
    policy = -np.minimum(ua, ca)
    err = value - ret
    vloss = err * err
    if h.clip_value:
        cv = ov + np.clip(value - ov, -eps, eps)
        cerr = cv - ret
        vloss = np.maximum(vloss, cerr * cerr)
    vloss = h.value_loss_scale * vloss
    sc = 1.0 / M
    loss = sc * (policy + h.value_coefficient * vloss - h.entropy_coefficient * entropy).sum()
    metrics = np.array([sc * policy.sum(), sc * vloss.sum(), sc * entropy.sum()])
    # adjoint (Warp rules: min -> first arg if strictly smaller; clamp passes inside/at bounds)
    first = ua < ca
    inside = (ratio >= 1.0 - eps) & (ratio <= 1.0 + eps)
    d_ratio = np.where(first, -adv, np.where(inside, -adv, 0.0)) * sc
    d_logp = d_ratio * ratio
    d_mean = d_logp[:, None] * r * np.exp(-s)
    d_s = (d_logp[:, None] * (r * r - 1.0)).sum(0) - h.entropy_coefficient * sc * M
    if h.clip_value:
        vin = (value - ov >= -eps) & (value - ov <= eps)
        unc = err * err > cerr * cerr
        d_value = np.where(unc, 2.0 * err, np.where(vin, 2.0 * cerr, 0.0))
    else:
        d_value = 2.0 * err
    d_value = d_value * h.value_loss_scale * h.value_coefficient * sc
    return loss, metrics, d_mean, d_value, d_s * ds_dp


def kl_mean(mean, std_param, old_mean, old_std, h: PPOHyper) -> float:
    """KL(old || new) per row in float32 with the kernel's operation order (ppo.py:207-230),
    mean over rows. The adaptive schedule compares this value with zero and with
    thresholds, so the float32 rounding of the reference decides: for a policy that has
    not moved, 1 + md^2 rounds to 1 and every row contributes exactly zero."""
    f = np.float32
    mean = np.asarray(mean, f)
    p = np.asarray(std_param, f)
    sd = np.clip(p, f(h.std_range[0]), f(h.std_range[1])) if h.std_type == "scalar" else np.exp(p)
    vr = np.asarray(old_std, f) / sd
    md = (np.asarray(old_mean, f) - mean) / sd
    acc = np.zeros(mean.shape[0], f)
    for j in range(mean.shape[1]):
        acc = acc + f(0.5) * (vr[:, j] * vr[:, j] + md[:, j] * md[:, j] - f(1.0))
        acc = acc - np.log(vr[:, j])
    return float(acc.astype(np.float64).sum() / mean.shape[0])


def adapt_learning_rate(kl: float, desired_kl: float, lr: float) -> float:
    if kl > desired_kl * 2.0:
        return max(1.0e-5, lr / 1.5)
    if kl < desired_kl / 2.0 and kl > 0.0:
        return min(1.0e-2, lr * 1.5)
    return lr


def clip_coefficient(grads: list, max_norm: float) -> float:
    ss = sum(float((np.asarray(g, np.float64) ** 2).sum()) for g in grads)
    return min(1.0, max_norm / (math.sqrt(ss) + 1.0e-6))


def adam_warp(p, g, m1, m2, t: int, lr: float, b1=0.9, b2=0.999, eps=1e-8):
    m1 = b1 * m1 + (1.0 - b1) * g
    m2 = b2 * m2 + (1.0 - b2) * g * g
    c1 = 1.0 / (1.0 - b1**t)
    c2 = 1.0 / (1.0 - b2**t)
    p = p - lr * (m1 * c1 / (np.sqrt(m2 * c2) + eps))
    return p, m1, m2


# ---------------------------------------------------------------------------
# one full update
# ---------------------------------------------------------------------------
@dataclass
class PPOState:
    params: list
    m1: list = field(default_factory=list)
    m2: list = field(default_factory=list)
    timestep: int = 0
    lr: float = 0.0

    @staticmethod
    def fresh(params: list, lr: float) -> "PPOState":
        p = [np.asarray(x, _FT()) for x in params]
        return PPOState(p, [np.zeros_like(x) for x in p], [np.zeros_like(x) for x in p], 0, lr)


def returns_and_advantages(data: dict, horizon: int, num_envs: int, h: PPOHyper):
    adv, ret = gae(data["rewards"], data["values"], data["next_values"], data["terminated"], data["truncated"],
                   horizon, num_envs, h.gamma, h.gae_lambda, h.timeout_bootstrap == "current")
    if h.normalize_advantages:
        adv = normalize_advantages(adv, h.advantage_sample_std)
    return np.asarray(adv, _FT()), np.asarray(ret, _FT())


def minibatch_step(state: PPOState, batch: dict, h: PPOHyper) -> dict:
    """Loss, backward, clipping and Adam for one minibatch; returns diagnostics."""
    hid = tuple(h.hidden_dims)
    actor, critic, std_p = split(state.params, hid)
    mean, a_acts = mlp_forward(actor, batch["observations"], h.activation)
    value, c_acts = mlp_forward(critic, batch["observations"], h.activation)
    kl = 0.0
    if h.schedule == "adaptive":
        kl = kl_mean(mean, std_p, batch["means"], batch["stds"], h)
        state.lr = adapt_learning_rate(kl, h.desired_kl, state.lr)
    loss, metrics, d_mean, d_value, d_std = ppo_loss(mean, value[:, 0], std_p, batch["actions"],
                                                     batch["log_probs"], batch["values"], batch["advantages"],
                                                     batch["returns"], h)
    ga = mlp_backward(actor, a_acts, d_mean, h.activation)
    gc = mlp_backward(critic, c_acts, d_value[:, None], h.activation)
    grads = ga + gc + [d_std]
    norms = {}
    if h.separate_grad_clipping:
        na = len(ga)
        group_a = ga + [d_std]
        ca = clip_coefficient(group_a, h.max_grad_norm)
        cc = clip_coefficient(gc, h.max_grad_norm)
        norms = {"actor": math.sqrt(sum(float((g**2).sum()) for g in group_a)),
                 "critic": math.sqrt(sum(float((g**2).sum()) for g in gc))}
        grads = [g * ca for g in ga] + [g * cc for g in gc] + [d_std * ca]
        assert len(grads) == 2 * na + 1
    else:
        c = clip_coefficient(grads, h.max_grad_norm)
        grads = [g * c for g in grads]
    state.timestep += 1
    for i, g in enumerate(grads):
        state.params[i], state.m1[i], state.m2[i] = adam_warp(state.params[i], g, state.m1[i], state.m2[i],
                                                              state.timestep, state.lr)
    return {"loss": loss, "metrics": metrics, "kl": kl, "norms": norms, "grads": grads}


def update(state: PPOState, data: dict, horizon: int, num_envs: int, h: PPOHyper, permutation=None) -> dict:
    """``launch_update``: returns/advantages, then epochs x minibatches over ``permutation``."""
    adv, ret = returns_and_advantages(data, horizon, num_envs, h)
    n = horizon * num_envs
    mb = n // h.num_mini_batches
    perm = np.arange(n) if h.num_mini_batches == 1 else np.asarray(permutation)
    rows = {k: np.asarray(data[k]) for k in ("observations", "actions", "means", "stds", "log_probs", "values")}
    rows["advantages"], rows["returns"] = adv, ret
    last = None
    for _ in range(h.epochs):
        for b in range(h.num_mini_batches):
            sel = perm[b * mb:(b + 1) * mb]
            last = minibatch_step(state, {k: v[sel] for k, v in rows.items()}, h)
    return {"advantages": adv, "returns": ret, "last": last}
