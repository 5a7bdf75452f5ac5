"""Generate golden tensors by running the reference's own Torch FlashSAC on CPU.

Run in a container where the reference project's ``src`` directory is available
(``--reference-src``); the outputs are small ``.npz`` fixtures committed beside
this script, so the tests never need the reference at run time.

What is produced:

* ``flashsac_update_<case>.npz`` — parameters/buffers of actor, critic, target
  critic and temperature before and after two ``_update_networks`` calls (an
  actor+critic phase then a critic-only phase, ``agent.py:217-281``), the fixed
  batch, the fixed Gaussian noise injected by patching
  ``torch.distributions.Normal.rsample`` (the reference's own diagnostic
  technique, ``examples/diagnose_warp_flashsac.py:311-333``), Adam moments and the
  returned metrics.
* ``categorical_<case>.npz`` — inputs and outputs of ``_select_min_q_log_probs``,
  ``_compute_categorical_td_target`` and the CE loss / logits gradient
  (``updates.py:19-80,248-257``), including clamped, terminal and tied rows.
* ``replay_nstep.npz`` — the n-step replay KAT timeline of ``tests/test_flashsac.py``.

``gymnasium`` is absent here; the reference only needs ``gym.spaces.Box`` with
``shape``/``dtype``, so a test-only stand-in module is registered first.
"""

from __future__ import annotations

import argparse
import math
import sys
import types
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def _install_gym_shim() -> None:
    gym = types.ModuleType("gymnasium")
    spaces = types.ModuleType("gymnasium.spaces")

    class Space:
        def __class_getitem__(cls, item):
            return cls

    class Box(Space):
        def __init__(self, low, high, shape=None, dtype=np.float32):
            self.low, self.high = low, high
            self.shape = tuple(shape) if shape is not None else None
            self.dtype = np.dtype(dtype)

    spaces.Space, spaces.Box = Space, Box
    gym.spaces = spaces
    sys.modules["gymnasium"] = gym
    sys.modules["gymnasium.spaces"] = spaces


def _state(module) -> dict[str, np.ndarray]:
    return {k.removeprefix("_orig_mod."): v.detach().cpu().numpy().copy() for k, v in module.state_dict().items()}


def _moments(network) -> dict[str, np.ndarray]:
    out = {}
    names = [n for n, _ in network.network.named_parameters()]
    params = list(network.network.parameters())
    for name, p in zip(names, params):
        st = network.optimizer.state.get(p, {})
        if st:
            out["m." + name] = st["exp_avg"].cpu().numpy().copy()
            out["v." + name] = st["exp_avg_sq"].cpu().numpy().copy()
            out["step." + name] = np.array(float(st["step"]))
    return out


CASES = {
    # tiny network, odd sizes, 11 bins (the reference's own test configuration style)
    "tiny": dict(obs=5, act=3, actor_hidden=8, actor_blocks=1, critic_hidden=8, critic_blocks=1,
                 bins=11, min_v=-5.0, max_v=5.0, batch=6, critic_obs=None),
    # cfg1-style shapes at reduced width: 101 atoms on [-10, 10], two blocks
    "small": dict(obs=31, act=8, actor_hidden=16, actor_blocks=2, critic_hidden=32, critic_blocks=2,
                  bins=101, min_v=-10.0, max_v=10.0, batch=32, critic_obs=None),
    # asymmetric critic input (privileged observation suffix)
    "asym": dict(obs=7, act=4, actor_hidden=16, actor_blocks=1, critic_hidden=16, critic_blocks=1,
                 bins=21, min_v=-10.0, max_v=10.0, batch=12, critic_obs=11),
}


def make_update_case(name: str, spec: dict) -> None:
    import torch

    from robolearn.flashsac import FlashSACConfig
    from robolearn.flashsac.agent import _init_flashsac_networks, _update_networks

    torch.set_num_threads(1)
    cfg = FlashSACConfig(
        device="cpu", use_compile=False, use_amp=False, seed=0,
        actor_hidden_dim=spec["actor_hidden"], actor_num_blocks=spec["actor_blocks"],
        critic_hidden_dim=spec["critic_hidden"], critic_num_blocks=spec["critic_blocks"],
        critic_num_bins=spec["bins"], critic_min_v=spec["min_v"], critic_max_v=spec["max_v"],
        critic_target_update_tau=0.005, learning_rate_init=3e-4, learning_rate_peak=3e-4,
        learning_rate_end=1.5e-4, learning_rate_warmup_step=0, learning_rate_decay_step=10, n_step=1,
        buffer_max_length=64, buffer_min_length=8, sample_batch_size=spec["batch"],
    )
    obs_a = spec["obs"]
    obs_c = spec["critic_obs"] or obs_a
    act = spec["act"]
    target_entropy = 0.5 * act * math.log(2 * math.pi * math.e * cfg.temp_target_sigma**2)
    cfg.temp_target_entropy = target_entropy
    torch.manual_seed(0)
    actor, critic, target, temp = _init_flashsac_networks(obs_a, obs_c, act, cfg, torch.device("cpu"))
    out: dict[str, np.ndarray] = {}
    for tag, net in (("actor", actor), ("critic", critic), ("target", target), ("temp", temp)):
        for k, v in _state(net.network).items():
            out[f"before.{tag}.{k}"] = v

    rng = np.random.default_rng(2026)
    B = spec["batch"]
    batches, noises = [], []
    for update in range(2):
        batch = {
            "observation": rng.standard_normal((B, obs_c)).astype(np.float32),
            "next_observation": rng.standard_normal((B, obs_c)).astype(np.float32),
            "action": rng.uniform(-1, 1, (B, act)).astype(np.float32),
            "reward": (3.0 * rng.standard_normal(B)).astype(np.float32),
            "terminated": (rng.random(B) < 0.2).astype(np.float32),
            "truncated": np.zeros(B, np.float32),
            "discount": np.full(B, 0.99, np.float32),
        }
        noise = {
            "actor": rng.standard_normal((2 * B, act)).astype(np.float32),
            "next": rng.standard_normal((B, act)).astype(np.float32),
        }
        batches.append(batch)
        noises.append(noise)

    metrics_all = []
    for update in range(2):
        batch_t = {k: torch.from_numpy(v) for k, v in batches[update].items()}
        batch_t["actor_observation"] = batch_t["observation"][:, :obs_a]
        batch_t["actor_next_observation"] = batch_t["next_observation"][:, :obs_a]
        queue = []
        if update % cfg.actor_update_period == 0:
            queue.append(torch.from_numpy(noises[update]["actor"]))
        queue.append(torch.from_numpy(noises[update]["next"]))

        original = torch.distributions.Normal.rsample

        def rsample(self, sample_shape=torch.Size(), _q=queue):
            eps = _q.pop(0)
            assert tuple(eps.shape) == tuple(self.loc.shape)
            return self.loc + eps * self.scale

        torch.distributions.Normal.rsample = rsample
        try:
            info = _update_networks(batch_t, actor, critic, target, temp, cfg,
                                    do_actor_update=(update % cfg.actor_update_period == 0),
                                    device=torch.device("cpu"), grad_scaler=None)
        finally:
            torch.distributions.Normal.rsample = original
        assert not queue
        metrics_all.append({k: float(v) for k, v in info.items()})
        for tag, net in (("actor", actor), ("critic", critic), ("target", target), ("temp", temp)):
            for k, v in _state(net.network).items():
                out[f"after{update}.{tag}.{k}"] = v
        for tag, net in (("actor", actor), ("critic", critic), ("temp", temp)):
            for k, v in _moments(net).items():
                out[f"after{update}.opt.{tag}.{k}"] = v
        for k, v in batches[update].items():
            out[f"batch{update}.{k}"] = v
        for k, v in noises[update].items():
            out[f"noise{update}.{k}"] = v
        for k, v in metrics_all[-1].items():
            out[f"metrics{update}.{k}"] = np.array(v)
    for k, v in spec.items():
        out[f"spec.{k}"] = np.array(-1 if v is None else v)
    out["spec.target_entropy"] = np.array(target_entropy)
    np.savez_compressed(HERE / f"flashsac_update_{name}.npz", **out)
    print(f"flashsac_update_{name}: {len(out)} arrays, metrics {metrics_all}")


def make_categorical_case(name: str, batch: int, bins: int, min_v: float, max_v: float, seed: int) -> None:
    import torch

    from robolearn.flashsac.updates import _compute_categorical_td_target, _select_min_q_log_probs

    rng = np.random.default_rng(seed)
    target_logits = rng.standard_normal((2, batch, bins)).astype(np.float32)
    target_lp = torch.log_softmax(torch.from_numpy(target_logits), dim=-1)
    support = torch.linspace(min_v, max_v, bins)
    next_q = (target_lp.exp() * support).sum(-1)
    # force ties on a few rows: both twins equal -> argmin picks twin 0
    next_q[1, :3] = next_q[0, :3]
    reward = (4.0 * rng.standard_normal(batch)).astype(np.float32)
    reward[3] = 40.0   # clamps every atom to max_v
    reward[4] = -40.0  # clamps every atom to min_v
    done = (rng.random(batch) < 0.1).astype(np.float32)
    done[5] = 1.0
    discount = np.full(batch, 0.99, np.float32)
    discount[6] = 0.0
    next_lp = rng.standard_normal(batch).astype(np.float32)
    alpha = np.float32(0.01)
    entropy = torch.from_numpy(next_lp) * torch.tensor(alpha)
    selected = _select_min_q_log_probs(next_q, target_lp)
    target = _compute_categorical_td_target(
        target_log_probs=selected, reward=torch.from_numpy(reward), done=torch.from_numpy(done),
        actor_entropy=entropy, gamma=torch.from_numpy(discount), num_bins=bins, min_v=min_v, max_v=max_v,
    )
    online_logits = torch.from_numpy(rng.standard_normal((2, 2 * batch, bins)).astype(np.float32)).requires_grad_(True)
    pred_lp = torch.log_softmax(online_logits, dim=-1)
    ce = -(target.unsqueeze(0) * pred_lp[:, :batch]).sum(-1)
    loss = ce.mean()
    loss.backward()
    np.savez_compressed(
        HERE / f"categorical_{name}.npz",
        target_log_probs=target_lp.numpy(), next_q=next_q.numpy(), reward=reward, done=done,
        discount=discount, next_log_probs=next_lp, alpha=np.array(alpha), support=support.numpy(),
        selected=selected.numpy(), target=target.numpy(), online_logits=online_logits.detach().numpy(),
        loss=np.array(loss.item()), dlogits=online_logits.grad.numpy(), max_entropy=np.array(entropy.max().item()),
        min_v=np.array(min_v), max_v=np.array(max_v),
    )
    print(f"categorical_{name}: loss {loss.item():.6f}")


def make_replay_case() -> None:
    import torch

    from robolearn.flashsac.replay import TorchUniformBuffer

    Box = sys.modules["gymnasium"].spaces.Box
    replay = TorchUniformBuffer(
        observation_space=Box(-np.inf, np.inf, shape=(1,), dtype=np.float32),
        action_space=Box(-1.0, 1.0, shape=(1,), dtype=np.float32),
        n_step=3, gamma=0.5, max_length=16, min_length=3, sample_batch_size=3, device_type="cpu",
    )
    steps = []
    for step, rewards in enumerate(([1.0, 1.0, 1.0], [2.0, 2.0, 2.0], [100.0, 4.0, 100.0])):
        tr = {
            "observation": torch.tensor([[step * 10.0], [step * 10.0 + 1], [step * 10.0 + 2]]),
            "action": torch.zeros(3, 1),
            "reward": torch.tensor(rewards),
            "terminated": torch.tensor([False, False, step == 1]),
            "truncated": torch.tensor([step == 1, False, False]),
            "next_observation": torch.tensor([[(step + 1) * 10.0], [(step + 1) * 10.0 + 1], [(step + 1) * 10.0 + 2]]),
        }
        steps.append({k: v.numpy().astype(np.float32) for k, v in tr.items()})
        replay.add(tr)
    batch = replay.sample(np.array([0, 1, 2]))
    out = {f"step{i}.{k}": v for i, s in enumerate(steps) for k, v in s.items()}
    out.update({f"sample.{k}": v.numpy() for k, v in batch.items()})
    np.savez_compressed(HERE / "replay_nstep.npz", **out)
    print("replay_nstep:", {k: v.numpy().ravel().tolist() for k, v in batch.items()})


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--reference-src", required=True, help="path of the reference project's src directory")
    args = parser.parse_args()
    _install_gym_shim()
    sys.path.insert(0, args.reference_src)
    for name, spec in CASES.items():
        make_update_case(name, spec)
    make_categorical_case("b37", 37, 101, -10.0, 10.0, seed=1)
    make_categorical_case("b64_bins11", 64, 11, -5.0, 5.0, seed=2)
    make_replay_case()


if __name__ == "__main__":
    main()
