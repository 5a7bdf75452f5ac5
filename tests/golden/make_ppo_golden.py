"""PPO oracle pin: run the reference's own controlled-update check against the oracle.

The reference checks its Warp PPO update against a Torch restatement of the same RSL-style
update (``examples/diagnose_ppo_update.py``: fixed rollout, device permutation, adaptive
KL schedule, separate gradient clipping, Adam; thresholds at ``:197-206``). Warp is absent
here, so this script runs that file's ``main()`` unchanged with two stand-ins registered
first:

* ``warp``: ``init`` / ``synchronize`` do nothing;
* ``robolearn.warp``: ``PPOConfig`` is this repository's drop-in record, and ``WarpPPO``
  is a small agent whose arrays are numpy arrays and whose ``compute_returns`` /
  ``launch_update`` / ``update`` run the numpy oracle (``oracle/ppo_np.py``) with a fixed
  permutation that it reports as its device shuffle.

Torch tensors the script places on ``"cuda"`` are placed on the CPU. The reference's Torch
half then recomputes the update and compares every returned quantity with the oracle at
its own thresholds (it raises if any is missed). Written to ``ppo_controlled_update.npz``:
the inputs (initial parameters, rollout, permutation), the Torch half's final parameters,
Adam moments and learning rate, and the reference's reported errors, so
``tests/test_oracle_ppo.py`` re-checks the oracle without the reference.

    python tests/golden/make_ppo_golden.py --reference <reference project root>
"""

from __future__ import annotations

import argparse
import json
import runpy
import sys
import tempfile
import types
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))

from oracle import ppo_np as P  # noqa: E402
from robolearn_b200.ppo.config import PPOConfig  # noqa: E402

PERMUTATION_SEED = 7


class _Array:
    """Numpy stand-in for a Warp array: ``assign`` and ``numpy``."""

    def __init__(self, a):
        self.a = np.array(a)

    def assign(self, v):
        self.a[...] = np.asarray(v, dtype=self.a.dtype).reshape(self.a.shape)

    def numpy(self):
        return self.a.copy()


class _Net:
    """A network of the agent: called on an array, and its parameter list."""

    def __init__(self, params, activation):
        self.params, self.activation = params, activation

    def __call__(self, x):
        return _Array(P.mlp_forward(self.params, x.numpy(), self.activation)[0].astype(np.float32))

    def parameters(self):
        return list(self.params)


class OracleWarpPPO:
    """The slice of ``WarpPPO``'s interface the controlled-update check uses, on the oracle."""

    record: list = []

    def __init__(self, observation_dim, action_dim, num_envs, horizon, config):
        self.config = config
        self.observation_dim, self.action_dim = observation_dim, action_dim
        self.num_envs, self.horizon = num_envs, horizon
        self.batch_size = num_envs * horizon
        self.mini_batch_size = self.batch_size // config.num_mini_batches
        self.h = P.PPOHyper(**{k: getattr(config, k) for k in P.PPOHyper.__dataclass_fields__})
        self.initial = P.init_params(observation_dim, action_dim, self.h, seed=config.seed)
        self.state = P.PPOState.fresh(self.initial, config.learning_rate)
        B, O, A = self.batch_size, observation_dim, action_dim
        f32 = lambda *s: _Array(np.zeros(s, np.float32))  # noqa: E731
        self.observations, self.actions, self.means, self.stds = f32(B, O), f32(B, A), f32(B, A), f32(B, A)
        for name in ("values", "log_probs", "rewards", "next_values", "returns", "advantages"):
            setattr(self, name, f32(B))
        self.terminated, self.truncated = _Array(np.zeros(B, np.int32)), _Array(np.zeros(B, np.int32))
        self.perm = np.random.default_rng(PERMUTATION_SEED).permutation(B)
        self._shuffle_indices = _Array(np.concatenate([self.perm, self.perm]).astype(np.int32))
        actor, critic, _ = P.split(self.state.params, tuple(config.hidden_dims))
        self.actor, self.critic = _Net(actor, config.activation), _Net(critic, config.activation)
        OracleWarpPPO.record.append(self)

    @property
    def parameters(self):
        return list(self.state.params)

    def _data(self):
        keys = ("observations", "actions", "means", "stds", "values", "log_probs", "rewards", "next_values",
                "terminated", "truncated")
        return {k: getattr(self, k).numpy() for k in keys}

    def state_dict(self):
        n = len(self.state.params)
        out = {f"parameter_{i}": np.asarray(self.state.params[i], np.float32) for i in range(n)}
        out.update({f"adam_m1_{i}": np.asarray(self.state.m1[i], np.float32) for i in range(n)})
        out.update({f"adam_m2_{i}": np.asarray(self.state.m2[i], np.float32) for i in range(n)})
        return out

    def load_state_dict(self, state):
        n = len(self.state.params)
        self.state = P.PPOState([np.asarray(state[f"parameter_{i}"], np.float64) for i in range(n)],
                                [np.asarray(state[f"adam_m1_{i}"], np.float64) for i in range(n)],
                                [np.asarray(state[f"adam_m2_{i}"], np.float64) for i in range(n)], 0,
                                self.config.learning_rate)

    def compute_returns(self):
        adv, ret = P.returns_and_advantages(self._data(), self.horizon, self.num_envs, self.h)
        self.advantages.assign(adv)
        self.returns.assign(ret)

    def launch_update(self):
        out = P.update(self.state, self._data(), self.horizon, self.num_envs, self.h, permutation=self.perm)
        self.advantages.assign(out["advantages"])
        self.returns.assign(out["returns"])

    def update(self, capture=True):
        self.launch_update()

    def health_metrics(self):
        return {"learning_rate": float(self.state.lr), "optimizer_updates": int(self.state.timestep)}


def _cpu_only(torch):
    """Place tensors the script creates on ``"cuda"`` on the CPU instead."""
    def wrap(fn):
        def inner(*a, **kw):
            if str(kw.get("device", "")).startswith("cuda"):
                kw["device"] = "cpu"
            return fn(*a, **kw)
        return inner

    torch.tensor = wrap(torch.tensor)
    torch.zeros = wrap(torch.zeros)


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--reference", required=True, help="the reference project's root directory")
    args = parser.parse_args()
    import torch

    _cpu_only(torch)
    optimizers = []
    adam = torch.optim.Adam

    class RecordingAdam(adam):
        def __init__(self, *a, **kw):
            super().__init__(*a, **kw)
            optimizers.append(self)

    torch.optim.Adam = RecordingAdam
    warp = types.ModuleType("warp")
    warp.init = lambda: None
    warp.synchronize = lambda: None
    robolearn = types.ModuleType("robolearn")
    rwarp = types.ModuleType("robolearn.warp")
    rwarp.PPOConfig, rwarp.WarpPPO = PPOConfig, OracleWarpPPO
    robolearn.warp = rwarp
    sys.modules.update({"warp": warp, "robolearn": robolearn, "robolearn.warp": rwarp})
    script = Path(args.reference) / "examples" / "diagnose_ppo_update.py"
    with tempfile.TemporaryDirectory() as tmp:
        report = Path(tmp) / "report.json"
        sys.argv = [str(script), "--output", str(report)]
        runpy.run_path(str(script), run_name="__diagnose__")["main"]()
        result = json.loads(report.read_text())
    agent = OracleWarpPPO.record[0]
    opt = optimizers[-1]
    params = opt.param_groups[0]["params"]
    out = {f"initial.{i}": np.asarray(p, np.float32) for i, p in enumerate(agent.initial)}
    out.update({f"data.{k}": v for k, v in agent._data().items()})
    out["permutation"] = agent.perm
    for i, p in enumerate(params):
        out[f"torch.parameter.{i}"] = p.detach().numpy().copy()
        out[f"torch.exp_avg.{i}"] = opt.state[p]["exp_avg"].numpy().copy()
        out[f"torch.exp_avg_sq.{i}"] = opt.state[p]["exp_avg_sq"].numpy().copy()
    out["torch.learning_rate"] = np.array(result["torch_learning_rate"])
    out["torch.last_kl"] = np.array(result["torch_last_kl"])
    for k in ("returns_max_abs_error", "advantages_max_abs_error", "torch_warp_parameters_max_abs_error",
              "torch_warp_adam_moments_max_abs_error"):
        out[f"report.{k}"] = np.array(result[k])
    np.savez_compressed(HERE / "ppo_controlled_update.npz", **out)
    print(json.dumps({k: result[k] for k in result if k not in ("warp_health",)}, indent=1))


if __name__ == "__main__":
    main()
