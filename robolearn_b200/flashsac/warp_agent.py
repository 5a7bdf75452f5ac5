"""``WarpFlashSAC`` on the B200 learner: drop-in for ``robolearn.warp.WarpFlashSAC``
(``src/robolearn/warp/flashsac.py:318-1239``).

Same constructor (keyword flags accepted and validated as in the reference; every
dense product runs on the tcgen05 GEMM whatever ``dense_backend`` says), Warp-NN's
Adam formula, and the reference's methods: ``parameters``, ``act`` / ``sample_actions`` /
``observe`` / ``process_transition`` / ``ready`` / ``can_start_training``,
``launch_update(do_actor_update, sample, randomize_noise, apply_optimizer,
normalize_reward)``, ``update_from_batch``, ``prepare`` (= ``warmup``), ``capture_update``,
``update(tensor_metrics, capture)``, ``get_metrics``, ``state_dict(include_replay)`` /
``load_state_dict``, ``save(path, include_replay)`` / ``load`` (``config.json`` +
``agent.npz``, format tag ``robolearn-warp-flashsac-v1``, the reference's key families:
``actor.* / critic.* / target_critic.*``, ``optimizer.<net>.m1.i / m2.i / timestep / lr``,
``log_temperature``, ``update_counters``, ``replay.*``, ``normalizer.*``,
``replay_storage_included``). The random streams are this implementation's Philox
counters (``rng.epoch``), not Warp's.
"""

from __future__ import annotations

import json
import warnings
from dataclasses import asdict
from pathlib import Path
from typing import Mapping

import numpy as np
import torch

from .agent import _ATTEMPTS, _GROWTH, _LR, _SCALE, _STEPS, FlashSAC
from .config import FlashSACConfig
from .learner import METRIC_KEYS

_FORMAT = "robolearn-warp-flashsac-v1"


class WarpFlashSAC(FlashSAC):
    """FlashSAC with the reference's Warp-class interface and Warp-NN Adam."""

    def __init__(self, observation_dim: int, action_dim: int, num_envs: int = 1, cfg: FlashSACConfig | None = None,
                 critic_observation_dim: int | None = None, *, optimized_linear_backward: bool = True,
                 dense_backend: str = "warp", fused_updates: bool = False, cuda_autotune: bool = False,
                 fresh_training_gradients: bool = False):
        if dense_backend not in ("warp", "cuda"):
            raise ValueError("dense_backend must be 'warp' or 'cuda'.")
        cfg = cfg or FlashSACConfig()
        if (cfg.use_amp or fused_updates or cuda_autotune) and dense_backend != "cuda":
            raise ValueError("Mixed precision, fused updates and CUDA plan tuning require dense_backend='cuda'.")
        if fresh_training_gradients and (dense_backend != "cuda" or not cfg.use_amp or not fused_updates):
            raise ValueError("Fresh training gradients require native CUDA, AMP and fused_updates=True.")
        if min(observation_dim, action_dim, num_envs) < 1:
            raise ValueError("Observation, action and environment dimensions must be positive.")
        if cfg.temp_initial_value <= 0 or cfg.temp_target_sigma <= 0 or cfg.actor_noise_zeta_max < 1:
            raise ValueError("Temperature and exploration distribution parameters must be positive.")
        if not 0 <= cfg.critic_target_update_tau <= 1:
            raise ValueError("Target EMA tau must lie in [0, 1].")
        if cfg.learning_rate_warmup_step < 0 or cfg.learning_rate_warmup_step >= cfg.learning_rate_decay_step:
            raise ValueError("Learning-rate warmup must be nonnegative and shorter than decay.")
        warnings.warn("WarpFlashSAC is experimental; policy quality and speed must be measured for your task.",
                      RuntimeWarning, stacklevel=2)
        super().__init__(observation_dim, action_dim, num_envs, cfg, critic_observation_dim, _adam_formula=1)
        self.config = self.cfg = self._cfg
        self.optimized_linear_backward = optimized_linear_backward
        self.dense_backend = dense_backend
        self.fused_updates = fused_updates
        self.cuda_autotune = cuda_autotune
        self.fresh_training_gradients = fresh_training_gradients
        self.observation_dim, self.action_dim, self.num_envs = observation_dim, action_dim, num_envs
        self.critic_observation_dim = self._critic_observation_dim
        self.compute_dtype = "float16" if self._cfg.precision == "fp16" else "float32"
        self._prepared = False
        self._feeds: dict[tuple, list] = {}

    # ------------------------------------------------------------------ views
    def parameters(self) -> list[torch.Tensor]:
        L = self._learner
        return ([L.actor.param(k) for k in L.actor.param_names] + [L.critic.param(k) for k in L.critic.param_names]
                + [L.log_temp])

    @property
    def batch(self) -> dict:
        """The learner's batch buffers in network layout (observation rows, actions, reward, flags)."""
        L = self._learner
        return {"critic_x": L.critic_x, "actor_x": L.actor_x, "reward": L.reward, "terminated": L.terminated,
                "truncated": L.truncated, "discount": L.discount}

    # ------------------------------------------------------------------ update API
    def _feed_program(self, sample: bool, randomize_noise: bool, normalize_reward: bool) -> list:
        key = (sample, randomize_noise, normalize_reward)
        if key not in self._feeds:
            from .sampling import sampling_program

            L = self._learner
            if sample:
                rs = self._reward_state if (normalize_reward and self._cfg.normalize_reward) else None
                prog = sampling_program(L, self._replay, rs, g_max=self._cfg.normalized_G_max, seed=self._cfg.seed,
                                        noise=randomize_noise)
            else:
                full = sampling_program(L, self._replay, None, seed=self._cfg.seed, noise=True)
                prog = [full[1], full[2]] if randomize_noise else []  # noise and its epoch advance only
            self._feeds[key] = prog
        return self._feeds[key]

    def launch_update(self, do_actor_update: bool = True, *, sample: bool = True, randomize_noise: bool = True,
                      apply_optimizer: bool = True, normalize_reward: bool = True) -> None:
        """Launch one learning phase on the current stream without host reads or phase bookkeeping."""
        for f in self._feed_program(sample, randomize_noise, normalize_reward):
            f()
        self._learner.run(do_actor_update, apply_optimizer)

    def update_from_batch(self, batch: Mapping, *, actor_noise=None, next_noise=None, do_actor_update: bool | None = None,
                          apply_optimizer: bool = True, normalize_reward: bool = False,
                          tensor_metrics: bool = True) -> dict:
        """One update on an explicit batch (keys observation, next_observation, action, reward,
        terminated, truncated, discount) and optionally prescribed noise of shapes (2B, A), (B, A)."""
        if (actor_noise is None) != (next_noise is None):
            raise ValueError("Supply both actor_noise and next_noise for fixed-noise diagnostics.")
        L = self._learner
        reward = None
        if normalize_reward and self._cfg.normalize_reward:
            st = self._reward_state
            r = torch.as_tensor(batch["reward"], dtype=torch.float32, device=self._device)
            denom = torch.maximum(torch.sqrt(st[1] + 1e-8), st[3] / self._cfg.normalized_G_max)
            reward = r / denom
        L.load_batch(batch, actor_noise, next_noise, reward=reward)
        phase = self._update_step % self._cfg.actor_update_period == 0 if do_actor_update is None else do_actor_update
        self.launch_update(phase, sample=False, randomize_noise=actor_noise is None, apply_optimizer=apply_optimizer,
                           normalize_reward=False)
        if apply_optimizer:
            self._update_step += 1
        return self._metrics(phase, tensor_metrics)

    def _metrics(self, actor_phase: bool, tensor_metrics: bool) -> dict:
        values = self._learner.metric_values(actor_phase)
        if tensor_metrics:
            return {k: v.detach().clone().reshape(1) for k, v in values.items()}
        vals = torch.stack(list(values.values())).cpu().tolist()
        return dict(zip(values.keys(), vals))

    def prepare(self, *, capture: bool = False) -> None:
        """Load every kernel for both phases on a dummy batch, keeping the training state."""
        if not self._prepared:
            state = self.state_dict(include_replay=False)
            try:
                L = self._learner
                for t in (L.critic_x, L.critic_x_pi, L.actor_x, L.reward, L.terminated, L.truncated):
                    t.zero_()
                L.discount.fill_(self._cfg.gamma ** self._cfg.n_step)
                obs = torch.zeros(self.num_envs, self._critic_observation_dim, device=self._device)
                self.act(obs, training=False)
                self.act(obs, training=True)
                for phase in (True, False):
                    self.launch_update(phase, sample=False)
                torch.cuda.synchronize(self._device)
                self._prepared = True
            finally:
                self.load_state_dict(state)
        if capture:
            self.capture_update()

    warmup = prepare

    def capture_update(self) -> None:
        """Record both learning phases (replay sampling included) as CUDA graphs without running them."""
        self.prepare(capture=False)
        L = self._learner
        for phase in (True, False):
            if phase not in self._graphs:
                self._graphs[phase] = L.capture(phase, pre=self._feed_program(True, True, True))

    def update(self, *, tensor_metrics: bool = False, capture: bool = True) -> dict:
        if not self.ready:
            raise RuntimeError("Replay has not reached buffer_min_length.")
        phase = self._update_step % self._cfg.actor_update_period == 0
        if capture:
            self.capture_update()
            self._graphs[phase].replay()
        else:
            self.launch_update(phase)
        self._update_step += 1
        return self._metrics(phase, tensor_metrics)

    def get_metrics(self) -> dict:
        L = self._learner
        res = self._metrics(True, False)
        res["actor_optimizer_steps"] = float(L.actor.opt_state[_STEPS].cpu())
        res["critic_optimizer_steps"] = float(L.critic.opt_state[_STEPS].cpu())
        res["temperature_optimizer_steps"] = float(L.temp_state[0].cpu())
        if self._cfg.precision == "fp16":
            for name, net in (("actor", L.actor), ("critic", L.critic)):
                st = net.opt_state.cpu().tolist()
                res[f"{name}_amp_loss_scale"] = st[_SCALE]
                res[f"{name}_optimizer_attempts"] = int(st[_ATTEMPTS])
                res[f"{name}_optimizer_skips"] = int(st[8])
        return res

    # ------------------------------------------------------------------ checkpoints
    def _state_arrays(self) -> dict[str, torch.Tensor]:
        """name -> device tensor view (restored in place, so captured graphs stay valid)."""
        L = self._learner
        arrays = {}
        for name, net in (("actor", L.actor), ("critic", L.critic), ("target_critic", L.target)):
            for k in net.param_names:
                arrays[f"{name}.{k}"] = net.param(k)
            for pre, _ in net.bn_layers:
                arrays[f"{name}.{pre}.running_mean"] = net.buffer(pre + ".running_mean")
                arrays[f"{name}.{pre}.running_var"] = net.buffer(pre + ".running_var")
        for name, net in (("actor", L.actor), ("critic", L.critic)):
            for i, k in enumerate(net.param_names):
                arrays[f"optimizer.{name}.m1.{i}"] = net.moment("m", k)
                arrays[f"optimizer.{name}.m2.{i}"] = net.moment("v", k)
            arrays[f"optimizer.{name}.state"] = net.opt_state
        arrays["optimizer.temperature.state"] = L.temp_state
        arrays["log_temperature"] = L.log_temp
        arrays["rng.epoch"] = self._replay.epoch
        arrays["exploration.cached_noise"] = self._cached_noise
        return arrays

    def state_dict(self, include_replay: bool = True) -> dict[str, np.ndarray]:
        """Weights, BN buffers, optimizer state, RNG counters, normaliser and replay."""
        state = {k: v.detach().cpu().numpy().copy() for k, v in self._state_arrays().items()}
        L = self._learner
        for name, net in (("actor", L.actor), ("critic", L.critic)):
            st = net.opt_state.cpu().numpy()
            state[f"optimizer.{name}.timestep"] = st[_STEPS:_STEPS + 1].copy()
            state[f"optimizer.{name}.lr"] = st[_LR:_LR + 1].copy()
        state["optimizer.temperature.timestep"] = L.temp_state[:1].cpu().numpy().copy()
        state["update_counters"] = np.array([self._update_step], dtype=np.int64)
        state["exploration.repetition"] = np.array([int(self._cur_noise_repeat_count), int(self._cur_noise_repeat_n)],
                                                   dtype=np.int32)
        rep = self._replay.state()
        for k, v in rep.items():
            if include_replay or k in ("num_in_buffer", "current_idx"):
                state[f"replay.{k}"] = torch.as_tensor(v).cpu().numpy()
        state["normalizer.state"] = self._reward_state.cpu().numpy().copy()
        state["normalizer.returns"] = self._g_r.cpu().numpy().copy()
        state["replay_storage_included"] = np.array([include_replay], dtype=np.bool_)
        return state

    def load_state_dict(self, state: Mapping) -> None:
        """Restore in place; replay storage only when the checkpoint includes it."""
        arrays = self._state_arrays()
        for k, a in arrays.items():
            if k not in state or tuple(np.shape(state[k])) != tuple(a.shape):
                raise ValueError(f"Checkpoint array {k} is missing or has the wrong shape.")
        for k, a in arrays.items():
            a.copy_(torch.as_tensor(np.asarray(state[k])).to(a.dtype))
        L = self._learner
        for net in (L.actor, L.critic, L.target):
            net.refresh_planes()
        if self._cfg.precision == "fp16":
            for name, net in (("actor", L.actor), ("critic", L.critic)):
                sc = L.scalers[name]
                scale = float(net.opt_state[_SCALE])
                sc.scale.fill_(scale)
                sc.inv_scale.fill_(1.0 / scale)
        self._update_step = int(np.asarray(state["update_counters"])[0])
        rep = np.asarray(state["exploration.repetition"])
        self._cur_noise_repeat_count.fill_(int(rep[0]))
        self._cur_noise_repeat_n.fill_(int(rep[1]))
        if bool(np.asarray(state["replay_storage_included"])[0]):
            self._replay.load({k[len("replay."):]: torch.as_tensor(np.asarray(v)) for k, v in state.items()
                               if k.startswith("replay.")})
        self._reward_state.copy_(torch.as_tensor(np.asarray(state["normalizer.state"])))
        self._g_r.copy_(torch.as_tensor(np.asarray(state["normalizer.returns"])))

    def save(self, path: str | Path, *, include_replay: bool = False) -> None:
        """``config.json`` + ``agent.npz`` (replay storage only with include_replay)."""
        directory = Path(path)
        directory.mkdir(parents=True, exist_ok=True)
        meta = {"format": _FORMAT, "precision": self.compute_dtype, "observation_dim": self.observation_dim,
                "action_dim": self.action_dim,
                "critic_observation_dim": self.critic_observation_dim if self._cfg.asymmetric_observation else None,
                "num_envs": self.num_envs, "config": asdict(self._cfg),
                "optimized_linear_backward": self.optimized_linear_backward, "dense_backend": self.dense_backend,
                "fused_updates": self.fused_updates, "cuda_autotune": self.cuda_autotune,
                "fresh_training_gradients": self.fresh_training_gradients, "replay_included": include_replay}
        with (directory / "config.json").open("w") as f:
            json.dump(meta, f, indent=2)
            f.write("\n")
        with (directory / "agent.npz").open("wb") as f:
            np.savez(f, **self.state_dict(include_replay=include_replay))

    def load(self, path: str | Path) -> None:
        directory = Path(path)
        meta = json.loads((directory / "config.json").read_text())
        if meta.get("format") != _FORMAT:
            raise ValueError("Unrecognized WarpFlashSAC checkpoint format.")
        if meta["observation_dim"] != self.observation_dim or meta["action_dim"] != self.action_dim:
            raise ValueError("Checkpoint observation/action dimensions differ from this agent.")
        if (meta["critic_observation_dim"] or meta["observation_dim"]) != self.critic_observation_dim:
            raise ValueError("Checkpoint critic observation dimension differs from this agent.")
        if meta.get("precision", "float32") != self.compute_dtype and self._cfg.load_optimizer:
            raise ValueError("Switching checkpoint dense precision requires load_optimizer=False.")
        with np.load(directory / "agent.npz", allow_pickle=False) as archive:
            state = dict(archive)
        if meta["replay_included"] and meta["num_envs"] != self.num_envs:
            raise ValueError("Exact replay continuation requires the original num_envs.")
        current = self.state_dict(include_replay=False)
        if not meta["replay_included"]:
            self._replay.reset()
            state["normalizer.returns"] = np.zeros(self.num_envs, dtype=np.float32)
            state["exploration.cached_noise"] = current["exploration.cached_noise"]
        if not self._cfg.load_optimizer:
            state.update({k: v for k, v in current.items() if k.startswith("optimizer.")})
            state["update_counters"] = current["update_counters"]
        if not self._cfg.load_reward_normalizer:
            state["normalizer.state"] = current["normalizer.state"]
        self.load_state_dict(state)


__all__ = ["WarpFlashSAC", "FlashSACConfig", "METRIC_KEYS"]
