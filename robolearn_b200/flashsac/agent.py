"""Reference-facing FlashSAC agent on the B200 learner.

Mirrors ``FlashSAC`` (src/robolearn/flashsac/agent.py:294-601): the same constructor
and validation, ``act`` / ``observe`` / ``process_transition`` / ``sample_actions`` /
``update`` / ``save`` / ``load`` / ``save_replay_buffer`` / ``load_replay_buffer`` /
``ready`` / ``can_start_training`` / ``get_metrics``, the same metric keys and the
same checkpoint files (``config.json``, ``actor.pt``, ``critic.pt``,
``target_critic.pt``, ``temperature.pt``, ``agent_state.pt``,
``reward_normalizer.pt``; per-network ``network_state_dict`` /
``optimizer_state_dict`` (torch Adam layout) / ``scheduler_state_dict`` (LambdaLR) /
``update_step``, ``src/robolearn/flashsac/_utils/network.py:115-150``).

Every update runs the sm_100a kernels: the replay sampling / gather / noise launches
and the learner program of the phase, recorded as one CUDA graph per phase after a
first eager pass. Exploration actions (``act``) run the actor forward with eval-mode
batch norm and the fused policy kernel. There is no CPU path: the learner refuses a
non-CUDA device and the kernels fail loudly when the library is missing.
"""

from __future__ import annotations

import json
import math
import os
from dataclasses import asdict, replace
from typing import Any, MutableMapping

import torch

from .. import _native as N
from ..categorical import support
from .config import FlashSACConfig
from .engine import Run
from .learner import METRIC_KEYS, Learner
from .replay import DeviceReplay
from .sampling import sampling_program

# optimizer state layout of each network: [attempts, steps, step_size, bc2, lr, skip, scale, growth, skipped]
_ATTEMPTS, _STEPS, _LR, _SCALE, _GROWTH = 0, 1, 4, 6, 7
_BETAS = (0.9, 0.999)
_EPS = 1e-8
_RMS_EPSILON = 1e-4  # RunningMeanStd count epsilon (reward_normalization.py:171)


def truncated_zeta_cdf(mu: float, max_n: int) -> torch.Tensor:
    """CDF of the zeta(mu) law truncated to 1..max_n (agent.py:159-167)."""
    ns = torch.arange(1, max_n + 1, dtype=torch.float32)
    pmf = ns ** (-mu)
    pmf = pmf / torch.sum(pmf)
    return torch.cumsum(pmf, dim=0)


def _adam_state_dict(m: list[torch.Tensor], v: list[torch.Tensor], steps: float, lr: float, initial_lr: float) -> dict:
    """torch.optim.Adam state_dict layout for parameters 0..n-1 (one param group)."""
    state = {i: {"step": torch.tensor(float(steps)), "exp_avg": m[i].clone(), "exp_avg_sq": v[i].clone()}
             for i in range(len(m))} if steps > 0 else {}
    # fused: the reference builds Adam(fused=True) on CUDA devices (agent.py:64-65)
    group = {"lr": lr, "betas": _BETAS, "eps": _EPS, "weight_decay": 0, "amsgrad": False, "maximize": False,
             "foreach": None, "capturable": False, "differentiable": False, "fused": True, "decoupled_weight_decay": False,
             "initial_lr": initial_lr, "params": list(range(len(m)))}
    return {"state": state, "param_groups": [group]}


def _schedule_lr(cfg: FlashSACConfig, steps: float) -> float:
    """The learning rate the reference's optimisers hold after ``steps`` scheduler steps:
    LambdaLR multiplies the optimiser's initial rate (learning_rate_peak) by
    warmup_cosine_decay_lr(steps) / learning_rate_peak (agent.py:64-69,
    _utils/scheduler.py:43-65), in Python floats."""
    k = int(steps)
    init, peak, end = cfg.learning_rate_init, cfg.learning_rate_peak, cfg.learning_rate_end
    w, d = cfg.learning_rate_warmup_step, cfg.learning_rate_decay_step
    if k < w:
        v = init + (peak - init) * (k / w)
    elif k < d:
        v = end + (peak - end) * 0.5 * (1 + math.cos(math.pi * ((k - w) / (d - w))))
    else:
        v = end
    return peak * (v / peak)


def _scheduler_state_dict(attempts: float, lr: float, base_lr: float) -> dict:
    """LambdaLR state_dict layout (the lambda itself is not serialised by torch either)."""
    n = int(attempts)
    return {"base_lrs": [base_lr], "last_epoch": n, "_step_count": n + 1, "_is_initial": False,
            "_get_lr_called_within_step": False, "_last_lr": [lr], "lr_lambdas": [None]}


class FlashSAC:
    """Tensor agent for a vectorized environment (actions in normalised [-1, 1])."""

    def __init__(self, observation_dim: int, action_dim: int, num_envs: int = 1, cfg: FlashSACConfig | None = None,
                 critic_observation_dim: int | None = None, *, _adam_formula: int = 0):
        cfg = cfg or FlashSACConfig()
        if min(observation_dim, action_dim, num_envs) <= 0:
            raise ValueError("Observation, action, and environment dimensions must be positive.")
        if num_envs > cfg.buffer_max_length:
            raise ValueError("Replay capacity must fit one vector environment step.")
        total_dim = critic_observation_dim or observation_dim
        if total_dim < observation_dim:
            raise ValueError("Critic observations must contain the actor observation prefix.")
        cfg = replace(cfg, asymmetric_observation=critic_observation_dim is not None)
        target_entropy = 0.5 * action_dim * math.log(2 * math.pi * math.e * cfg.temp_target_sigma**2)
        cfg = replace(cfg, temp_target_entropy=target_entropy)
        self._cfg = cfg
        self._num_envs = num_envs
        self._actor_observation_dim = observation_dim
        self._critic_observation_dim = total_dim
        self._action_dim = action_dim
        device = torch.device(cfg.device_type)
        if device.type != "cuda":
            raise RuntimeError("the B200 FlashSAC learner runs on a CUDA device only")
        if device.index is None:
            device = torch.device("cuda", torch.cuda.current_device())
        self._device = device
        torch.manual_seed(cfg.seed)
        self._learner = L = Learner(observation_dim, total_dim, action_dim, cfg, device, adam_formula=_adam_formula)
        self._replay = DeviceReplay(total_dim, action_dim, num_envs, cfg.buffer_max_length, cfg.n_step, cfg.gamma,
                                    cfg.buffer_min_length, device, seed=cfg.seed)
        f32 = dict(dtype=torch.float32, device=device)
        # reward normaliser: [mean, var, count, G_r_max] of the discounted-return statistics + G_r per env
        self._reward_state = torch.tensor([0.0, 1.0, 0.0, 0.0], **f32)
        self._g_r = torch.zeros(num_envs, **f32)
        self._feed = sampling_program(L, self._replay, self._reward_state if cfg.normalize_reward else None,
                                      g_max=cfg.normalized_G_max, seed=cfg.seed)
        self._graphs: dict[bool, torch.cuda.CUDAGraph] = {}
        self._update_step = 0
        # exploration noise repetition (agent.py:382-389)
        self._zeta_cdf = truncated_zeta_cdf(cfg.actor_noise_zeta_mu, cfg.actor_noise_zeta_max).to(device)
        self._cur_noise_repeat_n = torch.tensor(1, dtype=torch.int32, device=device)
        self._cur_noise_repeat_count = torch.tensor(0, dtype=torch.int32, device=device)
        self._cached_noise = torch.randn(num_envs, action_dim, **f32)
        self._act_runs: dict[int, tuple] = {}

    # ------------------------------------------------------------------ acting
    def _act_run(self, rows: int) -> tuple:
        entry = self._act_runs.get(rows)
        if entry is None:
            L, A = self._learner, self._action_dim
            f32 = dict(dtype=torch.float32, device=self._device)
            x = torch.zeros(rows, L.ldax, **f32)
            run = Run(L.actor, rows, False, x.data_ptr(), L.ldax, update_running=False, need_param_grads=False,
                      need_input_grad=False)
            actions = torch.zeros(rows, A, **f32)
            log_pi = torch.zeros(rows, **f32)
            noise = torch.zeros(rows, A, **f32)
            args = L._policy_args(run, rows, noise, actions.data_ptr(), A, log_pi)
            entry = (x, run, actions, noise, args, log_pi)  # args hold raw pointers into these
            self._act_runs[rows] = entry
        return entry

    def sample_actions(self, interaction_step: int, prev_transition: MutableMapping[str, torch.Tensor],
                       training: bool) -> torch.Tensor:
        """tanh(mean + std * noise * temperature) from the actor in eval mode (agent.py:180-214, 400-444);
        temperature 1 while training (noise held for a zeta-distributed number of calls), else 0."""
        import ctypes

        obs = prev_transition["next_observation"]
        if self._cfg.asymmetric_observation:
            obs = obs[:, : self._actor_observation_dim]
        obs = torch.as_tensor(obs, dtype=torch.float32).to(self._device)
        rows = obs.shape[0]
        x, run, actions, noise, args, _ = self._act_run(rows)
        lib = self._learner.lib
        with torch.no_grad():
            x[:, : self._actor_observation_dim].copy_(obs)
            self._learner.actor.eval_prepare()
            for f in run.forward_program:
                f()
            if not training:
                N.check(lib.rl2_policy_sample(ctypes.byref(args), 1, N.stream_ptr()), "deterministic actions")
                return actions.clone()
            reinit = (self._cur_noise_repeat_count == 0) | (self._cur_noise_repeat_count >= self._cur_noise_repeat_n)
            new_noise = torch.randn_like(self._cached_noise)
            u = torch.rand((), device=self._device)
            new_n = (torch.argmax((u < self._zeta_cdf).to(torch.int32)) + 1).to(torch.int32)
            self._cached_noise = torch.where(reinit, new_noise, self._cached_noise)
            self._cur_noise_repeat_n = torch.where(reinit, new_n, self._cur_noise_repeat_n)
            self._cur_noise_repeat_count = torch.where(reinit, torch.zeros_like(self._cur_noise_repeat_count),
                                                       self._cur_noise_repeat_count)
            noise.copy_(self._cached_noise.expand(rows, -1) if self._cached_noise.shape[0] == 1 else self._cached_noise)
            N.check(lib.rl2_policy_sample(ctypes.byref(args), 0, N.stream_ptr()), "sample actions")
            self._cur_noise_repeat_count = self._cur_noise_repeat_count + 1
        return actions.clone()

    def act(self, observations: torch.Tensor, training: bool = True) -> torch.Tensor:
        """Return normalized actions on the agent device."""
        return self.sample_actions(0, {"next_observation": observations}, training)

    # ------------------------------------------------------------------ ingest
    def process_transition(self, transition: MutableMapping[str, torch.Tensor]) -> None:
        dev = self._device
        t = lambda k: torch.as_tensor(transition[k], dtype=torch.float32, device=dev)  # noqa: E731
        reward, term, trunc = t("reward").reshape(-1), t("terminated").reshape(-1), t("truncated").reshape(-1)
        self._replay.add(t("observation"), t("action"), reward, term, trunc, t("next_observation"))
        if self._cfg.normalize_reward:
            if reward.numel() != self._num_envs:
                raise ValueError(f"expected {self._num_envs} rewards per step, got {reward.numel()}")
            N.check(self._learner.lib.rl2_reward_stats_update(
                reward.data_ptr(), term.data_ptr(), trunc.data_ptr(), None, None, self._g_r.data_ptr(),
                self._num_envs, self._cfg.gamma, self._reward_state.data_ptr(), _RMS_EPSILON, N.stream_ptr()),
                "reward statistics")

    def observe(self, observations, actions, rewards, terminated, truncated, next_observations) -> None:
        """Store transitions; next_observations must precede automatic reset on done rows."""
        self.process_transition({"observation": observations, "action": actions, "reward": rewards,
                                 "terminated": terminated, "truncated": truncated,
                                 "next_observation": next_observations})

    def can_start_training(self) -> bool:
        return self._replay.can_sample()

    @property
    def ready(self) -> bool:
        """Whether the replay buffer has enough samples for an update."""
        return self.can_start_training()

    # ------------------------------------------------------------------ update
    def update(self, *, tensor_metrics: bool = False) -> dict[str, Any]:
        """One replay update (actor + temperature + critic every ``actor_update_period`` calls, else critic).

        ``tensor_metrics=True`` returns device scalars (no host read)."""
        if not self._replay.can_sample():
            raise RuntimeError("the replay buffer holds fewer than buffer_min_length transitions")
        phase = self._update_step % self._cfg.actor_update_period == 0
        L = self._learner
        graph = self._graphs.get(phase)
        if graph is None:
            for f in self._feed:
                f()
            L.run(phase)
            self._graphs[phase] = L.capture(phase, pre=self._feed)
        else:
            graph.replay()
        self._update_step += 1
        metrics = L.metric_values(phase)
        if tensor_metrics:
            return {k: v.detach().clone() for k, v in metrics.items()}
        values = torch.stack(list(metrics.values())).cpu().tolist()
        return dict(zip(metrics.keys(), values))

    def get_metrics(self) -> dict[str, Any]:
        return {}

    # ------------------------------------------------------------------ checkpoints
    def _network_ckpt(self, net, optimised: bool) -> dict:
        peak = self._cfg.learning_rate_peak
        # the reference's Network.update_step is never advanced by an update; it is whatever was
        # loaded (0 for a fresh agent), and is written back as such
        state = net.state_dict()
        if net.spec.critic:  # the categorical head's support buffer (layers.py:289-292), saved by the reference
            cfg = self._cfg
            state["predictor.bin_values"] = torch.from_numpy(
                support(cfg.critic_num_bins, cfg.critic_min_v, cfg.critic_max_v)).reshape(1, 1, -1)
        ckpt = {"network_state_dict": state, "optimizer_state_dict": None, "scheduler_state_dict": None,
                "update_step": getattr(net, "ckpt_update_step", 0)}
        if optimised:
            st = net.opt_state.cpu().tolist()
            m = [net.moment("m", k) for k in net.param_names]
            v = [net.moment("v", k) for k in net.param_names]
            lr = _schedule_lr(self._cfg, st[_ATTEMPTS])
            ckpt["optimizer_state_dict"] = _adam_state_dict(m, v, st[_STEPS], lr, peak)
            ckpt["scheduler_state_dict"] = _scheduler_state_dict(st[_ATTEMPTS], lr, peak)
        return ckpt

    def _temperature_ckpt(self) -> dict:
        peak = self._cfg.learning_rate_peak
        step, m, v = self._learner.temp_state.cpu().tolist()
        lr = _schedule_lr(self._cfg, step)  # the temperature shares the schedule, one step per actor update
        return {"network_state_dict": {"log_temp": self._learner.log_temp.detach().clone()},
                "optimizer_state_dict": _adam_state_dict([torch.tensor([m])], [torch.tensor([v])], step, lr, peak),
                "scheduler_state_dict": _scheduler_state_dict(step, lr, peak),
                "update_step": getattr(self._learner, "temp_ckpt_update_step", 0)}

    def save(self, path: str) -> None:
        os.makedirs(path, exist_ok=True)
        metadata = {
            "observation_dim": self._actor_observation_dim,
            "critic_observation_dim": self._critic_observation_dim if self._cfg.asymmetric_observation else None,
            "action_dim": self._action_dim,
            "config": asdict(self._cfg),
        }
        with open(os.path.join(path, "config.json"), "w") as stream:
            json.dump(metadata, stream, indent=2)
            stream.write("\n")
        L = self._learner
        torch.save(self._network_ckpt(L.actor, True), os.path.join(path, "actor.pt"))
        torch.save(self._network_ckpt(L.critic, True), os.path.join(path, "critic.pt"))
        torch.save(self._network_ckpt(L.target, False), os.path.join(path, "target_critic.pt"))
        torch.save(self._temperature_ckpt(), os.path.join(path, "temperature.pt"))
        if self._cfg.normalize_reward:
            mean, var, count, g_max = self._reward_state.detach().clone()
            torch.save({"G_r": self._g_r.detach().clone(), "G_r_max": g_max.reshape(1), "G_rms_mean": mean.reshape(1),
                        "G_rms_var": var.reshape(1), "G_rms_count": count}, os.path.join(path, "reward_normalizer.pt"))
        st = L.critic.opt_state.cpu().tolist()
        scaler = ({"scale": st[_SCALE], "growth_factor": 2.0, "backoff_factor": 0.5, "growth_interval": 2000,
                   "_growth_tracker": int(st[_GROWTH])} if self._cfg.precision == "fp16" else {})
        torch.save({"update_step": self._update_step, "grad_scaler_state_dict": scaler},
                   os.path.join(path, "agent_state.pt"))

    def _load_network(self, net, ckpt: dict, load_optimizer: bool) -> None:
        state = {k.removeprefix("_orig_mod."): v for k, v in ckpt["network_state_dict"].items()}
        net.load_state_dict(state)
        if load_optimizer:
            net.ckpt_update_step = int(ckpt.get("update_step", 0))
        opt = ckpt.get("optimizer_state_dict")
        if load_optimizer and opt is not None and getattr(net, "with_optimizer", False):
            for i, k in enumerate(net.param_names):
                s = opt["state"].get(i)
                net.moment("m", k).copy_(s["exp_avg"].reshape(net.shapes[k]) if s else 0.0)
                net.moment("v", k).copy_(s["exp_avg_sq"].reshape(net.shapes[k]) if s else 0.0)
            steps = float(opt["state"][0]["step"]) if opt["state"] else 0.0
            sched = ckpt.get("scheduler_state_dict") or {}
            st = net.opt_state
            st[_STEPS] = steps
            st[_ATTEMPTS] = float(sched.get("last_epoch", steps))
            st[_LR] = float(opt["param_groups"][0]["lr"])

    def load(self, path: str) -> None:
        load_optimizer = self._cfg.load_optimizer
        dev = self._device
        L = self._learner
        rd = lambda name: torch.load(os.path.join(path, name), map_location=dev, weights_only=False)  # noqa: E731
        self._load_network(L.actor, rd("actor.pt"), load_optimizer)
        self._load_network(L.critic, rd("critic.pt"), load_optimizer)
        self._load_network(L.target, rd("target_critic.pt"), False)
        temp = rd("temperature.pt")
        L.log_temp.copy_(temp["network_state_dict"]["log_temp"].reshape(1))
        if load_optimizer:
            L.temp_ckpt_update_step = int(temp.get("update_step", 0))
        opt = temp.get("optimizer_state_dict")
        if load_optimizer and opt is not None and opt["state"]:
            s = opt["state"][0]
            L.temp_state.copy_(torch.tensor([float(s["step"]), float(s["exp_avg"].reshape(-1)[0]),
                                             float(s["exp_avg_sq"].reshape(-1)[0])]))
        if load_optimizer:
            agent_state = rd("agent_state.pt")
            self._update_step = int(agent_state["update_step"])
            sc = agent_state.get("grad_scaler_state_dict") or {}
            if sc and self._cfg.precision == "fp16":
                for net, name in ((L.actor, "actor"), (L.critic, "critic")):
                    net.opt_state[_SCALE] = float(sc["scale"])
                    net.opt_state[_GROWTH] = float(sc.get("_growth_tracker", 0))
                    scaler = L.scalers[name]
                    scaler.scale.fill_(float(sc["scale"]))
                    scaler.inv_scale.fill_(1.0 / float(sc["scale"]))
        if self._cfg.load_reward_normalizer and self._cfg.normalize_reward:
            rn = rd("reward_normalizer.pt")
            self._reward_state.copy_(torch.stack([rn["G_rms_mean"].reshape(()), rn["G_rms_var"].reshape(()),
                                                  torch.as_tensor(rn["G_rms_count"], device=dev).reshape(()),
                                                  rn["G_r_max"].reshape(())]).float())
            self._g_r.zero_()

    def save_replay_buffer(self, path: str) -> None:
        torch.save(self._replay.state(), os.path.join(path, "replay_buffer.pt"))

    def load_replay_buffer(self, path: str) -> None:
        self._replay.load(torch.load(os.path.join(path, "replay_buffer.pt"), map_location=self._device,
                                     weights_only=False))

    # ------------------------------------------------------------------ views
    @property
    def learner(self) -> Learner:
        return self._learner

    @property
    def replay(self) -> DeviceReplay:
        return self._replay


__all__ = ["FlashSAC", "FlashSACConfig", "METRIC_KEYS", "truncated_zeta_cdf"]
