"""Device replay for the FlashSAC learner: n-step ingest, sampling and gather.

Storage follows ``TorchUniformBuffer`` (``src/robolearn/flashsac/replay.py:36-97``):
``[capacity, dim]`` fp32 rows of observation, next_observation, action and
``[capacity]`` reward / terminated / truncated / discount. Ingest, sampling and
gather are ``librl2`` kernels; the save / load format is the reference's
``replay_buffer.pt`` dictionary (``replay.py:196-240``).
"""

from __future__ import annotations

import ctypes

import torch

from .. import _native as N


class DeviceReplay:
    def __init__(self, obs_dim: int, act_dim: int, num_envs: int, capacity: int, n_step: int, gamma: float,
                 min_length: int, device, seed: int = 0):
        self.obs_dim, self.act_dim, self.num_envs = obs_dim, act_dim, num_envs
        self.capacity, self.n_step, self.gamma, self.min_length = capacity, n_step, gamma, min_length
        self.device = torch.device(device)
        self.seed = int(seed) & 0xFFFFFFFFFFFFFFFF
        f32 = dict(dtype=torch.float32, device=self.device)
        self.observation = torch.zeros(capacity, obs_dim, **f32)
        self.next_observation = torch.zeros(capacity, obs_dim, **f32)
        self.action = torch.zeros(capacity, act_dim, **f32)
        self.reward = torch.zeros(capacity, **f32)
        self.terminated = torch.zeros(capacity, **f32)
        self.truncated = torch.zeros(capacity, **f32)
        self.discount = torch.zeros(capacity, **f32)
        E = num_envs
        self.pend_obs = torch.zeros(n_step, E, obs_dim, **f32)
        self.pend_next_obs = torch.zeros(n_step, E, obs_dim, **f32)
        self.pend_act = torch.zeros(n_step, E, act_dim, **f32)
        self.pend_reward = torch.zeros(n_step, E, **f32)
        self.pend_term = torch.zeros(n_step, E, **f32)
        self.pend_trunc = torch.zeros(n_step, E, **f32)
        # [steps seen, write position, filled rows]
        self.counters = torch.zeros(3, dtype=torch.int64, device=self.device)
        self.epoch = torch.zeros(1, dtype=torch.int64, device=self.device)
        self.lib = N.load()
        self._host_count = 0  # host mirror of filled rows (readiness checks without a sync)
        self._host_steps = 0

    # ---- ingest ------------------------------------------------------------
    def add(self, obs, action, reward, terminated, truncated, next_obs) -> None:
        """Stage one vector-environment step (device tensors of shape [num_envs, ...])."""
        t = lambda x: torch.as_tensor(x, device=self.device)  # noqa: E731
        obs = t(obs).float().contiguous()
        next_obs = t(next_obs).float().contiguous()
        action = t(action).float().contiguous()
        reward = t(reward).float().reshape(-1).contiguous()
        term, trunc = t(terminated).reshape(-1), t(truncated).reshape(-1)
        a = N.ReplayIngestArgs(
            obs=obs.data_ptr(), next_obs=next_obs.data_ptr(), ld_obs=obs.shape[1], action=action.data_ptr(),
            ld_action=action.shape[1], reward=reward.data_ptr(), num_envs=self.num_envs, obs_dim=self.obs_dim,
            act_dim=self.act_dim, n_step=self.n_step, gamma=self.gamma,
            pend_obs=self.pend_obs.data_ptr(), pend_next_obs=self.pend_next_obs.data_ptr(),
            pend_act=self.pend_act.data_ptr(), pend_reward=self.pend_reward.data_ptr(),
            pend_term=self.pend_term.data_ptr(), pend_trunc=self.pend_trunc.data_ptr(),
            counters=self.counters.data_ptr(), capacity=self.capacity, r_obs=self.observation.data_ptr(),
            r_next_obs=self.next_observation.data_ptr(), ld_replay_obs=self.obs_dim, r_act=self.action.data_ptr(),
            ld_replay_act=self.act_dim, r_reward=self.reward.data_ptr(), r_term=self.terminated.data_ptr(),
            r_trunc=self.truncated.data_ptr(), r_discount=self.discount.data_ptr())
        keep = []
        for name, x in (("terminated", term), ("truncated", trunc)):
            if x.dtype == torch.bool or x.dtype == torch.uint8:
                x = x.to(torch.uint8).contiguous()
                setattr(a, name + "_u8", x.data_ptr())
            else:
                x = x.float().contiguous()
                setattr(a, name, x.data_ptr())
            keep.append(x)
        N.check(self.lib.rl2_replay_ingest(ctypes.byref(a), N.stream_ptr()), "replay ingest")
        self._host_steps += 1
        if self._host_steps >= self.n_step:
            self._host_count = min(self._host_count + self.num_envs, self.capacity)
        return keep

    def __len__(self) -> int:
        return self._host_count

    def can_sample(self) -> bool:
        return self._host_count >= self.min_length

    def reset(self) -> None:
        self.counters.zero_()
        self._host_count = self._host_steps = 0

    # ---- reference checkpoint format (replay.py:196-240) ------------------
    def state(self) -> dict:
        c = self.counters.tolist()
        n = int(c[2])
        return {
            "observation": self.observation[:n].cpu(), "action": self.action[:n].cpu(), "reward": self.reward[:n].cpu(),
            "terminated": self.terminated[:n].cpu(), "truncated": self.truncated[:n].cpu(),
            "next_observation": self.next_observation[:n].cpu(), "discount": self.discount[:n].cpu(),
            "num_in_buffer": n, "current_idx": int(c[1]),
        }

    def load(self, data: dict) -> None:
        n = int(data["num_in_buffer"])
        if n > self.capacity:
            raise ValueError("Saved replay buffer exceeds the configured capacity.")
        for key, dst in (("observation", self.observation), ("next_observation", self.next_observation),
                         ("action", self.action), ("reward", self.reward), ("terminated", self.terminated),
                         ("truncated", self.truncated), ("discount", self.discount)):
            dst[:n].copy_(torch.as_tensor(data[key], device=self.device).reshape(dst[:n].shape))
        # in-flight n-step transitions are not part of the format (replay.py:238-240)
        self.counters.copy_(torch.tensor([0, int(data["current_idx"]) % self.capacity, n], device=self.device))
        self._host_count, self._host_steps = n, 0
