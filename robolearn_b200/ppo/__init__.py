"""Clipped PPO learner update on sm_100a kernels (drop-in for ``robolearn.warp.WarpPPO``)."""

from .config import PPOConfig
from .learner import WarpPPO

__all__ = ["PPOConfig", "WarpPPO"]
