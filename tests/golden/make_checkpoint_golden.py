"""Checkpoint interoperability fixture: a directory written by the reference's own
``FlashSAC.save()`` (``src/robolearn/flashsac/agent.py:529-551``).

A small reference agent (``FlashSAC(5, 3, num_envs=4)``, hidden 8, one block, 11 atoms,
reward normalisation on) runs on CPU: 24 vector steps of seeded transitions through
``observe()``, then three ``update()`` calls (two actor phases), so every network,
optimiser, scheduler, temperature and reward-normaliser state is non-trivial. The
directory is saved under ``tests/golden/flashsac_ckpt_ref/`` together with
``flashsac_ckpt_ref.npz``: fixed observations and the reference's deterministic
``act(obs, training=False)`` on them.

    python tests/golden/make_checkpoint_golden.py --reference-src <reference>/src
"""

from __future__ import annotations

import argparse
import shutil
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))

from tests.golden.make_golden import _install_gym_shim  # noqa: E402

OBS, ACT, ENVS = 5, 3, 4
CONFIG = dict(device="cpu", use_compile=False, use_amp=False, seed=3, actor_hidden_dim=8, actor_num_blocks=1,
              critic_hidden_dim=8, critic_num_blocks=1, critic_num_bins=11, critic_min_v=-5.0, critic_max_v=5.0,
              buffer_max_length=256, buffer_min_length=16, sample_batch_size=8, n_step=1, normalize_reward=True,
              learning_rate_init=3e-4, learning_rate_peak=3e-4, learning_rate_end=1e-4, learning_rate_decay_step=50)


def rollout(rng: np.random.Generator, steps: int):
    """Seeded transitions of ENVS environments (obs ~N(0,1), act ~U[-1,1], rew ~N(0,1))."""
    for _ in range(steps):
        yield dict(observations=rng.standard_normal((ENVS, OBS)).astype(np.float32),
                   actions=rng.uniform(-1, 1, (ENVS, ACT)).astype(np.float32),
                   rewards=rng.standard_normal(ENVS).astype(np.float32),
                   terminated=(rng.random(ENVS) < 0.1), truncated=np.zeros(ENVS, bool),
                   next_observations=rng.standard_normal((ENVS, OBS)).astype(np.float32))


def probe_observations() -> np.ndarray:
    return np.random.default_rng(77).standard_normal((16, OBS)).astype(np.float32)


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--reference-src", required=True)
    args = parser.parse_args()
    _install_gym_shim()
    sys.path.insert(0, args.reference_src)
    import torch

    from robolearn.flashsac import FlashSAC, FlashSACConfig

    torch.set_num_threads(1)
    agent = FlashSAC(OBS, ACT, num_envs=ENVS, cfg=FlashSACConfig(**CONFIG))
    for tr in rollout(np.random.default_rng(5), 24):
        agent.observe(*(torch.from_numpy(np.asarray(tr[k])) for k in
                        ("observations", "actions", "rewards", "terminated", "truncated", "next_observations")))
    for _ in range(3):
        agent.update()
    out = HERE / "flashsac_ckpt_ref"
    if out.exists():
        shutil.rmtree(out)
    agent.save(str(out))
    obs = probe_observations()
    with torch.no_grad():
        actions = agent.act(torch.from_numpy(obs), training=False).numpy()
    np.savez_compressed(HERE / "flashsac_ckpt_ref.npz", observations=obs, actions=actions)
    print(sorted(p.name for p in out.iterdir()), actions[:2])


if __name__ == "__main__":
    main()
