"""Reverse checkpoint fixture: a directory written by this library's ``FlashSAC.save()``.

Runs on a CUDA device: loads the reference-written directory ``flashsac_ckpt_ref/``,
continues training for three updates on the next seeded transitions, saves the agent to
``<out>/flashsac_ckpt_ours/`` and its deterministic actions on the probe observations to
``<out>/flashsac_ckpt_ours.npz``. Committed beside this script, the directory is loaded by
the reference's own ``FlashSAC.load()`` in ``tests/test_checkpoint_interop_cpu.py``.

    python tests/golden/make_checkpoint_ours.py --out <directory>
"""

from __future__ import annotations

import argparse
import json
import shutil
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))

from tests.golden.make_checkpoint_golden import ENVS, probe_observations, rollout  # noqa: E402


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--out", required=True)
    args = parser.parse_args()
    import torch

    from robolearn_b200.flashsac.agent import FlashSAC
    from robolearn_b200.flashsac.config import FlashSACConfig

    ref = HERE / "flashsac_ckpt_ref"
    meta = json.loads((ref / "config.json").read_text())
    agent = FlashSAC(meta["observation_dim"], meta["action_dim"], num_envs=ENVS,
                     cfg=FlashSACConfig(**{**meta["config"], "device": "cuda"}))
    agent.load(str(ref))
    for tr in rollout(np.random.default_rng(6), 24):
        agent.observe(*(torch.as_tensor(np.asarray(tr[k]), device="cuda") for k in
                        ("observations", "actions", "rewards", "terminated", "truncated", "next_observations")))
    for _ in range(3):
        agent.update()
    out = Path(args.out)
    out.mkdir(parents=True, exist_ok=True)
    target = out / "flashsac_ckpt_ours"
    if target.exists():
        shutil.rmtree(target)
    agent.save(str(target))
    obs = probe_observations()
    with torch.no_grad():
        actions = agent.act(torch.from_numpy(obs).cuda(), training=False).cpu().numpy()
    np.savez_compressed(out / "flashsac_ckpt_ours.npz", observations=obs, actions=actions)
    print(sorted(p.name for p in target.iterdir()), actions[:2])


if __name__ == "__main__":
    main()
