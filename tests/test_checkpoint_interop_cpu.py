"""The reference loads a checkpoint directory this library wrote.

``tests/golden/flashsac_ckpt_ours/`` was written by this library's ``FlashSAC.save()``
on a B200 (``tests/golden/make_checkpoint_ours.py``: the reference-written directory
loaded, three more updates, saved). Every file must load with the reference's own
``torch.load(weights_only=True)`` (checked everywhere), and, where the reference's
sources are present, the reference's ``FlashSAC.load()`` takes the directory (optimiser,
scheduler, scaler and reward-normaliser state included) and then acts on the probe
observations as this library did before saving (deterministic actions within 2e-5).
"""

import json
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import build_ref

GOLDEN = Path(__file__).resolve().parent / "golden"
OURS = GOLDEN / "flashsac_ckpt_ours"


def test_every_file_loads_with_weights_only():
    for name in ("actor.pt", "critic.pt", "target_critic.pt", "temperature.pt", "reward_normalizer.pt",
                 "agent_state.pt"):
        ck = torch.load(OURS / name, map_location="cpu", weights_only=True)
        assert isinstance(ck, dict), name


def test_reference_loads_our_directory_and_acts_alike():
    src = build_ref.reference_root() / "src"
    if not (src / "robolearn" / "flashsac" / "agent.py").is_file():
        pytest.skip("reference sources absent")
    sys.path.insert(0, str(Path(__file__).resolve().parent / "golden"))
    from make_golden import _install_gym_shim

    _install_gym_shim()
    sys.path.insert(0, str(src))
    from robolearn.flashsac import FlashSAC, FlashSACConfig

    meta = json.loads((OURS / "config.json").read_text())
    fields = set(FlashSACConfig.__dataclass_fields__)
    cfg = FlashSACConfig(**{k: v for k, v in {**meta["config"], "device": "cpu"}.items() if k in fields})
    agent = FlashSAC(meta["observation_dim"], meta["action_dim"], num_envs=4, cfg=cfg)
    agent.load(str(OURS))
    g = np.load(GOLDEN / "flashsac_ckpt_ours.npz")
    with torch.no_grad():
        got = agent.act(torch.from_numpy(g["observations"]), training=False).numpy()
    np.testing.assert_allclose(got, g["actions"], rtol=0, atol=2e-5)
