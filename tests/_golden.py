"""Helpers that turn the committed golden fixtures into oracle/engine inputs."""

from __future__ import annotations

from pathlib import Path

import numpy as np

from oracle import flashsac_np as fs

GOLDEN = Path(__file__).resolve().parent / "golden"


def load(name: str) -> dict[str, np.ndarray]:
    with np.load(GOLDEN / name) as data:
        return {k: data[k] for k in data.files}


def dims(g: dict) -> fs.Dims:
    s = lambda k: g[f"spec.{k}"].item()  # noqa: E731
    cobs = int(s("critic_obs"))
    return fs.Dims(
        obs=int(s("obs")), act=int(s("act")), actor_hidden=int(s("actor_hidden")),
        actor_blocks=int(s("actor_blocks")), critic_hidden=int(s("critic_hidden")),
        critic_blocks=int(s("critic_blocks")), bins=int(s("bins")), min_v=float(s("min_v")),
        max_v=float(s("max_v")), critic_obs=None if cobs < 0 else cobs,
    )


def network(g: dict, stage: str, tag: str) -> dict[str, np.ndarray]:
    pre = f"{stage}.{tag}."
    return {k[len(pre):]: v for k, v in g.items() if k.startswith(pre)}


def batch(g: dict, update: int) -> dict[str, np.ndarray]:
    pre = f"batch{update}."
    return {k[len(pre):]: v for k, v in g.items() if k.startswith(pre)}


def noise(g: dict, update: int) -> tuple[np.ndarray | None, np.ndarray]:
    a = g.get(f"noise{update}.actor")
    return a, g[f"noise{update}.next"]


def metrics(g: dict, update: int) -> dict[str, float]:
    pre = f"metrics{update}."
    return {k[len(pre):]: float(v) for k, v in g.items() if k.startswith(pre)}


def hyper(g: dict) -> fs.Hyper:
    return fs.Hyper(gamma=0.99, tau=0.005, lr_init=3e-4, lr_peak=3e-4, lr_end=1.5e-4, warmup=0, decay=10,
                    target_entropy=float(g["spec.target_entropy"]))


def initial_state(g: dict) -> dict:
    return dict(
        actor=network(g, "before", "actor"),
        critic=network(g, "before", "critic"),
        target=network(g, "before", "target"),
        log_temp=float(g["before.temp.log_temp"][0]),
        opt_actor=fs.OptState(), opt_critic=fs.OptState(), opt_temp=fs.OptState(),
    )


def rel_err(a, b) -> float:
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.max(np.abs(a - b)) / max(np.max(np.abs(b)), 1e-30))
