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


# ---------------------------------------------------------------------------
# Config-size fixtures: inputs regenerated from seeds, outputs stored as sketches.
#
# At the BASELINE configurations a full tensor dump of the reference's result is
# hundreds of MB, so ``tests/golden/make_config_golden.py`` stores, per tensor, a
# CountSketch (a fixed random signed bucketing, linear in the tensor) of the
# reference's float32 result and of the difference between its float64 and float32
# results. Because the sketch is linear, sketch(ours) - sketch(ref) = sketch(ours - ref),
# and its norm estimates ||ours - ref|| (exactly for sparse differences without
# bucket collisions, within a few percent for dense ones at 128 buckets).
# ---------------------------------------------------------------------------
SKETCH_BUCKETS = 128
_SKETCH_CACHE: dict[int, tuple[np.ndarray, np.ndarray]] = {}


def _sketch_hash(n: int) -> tuple[np.ndarray, np.ndarray]:
    if n not in _SKETCH_CACHE:
        rng = np.random.default_rng(1_000_003 + n)  # depends only on the tensor size
        bucket = rng.integers(0, SKETCH_BUCKETS, n)
        sign = rng.integers(0, 2, n).astype(np.float64) * 2.0 - 1.0
        _SKETCH_CACHE[n] = (bucket, sign)
    return _SKETCH_CACHE[n]


def sketch(x) -> np.ndarray:
    """CountSketch of a tensor (float64 sums of its float64 values)."""
    x = np.asarray(x, dtype=np.float64).ravel()
    bucket, sign = _sketch_hash(x.size)
    return np.bincount(bucket, weights=sign * x, minlength=SKETCH_BUCKETS)


CONFIG_CASES = {
    # exact config 1 of BASELINE.json (FlashSAC(31, 8), batch 512, critic 256 x 2, actor 128 x 2)
    "cfg1": dict(obs=31, act=8, actor_hidden=128, actor_blocks=2, critic_hidden=256, critic_blocks=2, batch=512,
                 updates=2),
    # config 3 widths (obs 123, act 37, batch 4096, critic 512 x 2, actor 256 x 2)
    "cfg3": dict(obs=123, act=37, actor_hidden=256, actor_blocks=2, critic_hidden=512, critic_blocks=2, batch=4096,
                 updates=2),
    # config 5 widths (critic 1024 x 3, actor 128 x 2 defaults) at a reduced batch of 1024 rows
    "cfg5w": dict(obs=123, act=37, actor_hidden=128, actor_blocks=2, critic_hidden=1024, critic_blocks=3, batch=1024,
                  updates=2),
}
CONFIG_BINS, CONFIG_MIN_V, CONFIG_MAX_V, CONFIG_LR, CONFIG_TAU = 101, -10.0, 10.0, 3e-4, 0.005


def config_inputs(spec: dict, seed: int = 2026) -> list[dict]:
    """Per update: batch with the BASELINE distributions (obs, next obs ~N(0,1), action ~U[-1,1],
    reward ~N(0,1), terminated ~Bernoulli(0.01), discount 0.99) and the policy noise
    (actor phase [2B, act], next actions [B, act], ~N(0,1)); draw order fixed."""
    rng = np.random.default_rng(seed)
    B, obs, act = spec["batch"], spec["obs"], spec["act"]
    out = []
    for _ in range(spec["updates"]):
        batch = {
            "observation": rng.standard_normal((B, obs)).astype(np.float32),
            "next_observation": rng.standard_normal((B, obs)).astype(np.float32),
            "action": rng.uniform(-1, 1, (B, act)).astype(np.float32),
            "reward": rng.standard_normal(B).astype(np.float32),
            "terminated": (rng.random(B) < 0.01).astype(np.float32),
            "truncated": np.zeros(B, np.float32),
            "discount": np.full(B, 0.99, np.float32),
        }
        noise = {"actor": rng.standard_normal((2 * B, act)).astype(np.float32),
                 "next": rng.standard_normal((B, act)).astype(np.float32)}
        out.append({"batch": batch, "noise": noise})
    return out


def config_target_entropy(act: int) -> float:
    return 0.5 * act * float(np.log(2 * np.pi * np.e * 0.15**2))


def config_oracle_state(spec: dict) -> dict:
    """Oracle start state of a config case: the reference's seeded initial networks (replayed
    by ``_init_reference_weights``), fresh BN buffers and optimiser states."""
    from robolearn_b200.flashsac.config import FlashSACConfig
    from robolearn_b200.flashsac.learner import _init_reference_weights

    cfg = FlashSACConfig(device="cpu", seed=0, actor_hidden_dim=spec["actor_hidden"],
                         actor_num_blocks=spec["actor_blocks"], critic_hidden_dim=spec["critic_hidden"],
                         critic_num_blocks=spec["critic_blocks"], critic_num_bins=CONFIG_BINS)
    a0, c0, lt = _init_reference_weights(spec["obs"], spec["obs"], spec["act"], cfg)

    def with_buffers(p, twin, H, cin, blocks):
        out = {k: v.numpy().astype(np.float64) for k, v in p.items()}
        for pre in fs.bn_buffer_prefixes(blocks):
            C = cin if pre == "embedder.norm" else (4 * H if pre.endswith("norm1") else H)
            shape = (2, C) if twin else (C,)
            out[pre + ".running_mean"] = np.zeros(shape)
            out[pre + ".running_var"] = np.ones(shape)
        return out

    obs, act = spec["obs"], spec["act"]
    return dict(actor=with_buffers(a0, False, spec["actor_hidden"], obs, spec["actor_blocks"]),
                critic=with_buffers(c0, True, spec["critic_hidden"], obs + act, spec["critic_blocks"]),
                target=with_buffers(c0, True, spec["critic_hidden"], obs + act, spec["critic_blocks"]),
                log_temp=lt, opt_actor=fs.OptState(), opt_critic=fs.OptState(), opt_temp=fs.OptState())


def config_dims(spec: dict) -> fs.Dims:
    return fs.Dims(obs=spec["obs"], act=spec["act"], actor_hidden=spec["actor_hidden"],
                   actor_blocks=spec["actor_blocks"], critic_hidden=spec["critic_hidden"],
                   critic_blocks=spec["critic_blocks"], bins=CONFIG_BINS, min_v=CONFIG_MIN_V, max_v=CONFIG_MAX_V)


def config_hyper(spec: dict) -> fs.Hyper:
    return fs.Hyper(gamma=0.99, tau=CONFIG_TAU, lr_init=CONFIG_LR, lr_peak=CONFIG_LR, lr_end=CONFIG_LR,
                    target_entropy=config_target_entropy(spec["act"]))


def oracle_tensors(state: dict, actor_done: bool) -> dict[str, np.ndarray]:
    """Oracle state in the fixture's key layout."""
    out = {}
    for tag in ("actor", "critic", "target"):
        for k, v in state[tag].items():
            if not k.endswith("bin_values"):
                out[f"{tag}.{k}"] = v
    for tag, opt in (("actor", state["opt_actor"]), ("critic", state["opt_critic"])):
        if tag == "actor" and not actor_done:
            continue
        for k in opt.m:
            out[f"opt.{tag}.m.{k}"] = opt.m[k]
            out[f"opt.{tag}.v.{k}"] = opt.v[k]
    return out
