"""Config-size golden fixtures: the reference's own Torch FlashSAC run on CPU at the
BASELINE configurations (exact config 1, config-3 widths, config-5 widths at 1024 rows).

For each case the reference is initialised exactly as ``FlashSAC`` does
(``torch.manual_seed(seed)`` then ``_init_flashsac_networks``,
``src/robolearn/flashsac/agent.py:52-155,320``) and ``_update_networks``
(``agent.py:217-281``) runs two updates (actor + critic, then critic only) on seeded
batches with the policy noise injected by patching ``Normal.rsample`` (the reference's
own diagnostic technique, ``examples/diagnose_warp_flashsac.py:311-333``). The inputs
are regenerated from their seed by ``tests/_golden.py:config_inputs`` and never stored.

The same update is run twice: in float32 (the reference as shipped) and in float64
(networks, optimiser state, batch and noise converted; the twin critics' BN running
buffers stay float32 because the reference casts their statistics to float32). The float64 run is only the
yardstick of the reference's own float32 rounding: it shows, per tensor, how far the
reference's float32 answer is from the exact one.

Yardsticks of the reference's own rounding, per tensor (relative L2 to its float32
result): ``floor`` (its float64 run), ``spread`` (float32 runs on inputs moved by +-1 ulp,
the largest of three), ``spread16`` (inputs restated at fp16 precision, +-2^-11), and ``spread17`` (inputs
moved by +-2^-17, the forward precision of the FP32 recipe's tensor-core products).

Stored per tensor (parameters, BN buffers, target parameters, Adam moments): the
CountSketch of the float32 result, the sketch of (float64 - float32), the float32
result's L2 norm and the yardsticks; every returned metric in float32 and float64 with
its spreads. A sketch of the initial networks pins the initialisation replay.

    python tests/golden/make_config_golden.py --reference-src <reference>/src [--cases cfg1 cfg3 cfg5w]
"""

from __future__ import annotations

import argparse
import sys
import time
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))

from tests import _golden as G  # noqa: E402
from tests.golden.make_golden import _install_gym_shim, _moments, _state  # noqa: E402


def _to_double(net) -> None:
    import torch

    net.network.double()
    for name, buf in net.network.named_buffers():
        # the twin critics' batch norm lerps float32 statistics into its running buffers
        # (layers.py:208-210); the actor's F.batch_norm keeps them in the input's type
        if name.endswith(("running_mean", "running_var")) and buf.dim() == 2:
            buf.data = buf.data.to(torch.float32)


def _perturbed(inputs: list[dict], seed: int, rel: float = 0.0) -> list[dict]:
    """The same inputs with every float32 value moved by -1, 0 or +1 ulp at random (``rel``
    = 0: the same problem as far as float32 can state it, evaluated with different
    rounding), or scaled by 1 - rel, 1 or 1 + rel at random (``rel`` = 2^-11: the problem as
    far as fp16 operands can state it)."""
    rng = np.random.default_rng(seed)
    out = []
    for x in inputs:
        y = {"batch": {}, "noise": {}}
        for part in ("batch", "noise"):
            for k, v in x[part].items():
                if k in ("terminated", "truncated", "discount"):
                    y[part][k] = v
                    continue
                step = rng.integers(-1, 2, v.shape)
                if rel > 0:
                    y[part][k] = (v * (1.0 + rel * step)).astype(np.float32)
                    continue
                up, down = np.nextafter(v, np.float32(np.inf)), np.nextafter(v, np.float32(-np.inf))
                y[part][k] = np.where(step > 0, up, np.where(step < 0, down, v)).astype(np.float32)
        out.append(y)
    return out


def _run_update(nets, cfg, inputs, actor_phase: bool, dtype, grad_scaler=None):
    import torch

    from robolearn.flashsac.agent import _update_networks

    actor, critic, target, temp = nets
    batch_t = {k: torch.from_numpy(v).to(dtype) for k, v in inputs["batch"].items()}
    batch_t["actor_observation"] = batch_t["observation"]
    batch_t["actor_next_observation"] = batch_t["next_observation"]
    queue = []
    if actor_phase:
        queue.append(torch.from_numpy(inputs["noise"]["actor"]).to(dtype))
    queue.append(torch.from_numpy(inputs["noise"]["next"]).to(dtype))
    original = torch.distributions.Normal.rsample

    def rsample(self, sample_shape=torch.Size(), _q=queue):
        eps = _q.pop(0)
        assert tuple(eps.shape) == tuple(self.loc.shape), (eps.shape, self.loc.shape)
        return self.loc + eps.to(self.loc.dtype) * self.scale

    torch.distributions.Normal.rsample = rsample
    try:
        info = _update_networks(batch_t, actor, critic, target, temp, cfg, do_actor_update=actor_phase,
                                device=torch.device("cpu"), grad_scaler=grad_scaler)
    finally:
        torch.distributions.Normal.rsample = original
    assert not queue
    return {k: float(v.detach()) if hasattr(v, 'detach') else float(v) for k, v in info.items()}


def _tensors(nets, actor_phase_done: bool) -> dict[str, np.ndarray]:
    actor, critic, target, temp = nets
    out = {}
    for tag, net in (("actor", actor), ("critic", critic), ("target", target)):
        for k, v in _state(net.network).items():
            if k.endswith("bin_values"):
                continue
            out[f"{tag}.{k}"] = v
    for tag, net in (("actor", actor), ("critic", critic)):
        if tag == "actor" and not actor_phase_done:
            continue
        for k, v in _moments(net).items():
            if not k.startswith("step."):
                out[f"opt.{tag}.{k}"] = v
    return out


def _config(spec: dict, use_amp: bool):
    from robolearn.flashsac import FlashSACConfig

    B = spec["batch"]
    cfg = FlashSACConfig(
        device="cpu", use_compile=False, use_amp=use_amp, seed=0,
        actor_hidden_dim=spec["actor_hidden"], actor_num_blocks=spec["actor_blocks"],
        critic_hidden_dim=spec["critic_hidden"], critic_num_blocks=spec["critic_blocks"],
        critic_num_bins=G.CONFIG_BINS, critic_min_v=G.CONFIG_MIN_V, critic_max_v=G.CONFIG_MAX_V,
        critic_target_update_tau=G.CONFIG_TAU, learning_rate_init=G.CONFIG_LR, learning_rate_peak=G.CONFIG_LR,
        learning_rate_end=G.CONFIG_LR, n_step=1, buffer_max_length=4 * B, buffer_min_length=B,
        sample_batch_size=B,
    )
    cfg.temp_target_entropy = G.config_target_entropy(spec["act"])
    return cfg


def _fresh(spec: dict, cfg, double: bool = False):
    """The reference's networks, initialised from the config seed (every run starts here)."""
    import torch

    from robolearn.flashsac.agent import _init_flashsac_networks

    torch.manual_seed(cfg.seed)
    nets = _init_flashsac_networks(spec["obs"], spec["obs"], spec["act"], cfg, torch.device("cpu"))
    if double:
        for net in nets:
            _to_double(net)
    return nets


def _trajectory(spec, cfg, nets, inputs, dtype, grad_scaler=None):
    """Yields (update, metrics, tensors, log_temp, seconds) for each update of the case."""
    actor_done = False
    for u in range(spec["updates"]):
        actor_phase = u % cfg.actor_update_period == 0
        actor_done |= actor_phase
        t0 = time.perf_counter()
        metrics = _run_update(nets, cfg, inputs[u], actor_phase, dtype, grad_scaler)
        yield u, metrics, _tensors(nets, actor_done), _state(nets[3].network)["log_temp"], time.perf_counter() - t0


def _rel(a, b) -> float:
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(np.asarray(a, np.float64) - b) / max(np.linalg.norm(b), 1e-30))


def make_case(name: str, spec: dict, threads: int, spread_runs: int = 3) -> None:
    import torch

    torch.set_num_threads(threads)
    cfg = _config(spec, use_amp=False)
    inputs = G.config_inputs(spec)
    out: dict[str, np.ndarray] = {}
    nets32 = _fresh(spec, cfg)
    for k, v in _tensors(nets32, False).items():
        out[f"before.{k}.sk"] = G.sketch(v)
    out["before.temp.log_temp"] = _state(nets32[3].network)["log_temp"]
    ref32 = {}  # update -> tensors of the shipped float32 reference
    for u, m32, t32, temp, sec in _trajectory(spec, cfg, nets32, inputs, torch.float32):
        ref32[u] = t32
        for k, v in t32.items():
            out[f"u{u}.{k}.sk"] = G.sketch(v).astype(np.float32)
            out[f"u{u}.{k}.norm"] = np.array(float(np.linalg.norm(np.asarray(v, np.float64))))
        for k, v in m32.items():
            out[f"u{u}.metric32.{k}"] = np.array(v)
        out[f"u{u}.temp32"] = temp
        print(f"{name} update {u}: float32 {sec:.1f} s, metrics {m32}", flush=True)
    # float64: how far the shipped float32 result is from exact arithmetic
    for u, m64, t64, temp, sec in _trajectory(spec, cfg, _fresh(spec, cfg, double=True), inputs, torch.float64):
        worst = (0.0, "")
        for k, v in t64.items():
            out[f"u{u}.{k}.dsk"] = (G.sketch(v) - out[f"u{u}.{k}.sk"].astype(np.float64)).astype(np.float32)
            out[f"u{u}.{k}.floor"] = np.array(_rel(v, ref32[u][k]))
            worst = max(worst, (float(out[f"u{u}.{k}.floor"]), k))
        for k, v in m64.items():
            out[f"u{u}.metric64.{k}"] = np.array(v)
        out[f"u{u}.temp64"] = temp.astype(np.float64)
        print(f"{name} update {u}: float64 {sec:.1f} s, float32 vs float64 worst {worst[1]} {worst[0]:.2e}",
              flush=True)
    # the spread of legitimate float32 evaluations: the same problem with +-1 ulp inputs
    for r in range(spread_runs):
        pert = _perturbed(inputs, seed=100 + r)
        for u, mp, tp, temp, sec in _trajectory(spec, cfg, _fresh(spec, cfg), pert, torch.float32):
            for k, v in tp.items():
                key = f"u{u}.{k}.spread"
                out[key] = np.array(max(float(out.get(key, 0.0)), _rel(v, ref32[u][k])))
            for k, v in mp.items():
                key = f"u{u}.metricspread.{k}"
                out[key] = np.array(max(float(out.get(key, 0.0)), abs(v - float(out[f"u{u}.metric32.{k}"]))))
            print(f"{name} update {u}: perturbed float32 run {r} {sec:.1f} s", flush=True)
    # the spread at fp16 scale: inputs restated at fp16 precision (+-2^-11 relative)
    for r in range(spread_runs):
        pert = _perturbed(inputs, seed=200 + r, rel=2.0 ** -11)
        for u, mp, tp, temp, sec in _trajectory(spec, cfg, _fresh(spec, cfg), pert, torch.float32):
            for k, v in tp.items():
                key = f"u{u}.{k}.spread16"
                out[key] = np.array(max(float(out.get(key, 0.0)), _rel(v, ref32[u][k])))
            for k, v in mp.items():
                key = f"u{u}.metricspread16.{k}"
                out[key] = np.array(max(float(out.get(key, 0.0)), abs(v - float(out[f"u{u}.metric32.{k}"]))))
            print(f"{name} update {u}: fp16-scale perturbed run {r} {sec:.1f} s", flush=True)
    # the spread at the FP32 recipe's forward precision: its tensor-core products accumulate
    # K terms with an error of about 7e-9 K relative (4e-6 at K = 512, 1.5e-5 at K = 2048,
    # measured against float64; CPU float32 stays below 1e-6), so the reference is also run
    # on inputs moved by +-2^-17 relative (7.6e-6)
    for r in range(spread_runs):
        pert = _perturbed(inputs, seed=300 + r, rel=2.0 ** -17)
        for u, mp, tp, temp, sec in _trajectory(spec, cfg, _fresh(spec, cfg), pert, torch.float32):
            for k, v in tp.items():
                key = f"u{u}.{k}.spread17"
                out[key] = np.array(max(float(out.get(key, 0.0)), _rel(v, ref32[u][k])))
            for k, v in mp.items():
                key = f"u{u}.metricspread17.{k}"
                out[key] = np.array(max(float(out.get(key, 0.0)), abs(v - float(out[f"u{u}.metric32.{k}"]))))
            print(f"{name} update {u}: 2^-17-perturbed run {r} {sec:.1f} s", flush=True)
    for k, v in spec.items():
        out[f"spec.{k}"] = np.array(v)
    out["spec.buckets"] = np.array(G.SKETCH_BUCKETS)
    out["spec.spread_runs"] = np.array(spread_runs)
    np.savez_compressed(HERE / f"flashsac_config_{name}.npz", **out)
    print(f"flashsac_config_{name}: {len(out)} arrays", flush=True)


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--reference-src", required=True, help="path of the reference project's src directory")
    parser.add_argument("--cases", nargs="*", default=list(G.CONFIG_CASES))
    parser.add_argument("--threads", type=int, default=8)
    args = parser.parse_args()
    _install_gym_shim()
    sys.path.insert(0, args.reference_src)
    for name in args.cases:
        make_case(name, G.CONFIG_CASES[name], args.threads)


if __name__ == "__main__":
    main()
