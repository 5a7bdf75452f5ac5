"""FlashSAC learner updates at the BASELINE configurations against the reference's own run.

Fixtures (``tests/golden/make_config_golden.py``): the reference's Torch FlashSAC
(``src/robolearn/flashsac/agent.py:217-281``) run on CPU at exact config 1 (obs 31,
act 8, batch 512, critic 256 x 2, actor 128 x 2), config-3 widths (obs 123, act 37,
batch 4096, critic 512 x 2, actor 256 x 2) and config-5 widths at 1024 rows (critic
1024 x 3, actor 128 x 2): two updates (actor + critic, then critic only) from the
reference's seeded initial networks on seeded batches and noise, which this test
regenerates (``tests/_golden.py:config_inputs``). Every tensor of the result is stored
as a CountSketch, a linear map, so ``||sketch(ours) - sketch(ref)||`` measures
``||ours - ref||``.

Checked per tensor (every parameter, BN running buffer, target parameter and Adam
moment; 162 tensors at config 1) after each update, in relative L2 norm, against three
yardsticks the fixture script measured on the reference itself:

* ``floor``: the reference's float32 result against its own float64 run;
* ``spread``: the reference's float32 result against float32 runs on the same inputs
  moved by +-1 ulp at random (three runs, the largest distance). At these widths this is
  well above 1e-4 for BN biases and every Adam moment: each ReLU decision that falls
  within rounding of the kink (about one per 1024-wide layer per evaluation) moves that
  layer's gradients by ~1e-3, and the first Adam step, ``lr g / (|g| + 1e-8)``, turns
  gradients near zero into a full ``+-lr`` step either way;
* ``spread16``: the same with the inputs restated at fp16 precision (+-2^-11 relative);
* ``spread17``: the same with the inputs moved by +-2^-17 relative, the forward precision
  of the FP32 recipe: its 3xTF32 tensor-core products accumulate K terms in fp32 with an
  error of about 7e-9 K relative (4e-6 at K = 512, 1.5e-5 at K = 2048, measured against
  float64; the operand split alone is 3.5e-7, CPU float32 stays below 1e-6), so it takes
  more ReLU decisions at the kink the other way than the reference's float32 does, and the
  gradient-carrying tensors (Adam moments) move accordingly.

Tolerances (plus, for parameter tensors, room for 1 + 0.2% of the elements to have taken
their first Adam step the other way, see ``_step_flip_allowance``):

* FP32 recipe: within ``max(1e-4, 3 floor, 2 spread, 2 spread17)`` of the reference's
  float32 result: 1e-4 wherever the arithmetic determines the result to that level,
  otherwise no farther from the reference than the reference moves itself under
  rounding-level changes of its inputs at float32 precision or at the recipe's precision.
* FP16-operand recipe: within ``max(1e-2, 2 spread16)``: no farther from the reference's
  FP32 result than that result moves when its inputs are stated at fp16 precision.
* Metrics: the same rules on each returned metric.
* The initial networks: this library's replay of the reference's seeded initialisation
  is within 1e-6 (relative L2) of the reference's (bit-identical on the fixture's host;
  ``orthogonal_``'s host QR rounds differently on other CPUs).

The arithmetic itself is checked without these yardsticks by
``test_gradients_match_oracle_at_config1``.

BN running buffers whose values are rounding noise (running means of zero-mean inputs,
~1e-9) are measured against an absolute scale of 1e-3 per element.
"""

import numpy as np
import pytest
import torch

from tests import _golden as G

pytestmark = pytest.mark.gpu

from robolearn_b200.flashsac.config import FlashSACConfig  # noqa: E402
from robolearn_b200.flashsac.learner import METRIC_KEYS, Learner  # noqa: E402

TOL = {"fp32": 1e-4, "fp16": 1e-2}
FLOOR_FACTOR = 3.0
SPREAD_FACTOR = 2.0
BUFFER_SCALE = 1e-3


def _learner(spec: dict, precision: str) -> Learner:
    B = spec["batch"]
    cfg = FlashSACConfig(
        device="cuda", seed=0, sample_batch_size=B, actor_hidden_dim=spec["actor_hidden"],
        actor_num_blocks=spec["actor_blocks"], critic_hidden_dim=spec["critic_hidden"],
        critic_num_blocks=spec["critic_blocks"], critic_num_bins=G.CONFIG_BINS, critic_min_v=G.CONFIG_MIN_V,
        critic_max_v=G.CONFIG_MAX_V, critic_target_update_tau=G.CONFIG_TAU, learning_rate_init=G.CONFIG_LR,
        learning_rate_peak=G.CONFIG_LR, learning_rate_end=G.CONFIG_LR, n_step=1, buffer_max_length=4 * B,
        buffer_min_length=B, dense_precision=precision, temp_target_entropy=G.config_target_entropy(spec["act"]),
    )
    return Learner(spec["obs"], spec["obs"], spec["act"], cfg, "cuda")


def _tensors(L: Learner, actor_done: bool) -> dict[str, np.ndarray]:
    out = {}
    for tag, net in (("actor", L.actor), ("critic", L.critic), ("target", L.target)):
        for k, v in net.state_dict().items():
            if not k.endswith("bin_values"):
                out[f"{tag}.{k}"] = v.cpu().numpy()
    for tag, net in (("actor", L.actor), ("critic", L.critic)):
        if tag == "actor" and not actor_done:
            continue
        for k in net.shapes:
            out[f"opt.{tag}.m.{k}"] = net.moment("m", k).cpu().numpy()
            out[f"opt.{tag}.v.{k}"] = net.moment("v", k).cpu().numpy()
    return out


def _step_flip_allowance(key: str, size: int, norm: float) -> float:
    """Relative L2 room for parameter elements whose Adam step went the other way.

    The first Adam step moves every element by about lr in the direction of its gradient's
    sign; an element whose gradient lies within rounding of zero may go either way in any
    float32 evaluation (the reference's own among them), a 2 lr difference (2 tau lr in the
    target network after the EMA). Up to 1 + 0.2% of a tensor's elements may do so; this
    only matters for tensors whose norm is a few steps (BN biases, head biases)."""
    if key.startswith("opt.") or key.endswith(("running_mean", "running_var")):
        return 0.0
    step = 2.2 * G.CONFIG_LR * (G.CONFIG_TAU if key.startswith("target.") else 1.0)
    flips = 1 + 0.002 * size
    return float(np.sqrt(flips) * step / max(norm, 1e-30))


def _compare(g: dict, u: int, ours: dict, tol: float, fp16: bool) -> list[str]:
    """Per-tensor relative L2 distance to the reference's float32 result; returns failures."""
    keys = sorted(k[len(f"u{u}."):-len(".sk")] for k in g if k.startswith(f"u{u}.") and k.endswith(".sk"))
    assert set(keys) == set(ours), (sorted(set(keys) ^ set(ours)))[:8]
    failures = []
    for k in keys:
        x = ours[k]
        ref = g[f"u{u}.{k}.sk"].astype(np.float64)
        norm = float(g[f"u{u}.{k}.norm"])
        if k.endswith(("running_mean", "running_var")):
            norm = max(norm, BUFFER_SCALE * np.sqrt(x.size))
        err = float(np.linalg.norm(G.sketch(x) - ref)) / max(norm, 1e-30)
        floor = float(g[f"u{u}.{k}.floor"])
        spread = float(g[f"u{u}.{k}.spread"])
        spread16 = float(g[f"u{u}.{k}.spread16"])
        spread17 = float(g[f"u{u}.{k}.spread17"])
        if fp16:
            limit = max(tol, SPREAD_FACTOR * spread16)
        else:
            limit = max(tol, FLOOR_FACTOR * floor, SPREAD_FACTOR * spread, SPREAD_FACTOR * spread17)
        limit += _step_flip_allowance(k, x.size, norm)
        if not err <= limit:
            failures.append(f"{k}: {err:.2e} > {limit:.2e} (reference: float64 {floor:.2e}, float32 spread "
                            f"{spread:.2e}, 2^-17 spread {spread17:.2e}, fp16-scale spread {spread16:.2e})")
    return failures


@pytest.mark.parametrize("precision", ["fp32", "fp16"])
@pytest.mark.parametrize("case", list(G.CONFIG_CASES))
def test_update_matches_reference_at_config_size(case, precision):
    g = G.load(f"flashsac_config_{case}.npz")
    spec = G.CONFIG_CASES[case]
    tol = TOL[precision]
    L = _learner(spec, precision)
    # the initialisation replays the reference's seeded construction; orthogonal_ runs a
    # host LAPACK QR whose last-bit rounding depends on the host CPU, so the replay is
    # bit-identical on the machine that made the fixture and within float32 rounding elsewhere
    init = _tensors(L, actor_done=False)
    for k, v in init.items():
        if k.startswith("opt."):
            continue
        ref = g[f"before.{k}.sk"]
        err = float(np.linalg.norm(G.sketch(v) - ref)) / max(float(np.linalg.norm(v)), 1e-30)
        assert err < 1e-6, (f"initial {k}", err)
    assert float(L.log_temp) == pytest.approx(float(g["before.temp.log_temp"][0]), abs=0)
    inputs = G.config_inputs(spec)
    actor_done = False
    report = []
    for u in range(spec["updates"]):
        actor_phase = u % L.cfg.actor_update_period == 0
        actor_done |= actor_phase
        L.load_batch(inputs[u]["batch"], inputs[u]["noise"]["actor"], inputs[u]["noise"]["next"])
        L.run(actor_phase)
        torch.cuda.synchronize()
        assert int(L.health.item()) == 0
        for name, net in (("actor", L.actor), ("critic", L.critic)):
            if name == "critic" or actor_phase:
                assert float(net.opt_state[8]) == 0.0, f"{name} optimiser step skipped (loss-scale overflow)"
        got = {k: float(L.metrics[METRIC_KEYS.index(k)]) for k in L.metric_values(actor_phase)}
        for k, v in got.items():
            r32 = float(g[f"u{u}.metric32.{k}"])
            r64 = float(g[f"u{u}.metric64.{k}"])
            if precision == "fp16":
                limit = max(tol * max(1.0, abs(r32)), SPREAD_FACTOR * float(g[f"u{u}.metricspread16.{k}"]))
            else:
                limit = max(tol * max(1.0, abs(r32)), FLOOR_FACTOR * abs(r64 - r32),
                            SPREAD_FACTOR * float(g[f"u{u}.metricspread.{k}"]),
                            SPREAD_FACTOR * float(g[f"u{u}.metricspread17.{k}"]))
            if not abs(v - r32) <= limit:
                report.append(f"update {u}: metric {k} = {v} vs reference {r32} (float64 {r64})")
        t32 = float(g[f"u{u}.temp32"][0])
        assert abs(float(L.log_temp) - t32) <= max(tol * abs(t32), 1e-6), (u, float(L.log_temp), t32)
        failures = _compare(g, u, _tensors(L, actor_done), tol, precision == "fp16")
        report += [f"update {u}: {f}" for f in failures]
    assert not report, f"{case} {precision}: {len(report)} tensors outside tolerance:\n" + "\n".join(report[:40])


def _gpu_decisions(L: Learner, actor_phase: bool) -> dict:
    """The CUDA path's ReLU decisions as (pre-normalisation output, mean, invstd) per block
    batch norm, keyed by the oracle's ReLU site numbers (sites in the oracle's call order:
    actor train forward, frozen critic, then next-action actor, target critic and online
    critic; two per residual block). The statistics are the ones the kernels used: the
    run's batch statistics in training mode, the evaluation (mean, invstd) prepared from
    the running buffers otherwise. Only runs with a backward matter: a decision taken the
    other way in a forward-only run changes its output by less than the pre-activation's
    own size, i.e. by rounding."""
    ab, cb = L.cfg.actor_num_blocks, L.cfg.critic_num_blocks
    runs = [(L.actor_train, ab), (L.critic_pi, cb)] if actor_phase else []
    runs += [(None, ab), (None, cb), (L.critic_run, cb)]
    adopt, site = {}, 0
    for run, blocks in runs:
        for i in range(blocks):
            for j, (pre, t) in enumerate(((f"encoder.{i}.norm1", run.t1[i] if run else None),
                                          (f"encoder.{i}.norm2", run.t2[i] if run else None))):
                if run is not None:
                    T, C = t.shape[0], t.shape[2]
                    if run.training:
                        mean, inv = run.stats[pre]
                    else:
                        o = run.net.buf_offsets[pre + ".running_mean"]
                        mean, inv = run.net.eval_mean[o:o + T * C], run.net.eval_invstd[o:o + T * C]
                    adopt[site + j] = (t.cpu().numpy(), mean.reshape(T, C).cpu().numpy(),
                                       inv.reshape(T, C).cpu().numpy())
            site += 2
    return adopt


@pytest.mark.parametrize("precision", ["fp32", "fp16"])
@pytest.mark.parametrize("phase", ["actor", "critic"])
def test_gradients_match_oracle_at_config1(phase, precision):
    """Every gradient tensor and metric of one update at exact config 1, against the float64
    oracle (which reproduces the reference at this size, ``tests/test_oracle_golden.py``)
    run from the same initial state with the CUDA path's own ReLU decisions: a decision
    whose pre-activation lies within rounding of the kink is not determined by the
    arithmetic, and each one taken differently moves a 1024-wide layer's gradients by
    ~1e-3, so the oracle rebuilds the CUDA path's decisions from its stored
    pre-normalisation outputs and batch statistics and takes them where they differ (a
    handful per update).
    FP32 recipe within 1e-4 relative L2; FP16 recipe within 1e-2 of the oracle run with
    fp16-rounded product operands. ``phase="critic"`` checks a critic-only update."""
    from oracle import flashsac_np as fs

    spec = G.CONFIG_CASES["cfg1"]
    d, h = G.config_dims(spec), G.config_hyper(spec)
    x = G.config_inputs(spec)[0]
    L = _learner(spec, precision)
    L.load_batch(x["batch"], x["noise"]["actor"], x["noise"]["next"])
    actor_phase = phase == "actor"
    L.run(actor_phase)
    torch.cuda.synchronize()
    state = G.config_oracle_state(spec)
    scale = float(L.critic.opt_state[6]) if precision == "fp16" else 1.0
    if precision == "fp16":
        fs.set_operand_rounding("fp16", scale)
    fs.relu_margin_reset(adopt=_gpu_decisions(L, actor_phase))
    try:
        ref_state, ref_metrics = fs.update_networks(state, x["batch"], x["noise"]["actor"], x["noise"]["next"], d, h,
                                                    do_actor=actor_phase)
        adopted = fs.relu_adopted()
    finally:
        fs.set_operand_rounding("fp32")
        fs.relu_margin_reset()
    tol = TOL[precision]
    bad = []
    for tag, net in (("actor", L.actor), ("critic", L.critic)):
        if tag == "actor" and not actor_phase:
            continue
        for k, ref in ref_state["grads"][tag].items():
            got = net.grad(k).cpu().numpy().astype(np.float64)
            err = float(np.linalg.norm(got - ref) / max(np.linalg.norm(ref), 1e-30))
            if not err <= tol:
                bad.append(f"{tag} {k}: {err:.2e}")
    got_m = {k: float(L.metrics[METRIC_KEYS.index(k)]) for k in L.metric_values(actor_phase)}
    for k, v in got_m.items():
        if abs(v - ref_metrics[k]) > tol * max(1.0, abs(ref_metrics[k])):
            bad.append(f"metric {k}: {v} vs {ref_metrics[k]}")
    assert not bad, f"({adopted} decisions adopted)\n" + "\n".join(bad)
