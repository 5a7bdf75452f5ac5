"""Pin the CPU oracle against golden tensors produced by the reference itself.

The fixtures come from ``tests/golden/make_golden.py``, which runs the reference's
Torch FlashSAC (``src/robolearn/flashsac``) on CPU with injected noise. If the
oracle agrees with them, every GPU parity test that compares against the oracle
is transitively compared against the reference.
"""

import numpy as np
import pytest

from oracle import flashsac_np as fs
from tests import _golden as G

UPDATE_CASES = ["tiny", "small", "asym"]


@pytest.mark.parametrize("case", UPDATE_CASES)
def test_oracle_two_updates_match_reference(case):
    g = G.load(f"flashsac_update_{case}.npz")
    d = G.dims(g)
    h = G.hyper(g)
    state = G.initial_state(g)
    for update in range(2):
        a_noise, n_noise = G.noise(g, update)
        state, metrics = fs.update_networks(state, G.batch(g, update), a_noise, n_noise, d, h,
                                            do_actor=(update % 2 == 0))
        ref = G.metrics(g, update)
        assert set(metrics) == set(ref)
        for k, v in ref.items():
            assert abs(metrics[k] - v) <= 1e-4 * max(1.0, abs(v)), (k, metrics[k], v)
        for tag, ours in (("actor", state["actor"]), ("critic", state["critic"]), ("target", state["target"])):
            theirs = G.network(g, f"after{update}", tag)
            for k, v in theirs.items():
                if k.endswith("num_batches_tracked") or k == "predictor.bin_values":
                    continue
                # running means of zero-mean BN inputs are pure rounding (~1e-10): absolute floor
                np.testing.assert_allclose(ours[k], v, rtol=1e-4, atol=1e-6, err_msg=f"{update} {tag} {k}")
        assert abs(state["log_temp"] - float(g[f"after{update}.temp.log_temp"][0])) < 1e-6
        for tag, opt in (("actor", state["opt_actor"]), ("critic", state["opt_critic"])):
            for k in opt.m:
                key = f"after{update}.opt.{tag}.m.{k}"
                if key in g:
                    assert G.rel_err(opt.m[k], g[key]) < 1e-3, (tag, k)
                    assert G.rel_err(opt.v[k], g[f"after{update}.opt.{tag}.v.{k}"]) < 1e-3, (tag, k)


@pytest.mark.parametrize("case", ["b37", "b64_bins11"])
def test_oracle_categorical_matches_reference(case):
    g = G.load(f"categorical_{case}.npz")
    bins = g["support"].shape[0]
    min_v, max_v = float(g["min_v"]), float(g["max_v"])
    np.testing.assert_array_equal(fs.support(bins, min_v, max_v), g["support"])
    sel = fs.select_min_q(g["next_q"], g["target_log_probs"])
    np.testing.assert_array_equal(sel, g["selected"])
    ent = (g["next_log_probs"] * g["alpha"]).astype(np.float32)
    tgt, _ = fs.categorical_target(sel, g["reward"], g["done"], ent, g["discount"], bins, min_v, max_v)
    np.testing.assert_allclose(tgt, g["target"], rtol=2e-6, atol=1e-7)
    B = g["reward"].shape[0]
    logits = g["online_logits"].astype(np.float64)
    lp = logits - np.log(np.exp(logits - logits.max(-1, keepdims=True)).sum(-1, keepdims=True)) - logits.max(-1, keepdims=True)
    loss, dlog = fs.categorical_loss_grad(lp[:, :B], g["target"].astype(np.float64), 2 * B)
    assert abs(loss - float(g["loss"])) < 1e-5 * abs(float(g["loss"]))
    np.testing.assert_allclose(dlog, g["dlogits"], rtol=1e-4, atol=1e-9)


def test_support_matches_linspace_rule_for_common_bin_counts():
    import torch

    for bins, lo, hi in ((101, -10.0, 10.0), (101, -5.0, 5.0), (11, -5.0, 5.0), (51, -1.0, 3.0), (2, -1.0, 1.0)):
        np.testing.assert_array_equal(fs.support(bins, lo, hi), torch.linspace(lo, hi, bins).numpy())
