"""Fused categorical critic objective (``rl2_critic_objective``) vs the reference.

Small cases compare with the golden tensors of the reference's own functions
(``updates.py:19-80,248-257``) and with the pinned oracle; the full cfg4 size
(65,536 rows x 101 atoms, config 4's distributions) is checked against the oracle at the
same tolerances as the small cases, and through size-independent properties: mass
conservation of the projected target, zero-sum logits gradients, bias gradient =
column sums, and bitwise run-to-run determinism.
"""

import numpy as np
import pytest
import torch

from oracle import flashsac_np as fs
from tests import _golden as G

pytestmark = pytest.mark.gpu

from robolearn_b200.categorical import CriticObjective, support  # noqa: E402


def _launch(target_lp, online_logits, reward, done, discount, next_lp, alpha, min_v, max_v, outputs=("fp32",),
            padded=False):
    """target_lp: [2, B, bins] next-half distributions; online_logits: [2, 2B, bins].
    ``padded``: logits rows padded to a multiple of four floats (16-byte rows, the layout the
    critic head product writes), which takes the shared-memory staged kernel."""
    twins, B, bins = target_lp.shape
    dev = "cuda"
    ld = (bins + 3) // 4 * 4 if padded else bins
    # the kernel reads the next half at rows B..2B-1 of a [2, 2B, ld] target tensor
    tgt_full = torch.zeros(2, 2 * B, ld, device=dev)
    tgt_full[:, B:, :bins] = torch.as_tensor(target_lp, device=dev)
    onl = torch.zeros(2, 2 * B, ld, device=dev)
    onl[:, :, :bins] = torch.as_tensor(online_logits, device=dev)
    obj = CriticObjective(B, bins, min_v, max_v)
    out = dict(
        loss=torch.zeros(1, device=dev), ent=torch.zeros(1, device=dev),
        bias=torch.zeros(2, bins, device=dev), target=torch.zeros(B, bins, device=dev),
        dlogits=torch.zeros(2, 2 * B, bins, device=dev),
    )
    kw = {}
    if "fp16" in outputs:
        out["d16"] = torch.zeros(2, 2 * B, bins + 3, device=dev, dtype=torch.float16)
        out["scale"] = torch.tensor([1024.0], device=dev)
        kw.update(d16=out["d16"], d16_row_stride=bins + 3, d16_twin_stride=2 * B * (bins + 3), d16_scale=out["scale"])
    if "tf32" in outputs:
        out["hi"] = torch.zeros(2, 2 * B, bins, device=dev)
        out["lo"] = torch.zeros(2, 2 * B, bins, device=dev)
        kw.update(d_hi=out["hi"], d_lo=out["lo"], dplane_row_stride=bins, dplane_twin_stride=2 * B * bins)
    t = lambda x: torch.as_tensor(np.asarray(x, dtype=np.float32), device=dev)  # noqa: E731
    obj.run(target_logits=tgt_full, target_row_stride=ld, target_twin_stride=2 * B * ld, target_row_offset=B,
            online_logits=onl, online_row_stride=ld, online_twin_stride=2 * B * ld, reward=t(reward),
            terminated=t(done), discount=t(discount), next_log_pi=t(next_lp), alpha=t([alpha]),
            loss_weight=1.0 / (2 * B), loss_out=out["loss"], max_entropy_out=out["ent"], bias_grad_out=out["bias"],
            dlogits=out["dlogits"], dlogits_row_stride=bins, dlogits_twin_stride=2 * B * bins,
            target_out=out["target"], target_out_row_stride=bins, **kw)
    torch.cuda.synchronize()
    return {k: v.cpu().numpy() for k, v in out.items()}


def _oracle(target_lp, online_logits, reward, done, discount, next_lp, alpha, min_v, max_v):
    bins = target_lp.shape[-1]
    z = fs.support(bins, min_v, max_v).astype(np.float64)
    q = (np.exp(target_lp.astype(np.float64)) * z).sum(-1)
    sel = fs.select_min_q(q, target_lp)
    ent = (np.float32(alpha) * next_lp.astype(np.float32)).astype(np.float32)
    tgt, _ = fs.categorical_target(sel, reward, done, ent, discount, bins, min_v, max_v)
    B = reward.shape[0]
    lg = online_logits.astype(np.float64)
    lp = lg - lg.max(-1, keepdims=True)
    lp = lp - np.log(np.exp(lp).sum(-1, keepdims=True))
    loss, d = fs.categorical_loss_grad(lp[:, :B], tgt, 2 * B)
    return tgt, loss, d, ent.max()


@pytest.mark.parametrize("case", ["b37", "b64_bins11"])
def test_matches_golden_and_oracle(case):
    g = G.load(f"categorical_{case}.npz")
    min_v, max_v = float(g["min_v"]), float(g["max_v"])
    args = (g["target_log_probs"], g["online_logits"], g["reward"], g["done"], g["discount"],
            g["next_log_probs"], float(g["alpha"]), min_v, max_v)
    out = _launch(*args)
    tgt, loss, d, ent = _oracle(*args)
    B = g["reward"].shape[0]
    np.testing.assert_allclose(out["target"], tgt, rtol=2e-5, atol=2e-7)
    # rows >= 3 were not forced to q-ties in the fixture: direct comparison with the reference
    np.testing.assert_allclose(out["target"][3:], g["target"][3:], rtol=2e-5, atol=2e-7)
    assert abs(out["loss"][0] - loss) <= 1e-5 * abs(loss)
    np.testing.assert_allclose(out["dlogits"], d, rtol=1e-4, atol=1e-9)
    np.testing.assert_allclose(out["dlogits"][:, 3:B], g["dlogits"][:, 3:B], rtol=1e-4, atol=1e-9)
    assert abs(out["ent"][0] - float(g["max_entropy"])) <= 1e-7
    np.testing.assert_allclose(out["bias"], d.sum(axis=1), rtol=1e-4, atol=1e-8)


@pytest.mark.parametrize("padded", [False, True])
@pytest.mark.parametrize("B,bins,min_v,max_v", [(4096, 101, -10.0, 10.0), (999, 51, -5.0, 5.0), (257, 128, -1.0, 3.0),
                                               (37, 11, -5.0, 5.0)])
def test_random_against_oracle(B, bins, min_v, max_v, padded):
    rng = np.random.default_rng(B + bins)
    tl = rng.standard_normal((2, B, bins)).astype(np.float32)
    target_lp = tl - np.log(np.exp(tl).sum(-1, keepdims=True))
    online = rng.standard_normal((2, 2 * B, bins)).astype(np.float32)
    reward = (3 * rng.standard_normal(B)).astype(np.float32)
    done = (rng.random(B) < 0.01).astype(np.float32)
    discount = np.full(B, 0.99, np.float32)
    next_lp = rng.standard_normal(B).astype(np.float32)
    args = (target_lp.astype(np.float32), online, reward, done, discount, next_lp, 0.01, min_v, max_v)
    out = _launch(*args, outputs=("fp32", "fp16", "tf32"), padded=padded)
    tgt, loss, d, ent = _oracle(*args)
    np.testing.assert_allclose(out["target"], tgt, rtol=2e-5, atol=2e-7)
    assert abs(out["loss"][0] - loss) <= 1e-5 * abs(loss)
    np.testing.assert_allclose(out["dlogits"], d, rtol=1e-4, atol=1e-9)
    np.testing.assert_array_equal(out["hi"] + out["lo"], out["dlogits"])
    d16 = out["d16"][:, :, :bins].astype(np.float32) / 1024.0
    np.testing.assert_allclose(d16[:, :B], out["dlogits"][:, :B], rtol=2e-3, atol=1e-7)


@pytest.mark.parametrize("padded", [False, True])
def test_full_size_against_oracle_properties_and_determinism(padded):
    B, bins = 65536, 101
    g = torch.Generator(device="cuda").manual_seed(4)
    tl = torch.log_softmax(torch.randn(2, B, bins, device="cuda", generator=g), -1)
    online = torch.randn(2, 2 * B, bins, device="cuda", generator=g)
    reward = torch.randn(B, device="cuda", generator=g)
    done = (torch.rand(B, device="cuda", generator=g) < 0.01).float()
    args = (tl.cpu().numpy(), online.cpu().numpy(), reward.cpu().numpy(), done.cpu().numpy(),
            np.full(B, 0.99, np.float32), torch.randn(B, generator=None).numpy(), 0.01, -10.0, 10.0)
    first = _launch(*args, padded=padded)
    second = _launch(*args, padded=padded)
    for k in ("target", "loss", "dlogits", "bias", "ent"):
        np.testing.assert_array_equal(first[k], second[k])
    np.testing.assert_allclose(first["target"].sum(-1), 1.0, atol=2e-6)
    assert np.abs(first["dlogits"].sum(-1)).max() < 1e-9
    assert np.all(first["dlogits"][:, B:] == 0)
    np.testing.assert_allclose(first["bias"], first["dlogits"].astype(np.float64).sum(1), rtol=1e-3, atol=1e-7)
    assert np.isfinite(first["loss"]).all()
    tgt, loss, d, ent = _oracle(*args)
    np.testing.assert_allclose(first["target"], tgt, rtol=2e-5, atol=2e-7)
    assert abs(first["loss"][0] - loss) <= 1e-5 * abs(loss)
    np.testing.assert_allclose(first["dlogits"], d, rtol=1e-4, atol=1e-9)
    assert abs(first["ent"][0] - ent) <= 1e-7 * max(1.0, abs(ent))


def test_support_matches_oracle_rule():
    for bins, lo, hi in ((101, -10.0, 10.0), (11, -5.0, 5.0), (51, -1.0, 3.0)):
        np.testing.assert_array_equal(support(bins, lo, hi), fs.support(bins, lo, hi))
