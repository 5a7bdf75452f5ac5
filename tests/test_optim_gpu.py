"""The fused optimizer pass (``rl2_adam_step``) unit by unit against a float32 restatement.

Units cover every path of the kernel: one warp per unit (lengths <= the warp limit) and one
CTA per unit, 16-byte vectors (offsets and lengths multiples of four floats) and the scalar
form (odd lengths, odd offsets), every projection kind (plain, unit-linear row, BN pair, RMS
scale), both Adam formulas, the skipped step of the loss scaler, the refresh-only call (no
gradients), the target EMA and the fp16 / tf32 hi + lo operand planes. Semantics:
torch Adam / Warp-NN Adam (``src/robolearn/cuda/kernels.cu:310-337``), projection
(``src/robolearn/flashsac/layers.py:24-29,57-64,76-81``), EMA (``flashsac/_utils/network.py:66-80``).
"""

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

from robolearn_b200 import _native as N  # noqa: E402

# (kind, length, count, misalign): misalign shifts the unit's offset by one float
UNITS = [(1, 512, 6, 0), (1, 123, 5, 0), (1, 2048, 3, 0), (1, 1000, 2, 1), (1, 4096, 1, 0), (2, 256, 2, 0),
         (2, 1024, 2, 0), (2, 300, 1, 1), (3, 512, 1, 0), (3, 4096, 1, 0), (0, 37, 2, 0), (0, 4096, 1, 0),
         (1, 8, 3, 0)]


def _layout():
    rows, off, plane_off = [], 0, 0
    for kind, n, count, mis in UNITS:
        for _ in range(count):
            off += mis
            o2 = -1
            if kind == 2:
                o2 = off + n + 4 + mis
            po = -1
            if kind == 1:
                po = plane_off
                plane_off += (n + 7) // 8 * 8
            rows.append((off, o2, po, n, kind))
            off = (max(off + n, o2 + n if o2 >= 0 else 0) + 3) // 4 * 4 + 4
    return rows, off, plane_off


def _reference(rows, arrays, formula, st, project, tau, with_grads):
    p, g, m, v, t = (arrays[k].clone() for k in ("p", "g", "m", "v", "t"))
    def f32(x):  # a float32 value as a Python float (exact)
        return float(np.float32(x))

    b1, b2, eps = f32(0.9), f32(0.999), f32(1e-8)
    c1, c2 = f32(np.float32(1) - np.float32(0.9)), f32(np.float32(1) - np.float32(0.999))  # the kernel's (1 - beta)
    update = st[5] == 0
    for off, o2, _, n, kind in rows:
        idx = [torch.arange(off, off + n)] + ([torch.arange(o2, o2 + n)] if kind == 2 else [])
        vals = []
        for ix in idx:
            pv = p[ix]
            if update and with_grads:
                gv, mv, vv = g[ix], m[ix], v[ix]
                s2, s3, s4 = (torch.tensor(st[i], dtype=torch.float32) for i in (2, 3, 4))
                if formula == 0:
                    mv = mv + c1 * (gv - mv)
                    vv = vv * b2 + c2 * gv * gv
                    pv = pv - s2 * (mv / (torch.sqrt(vv) / s3 + eps))
                else:
                    mv = b1 * mv + c1 * gv
                    vv = b2 * vv + c2 * (gv * gv)
                    pv = pv - s4 * ((mv * s2) / (torch.sqrt(vv * s3) + eps))
                m[ix], v[ix] = mv, vv
            vals.append(pv)
        if kind != 0 and project:
            total = sum(float((x.double() ** 2).sum()) for x in vals)
            if kind == 1:
                vals = [x / max(np.sqrt(total), 1e-8) for x in vals]
            else:
                vals = [x * np.float32(np.sqrt(n) / np.sqrt(total + 1e-8)) for x in vals]
        for ix, pv in zip(idx, vals):
            p[ix] = pv
            if tau is not None:
                t[ix] = t[ix] + f32(tau) * (pv - t[ix])
    return p, m, v, t


@pytest.mark.parametrize("formula", [0, 1])
@pytest.mark.parametrize("plane", ["fp16", "tf32"])
@pytest.mark.parametrize("mode", ["step", "skip", "refresh"])
def test_fused_step_matches_float32_restatement(formula, plane, mode):
    lib = N.load()
    rows, size, plane_size = _layout()
    gen = torch.Generator().manual_seed(formula * 7 + len(plane) + len(mode))
    arrays = {k: torch.randn(size, generator=gen) for k in ("p", "g", "t")}
    arrays["m"] = torch.randn(size, generator=gen) * 0.1
    arrays["v"] = torch.rand(size, generator=gen) * 0.01
    st = torch.tensor([3, 2, 1e-3 / 0.19, 0.0446, 1e-3, 1.0 if mode == "skip" else 0.0, 1, 0, 0], dtype=torch.float32)
    if formula == 1:
        st[2], st[3] = 1 / 0.19, 1 / 0.002
    with_grads = mode != "refresh"
    tau = 0.005 if mode != "refresh" else None
    dev = {k: x.cuda() for k, x in arrays.items()}
    dst = st.cuda()
    table, count, warp_units = N.segment_table(rows, "cuda")
    assert 0 < warp_units < count
    wp_t = {"h16": torch.zeros(plane_size, dtype=torch.float16, device="cuda")} if plane == "fp16" else \
        {"hi": torch.zeros(plane_size, device="cuda"), "lo": torch.zeros(plane_size, device="cuda")}
    tp_t = {k: torch.zeros_like(x) for k, x in wp_t.items()}
    wp = N.Plane(**{k: x.data_ptr() for k, x in wp_t.items()})
    tp = N.Plane(**{k: x.data_ptr() for k, x in tp_t.items()}) if tau is not None else N.Plane()
    a = N.AdamArgs(params=dev["p"].data_ptr(), grads=dev["g"].data_ptr() if with_grads else None,
                   m=dev["m"].data_ptr() if with_grads else None, v=dev["v"].data_ptr() if with_grads else None,
                   segments=table.data_ptr(), count=count, state=dst.data_ptr() if with_grads else None,
                   formula=formula, beta1=0.9, beta2=0.999, eps=1e-8, project=1, weight_plane=wp,
                   target_params=dev["t"].data_ptr() if tau is not None else None, tau=tau or 0.0, target_plane=tp,
                   warp_segments=warp_units)
    N.check(lib.rl2_adam_step(ctypes.byref(a), N.stream_ptr()), "adam step")
    torch.cuda.synchronize()
    ref_st = st if with_grads else torch.tensor([0, 0, 0, 1, 0, 0, 0, 0, 0], dtype=torch.float32)
    p, m, v, t = _reference(rows, arrays, formula, ref_st.tolist(), True, tau, with_grads)
    for name, want in (("params", p), ("m", m), ("v", v), ("target", t)):
        got = dev[{"params": "p", "target": "t"}.get(name, name)].cpu()
        torch.testing.assert_close(got, want, rtol=2e-6, atol=2e-7, msg=name)
    # untouched gaps between units stay as they were
    covered = torch.zeros(size, dtype=torch.bool)
    for off, o2, _, n, kind in rows:
        covered[off:off + n] = True
        if kind == 2:
            covered[o2:o2 + n] = True
    assert torch.equal(dev["p"].cpu()[~covered], arrays["p"][~covered])
    for planes, src in ((wp_t, dev["p"]), (tp_t, dev["t"]) if tau is not None else (None, None)):
        if planes is None:
            continue
        for off, _, po, n, kind in rows:
            if po < 0:
                continue
            vals = src[off:off + n]
            if plane == "fp16":
                assert torch.equal(planes["h16"][po:po + n], vals.half())
            else:
                hi, lo = planes["hi"][po:po + n], planes["lo"][po:po + n]
                assert torch.equal(hi, (vals.view(torch.int32) & -8192).view(torch.float32))
                assert torch.equal(lo, vals - hi)


def test_segment_table_puts_warp_units_first():
    lib = N.load()
    rows, _, _ = _layout()
    table, count, warp_units = N.segment_table(rows, "cpu")
    recs = (N.Segment * count).from_buffer_copy(table.numpy().tobytes())
    lens = [r.length for r in recs]
    limit = lib.rl2_segment_warp_max_length()
    assert all(n <= limit for n in lens[:warp_units]) and all(n > limit for n in lens[warp_units:])
    assert sorted(lens) == sorted(r[3] for r in rows)
