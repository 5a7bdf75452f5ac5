"""librl2's ``rl_*`` entry points against the reference's own native library on the same
inputs: ``oracle/_ref/librobolearn_cuda.so``, compiled from the reference's
``src/robolearn/cuda/kernels.cu`` by ``oracle/build_ref.py``. Both libraries are bound with
the reference's ctypes declarations and called with identical arguments; only the output
buffers differ. Tolerances: dense fp32 products 1e-4 of the result's scale (cuBLASLt
pedantic fp32 against three tf32 products per step), everything else 1e-5 or tighter;
fp16 casts, zeroing, loss-scaler state and the timestep exact."""

import ctypes
from pathlib import Path

import numpy as np
import pytest
import torch

from tests._rl_abi import CTYPES, TABLE, bound_library, ints, pointers, sizes

pytestmark = pytest.mark.gpu

REF_LIB = Path(__file__).resolve().parents[1] / "oracle" / "_ref" / "librobolearn_cuda.so"


@pytest.fixture(scope="module")
def libs():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    if not REF_LIB.is_file():
        pytest.skip("oracle/_ref/librobolearn_cuda.so not built (reference sources absent at build time)")
    ref = ctypes.CDLL(str(REF_LIB))
    for name, sig in TABLE.items():
        fn = getattr(ref, name)
        fn.argtypes = [CTYPES[k] for k in sig["argtypes"]]
        fn.restype = CTYPES[sig["restype"]]
    return {"rl2": bound_library(), "ref": ref}


def _s():
    return torch.cuda.current_stream().cuda_stream


def _ok(lib, rc):
    assert rc == 0, lib.rl_last_error().decode()


def _close(a, b, tol):
    a, b = a.double().cpu(), b.double().cpu()
    scale = max(1.0, b.abs().max().item())
    err = (a - b).abs().max().item()
    assert err <= tol * scale, f"max difference {err:.3e} over scale {scale:.3e}"


def _both(libs, fn):
    """Run fn(lib) for librl2 and for the reference library; returns (ours, reference)."""
    out = {k: fn(lib) for k, lib in libs.items()}
    torch.cuda.synchronize()
    return out["rl2"], out["ref"]


@pytest.mark.parametrize(
    "m,n,k,ta,tb,dtype,bias,beta",
    [(37, 101, 39, 0, 0, 0, 1, 0.0), (512, 256, 160, 1, 0, 0, 1, 1.0), (2048, 1024, 512, 0, 1, 1, 1, 0.0),
     (101, 4096, 512, 1, 0, 0, 0, 0.5)],
)
def test_dense_plans_agree(libs, m, n, k, ta, tb, dtype, bias, beta):
    g = torch.Generator().manual_seed(m + n + k)
    lda, ldb, ldd = (k if ta else m), (n if tb else k), m
    dt = torch.float16 if dtype else torch.float32
    A = torch.randn(k if not ta else m, lda, generator=g).to(dt).cuda()
    B = torch.randn(n if not tb else k, ldb, generator=g).to(dt).cuda()
    C = torch.randn(n, ldd, generator=g).cuda()
    bv = torch.randn(m, generator=g).cuda()

    def run(lib):
        plan = lib.rl_plan_create_mixed(m, n, k, ta, tb, lda, ldb, ldd, bias, 0, dtype, 32 << 20)
        assert plan, lib.rl_last_error().decode()
        ws_bytes = lib.rl_plan_workspace(plan)
        ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device="cuda")
        D = C.clone()
        _ok(lib, lib.rl_plan_run(plan, A.data_ptr(), B.data_ptr(), D.data_ptr() if beta else None, D.data_ptr(),
                                 bv.data_ptr() if bias else None, ws.data_ptr(), ws_bytes, beta, _s()))
        torch.cuda.synchronize()
        lib.rl_plan_destroy(plan)
        return D

    ours, ref = _both(libs, run)
    _close(ours, ref, 1e-4 if dtype == 0 else 1e-5)


def _linear_specs(batch, fan_in, fan_out):
    """The three plans the reference's CudaLinear makes per layer (cuda/linear.py:178-186):
    Y^T = W X^T (+ bias), dX^T += W^T dY^T and dW^T += X^T dY on row-major arrays."""
    return (
        (fan_out, batch, fan_in, 1, 0, fan_in, fan_in, fan_out, 1),
        (fan_in, batch, fan_out, 0, 0, fan_in, fan_out, fan_in, 0),
        (fan_in, fan_out, batch, 0, 1, fan_in, fan_out, fan_in, 0),
    )


def _linear_step(lib, dtype, specs, x, w, dy, bias, dx0, dw0, timer=None):
    """Forward, input-gradient and weight-gradient plans of one layer, as CudaLinear runs them."""
    plans, out = [], {}
    try:
        for spec in specs:
            h = (lib.rl_plan_create_mixed(*spec, 0, 1, 32 << 20) if dtype == 1
                 else lib.rl_plan_create(*spec, 0, 32 << 20))
            assert h, lib.rl_last_error().decode()
            plans.append(h)
        ws_bytes = max(lib.rl_plan_workspace(h) for h in plans)
        ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device="cuda")
        y = torch.empty(x.shape[0], w.shape[0], device="cuda")
        dx, dw = dx0.clone(), dw0.clone()
        calls = {
            "forward": lambda: lib.rl_plan_run(plans[0], w.data_ptr(), x.data_ptr(), None, y.data_ptr(),
                                               bias.data_ptr(), ws.data_ptr(), ws_bytes, 0.0, _s()),
            "input_gradient": lambda: lib.rl_plan_run(plans[1], w.data_ptr(), dy.data_ptr(), dx.data_ptr(),
                                                      dx.data_ptr(), None, ws.data_ptr(), ws_bytes, 1.0, _s()),
            "weight_gradient": lambda: lib.rl_plan_run(plans[2], x.data_ptr(), dy.data_ptr(), dw.data_ptr(),
                                                       dw.data_ptr(), None, ws.data_ptr(), ws_bytes, 1.0, _s()),
        }
        for name, call in calls.items():
            _ok(lib, call())
        torch.cuda.synchronize()
        out = {"y": y, "dx": dx, "dw": dw}
        if timer is not None:
            for name, call in calls.items():
                out[name] = timer(lambda call=call: _ok(lib, call()))
    finally:
        for h in plans:
            lib.rl_plan_destroy(h)
    return out


@pytest.mark.parametrize("dtype", [0, 1])
@pytest.mark.parametrize("fan_in,fan_out", [(512, 2048), (2048, 512)])
def test_linear_layer_plans_agree(libs, dtype, fan_in, fan_out):
    g = torch.Generator().manual_seed(fan_in + 3 * fan_out + dtype)
    B = 8192
    dt = torch.float16 if dtype else torch.float32
    x = torch.randn(B, fan_in, generator=g).to(dt).cuda()
    w = (torch.randn(fan_out, fan_in, generator=g) / fan_in ** 0.5).to(dt).cuda()
    dy = (torch.randn(B, fan_out, generator=g) / B).to(dt).cuda()
    bias = torch.randn(fan_out, generator=g).cuda()
    dx0 = torch.randn(B, fan_in, generator=g).cuda()
    dw0 = torch.randn(fan_out, fan_in, generator=g).cuda()
    specs = _linear_specs(B, fan_in, fan_out)
    ours, ref = _both(libs, lambda lib: _linear_step(lib, dtype, specs, x, w, dy, bias, dx0, dw0))
    for name in ("y", "dx", "dw"):
        try:
            _close(ours[name], ref[name], 1e-4 if dtype == 0 else 5e-5)
        except AssertionError as e:
            raise AssertionError(f"{name}: {e}") from None


def test_cast_bias_grad_zero_agree(libs):
    g = torch.Generator().manual_seed(1)
    x = (torch.randn(100003, generator=g) * 5000).cuda()
    dy = torch.randn(4096, 101, generator=g).cuda()
    db0 = torch.randn(101, generator=g).cuda()

    def run(lib):
        h = torch.empty(x.numel(), dtype=torch.float16, device="cuda")
        _ok(lib, lib.rl_cast_f32_f16(x.data_ptr(), h.data_ptr(), x.numel(), _s()))
        db = db0.clone()
        _ok(lib, lib.rl_bias_grad(dy.data_ptr(), db.data_ptr(), 4096, 101, _s()))
        z = torch.ones(70000, device="cuda")
        plan = lib.rl_zero_create(2, pointers([z[3:].data_ptr(), z[9000:].data_ptr()]), sizes([5000, 50001]))
        assert plan
        _ok(lib, lib.rl_zero_step(plan, _s()))
        torch.cuda.synchronize()
        lib.rl_zero_destroy(plan)
        return h, db, z

    (h1, db1, z1), (h2, db2, z2) = _both(libs, run)
    assert torch.equal(h1.view(torch.int16), h2.view(torch.int16))
    _close(db1, db2, 1e-5)
    assert torch.equal(z1, z2)


def test_adam_with_loss_scaling_agrees(libs):
    g = torch.Generator().manual_seed(2)
    shapes = [3, 4096, 70001]
    p0 = [torch.randn(s, generator=g).cuda() for s in shapes]
    grads = [[torch.randn(s, generator=g).cuda() for s in shapes] for _ in range(4)]
    grads[1][2][5] = float("nan")  # the second step is skipped

    def run(lib):
        ps = [t.clone() for t in p0]
        gs = [torch.empty_like(t) for t in p0]
        m1 = [torch.zeros_like(t) for t in p0]
        m2 = [torch.zeros_like(t) for t in p0]
        ts, lr = torch.zeros(1, device="cuda"), torch.tensor([3e-3], device="cuda")
        scale = torch.tensor([256.0], device="cuda")
        ints_state = [torch.zeros(1, dtype=torch.int32, device="cuda") for _ in range(3)]
        counts = [torch.zeros(1, dtype=torch.int64, device="cuda") for _ in range(2)]
        plan = lib.rl_adam_create(3, pointers([t.data_ptr() for t in ps]), pointers([t.data_ptr() for t in gs]),
                                  pointers([t.data_ptr() for t in m1]), pointers([t.data_ptr() for t in m2]),
                                  sizes(shapes), ts.data_ptr(), lr.data_ptr(), 0.9, 0.999, 1e-8)
        assert plan
        _ok(lib, lib.rl_adam_set_scaler(plan, scale.data_ptr(), *[t.data_ptr() for t in ints_state],
                                        *[t.data_ptr() for t in counts], 2.0, 0.5, 3))
        for step in grads:
            for dst, src in zip(gs, step):
                dst.copy_(src * scale)
            _ok(lib, lib.rl_adam_unscale(plan, _s()))
            _ok(lib, lib.rl_adam_step(plan, _s()))
        torch.cuda.synchronize()
        lib.rl_adam_destroy(plan)
        state = [ts.item(), scale.item()] + [t.item() for t in ints_state] + [t.item() for t in counts]
        return ps, m1, m2, state

    (p1, a1, b1, s1), (p2, a2, b2, s2) = _both(libs, run)
    assert s1 == s2
    for x, y in zip(p1 + a1 + b1, p2 + a2 + b2):
        _close(x, y, 1e-6)


def test_projection_and_ema_agree(libs):
    g = torch.Generator().manual_seed(3)
    rows = [torch.randn(n, generator=g).cuda() for n in (1, 160, 2048)]
    w, b, q = torch.randn(512, generator=g).cuda(), torch.randn(512, generator=g).cuda(), torch.randn(99, generator=g).cuda()
    src, dst = torch.randn(123457, generator=g).cuda(), torch.randn(123457, generator=g).cuda()

    def run(lib):
        r = [t.clone() for t in rows]
        ww, bb, qq = w.clone(), b.clone(), q.clone()
        sh = [torch.zeros(t.numel(), dtype=torch.float16, device="cuda") for t in r]
        first = [*r, ww, qq]
        second = [*r, bb, qq]
        plan = lib.rl_flash_projection_create_with_shadows(
            5, pointers([t.data_ptr() for t in first]), pointers([t.data_ptr() for t in second]),
            sizes([t.numel() for t in first]), ints([0, 0, 0, 1, 2]), pointers([t.data_ptr() for t in sh] + [0, 0]))
        assert plan
        _ok(lib, lib.rl_flash_projection_step(plan, _s()))
        d = dst.clone()
        esh = torch.zeros(d.numel(), dtype=torch.float16, device="cuda")
        eplan = lib.rl_flash_ema_create_with_shadows(1, pointers([src.data_ptr()]), pointers([d.data_ptr()]),
                                                     sizes([d.numel()]), 0.005, pointers([esh.data_ptr()]))
        assert eplan
        _ok(lib, lib.rl_flash_ema_step(eplan, _s()))
        torch.cuda.synchronize()
        lib.rl_flash_projection_destroy(plan)
        lib.rl_flash_ema_destroy(eplan)
        return [*r, ww, bb, qq, d], [*sh, esh]

    (v1, h1), (v2, h2) = _both(libs, run)
    for x, y in zip(v1, v2):
        _close(x, y, 1e-6)
    for x, y in zip(h1, h2):  # fp16 copies may differ only where the fp32 values differ by an ulp
        assert (x.float() - y.float()).abs().max().item() <= 1e-3 * max(1.0, y.float().abs().max().item())


@pytest.mark.parametrize("batch,channels,training,relu", [(8192, 2048, 1, 1), (700, 45, 1, 0), (300, 160, 0, 1)])
def test_batch_norm_agrees(libs, batch, channels, training, relu):
    g = torch.Generator().manual_seed(batch + channels)
    x = (1.5 + torch.randn(batch, channels, generator=g)).cuda()
    w, b = torch.randn(channels, generator=g).cuda(), torch.randn(channels, generator=g).cuda()
    dy = torch.randn(batch, channels, generator=g).cuda()
    dx0 = torch.randn(batch, channels, generator=g).cuda()
    chunks = (batch + 255) // 256

    def run(lib):
        rm, rv = torch.full((channels,), 0.2, device="cuda"), torch.full((channels,), 1.3, device="cuda")
        mean, var = torch.zeros(channels, device="cuda"), torch.zeros(channels, device="cuda")
        partial = torch.zeros(2 * chunks * channels, device="cuda")
        sums = torch.zeros(2 * channels, device="cuda")
        y = torch.empty_like(x)
        y16 = torch.empty(batch, channels, dtype=torch.float16, device="cuda")
        _ok(lib, lib.rl_flash_bn_forward_with_fp16(x.data_ptr(), w.data_ptr(), b.data_ptr(), rm.data_ptr(),
                                                   rv.data_ptr(), mean.data_ptr(), var.data_ptr(), partial.data_ptr(),
                                                   y.data_ptr(), y16.data_ptr(), batch, channels, 1e-5, 0.01, training,
                                                   relu, _s()))
        m_ptr, v_ptr = (mean, var) if training else (rm, rv)
        dx, dw, db = dx0.clone(), torch.zeros(channels, device="cuda"), torch.zeros(channels, device="cuda")
        dx16 = torch.empty(batch, channels, dtype=torch.float16, device="cuda")
        _ok(lib, lib.rl_flash_bn_backward_with_fp16(x.data_ptr(), dy.data_ptr(), y.data_ptr(), w.data_ptr(),
                                                    m_ptr.data_ptr(), v_ptr.data_ptr(), partial.data_ptr(),
                                                    sums.data_ptr(), dx.data_ptr(), dw.data_ptr(), db.data_ptr(),
                                                    dx16.data_ptr(), batch, channels, 1e-5, training, relu, _s()))
        return [y, mean, var, rm, rv, dx, dw, db], [y16, dx16]

    (v1, h1), (v2, h2) = _both(libs, run)
    names = ["y", "mean", "var", "running_mean", "running_var", "dx", "dw", "db"]
    for name, x1, x2 in zip(names, v1, v2):
        tol = 1e-4 if name in ("dw", "db") else 1e-5
        try:
            _close(x1, x2, tol)
        except AssertionError as e:
            raise AssertionError(f"{name}: {e}") from None
    for x1, x2 in zip(h1, h2):
        assert (x1.float() - x2.float()).abs().max().item() <= 1e-3 * max(1.0, x2.float().abs().max().item())


def test_rms_norm_agrees(libs):
    g = torch.Generator().manual_seed(4)
    B, C = 8192, 512
    x = torch.randn(B, C, generator=g).cuda()
    w = torch.randn(C, generator=g).cuda()
    dy = torch.randn(B, C, generator=g).cuda()

    def run(lib):
        var, y = torch.empty(B, device="cuda"), torch.empty(B, C, device="cuda")
        _ok(lib, lib.rl_flash_rms_forward(x.data_ptr(), w.data_ptr(), var.data_ptr(), y.data_ptr(), B, C, 1e-6, _s()))
        dx, dw = torch.zeros(B, C, device="cuda"), torch.zeros(C, device="cuda")
        partial = torch.zeros(((B + 255) // 256) * C, device="cuda")
        _ok(lib, lib.rl_flash_rms_backward(x.data_ptr(), dy.data_ptr(), w.data_ptr(), var.data_ptr(),
                                           partial.data_ptr(), dx.data_ptr(), dw.data_ptr(), B, C, 1e-6, _s()))
        return var, y, dx, dw

    for x1, x2 in zip(*_both(libs, run)):
        _close(x1, x2, 1e-5)


@pytest.mark.parametrize("batch,bins", [(4096, 101), (300, 51)])
def test_categorical_heads_agree(libs, batch, bins):
    rng = np.random.default_rng(batch + bins)
    f32 = lambda a: torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).cuda()  # noqa: E731
    raw, bias = f32(rng.standard_normal((batch, bins))), f32(rng.standard_normal(bins))
    support = torch.linspace(-10, 10, bins).cuda()
    dlp, dq = f32(rng.standard_normal((batch, bins))), f32(rng.standard_normal(batch))
    q = f32(rng.standard_normal((2, 2 * batch)))
    logits = rng.standard_normal((2, 2 * batch, bins))
    lp_in = f32(logits - np.log(np.exp(logits).sum(-1, keepdims=True)))
    reward, term = f32(rng.standard_normal(batch) * 2), f32(rng.random(batch) < 0.1)
    disc, nlp, alpha = f32(np.full(batch, 0.99)), f32(rng.standard_normal(batch)), f32([0.05])

    def run(lib):
        lp, val = torch.empty(batch, bins, device="cuda"), torch.empty(batch, device="cuda")
        _ok(lib, lib.rl_flash_categorical_forward(raw.data_ptr(), bias.data_ptr(), support.data_ptr(), lp.data_ptr(),
                                                  val.data_ptr(), batch, bins, _s()))
        draw, dbias = torch.zeros(batch, bins, device="cuda"), torch.zeros(bins, device="cuda")
        scratch = torch.empty(batch, bins, device="cuda")
        _ok(lib, lib.rl_flash_categorical_backward(lp.data_ptr(), support.data_ptr(), dlp.data_ptr(), dq.data_ptr(),
                                                   scratch.data_ptr(), draw.data_ptr(), dbias.data_ptr(), batch, bins,
                                                   _s()))
        target = torch.empty(batch, bins, device="cuda")
        max_ent = torch.tensor([-3.0e38], device="cuda")
        _ok(lib, lib.rl_flash_categorical_target(q.data_ptr(), lp_in.data_ptr(), reward.data_ptr(), term.data_ptr(),
                                                 disc.data_ptr(), nlp.data_ptr(), alpha.data_ptr(), target.data_ptr(),
                                                 max_ent.data_ptr(), batch, bins, -10.0, 10.0, _s()))
        return lp, val, draw, dbias, target, max_ent

    ours, ref = _both(libs, run)
    for name, x1, x2 in zip(["log_probs", "values", "draw", "dbias", "target", "max_entropy"], ours, ref):
        try:
            _close(x1, x2, 1e-4 if name == "dbias" else 1e-5)
        except AssertionError as e:
            raise AssertionError(f"{name}: {e}") from None
    assert ours[5].item() == ref[5].item()


def test_reference_library_timing(libs):
    """Times each entry-point family at cfg3 sizes in both libraries (CUDA events, 200 MB L2
    flush before every timed call, median of 10 after 3 warm-up calls) and writes the table
    as JSON to ``$RL2_REFOPS_OUT`` when that is set; asserts only that every call succeeds.
    The reference library is the GPU baseline of the reference's native backend."""
    import json
    import os

    g = torch.Generator().manual_seed(5)
    flush = torch.empty(50 * 1024 * 1024, device="cuda")
    rows, hidden, wide, bins = 8192, 512, 2048, 101

    def timed(fn, reps=10, warm=3):
        for _ in range(warm):
            fn()
        ts = []
        for _ in range(reps):
            flush.zero_()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            fn()
            b.record()
            torch.cuda.synchronize()
            ts.append(a.elapsed_time(b) * 1e3)
        return float(np.median(ts))

    x16 = torch.randn(rows, hidden, generator=g).half().cuda()
    w16 = torch.randn(wide, hidden, generator=g).half().cuda()
    x32, w32 = x16.float(), w16.float()
    bias = torch.randn(wide, generator=g).cuda()
    xb = torch.randn(rows, wide, generator=g).cuda()
    dyb = torch.randn(rows, wide, generator=g).cuda()
    wb, bb = torch.randn(wide, generator=g).cuda(), torch.randn(wide, generator=g).cuda()
    xr, dyr, wr = xb[:, :hidden].contiguous(), dyb[:, :hidden].contiguous(), wb[:hidden].contiguous()
    raw = torch.randn(rows, bins, generator=g).cuda()
    cb, support = torch.randn(bins, generator=g).cuda(), torch.linspace(-10, 10, bins).cuda()
    q = torch.randn(2, rows, generator=g).cuda()
    lp_in = torch.log_softmax(torch.randn(2, rows, bins, generator=g), -1).cuda()
    half = rows // 2
    rew, term = torch.randn(half, generator=g).cuda(), torch.zeros(half, device="cuda")
    disc, nlp, alpha = torch.full((half,), 0.99, device="cuda"), torch.randn(half, generator=g).cuda(), torch.tensor([0.05], device="cuda")
    n_params = [wide * hidden] * 4 + [hidden * wide] * 4 + [wide] * 16 + [hidden * 160] * 2
    params = [torch.randn(n, generator=g).cuda() for n in n_params]
    table = {}

    for name, lib in libs.items():
        res = {}
        # dense: Y^T (wide x rows) = W (wide x hidden) . X^T, column-major views of row-major X, W
        for dtype, (xa, wa) in ((1, (x16, w16)), (0, (x32, w32))):
            plan = lib.rl_plan_create_mixed(wide, rows, hidden, 1, 0, hidden, hidden, wide, 1, 0, dtype, 32 << 20)
            assert plan, lib.rl_last_error().decode()
            wsb = lib.rl_plan_workspace(plan)
            ws = torch.empty(max(wsb, 1), dtype=torch.uint8, device="cuda")
            out = torch.empty(rows, wide, device="cuda")
            res[f"dense_fp{16 if dtype else 32}_{wide}x{rows}x{hidden}"] = timed(lambda: _ok(lib, lib.rl_plan_run(
                plan, wa.data_ptr(), xa.data_ptr(), None, out.data_ptr(), bias.data_ptr(), ws.data_ptr(), wsb, 0.0, _s())))
            lib.rl_plan_destroy(plan)
        for dtype, (xa, wa) in ((1, (x16, w16)), (0, (x32, w32))):
            dy_l = torch.randn(rows, wide, generator=g).to(xa.dtype).cuda()
            dx_l, dw_l = torch.zeros(rows, hidden, device="cuda"), torch.zeros(wide, hidden, device="cuda")
            t = _linear_step(lib, dtype, _linear_specs(rows, hidden, wide), xa, wa, dy_l, bias, dx_l, dw_l, timed)
            for part in ("forward", "input_gradient", "weight_gradient"):
                res[f"linear_{part}_fp{16 if dtype else 32}_{rows}x{hidden}->{wide}"] = t[part]
        chunks = (rows + 255) // 256
        rm, rv = torch.zeros(wide, device="cuda"), torch.ones(wide, device="cuda")
        mean, var = torch.zeros(wide, device="cuda"), torch.zeros(wide, device="cuda")
        partial, sums = torch.zeros(2 * chunks * wide, device="cuda"), torch.zeros(2 * wide, device="cuda")
        y, y16 = torch.empty_like(xb), torch.empty(rows, wide, dtype=torch.float16, device="cuda")
        dx, dw, db = torch.zeros_like(xb), torch.zeros(wide, device="cuda"), torch.zeros(wide, device="cuda")
        res[f"bn_forward_train_relu_{rows}x{wide}"] = timed(lambda: _ok(lib, lib.rl_flash_bn_forward_with_fp16(
            xb.data_ptr(), wb.data_ptr(), bb.data_ptr(), rm.data_ptr(), rv.data_ptr(), mean.data_ptr(), var.data_ptr(),
            partial.data_ptr(), y.data_ptr(), y16.data_ptr(), rows, wide, 1e-5, 0.01, 1, 1, _s())))
        res[f"bn_backward_train_relu_{rows}x{wide}"] = timed(lambda: _ok(lib, lib.rl_flash_bn_backward(
            xb.data_ptr(), dyb.data_ptr(), y.data_ptr(), wb.data_ptr(), mean.data_ptr(), var.data_ptr(),
            partial.data_ptr(), sums.data_ptr(), dx.data_ptr(), dw.data_ptr(), db.data_ptr(), rows, wide, 1e-5, 1, 1,
            _s())))
        rvar, ry = torch.empty(rows, device="cuda"), torch.empty_like(xr)
        rdx, rdw = torch.zeros_like(xr), torch.zeros(hidden, device="cuda")
        rpart = torch.zeros(chunks * hidden, device="cuda")
        res[f"rms_forward_{rows}x{hidden}"] = timed(lambda: _ok(lib, lib.rl_flash_rms_forward(
            xr.data_ptr(), wr.data_ptr(), rvar.data_ptr(), ry.data_ptr(), rows, hidden, 1e-6, _s())))
        res[f"rms_backward_{rows}x{hidden}"] = timed(lambda: _ok(lib, lib.rl_flash_rms_backward(
            xr.data_ptr(), dyr.data_ptr(), wr.data_ptr(), rvar.data_ptr(), rpart.data_ptr(), rdx.data_ptr(),
            rdw.data_ptr(), rows, hidden, 1e-6, _s())))
        lp, val = torch.empty(rows, bins, device="cuda"), torch.empty(rows, device="cuda")
        draw, dcb, scratch = torch.zeros(rows, bins, device="cuda"), torch.zeros(bins, device="cuda"), torch.empty(rows, bins, device="cuda")
        res[f"categorical_forward_{rows}x{bins}"] = timed(lambda: _ok(lib, lib.rl_flash_categorical_forward(
            raw.data_ptr(), cb.data_ptr(), support.data_ptr(), lp.data_ptr(), val.data_ptr(), rows, bins, _s())))
        res[f"categorical_backward_{rows}x{bins}"] = timed(lambda: _ok(lib, lib.rl_flash_categorical_backward(
            lp.data_ptr(), support.data_ptr(), raw.data_ptr(), val.data_ptr(), scratch.data_ptr(), draw.data_ptr(),
            dcb.data_ptr(), rows, bins, _s())))
        tgt, ment = torch.empty(half, bins, device="cuda"), torch.zeros(1, device="cuda")
        res[f"categorical_target_{half}x{bins}"] = timed(lambda: _ok(lib, lib.rl_flash_categorical_target(
            q.data_ptr(), lp_in.data_ptr(), rew.data_ptr(), term.data_ptr(), disc.data_ptr(), nlp.data_ptr(),
            alpha.data_ptr(), tgt.data_ptr(), ment.data_ptr(), half, bins, -10.0, 10.0, _s())))
        gr = [torch.randn_like(t) * 1e-3 for t in params]
        m1, m2 = [torch.zeros_like(t) for t in params], [torch.zeros_like(t) for t in params]
        ts, lr = torch.zeros(1, device="cuda"), torch.tensor([1e-4], device="cuda")
        tab = lambda ts_: pointers([t.data_ptr() for t in ts_])  # noqa: E731
        adam = lib.rl_adam_create(len(params), tab(params), tab(gr), tab(m1), tab(m2), sizes(n_params),
                                  ts.data_ptr(), lr.data_ptr(), 0.9, 0.999, 1e-8)
        assert adam
        res[f"adam_{sum(n_params)}_params"] = timed(lambda: _ok(lib, lib.rl_adam_step(adam, _s())))
        lib.rl_adam_destroy(adam)
        targets = [t.clone() for t in params]
        ema = lib.rl_flash_ema_create(len(params), tab(params), tab(targets), sizes(n_params), 0.005)
        assert ema
        res[f"ema_{sum(n_params)}_params"] = timed(lambda: _ok(lib, lib.rl_flash_ema_step(ema, _s())))
        lib.rl_flash_ema_destroy(ema)
        table[name] = res

    out = {k: {"rl2_us": round(table["rl2"][k], 2), "reference_us": round(table["ref"][k], 2),
               "reference_over_rl2": round(table["ref"][k] / table["rl2"][k], 2)} for k in table["rl2"]}
    path = os.environ.get("RL2_REFOPS_OUT")
    if path:
        Path(path).write_text(json.dumps({"device": torch.cuda.get_device_name(0), "ops": out}, indent=1) + "\n")
