"""The reference's native ABI (``rl_*``) on librl2, called through the reference's own ctypes
declarations, against the oracle / float64 restatements of the reference kernels
(``src/robolearn/cuda/kernels.cu``, ``flash_kernels.cuh``, ``categorical_kernels.cuh``,
``zero_kernels.cuh``). Tolerances: fp32 results 1e-4 relative to the result's scale
(dense products: three tf32 products per step); fp16 copies bit-equal to rounding the
fp32 result; zeroing and index-derived values exact."""

import json
import math

import numpy as np
import pytest
import torch

from oracle import flashsac_np as O
from tests._rl_abi import bound_library, ints, pointers, sizes

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    return bound_library()


def _s():
    return torch.cuda.current_stream().cuda_stream


def _ok(lib, rc):
    assert rc == 0, lib.rl_last_error().decode()


def _close(got, ref, tol=1e-4):
    got = got.double().cpu()
    ref = torch.as_tensor(ref).double().cpu()
    scale = max(1.0, ref.abs().max().item())
    err = (got - ref).abs().max().item()
    assert err <= tol * scale, f"max error {err:.3e} over scale {scale:.3e}"


def _gen(seed):
    return torch.Generator().manual_seed(seed)


# ---------------------------------------------------------------------------- dense plans


@pytest.mark.parametrize(
    "m,n,k,ta,tb,dtype,bias,beta,alias",
    [
        (37, 101, 39, 0, 0, 0, 1, 0.0, False),
        (37, 101, 39, 1, 1, 0, 0, 1.0, True),
        (256, 300, 160, 1, 0, 0, 1, 1.0, False),  # >= 128 output columns: transposed epilogue
        (512, 128, 64, 0, 1, 1, 1, 0.5, False),  # fp16 operands, general beta
        (130, 70, 512, 0, 0, 1, 0, 1.0, True),
    ],
)
def test_dense_plan_matches_column_major_product(lib, m, n, k, ta, tb, dtype, bias, beta, alias):
    g = _gen(m * 1000 + n * 10 + k)
    lda, ldb, ldd = (k if ta else m) + 3, (n if tb else k) + 5, m + 2
    a_rows, a_cols = (k, m) if ta else (m, k)
    b_rows, b_cols = (n, k) if tb else (k, n)
    dt = torch.float16 if dtype else torch.float32
    A = torch.randn(a_cols, lda, generator=g).to(dt)  # column-major storage: one row per column
    B = torch.randn(b_cols, ldb, generator=g).to(dt)
    C = torch.randn(n, ldd, generator=g)
    bv = torch.randn(m, generator=g)
    amat = A[:, :a_rows].T.double()
    bmat = B[:, :b_rows].T.double()
    prod = (amat.T if ta else amat) @ (bmat.T if tb else bmat)  # m x n
    if bias:
        prod = prod + bv.double()[:, None]
    ref = prod + beta * C[:, :m].T.double() if beta else prod

    plan = lib.rl_plan_create_mixed(m, n, k, ta, tb, lda, ldb, ldd, bias, 0, dtype, 32 << 20)
    assert plan, lib.rl_last_error().decode()
    try:
        assert lib.rl_plan_workspace(plan) == 0
        _ok(lib, lib.rl_plan_autotune(plan, 1.0 if beta == 1.0 else 0.0, _s()))
        meta = json.loads(lib.rl_plan_tuning_metadata(plan))
        assert meta["enabled"] is True and len(meta["candidates"]) == 1
        assert lib.rl_plan_autotune(plan, 0.0, _s()) == -1  # once only
        Ad, Bd, Cd, bd = A.cuda(), B.cuda(), C.cuda(), bv.cuda()
        D = Cd if alias else torch.full((n, ldd), float("nan"), device="cuda")
        _ok(lib, lib.rl_plan_run(plan, Ad.data_ptr(), Bd.data_ptr(), Cd.data_ptr() if beta else None,
                                 D.data_ptr(), bd.data_ptr() if bias else None, None, 0, beta, _s()))
        # the same plan into another output (pointers are bound per launch)
        D2 = torch.full((n, ldd), float("nan"), device="cuda")
        _ok(lib, lib.rl_plan_run(plan, Ad.data_ptr(), Bd.data_ptr(), None, D2.data_ptr(),
                                 bd.data_ptr() if bias else None, None, 0, 0.0, _s()))
        torch.cuda.synchronize()
        _close(D[:, :m].T, ref)
        _close(D2[:, :m].T, prod)
        assert torch.isnan(D2[:, m:]).all()  # the rows between m and ldd are not written
    finally:
        assert lib.rl_plan_destroy(plan) == 0


def test_dense_plan_replays_in_a_cuda_graph(lib):
    g = _gen(4)
    m, n, k = 64, 256, 96
    plan = lib.rl_plan_create(m, n, k, 0, 0, m, k, m, 1, 0, 0)
    assert plan, lib.rl_last_error().decode()
    try:
        A = torch.randn(k, m, generator=g).cuda()  # column-major m x k
        B = torch.randn(n, k, generator=g).cuda()  # column-major k x n
        bias = torch.randn(m, generator=g).cuda()
        D = torch.empty(n, m, device="cuda")

        def run():
            _ok(lib, lib.rl_plan_run(plan, A.data_ptr(), B.data_ptr(), None, D.data_ptr(), bias.data_ptr(), None, 0,
                                     0.0, _s()))

        run()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            run()
        A.copy_(torch.randn(k, m, generator=g))
        graph.replay()
        torch.cuda.synchronize()
        _close(D.T, A.T.double() @ B.T.double() + bias.double()[:, None])
        del graph
    finally:
        lib.rl_plan_destroy(plan)


def test_cast_and_bias_gradient(lib):
    g = _gen(5)
    x = (torch.randn(1001, generator=g) * 3000).cuda()
    for src in (x, x[1:]):  # 16-byte aligned and merely 4-byte aligned sources
        out = torch.empty(src.numel(), dtype=torch.float16, device="cuda")
        _ok(lib, lib.rl_cast_f32_f16(src.data_ptr(), out.data_ptr(), src.numel(), _s()))
        torch.cuda.synchronize()
        assert torch.equal(out.view(torch.int16), src.half().view(torch.int16))
    dy = torch.randn(300, 101, generator=g).cuda()
    db = torch.randn(101, generator=g).cuda()
    ref = db.double() + dy.double().sum(0)
    _ok(lib, lib.rl_bias_grad(dy.data_ptr(), db.data_ptr(), 300, 101, _s()))
    torch.cuda.synchronize()
    _close(db, ref, 1e-5)


# ---------------------------------------------------------------------------- Adam


def test_adam_plan_matches_bias_corrected_formula(lib):
    g = _gen(7)
    shapes = [1, 4097, 10000]
    params = [torch.randn(s, generator=g).cuda() for s in shapes]
    grads = [torch.zeros(s, device="cuda") for s in shapes]
    m1 = [torch.zeros(s, device="cuda") for s in shapes]
    m2 = [torch.zeros(s, device="cuda") for s in shapes]
    ts = torch.zeros(1, device="cuda")
    lr = torch.tensor([1e-3], device="cuda")
    ref = [(p.double().cpu().numpy(), np.zeros(p.numel()), np.zeros(p.numel())) for p in params]
    plan = lib.rl_adam_create(3, pointers([t.data_ptr() for t in params]), pointers([t.data_ptr() for t in grads]),
                              pointers([t.data_ptr() for t in m1]), pointers([t.data_ptr() for t in m2]),
                              sizes(shapes), ts.data_ptr(), lr.data_ptr(), 0.9, 0.999, 1e-8)
    assert plan, lib.rl_last_error().decode()
    try:
        for step in range(1, 4):
            for t in grads:
                t.copy_(torch.randn(t.numel(), generator=g))
            ref = [O.adam_warp(p, gr.double().cpu().numpy(), a, b, step, 1e-3) for (p, a, b), gr in zip(ref, grads)]
            _ok(lib, lib.rl_adam_step(plan, _s()))
        torch.cuda.synchronize()
        assert ts.item() == 3.0
        for p, a, b, (rp, ra, rb) in zip(params, m1, m2, ref):
            _close(p, rp, 1e-5)
            _close(a, ra, 1e-5)
            _close(b, rb, 1e-5)
    finally:
        assert lib.rl_adam_destroy(plan) == 0


def test_adam_dynamic_loss_scaling_skips_and_grows(lib):
    g = _gen(8)
    n = 5000
    p = torch.randn(n, generator=g).cuda()
    grad = torch.zeros(n, device="cuda")
    m1, m2 = torch.zeros(n, device="cuda"), torch.zeros(n, device="cuda")
    ts, lr = torch.zeros(1, device="cuda"), torch.tensor([1e-2], device="cuda")
    scale = torch.tensor([1024.0], device="cuda")
    tracker, found, skipped_flag = (torch.zeros(1, dtype=torch.int32, device="cuda") for _ in range(3))
    attempted, skipped = torch.zeros(1, dtype=torch.int64, device="cuda"), torch.zeros(1, dtype=torch.int64, device="cuda")
    plan = lib.rl_adam_create(1, pointers([p.data_ptr()]), pointers([grad.data_ptr()]), pointers([m1.data_ptr()]),
                              pointers([m2.data_ptr()]), sizes([n]), ts.data_ptr(), lr.data_ptr(), 0.9, 0.999, 1e-8)
    assert plan
    try:
        _ok(lib, lib.rl_adam_set_scaler(plan, scale.data_ptr(), tracker.data_ptr(), found.data_ptr(),
                                        skipped_flag.data_ptr(), attempted.data_ptr(), skipped.data_ptr(), 2.0, 0.5, 2))
        rp, ra, rb = p.double().cpu().numpy(), np.zeros(n), np.zeros(n)
        step = 0
        expected_scale = [1024.0, 512.0, 512.0, 1024.0]
        for i in range(4):
            true_grad = torch.randn(n, generator=g)
            grad.copy_(true_grad * scale.item())
            if i == 1:
                grad[17] = float("inf")
            before = p.clone()
            _ok(lib, lib.rl_adam_unscale(plan, _s()))
            _ok(lib, lib.rl_adam_step(plan, _s()))
            torch.cuda.synchronize()
            if i == 1:
                assert found.item() == 1 and skipped_flag.item() == 1
                assert torch.equal(p, before)
            else:
                step += 1
                rp, ra, rb = O.adam_warp(rp, true_grad.double().numpy(), ra, rb, step, 1e-2)
                _close(p, rp, 1e-5)
            assert scale.item() == expected_scale[i]
        assert attempted.item() == 4 and skipped.item() == 1 and ts.item() == 3.0 and tracker.item() == 0
    finally:
        lib.rl_adam_destroy(plan)


# ---------------------------------------------------------------------------- projection, EMA, zero


def test_projection_plan(lib):
    g = _gen(9)
    rows = [torch.randn(7, generator=g).cuda(), torch.randn(512, generator=g).cuda() * 5]
    bn_w, bn_b = torch.randn(64, generator=g).cuda(), torch.randn(64, generator=g).cuda()
    rms = torch.randn(33, generator=g).cuda() * 0.1
    shadows = [torch.zeros(7, dtype=torch.float16, device="cuda"), torch.zeros(512, dtype=torch.float16, device="cuda")]
    before = [t.double().cpu() for t in (*rows, bn_w, bn_b, rms)]
    firsts = [rows[0], rows[1], bn_w, rms]
    seconds = [rows[0], rows[1], bn_b, rms]
    plan = lib.rl_flash_projection_create_with_shadows(
        4, pointers([t.data_ptr() for t in firsts]), pointers([t.data_ptr() for t in seconds]), sizes([7, 512, 64, 33]),
        ints([0, 0, 1, 2]), pointers([shadows[0].data_ptr(), shadows[1].data_ptr(), 0, 0]))
    assert plan, lib.rl_last_error().decode()
    try:
        _ok(lib, lib.rl_flash_projection_step(plan, _s()))
        torch.cuda.synchronize()
    finally:
        lib.rl_flash_projection_destroy(plan)
    r0, r1, w, b, q = before
    _close(rows[0], r0 / max(r0.norm().item(), 1e-8), 1e-6)
    _close(rows[1], r1 / max(r1.norm().item(), 1e-8), 1e-6)
    f = math.sqrt(64) / math.sqrt((w * w).sum().item() + (b * b).sum().item() + 1e-8)
    _close(bn_w, w * f, 1e-5)
    _close(bn_b, b * f, 1e-5)
    _close(rms, q * (math.sqrt(33) / math.sqrt((q * q).sum().item() + 1e-8)), 1e-5)
    for row, sh in zip(rows, shadows):
        assert torch.equal(sh.view(torch.int16), row.half().view(torch.int16))


def test_ema_and_zero_plans(lib):
    g = _gen(10)
    src = [torch.randn(5, generator=g).cuda(), torch.randn(20000, generator=g).cuda()]
    dst = [torch.randn(5, generator=g).cuda(), torch.randn(20000, generator=g).cuda()]
    shadow = torch.zeros(20000, dtype=torch.float16, device="cuda")
    ref = [(1 - 0.005) * d.double() + 0.005 * s.double() for s, d in zip(src, dst)]
    plan = lib.rl_flash_ema_create_with_shadows(2, pointers([t.data_ptr() for t in src]),
                                                pointers([t.data_ptr() for t in dst]), sizes([5, 20000]), 0.005,
                                                pointers([0, shadow.data_ptr()]))
    assert plan
    try:
        _ok(lib, lib.rl_flash_ema_step(plan, _s()))
        torch.cuda.synchronize()
    finally:
        lib.rl_flash_ema_destroy(plan)
    for d, r in zip(dst, ref):
        _close(d, r, 1e-6)
    assert torch.equal(shadow.view(torch.int16), dst[1].half().view(torch.int16))

    buf = torch.ones(50000, device="cuda")
    spans = [(1, 3), (10, 9000), (20000, 20001)]
    zplan = lib.rl_zero_create(3, pointers([buf[o:].data_ptr() for o, _ in spans]), sizes([n for _, n in spans]))
    assert zplan
    try:
        _ok(lib, lib.rl_zero_step(zplan, _s()))
        torch.cuda.synchronize()
    finally:
        lib.rl_zero_destroy(zplan)
    expect = torch.ones(50000)
    for o, n in spans:
        expect[o:o + n] = 0
    assert torch.equal(buf.cpu(), expect)


# ---------------------------------------------------------------------------- BN / RMS


def _bn_buffers(batch, channels):
    chunks = (batch + 255) // 256
    return torch.zeros(2 * chunks * channels, device="cuda"), torch.zeros(2 * channels, device="cuda")


def test_batch_norm_training_and_evaluation(lib):
    g = _gen(11)
    B, C, eps, mom = 700, 45, 1e-5, 0.01
    x = (3.0 + 2.0 * torch.randn(B, C, generator=g)).cuda()
    w, b = torch.randn(C, generator=g).cuda(), torch.randn(C, generator=g).cuda()
    rm, rv = torch.full((C,), 0.1, device="cuda"), torch.full((C,), 1.5, device="cuda")
    mean, var = torch.zeros(C, device="cuda"), torch.zeros(C, device="cuda")
    partial, sums = _bn_buffers(B, C)
    y = torch.empty(B, C, device="cuda")
    y16 = torch.empty(B, C, dtype=torch.float16, device="cuda")
    xn, wn, bn_ = (t.double().cpu().numpy() for t in (x, w, b))
    yr, cache, nrm, nrv = O.bn_forward(xn[None], wn[None], bn_[None], np.full((1, C), 0.1), np.full((1, C), 1.5), True,
                                       eps=eps, momentum=mom)
    pre = yr[0]
    yr = np.maximum(pre, 0.0)
    _ok(lib, lib.rl_flash_bn_forward_with_fp16(x.data_ptr(), w.data_ptr(), b.data_ptr(), rm.data_ptr(), rv.data_ptr(),
                                               mean.data_ptr(), var.data_ptr(), partial.data_ptr(), y.data_ptr(),
                                               y16.data_ptr(), B, C, eps, mom, 1, 1, _s()))
    torch.cuda.synchronize()
    _close(y, yr)
    _close(mean, xn.mean(0), 1e-5)
    _close(var, xn.var(0), 1e-5)
    _close(rm, nrm[0], 1e-5)
    _close(rv, nrv[0], 1e-5)
    assert torch.equal(y16.view(torch.int16), y.half().view(torch.int16))

    dy = torch.randn(B, C, generator=g).cuda()
    dx = torch.randn(B, C, generator=g).cuda()
    dw, db = torch.randn(C, generator=g).cuda(), torch.randn(C, generator=g).cuda()
    gmask = dy.double().cpu().numpy() * (y.double().cpu().numpy() > 0)
    dxr, dwr, dbr = O.bn_backward(gmask[None], cache)
    exp_dx, exp_dw, exp_db = (t.double().cpu() + torch.from_numpy(r[0]) for t, r in ((dx, dxr), (dw, dwr), (db, dbr)))
    _ok(lib, lib.rl_flash_bn_backward(x.data_ptr(), dy.data_ptr(), y.data_ptr(), w.data_ptr(), mean.data_ptr(),
                                      var.data_ptr(), partial.data_ptr(), sums.data_ptr(), dx.data_ptr(), dw.data_ptr(),
                                      db.data_ptr(), B, C, eps, 1, 1, _s()))
    torch.cuda.synchronize()
    _close(dx, exp_dx)
    _close(dw, exp_dw)
    _close(db, exp_db)

    # evaluation mode: running statistics, no ReLU; controlled backward overwrites dx
    ye = torch.empty(B, C, device="cuda")
    _ok(lib, lib.rl_flash_bn_forward(x.data_ptr(), w.data_ptr(), b.data_ptr(), rm.data_ptr(), rv.data_ptr(),
                                     mean.data_ptr(), var.data_ptr(), partial.data_ptr(), ye.data_ptr(), B, C, eps, mom,
                                     0, 0, _s()))
    rmn, rvn = rm.double().cpu().numpy(), rv.double().cpu().numpy()
    yer, ecache, _, _ = O.bn_forward(xn[None], wn[None], bn_[None], rmn[None], rvn[None], False, eps=eps)
    dxe = torch.full((B, C), 7.0, device="cuda")
    dxe16 = torch.empty(B, C, dtype=torch.float16, device="cuda")
    _ok(lib, lib.rl_flash_bn_backward_controlled(x.data_ptr(), dy.data_ptr(), ye.data_ptr(), w.data_ptr(),
                                                 rm.data_ptr(), rv.data_ptr(), partial.data_ptr(), sums.data_ptr(),
                                                 dxe.data_ptr(), None, None, dxe16.data_ptr(), 1, B, C, eps, 0, 0, _s()))
    torch.cuda.synchronize()
    _close(ye, yer[0])
    dxer, _, _ = O.bn_backward(dy.double().cpu().numpy()[None], ecache)
    _close(dxe, dxer[0])
    assert torch.equal(dxe16.view(torch.int16), dxe.half().view(torch.int16))


def test_rms_norm(lib):
    g = _gen(12)
    B, C, eps = 300, 77, 1e-6
    x = torch.randn(B, C, generator=g).cuda()
    w = torch.randn(C, generator=g).cuda()
    var, y = torch.empty(B, device="cuda"), torch.empty(B, C, device="cuda")
    _ok(lib, lib.rl_flash_rms_forward(x.data_ptr(), w.data_ptr(), var.data_ptr(), y.data_ptr(), B, C, eps, _s()))
    xn, wn = x.double().cpu().numpy(), w.double().cpu().numpy()
    yr, cache = O.rms_forward(xn[None], wn[None], eps=eps)
    dy = torch.randn(B, C, generator=g).cuda()
    dx, dw = torch.randn(B, C, generator=g).cuda(), torch.randn(C, generator=g).cuda()
    partial = torch.zeros(((B + 255) // 256) * C, device="cuda")
    dxr, dwr = O.rms_backward(dy.double().cpu().numpy()[None], cache)
    exp_dx, exp_dw = dx.double().cpu() + torch.from_numpy(dxr[0]), dw.double().cpu() + torch.from_numpy(dwr[0])
    _ok(lib, lib.rl_flash_rms_backward(x.data_ptr(), dy.data_ptr(), w.data_ptr(), var.data_ptr(), partial.data_ptr(),
                                       dx.data_ptr(), dw.data_ptr(), B, C, eps, _s()))
    torch.cuda.synchronize()
    _close(y, yr[0])
    _close(var, (xn * xn).mean(1), 1e-5)
    _close(dx, exp_dx)
    _close(dw, exp_dw)


# ---------------------------------------------------------------------------- categorical


def test_categorical_forward_backward(lib):
    g = _gen(13)
    B, K = 50, 101
    raw = torch.randn(B, K, generator=g).cuda()
    bias = torch.randn(K, generator=g).cuda()
    support = torch.linspace(-10, 10, K).cuda()
    lp, q = torch.empty(B, K, device="cuda"), torch.empty(B, device="cuda")
    _ok(lib, lib.rl_flash_categorical_forward(raw.data_ptr(), bias.data_ptr(), support.data_ptr(), lp.data_ptr(),
                                              q.data_ptr(), B, K, _s()))
    r = raw.double().cpu().requires_grad_(True)
    bb = bias.double().cpu()
    ref_lp = torch.log_softmax(r + bb, dim=-1)
    ref_q = (ref_lp.exp() * support.double().cpu()).sum(-1)
    dlp, dq = torch.randn(B, K, generator=g), torch.randn(B, generator=g)
    ((ref_lp * dlp.double()).sum() + (ref_q * dq.double()).sum()).backward()
    draw = torch.randn(B, K, generator=g).cuda()
    dbias = torch.randn(K, generator=g).cuda()
    scratch = torch.empty(B, K, device="cuda")
    exp_draw, exp_db = draw.double().cpu() + r.grad, dbias.double().cpu() + r.grad.sum(0)
    dlpd, dqd = dlp.cuda(), dq.cuda()
    _ok(lib, lib.rl_flash_categorical_backward(lp.data_ptr(), support.data_ptr(), dlpd.data_ptr(), dqd.data_ptr(),
                                               scratch.data_ptr(), draw.data_ptr(), dbias.data_ptr(), B, K, _s()))
    torch.cuda.synchronize()
    _close(lp, ref_lp.detach(), 1e-5)
    _close(q, ref_q.detach(), 1e-5)
    _close(draw, exp_draw)
    _close(dbias, exp_db)
    # value gradient alone, into the bias only
    r2 = raw.double().cpu().requires_grad_(True)
    q2 = (torch.log_softmax(r2 + bb, dim=-1).exp() * support.double().cpu()).sum(-1)
    (q2 * dq.double()).sum().backward()
    db2 = torch.zeros(K, device="cuda")
    _ok(lib, lib.rl_flash_categorical_backward(lp.data_ptr(), support.data_ptr(), None, dqd.data_ptr(),
                                               scratch.data_ptr(), None, db2.data_ptr(), B, K, _s()))
    torch.cuda.synchronize()
    _close(db2, r2.grad.sum(0))


@pytest.mark.parametrize("batch,bins", [(64, 101), (37, 11)])
def test_categorical_target_projection(lib, batch, bins):
    rng = np.random.default_rng(batch * bins)
    min_v, max_v = -10.0, 10.0
    q = rng.standard_normal((2, 2 * batch)).astype(np.float32)
    q[1, batch + 3] = q[0, batch + 3]  # a tie picks twin 0
    logits = rng.standard_normal((2, 2 * batch, bins))
    lp = (logits - np.log(np.exp(logits).sum(-1, keepdims=True))).astype(np.float32)
    reward = (rng.standard_normal(batch) * 3).astype(np.float32)
    term = (rng.random(batch) < 0.2).astype(np.float32)
    disc = np.full(batch, 0.99, np.float32)
    nlp = rng.standard_normal(batch).astype(np.float32)
    alpha = np.array([0.2], np.float32)
    dev = [torch.from_numpy(a).cuda() for a in (q, lp, reward, term, disc, nlp, alpha)]
    target = torch.full((batch, bins), float("nan"), device="cuda")
    max_ent = torch.tensor([-1e30], device="cuda")
    _ok(lib, lib.rl_flash_categorical_target(*[t.data_ptr() for t in dev], target.data_ptr(), max_ent.data_ptr(),
                                             batch, bins, min_v, max_v, _s()))
    torch.cuda.synchronize()
    twin = (q[1, batch:] < q[0, batch:]).astype(np.int64)
    sel = lp[twin, batch + np.arange(batch)]
    ent = alpha[0] * nlp
    ref, _ = O.categorical_target(sel, reward, term, ent, disc, bins, min_v, max_v)
    _close(target, ref, 1e-5)
    np.testing.assert_allclose(target.sum(-1).cpu().numpy(), np.exp(sel.astype(np.float64)).sum(-1), rtol=1e-5)
    assert max_ent.item() == float(ent.max())


def test_entry_points_are_deterministic_and_capture_equals_eager(lib):
    """Every family run twice on the same inputs gives bitwise equal results (fixed-order sums,
    no scheduling-dependent atomics), and a CUDA-graph replay of a dense plan equals the eager
    call bitwise (the reference's diagnostics hold capture to eager within 2e-6,
    examples/diagnose_cuda_flashsac.py:250-256)."""
    g = _gen(21)
    B, C, K = 1000, 96, 101
    x = (1.0 + torch.randn(B, C, generator=g)).cuda()
    w, b = torch.randn(C, generator=g).cuda(), torch.randn(C, generator=g).cuda()
    dy = torch.randn(B, C, generator=g).cuda()
    q = torch.randn(2, 2 * B, generator=g).cuda()
    lp = torch.log_softmax(torch.randn(2, 2 * B, K, generator=g), -1).cuda()
    rew, term = torch.randn(B, generator=g).cuda(), (torch.rand(B, generator=g) < 0.1).float().cuda()
    disc, nlp, alpha = torch.full((B,), 0.99, device="cuda"), torch.randn(B, generator=g).cuda(), torch.tensor([0.1], device="cuda")
    support = torch.linspace(-10, 10, K).cuda()
    A = torch.randn(300, 256, generator=g).half().cuda()  # column-major 256 x 300 (lda 256)
    Bm = torch.randn(512, 300, generator=g).half().cuda()  # column-major 300 x 512 (ldb 300, staged)

    def run():
        chunks = (B + 255) // 256
        mean, var = torch.zeros(C, device="cuda"), torch.zeros(C, device="cuda")
        rm, rv = torch.zeros(C, device="cuda"), torch.ones(C, device="cuda")
        partial, sums = torch.zeros(2 * chunks * C, device="cuda"), torch.zeros(2 * C, device="cuda")
        y = torch.empty_like(x)
        _ok(lib, lib.rl_flash_bn_forward(x.data_ptr(), w.data_ptr(), b.data_ptr(), rm.data_ptr(), rv.data_ptr(),
                                         mean.data_ptr(), var.data_ptr(), partial.data_ptr(), y.data_ptr(), B, C,
                                         1e-5, 0.01, 1, 1, _s()))
        dx, dw, db = torch.zeros_like(x), torch.zeros(C, device="cuda"), torch.zeros(C, device="cuda")
        _ok(lib, lib.rl_flash_bn_backward(x.data_ptr(), dy.data_ptr(), y.data_ptr(), w.data_ptr(), mean.data_ptr(),
                                          var.data_ptr(), partial.data_ptr(), sums.data_ptr(), dx.data_ptr(),
                                          dw.data_ptr(), db.data_ptr(), B, C, 1e-5, 1, 1, _s()))
        tgt, ment = torch.empty(B, K, device="cuda"), torch.tensor([-1e30], device="cuda")
        _ok(lib, lib.rl_flash_categorical_target(q.data_ptr(), lp.data_ptr(), rew.data_ptr(), term.data_ptr(),
                                                 disc.data_ptr(), nlp.data_ptr(), alpha.data_ptr(), tgt.data_ptr(),
                                                 ment.data_ptr(), B, K, -10.0, 10.0, _s()))
        logp, val = torch.empty(B, K, device="cuda"), torch.empty(B, device="cuda")
        _ok(lib, lib.rl_flash_categorical_forward(tgt.data_ptr(), support.data_ptr(), support.data_ptr(),
                                                  logp.data_ptr(), val.data_ptr(), B, K, _s()))
        draw, dcb, scratch = torch.zeros(B, K, device="cuda"), torch.zeros(K, device="cuda"), torch.empty(B, K, device="cuda")
        _ok(lib, lib.rl_flash_categorical_backward(logp.data_ptr(), support.data_ptr(), tgt.data_ptr(),
                                                   val.data_ptr(), scratch.data_ptr(), draw.data_ptr(),
                                                   dcb.data_ptr(), B, K, _s()))
        torch.cuda.synchronize()
        return [y, mean, var, dx, dw, db, tgt, ment, logp, val, draw, dcb]

    first, second = run(), run()
    for t1, t2 in zip(first, second):
        assert torch.equal(t1, t2)

    plans = [lib.rl_plan_create_mixed(256, 512, 300, 0, 0, 256, 300, 256, 0, 0, 1, 0),  # fp16 staged (ldb 300)
             lib.rl_plan_create_mixed(256, 512, 296, 0, 1, 256, 512, 256, 0, 0, 1, 0)]  # fp16 in place
    try:
        assert all(plans), lib.rl_last_error().decode()
        Bt = torch.randn(296, 512, generator=g).half().cuda()  # column-major 512 x 296 (ldb 512)
        operands = [(A, Bm), (A, Bt)]
        for plan, (a, bb) in zip(plans, operands):
            eager, replay = torch.empty(512, 256, device="cuda"), torch.empty(512, 256, device="cuda")
            _ok(lib, lib.rl_plan_run(plan, a.data_ptr(), bb.data_ptr(), None, eager.data_ptr(), None, None, 0, 0.0,
                                     _s()))
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                _ok(lib, lib.rl_plan_run(plan, a.data_ptr(), bb.data_ptr(), None, replay.data_ptr(), None, None, 0,
                                         0.0, _s()))
            graph.replay()
            torch.cuda.synchronize()
            assert torch.equal(eager, replay)
            del graph
    finally:
        for plan in plans:
            lib.rl_plan_destroy(plan)
