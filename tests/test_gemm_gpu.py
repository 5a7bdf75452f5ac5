"""tcgen05 GEMM numerics against torch fp32/fp64 references of the same product.

Covers both operand kinds (fp16, tf32x3 split), all four operand-major
combinations, ragged M/N/K tails, twin batching, shared operands, the fused
epilogue (bias, residual, accumulate, scale, 32-row column moments) and split-K.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu

from robolearn_b200 import dense  # noqa: E402


def _store(logical: torch.Tensor, major: int, kind: int) -> tuple[torch.Tensor, int]:
    """Lay out logical [batch, rows, k] as K-contiguous (major 0) or rows-contiguous (major 1)."""
    bsz, rows, k = logical.shape
    src = logical if major == 0 else logical.transpose(1, 2)
    inner = k if major == 0 else rows
    ld = dense.operand_ld(inner, kind)
    buf = torch.zeros(bsz, src.shape[1], ld, device="cuda", dtype=torch.float16 if kind == 0 else torch.float32)
    buf[:, :, :inner] = src.to(buf.dtype)
    return buf, ld


def _run(kind, m, n, k, a_major, b_major, batch=2, shared_a=False, ldd=None, d_rows=None, **epi):
    g = torch.Generator(device="cuda").manual_seed(m * 131 + n * 7 + k)
    A = torch.randn(1 if shared_a else batch, m, k, device="cuda", generator=g)
    B = torch.randn(batch, n, k, device="cuda", generator=g) / k**0.5
    if kind == 0:
        A, B = A.half().float(), B.half().float()
    a_st, lda = _store(A, a_major, kind)
    b_st, ldb = _store(B, b_major, kind)
    ldd = ldd or n + 3
    D = torch.zeros(batch, d_rows or m, ldd, device="cuda")
    if isinstance(epi.get("residual"), str):  # "D": the residual is the output itself
        epi["residual"] = D
    kw = {}
    if kind == 1:
        a_hi, a_lo = dense.tf32_split(a_st)
        b_hi, b_lo = dense.tf32_split(b_st)
        a_st, b_st = a_hi, b_hi
        kw = dict(a_lo=a_lo, b_lo=b_lo)
    ref = torch.einsum("zmk,znk->zmn", A.double().expand(batch, m, k), B.double())
    plan = dense.DensePlan(
        kind=kind, m=m, n=n, k=k, a=a_st, b=b_st, d=D, lda=lda, ldb=ldb, ldd=ldd, a_major=a_major,
        b_major=b_major, batch=batch, a_batch_stride=0 if shared_a else a_st[0].numel(),
        b_batch_stride=b_st[0].numel(), d_batch_stride=D[0].numel(), **kw, **epi,
    )
    return plan, D, ref


@pytest.mark.parametrize("kind", [0, 1])
@pytest.mark.parametrize("a_major,b_major", [(0, 0), (0, 1), (1, 0), (1, 1)])
@pytest.mark.parametrize("m,n,k", [(128, 128, 64), (300, 200, 160), (257, 101, 123), (64, 512, 520)])
def test_gemm_matches_reference(kind, a_major, b_major, m, n, k):
    plan, D, ref = _run(kind, m, n, k, a_major, b_major)
    plan.run()
    torch.cuda.synchronize()
    out = D[:, :, :n].double()
    tol = 2e-3 if kind == 0 else 2e-5
    err = (out - ref).abs().max().item() / ref.abs().max().item()
    assert err < tol, (err, plan.tile_n)


def test_gemm_epilogue_bias_residual_accumulate_scale_and_shared_operand():
    m, n, k, batch = 200, 96, 64, 2
    bias = torch.randn(batch, n, device="cuda")
    res = torch.randn(batch, m, n, device="cuda")
    scale = torch.tensor([0.25], device="cuda")
    plan, D, ref = _run(0, m, n, k, 0, 0, batch=batch, shared_a=True, bias=bias, bias_batch_stride=n,
                        residual=res, ldr=n, residual_batch_stride=m * n, scale=scale, accumulate=True)
    D.fill_(1.5)
    plan.run()
    torch.cuda.synchronize()
    expect = 0.25 * ref + bias.double()[:, None, :] + res.double() + 1.5
    assert (D[:, :, :n].double() - expect).abs().max().item() < 2e-3 * expect.abs().max().item()


@pytest.mark.parametrize("kind", [0, 1])
def test_gemm_column_moments(kind):
    m, n, k, batch = 300, 80, 96, 2
    groups = (m + 31) // 32
    mean = torch.zeros(batch, groups, n, device="cuda")
    m2 = torch.zeros(batch, groups, n, device="cuda")
    plan, D, ref = _run(kind, m, n, k, 0, 0, batch=batch, stat_mean=mean, stat_m2=m2, stat_batch_stride=groups * n)
    plan.run()
    torch.cuda.synchronize()
    out = D[:, :, :n].double()
    for gidx in range(groups):
        rows = out[:, gidx * 32:(gidx + 1) * 32]
        mu = rows.mean(1)
        assert torch.allclose(mean[:, gidx].double(), mu, atol=1e-4, rtol=1e-4)
        assert torch.allclose(m2[:, gidx].double(), ((rows - mu[:, None]) ** 2).sum(1), atol=1e-3, rtol=1e-4)


@pytest.mark.parametrize("kind", [0, 1])
def test_gemm_split_k_partials_reduce(kind):
    m, n, k, batch, splits = 256, 128, 1024, 2, 4
    stride = batch * m * (n + 3)
    part = torch.zeros(splits, stride, device="cuda")
    g = torch.Generator(device="cuda").manual_seed(5)
    A = torch.randn(batch, m, k, device="cuda", generator=g)
    B = torch.randn(batch, n, k, device="cuda", generator=g) / k**0.5
    if kind == 0:
        A, B = A.half().float(), B.half().float()
    a_st, lda = _store(A, 1, kind)
    b_st, ldb = _store(B, 1, kind)
    kw = {}
    if kind == 1:
        a_st, a_lo = dense.tf32_split(a_st)
        b_st, b_lo = dense.tf32_split(b_st)
        kw = dict(a_lo=a_lo, b_lo=b_lo)
    plan = dense.DensePlan(kind=kind, m=m, n=n, k=k, a=a_st, b=b_st, d=part, lda=lda, ldb=ldb, ldd=n + 3,
                           a_major=1, b_major=1, batch=batch, a_batch_stride=a_st[0].numel(),
                           b_batch_stride=b_st[0].numel(), d_batch_stride=m * (n + 3), k_splits=splits,
                           d_split_stride=stride, **kw)
    out = torch.zeros(stride, device="cuda")
    plan.run()
    dense.split_reduce(part, stride, splits, out, stride)
    torch.cuda.synchronize()
    got = out.view(batch, m, n + 3)[:, :, :n].double()
    ref = torch.einsum("zmk,znk->zmn", A.double(), B.double())
    tol = 2e-3 if kind == 0 else 2e-5
    assert (got - ref).abs().max().item() < tol * ref.abs().max().item()


def test_gemm_rejects_misaligned_stride():
    a = torch.zeros(16, 10, device="cuda", dtype=torch.float16)
    b = torch.zeros(16, 16, device="cuda", dtype=torch.float16)
    d = torch.zeros(16, 16, device="cuda")
    with pytest.raises(RuntimeError, match="16 bytes"):
        dense.DensePlan(kind=0, m=16, n=16, k=10, a=a, b=b, d=d, lda=10, ldb=16, ldd=16)


@pytest.mark.parametrize("kind,tile_n", [(0, 0), (0, 48), (1, 0)])
def test_gemm_multi_wave_epilogue_moments_and_plane(kind, tile_n):
    """More CTAs than SMs (two co-resident CTAs per SM for fp16 tiles), ragged M and N,
    bias + residual, 32-row column moments and an operand-plane copy of the output."""
    from robolearn_b200 import _native as N

    m, n, k, batch = 8200, 600, 256, 2
    groups = (m + 31) // 32
    bias = torch.randn(batch, n, device="cuda")
    res = torch.randn(batch, m, n, device="cuda")
    mean = torch.zeros(batch, groups, n, device="cuda")
    m2 = torch.zeros(batch, groups, n, device="cuda")
    pld = dense.operand_ld(n, kind)
    if kind == 0:
        h16 = torch.zeros(batch, m, pld, device="cuda", dtype=torch.float16)
        plane = N.Plane(h16=h16.data_ptr(), ld=pld, twin_stride=m * pld)
        keep = [h16]
    else:
        hi = torch.zeros(batch, m, pld, device="cuda")
        lo = torch.zeros(batch, m, pld, device="cuda")
        plane = N.Plane(hi=hi.data_ptr(), lo=lo.data_ptr(), ld=pld, twin_stride=m * pld)
        keep = [hi, lo]
    plan, D, ref = _run(kind, m, n, k, 0, 0, batch=batch, bias=bias, bias_batch_stride=n, residual=res, ldr=n,
                        residual_batch_stride=m * n, stat_mean=mean, stat_m2=m2, stat_batch_stride=groups * n,
                        out_plane=plane, tile_n=tile_n)
    plan.run()
    torch.cuda.synchronize()
    expect = ref + bias.double()[:, None, :] + res.double()
    out = D[:, :, :n].double()
    tol = 2e-3 if kind == 0 else 2e-5
    assert (out - expect).abs().max().item() < tol * expect.abs().max().item()
    if kind == 0:
        assert torch.equal(keep[0][:, :, :n], D[:, :, :n].half())
    else:
        hi_ref = (D[:, :, :n].view(torch.int32) & -8192).view(torch.float32)
        assert torch.equal(keep[0][:, :, :n], hi_ref)
        assert torch.equal(keep[1][:, :, :n], D[:, :, :n] - hi_ref)
    full = torch.zeros(batch, groups * 32, n, device="cuda", dtype=torch.float64)
    full[:, :m] = out
    rows = full.view(batch, groups, 32, n)
    counts = torch.full((groups,), 32.0, device="cuda", dtype=torch.float64)
    counts[-1] = m - 32 * (groups - 1)
    mu = rows.sum(2) / counts[None, :, None]
    valid = (torch.arange(groups * 32, device="cuda") < m).view(groups, 32)[None, :, :, None]
    dev = torch.where(valid, rows - mu[:, :, None, :], torch.zeros_like(rows))
    assert torch.allclose(mean.double(), mu, atol=1e-4, rtol=1e-4)
    assert torch.allclose(m2.double(), (dev**2).sum(2), atol=1e-3, rtol=1e-4)
    del keep


@pytest.mark.parametrize("kind", [0, 1])
@pytest.mark.parametrize("activation", [dense.ELU, dense.TANH])
@pytest.mark.parametrize("m,n", [(300, 200), (4096, 512)])
def test_gemm_activation_forward_and_derivative(kind, activation, m, n):
    """out = f(A B^T + bias) and, with act_aux = y, out = (A B^T + bias) * f'(y)."""
    k, batch = 96, 2
    bias = torch.randn(batch, n, device="cuda")
    plan, D, ref = _run(kind, m, n, k, 0, 0, batch=batch, bias=bias, bias_batch_stride=n, activation=activation)
    plan.run()
    torch.cuda.synchronize()
    pre = ref + bias.double()[:, None, :]
    f = (lambda x: torch.where(x > 0, x, torch.expm1(x))) if activation == dense.ELU else torch.tanh
    expect = f(pre)
    tol = 2e-3 if kind == 0 else 2e-5
    assert (D[:, :, :n].double() - expect).abs().max().item() < tol * max(expect.abs().max().item(), 1.0)
    # derivative mode: y = stored outputs (any values in f's range), out = x * f'(y)
    y = f(torch.randn(batch, m, n, device="cuda"))
    plan2, D2, ref2 = _run(kind, m, n, k, 0, 0, batch=batch, bias=bias, bias_batch_stride=n, activation=activation,
                           act_aux=y, ld_aux=n, aux_batch_stride=m * n)
    plan2.run()
    torch.cuda.synchronize()
    yd = y.double()
    grad = torch.where(yd > 0, torch.ones_like(yd), yd + 1) if activation == dense.ELU else 1 - yd * yd
    expect2 = (ref2 + bias.double()[:, None, :]) * grad
    assert (D2[:, :, :n].double() - expect2).abs().max().item() < tol * max(expect2.abs().max().item(), 1.0)


@pytest.mark.parametrize("kind", [0, 1])
def test_gemm_column_sums_mode(kind):
    """stat_m2 == null: per-32-row-group column sums (bias gradients of the PPO layers)."""
    m, n, k, batch = 4100, 200, 64, 2
    groups = (m + 31) // 32
    sums = torch.zeros(batch, groups, n, device="cuda")
    plan, D, ref = _run(kind, m, n, k, 0, 0, batch=batch, stat_mean=sums, stat_batch_stride=groups * n)
    plan.run()
    torch.cuda.synchronize()
    full = torch.zeros(batch, groups * 32, n, device="cuda", dtype=torch.float64)
    full[:, :m] = D[:, :, :n].double()
    expect = full.view(batch, groups, 32, n).sum(2)
    assert torch.allclose(sums.double(), expect, atol=1e-3, rtol=1e-4)


@pytest.mark.parametrize("kind", [0, 1])
@pytest.mark.parametrize("m,n,k,tile_n", [(300, 200, 96, 0), (8200, 600, 256, 0), (4096, 2048, 512, 0),
                                          (1000, 72, 64, 48)])
@pytest.mark.parametrize("mode", ["moments", "sums", "plane"])
def test_gemm_tma_store_epilogue(kind, m, n, k, tile_n, mode):
    """Store-engine epilogue (outputs written by TMA stores; with column statistics and
    n >= 128 the accumulator is kept transposed): output, bias, scale, 32-row column
    moments or sums and the fp16 plane against fp64 references; rows past M and columns
    past N (up to the row stride) stay untouched."""
    from robolearn_b200 import _native as N

    batch = 2
    groups = (m + 31) // 32
    ldd = (n + 3) // 4 * 4 + 4
    extra = 40  # rows after each twin's M rows that must stay untouched
    bias = torch.randn(batch, n, device="cuda")
    scale = torch.tensor([0.5], device="cuda")
    epi = dict(bias=bias, bias_batch_stride=n, scale=scale)
    mean = torch.zeros(batch, groups, n, device="cuda")
    m2 = torch.zeros(batch, groups, n, device="cuda")
    keep = []
    if mode == "moments":
        epi.update(stat_mean=mean, stat_m2=m2, stat_batch_stride=groups * n)
    elif mode == "sums":
        epi.update(stat_mean=mean, stat_batch_stride=groups * n)
    elif kind == 0:
        pld = dense.operand_ld(n, 0)
        h16 = torch.full((batch, m + extra, pld), 7.0, device="cuda", dtype=torch.float16)
        pscale = torch.tensor([4.0], device="cuda")
        found = torch.zeros(1, dtype=torch.int32, device="cuda")
        epi["out_plane"] = N.Plane(h16=h16.data_ptr(), ld=pld, twin_stride=(m + extra) * pld,
                                   scale=pscale.data_ptr(), found_inf=found.data_ptr())
        epi.update(stat_mean=mean, stat_m2=m2, stat_batch_stride=groups * n)
        keep = [h16, pscale, found]
    else:
        pytest.skip("tf32 output planes take the register-store epilogue")
    plan, D, ref = _run(kind, m, n, k, 0, 0, batch=batch, ldd=ldd, d_rows=m + extra, tile_n=tile_n, **epi)
    assert plan.transposed if n >= 128 and tile_n == 0 else plan.tma_store
    D.fill_(float("nan"))
    plan.run()
    torch.cuda.synchronize()
    expect = ref * 0.5 + bias.double()[:, None, :]
    out = D[:, :m, :n].double()
    tol = 2e-3 if kind == 0 else 2e-5
    assert (out - expect).abs().max().item() < tol * expect.abs().max().item()
    assert torch.isnan(D[:, :m, n:]).all() and torch.isnan(D[:, m:]).all()
    full = torch.zeros(batch, groups * 32, n, device="cuda", dtype=torch.float64)
    full[:, :m] = out
    rows = full.view(batch, groups, 32, n)
    counts = torch.full((groups,), 32.0, device="cuda", dtype=torch.float64)
    counts[-1] = m - 32 * (groups - 1)
    if mode == "sums":
        assert torch.allclose(mean.double(), rows.sum(2), atol=1e-3, rtol=1e-4)
    else:
        mu = rows.sum(2) / counts[None, :, None]
        valid = (torch.arange(groups * 32, device="cuda") < m).view(groups, 32)[None, :, :, None]
        dev = torch.where(valid, rows - mu[:, :, None, :], torch.zeros_like(rows))
        assert torch.allclose(mean.double(), mu, atol=1e-4, rtol=1e-4)
        assert torch.allclose(m2.double(), (dev**2).sum(2), atol=1e-3, rtol=1e-4)
    if mode == "plane":
        h16, _, found = keep
        assert torch.equal(h16[:, :m, :n], (D[:, :m, :n] * 4.0).half())
        assert (h16[:, m:] == 7.0).all() and (h16[:, :m, n:] == 7.0).all()
        assert int(found.item()) == 0


@pytest.mark.parametrize("tile_n", [0, 64])
def test_gemm_plane_overflow_flag(tile_n):
    """fp16 plane through the transposed epilogue (plan-chosen tile) and the store engine
    (explicit tile width): a loss scale that overflows fp16 sets found_inf."""
    from robolearn_b200 import _native as N

    m, n, k, batch = 256, 128, 64, 2
    pld = dense.operand_ld(n, 0)
    h16 = torch.zeros(batch, m, pld, device="cuda", dtype=torch.float16)
    pscale = torch.tensor([1e6], device="cuda")
    found = torch.zeros(1, dtype=torch.int32, device="cuda")
    plane = N.Plane(h16=h16.data_ptr(), ld=pld, twin_stride=m * pld, scale=pscale.data_ptr(),
                    found_inf=found.data_ptr())
    plan, D, _ = _run(0, m, n, k, 0, 0, batch=batch, ldd=n, out_plane=plane, tile_n=tile_n)
    assert plan.transposed if tile_n == 0 else plan.tma_store
    plan.run()
    torch.cuda.synchronize()
    assert int(found.item()) == 1


@pytest.mark.parametrize("kind", [0, 1])
@pytest.mark.parametrize("how,plane,tile_n,path", [
    ("residual_in_place", False, 0, "tma"),  # D += result as TMA reduce-add stores
    ("accumulate", False, 0, "tma"),
    ("residual_in_place", True, 0, "transposed"),  # the plane needs the final values
    ("residual_in_place", True, 64, "registers"),
    ("residual", True, 0, "transposed"),  # a separate residual array, rows loaded per lane
])
def test_gemm_residual_and_accumulate_paths(kind, how, plane, tile_n, path):
    """D = scale * A B^T + bias + residual (the residual being D itself or another array), or
    D += ... (accumulate), through each epilogue form; ragged M / N tails; rows past M and
    columns past N untouched; the operand plane equals the output."""
    from robolearn_b200 import _native as N

    m, n, k, batch = 1000, 600, 192, 2
    ldd = (n + 3) // 4 * 4 + 4
    bias = torch.randn(batch, n, device="cuda")
    scale = torch.tensor([0.25], device="cuda")
    old = torch.randn(batch, m + 8, ldd, device="cuda")
    res = torch.randn(batch, m, n, device="cuda")
    epi = dict(bias=bias, bias_batch_stride=n, scale=scale, tile_n=tile_n)
    keep = []
    if plane:
        pld = dense.operand_ld(n, kind)
        if kind == 0:
            h16 = torch.zeros(batch, m, pld, device="cuda", dtype=torch.float16)
            epi["out_plane"] = N.Plane(h16=h16.data_ptr(), ld=pld, twin_stride=m * pld)
            keep = [h16]
        else:
            hi = torch.zeros(batch, m, pld, device="cuda")
            lo = torch.zeros(batch, m, pld, device="cuda")
            epi["out_plane"] = N.Plane(hi=hi.data_ptr(), lo=lo.data_ptr(), ld=pld, twin_stride=m * pld)
            keep = [hi, lo]
    if how == "accumulate":
        epi["accumulate"] = 1
    elif how == "residual_in_place":
        epi.update(residual="D", ldr=ldd, residual_batch_stride=(m + 8) * ldd)
    else:
        epi.update(residual=res, ldr=n, residual_batch_stride=m * n)
    plan, D, ref = _run(kind, m, n, k, 0, 0, batch=batch, ldd=ldd, d_rows=m + 8, **epi)
    assert (plan.transposed, plan.tma_store) == (path == "transposed", path == "tma")
    D.copy_(old)
    plan.run()
    torch.cuda.synchronize()
    add = res.double() if how == "residual" else old[:, :m, :n].double()
    expect = ref * 0.25 + bias.double()[:, None, :] + add
    tol = 2e-3 if kind == 0 else 2e-5
    out = D[:, :m, :n]
    assert (out.double() - expect).abs().max().item() < tol * expect.abs().max().item()
    assert torch.equal(D[:, :m, n:], old[:, :m, n:]) and torch.equal(D[:, m:], old[:, m:])
    if plane and kind == 0:
        assert torch.equal(keep[0][:, :, :n], out.half())
    elif plane:
        hi_ref = (out.contiguous().view(torch.int32) & -8192).view(torch.float32)
        assert torch.equal(keep[0][:, :, :n], hi_ref) and torch.equal(keep[1][:, :, :n], out - hi_ref)


def test_tf32_operands_read_raw_fp32_as_hi():
    """kind::tf32 products ignore the low 13 mantissa bits: raw fp32 in the hi operand slot
    gives bit-identical results to the truncated hi plane (the PPO activations rely on it),
    and a GEMM given a lo-only plane writes lo = D - trunc(D) beside its fp32 output."""
    from robolearn_b200 import _native as N

    m, n, k, batch = 300, 256, 96, 2
    plan, D, ref = _run(1, m, n, k, 0, 0, batch=batch, ldd=n)
    lo = torch.zeros(batch, m, n, device="cuda")
    plan2, D2, _ = _run(1, m, n, k, 0, 0, batch=batch, ldd=n,
                        out_plane=N.Plane(lo=lo.data_ptr(), ld=n, twin_stride=m * n))
    plan2._keep.append(lo)
    plan.run()
    plan2.run()
    torch.cuda.synchronize()
    assert torch.equal(D, D2)
    hi = (D2.view(torch.int32) & -8192).view(torch.float32)
    assert torch.equal(lo, D2 - hi)
    # next product with the output as operand: (raw fp32, lo) == (truncated hi, lo)
    w = torch.randn(batch, 64, n, device="cuda") / n**0.5
    w_hi, w_lo = dense.tf32_split(w)
    outs = []
    for a_hi in (D2, hi):
        out = torch.zeros(batch, m, 64, device="cuda")
        p = dense.DensePlan(kind=1, m=m, n=64, k=n, a=a_hi, a_lo=lo, b=w_hi, b_lo=w_lo, lda=n, ldb=n, d=out, ldd=64,
                            a_major=0, b_major=0, batch=batch, a_batch_stride=m * n, b_batch_stride=64 * n,
                            d_batch_stride=m * 64)
        p.run()
        outs.append(out)
    torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[1])


@pytest.mark.parametrize("kind", [0, 1])
def test_gemm_eval_batch_norm_epilogue(kind):
    """Evaluation-mode batch norm fused into a transposed plan's epilogue:
    out = residual + relu((x - mean) * invstd * gamma + beta), plus the operand plane."""
    from robolearn_b200 import _native as N

    m, n, k, batch = 1000, 384, 160, 2
    g = torch.Generator(device="cuda").manual_seed(11)
    mean = torch.randn(batch, n, device="cuda", generator=g)
    invstd = torch.rand(batch, n, device="cuda", generator=g) + 0.5
    gamma = torch.randn(batch, n, device="cuda", generator=g)
    beta = torch.randn(batch, n, device="cuda", generator=g)
    res = torch.randn(batch, m, n, device="cuda", generator=g)
    pld = dense.operand_ld(n, kind)
    if kind == 0:
        h16 = torch.zeros(batch, m, pld, device="cuda", dtype=torch.float16)
        plane, keep = N.Plane(h16=h16.data_ptr(), ld=pld, twin_stride=m * pld), [h16]
    else:
        hi = torch.zeros(batch, m, pld, device="cuda")
        lo = torch.zeros(batch, m, pld, device="cuda")
        plane, keep = N.Plane(hi=hi.data_ptr(), lo=lo.data_ptr(), ld=pld, twin_stride=m * pld), [hi, lo]
    bn = (mean.data_ptr(), invstd.data_ptr(), gamma.data_ptr(), beta.data_ptr(), n, 1)
    plan, D, ref = _run(kind, m, n, k, 0, 0, batch=batch, ldd=n, residual=res, ldr=n, residual_batch_stride=m * n,
                        out_plane=plane, bn=bn)
    assert plan.transposed
    plan.run()
    torch.cuda.synchronize()
    y = (ref - mean.double()[:, None]) * invstd.double()[:, None] * gamma.double()[:, None] + beta.double()[:, None]
    expect = res.double() + torch.clamp(y, min=0)
    tol = 2e-3 if kind == 0 else 2e-5
    assert (D.double() - expect).abs().max().item() < tol * expect.abs().max().item()
    if kind == 0:
        assert torch.equal(keep[0][:, :, :n], D.half())
    else:
        assert torch.equal(keep[0][:, :, :n] + keep[1][:, :, :n], D)


def test_split_reduce_batched_matches_per_batch_reduce():
    """rl2_split_reduce_batched (one launch for several same-shape reductions, output stride
    possibly negative) equals one rl2_split_reduce per batch, bit for bit."""
    from robolearn_b200 import _native as N

    lib = N.load()
    splits, count, batch = 5, 3001, 2
    part = torch.randn(splits, batch, count, device="cuda")
    out = torch.zeros(2 * count + 17, device="cuda")
    ref = torch.zeros_like(out)
    s = torch.cuda.current_stream().cuda_stream
    base1 = out.data_ptr() + 4 * (count + 17)  # batch 0 written after batch 1: negative stride
    assert lib.rl2_split_reduce_batched(part.data_ptr(), batch * count, splits, base1, count, 0, batch, count,
                                        -(count + 17), s) == 0
    for b, off in ((0, count + 17), (1, 0)):
        assert lib.rl2_split_reduce(part.data_ptr() + 4 * b * count, batch * count, splits, ref.data_ptr() + 4 * off,
                                    count, 0, s) == 0
    torch.cuda.synchronize()
    assert torch.equal(out, ref)
    assert torch.allclose(out[count + 17:], part[:, 0].sum(0), rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("with_residual", [True, False])
@pytest.mark.parametrize("a_major,b_major", [(0, 0), (0, 1), (1, 0), (1, 1)])
@pytest.mark.parametrize("m,n,k", [(1000, 96, 1040), (600, 96, 1100), (512, 1000, 1030), (2048, 640, 1024)])
def test_gemm_cta_pair_plans(a_major, b_major, m, n, k, with_residual):
    """fp16 products with >= 512 kernel rows and >= 16 k-blocks run on CTA pairs (256-row
    tiles over two SMs):
    ragged pair tiles (a follower half partly or wholly outside M), both orientations
    (n >= 128: transposed accumulator, kernel rows = n; without a residual such plans
    take sixteen epilogue warps), all operand majors, bias (+ residual) + column moments,
    against float64."""
    batch = 2
    groups = (m + 31) // 32
    bias = torch.randn(batch, n, device="cuda")
    res = torch.randn(batch, m, n, device="cuda") if with_residual else None
    mean = torch.zeros(batch, groups, n, device="cuda")
    m2 = torch.zeros(batch, groups, n, device="cuda")
    plan, D, ref = _run(0, m, n, k, a_major, b_major, batch=batch, bias=bias, bias_batch_stride=n, residual=res,
                        ldr=n if with_residual else 0, residual_batch_stride=m * n if with_residual else 0,
                        stat_mean=mean, stat_m2=m2, stat_batch_stride=groups * n)
    assert plan.cta_pair, plan.shape
    plan.run()
    torch.cuda.synchronize()
    expect = ref + bias.double()[:, None, :] + (res.double() if with_residual else 0.0)
    out = D[:, :, :n].double()
    assert (out - expect).abs().max().item() < 2e-3 * expect.abs().max().item()
    full = torch.zeros(batch, groups * 32, n, device="cuda", dtype=torch.float64)
    full[:, :m] = out
    rows = full.view(batch, groups, 32, n)
    counts = torch.full((groups,), 32.0, device="cuda", dtype=torch.float64)
    counts[-1] = m - 32 * (groups - 1)
    mu = rows.sum(2) / counts[None, :, None]
    assert torch.allclose(mean.double(), mu, atol=1e-4, rtol=1e-4)


def test_gemm_cta_pair_split_k_and_graph_replay():
    """A CTA-pair plan with split-K partials, replayed from a CUDA graph, equals its eager run."""
    m, n, k, batch, splits = 512, 64, 2048, 2, 2
    stride = batch * m * n
    part = torch.zeros(splits, stride, device="cuda")
    g = torch.Generator(device="cuda").manual_seed(9)
    A = torch.randn(batch, m, k, device="cuda", generator=g).half().float()
    B = (torch.randn(batch, n, k, device="cuda", generator=g) / k**0.5).half().float()
    a_st, lda = _store(A, 0, 0)
    b_st, ldb = _store(B, 0, 0)
    plan = dense.DensePlan(kind=0, m=m, n=n, k=k, a=a_st, b=b_st, d=part, lda=lda, ldb=ldb, ldd=n, a_major=0,
                           b_major=0, batch=batch, a_batch_stride=a_st[0].numel(), b_batch_stride=b_st[0].numel(),
                           d_batch_stride=m * n, k_splits=splits, d_split_stride=stride)
    assert plan.cta_pair
    plan.run()
    torch.cuda.synchronize()
    eager = part.clone()
    got = eager.view(splits, batch, m, n).sum(0).double()
    ref = torch.einsum("zmk,znk->zmn", A.double(), B.double())
    assert (got - ref).abs().max().item() < 2e-3 * ref.abs().max().item()
    part.zero_()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s), torch.cuda.graph(graph, stream=s):
        plan.run()
    torch.cuda.current_stream().wait_stream(s)
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(part, eager)
