"""NumPy restatement of one FlashSAC learner update (test infrastructure only).

Every function follows the reference's Torch FlashSAC; the citations are paths
inside the reference project:

* networks: ``src/robolearn/flashsac/layers.py:15-303`` and ``networks.py:23-119``;
* update order and losses: ``src/robolearn/flashsac/updates.py:19-326`` and
  ``agent.py:217-281``;
* optimizer, scheduler, projection and EMA: ``agent.py:47-156``,
  ``_utils/network.py:56-80``, ``_utils/scheduler.py:43-65``.

Autograd is replaced by explicit analytic backward passes so that the CUDA path
(which also writes its backward out) can be compared stage by stage. Arithmetic
runs in ``dtype`` (float64 by default, so the oracle's own rounding is far below
the parity tolerances).
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np

BN_EPS = 1e-5
BN_MOMENTUM = 0.01
RMS_EPS = 1e-6
LOG_STD_MIN = -10.0
LOG_STD_MAX = 2.0
HALF_LOG_2PI = 0.5 * math.log(2.0 * math.pi)


# ----------------------------------------------------------------------------
# configuration and parameter layout
# ----------------------------------------------------------------------------


@dataclass
class Dims:
    """Network dimensions of one FlashSAC agent (``agent.py:56-130``)."""

    obs: int
    act: int
    actor_hidden: int
    actor_blocks: int
    critic_hidden: int
    critic_blocks: int
    bins: int
    min_v: float
    max_v: float
    critic_obs: int | None = None  # asymmetric critic input; None = obs
    expansion: int = 4

    @property
    def critic_in(self) -> int:
        return (self.critic_obs or self.obs) + self.act


def support(bins: int, min_v: float, max_v: float) -> np.ndarray:
    """``torch.linspace(min_v, max_v, bins)`` in float32 (``updates.py:53-55``, ``layers.py:291``).

    Torch's kernel evaluates the first half forwards from ``start`` and the second
    half backwards from ``end`` with a float32 step, each as one fused multiply-add
    (a single rounding). ``step * i`` and the sum are exact in float64 here, so one
    cast to float32 reproduces the fused result.
    """
    start, end = np.float32(min_v), np.float32(max_v)
    step = np.float64(np.float32((end - start) / np.float32(bins - 1)))
    out = np.empty(bins, dtype=np.float32)
    half = bins // 2
    for i in range(bins):
        if i < half:
            out[i] = np.float32(np.float64(start) + step * i)
        else:
            out[i] = np.float32(np.float64(end) - step * (bins - i - 1))
    return out


def actor_param_names(d: Dims) -> list[str]:
    """Actor ``state_dict`` parameter keys in ``nn.Module.parameters()`` order (``networks.py:23-61``)."""
    names = ["embedder.norm.weight", "embedder.norm.bias", "embedder.w.w.weight"]
    for i in range(d.actor_blocks):
        names += [
            f"encoder.{i}.w1.w.weight",
            f"encoder.{i}.w2.w.weight",
            f"encoder.{i}.norm1.weight",
            f"encoder.{i}.norm1.bias",
            f"encoder.{i}.norm2.weight",
            f"encoder.{i}.norm2.bias",
        ]
    names += [
        "post_norm.weight",
        "predictor.mean_bias",
        "predictor.std_bias",
        "predictor.mean_w.w.weight",
        "predictor.std_w.w.weight",
    ]
    return names


def critic_param_names(d: Dims) -> list[str]:
    """Double-critic parameter keys in ``parameters()`` order (``networks.py:64-110``)."""
    names = ["embedder.norm.weight", "embedder.norm.bias", "embedder.w.weight"]
    for i in range(d.critic_blocks):
        names += [
            f"encoder.{i}.w1.weight",
            f"encoder.{i}.w2.weight",
            f"encoder.{i}.norm1.weight",
            f"encoder.{i}.norm1.bias",
            f"encoder.{i}.norm2.weight",
            f"encoder.{i}.norm2.bias",
        ]
    names += ["post_norm.weight", "predictor.bias", "predictor.w.weight"]
    return names


def bn_buffer_prefixes(blocks: int) -> list[str]:
    out = ["embedder.norm"]
    for i in range(blocks):
        out += [f"encoder.{i}.norm1", f"encoder.{i}.norm2"]
    return out


# ----------------------------------------------------------------------------
# layer primitives over a leading "network" axis T (1 for the actor, 2 twins)
# ----------------------------------------------------------------------------


def _bn_forward_cols(x, w, b, rm, rv, training, eps=BN_EPS, momentum=BN_MOMENTUM):
    """Batch norm over rows of ``x[T,R,C]`` (``layers.py:32-55,189-214``).

    Training uses the biased variance and moves running statistics by
    ``lerp(momentum)`` with the unbiased variance; evaluation uses the buffers.
    Returns ``(y, cache, new_rm, new_rv)``.
    """
    if training:
        rows = x.shape[1]
        mean = x.mean(axis=1, keepdims=True)
        var = ((x - mean) ** 2).mean(axis=1, keepdims=True)
        inv = 1.0 / np.sqrt(var + eps)
        xhat = (x - mean) * inv
        new_rm = rm + momentum * (mean[:, 0] - rm)
        new_rv = rv + momentum * (var[:, 0] * (rows / (rows - 1)) - rv)
    else:
        inv = 1.0 / np.sqrt(rv[:, None, :] + eps)
        xhat = (x - rm[:, None, :]) * inv
        new_rm, new_rv = rm, rv
    y = xhat * w[:, None, :] + b[:, None, :]
    return y, (xhat, inv, w, training), new_rm, new_rv


def _bn_backward_cols(dy, cache):
    """Adjoint of :func:`bn_forward`; returns ``(dx, dw, db)``."""
    xhat, inv, w, training = cache
    dw = (dy * xhat).sum(axis=1)
    db = dy.sum(axis=1)
    g = dy * w[:, None, :]
    if training:
        dx = inv * (g - g.mean(axis=1, keepdims=True) - xhat * (g * xhat).mean(axis=1, keepdims=True))
    else:
        dx = g * inv
    return dx, dw, db


# Host threads for the column-independent batch-norm passes (off by default; the CPU
# baseline turns them on). Every column is computed by the same expressions whichever
# thread runs it, so the result does not depend on the thread count.
_THREADS = {"n": 1, "pool": None}


def set_threads(n: int) -> None:
    """Run the batch-norm passes of large arrays over ``n`` host threads (numpy releases
    the interpreter lock inside its array loops)."""
    from concurrent.futures import ThreadPoolExecutor

    n = max(1, int(n))
    if _THREADS["pool"] is not None:
        _THREADS["pool"].shutdown()
    _THREADS.update(n=n, pool=ThreadPoolExecutor(n) if n > 1 else None)


def _col_chunks(cols: int):
    n = _THREADS["n"]
    step = -(-cols // n)
    return [(c, min(c + step, cols)) for c in range(0, cols, step)]


def bn_forward(x, w, b, rm, rv, training, eps=BN_EPS, momentum=BN_MOMENTUM):
    """Batch norm over rows of ``x[T,R,C]`` (see :func:`_bn_forward_cols`), over column
    chunks on the host threads of :func:`set_threads` for large arrays."""
    pool = _THREADS["pool"]
    if pool is None or x.size < (1 << 20):
        return _bn_forward_cols(x, w, b, rm, rv, training, eps, momentum)
    T, _, C = x.shape
    dt = np.result_type(x, w)
    y, xhat = np.empty(x.shape, dt), np.empty(x.shape, dt)
    inv = np.empty((T, 1, C), dt)
    nrm, nrv = np.empty(rm.shape, np.result_type(rm, x)), np.empty(rv.shape, np.result_type(rv, x))

    def work(c):
        sl = slice(*c)
        yy, (xh, iv, _, _), r1, r2 = _bn_forward_cols(x[..., sl], w[:, sl], b[:, sl], rm[:, sl], rv[:, sl], training,
                                                     eps, momentum)
        y[..., sl], xhat[..., sl], inv[..., sl] = yy, xh, np.broadcast_to(iv, (T, 1, c[1] - c[0]))
        nrm[..., sl], nrv[..., sl] = r1, r2

    list(pool.map(work, _col_chunks(C)))
    return y, (xhat, inv, w, training), nrm, nrv


def bn_backward(dy, cache):
    """Adjoint of :func:`bn_forward` (see :func:`_bn_backward_cols`), column-chunked like it."""
    pool = _THREADS["pool"]
    if pool is None or dy.size < (1 << 20):
        return _bn_backward_cols(dy, cache)
    xhat, inv, w, training = cache
    T, _, C = dy.shape
    dt = np.result_type(dy, xhat)
    dx, dw, db = np.empty(dy.shape, dt), np.empty((T, C), dt), np.empty((T, C), dt)

    def work(c):
        sl = slice(*c)
        dx[..., sl], dw[:, sl], db[:, sl] = _bn_backward_cols(dy[..., sl], (xhat[..., sl], inv[..., sl], w[:, sl],
                                                                             training))

    list(pool.map(work, _col_chunks(C)))
    return dx, dw, db


def rms_forward(x, w, eps=RMS_EPS):
    """Row RMS norm ``x / sqrt(mean(x^2) + eps) * w`` (``layers.py:67-81,225-240``)."""
    r = 1.0 / np.sqrt((x * x).mean(axis=-1, keepdims=True) + eps)
    return x * r * w[:, None, :], (x, r, w)


def rms_backward(dy, cache):
    x, r, w = cache
    c = x.shape[-1]
    g = dy * w[:, None, :]
    dx = r * g - x * (r**3) * (g * x).sum(axis=-1, keepdims=True) / c
    dw = (dy * x * r).sum(axis=1)
    return dx, dw


def linear(x, w):
    """``x[T,R,K] @ w[T,N,K]^T`` (``layers.py:15-22,174-183``)."""
    return np.matmul(x, np.swapaxes(w, -1, -2))


def _tn(d, x):
    """weight gradient ``d[T,R,N]^T @ x[T,R,K] -> [T,N,K]``"""
    return np.matmul(np.swapaxes(d, -1, -2), x)


def _nn(d, w):
    """input gradient ``d[T,R,N] @ w[T,N,K] -> [T,R,K]``"""
    return np.matmul(d, w)


# Operand rounding of the dense products. The FP32 recipe leaves operands as they
# are; the FP16-operand recipe rounds every product operand to fp16 (gradient
# operands after multiplying by the loss scale S, then divided by S), which is
# what both the reference's autocast path and the CUDA path feed the tensor cores.
_ROUND = {"mode": "fp32", "scale": 1.0}


def set_operand_rounding(mode: str = "fp32", scale: float = 1.0) -> None:
    """Round every dense-product operand as a CUDA recipe does before its tensor-core
    products: "fp16" (operands rounded to fp16, gradient operands carrying ``scale``), or
    "tf32x3" (the FP32 recipe's split: the fp32 value's high part with the low 13 mantissa
    bits cleared, plus the remainder as the tensor core reads it, truncated to tf32; the
    model multiplies the two rounded sums, so it keeps the lo x lo term the recipe drops,
    about 2^-22 of each product). "fp32" leaves operands exact."""
    if mode not in ("fp32", "fp16", "tf32x3"):
        raise ValueError(mode)
    _ROUND["mode"], _ROUND["scale"] = mode, float(scale)


def _tf32_trunc(v32):
    return (np.asarray(v32, np.float32).view(np.uint32) & np.uint32(0xFFFFE000)).view(np.float32)


def _tf32x3(x):
    x32 = np.asarray(x, np.float32)
    hi = _tf32_trunc(x32)
    lo = _tf32_trunc(x32 - hi)
    return hi.astype(np.float64) + lo.astype(np.float64)


def _rf(x):
    """forward / weight operand"""
    if _ROUND["mode"] == "fp16":
        return np.asarray(x).astype(np.float16).astype(np.float64)
    if _ROUND["mode"] == "tf32x3":
        return _tf32x3(x)
    return x


def _rg(x):
    """gradient operand (carries the loss scale while rounded)"""
    if _ROUND["mode"] == "fp16":
        s = _ROUND["scale"]
        return (np.asarray(x) * s).astype(np.float16).astype(np.float64) / s
    if _ROUND["mode"] == "tf32x3":
        return _tf32x3(x)
    return x


def relu(x):
    return np.maximum(x, 0.0)


def softplus(x):
    return np.where(x > 0, x + np.log1p(np.exp(-np.abs(x))), np.log1p(np.exp(x)))


def sigmoid(x):
    return 0.5 * (1.0 + np.tanh(0.5 * x))


# ----------------------------------------------------------------------------
# backbone (embedder -> residual blocks -> RMS post-norm), shared by actor and critic
# ----------------------------------------------------------------------------


_MARGIN = [np.inf]
# ReLU sites are numbered in call order since the last reset; a near-kink element is
# (site, flat index) with |pre-activation| below _KINK["margin"]; _KINK["flips"] holds
# the elements whose decision is evaluated the other way (the pre-activation's sign is
# flipped there, so the forward value and the backward mask both take the other branch);
# _KINK["adopt"] maps a site to another evaluation's pre-normalisation output, whose
# decisions (rebuilt with this evaluation's batch-norm statistics) are taken wherever
# they differ from this one's
_KINK = {"site": 0, "margin": 0.0, "near": [], "flips": set(), "adopt": {}, "adopted": 0, "track": False,
         "keep": False, "pre": {}}


def _kink(pre_relu, bn=None):
    """Note how close this ReLU's decisions are to the kink, record near-kink elements and
    apply requested decision flips. ``bn`` = (pre-normalisation input, mean, invstd,
    weight, bias) of the batch norm that produced ``pre_relu``, used to rebuild adopted
    decisions. Returns the pre-activation to feed the ReLU."""
    site = _KINK["site"]
    _KINK["site"] += 1
    if not _KINK["track"]:  # no reset since import: plain evaluation, nothing recorded
        return pre_relu
    a = np.abs(pre_relu)
    _MARGIN[0] = min(_MARGIN[0], float(a.min()))
    if _KINK["margin"] > 0:
        for i in np.flatnonzero(a.ravel() < _KINK["margin"]):
            _KINK["near"].append((site, int(i)))
    flip = np.zeros(pre_relu.size, dtype=bool)
    mine = [i for (s_, i) in _KINK["flips"] if s_ == site]
    flip[mine] = True
    if _KINK["keep"] and bn is not None:
        _KINK["pre"][site] = np.array(bn[0], copy=True)
    other = _KINK["adopt"].get(site)
    if other is not None and bn is not None:
        _, mean, inv, w, b = bn
        if isinstance(other, tuple):
            # (pre-normalisation output, mean, invstd) of a float32 evaluation: its decision
            # is the sign of fma((x - mean) * invstd, weight, bias) with float32 roundings of
            # the difference and the product; the fused multiply-add's sign is that of the
            # exact value, which float64 holds exactly for float32 factors
            ox, om, oi = (np.asarray(v, np.float32) for v in other)
            f32 = np.float32
            xh = ((ox.reshape(pre_relu.shape) - om[:, None, :]).astype(f32) * oi[:, None, :]).astype(f32)
            rebuilt = xh.astype(np.float64) * w.astype(f32)[:, None, :].astype(np.float64) \
                + b.astype(f32)[:, None, :].astype(np.float64)
        else:
            rebuilt = (np.asarray(other, np.float64).reshape(pre_relu.shape) - mean) * inv * w[:, None, :] + b[:, None, :]
        differ = ((rebuilt > 0) != (pre_relu > 0)).ravel()
        _KINK["adopted"] += int(differ.sum())
        flip ^= differ
    if flip.any():
        pre_relu = np.array(pre_relu, copy=True)
        flat = pre_relu.reshape(-1)
        flat[flip] = -flat[flip]
    return pre_relu


def relu_margin_reset(record_below: float = 0.0, flips=(), adopt=None, keep_pre: bool = False) -> None:
    """Start a new update: reset the margin and the site counter; record elements whose
    |pre-activation| is below ``record_below``; evaluate the decisions of ``flips``
    ((site, flat index) pairs from :func:`relu_near_kinks`) the other way; take the
    decisions of another evaluation at the sites of ``adopt`` (site -> its
    pre-normalisation output, same shape as this evaluation's, rebuilt with this
    evaluation's statistics; or a float32 evaluation's (output, mean [T,C], invstd [T,C]),
    rebuilt with its own statistics and float32 roundings); with ``keep_pre`` keep
    this evaluation's own pre-normalisation outputs (:func:`relu_pre_outputs`)."""
    _MARGIN[0] = np.inf
    _KINK.update(site=0, margin=float(record_below), near=[], flips=set(flips), adopt=dict(adopt or {}), adopted=0,
                 track=True, keep=bool(keep_pre), pre={})


def relu_near_kinks() -> list[tuple[int, int]]:
    """(site, flat index) of the pre-activations below the recording margin since the reset."""
    return list(_KINK["near"])


def relu_pre_outputs() -> dict:
    """Site -> pre-normalisation output kept since a ``keep_pre`` reset."""
    return dict(_KINK["pre"])


def relu_adopted() -> int:
    """How many decisions were taken from the other evaluation since the reset."""
    return _KINK["adopted"]


def relu_margin() -> float:
    """Smallest |pre-ReLU| value since the last reset (tracking starts at the first reset);
    a decision closer to 0 than the arithmetic's rounding is not determined by fp32
    evaluation order."""
    return _MARGIN[0]


def _bn_ctx(x, cache, running_mean, bias):
    """(input, mean, invstd, weight, bias) of a batch norm, for rebuilding decisions."""
    if not (_KINK["adopt"] or _KINK["keep"]):
        return None
    _, inv, w, training = cache
    mean = x.mean(axis=1, keepdims=True) if training else running_mean[:, None, :]
    return x, mean, inv, w, bias


def _stack(p: dict, key: str, twin: bool) -> np.ndarray:
    v = p[key]
    return v if twin else v[None]


def backbone_forward(p, x, blocks, training, twin, dtype):
    """Embedder + residual blocks + post-norm (``layers.py:84-113``, ``networks.py:50-61,97-110``).

    ``x`` is ``[T,R,C]``. Returns ``(features, cache, running_stat_updates)``.
    """
    wkey = "embedder.w.weight" if twin else "embedder.w.w.weight"
    stats = {}
    caches = []
    g = lambda k: _stack(p, k, twin).astype(dtype)  # noqa: E731
    y, c_bn, rm, rv = bn_forward(
        x, g("embedder.norm.weight"), g("embedder.norm.bias"),
        g("embedder.norm.running_mean"), g("embedder.norm.running_var"), training,
    )
    stats["embedder.norm"] = (rm, rv)
    w_e = g(wkey)
    h = linear(_rf(y), _rf(w_e))
    caches.append(("embed", y, c_bn, w_e))
    for i in range(blocks):
        suffix = ".weight" if twin else ".w.weight"
        w1 = g(f"encoder.{i}.w1{suffix}")
        w2 = g(f"encoder.{i}.w2{suffix}")
        t1 = linear(_rf(h), _rf(w1))
        n1, c1, rm1, rv1 = bn_forward(
            t1, g(f"encoder.{i}.norm1.weight"), g(f"encoder.{i}.norm1.bias"),
            g(f"encoder.{i}.norm1.running_mean"), g(f"encoder.{i}.norm1.running_var"), training,
        )
        n1 = _kink(n1, _bn_ctx(t1, c1, g(f"encoder.{i}.norm1.running_mean"), g(f"encoder.{i}.norm1.bias")))
        a1 = relu(n1)
        t2 = linear(_rf(a1), _rf(w2))
        n2, c2, rm2, rv2 = bn_forward(
            t2, g(f"encoder.{i}.norm2.weight"), g(f"encoder.{i}.norm2.bias"),
            g(f"encoder.{i}.norm2.running_mean"), g(f"encoder.{i}.norm2.running_var"), training,
        )
        n2 = _kink(n2, _bn_ctx(t2, c2, g(f"encoder.{i}.norm2.running_mean"), g(f"encoder.{i}.norm2.bias")))
        a2 = relu(n2)
        stats[f"encoder.{i}.norm1"] = (rm1, rv1)
        stats[f"encoder.{i}.norm2"] = (rm2, rv2)
        caches.append(("block", h, w1, w2, c1, n1, a1, c2, n2))
        h = a2 + h
    u, c_rms = rms_forward(h, g("post_norm.weight"))
    caches.append(("rms", c_rms))
    return u, caches, stats


def backbone_backward(du, caches, blocks, twin, need_input_grad):
    """Adjoint of :func:`backbone_forward`. Returns ``(grads, dx)`` with twin-shaped grads."""
    grads = {}
    dh, grads["post_norm.weight"] = rms_backward(du, caches[-1][1])
    for i in reversed(range(blocks)):
        _, h_in, w1, w2, c1, n1, a1, c2, n2 = caches[1 + i]
        suffix = ".weight" if twin else ".w.weight"
        d_n2 = dh * (n2 > 0)
        d_t2, grads[f"encoder.{i}.norm2.weight"], grads[f"encoder.{i}.norm2.bias"] = bn_backward(d_n2, c2)
        grads[f"encoder.{i}.w2{suffix}"] = _tn(_rg(d_t2), _rf(a1))
        d_a1 = _nn(_rg(d_t2), _rf(w2))
        d_n1 = d_a1 * (n1 > 0)
        d_t1, grads[f"encoder.{i}.norm1.weight"], grads[f"encoder.{i}.norm1.bias"] = bn_backward(d_n1, c1)
        grads[f"encoder.{i}.w1{suffix}"] = _tn(_rg(d_t1), _rf(h_in))
        dh = _nn(_rg(d_t1), _rf(w1)) + dh
    _, y_e, c_bn, w_e = caches[0]
    grads["embedder.w.weight" if twin else "embedder.w.w.weight"] = _tn(_rg(dh), _rf(y_e))
    d_y = _nn(_rg(dh), _rf(w_e))
    dx, grads["embedder.norm.weight"], grads["embedder.norm.bias"] = bn_backward(d_y, c_bn)
    if not twin:
        grads = {k: v[0] for k, v in grads.items()}
    return grads, (dx if need_input_grad else None)


# ----------------------------------------------------------------------------
# actor (NormalTanhPolicy) and double critic (categorical value)
# ----------------------------------------------------------------------------


def actor_forward(p, d: Dims, obs, noise, training, dtype=np.float64):
    """``FlashSACActor.forward`` with reparameterised noise (``layers.py:116-166``).

    Returns ``(actions, log_probs, cache, stats)``.
    """
    x = obs.astype(dtype)[None]
    u, caches, stats = backbone_forward(p, x, d.actor_blocks, training, False, dtype)
    u0 = u[0]
    wm = p["predictor.mean_w.w.weight"].astype(dtype)
    ws = p["predictor.std_w.w.weight"].astype(dtype)
    mean = _rf(u0) @ _rf(wm).T + p["predictor.mean_bias"].astype(dtype)
    s = _rf(u0) @ _rf(ws).T + p["predictor.std_bias"].astype(dtype)
    ts = np.tanh(s)
    log_std = LOG_STD_MIN + (LOG_STD_MAX - LOG_STD_MIN) * 0.5 * (1.0 + ts)
    std = np.exp(log_std)
    eps = noise.astype(dtype)
    raw = mean + std * eps
    action = np.tanh(raw)
    jac = 2.0 * (math.log(2.0) - raw - softplus(-2.0 * raw))
    log_prob = (-0.5 * eps * eps - log_std - HALF_LOG_2PI - jac).sum(axis=1)
    cache = dict(caches=caches, u=u0, wm=wm, ws=ws, ts=ts, std=std, eps=eps, raw=raw, action=action)
    return action, log_prob, cache, stats


def actor_backward(cache, d: Dims, d_action, d_log_prob):
    """Adjoint of :func:`actor_forward` w.r.t. actor parameters."""
    raw, action, std, eps, ts = cache["raw"], cache["action"], cache["std"], cache["eps"], cache["ts"]
    dlp = d_log_prob[:, None]
    # d logp / d raw = 2 tanh(raw) (tanh Jacobian correction, distribution.py:12-19)
    d_raw = d_action * (1.0 - action * action) + dlp * 2.0 * action
    d_mean = d_raw
    d_log_std = d_raw * std * eps - dlp
    d_s = d_log_std * (LOG_STD_MAX - LOG_STD_MIN) * 0.5 * (1.0 - ts * ts)
    u = cache["u"]
    grads = {
        "predictor.mean_w.w.weight": _rg(d_mean).T @ _rf(u),
        "predictor.std_w.w.weight": _rg(d_s).T @ _rf(u),
        "predictor.mean_bias": d_mean.sum(axis=0),
        "predictor.std_bias": d_s.sum(axis=0),
    }
    du = _rg(d_mean) @ _rf(cache["wm"]) + _rg(d_s) @ _rf(cache["ws"])
    g2, _ = backbone_backward(du[None], cache["caches"], d.actor_blocks, False, False)
    grads.update(g2)
    return grads


def critic_forward(p, d: Dims, obs, act, training, dtype=np.float64):
    """``FlashSACDoubleCritic.forward`` (``networks.py:97-110``, ``layers.py:275-303``).

    Returns ``(q[2,R], log_probs[2,R,bins], cache, stats)``.
    """
    x = np.concatenate([obs, act], axis=-1).astype(dtype)
    x = np.broadcast_to(x[None], (2,) + x.shape)
    u, caches, stats = backbone_forward(p, x, d.critic_blocks, training, True, dtype)
    w = p["predictor.w.weight"].astype(dtype)
    logits = linear(_rf(u), _rf(w)) + p["predictor.bias"].astype(dtype)[:, None, :]
    mx = logits.max(axis=-1, keepdims=True)
    lse = mx + np.log(np.exp(logits - mx).sum(axis=-1, keepdims=True))
    log_probs = logits - lse
    z = support(d.bins, d.min_v, d.max_v).astype(dtype)
    probs = np.exp(log_probs)
    q = (probs * z).sum(axis=-1)
    cache = dict(caches=caches, u=u, w=w, probs=probs, q=q, z=z)
    return q, log_probs, cache, stats


def critic_backward(cache, d: Dims, d_log_probs=None, d_q=None, need_input_grad=False):
    """Adjoint of :func:`critic_forward`: log-softmax + expected value, head, backbone."""
    probs, z, q = cache["probs"], cache["z"], cache["q"]
    d_logits = np.zeros_like(probs)
    if d_log_probs is not None:
        d_logits += d_log_probs - probs * d_log_probs.sum(axis=-1, keepdims=True)
    if d_q is not None:
        d_logits += d_q[..., None] * probs * (z - q[..., None])
    u = cache["u"]
    grads = {
        "predictor.w.weight": _tn(_rg(d_logits), _rf(u)),
        "predictor.bias": d_logits.sum(axis=1),
    }
    du = _nn(_rg(d_logits), _rf(cache["w"]))
    g2, dx = backbone_backward(du, cache["caches"], d.critic_blocks, True, need_input_grad)
    grads.update(g2)
    return grads, (dx.sum(axis=0) if need_input_grad else None)


# ----------------------------------------------------------------------------
# categorical Bellman target and cross-entropy (updates.py:19-80, 248-257)
# ----------------------------------------------------------------------------


def select_min_q(next_qs, next_log_probs):
    """``_select_min_q_log_probs``: per row the twin with the smaller Q; ties pick twin 0."""
    idx = np.argmin(next_qs, axis=0)
    return next_log_probs[idx, np.arange(next_qs.shape[1])]


def categorical_target(log_probs, reward, done, entropy, gamma, bins, min_v, max_v):
    """``_compute_categorical_td_target`` evaluated in float32 exactly as Torch does on CPU.

    The floor of the fractional bin index is index arithmetic, so this is done in
    float32 with the same operation order to keep the lower/upper split identical.
    """
    f = np.float32
    lp = log_probs.astype(f)
    r = reward.astype(f)[:, None]
    dn = done.astype(f)[:, None]
    ent = entropy.astype(f)[:, None]
    g = np.asarray(gamma, dtype=f).reshape(-1, 1)
    width = f((max_v - min_v) / (bins - 1))
    z = support(bins, min_v, max_v)[None]
    v = r + g * (z - ent) * (f(1.0) - dn)
    v = np.clip(v, f(min_v), f(max_v)).astype(f)
    b = ((v - f(min_v)) / width).astype(f)
    lower = np.floor(b).astype(np.int64)
    upper = np.clip(lower + 1, 0, bins - 1)
    frac = (b - lower.astype(f)).astype(f)
    p = np.exp(lp.astype(np.float64))
    out = np.zeros(lp.shape, dtype=np.float64)
    rows = np.arange(lp.shape[0])[:, None]
    np.add.at(out, (np.broadcast_to(rows, lower.shape), lower), p * (1.0 - frac))
    np.add.at(out, (np.broadcast_to(rows, upper.shape), upper), p * frac)
    return out, (lower, upper, frac)


def categorical_loss_grad(pred_log_probs, target, rows_total):
    """CE ``-(t * logp).sum(-1)`` averaged over ``[2, B]`` and its logits gradient.

    ``pred_log_probs`` is ``[2, B, bins]`` (current-observation half), ``rows_total``
    the number of rows in the critic batch (2B): the rows of the next-observation
    half receive a zero gradient. Returns ``(loss, dlogits[2, rows_total, bins])``.
    """
    twins, b, bins = pred_log_probs.shape
    ce = -(target[None] * pred_log_probs).sum(axis=-1)
    loss = ce.mean()
    p = np.exp(pred_log_probs)
    d = np.zeros((twins, rows_total, bins))
    d[:, :b] = (p * target[None].sum(axis=-1, keepdims=True) - target[None]) / (twins * b)
    return loss, d


# ----------------------------------------------------------------------------
# optimizer, schedule, projection, EMA
# ----------------------------------------------------------------------------


def warmup_cosine(step, init, peak, end, warmup, decay):
    """``warmup_cosine_decay_scheduler`` (``_utils/scheduler.py:43-65``)."""
    if step < warmup:
        return init + (peak - init) * (step / warmup)
    if step < decay:
        progress = (step - warmup) / (decay - warmup)
        return end + (peak - end) * 0.5 * (1 + math.cos(math.pi * progress))
    return end


def adam_torch(p, g, m, v, step, lr, b1=0.9, b2=0.999, eps=1e-8):
    """Torch single-tensor Adam (no weight decay): ``p -= lr/bc1 * m / (sqrt(v)/sqrt(bc2) + eps)``."""
    m = m + (1 - b1) * (g - m)
    v = b2 * v + (1 - b2) * g * g
    bc1 = 1 - b1**step
    bc2 = 1 - b2**step
    p = p - (lr / bc1) * m / (np.sqrt(v) / math.sqrt(bc2) + eps)
    return p, m, v


def adam_warp(p, g, m, v, step, lr, b1=0.9, b2=0.999, eps=1e-8):
    """Warp-NN Adam as restated by the reference (``cuda/kernels.cu:310-337``)."""
    m = b1 * m + (1 - b1) * g
    v = b2 * v + (1 - b2) * g * g
    c1 = 1.0 / (1.0 - b1**step)
    c2 = 1.0 / (1.0 - b2**step)
    p = p - lr * (m * c1) / (np.sqrt(v * c2) + eps)
    return p, m, v


def project(p: dict, names: list[str], twin: bool, blocks: int) -> dict:
    """``Network.normalize_parameters`` (``_utils/network.py:56-67``, ``layers.py:24-29,57-64,76-81``).

    Unit-linear rows -> unit L2 norm (eps 1e-8); BN (weight, bias) -> joint norm
    sqrt(C); RMS weight -> norm sqrt(C). Head biases are not projected.
    """
    out = dict(p)
    for k in names:
        if is_unit_linear(k):
            w = p[k]
            n = np.sqrt((w * w).sum(axis=-1, keepdims=True))
            out[k] = w / np.maximum(n, 1e-8)
    for pre in bn_buffer_prefixes(blocks):
        w, b = p[pre + ".weight"], p[pre + ".bias"]
        c = w.shape[-1]
        f = math.sqrt(c) / np.sqrt((w * w + b * b).sum(axis=-1, keepdims=True) + 1e-8)
        out[pre + ".weight"], out[pre + ".bias"] = w * f, b * f
    w = p["post_norm.weight"]
    c = w.shape[-1]
    out["post_norm.weight"] = w * (math.sqrt(c) / np.sqrt((w * w).sum(axis=-1, keepdims=True) + 1e-8))
    return out


def is_unit_linear(name: str) -> bool:
    """Whether a parameter key names a projected unit-linear weight (``layers.py:15-29,174-186``)."""
    return name.endswith(".weight") and "norm" not in name and not name.endswith("bias")


def ema(target: dict, online: dict, names: list[str], tau: float) -> dict:
    """``torch._foreach_lerp_(target, online, tau)`` over parameters only (``_utils/network.py:66-80``)."""
    out = dict(target)
    for k in names:
        out[k] = target[k] + tau * (online[k] - target[k])
    return out


# ----------------------------------------------------------------------------
# one full update (agent.py:217-281, updates.py:83-326)
# ----------------------------------------------------------------------------


@dataclass
class OptState:
    m: dict = field(default_factory=dict)
    v: dict = field(default_factory=dict)
    step: int = 0


@dataclass
class Hyper:
    gamma: float = 0.99
    tau: float = 0.005
    lr_init: float = 3e-4
    lr_peak: float = 3e-4
    lr_end: float = 1.5e-4
    warmup: int = 0
    decay: int = 10_000
    target_entropy: float = 0.0
    bc_alpha: float = 0.0
    adam: str = "torch"  # "torch" (FlashSAC) or "warp" (Warp-NN formula, WarpFlashSAC)


def _adam_net(params: dict, grads: dict, opt: OptState, names: list[str], lr: float, dtype, formula: str = "torch"):
    opt.step += 1
    out = dict(params)
    rule = adam_warp if formula == "warp" else adam_torch
    for k in names:
        p = params[k].astype(dtype)
        m = opt.m.get(k, np.zeros_like(p))
        v = opt.v.get(k, np.zeros_like(p))
        out[k], opt.m[k], opt.v[k] = rule(p, grads[k].astype(dtype), m, v, opt.step, lr)
    return out


def _apply_stats(params: dict, stats: dict) -> dict:
    out = dict(params)
    for pre, (rm, rv) in stats.items():
        out[pre + ".running_mean"] = rm if rm.ndim == out[pre + ".running_mean"].ndim else rm[0]
        out[pre + ".running_var"] = rv if rv.ndim == out[pre + ".running_var"].ndim else rv[0]
    return out


def update_networks(state: dict, batch: dict, actor_noise, next_noise, d: Dims, h: Hyper,
                    do_actor: bool, dtype=np.float64) -> tuple[dict, dict]:
    """One ``_update_networks`` call with fixed batch and noise.

    ``state`` holds ``actor``, ``critic``, ``target`` (state-dict-like mappings),
    ``log_temp`` and optimizer states ``opt_actor``, ``opt_critic``, ``opt_temp``.
    ``batch`` holds observation, next_observation, action, reward (already
    normalised), terminated, discount; ``actor_observation`` keys are derived from
    the observation prefix. Returns ``(new_state, metrics)``.
    """
    a_names = actor_param_names(d)
    c_names = critic_param_names(d)
    actor = dict(state["actor"])
    critic = dict(state["critic"])
    target = dict(state["target"])
    log_temp = float(state["log_temp"])
    opt_a, opt_c, opt_t = state["opt_actor"], state["opt_critic"], state["opt_temp"]
    obs = batch["observation"].astype(dtype)
    nobs = batch["next_observation"].astype(dtype)
    a_obs = obs[:, : d.obs]
    a_nobs = nobs[:, : d.obs]
    B = obs.shape[0]
    metrics = {}
    grads_out = {}

    if do_actor:
        # ---- update_actor (updates.py:83-166)
        alpha = math.exp(log_temp)
        obs_all = np.concatenate([a_obs, a_nobs], axis=0)
        acts_all, lp_all, a_cache, a_stats = actor_forward(actor, d, obs_all, actor_noise, True, dtype)
        acts, lps = acts_all[:B], lp_all[:B]
        qs, _, c_cache, _ = critic_forward(critic, d, obs, acts, False, dtype)
        q = np.minimum(qs[0], qs[1])
        loss = (lps * alpha - q).mean()
        d_q = np.zeros_like(qs)
        tie = qs[0] == qs[1]
        d_q[0] = np.where(qs[0] < qs[1], -1.0 / B, np.where(tie, -0.5 / B, 0.0))
        d_q[1] = np.where(qs[1] < qs[0], -1.0 / B, np.where(tie, -0.5 / B, 0.0))
        d_act = np.zeros_like(acts_all)
        if h.bc_alpha > 0:
            q_abs = np.abs(q).mean()
            bc = ((acts - batch["action"].astype(dtype)) ** 2).mean()
            loss = loss + h.bc_alpha * q_abs * bc
            d_act[:B] += h.bc_alpha * q_abs * 2.0 * (acts - batch["action"].astype(dtype)) / acts.size
        _, dx = critic_backward(c_cache, d, d_q=d_q, need_input_grad=True)
        d_act[:B] += dx[:, -d.act:]
        d_lp = np.zeros(2 * B)
        d_lp[:B] = alpha / B
        grads = actor_backward(a_cache, d, d_act, d_lp)
        grads_out["actor"] = grads
        entropy = -lps.mean()
        metrics["actor/loss"] = loss
        metrics["actor/entropy"] = entropy
        metrics["actor/mean_action"] = acts.mean()
        lr = warmup_cosine(opt_a.step, h.lr_init, h.lr_peak, h.lr_end, h.warmup, h.decay)
        actor = _apply_stats(actor, a_stats)
        actor = _adam_net(actor, grads, opt_a, a_names, lr, dtype, h.adam)
        actor = project(actor, a_names, False, d.actor_blocks)
        # ---- update_temperature (updates.py:297-326)
        tval = math.exp(log_temp)
        t_loss = tval * (entropy - h.target_entropy)
        g_t = np.array([tval * (entropy - h.target_entropy)])
        lr_t = warmup_cosine(opt_t.step, h.lr_init, h.lr_peak, h.lr_end, h.warmup, h.decay)
        tp = _adam_net({"log_temp": np.array([log_temp])}, {"log_temp": g_t}, opt_t, ["log_temp"], lr_t, dtype,
                       h.adam)
        log_temp = float(tp["log_temp"][0])
        metrics["temperature/value"] = tval
        metrics["temperature/loss"] = t_loss

    # ---- update_critic (updates.py:169-284)
    n_act, n_lp, _, _ = actor_forward(actor, d, a_nobs, next_noise, False, dtype)
    tval = math.exp(log_temp)
    n_ent = tval * n_lp
    obs_all = np.concatenate([obs, nobs], axis=0)
    act_all = np.concatenate([batch["action"].astype(dtype), n_act], axis=0)
    t_q, t_lp, _, t_stats = critic_forward(target, d, obs_all, act_all, True, dtype)
    sel = select_min_q(t_q[:, B:], t_lp[:, B:])
    tgt, _ = categorical_target(sel, batch["reward"], batch["terminated"], n_ent, batch["discount"],
                                d.bins, d.min_v, d.max_v)
    metrics["critic/max_entropy_bonus"] = n_ent.max()
    target = _apply_stats(target, t_stats)
    _, p_lp, c_cache, c_stats = critic_forward(critic, d, obs_all, act_all, True, dtype)
    loss, d_logits = categorical_loss_grad(p_lp[:, :B], tgt, 2 * B)
    metrics["critic/loss"] = loss
    grads, _ = _critic_backward_from_logits(c_cache, d, d_logits)
    grads_out["critic"] = grads
    lr = warmup_cosine(opt_c.step, h.lr_init, h.lr_peak, h.lr_end, h.warmup, h.decay)
    critic = _apply_stats(critic, c_stats)
    critic = _adam_net(critic, grads, opt_c, c_names, lr, dtype, h.adam)
    critic = project(critic, c_names, True, d.critic_blocks)
    # ---- update_target_network (updates.py:287-294)
    target = ema(target, critic, c_names, h.tau)

    new_state = dict(state)
    new_state.update(actor=actor, critic=critic, target=target, log_temp=log_temp,
                     opt_actor=opt_a, opt_critic=opt_c, opt_temp=opt_t, grads=grads_out)
    return new_state, metrics


def _critic_backward_from_logits(cache, d: Dims, d_logits):
    u = cache["u"]
    grads = {
        "predictor.w.weight": _tn(_rg(d_logits), _rf(u)),
        "predictor.bias": d_logits.sum(axis=1),
    }
    du = _nn(_rg(d_logits), _rf(cache["w"]))
    g2, _ = backbone_backward(du, cache["caches"], d.critic_blocks, True, False)
    grads.update(g2)
    return grads, None
