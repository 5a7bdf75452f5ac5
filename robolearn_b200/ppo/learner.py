"""``WarpPPO`` on sm_100a kernels: drop-in for ``robolearn.warp.WarpPPO``
(``src/robolearn/warp/ppo.py:353-778``).

Same constructor and validation, ``act`` / ``store`` / ``compute_returns`` /
``launch_update`` / ``warmup`` / ``update(capture)`` / ``health_metrics`` /
``state_dict`` / ``load_state_dict`` / ``save`` / ``load`` and the public rollout
arrays (``observations, actions, means, stds, log_probs, values, rewards,
next_values, advantages, returns, terminated, truncated``) as torch CUDA tensors.

Device layout. All parameters live in one fp32 arena in the reference's order --
actor (W [out, in], b [out, 1]) per layer, critic likewise, then the std parameter --
so ``state_dict`` keys ``parameter_i`` map to views. Actor and critic share hidden
widths and their input, so every layer runs as ONE twin-batched tcgen05 GEMM (batch 0 =
actor, 1 = critic; the twin stride through the arena is the actor's size). The heads
differ (act outputs vs 1): the critic head's weight-plane rows past the first are zero,
its extra outputs are ignored and receive zero gradient. GEMM operands are three-
product tf32 planes (fp32-accurate, hi + lo) written by the producers: the minibatch
gather, each layer's epilogue (bias + ELU / tanh fused) and the optimizer (weights).
Backward: the loss kernel writes the head gradient plane; each layer's input-gradient
GEMM multiplies by the activation derivative in its epilogue (from the stored outputs)
and emits per-32-row column sums for the bias gradient; weight gradients use split-K
GEMMs reduced in a fixed order; clipping and Warp-NN Adam (with the weight-plane
refresh) finish the step. ``update()`` records the whole update as one CUDA graph.
"""

from __future__ import annotations

import ctypes
import math
from pathlib import Path

import numpy as np
import torch

from .. import _native as N
from ..dense import ELU, TANH, TF32X3, DensePlan, operand_ld
from .config import PPOConfig

SM_COUNT = 148
_STATE_FLOATS = 9  # optimizer state [attempts, steps, step_size, bc2, lr, skip, scale, growth, skipped]


class _Layout:
    """Offsets of every parameter in the flat arena (reference parameter order)."""

    def __init__(self, obs: int, act: int, hidden: tuple[int, ...]):
        self.obs, self.act, self.hidden = obs, act, tuple(hidden)
        self.layers = len(self.hidden) + 1
        self.widths = (obs, *self.hidden)  # layer inputs
        self.outs = {"actor": (*self.hidden, act), "critic": (*self.hidden, 1)}
        self.shapes: list[tuple] = []
        self.offsets: list[int] = []
        self.w_off = {"actor": [], "critic": []}
        self.b_off = {"actor": [], "critic": []}
        o = 0
        for net in ("actor", "critic"):
            for li in range(self.layers):
                out, inp = self.outs[net][li], self.widths[li]
                for shape, table in (((out, inp), self.w_off), ((out, 1), self.b_off)):
                    self.shapes.append(shape)
                    self.offsets.append(o)
                    table[net].append(o)
                    o += shape[0] * shape[1]
            if net == "actor":
                self.actor_size = o
        self.critic_size = o - self.actor_size
        self.std_off = o
        self.shapes.append((act,))
        self.offsets.append(o)
        self.size = o + act
        # weight planes: per layer [2][rows = actor outputs][operand_ld(in)]
        self.kp = [operand_ld(w, TF32X3) for w in self.widths]
        self.plane_off = []
        p = 0
        for li in range(self.layers):
            self.plane_off.append(p)
            p += 2 * self.outs["actor"][li] * self.kp[li]
        self.plane_size = p

    def segments(self) -> list[tuple[int, int, int, int, int]]:
        """(offset, offset2, plane_offset, length, kind) per optimizer unit: one per weight
        row (refreshing its operand-plane row), one per bias, one for the std parameter."""
        rows = []
        for z, net in enumerate(("actor", "critic")):
            for li in range(self.layers):
                out, inp = self.outs[net][li], self.widths[li]
                ra = self.outs["actor"][li]
                for r in range(out):
                    rows.append((self.w_off[net][li] + r * inp, -1,
                                 self.plane_off[li] + (z * ra + r) * self.kp[li], inp, 0))
                rows.append((self.b_off[net][li], -1, -1, out, 0))
        rows.append((self.std_off, -1, -1, self.act, 0))
        return rows


def _init_parameters(layout: _Layout, cfg: PPOConfig) -> np.ndarray:
    """Uniform(+-1/sqrt(in)) weights then biases per layer, actor then critic, from one
    ``default_rng(seed)`` stream (ppo.py:313-350, 405-433); std parameter at its initial value."""
    rng = np.random.default_rng(cfg.seed)
    flat = np.zeros(layout.size, np.float32)
    for i, (shape, off) in enumerate(zip(layout.shapes[:-1], layout.offsets[:-1])):
        inp = layout.shapes[i - (i % 2)][1]  # the weight of this (weight, bias) pair
        bound = 1.0 / math.sqrt(inp)
        n = shape[0] * shape[1]
        flat[off:off + n] = rng.uniform(-bound, bound, shape).astype(np.float32).ravel()
    s0 = math.log(cfg.initial_std) if cfg.std_type == "log" else cfg.initial_std
    flat[layout.std_off:] = s0
    return flat


class WarpPPO:
    """Fixed-shape continuous-action PPO with optional shuffled minibatches.

    Call :meth:`act`, step the environment, then :meth:`store` for each rollout step.
    ``next_observations`` passed to ``store`` must be the observations before an
    automatic reset, including terminal observations at timeouts.
    """

    def __init__(self, observation_dim: int, action_dim: int, num_envs: int, horizon: int,
                 config: PPOConfig | None = None, device: str = "cuda"):
        self.config = cfg = config or PPOConfig()
        if cfg.dense_backend not in ("warp", "cuda"):
            raise ValueError("dense_backend must be 'warp' or 'cuda'.")
        if min(observation_dim, action_dim, num_envs, horizon, cfg.epochs, *cfg.hidden_dims) < 1:
            raise ValueError("Dimensions, horizon, and epochs must be positive.")
        if cfg.initial_std <= 0:
            raise ValueError("initial_std must be positive.")
        if cfg.activation not in ("tanh", "elu") or cfg.std_type not in ("log", "scalar"):
            raise ValueError("activation must be 'tanh' or 'elu', and std_type must be 'log' or 'scalar'.")
        if cfg.schedule not in ("fixed", "adaptive") or cfg.desired_kl <= 0:
            raise ValueError("schedule must be 'fixed' or 'adaptive', and desired_kl must be positive.")
        if cfg.timeout_bootstrap not in ("next", "current"):
            raise ValueError("timeout_bootstrap must be 'next' or 'current'.")
        if cfg.std_range[0] <= 0 or cfg.std_range[0] > cfg.std_range[1]:
            raise ValueError("std_range must contain positive increasing bounds.")
        dev = torch.device(device)
        if dev.type != "cuda":
            raise ValueError("WarpPPO requires a CUDA device.")
        if dev.index is None:
            dev = torch.device("cuda", torch.cuda.current_device())
        self.device = dev
        self.num_envs, self.horizon = num_envs, horizon
        self.observation_dim, self.action_dim = observation_dim, action_dim
        self.batch_size = num_envs * horizon
        if cfg.num_mini_batches < 1 or self.batch_size % cfg.num_mini_batches:
            raise ValueError("num_mini_batches must be positive and divide the rollout batch size.")
        if action_dim > 64:
            raise ValueError("the fused PPO loss supports up to 64 actions")
        self.mini_batch_size = self.batch_size // cfg.num_mini_batches
        self.lib = lib = N.load()
        self.layout = lo = _Layout(observation_dim, action_dim, cfg.hidden_dims)
        self._act_fn = ELU if cfg.activation == "elu" else TANH
        self._std_type = int(cfg.std_type == "scalar")
        f32 = dict(dtype=torch.float32, device=dev)
        i32 = dict(dtype=torch.int32, device=dev)
        B, O, A = self.batch_size, observation_dim, action_dim
        # ---- rollout storage (public, as in the reference)
        self.observations = torch.zeros(B, O, **f32)
        self.actions = torch.zeros(B, A, **f32)
        self.means = torch.zeros(B, A, **f32)
        self.stds = torch.zeros(B, A, **f32)
        for name in ("log_probs", "values", "rewards", "next_values", "advantages", "returns"):
            setattr(self, name, torch.zeros(B, **f32))
        self.terminated = torch.zeros(B, **i32)
        self.truncated = torch.zeros(B, **i32)
        # ---- parameters, gradients, Adam moments, weight planes, optimizer state
        self.params = torch.from_numpy(_init_parameters(lo, cfg)).to(dev)
        self.grads = torch.zeros(lo.size, **f32)
        self.m1 = torch.zeros(lo.size, **f32)
        self.m2 = torch.zeros(lo.size, **f32)
        self.plane_hi = torch.zeros(lo.plane_size, **f32)
        self.plane_lo = torch.zeros(lo.plane_size, **f32)
        self.opt_state = torch.zeros(_STATE_FLOATS, **f32)
        self.learning_rate = torch.full((1,), cfg.learning_rate, **f32)
        self._seed = torch.tensor([cfg.seed], dtype=torch.int64, device=dev)  # advanced like the reference's
        segs = lo.segments()
        if max(s[3] for s in segs) > lib.rl2_segment_max_length():
            raise ValueError("a layer is wider than the optimizer's vector limit")
        self._segments, self._segment_count, self._warp_segments = N.segment_table(segs, dev)
        # ---- scalars and reduction workspace (tickets start at zero and are left at zero)
        self.loss = torch.zeros(1, **f32)
        self.metrics = torch.zeros(3, **f32)
        self.kl = torch.zeros(1, **f32)
        self.norms = torch.zeros(5, **f32)
        self.health = torch.zeros(1, **i32)
        self._counters = torch.zeros(8, **i32)
        self._adv_stats = torch.zeros(2, dtype=torch.float64, device=dev)
        self._adv_partials = torch.zeros(lib.rl2_ppo_partials(B), dtype=torch.float64, device=dev)
        self._grad_partials = torch.zeros(3 * lib.rl2_ppo_partials(lo.size), dtype=torch.float64, device=dev)
        self._kl_partials = torch.zeros(lib.rl2_ppo_partials(self.mini_batch_size), dtype=torch.float64, device=dev)
        self._loss_partials = torch.zeros(lib.rl2_ppo_loss_partials(self.mini_batch_size, A), dtype=torch.float64,
                                          device=dev)
        self._perm = torch.arange(B, **i32)
        self._keep: list = []
        self._mb = self._network_buffers(self.mini_batch_size, backward=True)
        self._program = self._build_update_program()
        self._act_bufs = {}
        self._update_graph = None
        self.refresh_weight_planes()

    # ------------------------------------------------------------------ helpers
    def _ctr(self, i: int) -> int:
        return self._counters.data_ptr() + 4 * i

    def parameter(self, i: int) -> torch.Tensor:
        """View of the i-th parameter (reference order)."""
        lo = self.layout
        shape, off = lo.shapes[i], lo.offsets[i]
        return self.params[off:off + int(np.prod(shape))].view(shape)

    @property
    def parameters(self) -> list[torch.Tensor]:
        return [self.parameter(i) for i in range(len(self.layout.shapes))]

    def _view(self, arena: torch.Tensor, i: int) -> torch.Tensor:
        lo = self.layout
        shape, off = lo.shapes[i], lo.offsets[i]
        return arena[off:off + int(np.prod(shape))].view(shape)

    def refresh_weight_planes(self) -> None:
        """Rewrite the tf32 hi/lo weight planes from the fp32 parameters."""
        a = N.AdamArgs(params=self.params.data_ptr(), grads=None, m=None, v=None,
                       segments=self._segments.data_ptr(), count=self._segment_count, state=None, formula=1,
                       beta1=0.9, beta2=0.999, eps=1e-8, project=0, weight_plane=self._weight_plane(),
                       target_params=None, tau=0.0, target_plane=N.Plane(), warp_segments=self._warp_segments)
        N.check(self.lib.rl2_adam_step(ctypes.byref(a), N.stream_ptr()), "refresh weight planes")

    def _weight_plane(self) -> N.Plane:
        return N.Plane(hi=self.plane_hi.data_ptr(), lo=self.plane_lo.data_ptr(), ld=0, twin_stride=0)

    # ------------------------------------------------------------------ buffers
    def _network_buffers(self, rows: int, backward: bool) -> dict:
        lo, dev = self.layout, self.device
        f32 = dict(dtype=torch.float32, device=dev)
        L = lo.layers
        G = (rows + 31) // 32
        ldh = operand_ld(self.action_dim, TF32X3)
        b = {"rows": rows, "G": G, "ldh": ldh,
             "x0": _PlanePair(1, rows, lo.kp[0], dev),
             "y": {i: torch.zeros(2, rows, lo.widths[i], **f32) for i in range(1, L)},
             "head": torch.zeros(2, rows, ldh, **f32)}
        # hidden activations as operands: hi = the fp32 activations themselves (kind::tf32
        # products ignore the low 13 mantissa bits), lo = a separate plane in the same layout
        b["yp"] = {i: _LoPlane(b["y"][i], lo.kp[i]) for i in range(1, L)}
        if backward:
            b["dz"] = {i: _PlanePair(2, rows, lo.kp[i + 1], dev) for i in range(L - 1)}
            b["dz"][L - 1] = _PlanePair(2, rows, ldh, dev)
            b["sums"] = {i: torch.zeros(2, G, lo.widths[i + 1], **f32) for i in range(L - 1)}
            A = self.action_dim
            b["batch"] = {k: torch.zeros(rows, A, **f32) for k in ("actions", "means", "stds")}
            b["batch"].update({k: torch.zeros(rows, **f32)
                               for k in ("log_probs", "values", "advantages", "returns")})
        return b

    def _input_plane(self, b: dict, li: int):
        return b["x0"] if li == 0 else b["yp"][li]

    # ------------------------------------------------------------------ programs
    def _forward_plans(self, b: dict) -> list:
        """Twin-batched layer GEMMs: y = f(x W^T + b) (hidden), head = x W^T + b."""
        lo, rows = self.layout, b["rows"]
        p = self.params.data_ptr()
        plans = []
        for li in range(lo.layers):
            x = self._input_plane(b, li)
            n, k = lo.outs["actor"][li], lo.widths[li]
            last = li == lo.layers - 1
            kw = dict(kind=TF32X3, m=rows, n=n, k=k, batch=2,
                      a=x.hi, a_lo=x.lo, a_major=0, lda=x.ld, a_batch_stride=x.tstride,
                      b=self.plane_hi.data_ptr() + 4 * lo.plane_off[li],
                      b_lo=self.plane_lo.data_ptr() + 4 * lo.plane_off[li], b_major=0, ldb=lo.kp[li],
                      b_batch_stride=n * lo.kp[li],
                      bias=p + 4 * lo.b_off["actor"][li],
                      bias_batch_stride=lo.b_off["critic"][li] - lo.b_off["actor"][li])
            if last:
                kw.update(d=b["head"], ldd=b["ldh"], d_batch_stride=rows * b["ldh"])
            else:
                y, yp = b["y"][li + 1], b["yp"][li + 1]
                kw.update(d=y, ldd=lo.widths[li + 1], d_batch_stride=rows * lo.widths[li + 1],
                          out_plane=yp.c(), activation=self._act_fn)
            plans.append(DensePlan(**kw))
        return plans


    def _split_ws(self, floats: int) -> torch.Tensor:
        ws = getattr(self, "_ws", None)
        if ws is None or ws.numel() < floats:
            self._ws = torch.zeros(floats, dtype=torch.float32, device=self.device)
        return self._ws

    def _dw_plans(self, b: dict, li: int, z_list, m: int) -> list:
        """dW[z] = dz[z]^T x[z] for layer li into the gradient arena (split-K + fixed-order reduce)."""
        lo, rows = self.layout, b["rows"]
        n = lo.widths[li]
        dz, x = b["dz"][li], self._input_plane(b, li)
        batch = len(z_list)
        # long K (24576 rows) over few small tiles: split up to 32 ways to fill the SMs
        tiles = math.ceil(m / 128) * math.ceil(n / min(256, max(32, n))) * batch
        kblocks = math.ceil(rows / 32)
        splits = max(1, min(math.ceil(2 * SM_COUNT / tiles), kblocks // 8, 32))
        count = m * n
        z0 = z_list[0]
        a_hi, a_lo = dz.twin(z0)
        b_hi, b_lo = x.twin(z0)
        common = dict(kind=TF32X3, m=m, n=n, k=rows, batch=batch,
                      a=a_hi, a_lo=a_lo, a_major=1, lda=dz.ld, a_batch_stride=dz.tstride,
                      b=b_hi, b_lo=b_lo, b_major=1, ldb=x.ld, b_batch_stride=x.tstride, ldd=n,
                      d_batch_stride=count)
        nets = ("actor", "critic")
        outs = [self.grads.data_ptr() + 4 * lo.w_off[nets[z]][li] for z in z_list]
        if splits == 1:
            if batch == 2:
                common["d_batch_stride"] = lo.w_off["critic"][li] - lo.w_off["actor"][li]
            return [DensePlan(d=outs[0], **common)]
        ws = self._split_ws(splits * batch * count)
        plan = DensePlan(d=ws, k_splits=splits, d_split_stride=batch * count, **common)
        lib = self.lib

        out_stride = (outs[1] - outs[0]) // 4 if batch == 2 else 0

        def reduce_launch():  # both twins in one launch (their outputs sit a fixed distance apart)
            N.check(lib.rl2_split_reduce_batched(ws.data_ptr(), batch * count, splits, outs[0], count, 0, batch, count,
                                                 out_stride, N.stream_ptr()), "PPO weight-gradient reduce")

        reduce_launch.launches = 1
        return [plan, reduce_launch]

    def _backward_plans(self, b: dict) -> list:
        lo, rows, G = self.layout, b["rows"], b["G"]
        L = lo.layers
        prog = []
        lib = self.lib
        for li in range(L - 1, -1, -1):
            if li == L - 1:  # heads differ in width: one plan per twin
                prog += self._dw_plans(b, li, [0], lo.outs["actor"][li])
                prog += self._dw_plans(b, li, [1], lo.outs["critic"][li])
            else:
                prog += self._dw_plans(b, li, [0, 1], lo.outs["actor"][li])
                sums, C = b["sums"][li], lo.widths[li + 1]
                out = self.grads.data_ptr() + 4 * lo.b_off["actor"][li]
                stride = lo.b_off["critic"][li] - lo.b_off["actor"][li]

                def bias_grad(sums=sums, C=C, out=out, stride=stride):
                    N.check(lib.rl2_colsum_finalize(sums.data_ptr(), 2, G, C, out, stride, 0, N.stream_ptr()),
                            "PPO bias gradient")

                prog.append(bias_grad)
            if li > 0:  # dz[li-1] = (dz[li] W) * f'(y[li]); column sums -> bias gradient of layer li-1
                dz, nxt = b["dz"][li], b["dz"][li - 1]
                n_out = lo.outs["actor"][li]
                w = lo.widths[li]
                prog.append(DensePlan(
                    kind=TF32X3, m=rows, n=w, k=n_out, batch=2,
                    a=dz.hi, a_lo=dz.lo, a_major=0, lda=dz.ld, a_batch_stride=dz.tstride,
                    b=self.plane_hi.data_ptr() + 4 * lo.plane_off[li],
                    b_lo=self.plane_lo.data_ptr() + 4 * lo.plane_off[li], b_major=1, ldb=lo.kp[li],
                    b_batch_stride=n_out * lo.kp[li], d=None, ldd=0, out_plane=nxt.c(),
                    activation=self._act_fn, act_aux=b["y"][li], ld_aux=w, aux_batch_stride=rows * w,
                    stat_mean=b["sums"][li - 1], stat_batch_stride=G * w))
        return prog


    def _returns_program(self) -> list:
        cfg, lib = self.config, self.lib
        g = N.PPOGaeArgs(rewards=self.rewards.data_ptr(), values=self.values.data_ptr(),
                         next_values=self.next_values.data_ptr(), terminated=self.terminated.data_ptr(),
                         truncated=self.truncated.data_ptr(), horizon=self.horizon, num_envs=self.num_envs,
                         gamma=cfg.gamma, gae_lambda=cfg.gae_lambda,
                         current_timeout_bootstrap=int(cfg.timeout_bootstrap == "current"),
                         advantages=self.advantages.data_ptr(), returns=self.returns.data_ptr())
        self._keep.append(g)
        gref = ctypes.byref(g)

        def gae():
            N.check(lib.rl2_ppo_gae(gref, N.stream_ptr()), "PPO GAE")

        prog = [gae]
        if cfg.normalize_advantages:
            def normalize():
                N.check(lib.rl2_ppo_normalize_advantages(
                    self.advantages.data_ptr(), self.batch_size, int(cfg.advantage_sample_std),
                    self._adv_stats.data_ptr(), self._adv_partials.data_ptr(), self._ctr(0), N.stream_ptr()),
                    "PPO advantage normalisation")

            prog.append(normalize)
        return prog

    def _minibatch_program(self, mb: int) -> list:
        cfg, lib, lo = self.config, self.lib, self.layout
        b = self._mb
        rows, A = b["rows"], self.action_dim
        bt = b["batch"]
        shuffled = cfg.num_mini_batches > 1
        ga = N.PPOGatherArgs(indices=self._perm.data_ptr() if shuffled else None, offset=mb * rows, rows=rows,
                             obs_dim=self.observation_dim, act_dim=A, observations=self.observations.data_ptr(),
                             actions=self.actions.data_ptr(), means=self.means.data_ptr(), stds=self.stds.data_ptr(),
                             log_probs=self.log_probs.data_ptr(), values=self.values.data_ptr(),
                             advantages=self.advantages.data_ptr(), returns=self.returns.data_ptr(),
                             obs_plane=b["x0"].c(), batch_actions=bt["actions"].data_ptr(),
                             batch_means=bt["means"].data_ptr() if cfg.schedule == "adaptive" else None,
                             batch_stds=bt["stds"].data_ptr() if cfg.schedule == "adaptive" else None,
                             batch_log_probs=bt["log_probs"].data_ptr(), batch_values=bt["values"].data_ptr(),
                             batch_advantages=bt["advantages"].data_ptr(), batch_returns=bt["returns"].data_ptr())
        self._keep.append(ga)
        gref = ctypes.byref(ga)

        def gather():
            N.check(lib.rl2_ppo_gather(gref, N.stream_ptr()), "PPO gather")

        prog = [gather] + self._forward_plans_cached(b)
        p = self.params.data_ptr()
        if cfg.schedule == "adaptive":
            def kl():
                N.check(lib.rl2_ppo_kl(b["head"].data_ptr(), b["ldh"], p + 4 * lo.std_off, bt["means"].data_ptr(),
                                       bt["stds"].data_ptr(), rows, A, self._std_type, cfg.std_range[0],
                                       cfg.std_range[1], cfg.desired_kl, self.kl.data_ptr(),
                                       self.learning_rate.data_ptr(), self._kl_partials.data_ptr(), self._ctr(1),
                                       N.stream_ptr()), "PPO KL schedule")

            prog.append(kl)
        g = self.grads.data_ptr()
        la = N.PPOLossArgs(
            head=b["head"].data_ptr(), ld_head=b["ldh"], head_twin_stride=rows * b["ldh"], std_param=p + 4 * lo.std_off,
            rows=rows, act=A, actions=bt["actions"].data_ptr(), old_log_probs=bt["log_probs"].data_ptr(),
            old_values=bt["values"].data_ptr(), advantages=bt["advantages"].data_ptr(),
            returns=bt["returns"].data_ptr(), clip_ratio=cfg.clip_ratio, value_coefficient=cfg.value_coefficient,
            entropy_coefficient=cfg.entropy_coefficient, value_loss_scale=cfg.value_loss_scale,
            clip_value=int(cfg.clip_value), std_type=self._std_type, std_min=cfg.std_range[0],
            std_max=cfg.std_range[1], loss=self.loss.data_ptr(), metrics=self.metrics.data_ptr(), d_head=None,
            ld_d_head=b["ldh"], d_head_twin_stride=rows * b["ldh"], d_plane=b["dz"][lo.layers - 1].c(),
            d_bias_actor=g + 4 * lo.b_off["actor"][lo.layers - 1],
            d_bias_critic=g + 4 * lo.b_off["critic"][lo.layers - 1], d_std_param=g + 4 * lo.std_off,
            partials=self._loss_partials.data_ptr(), counter=self._ctr(2))
        self._keep.append(la)
        lref = ctypes.byref(la)

        def loss():
            N.check(lib.rl2_ppo_loss(lref, N.stream_ptr()), "PPO loss")

        prog.append(loss)
        prog += self._backward_plans_cached(b)
        na, nc = lo.actor_size, lo.critic_size

        def clip():
            N.check(lib.rl2_ppo_clip_gradients(g, na, nc, A, int(cfg.separate_grad_clipping), cfg.max_grad_norm,
                                               self.norms.data_ptr(), self._grad_partials.data_ptr(), self._ctr(3),
                                               N.stream_ptr()), "PPO gradient clipping")

        prog += [clip] + self._optimizer_program()
        return prog

    def _forward_plans_cached(self, b: dict) -> list:
        if "fwd" not in b:
            b["fwd"] = self._forward_plans(b)
        return b["fwd"]

    def _backward_plans_cached(self, b: dict) -> list:
        if "bwd" not in b:
            b["bwd"] = self._backward_plans(b)
        return b["bwd"]

    def _optimizer_program(self) -> list:
        if hasattr(self, "_opt_prog"):
            return self._opt_prog
        lib = self.lib
        prep = N.AdamPrepareArgs(state=self.opt_state.data_ptr(), found_inf=None, formula=1, beta1=0.9, beta2=0.999,
                                 lr_init=self.config.learning_rate, lr_peak=self.config.learning_rate,
                                 lr_end=self.config.learning_rate, warmup_steps=0.0, decay_steps=1.0,
                                 schedule_on_attempts=0, lr_override=self.learning_rate.data_ptr(), scaler=0,
                                 growth=2.0, backoff=0.5, growth_interval=2000, scale_out=None, inv_scale_out=None)
        step = N.AdamArgs(params=self.params.data_ptr(), grads=self.grads.data_ptr(), m=self.m1.data_ptr(),
                          v=self.m2.data_ptr(), segments=self._segments.data_ptr(), count=self._segment_count,
                          state=self.opt_state.data_ptr(), formula=1, beta1=0.9, beta2=0.999, eps=1e-8, project=0,
                          weight_plane=self._weight_plane(), target_params=None, tau=0.0, target_plane=N.Plane(),
                          warp_segments=self._warp_segments)
        self._keep += [prep, step]
        pref, sref = ctypes.byref(prep), ctypes.byref(step)

        def adam():
            s = N.stream_ptr()
            N.check(lib.rl2_adam_prepare(pref, s), "PPO Adam prepare")
            N.check(lib.rl2_adam_step(sref, s), "PPO Adam step")

        adam.launches = 2
        self._opt_prog = [adam]
        return self._opt_prog

    def _build_update_program(self) -> list:
        cfg, lib = self.config, self.lib
        prog = self._returns_program()
        if cfg.num_mini_batches > 1:
            seed = (cfg.seed * 0x9E3779B97F4A7C15 + 53) & 0xFFFFFFFFFFFFFFFF

            def shuffle():
                s = N.stream_ptr()
                N.check(lib.rl2_counter_advance(self._seed.data_ptr(), 1, s), "PPO seed advance")
                N.check(lib.rl2_ppo_permutation(seed, self._seed.data_ptr(), self.batch_size, self._perm.data_ptr(),
                                                self.health.data_ptr(), s), "PPO permutation")

            shuffle.launches = 2
            prog.append(shuffle)
        per_mb = [self._minibatch_program(mb) for mb in range(cfg.num_mini_batches)]
        for _ in range(cfg.epochs):
            for mb_prog in per_mb:
                prog += mb_prog
        return prog

    # ------------------------------------------------------------------ public update API
    def compute_returns(self) -> None:
        """Compute GAE, preserving timeout bootstraps and stopping traces at all resets."""
        for f in self._returns_program_cached():
            f()

    def _returns_program_cached(self) -> list:
        if not hasattr(self, "_ret_prog"):
            self._ret_prog = self._returns_program()
        return self._ret_prog

    def launch_update(self) -> None:
        """Launch the entire PPO update (capturable): returns, shuffle, epochs x minibatches."""
        for f in self._program:
            f()

    def warmup(self) -> None:
        """Load every kernel without changing the optimizer state or parameters."""
        state = self.state_dict()
        saved = {k: getattr(self, k).clone() for k in ("advantages", "returns")}
        self.launch_update()
        self.load_state_dict(state)
        for k, v in saved.items():
            getattr(self, k).copy_(v)

    def update(self, capture: bool = True) -> None:
        """Execute one complete update, capturing and replaying it as a CUDA graph by default."""
        if not capture:
            self.launch_update()
            return
        if self._update_graph is None:
            self.warmup()
            graph = torch.cuda.CUDAGraph()
            stream = torch.cuda.Stream(device=self.device)
            stream.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(stream), torch.cuda.graph(graph, stream=stream):
                self.launch_update()
            torch.cuda.current_stream(self.device).wait_stream(stream)
            self._update_graph = graph
        self._update_graph.replay()

    def launch_count(self) -> int:
        """Kernel launches of one update (every DensePlan / helper counted by its launches)."""
        return sum(getattr(f, "launches", 1) for f in self._program)


    # ------------------------------------------------------------------ rollout API
    def _rollout_bufs(self, name: str) -> dict:
        if name not in self._act_bufs:
            b = self._network_buffers(self.num_envs, backward=False)
            b["obs"] = torch.zeros(self.num_envs, self.observation_dim, dtype=torch.float32, device=self.device)
            self._forward_plans_cached(b)
            self._act_bufs[name] = b
        return self._act_bufs[name]

    def _forward(self, b: dict, observations) -> None:
        obs = torch.as_tensor(observations, dtype=torch.float32, device=self.device)
        b["obs"].copy_(obs.reshape(self.num_envs, self.observation_dim))
        ga = N.PPOGatherArgs(indices=None, offset=0, rows=self.num_envs, obs_dim=self.observation_dim, act_dim=0,
                             observations=b["obs"].data_ptr(), obs_plane=b["x0"].c())
        N.check(self.lib.rl2_ppo_gather(ctypes.byref(ga), N.stream_ptr()), "PPO observation planes")
        for f in b["fwd"]:
            f()

    def act(self, observations, deterministic: bool = False) -> torch.Tensor:
        """Return raw Gaussian actions in a reusable tensor (ppo.py:482-503)."""
        lib, cfg, A = self.lib, self.config, self.action_dim
        b = self._rollout_bufs("act")
        if "actions" not in b:
            f32 = dict(dtype=torch.float32, device=self.device)
            b["actions"] = torch.zeros(self.num_envs, A, **f32)
            b["log_probs"] = torch.zeros(self.num_envs, **f32)
            b["values"] = torch.zeros(self.num_envs, **f32)
            b["noise"] = torch.zeros(self.num_envs, A, **f32)
            b["sampled_std"] = torch.zeros(A, **f32)
        s = N.stream_ptr()
        N.check(lib.rl2_counter_advance(self._seed.data_ptr(), 1, s), "PPO seed advance")
        self._forward(b, observations)
        if not deterministic:
            seed = (cfg.seed * 0x9E3779B97F4A7C15 + 71) & 0xFFFFFFFFFFFFFFFF
            N.check(lib.rl2_normal_noise(seed, self._seed.data_ptr(), self.num_envs, A, b["noise"].data_ptr(), A, s),
                    "PPO action noise")
        sa = N.PPOSampleArgs(head=b["head"].data_ptr(), ld_head=b["ldh"], head_twin_stride=self.num_envs * b["ldh"],
                             std_param=self.params.data_ptr() + 4 * self.layout.std_off, std_type=self._std_type,
                             std_min=cfg.std_range[0], std_max=cfg.std_range[1],
                             noise=None if deterministic else b["noise"].data_ptr(), rows=self.num_envs, act=A,
                             actions=b["actions"].data_ptr(), log_probs=b["log_probs"].data_ptr(),
                             values=b["values"].data_ptr(), sampled_std=b["sampled_std"].data_ptr())
        N.check(lib.rl2_ppo_sample(ctypes.byref(sa), s), "PPO sample")
        return b["actions"]

    def store(self, step: int, observations, rewards, terminated, truncated, next_observations) -> None:
        """Store the last sampled action and bootstrap from the pre-reset next observation."""
        if not 0 <= step < self.horizon:
            raise ValueError("step must be within the rollout horizon.")
        if "act" not in self._act_bufs or "actions" not in self._act_bufs["act"]:
            raise RuntimeError("store() needs a preceding act()")
        a, nb = self._act_bufs["act"], self._rollout_bufs("next")
        self._forward(nb, next_observations)
        dev = self.device
        obs = a["obs"]  # store the observations the last act() saw unless new ones are given
        if observations is not None:
            obs = torch.as_tensor(observations, dtype=torch.float32, device=dev).reshape(self.num_envs, -1).contiguous()
        rew = torch.as_tensor(rewards, dtype=torch.float32, device=dev).reshape(-1).contiguous()
        term = torch.as_tensor(terminated, device=dev).reshape(-1).to(torch.int32).contiguous()
        trunc = torch.as_tensor(truncated, device=dev).reshape(-1).to(torch.int32).contiguous()
        st = N.PPOStoreArgs(
            step=step, num_envs=self.num_envs, obs_dim=self.observation_dim, act=self.action_dim,
            observations=obs.data_ptr(), actions=a["actions"].data_ptr(), log_probs=a["log_probs"].data_ptr(),
            values=a["values"].data_ptr(), rewards=rew.data_ptr(), terminated=term.data_ptr(), truncated=trunc.data_ptr(),
            mean=a["head"].data_ptr(), ld_mean=a["ldh"], next_values=nb["head"].data_ptr() + 4 * self.num_envs * nb["ldh"],
            next_values_stride=nb["ldh"], sampled_std=a["sampled_std"].data_ptr(),
            r_observations=self.observations.data_ptr(), r_actions=self.actions.data_ptr(),
            r_log_probs=self.log_probs.data_ptr(), r_values=self.values.data_ptr(), r_rewards=self.rewards.data_ptr(),
            r_terminated=self.terminated.data_ptr(), r_truncated=self.truncated.data_ptr(),
            r_next_values=self.next_values.data_ptr(), r_means=self.means.data_ptr(), r_stds=self.stds.data_ptr())
        N.check(self.lib.rl2_ppo_store(ctypes.byref(st), N.stream_ptr()), "PPO store")

    # ------------------------------------------------------------------ diagnostics / checkpoints
    def health_metrics(self) -> dict[str, float]:
        """Distribution and optimizer diagnostics (synchronises; ppo.py:697-725)."""
        cfg = self.config
        param = self.parameter(len(self.layout.shapes) - 1).detach().cpu().numpy()
        std = np.clip(param, *cfg.std_range) if cfg.std_type == "scalar" else np.exp(param)
        m = self.metrics.cpu().numpy()
        res = {"std_min": float(std.min()), "std_mean": float(std.mean()), "std_max": float(std.max()),
               "std_parameter_min": float(param.min()), "std_parameter_max": float(param.max()),
               "learning_rate": float(self.learning_rate.cpu()[0]), "kl": float(self.kl.cpu()[0]),
               "policy_loss": float(m[0]), "value_loss": float(m[1]), "entropy": float(m[2]),
               "optimizer_updates": float(self.opt_state[1].cpu())}
        if cfg.separate_grad_clipping:
            n = self.norms.cpu().numpy()
            res["actor_grad_norm"] = float(np.sqrt(n[0]))
            res["critic_grad_norm"] = float(np.sqrt(n[1]))
        return res

    def state_dict(self) -> dict[str, np.ndarray]:
        """Model, Adam and sampling state as numpy arrays (synchronises)."""
        n = len(self.layout.shapes)
        state = {f"parameter_{i}": self._view(self.params, i).cpu().numpy() for i in range(n)}
        state.update({f"adam_m1_{i}": self._view(self.m1, i).cpu().numpy() for i in range(n)})
        state.update({f"adam_m2_{i}": self._view(self.m2, i).cpu().numpy() for i in range(n)})
        state["adam_timestep"] = self.opt_state[1:2].cpu().numpy().astype(np.float32)
        state["adam_lr"] = self.learning_rate.cpu().numpy().astype(np.float32)
        state["seed"] = self._seed.cpu().numpy().astype(np.int32)
        return state

    def load_state_dict(self, state: dict[str, np.ndarray]) -> None:
        """Restore in place so captured graphs keep valid pointers."""
        n = len(self.layout.shapes)
        keys = {f"{p}_{i}" for p in ("parameter", "adam_m1", "adam_m2") for i in range(n)}
        keys |= {"adam_timestep", "adam_lr", "seed"}
        if set(state) != keys:
            raise ValueError("Checkpoint parameter or optimizer keys do not match this model.")
        for i in range(n):
            for p in ("parameter", "adam_m1", "adam_m2"):
                if tuple(np.shape(state[f"{p}_{i}"])) != tuple(self.layout.shapes[i]):
                    raise ValueError(f"Checkpoint shape for {p}_{i} does not match this model.")
        for k in ("adam_timestep", "adam_lr", "seed"):
            if np.shape(state[k]) != (1,):
                raise ValueError(f"Checkpoint shape for {k} does not match this model.")
        for i in range(n):
            for p, arena in (("parameter", self.params), ("adam_m1", self.m1), ("adam_m2", self.m2)):
                self._view(arena, i).copy_(torch.as_tensor(np.asarray(state[f"{p}_{i}"], np.float32)))
        self.opt_state.zero_()
        self.opt_state[1] = float(state["adam_timestep"][0])
        self.opt_state[0] = float(state["adam_timestep"][0])
        self.learning_rate.fill_(float(state["adam_lr"][0]))
        self._seed.fill_(int(state["seed"][0]))
        self.refresh_weight_planes()

    def save(self, path: str | Path) -> None:
        """Save model and optimizer state to an NPZ checkpoint."""
        with Path(path).open("wb") as f:
            np.savez(f, **self.state_dict())

    def load(self, path: str | Path) -> None:
        """Load an NPZ checkpoint into a model with the same architecture."""
        with np.load(path, allow_pickle=False) as state:
            self.load_state_dict(dict(state))


class _LoPlane:
    """tf32 operand [2][rows][ld] whose hi part is an fp32 array of that layout (the tensor
    cores read raw fp32 as tf32 by ignoring the low mantissa bits); only lo is stored."""

    def __init__(self, values: torch.Tensor, ld: int):
        twins, rows, width = values.shape
        if width != ld:
            raise ValueError("the fp32 activations must have the operand row stride")
        self.twins, self.rows, self.ld = twins, rows, ld
        self.values = values
        self.lo_t = torch.zeros_like(values)
        self.hi, self.lo = values.data_ptr(), self.lo_t.data_ptr()
        self.tstride = rows * ld

    def c(self) -> N.Plane:
        return N.Plane(lo=self.lo, ld=self.ld, twin_stride=self.rows * self.ld)

    def twin(self, z: int) -> tuple[int, int]:
        off = 4 * z * self.rows * self.ld
        return self.hi + off, self.lo + off

    def value(self) -> torch.Tensor:
        hi = (self.values.view(torch.int32) & -8192).view(torch.float32)
        return hi + self.lo_t


class _PlanePair:
    """tf32 hi / lo operand planes [twins][rows][ld] (twins == 1: shared by both twins)."""

    def __init__(self, twins: int, rows: int, ld: int, device):
        self.twins, self.rows, self.ld = twins, rows, ld
        self.hi_t = torch.zeros(twins, rows, ld, dtype=torch.float32, device=device)
        self.lo_t = torch.zeros(twins, rows, ld, dtype=torch.float32, device=device)
        self.hi, self.lo = self.hi_t.data_ptr(), self.lo_t.data_ptr()
        self.tstride = rows * ld if twins > 1 else 0

    def c(self) -> N.Plane:
        return N.Plane(hi=self.hi, lo=self.lo, ld=self.ld, twin_stride=self.rows * self.ld)

    def twin(self, z: int) -> tuple[int, int]:
        off = 4 * z * self.rows * self.ld if self.twins > 1 else 0
        return self.hi + off, self.lo + off

    def value(self) -> torch.Tensor:
        return self.hi_t + self.lo_t
