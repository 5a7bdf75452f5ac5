"""One FlashSAC learner update as a fixed launch program over persistent buffers.

Order and semantics follow ``_update_networks`` (``src/robolearn/flashsac/agent.py:217-281``)
and the Warp learner's ``launch_update`` (``src/robolearn/warp/flashsac.py:880-938``):

actor phase (every ``actor_update_period`` updates)
    actor forward (training, current || next observations) -> tanh-Gaussian sample ->
    frozen critic forward (evaluation BN) on (obs, policy action) -> actor objective ->
    critic backward to the action input -> policy backward -> actor backward ->
    fused Adam / projection / plane refresh -> temperature step
critic phase (every update)
    actor forward (evaluation) on next observations -> next action / log pi ->
    target critic forward (training BN, moves target running statistics) ->
    online critic forward (training) -> fused categorical projection + CE + gradient ->
    critic backward -> fused Adam / projection / plane refresh / target EMA.

All launches go to the current torch stream; ``Learner.capture`` records each phase
as a CUDA graph so one update is one or two graph launches.
"""

from __future__ import annotations

import ctypes
import math

import numpy as np
import torch

from .. import _native as N
from ..categorical import CriticObjective, support
from ..dense import FP16, TF32X3
from .config import FlashSACConfig
from .engine import Net, PlaneBuf, Run, Scaler, Spec, _a4

METRIC_KEYS = (
    "actor/loss",
    "actor/entropy",
    "actor/mean_action",
    "critic/loss",
    "critic/max_entropy_bonus",
    "temperature/value",
    "temperature/loss",
)


def _init_reference_weights(obs_a: int, obs_c: int, act: int, cfg: FlashSACConfig) -> tuple[dict, dict, float]:
    """Initial parameters drawn exactly as the reference constructs its networks.

    ``torch.manual_seed(cfg.seed)`` then, in module construction order, every
    ``UnitLinear`` draws ``nn.Linear``'s default init and then ``orthogonal_``
    (``layers.py:15-20``), every ``EnsembleUnitLinear`` draws ``orthogonal_`` per
    member (``layers.py:174-180``); finally both networks are weight-projected
    (``agent.py:151-154``). Runs on the host once at construction.
    """
    import torch.nn as nn
    import torch.nn.functional as F

    gen_state = torch.random.get_rng_state()
    torch.manual_seed(cfg.seed)

    def unit_linear(inp, out):
        lin = nn.Linear(inp, out, bias=False)
        nn.init.orthogonal_(lin.weight, gain=1)
        return lin.weight.detach().clone()

    def ensemble(n, inp, out):
        w = torch.empty(n, out, inp)
        for i in range(n):
            nn.init.orthogonal_(w[i], gain=1)
        return w

    H, E = cfg.actor_hidden_dim, 4 * cfg.actor_hidden_dim
    actor = {"embedder.norm.weight": torch.ones(obs_a), "embedder.norm.bias": torch.zeros(obs_a)}
    actor["embedder.w.w.weight"] = unit_linear(obs_a, H)
    for i in range(cfg.actor_num_blocks):
        actor[f"encoder.{i}.w1.w.weight"] = unit_linear(H, E)
        actor[f"encoder.{i}.w2.w.weight"] = unit_linear(E, H)
        actor[f"encoder.{i}.norm1.weight"] = torch.ones(E)
        actor[f"encoder.{i}.norm1.bias"] = torch.zeros(E)
        actor[f"encoder.{i}.norm2.weight"] = torch.ones(H)
        actor[f"encoder.{i}.norm2.bias"] = torch.zeros(H)
    actor["post_norm.weight"] = torch.ones(H)
    actor["predictor.mean_w.w.weight"] = unit_linear(H, act)
    actor["predictor.mean_bias"] = torch.zeros(act)
    actor["predictor.std_w.w.weight"] = unit_linear(H, act)
    actor["predictor.std_bias"] = torch.zeros(act)
    Hc, Ec, cin = cfg.critic_hidden_dim, 4 * cfg.critic_hidden_dim, obs_c + act
    critic = {"embedder.norm.weight": torch.ones(2, cin), "embedder.norm.bias": torch.zeros(2, cin)}
    critic["embedder.w.weight"] = ensemble(2, cin, Hc)
    for i in range(cfg.critic_num_blocks):
        critic[f"encoder.{i}.w1.weight"] = ensemble(2, Hc, Ec)
        critic[f"encoder.{i}.w2.weight"] = ensemble(2, Ec, Hc)
        critic[f"encoder.{i}.norm1.weight"] = torch.ones(2, Ec)
        critic[f"encoder.{i}.norm1.bias"] = torch.zeros(2, Ec)
        critic[f"encoder.{i}.norm2.weight"] = torch.ones(2, Hc)
        critic[f"encoder.{i}.norm2.bias"] = torch.zeros(2, Hc)
    critic["post_norm.weight"] = torch.ones(2, Hc)
    critic["predictor.w.weight"] = ensemble(2, Hc, cfg.critic_num_bins)
    critic["predictor.bias"] = torch.zeros(2, cfg.critic_num_bins)
    torch.random.set_rng_state(gen_state)

    def project(params):
        out = {}
        for k, v in params.items():
            if k == "post_norm.weight":
                out[k] = v * (math.sqrt(v.shape[-1]) * torch.rsqrt((v * v).sum(-1, keepdim=True) + 1e-8))
            elif k.endswith("norm.weight") or "norm1.weight" in k or "norm2.weight" in k:
                b = params[k[: -len("weight")] + "bias"]
                f = math.sqrt(v.shape[-1]) * torch.rsqrt((v * v + b * b).sum(-1, keepdim=True) + 1e-8)
                out[k], out[k[: -len("weight")] + "bias"] = v * f, b * f
            elif k.endswith("weight") and "norm" not in k:
                out[k] = F.normalize(v, dim=-1, eps=1e-8)
            elif k not in out:
                out[k] = v
        return out

    return project(actor), project(critic), math.log(cfg.temp_initial_value)


class Learner:
    """Device state and launch programs of one FlashSAC learner."""

    def __init__(self, obs_a: int, obs_c: int, act: int, cfg: FlashSACConfig, device, *, adam_formula: int = 0,
                 init_weights: bool = True, init_loss_scale: float = 65536.0, dp=None):
        """``cfg.sample_batch_size`` is this rank's batch; with ``dp`` (a ``DataParallel``) the
        update runs on the global batch of all ranks (batch-norm statistics, gradients and
        the temperature's entropy exchanged; see ``dp.py``)."""
        self.cfg = cfg
        self.dp = dp if (dp is not None and dp.world > 1) else None
        self.device = device = torch.device(device)
        self.obs_a, self.obs_c, self.act = obs_a, obs_c, act
        self.kind = FP16 if cfg.precision == "fp16" else TF32X3
        self.adam_formula = adam_formula
        B = self.B = cfg.sample_batch_size
        bins = cfg.critic_num_bins
        if bins > 128:
            raise ValueError("the fused categorical kernels support up to 128 atoms")
        self.target_entropy = cfg.temp_target_entropy
        if self.target_entropy is None:
            self.target_entropy = 0.5 * act * math.log(2 * math.pi * math.e * cfg.temp_target_sigma**2)
        a_spec = Spec(1, obs_a, cfg.actor_hidden_dim, cfg.actor_num_blocks, 2 * act, actor_act=act)
        c_spec = Spec(2, obs_c + act, cfg.critic_hidden_dim, cfg.critic_num_blocks, bins)
        self.actor = Net(a_spec, self.kind, device)
        self.critic = Net(c_spec, self.kind, device)
        self.target = Net(c_spec, self.kind, device, with_optimizer=False)
        f32 = dict(dtype=torch.float32, device=device)
        self.log_temp = torch.zeros(1, **f32)
        self.temp_state = torch.zeros(3, **f32)  # [step, m, v]
        if init_weights:
            a0, c0, lt = _init_reference_weights(obs_a, obs_c, act, cfg)
            self.actor.load_state_dict(a0)
            self.critic.load_state_dict(c0)
            self.target.load_state_dict(c0)
            self.log_temp.fill_(lt)
        # ---- scalers (fp16 recipe): dynamic loss scale per optimised network
        self.scalers = {}
        for name, net in (("actor", self.actor), ("critic", self.critic)):
            if self.kind == FP16:
                # GradScaler defaults: initial scale 2^16, x2 after 2000 clean steps, x0.5 on overflow
                sc = Scaler(torch.full((1,), init_loss_scale, **f32), torch.full((1,), 1.0 / init_loss_scale, **f32),
                            torch.zeros(1, dtype=torch.int32, device=device))
                net.opt_state[6] = init_loss_scale
            else:
                sc = Scaler(found_inf=torch.zeros(1, dtype=torch.int32, device=device))
            self.scalers[name] = sc
        # ---- batch buffers (network layouts)
        cin = obs_c + act
        self.ldx = _a4(cin)
        self.ldax = _a4(obs_a)
        self.critic_x = torch.zeros(2 * B, self.ldx, **f32)
        self.critic_x_pi = torch.zeros(2 * B, self.ldx, **f32)
        self.actor_x = torch.zeros(2 * B, self.ldax, **f32)
        self.reward = torch.zeros(B, **f32)
        self.terminated = torch.zeros(B, **f32)
        self.truncated = torch.zeros(B, **f32)
        self.discount = torch.zeros(B, **f32)
        self.actor_noise = torch.zeros(2 * B, act, **f32)
        self.next_noise = torch.zeros(B, act, **f32)
        self.log_pi = torch.zeros(2 * B, **f32)
        self.next_log_pi = torch.zeros(B, **f32)
        self.alpha = torch.zeros(1, **f32)
        self.metrics = torch.zeros(len(METRIC_KEYS), **f32)
        self.scratch = torch.zeros(8, **f32)  # [q_abs, d_log_pi, ...]
        self.health = torch.zeros(1, dtype=torch.int32, device=device)
        # data parallel: gradient suffixes are averaged on this stream during the backward
        self._grad_stream = torch.cuda.Stream(device) if (self.dp is not None and device.type == "cuda") else None
        self.counters = torch.zeros(4, dtype=torch.int64, device=device)  # [noise epoch, ...]
        self.noise_epoch = torch.zeros(1, dtype=torch.int64, device=device)
        self.support = torch.from_numpy(support(bins, cfg.critic_min_v, cfg.critic_max_v)).to(device)
        self.bias_part = torch.zeros((2 * B + 31) // 32, 2 * act, **f32)
        lib = N.load()
        self.lib = lib
        self.actor_ws = torch.zeros(lib.rl2_actor_objective_workspace_floats(B), **f32)
        self.counter = torch.zeros(2, dtype=torch.int32, device=device)
        self.objective = CriticObjective(B, bins, cfg.critic_min_v, cfg.critic_max_v, device=device)
        # ---- backbone runs
        if self.dp is not None and self.dp.peer is None:
            # one peer-exchange slot per batch-norm sync point: forward + backward of the
            # actor and online critic, forward of the target critic
            # (plus slots for the scalar reductions of the phase programs)
            la, lc = self.actor.bn_layers, self.critic.bn_layers
            self.dp.enable_peer(device, 2 * len(la) + 3 * len(lc) + 16, max([32] + [C for _, C in la + lc]),
                                self.health.data_ptr())
            # gradient arenas in symmetric memory: one peer-memory mean per optimizer step
            self.dp.enable_peer_gradients([self.actor, self.critic], device, self.health.data_ptr())
        pa, pa_eval, pc, pc_eval = {}, {}, {}, {}
        sa, scc = self.scalers["actor"], self.scalers["critic"]
        self.actor_train = Run(self.actor, 2 * B, True, self.actor_x.data_ptr(), self.ldax, update_running=True,
                               need_param_grads=True, need_input_grad=False, scaler=sa, pool=pa, dp=self.dp)
        self.actor_next = Run(self.actor, B, False, self.actor_x.data_ptr() + 4 * B * self.ldax, self.ldax,
                              update_running=False, need_param_grads=False, need_input_grad=False, pool=pa_eval)
        self.critic_pi = Run(self.critic, B, False, self.critic_x_pi.data_ptr(), self.ldx, update_running=False,
                             need_param_grads=False, need_input_grad=True, scaler=sa, pool=pc_eval)
        self.target_run = Run(self.target, 2 * B, True, self.critic_x.data_ptr(), self.ldx, update_running=True,
                              need_param_grads=False, need_input_grad=False, pool=pc, dp=self.dp)
        pc_online = {k: v for k, v in pc.items() if k != "out"}
        self.critic_run = Run(self.critic, 2 * B, True, self.critic_x.data_ptr(), self.ldx, update_running=True,
                              need_param_grads=True, need_input_grad=False, scaler=scc, pool=pc_online, dp=self.dp)
        self.graphs = {}
        self._extra_programs = {}
        self.programs = {True: self._program(True), False: self._program(False)}

    # ------------------------------------------------------------------
    def _policy_args(self, run: Run, rows: int, noise: torch.Tensor, actions_addr: int, ld_actions: int,
                     log_pi: torch.Tensor) -> N.PolicyArgs:
        return N.PolicyArgs(head=run.out.data_ptr(), ld_head=run.head_ld, noise=noise.data_ptr(), ld_noise=self.act,
                            rows=rows, act=self.act, actions=actions_addr, ld_actions=ld_actions,
                            log_pi=log_pi.data_ptr())

    def _backward_with_exchange(self, run: Run, net: Net, apply_optimizer: bool):
        """The run's backward launches; with data parallelism and an optimizer step, each
        finished suffix of the gradient arena is averaged over the ranks on a side stream
        while the earlier layers' backward continues. Returns (launches, prefix end): the
        gradients below the prefix end are left to the optimizer launch."""
        prog = list(run.backward_program)
        dp = self.dp
        if dp is None or not apply_optimizer or not dp.nccl or not run.grad_marks or self._peer_mean(net):
            return prog, net.size
        side = self._grad_stream
        out, hi = [], net.size
        marks = dict(run.grad_marks)
        for i, f in enumerate(prog):
            out.append(f)
            if i + 1 in marks:
                lo = marks[i + 1]

                def bucket(lo=lo, hi=hi):
                    side.wait_stream(torch.cuda.current_stream())
                    with torch.cuda.stream(side):
                        dp.all_reduce_mean(net.grads[lo:hi])

                bucket.launches = 0
                out.append(bucket)
                hi = lo
        return out, hi

    def _peer_mean(self, net: Net) -> bool:
        """Whether ``net``'s gradients are averaged by the peer-memory kernel (whole arena,
        once, just before the optimizer step)."""
        dp = self.dp
        return dp is not None and dp.peer_grads is not None and dp.peer_grads.holds(net)

    def _optimizer(self, name: str, net: Net, target: Net | None = None, prefix: int | None = None):
        """Fused optimizer pass; under data parallelism the gradients are averaged first
        (only [0, prefix) here when the backward already averaged the rest on the side stream)."""
        cfg, lib = self.cfg, self.lib
        sc = self.scalers[name]
        prep = N.AdamPrepareArgs(
            state=net.opt_state.data_ptr(), found_inf=N.addr(sc.found_inf), formula=self.adam_formula,
            beta1=0.9, beta2=0.999, lr_init=cfg.learning_rate_init, lr_peak=cfg.learning_rate_peak,
            lr_end=cfg.learning_rate_end, warmup_steps=float(cfg.learning_rate_warmup_step),
            decay_steps=float(cfg.learning_rate_decay_step), schedule_on_attempts=1, lr_override=None,
            scaler=int(self.kind == FP16), growth=2.0, backoff=0.5, growth_interval=2000,
            scale_out=N.addr(sc.scale), inv_scale_out=N.addr(sc.inv_scale))
        step = N.AdamArgs(
            params=net.params.data_ptr(), grads=net.grads.data_ptr(), m=net.m.data_ptr(), v=net.v.data_ptr(),
            segments=net.segments.data_ptr(), count=net.segment_count, state=net.opt_state.data_ptr(),
            formula=self.adam_formula, beta1=0.9, beta2=0.999, eps=1e-8, project=1, weight_plane=net.plane_c(),
            target_params=target.params.data_ptr() if target is not None else None,
            tau=cfg.critic_target_update_tau if target is not None else 0.0,
            target_plane=target.plane_c() if target is not None else N.Plane(),
            warp_segments=net.warp_segment_count)
        pref, sref = ctypes.byref(prep), ctypes.byref(step)
        dp = self.dp
        # skip the step on any rank's overflow
        flags = dp.scalar_reducer(max_int=sc.found_inf) if (
            dp is not None and sc.found_inf is not None and self.kind == FP16) else None
        mean = dp.gradient_mean(net) if self._peer_mean(net) else None

        def launch():
            if mean is not None:
                mean()
                if flags is not None:
                    flags()
            elif dp is not None:  # average the gradients of all ranks
                if prefix is not None and prefix < net.size:
                    torch.cuda.current_stream().wait_stream(self._grad_stream)
                    if prefix > 0:
                        dp.all_reduce_mean(net.grads[:prefix])
                else:
                    dp.all_reduce_mean(net.grads)
                if flags is not None:
                    flags()
            N.check(lib.rl2_adam_prepare(pref, N.stream_ptr()), f"{name} adam prepare")
            N.check(lib.rl2_adam_step(sref, N.stream_ptr()), f"{name} adam step")

        launch.keep = (prep, step, flags, mean)
        launch.launches = 2 + (flags.launches if flags is not None else 0) + (mean.launches if mean is not None else 0)
        return launch

    def _program(self, actor_phase: bool, apply_optimizer: bool = True):
        """Launch list of one phase; ``apply_optimizer=False`` stops after the gradients
        (no Adam / projection / EMA / temperature step), for diagnostics."""
        cfg, lib, B, A = self.cfg, self.lib, self.B, self.act
        prog = []
        m = self.metrics.data_ptr()
        mi = {k: m + 4 * i for i, k in enumerate(METRIC_KEYS)}
        s = self.scratch.data_ptr()
        q_abs_addr, dlp_addr = s, s + 4
        if actor_phase:
            prog += self.actor_train.forward_program
            pa = self._policy_args(self.actor_train, 2 * B, self.actor_noise, self.critic_x_pi.data_ptr() + 4 * self.obs_c,
                                   self.ldx, self.log_pi)
            prog.append(_wrap(lib.rl2_policy_sample, pa, 0, "policy sample (actor phase)"))
            prog += self.critic_pi.forward_program
            sa = self.scalers["actor"]
            cp = self.critic_pi
            ao = N.ActorObjectiveArgs(
                logits=cp.out.data_ptr(), logits_row_stride=cp.head_ld, logits_twin_stride=B * cp.head_ld,
                support=self.support.data_ptr(), bins=cfg.critic_num_bins, batch=B, act=A,
                log_pi=self.log_pi.data_ptr(), actions=self.critic_x_pi.data_ptr() + 4 * self.obs_c,
                actions_row_stride=self.ldx, replay_action=self.critic_x.data_ptr() + 4 * self.obs_c,
                replay_row_stride=self.ldx, bc_alpha=cfg.actor_bc_alpha, alpha=self.alpha.data_ptr(),
                d_logits=cp.dhead.c(sa.scale, sa.found_inf), workspace=self.actor_ws.data_ptr(),
                counter=self.counter.data_ptr(), loss_out=mi["actor/loss"], entropy_out=mi["actor/entropy"],
                mean_action_out=mi["actor/mean_action"], q_abs_out=q_abs_addr, d_log_pi_out=dlp_addr)
            temp0 = N.TemperatureArgs(log_temp=self.log_temp.data_ptr(), update=0, alpha_out=self.alpha.data_ptr())
            prog.append(_wrap(lib.rl2_temperature_step, temp0, None, "alpha"))
            prog.append(_wrap(lib.rl2_actor_objective, ao, None, "actor objective"))
            prog += self.critic_pi.backward_program
            at = self.actor_train
            pb = self._policy_args(at, 2 * B, self.actor_noise, None, 0, self.log_pi)
            pb.log_pi = None
            pb.grad_rows = B
            pb.d_action = self.critic_pi.dx.data_ptr() + 4 * self.obs_c
            pb.ld_d_action = self.critic_pi.dx.shape[1]
            pb.d_log_pi_value = dlp_addr
            pb.bc_alpha = cfg.actor_bc_alpha
            pb.q_abs = q_abs_addr
            pb.replay_action = self.critic_x.data_ptr() + 4 * self.obs_c
            pb.ld_replay_action = self.ldx
            pb.d_plane = at.dhead.c(sa.scale, sa.found_inf)
            pb.bias_part = self.bias_part.data_ptr()
            prog.append(_wrap(lib.rl2_policy_backward, pb, None, "policy backward"))
            groups = (2 * B + 31) // 32
            bp, gb = self.bias_part, self.actor.addr("predictor.mean_bias", "grads")

            def bias_fin():
                N.check(lib.rl2_colsum_finalize(bp.data_ptr(), 1, groups, 2 * A, gb, 0, 0, N.stream_ptr()),
                        "policy bias gradient")

            prog.append(bias_fin)
            bw, prefix = self._backward_with_exchange(self.actor_train, self.actor, apply_optimizer)
            prog += bw
            if apply_optimizer:
                prog.append(self._optimizer("actor", self.actor, prefix=prefix))
            temp = N.TemperatureArgs(
                log_temp=self.log_temp.data_ptr(), entropy=mi["actor/entropy"], target_entropy=self.target_entropy,
                adam_state=self.temp_state.data_ptr(), beta1=0.9, beta2=0.999, eps=1e-8,
                lr_init=cfg.learning_rate_init, lr_peak=cfg.learning_rate_peak, lr_end=cfg.learning_rate_end,
                warmup_steps=float(cfg.learning_rate_warmup_step), decay_steps=float(cfg.learning_rate_decay_step),
                update=1, value_out=mi["temperature/value"], loss_out=mi["temperature/loss"],
                alpha_out=self.alpha.data_ptr())
            if self.dp is not None:
                ent = self.metrics[METRIC_KEYS.index("actor/entropy"):METRIC_KEYS.index("actor/entropy") + 1]
                prog.append(self.dp.scalar_reducer(mean=ent))
            if apply_optimizer:
                prog.append(_wrap(lib.rl2_temperature_step, temp, None, "temperature step"))
        else:
            temp = N.TemperatureArgs(log_temp=self.log_temp.data_ptr(), update=0, alpha_out=self.alpha.data_ptr())
            prog.append(_wrap(lib.rl2_temperature_step, temp, None, "alpha"))
        # ---- critic phase
        prog += self.actor_next.forward_program
        pn = self._policy_args(self.actor_next, B, self.next_noise,
                               self.critic_x.data_ptr() + 4 * (B * self.ldx + self.obs_c), self.ldx, self.next_log_pi)
        prog.append(_wrap(lib.rl2_policy_sample, pn, 0, "policy sample (next actions)"))
        prog += self.target_run.forward_program
        prog += self.critic_run.forward_program
        scc = self.scalers["critic"]
        cr, tr = self.critic_run, self.target_run
        dplane = cr.dhead.c(scc.scale, scc.found_inf)
        co = N.CriticObjectiveArgs(
            target_logits=tr.out.data_ptr(), target_row_stride=tr.head_ld, target_twin_stride=2 * B * tr.head_ld,
            target_row_offset=B, online_logits=cr.out.data_ptr(), online_row_stride=cr.head_ld,
            online_twin_stride=2 * B * cr.head_ld, reward=self.reward.data_ptr(),
            terminated=self.terminated.data_ptr(), discount=self.discount.data_ptr(),
            next_log_pi=self.next_log_pi.data_ptr(), alpha=self.alpha.data_ptr(), support=self.support.data_ptr(),
            min_v=cfg.critic_min_v, max_v=cfg.critic_max_v, bins=cfg.critic_num_bins, batch=B,
            loss_weight=1.0 / (2 * B), workspace=self.objective.workspace.data_ptr(),
            counter=self.objective.counter.data_ptr(), loss_out=mi["critic/loss"],
            max_entropy_out=mi["critic/max_entropy_bonus"], bias_grad_out=self.critic.addr("predictor.bias", "grads"),
            bias_grad_accumulate=0, health=self.health.data_ptr())
        if self.kind == FP16:
            co.d16 = dplane.h16
            co.d16_row_stride = cr.dhead.ld
            co.d16_twin_stride = cr.dhead.tstride
            co.d16_scale = N.addr(scc.scale)
        else:
            co.d_hi, co.d_lo = dplane.hi, dplane.lo
            co.dplane_row_stride = cr.dhead.ld
            co.dplane_twin_stride = cr.dhead.tstride
        prog.append(_wrap(lib.rl2_critic_objective, co, None, "critic objective"))
        bw, prefix = self._backward_with_exchange(self.critic_run, self.critic, apply_optimizer)
        prog += bw
        if apply_optimizer:
            prog.append(self._optimizer("critic", self.critic, target=self.target, prefix=prefix))
        if self.dp is not None:  # reported metrics over the global batch
            mx = METRIC_KEYS.index("critic/max_entropy_bonus")
            prog.append(self.dp.scalar_reducer(mean=self.metrics, max=self.metrics[mx:mx + 1]))
        return prog

    # ------------------------------------------------------------------
    def load_batch(self, batch: dict, actor_noise=None, next_noise=None, reward=None) -> None:
        """Stage an explicit batch (and noise) into the network layouts (diagnostics / parity)."""
        B, oc, oa, A = self.B, self.obs_c, self.obs_a, self.act
        t = lambda k: torch.as_tensor(batch[k], dtype=torch.float32, device=self.device)  # noqa: E731
        obs, nobs, act = t("observation"), t("next_observation"), t("action")
        self.critic_x[:B, :oc] = obs
        self.critic_x[:B, oc:oc + A] = act
        self.critic_x[B:, :oc] = nobs
        self.critic_x_pi[:B, :oc] = obs
        self.actor_x[:B, :oa] = obs[:, :oa]
        self.actor_x[B:, :oa] = nobs[:, :oa]
        self.reward.copy_(t("reward") if reward is None else torch.as_tensor(reward, device=self.device))
        self.terminated.copy_(t("terminated"))
        self.discount.copy_(t("discount"))
        if "truncated" in batch:
            self.truncated.copy_(t("truncated"))
        if actor_noise is not None:
            self.actor_noise.copy_(torch.as_tensor(actor_noise, dtype=torch.float32, device=self.device))
        if next_noise is not None:
            self.next_noise.copy_(torch.as_tensor(next_noise, dtype=torch.float32, device=self.device))

    def program(self, actor_phase: bool, apply_optimizer: bool = True) -> list:
        if apply_optimizer:
            return self.programs[actor_phase]
        key = (actor_phase, False)
        if key not in self._extra_programs:
            self._extra_programs[key] = self._program(actor_phase, apply_optimizer=False)
        return self._extra_programs[key]

    def run(self, actor_phase: bool, apply_optimizer: bool = True) -> None:
        for f in self.program(actor_phase, apply_optimizer):
            f()

    def capture(self, actor_phase: bool, pre=()) -> torch.cuda.CUDAGraph:
        """Record ``pre`` launches + one update phase as a CUDA graph (after one eager warm run)."""
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream(device=self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                for f in pre:
                    f()
                self.run(actor_phase)
        torch.cuda.current_stream(self.device).wait_stream(s)
        return g

    def metric_values(self, actor_phase: bool) -> dict[str, torch.Tensor]:
        keys = METRIC_KEYS if actor_phase else ("critic/loss", "critic/max_entropy_bonus")
        return {k: self.metrics[METRIC_KEYS.index(k)] for k in keys}


def _wrap(fn, args, extra, what):
    ref = ctypes.byref(args)
    if extra is None:
        def launch():
            N.check(fn(ref, N.stream_ptr()), what)
    else:
        def launch():
            N.check(fn(ref, extra, N.stream_ptr()), what)
    launch.keep = args
    return launch
