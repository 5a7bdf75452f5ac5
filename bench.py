"""FlashSAC learner-update benchmark (BASELINE.json metric: FlashSAC updates/s, obs 123 / act 37, batch 4096).

``python bench.py --gpus N --steps K --warmup W`` times K learner updates after W
warm-up updates and prints ONE JSON line on rank 0. A step is one ``update()``:
replay index sampling + fused gather + one learner phase (actor + critic every
``actor_update_period`` = 2 updates, critic otherwise), each phase one CUDA graph.

Workload: obs 123 ~N(0,1), act 37 ~U[-1,1], 4096
environments, batch 4096 per GPU, twin critics hidden 512 x 2 blocks, 101 atoms on
[-10, 10], actor hidden 256 x 2 blocks, FP16 dense operands with FP32 activations,
master weights and Adam. Synthetic data (no simulator, no dataset); random-init
weights of the reference architecture. The replay holds 16 x 4096 rows; the
per-update working set (> 1 GB of activations) exceeds the 126 MB L2, so no flush
is needed between steps.

With ``--gpus N`` (one process per GPU under torch.distributed.run) the ranks train ONE
learner data-parallel: every rank processes 4096 rows of the N x 4096 global batch
(same replay, indices and noise streams), batch-norm statistics are merged over all
ranks and gradients averaged with NCCL before Adam; ``value`` counts N x 4096-row
updates per second (weak scaling).

``optimizer_updates_per_s`` is the learner's optimizer-update rate (steps / s) beside
that weak-scaled ``value``.

Extra keys of the FlashSAC line (``--no-extras`` leaves them out): ``cfg5``, config 5 of
BASELINE.json (critic 1024 x 3 blocks, actor 128 x 2, FP32 recipe, a global batch of
32768 split over the ranks: strong scaling) timed on every rank count with its own
roofline, clocks and end-to-end figure; at N = 1 also ``ppo`` (the config-2 WarpPPO
update with its CPU baseline) and ``cfg4`` (the config-4 categorical objective, HBM
roofline, CPU baseline). ``cpu_baseline`` (N = 1) is the numpy restatement of the
reference update on all host cores: one actor + critic and one critic update at batch
4096, no extrapolation.

``--workload cfg5 | ppo | categorical`` time one of those alone; ``--workload gemm`` one
product shape of the update in isolation (the small case for ncu captures). Only the
JSON line goes to stdout.

``--impl reference`` times the CPU restatement of the reference update (the reference is
Python/Torch and cannot travel to the GPU box) on all host cores: real batch-4096
updates, at most six timed.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

OBS, ACT, ENVS, BATCH = 123, 37, 4096, 4096
METRIC = "FlashSAC updates/s (obs123/act37, batch 4096)"
# data-parallel FlashSAC, global batch 32768 split over the ranks
# (strong scaling), critics 1024 x 3 blocks, actor 128 x 2 (defaults), FP32 recipe
CFG5_METRIC = "FlashSAC cfg5 updates/s (obs123/act37, global batch 32768, critic 1024x3, FP32)"
CFG5_BATCH = 32768
CFG5_STEPS = 5  # timed cfg5 updates in the headline line's summary (about 1 s on one GPU)
# DRAM traffic of the GEMM family over one cfg3 update pair: the per-launch
# dram__bytes_read.sum + dram__bytes_write.sum of every product of one actor + critic
# update pair, summed (ncu launch list with those metrics, one pass, caches flushed before
# each launch; profiles/gemm_family_dram_cfg3.md).
GEMM_TRAFFIC_PER_PAIR = 3480483072
GEMM_TRAFFIC_SOURCE = ("ncu dram__bytes_read.sum + dram__bytes_write.sum summed over the 94 GEMM launches of one "
                       "update pair (2765.0 MB read + 715.4 MB written; caches flushed before each launch)")


def parse():
    p = argparse.ArgumentParser(description=__doc__)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=None,
                   help="timed steps (default 400 for the FlashSAC headline, about one second so the clock "
                        "sampler sees several samples; 40 for the other workloads and the reference arm)")
    p.add_argument("--warmup", type=int, default=6)
    p.add_argument("--impl", choices=("b200", "reference"), default="b200")
    p.add_argument("--precision", choices=("fp16", "fp32"), default="fp16")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-ppo", action="store_true", help="leave the PPO summary out of the FlashSAC line")
    p.add_argument("--workload", choices=("flashsac", "ppo", "categorical", "cfg5", "gemm"), default="flashsac",
                   help="flashsac: the headline FlashSAC update; ppo: the cfg2 WarpPPO update (ms); "
                        "categorical: the cfg4 objective microbench; cfg5: the data-parallel FP32 config "
                        "(global batch 32768 split over --gpus ranks); gemm: one tcgen05 product shape in "
                        "isolation (the small case for ncu captures)")
    p.add_argument("--no-extras", action="store_true",
                   help="leave the ppo / cfg4 / cfg5 summaries out of the FlashSAC line")
    g = p.add_argument_group("gemm workload: D[z] = A[z] B[z]^T with the update's forward epilogue")
    g.add_argument("--gemm-m", type=int, default=8192)
    g.add_argument("--gemm-n", type=int, default=2048)
    g.add_argument("--gemm-k", type=int, default=512)
    g.add_argument("--gemm-batch", type=int, default=2)
    g.add_argument("--gemm-kind", type=int, choices=(0, 1), default=0, help="0 fp16 operands, 1 3xTF32")
    g.add_argument("--gemm-a-major", type=int, choices=(0, 1), default=0)
    g.add_argument("--gemm-b-major", type=int, choices=(0, 1), default=0)
    g.add_argument("--gemm-tile-n", type=int, default=0)
    g.add_argument("--gemm-splits", type=int, default=1)
    g.add_argument("--gemm-stats", action="store_true", help="32-row column moments in the epilogue")
    g.add_argument("--gemm-plane", action="store_true", help="fp16 / tf32 operand-plane copy of the output")
    g.add_argument("--gemm-residual", action="store_true")
    g.add_argument("--gemm-in-place", action="store_true", help="residual = the output itself")
    g.add_argument("--gemm-act", type=int, choices=(0, 1, 2), default=0, help="epilogue activation: 1 ELU, 2 tanh")
    args = p.parse_args()
    if args.steps is None:
        args.steps = 400 if args.workload == "flashsac" and args.impl == "b200" else 40
    if args.no_ppo:
        args.no_extras = True
    return args


class Clocks:
    """nvidia-smi sampling during the timed region (SM clock, throttle reasons)."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index, self.rows, self.proc = index, [], None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
        except OSError:
            self.proc = None
            return self
        # the sampler's own start (driver initialisation) stays out of the timed region
        deadline = time.time() + 5.0
        while not self.rows and time.time() < deadline and self.proc.poll() is None:
            time.sleep(0.02)
        return self

    def _read(self):
        for line in self.proc.stdout:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) == 7:
                self.rows.append(parts)

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[0]) for r in self.rows if r[0].replace(".", "").isdigit()]
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        reasons = sorted({n for r in self.rows for n, v in zip(names, r[3:]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": float(self.rows[0][1]) if self.rows[0][1].replace(".", "").isdigit() else None,
                "samples": len(self.rows), "reasons": reasons}


def peaks():
    try:
        return json.loads((ROOT / "MEASURED_PEAKS.json").read_text()), "measured"
    except (OSError, ValueError):
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def build(precision: str, device, seed: int = 0, dp=None, batch: int = BATCH, critic=(512, 2), actor=(256, 2)):
    """Learner + synthetic device replay (config-3 shapes by default: batch 4096 per rank;
    with ``dp`` the ranks train one learner on the global batch, replay replicated)."""
    import torch

    from robolearn_b200.flashsac.config import FlashSACConfig
    from robolearn_b200.flashsac.learner import Learner
    from robolearn_b200.flashsac.replay import DeviceReplay
    from robolearn_b200.flashsac.sampling import sampling_program

    world = dp.world if dp is not None else 1
    cap = max(16 * ENVS, 2 * batch * world)
    cfg = FlashSACConfig(device=str(device), sample_batch_size=batch, critic_hidden_dim=critic[0],
                         critic_num_blocks=critic[1], actor_hidden_dim=actor[0], actor_num_blocks=actor[1],
                         critic_num_bins=101, critic_min_v=-10.0, critic_max_v=10.0, critic_target_update_tau=0.005,
                         learning_rate_init=3e-4, learning_rate_peak=3e-4, learning_rate_end=3e-4, n_step=1,
                         buffer_max_length=cap, buffer_min_length=batch * world, dense_precision=precision, seed=seed)
    L = Learner(OBS, OBS, ACT, cfg, device, dp=dp)
    R = DeviceReplay(OBS, ACT, ENVS, cap, 1, 0.99, batch * world, device, seed=seed)
    g = torch.Generator(device=device).manual_seed(2026 + seed)
    cap = R.capacity
    R.observation.copy_(torch.randn(cap, OBS, device=device, generator=g))
    R.next_observation.copy_(torch.randn(cap, OBS, device=device, generator=g))
    R.action.uniform_(-1, 1, generator=g)
    R.reward.copy_(torch.randn(cap, device=device, generator=g))
    R.terminated.copy_((torch.rand(cap, device=device, generator=g) < 0.01).float())
    R.discount.fill_(0.99)
    R.counters.copy_(torch.tensor([0, 0, cap], device=device))
    R._host_count = cap
    feed = sampling_program(L, R, seed=seed)
    return L, R, feed


def count_launches(prog) -> int:
    from robolearn_b200.dense import DensePlan

    n = 0
    for f in prog:
        n += 1 if isinstance(f, DensePlan) else getattr(f, "launches", 1)
    return n


def gemm_roofline(L, peak_tflops):
    """Average tcgen05 GEMM throughput over one update's products, timed as one CUDA graph
    (algorithmic FLOPs: products computed twice count once; their time is included)."""
    import torch

    from robolearn_b200.dense import DensePlan

    plans = []
    for phase in (True, False):
        plans += [f for f in L.programs[phase] if isinstance(f, DensePlan)]
    flops = sum(p.flops for p in plans if not p.recompute)  # algorithmic: a recomputed product counts once
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s), torch.cuda.graph(g, stream=s):
        for p in plans:
            p.run()
    torch.cuda.current_stream().wait_stream(s)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 10
    e0.record()
    for _ in range(reps):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    sec = e0.elapsed_time(e1) / 1e3 / reps
    achieved = flops / sec / 1e12
    return {"kernel": "rl2 tcgen05 GEMM (all products of one actor+critic update pair)", "bound": "tensor",
            "achieved": round(achieved, 1), "peak": peak_tflops, "unit": "TFLOP/s",
            "frac": round(achieved / peak_tflops, 4), "traffic": None, "launches": len(plans),
            "flops_per_pair": flops, "algorithmic_bytes_per_pair": sum(p.bytes for p in plans),
            "ms_per_pair": round(sec * 1e3, 4)}


def cpu_threads() -> int:
    """Size the host thread pools of the CPU restatement to every core this process may run
    on: BLAS (the products) and the oracle's column-chunked batch-norm passes, which never
    run at the same time (so the cores are not oversubscribed). Returns the core count."""
    import numpy as np
    from threadpoolctl import threadpool_limits

    from oracle import flashsac_np as fs

    cores = len(os.sched_getaffinity(0))
    np.ones((8, 8), np.float32) @ np.ones((8, 8), np.float32)  # load BLAS so its pool can be sized
    threadpool_limits(limits=cores)
    fs.set_threads(cores)
    return cores


def cpu_update_rate(batch: int, updates: int = 2, critic=(512, 2), actor=(256, 2)):
    """CPU restatement of the reference update (oracle, float32, all host cores): ``updates``
    real updates at ``batch`` rows, alternating actor + critic and critic-only phases like
    ``update()`` with ``actor_update_period`` = 2. Returns (updates/s, seconds, cores).
    Used by the cpu_baseline field and by ``--impl reference``; the oracle is the checker,
    never the product path."""
    import numpy as np

    from oracle import flashsac_np as fs
    from robolearn_b200.flashsac.config import FlashSACConfig
    from robolearn_b200.flashsac.learner import _init_reference_weights

    cores = cpu_threads()
    d = fs.Dims(obs=OBS, act=ACT, actor_hidden=actor[0], actor_blocks=actor[1], critic_hidden=critic[0],
                critic_blocks=critic[1], bins=101, min_v=-10.0, max_v=10.0)
    a0, c0, lt = _init_reference_weights(OBS, OBS, ACT, FlashSACConfig(
        device="cpu", actor_hidden_dim=actor[0], actor_num_blocks=actor[1], critic_hidden_dim=critic[0],
        critic_num_blocks=critic[1]))

    def with_buffers(p, twin, H, cin, blocks):
        out = {k: v.numpy() for k, v in p.items()}
        for pre in fs.bn_buffer_prefixes(blocks):
            C = cin if pre == "embedder.norm" else (4 * H if pre.endswith("norm1") else H)
            shape = (2, C) if twin else (C,)
            out[pre + ".running_mean"] = np.zeros(shape, np.float32)
            out[pre + ".running_var"] = np.ones(shape, np.float32)
        return out

    st = dict(actor=with_buffers(a0, False, actor[0], OBS, actor[1]),
              critic=with_buffers(c0, True, critic[0], OBS + ACT, critic[1]),
              target=with_buffers(c0, True, critic[0], OBS + ACT, critic[1]), log_temp=lt, opt_actor=fs.OptState(),
              opt_critic=fs.OptState(), opt_temp=fs.OptState())
    rng = np.random.default_rng(2026)
    B = batch
    bt = dict(observation=rng.standard_normal((B, OBS)).astype(np.float32),
              next_observation=rng.standard_normal((B, OBS)).astype(np.float32),
              action=rng.uniform(-1, 1, (B, ACT)).astype(np.float32), reward=rng.standard_normal(B).astype(np.float32),
              terminated=(rng.random(B) < 0.01).astype(np.float32), discount=np.full(B, 0.99, np.float32))
    an = rng.standard_normal((2 * B, ACT)).astype(np.float32)
    nn = rng.standard_normal((B, ACT)).astype(np.float32)
    h = fs.Hyper(tau=0.005, lr_end=3e-4, target_entropy=float(0.5 * ACT * np.log(2 * np.pi * np.e * 0.15**2)))
    t0 = time.perf_counter()
    for i in range(updates):
        st, _ = fs.update_networks(st, bt, an, nn, d, h, do_actor=(i % 2 == 0), dtype=np.float32)
    sec = time.perf_counter() - t0
    return updates / sec, sec, cores


def run_flashsac(workload: str, precision: str, steps: int, warmup: int, world: int, local_rank: int):
    """Device-timed and end-to-end FlashSAC updates. ``workload`` "cfg3": batch 4096 per rank
    (weak scaling), ``precision`` as given; "cfg5": global batch 32768 split over the ranks,
    critic 1024 x 3, actor 128 x 2, FP32 recipe (strong scaling). Returns (learner, device
    seconds, end-to-end seconds, host->device bytes per step, launches, clocks)."""
    import torch

    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    dp = None
    if world > 1:
        from robolearn_b200.flashsac.dp import DataParallel

        dp = DataParallel()
    if workload == "cfg5":
        if CFG5_BATCH % world:
            raise SystemExit("cfg5 needs a rank count that divides 32768")
        L, R, feed = build("fp32", device, seed=0, dp=dp, batch=CFG5_BATCH // world, critic=(1024, 3), actor=(128, 2))
    else:
        L, R, feed = build(precision, device, seed=0, dp=dp)
    for phase in (True, False):  # one eager pass loads every kernel module before capture
        for f in feed:
            f()
        L.run(phase)
    torch.cuda.synchronize()
    graphs = {phase: L.capture(phase, pre=feed) for phase in (True, False)}
    period = L.cfg.actor_update_period

    def step(i):
        graphs[i % period == 0].replay()

    for i in range(warmup):
        step(i)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local_rank) as clocks:
        if world > 1:  # every rank's sampler is up before the ranks start together
            import torch.distributed as dist

            dist.barrier()
        torch.cuda.synchronize()
        e0.record()
        for i in range(steps):
            step(warmup + i)
        e1.record()
        torch.cuda.synchronize()
    sec = e0.elapsed_time(e1) / 1e3
    launches = sum(count_launches(feed) + count_launches(L.programs[(warmup + i) % period == 0])
                   for i in range(steps))
    # ---- end to end through the public replay + learner API with host buffers:
    # each step copies one vector-environment step of transitions from pinned host
    # memory, ingests it, runs the update and reads the critic loss back to the host.
    torch.manual_seed(1234)  # the same transitions on every rank (replicated replay)
    host = {k: torch.randn(ENVS, d).pin_memory() for k, d in (("obs", OBS), ("next_obs", OBS))}
    host["act"] = torch.rand(ENVS, ACT).mul_(2).sub_(1).pin_memory()
    host["rew"] = torch.randn(ENVS).pin_memory()
    host["term"] = (torch.rand(ENVS) < 0.01).float().pin_memory()
    host["trunc"] = torch.zeros(ENVS).pin_memory()
    # two device staging sets: step i + 1's host->device copy runs on a copy stream while
    # step i's ingest and update run (the copy into a set waits for the ingest that read it)
    dev = [{k: torch.empty(v.shape, device=device) for k, v in host.items()} for _ in range(2)]
    loss_host = torch.zeros(1).pin_memory()
    h2d = sum(v.numel() * 4 for v in host.values())
    main = torch.cuda.current_stream()
    copy_stream = torch.cuda.Stream()
    landed = [torch.cuda.Event() for _ in range(2)]
    consumed = [torch.cuda.Event() for _ in range(2)]

    def upload(i):
        b = i % 2
        with torch.cuda.stream(copy_stream):
            if i >= 2:
                copy_stream.wait_event(consumed[b])
            for k in host:
                dev[b][k].copy_(host[k], non_blocking=True)
            landed[b].record(copy_stream)

    torch.cuda.synchronize()
    if world > 1:  # every rank has its host buffers before the timed region (as for the device timing)
        import torch.distributed as dist

        dist.barrier()
        torch.cuda.synchronize()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record()
    upload(0)
    for i in range(steps):
        b = i % 2
        if i + 1 < steps:
            upload(i + 1)
        main.wait_event(landed[b])
        d = dev[b]
        R.add(d["obs"], d["act"], d["rew"], d["term"], d["trunc"], d["next_obs"])
        consumed[b].record(main)
        step(i)
        loss_host.copy_(L.metrics[3:4], non_blocking=True)
    t1.record()
    torch.cuda.synchronize()
    e2e_sec = t0.elapsed_time(t1) / 1e3
    for gr in graphs.values():  # graphs holding NCCL calls go before the process group does
        gr.reset()
    return L, sec, e2e_sec, h2d, launches, clocks.summary()


# ---------------------------------------------------------------------------
# PPO: WarpPPO(48, 12, 4096, 24), 512-256-128 ELU,
# 5 epochs x 4 minibatches of 24576 rows, clip 0.2, value coef 1.0, entropy 0.01, lr 1e-3
# ---------------------------------------------------------------------------
PPO_METRIC = "PPO update ms (4096 envs x 24 steps, obs 48, act 12, 512-256-128 ELU, 5x4 minibatches)"
PPO_OBS, PPO_ACT, PPO_ENVS, PPO_T, PPO_HIDDEN = 48, 12, 4096, 24, (512, 256, 128)


def ppo_config():
    from robolearn_b200.ppo import PPOConfig

    return PPOConfig(hidden_dims=PPO_HIDDEN, activation="elu", epochs=5, num_mini_batches=4, clip_ratio=0.2,
                     value_coefficient=1.0, entropy_coefficient=0.01, learning_rate=1e-3, gamma=0.99,
                     gae_lambda=0.95)


def ppo_flops() -> float:
    """Executed GEMM FLOPs of one update: per minibatch row, forward 2*sum(K*N) per net, backward
    dW 2*sum(K*N) and dX 2*sum(K*N) without the first layer's input gradient; 20 minibatches."""
    widths = (PPO_OBS, *PPO_HIDDEN)
    total = 0
    for out in (PPO_ACT, 1):
        kn = [k * n for k, n in zip(widths, (*PPO_HIDDEN, out))]
        total += 2 * sum(kn) + 2 * sum(kn) + 2 * sum(kn[1:])
    return float(total) * PPO_ENVS * PPO_T * 5


def ppo_rollout(agent, seed: int = 0) -> dict:
    """Synthetic rollout with the cfg2 distributions: obs ~N(0,1), actions = initial means + N(0,1),
    rewards ~N(0,1), terminated ~Bernoulli(0.005), truncated 0, next values from N(0,1)."""
    import torch

    g = torch.Generator(device=agent.device).manual_seed(2026 + seed)
    B = agent.batch_size
    data = {"observations": torch.randn(B, PPO_OBS, device=agent.device, generator=g)}
    data["means"] = torch.randn(B, PPO_ACT, device=agent.device, generator=g) * 0.1
    data["actions"] = data["means"] + torch.randn(B, PPO_ACT, device=agent.device, generator=g)
    data["stds"] = torch.ones(B, PPO_ACT, device=agent.device)
    data["log_probs"] = (-0.5 * ((data["actions"] - data["means"]) ** 2 + 1.8378770664093453)).sum(1)
    data["values"] = torch.randn(B, device=agent.device, generator=g)
    data["rewards"] = torch.randn(B, device=agent.device, generator=g)
    data["next_values"] = torch.randn(B, device=agent.device, generator=g)
    data["terminated"] = (torch.rand(B, device=agent.device, generator=g) < 0.005).int()
    data["truncated"] = torch.zeros(B, dtype=torch.int32, device=agent.device)
    for k, v in data.items():
        getattr(agent, k).copy_(v)
    return data


def ppo_cpu_update_seconds() -> tuple[float, int]:
    """One full cfg2 update of the oracle restatement in float32 on all host cores: GAE and
    advantage normalisation over 4096 x 24 steps, then 5 epochs x 4 minibatches of 24576
    rows (forward, loss, backward, clipping, Adam), the cfg2 rollout distributions."""
    import numpy as np

    from oracle import ppo_np as P

    cores = cpu_threads()
    h = P.PPOHyper(hidden_dims=PPO_HIDDEN, activation="elu", epochs=5, num_mini_batches=4, clip_ratio=0.2,
                   value_coefficient=1.0, entropy_coefficient=0.01, learning_rate=1e-3)
    n = PPO_ENVS * PPO_T
    rng = np.random.default_rng(0)
    f32 = lambda x: np.asarray(x, np.float32)  # noqa: E731
    means = f32(0.1 * rng.standard_normal((n, PPO_ACT)))
    actions = f32(means + rng.standard_normal((n, PPO_ACT)))
    data = dict(observations=f32(rng.standard_normal((n, PPO_OBS))), actions=actions, means=means,
                stds=np.ones((n, PPO_ACT), np.float32),
                log_probs=f32((-0.5 * ((actions - means) ** 2 + 1.8378770664093453)).sum(1)),
                values=f32(rng.standard_normal(n)), rewards=f32(rng.standard_normal(n)),
                next_values=f32(rng.standard_normal(n)), terminated=(rng.random(n) < 0.005).astype(np.int32),
                truncated=np.zeros(n, np.int32))
    perm = rng.permutation(n)
    P.set_dtype(np.float32)
    try:
        state = P.PPOState.fresh(P.init_params(PPO_OBS, PPO_ACT, h, seed=42), h.learning_rate)
        t0 = time.perf_counter()
        P.update(state, data, PPO_T, PPO_ENVS, h, permutation=perm)
        sec = time.perf_counter() - t0
    finally:
        P.set_dtype(np.float64)
    return sec, cores


def run_ppo(args) -> dict:
    import torch

    from robolearn_b200.ppo import WarpPPO

    device = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(device)
    agent = WarpPPO(PPO_OBS, PPO_ACT, PPO_ENVS, PPO_T, ppo_config(), device=str(device))
    data = ppo_rollout(agent)
    agent.update()  # warm-up pass + capture
    for _ in range(max(args.warmup - 1, 0)):
        agent.update()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(device.index) as clocks:
        torch.cuda.synchronize()
        e0.record()
        for _ in range(args.steps):
            agent.update()
        e1.record()
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    # end to end through the public API: rollout copied from pinned host memory, update, loss
    # read back. Update i + 1's rollout goes host -> device on a copy stream into one of two
    # staging sets while update i runs; the update stream moves it into the agent's arrays.
    host = {k: v.cpu().pin_memory() for k, v in data.items()}
    loss_host = torch.zeros(4).pin_memory()
    h2d = sum(v.numel() * v.element_size() for v in host.values())
    stage = [{k: torch.empty_like(getattr(agent, k)) for k in host} for _ in range(2)]
    main = torch.cuda.current_stream()
    copy_stream = torch.cuda.Stream()
    landed = [torch.cuda.Event() for _ in range(2)]
    consumed = [torch.cuda.Event() for _ in range(2)]

    def upload(i):
        b = i % 2
        with torch.cuda.stream(copy_stream):
            if i >= 2:
                copy_stream.wait_event(consumed[b])
            for k, v in host.items():
                stage[b][k].copy_(v, non_blocking=True)
            landed[b].record(copy_stream)

    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    t0.record()
    upload(0)
    for i in range(args.steps):
        b = i % 2
        if i + 1 < args.steps:
            upload(i + 1)
        main.wait_event(landed[b])
        for k in host:
            getattr(agent, k).copy_(stage[b][k])
        consumed[b].record(main)
        agent.update()
        loss_host[:1].copy_(agent.loss, non_blocking=True)
        loss_host[1:].copy_(agent.metrics, non_blocking=True)
    t1.record()
    torch.cuda.synchronize()
    e2e_ms = t0.elapsed_time(t1) / args.steps
    pk, src = peaks()
    peak = pk["bf16_tflops"] / 6.0
    achieved = ppo_flops() / (ms * 1e-3) / 1e12
    out = {"metric": PPO_METRIC, "value": ms, "unit": "ms/update", "higher_is_better": False, "ms_per_step": ms,
           "gpu_launches": agent.launch_count(), "clocks": clocks.summary(), "dtype": "f32 (tf32x3 GEMMs)",
           "roofline": {"bound": "tensor", "achieved": round(achieved, 1), "peak": round(peak, 1),
                        "unit": "TFLOP/s", "frac": round(achieved / peak, 4), "traffic": None,
                        "flops_per_update": ppo_flops(),
                        "peak_source": f"{src} bf16_tflops / 6 (tf32 dense = bf16 / 2; three tf32 products per "
                                       "fp32 product)"},
           "e2e": {"value": e2e_ms, "unit": "ms/update", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 16},
           "config": {"workload": "cfg2 WarpPPO update (4096 envs x 24, obs 48, act 12, 512-256-128 ELU, "
                                  "5 epochs x 4 minibatches)", "global_batch": agent.batch_size,
                      "parallelism": "single", "l2": "rollout + activations > 126 MB L2 (no flush needed)"}}
    if not args.no_cpu_baseline:
        sec, cores = ppo_cpu_update_seconds()
        out["cpu_baseline"] = {"value": sec * 1e3, "unit": "ms/update", "cores": cores, "kind": "port",
                               "sample": "one full update (GAE + 5 epochs x 4 minibatches of 24576 rows) of the "
                                         "numpy restatement, float32, no extrapolation"}
    return out


# ---------------------------------------------------------------------------
# categorical critic objective microbench
# ---------------------------------------------------------------------------
CAT_METRIC = "categorical critic objective us/launch (B 65536, 101 atoms, twin logits, fp32 dlogits)"
CAT_B, CAT_BINS = 65536, 101
CAT_LD = 104  # logits / gradient rows padded to 16 bytes, as the critic head GEMM writes them


def categorical_inputs(device, seed: int = 0) -> dict:
    """Target and online logits [2][B][101] ~N(0,1) (rows padded to 104 floats, the layout the
    critic head product writes), rewards ~N(0,1), discount 0.99, done ~Bernoulli(0.01), next
    log-probs ~N(0,1), alpha 0.01."""
    import torch

    g = torch.Generator(device=device).manual_seed(4000 + seed)
    B, K = CAT_B, CAT_BINS
    def logits():
        buf = torch.zeros(2, B, CAT_LD, device=device)
        buf[:, :, :K] = torch.randn(2, B, K, device=device, generator=g)
        return buf

    return {"target": logits(), "online": logits(),
            "reward": torch.randn(B, device=device, generator=g),
            "terminated": (torch.rand(B, device=device, generator=g) < 0.01).float(),
            "discount": torch.full((B,), 0.99, device=device),
            "next_log_pi": torch.randn(B, device=device, generator=g),
            "alpha": torch.full((1,), 0.01, device=device)}


def categorical_bytes() -> int:
    # read target + online logits, write dlogits (fp32), read 4 per-row vectors
    return 3 * 2 * CAT_B * CAT_BINS * 4 + 4 * CAT_B * 4


def run_categorical(args) -> dict:
    import torch

    from robolearn_b200.categorical import CriticObjective

    device = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(device)
    x = categorical_inputs(device)
    obj = CriticObjective(CAT_B, CAT_BINS, -10.0, 10.0, device=device)
    dlogits = torch.zeros(2, CAT_B, CAT_LD, device=device)
    loss = torch.zeros(1, device=device)
    mx = torch.zeros(1, device=device)

    def launch():
        obj.run(target_logits=x["target"], target_row_stride=CAT_LD, target_twin_stride=CAT_B * CAT_LD,
                target_row_offset=0, online_logits=x["online"], online_row_stride=CAT_LD,
                online_twin_stride=CAT_B * CAT_LD, reward=x["reward"], terminated=x["terminated"],
                discount=x["discount"], next_log_pi=x["next_log_pi"], alpha=x["alpha"], loss_weight=1.0 / (2 * CAT_B),
                loss_out=loss, max_entropy_out=mx, dlogits=dlogits, dlogits_row_stride=CAT_LD,
                dlogits_twin_stride=CAT_B * CAT_LD)

    flush = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device=device)  # 256 MB > L2
    for _ in range(max(args.warmup, 3)):
        launch()
    torch.cuda.synchronize()
    times = []
    for _ in range(args.steps):
        flush.zero_()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        launch()
        e1.record()
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1) * 1e3)
    us = statistics.median(times)
    pk, src = peaks()
    gbs = categorical_bytes() / (us * 1e-6) / 1e9
    out = {"metric": CAT_METRIC, "value": us, "unit": "us/launch", "higher_is_better": False, "ms_per_step": us / 1e3,
           "gpu_launches": 1, "dtype": "f32", "rows_per_s": CAT_B / (us * 1e-6),
           "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
                        "frac": round(gbs / pk["hbm_gbs"], 4), "traffic": None,
                        "algorithmic_bytes": categorical_bytes(), "peak_source": f"{src} hbm_gbs"},
           "config": {"workload": "cfg4 categorical projection + CE + gradient, B 65536, 101 atoms on [-10, 10], "
                                  "both twins", "layout": "logits and gradient rows padded to 104 floats",
                      "l2": "L2 flushed (256 MB write) before every timed launch",
                      "timing": "median of per-launch CUDA-event times"}}
    if not args.no_cpu_baseline:
        import numpy as np

        from oracle import flashsac_np as fs

        xs = {k: (v[:, :, :CAT_BINS] if v.dim() == 3 else v).cpu().numpy() for k, v in x.items()}
        t0 = time.perf_counter()
        tl = xs["target"] - np.log(np.exp(xs["target"]).sum(-1, keepdims=True))
        q = (np.exp(tl) * fs.support(CAT_BINS, -10.0, 10.0)).sum(-1)
        lp = fs.select_min_q(q, tl)
        ent = 0.01 * xs["next_log_pi"]
        tgt, _ = fs.categorical_target(lp, xs["reward"], xs["terminated"], ent, 0.99, CAT_BINS, -10.0, 10.0)
        ol = xs["online"] - np.log(np.exp(xs["online"]).sum(-1, keepdims=True))
        fs.categorical_loss_grad(ol, tgt, CAT_B)
        sec = time.perf_counter() - t0
        out["cpu_baseline"] = {"value": sec * 1e6, "unit": "us/launch", "cores": len(os.sched_getaffinity(0)),
                               "kind": "port", "sample": "one full launch (B 65536) of the numpy restatement"}
    return out


# ---------------------------------------------------------------------------
# one tcgen05 product shape in isolation (the small, self-contained ncu case)
# ---------------------------------------------------------------------------
def run_gemm(args) -> dict:
    """Times ``--steps`` launches of one product ``D[z] = A[z] B[z]^T`` with the forward
    epilogue the update uses (bias, optional residual, 32-row column moments, operand-plane
    copy of the output), CUDA events on the launching stream after ``--warmup`` launches."""
    import torch

    from robolearn_b200 import _native as N
    from robolearn_b200 import dense

    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    m, n, k, z, kind = args.gemm_m, args.gemm_n, args.gemm_k, args.gemm_batch, args.gemm_kind
    dt = torch.float16 if kind == 0 else torch.float32
    g = torch.Generator(device=dev).manual_seed(0)

    def operand(rows: int, major: int):
        inner, outer = (k, rows) if major == 0 else (rows, k)
        ld = dense.operand_ld(inner, kind)
        t = torch.zeros(z, outer, ld, device=dev, dtype=dt)
        t[:, :, :inner] = (torch.randn(z, outer, inner, device=dev, generator=g) / k**0.5).to(dt)
        return t, ld

    A, lda = operand(m, args.gemm_a_major)
    B, ldb = operand(n, args.gemm_b_major)
    kw = {}
    if kind == 1:
        A, a_lo = dense.tf32_split(A)
        B, b_lo = dense.tf32_split(B)
        kw.update(a_lo=a_lo, b_lo=b_lo)
    ldd = dense.operand_ld(n, 1)
    splits = max(1, args.gemm_splits)
    D = torch.zeros(splits, z, m, ldd, device=dev)
    kw.update(d=D, ldd=ldd, d_batch_stride=m * ldd)
    if splits > 1:
        kw.update(k_splits=splits, d_split_stride=z * m * ldd)
    else:
        kw.update(bias=torch.randn(z, n, device=dev, generator=g), bias_batch_stride=n)
    if args.gemm_in_place and splits == 1:
        kw.update(residual=D[0], ldr=ldd, residual_batch_stride=m * ldd)
    elif args.gemm_residual and splits == 1:
        kw.update(residual=torch.randn(z, m, n, device=dev, generator=g), ldr=n, residual_batch_stride=m * n)
    groups = (m + 31) // 32
    if args.gemm_stats and splits == 1:
        kw.update(stat_mean=torch.zeros(z, groups, n, device=dev), stat_m2=torch.zeros(z, groups, n, device=dev),
                  stat_batch_stride=groups * n)
    keep = []
    if args.gemm_plane and splits == 1:
        pld = dense.operand_ld(n, kind)
        if kind == 0:
            h = torch.zeros(z, m, pld, device=dev, dtype=torch.float16)
            keep.append(h)
            kw["out_plane"] = N.Plane(h16=h.data_ptr(), ld=pld, twin_stride=m * pld)
        else:
            hi, lo = torch.zeros(z, m, pld, device=dev), torch.zeros(z, m, pld, device=dev)
            keep += [hi, lo]
            kw["out_plane"] = N.Plane(hi=hi.data_ptr(), lo=lo.data_ptr(), ld=pld, twin_stride=m * pld)
    if args.gemm_act:
        kw["activation"] = args.gemm_act
    plan = dense.DensePlan(kind=kind, m=m, n=n, k=k, a=A, b=B, lda=lda, ldb=ldb, a_major=args.gemm_a_major,
                           b_major=args.gemm_b_major, batch=z, a_batch_stride=A[0].numel(),
                           b_batch_stride=B[0].numel(), tile_n=args.gemm_tile_n, **kw)
    stream = torch.cuda.current_stream()
    for _ in range(max(args.warmup, 3)):
        plan.run()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        plan.run()
    e1.record(stream)
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1000.0 / max(args.steps, 1)
    el = 2 if kind == 0 else 8
    out_bytes = z * m * n * 4 * splits + (z * m * n * el if args.gemm_plane and splits == 1 else 0)
    in_bytes = z * (m + n) * k * el + (z * m * n * 4 if args.gemm_residual and splits == 1 else 0)
    flops = 2.0 * z * m * n * k * (1 if kind == 0 else 3)
    pk, src = peaks()
    peak = pk["bf16_tflops"] if kind == 0 else pk["bf16_tflops"] / 2
    tflops = flops / us / 1e6
    del keep
    return {"metric": f"tcgen05 GEMM us/launch (M {m}, N {n}, K {k}, batch {z}, {'fp16' if kind == 0 else '3xTF32'})",
            "value": us, "unit": "us/launch", "higher_is_better": False, "ms_per_step": us / 1e3,
            "gpu_launches": args.steps, "dtype": "fp16" if kind == 0 else "f32 (tf32x3)",
            "roofline": {"bound": "tensor", "achieved": round(tflops, 1), "peak": round(peak, 1), "unit": "TFLOP/s",
                         "frac": round(tflops / peak, 4), "traffic": None, "algorithmic_bytes": in_bytes + out_bytes,
                         "peak_source": f"{src} bf16_tflops" + (" / 2 (tf32 dense rate; FLOPs per tf32 pass)"
                                                                 if kind == 1 else " (burst)")},
            "config": {"workload": "one product of the update in isolation", "tile_n": plan.tile_n,
                       "splits": splits, "stats": args.gemm_stats, "plane": args.gemm_plane,
                       "residual": args.gemm_residual or args.gemm_in_place, "activation": args.gemm_act,
                       "a_major": args.gemm_a_major, "b_major": args.gemm_b_major,
                       "l2": "operands resident (launch-to-launch timing of one shape)"}}


_JSON_OUT = None


def emit(line: str) -> None:
    """Write the result line to the process's original standard output (everything else,
    including libraries that print to stdout, goes to standard error)."""
    out = _JSON_OUT if _JSON_OUT is not None else sys.stdout
    out.write(line + "\n")
    out.flush()


REF_MAX_STEPS = 6  # timed CPU updates of the reference arm (about 10 s each at batch 4096 on 16 cores)


def reference_line(args, base) -> dict:
    """``--impl reference``: the CPU restatement of the reference path on all host cores, on
    the same workload, metric and unit as the b200 arm. FlashSAC cfg3: real updates at batch
    4096 (alternating actor + critic and critic-only phases, as ``update()`` does), one
    warm-up update and at most ``REF_MAX_STEPS`` timed. cfg5 (30 TFLOP per update, beyond a
    bounded CPU sample): one update pair at 1024 and at 2048 rows, time extrapolated
    linearly in the rows to 32768, labelled as such. PPO: one full cfg2 update. The CPU
    path has no warm-up to do (no compilation, no caches to fill at these sizes)."""
    if args.workload == "ppo":
        sec, cores = ppo_cpu_update_seconds()
        value = sec * 1e3
        return {"metric": PPO_METRIC, "impl": "reference", "value": value, "unit": "ms/update",
                "higher_is_better": False, "n_gpus": args.gpus, "steps": 1, "warmup": 0, "ms_per_step": value,
                "dtype": "f32", "data": "synthetic",
                "config": {"workload": "cfg2 WarpPPO update, CPU restatement of the reference (oracle port)"},
                "cpu_baseline": {"value": value, "unit": "ms/update", "cores": cores, "kind": "port",
                                 "sample": "one full update (GAE + 5 epochs x 4 minibatches of 24576 rows), float32"},
                "e2e": {"value": value, "unit": "ms/update", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    if args.workload == "cfg5":
        rates = []
        for rows in (1024, 2048):
            r, sec, cores = cpu_update_rate(rows, 2, critic=(1024, 3), actor=(128, 2))
            rates.append((rows, 1.0 / r))
        (b1, t1), (b2, t2) = rates
        per_update = t2 + max(t2 - t1, 0.0) / (b2 - b1) * (CFG5_BATCH - b2)
        value = 1.0 / per_update
        return dict(base, metric=CFG5_METRIC, scaling="strong", impl="reference", value=value, steps=2, warmup=0,
                    ms_per_step=per_update * 1e3, dtype="f32",
                    config={"workload": "cfg5 FlashSAC update, CPU restatement of the reference (oracle port)",
                            "global_batch": CFG5_BATCH, "parallelism": "cpu"},
                    cpu_baseline={"value": value, "unit": "updates/s", "cores": cores, "kind": "port",
                                  "sample": f"one actor+critic update pair at {b1} rows and one at {b2} "
                                            f"(EXTRAPOLATED linearly in the rows to {CFG5_BATCH})"},
                    e2e={"value": value, "unit": "updates/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0})
    steps = min(args.steps, REF_MAX_STEPS)
    value, sec, cores = cpu_update_rate(BATCH, steps)  # the CPU path has nothing to warm up
    return dict(base, impl="reference", value=value, steps=steps, warmup=0, steps_requested=args.steps,
                ms_per_step=1e3 / value, dtype="f32",
                config={"workload": "cfg3 FlashSAC update, CPU restatement of the reference (oracle port)",
                        "global_batch": BATCH, "parallelism": "cpu"},
                cpu_baseline={"value": value, "unit": "updates/s", "cores": cores, "kind": "port",
                              "sample": f"{steps} real updates at batch {BATCH} (alternating actor + critic "
                                        "and critic-only, no extrapolation), float32"},
                e2e={"value": value, "unit": "updates/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0})


def flashsac_summary(workload: str, precision: str, steps: int, warmup: int, world: int, local_rank: int) -> dict:
    """One FlashSAC workload timed on every rank (device time and end-to-end: max over ranks)
    with its GEMM-family roofline; the learner is released before returning."""
    import torch

    L, sec, e2e_sec, h2d, launches, clocks = run_flashsac(workload, precision, steps, warmup, world, local_rank)
    if world > 1:
        import torch.distributed as dist

        t = torch.tensor([sec, e2e_sec], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        sec, e2e_sec = t.tolist()
    pk, src = peaks()
    if workload == "cfg5":
        # three tf32 tensor passes per product (counted in the executed FLOPs) at the dense
        # tf32 rate, half the bf16 rate
        roof = gemm_roofline(L, pk["bf16_tflops"] / 2)
        roof["peak_source"] = f"{src} bf16_tflops / 2 (dense tf32 rate; FLOPs counted per tf32 pass, 3 per product)"
        rows, scaling, dtype = CFG5_BATCH, "strong", "f32 (3xTF32 products)"
        workload_name = ("cfg5 data-parallel FlashSAC update (obs 123, act 37, global batch 32768 split over the "
                         "ranks, critic 1024x3, actor 128x2, 101 atoms, FP32 recipe)")
        value = steps / sec  # global-batch updates per second
    else:
        roof = gemm_roofline(L, pk["bf16_tflops"])
        roof["peak_source"] = f"{src} bf16_tflops (burst; fp16 dense rate taken equal)"
        roof["traffic"] = GEMM_TRAFFIC_PER_PAIR
        roof["traffic_source"] = GEMM_TRAFFIC_SOURCE
        rows, scaling, dtype = BATCH * world, "weak", precision
        workload_name = ("cfg3 FlashSAC update (obs 123, act 37, batch 4096 per GPU, critic 512x2, actor 256x2, "
                         "101 atoms)")
        value = world * steps / sec  # 4096-row batches per second over all ranks
    out = {"value": value, "optimizer_updates_per_s": steps / sec, "ms_per_step": sec / steps * 1e3,
           "steps": steps, "warmup": warmup, "scaling": scaling, "dtype": dtype, "gpu_launches": launches,
           "clocks": clocks, "roofline": roof,
           "config": {"workload": workload_name, "global_batch": rows, "seq_len": None,
                      "parallelism": f"dp{world}" if world > 1 else "single",
                      "l2": "working set > 126 MB L2 (no flush needed)"},
           "e2e": {"value": value * sec / e2e_sec, "unit": "updates/s", "h2d_bytes_per_step": h2d,
                   "d2h_bytes_per_step": 4}}
    del L
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    return out


def main():
    global _JSON_OUT
    # keep stdout for the JSON line alone: NCCL prints its version on the first collective
    sys.stdout.flush()
    _JSON_OUT = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)
    args = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    base = {"metric": METRIC, "unit": "updates/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "data": "synthetic"}
    common = dict(n_gpus=1, steps=args.steps, warmup=args.warmup, scaling="weak", vs_baseline=None, data="synthetic")
    if args.impl == "reference":
        if rank == 0:  # the CPU arm runs once per job; other ranks exit without work
            emit(json.dumps(reference_line(args, base)))
        return
    if args.workload in ("categorical", "gemm", "ppo"):
        if rank == 0:
            run = {"categorical": run_categorical, "gemm": run_gemm, "ppo": run_ppo}[args.workload]
            emit(json.dumps(dict(common, impl="b200", **run(args))))
        return
    import torch

    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    if args.workload == "cfg5":
        head = flashsac_summary("cfg5", "fp32", args.steps, args.warmup, world, local_rank)
        out = dict(base, impl="b200", metric=CFG5_METRIC, **head)
    else:
        head = flashsac_summary("cfg3", args.precision, args.steps, args.warmup, world, local_rank)
        out = dict(base, impl="b200", **head)
        if not args.no_extras:
            # config 5 (strong scaling of the global batch 32768) on every rank count
            c5 = flashsac_summary("cfg5", "fp32", CFG5_STEPS, 3, world, local_rank)
            out["cfg5"] = dict(metric=CFG5_METRIC, unit="updates/s", **c5)
        if rank == 0 and world == 1 and not args.no_cpu_baseline:
            rate, csec, cores = cpu_update_rate(BATCH, 2)
            out["cpu_baseline"] = {"value": rate, "unit": "updates/s", "cores": cores, "kind": "port",
                                   "sample": f"one actor + critic update and one critic update at batch {BATCH} "
                                             f"({csec:.1f} s, numpy restatement in float32, no extrapolation)"}
        if rank == 0 and world == 1 and not args.no_extras:
            import types

            sub = types.SimpleNamespace(steps=10, warmup=3, no_cpu_baseline=args.no_cpu_baseline)
            pp = run_ppo(sub)
            out["ppo"] = {k: pp[k] for k in ("metric", "value", "unit", "higher_is_better", "ms_per_step",
                                             "gpu_launches", "clocks", "roofline", "e2e", "config")
                          if k in pp}
            if "cpu_baseline" in pp:
                out["ppo"]["cpu_baseline"] = pp["cpu_baseline"]
            sub = types.SimpleNamespace(steps=20, warmup=3, no_cpu_baseline=args.no_cpu_baseline)
            cat = run_categorical(sub)
            out["cfg4"] = {k: cat[k] for k in ("metric", "value", "unit", "higher_is_better", "roofline", "config",
                                               "rows_per_s", "cpu_baseline") if k in cat}
    if rank == 0:
        emit(json.dumps(out))
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
