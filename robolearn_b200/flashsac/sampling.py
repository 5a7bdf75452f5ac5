"""Launches that feed one learner update from the device replay: index sampling,
fused gather into the network layouts (with reward normalisation) and policy noise.
Replaces ``WarpFlashReplay.sample`` + ``normalize_rewards`` + ``_normal_noise``
(``src/robolearn/warp/_flash_replay.py:281-301,434-444``, ``warp/flashsac.py:44-50``)."""

from __future__ import annotations

import ctypes

from .. import _native as N


def sampling_program(learner, replay, reward_state=None, g_max: float = 5.0, seed: int = 0, noise: bool = True):
    """Return a list of launches (capturable) that fill ``learner``'s batch buffers.

    ``reward_state`` is the device normaliser state ``[mean, var, count, G_r_max]``;
    None leaves rewards unnormalised.
    """
    lib = N.load()
    L = learner
    B = L.B
    dp = getattr(L, "dp", None)
    world, rank = (dp.world, dp.rank) if dp is not None else (1, 0)
    BG, row0 = B * world, B * rank  # global batch and this rank's first row
    idx = replay_indices(L, BG)
    g = N.ReplayGatherArgs(
        indices=idx.data_ptr() + 4 * row0, batch=B, obs=replay.observation.data_ptr(),
        next_obs=replay.next_observation.data_ptr(), ld_obs=replay.obs_dim, action=replay.action.data_ptr(),
        ld_action=replay.act_dim, reward=replay.reward.data_ptr(), terminated=replay.terminated.data_ptr(),
        truncated=replay.truncated.data_ptr(), discount=replay.discount.data_ptr(), obs_dim=L.obs_c,
        act_dim=L.act, actor_obs_dim=L.obs_a, critic_x=L.critic_x.data_ptr(), ld_critic_x=L.ldx,
        actor_x=L.actor_x.data_ptr(), ld_actor_x=L.ldax, reward_out=L.reward.data_ptr(),
        terminated_out=L.terminated.data_ptr(), truncated_out=L.truncated.data_ptr(),
        discount_out=L.discount.data_ptr(), g_max=g_max, norm_eps=1e-8,
        critic_x_pi=L.critic_x_pi.data_ptr(), ld_critic_x_pi=L.ldx)
    if reward_state is not None:
        g.g_var = reward_state.data_ptr() + 4
        g.g_r_max = reward_state.data_ptr() + 12
    gref = ctypes.byref(g)
    epoch = replay.epoch
    pop = replay.counters.data_ptr() + 16  # filled rows
    health = L.health.data_ptr()
    seed_idx = (seed * 0x9E3779B97F4A7C15 + 11) & 0xFFFFFFFFFFFFFFFF
    seed_a = (seed * 0x9E3779B97F4A7C15 + 23) & 0xFFFFFFFFFFFFFFFF
    seed_n = (seed * 0x9E3779B97F4A7C15 + 37) & 0xFFFFFFFFFFFFFFFF

    def sample():
        s = N.stream_ptr()
        N.check(lib.rl2_replay_sample(seed_idx, epoch.data_ptr(), pop, 0, BG, idx.data_ptr(), health, s), "sample")
        N.check(lib.rl2_replay_gather(gref, s), "gather")

    # global noise arrays: actor phase [observations (BG) | next observations (BG)], next actions [BG];
    # this rank draws its rows of each
    an, A = L.actor_noise.data_ptr(), L.act

    def make_noise():
        s = N.stream_ptr()
        N.check(lib.rl2_normal_noise_rows(seed_a, epoch.data_ptr(), row0, B, A, an, A, s), "actor noise")
        N.check(lib.rl2_normal_noise_rows(seed_a, epoch.data_ptr(), BG + row0, B, A, an + 4 * B * A, A, s),
                "actor noise (next observations)")
        N.check(lib.rl2_normal_noise_rows(seed_n, epoch.data_ptr(), row0, B, A, L.next_noise.data_ptr(), A, s),
                "next noise")

    def advance():
        N.check(lib.rl2_counter_advance(epoch.data_ptr(), 1, N.stream_ptr()), "advance epoch")

    sample.keep = g
    sample.launches, make_noise.launches, advance.launches = 2, 3, 1
    return [sample, make_noise, advance] if noise else [sample, advance]


def replay_indices(learner, rows: int | None = None):
    """The learner's replay-index buffer (the global batch's indices under data parallelism)."""
    import torch

    rows = rows or learner.B
    if not hasattr(learner, "_indices") or learner._indices.numel() < rows:
        learner._indices = torch.zeros(rows, dtype=torch.int32, device=learner.device)
    return learner._indices
