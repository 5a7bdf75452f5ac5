"""ctypes binding of ``librl2.so`` (the C ABI declared in ``include/rl2.h``).

Mirrors the reference's loader contract (``src/robolearn/cuda/_runtime.py:77-135``):
explicit ``argtypes``/``restype`` per entry point and ``check()`` that turns a -1
status into ``RuntimeError`` with the library's thread-local message. There is no
CPU or library fallback: if the shared library cannot be found or built, loading
raises.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

from . import build as _build

_LOCK = threading.Lock()
_LIB: ctypes.CDLL | None = None

P = ctypes.c_void_p
I = ctypes.c_int  # noqa: E741
LL = ctypes.c_longlong
F = ctypes.c_float
D = ctypes.c_double
SZ = ctypes.c_size_t
U64 = ctypes.c_uint64


class Plane(ctypes.Structure):
    """``rl2_plane`` (include/rl2.h): fp16 operand plane or tf32 hi/lo pair."""

    _fields_ = [("h16", P), ("hi", P), ("lo", P), ("ld", LL), ("twin_stride", LL), ("scale", P), ("found_inf", P)]


class GemmDesc(ctypes.Structure):
    """``rl2_gemm_desc`` (include/rl2.h)."""

    _fields_ = [
        ("kind", I), ("m", I), ("n", I), ("k", I), ("batch", I),
        ("a", P), ("a_lo", P), ("a_major", I), ("lda", LL), ("a_batch_stride", LL),
        ("b", P), ("b_lo", P), ("b_major", I), ("ldb", LL), ("b_batch_stride", LL),
        ("d", P), ("ldd", LL), ("d_batch_stride", LL), ("accumulate", I),
        ("bias", P), ("bias_batch_stride", LL),
        ("residual", P), ("ldr", LL), ("residual_batch_stride", LL),
        ("stat_mean", P), ("stat_m2", P), ("stat_batch_stride", LL),
        ("scale", P), ("k_splits", I), ("d_split_stride", LL), ("tile_n", I), ("health", P),
        ("out_plane", Plane),
        ("activation", I), ("act_aux", P), ("ld_aux", LL), ("aux_batch_stride", LL),
        ("bn_mean", P), ("bn_invstd", P), ("bn_gamma", P), ("bn_beta", P), ("bn_twin_stride", LL), ("bn_relu", I),
    ]


class CriticObjectiveArgs(ctypes.Structure):
    """``rl2_critic_objective_args`` (include/rl2.h)."""

    _fields_ = [
        ("target_logits", P), ("target_row_stride", LL), ("target_twin_stride", LL), ("target_row_offset", I),
        ("online_logits", P), ("online_row_stride", LL), ("online_twin_stride", LL),
        ("reward", P), ("terminated", P), ("discount", P), ("next_log_pi", P), ("alpha", P), ("support", P),
        ("min_v", D), ("max_v", D), ("bins", I), ("batch", I), ("loss_weight", F),
        ("dlogits", P), ("dlogits_row_stride", LL), ("dlogits_twin_stride", LL),
        ("d16", P), ("d16_row_stride", LL), ("d16_twin_stride", LL), ("d16_scale", P),
        ("d_hi", P), ("d_lo", P), ("dplane_row_stride", LL), ("dplane_twin_stride", LL),
        ("target_out", P), ("target_out_row_stride", LL),
        ("workspace", P), ("counter", P), ("loss_out", P), ("max_entropy_out", P), ("bias_grad_out", P),
        ("bias_grad_accumulate", I), ("health", P),
    ]


class BnApplyArgs(ctypes.Structure):
    _fields_ = [
        ("x", P), ("ldx", LL), ("x_twin_stride", LL), ("twins", I), ("rows", I), ("cols", I),
        ("mean", P), ("invstd", P), ("gamma", P), ("beta", P), ("relu", I),
        ("residual", P), ("ldr", LL), ("residual_twin_stride", LL),
        ("y", P), ("ldy", LL), ("y_twin_stride", LL), ("plane", Plane),
    ]


class BnBackwardArgs(ctypes.Structure):
    _fields_ = [
        ("dy", P), ("lddy", LL), ("dy_twin_stride", LL), ("x", P), ("ldx", LL), ("x_twin_stride", LL),
        ("twins", I), ("rows", I), ("cols", I), ("mean", P), ("invstd", P), ("gamma", P), ("beta", P),
        ("relu", I), ("training", I), ("s1_part", P), ("s2_part", P), ("coef1", P), ("coef2", P),
        ("dx", P), ("lddx", LL), ("dx_twin_stride", LL), ("sum_twins", I), ("plane", Plane),
    ]


class PolicyArgs(ctypes.Structure):
    _fields_ = [
        ("head", P), ("ld_head", LL), ("noise", P), ("ld_noise", LL), ("rows", I), ("act", I),
        ("actions", P), ("ld_actions", LL), ("log_pi", P), ("grad_rows", I), ("d_action", P), ("ld_d_action", LL),
        ("d_log_pi", P), ("d_log_pi_value", P), ("bc_alpha", F), ("q_abs", P), ("replay_action", P),
        ("ld_replay_action", LL), ("d_head", P), ("ld_d_head", LL), ("d_plane", Plane), ("bias_part", P),
    ]


class ActorObjectiveArgs(ctypes.Structure):
    _fields_ = [
        ("logits", P), ("logits_row_stride", LL), ("logits_twin_stride", LL), ("support", P),
        ("bins", I), ("batch", I), ("act", I), ("log_pi", P), ("actions", P), ("actions_row_stride", LL),
        ("replay_action", P), ("replay_row_stride", LL), ("bc_alpha", F), ("alpha", P), ("d_logits", Plane),
        ("workspace", P), ("counter", P), ("loss_out", P), ("entropy_out", P), ("mean_action_out", P),
        ("q_abs_out", P), ("d_log_pi_out", P),
    ]


class TemperatureArgs(ctypes.Structure):
    _fields_ = [
        ("log_temp", P), ("entropy", P), ("target_entropy", F), ("adam_state", P), ("beta1", F), ("beta2", F),
        ("eps", F), ("lr_init", D), ("lr_peak", D), ("lr_end", D), ("warmup_steps", D), ("decay_steps", D),
        ("update", I), ("value_out", P), ("loss_out", P), ("alpha_out", P),
    ]


class Segment(ctypes.Structure):
    _fields_ = [("offset", LL), ("offset2", LL), ("plane_offset", LL), ("length", I), ("kind", I)]


class AdamPrepareArgs(ctypes.Structure):
    _fields_ = [
        ("state", P), ("found_inf", P), ("formula", I), ("beta1", F), ("beta2", F),
        ("lr_init", D), ("lr_peak", D), ("lr_end", D), ("warmup_steps", D), ("decay_steps", D),
        ("schedule_on_attempts", I), ("lr_override", P), ("scaler", I), ("growth", F), ("backoff", F),
        ("growth_interval", I), ("scale_out", P), ("inv_scale_out", P),
    ]


class AdamArgs(ctypes.Structure):
    _fields_ = [
        ("params", P), ("grads", P), ("m", P), ("v", P), ("segments", P), ("count", I), ("state", P),
        ("formula", I), ("beta1", F), ("beta2", F), ("eps", F), ("project", I), ("weight_plane", Plane),
        ("target_params", P), ("tau", F), ("target_plane", Plane), ("warp_segments", I),
    ]


class ReplayGatherArgs(ctypes.Structure):
    _fields_ = [
        ("indices", P), ("batch", I), ("obs", P), ("next_obs", P), ("ld_obs", LL), ("action", P),
        ("ld_action", LL), ("reward", P), ("terminated", P), ("truncated", P), ("discount", P),
        ("obs_dim", I), ("act_dim", I), ("actor_obs_dim", I), ("critic_x", P), ("ld_critic_x", LL),
        ("actor_x", P), ("ld_actor_x", LL), ("reward_out", P), ("terminated_out", P), ("truncated_out", P),
        ("discount_out", P), ("g_var", P), ("g_r_max", P), ("g_max", F), ("norm_eps", F),
        ("batch_obs", P), ("batch_next_obs", P), ("batch_action", P), ("batch_reward", P),
        ("critic_x_pi", P), ("ld_critic_x_pi", LL),
    ]


# name -> (argtypes, restype); every symbol here is declared in include/rl2.h
SIGNATURES: dict[str, tuple[list, object]] = {
    "rl2_last_error": ([], ctypes.c_char_p),
    "rl2_abi_version": ([], I),
    "rl2_gemm_create": ([ctypes.POINTER(GemmDesc)], P),
    "rl2_gemm_run": ([P, P], I),
    "rl2_gemm_destroy": ([P], I),
    "rl2_gemm_tile_n": ([P], I),
    "rl2_gemm_uses_tma_store": ([P], I),
    "rl2_gemm_cta_pair": ([P], I),
    "rl2_split_reduce": ([P, LL, I, P, LL, I, P], I),
    "rl2_split_reduce_batched": ([P, LL, I, P, LL, I, I, LL, LL, P], I),
    "rl2_categorical_workspace_floats": ([I, I], I),
    "rl2_categorical_counter_words": ([I, I], I),
    "rl2_critic_objective": ([ctypes.POINTER(CriticObjectiveArgs), P], I),
    "rl2_colstats": ([P, LL, LL, I, I, I, P, P, LL, P], I),
    "rl2_bn_finalize": ([P, P, LL, I, I, I, P, P, P, P, F, F, I, P], I),
    "rl2_bn_eval_prepare": ([P, P, LL, F, P, P, P], I),
    "rl2_bn_apply": ([ctypes.POINTER(BnApplyArgs), P], I),
    "rl2_bn_backward_reduce": ([ctypes.POINTER(BnBackwardArgs), P], I),
    "rl2_bn_backward_finalize": ([P, P, I, I, I, P, P, LL, I, P, P, P], I),
    "rl2_bn_backward_apply": ([ctypes.POINTER(BnBackwardArgs), P], I),
    "rl2_rms_forward": ([P, LL, LL, I, I, I, P, F, P, P, LL, LL, ctypes.POINTER(Plane), P], I),
    "rl2_rms_backward": ([P, LL, LL, P, LL, LL, P, P, I, I, I, P, LL, LL, P, P], I),
    "rl2_colsum_finalize": ([P, I, I, I, P, LL, I, P], I),
    "rl2_policy_sample": ([ctypes.POINTER(PolicyArgs), I, P], I),
    "rl2_policy_backward": ([ctypes.POINTER(PolicyArgs), P], I),
    "rl2_actor_objective_workspace_floats": ([I], I),
    "rl2_actor_objective": ([ctypes.POINTER(ActorObjectiveArgs), P], I),
    "rl2_temperature_step": ([ctypes.POINTER(TemperatureArgs), P], I),
    "rl2_adam_prepare": ([ctypes.POINTER(AdamPrepareArgs), P], I),
    "rl2_adam_step": ([ctypes.POINTER(AdamArgs), P], I),
    "rl2_segment_max_length": ([], I),
    "rl2_segment_warp_max_length": ([], I),
    "rl2_replay_sample": ([ctypes.c_ulonglong, P, P, LL, I, P, P, P], I),
    "rl2_counter_advance": ([P, ctypes.c_ulonglong, P], I),
    "rl2_replay_gather": ([ctypes.POINTER(ReplayGatherArgs), P], I),
    "rl2_normal_noise": ([ctypes.c_ulonglong, P, I, I, P, LL, P], I),
    "rl2_philox4x32": ([ctypes.c_uint] * 6 + [ctypes.POINTER(ctypes.c_uint)], None),
}


def library_path() -> Path:
    return _build.LIBRARY


def load(build_if_missing: bool = True) -> ctypes.CDLL:
    """Load (building first if needed and possible) and declare the library."""
    global _LIB
    with _LOCK:
        if _LIB is not None:
            return _LIB
        path = library_path()
        if build_if_missing:
            try:
                path = _build.build()
            except RuntimeError:
                if not path.exists():
                    raise
        if not path.exists():
            raise RuntimeError(f"librl2.so not found at {path}; run robolearn_b200/build.py (needs nvcc)")
        lib = ctypes.CDLL(str(path))
        for name, (args, res) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.argtypes, fn.restype = args, res
        _LIB = lib
        return lib


def check(status: int, what: str) -> None:
    if status:
        message = load().rl2_last_error()
        detail = message.decode("utf-8", errors="replace") if message else "no native error message"
        raise RuntimeError(f"{what}: {detail}")


def created(handle, what: str):
    if not handle:
        message = load().rl2_last_error()
        raise RuntimeError(f"{what}: {message.decode('utf-8', errors='replace') if message else 'creation failed'}")
    return handle


def ptr(t) -> int | None:
    """Device address of a torch tensor (None passes a null pointer)."""
    return None if t is None else t.data_ptr()


def addr(x) -> int | None:
    """Device address of a tensor, or an integer address passed through; None stays null."""
    if x is None:
        return None
    if isinstance(x, int):
        return x
    return x.data_ptr()


def segment_table(rows, device):
    """Device table of optimizer units (offset, offset2, plane_offset, length, kind) for
    ``rl2_adam_step``: units short enough for one warp first (in their given order), then
    the rest. Returns (uint8 tensor, unit count, leading warp units)."""
    import torch

    lib = load()
    longest, warp_max = lib.rl2_segment_max_length(), lib.rl2_segment_warp_max_length()
    if any(r[3] > longest for r in rows):
        raise ValueError(f"a projection unit is longer than {longest} elements")
    ordered = [r for r in rows if r[3] <= warp_max] + [r for r in rows if r[3] > warp_max]
    warp_units = sum(1 for r in rows if r[3] <= warp_max)
    arr = (Segment * len(ordered))(*[Segment(offset=a, offset2=b, plane_offset=c, length=d, kind=e)
                                     for a, b, c, d, e in ordered])
    raw = torch.frombuffer(bytearray(bytes(arr)), dtype=torch.uint8).clone()
    return raw.to(device), len(ordered), warp_units


def stream_ptr(stream=None) -> int:
    import torch

    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


class ReplayIngestArgs(ctypes.Structure):
    """``rl2_replay_ingest_args`` (include/rl2.h)."""

    _fields_ = [
        ("obs", P), ("next_obs", P), ("ld_obs", LL), ("action", P), ("ld_action", LL), ("reward", P),
        ("terminated", P), ("truncated", P), ("terminated_u8", P), ("truncated_u8", P), ("num_envs", LL),
        ("obs_dim", I), ("act_dim", I), ("n_step", I), ("gamma", F),
        ("pend_obs", P), ("pend_next_obs", P), ("pend_act", P), ("pend_reward", P), ("pend_term", P),
        ("pend_trunc", P), ("counters", P), ("capacity", LL), ("r_obs", P), ("r_next_obs", P),
        ("ld_replay_obs", LL), ("r_act", P), ("ld_replay_act", LL), ("r_reward", P), ("r_term", P),
        ("r_trunc", P), ("r_discount", P),
    ]


SIGNATURES.update({
    "rl2_replay_ingest": ([ctypes.POINTER(ReplayIngestArgs), P], I),
    "rl2_reward_stats_update": ([P, P, P, P, P, P, I, F, P, F, P], I),
})

SIGNATURES["rl2_critic_objective_noalloc"] = ([ctypes.POINTER(CriticObjectiveArgs), P], I)


class PPOGaeArgs(ctypes.Structure):
    """``rl2_ppo_gae_args`` (include/rl2.h)."""

    _fields_ = [
        ("rewards", P), ("values", P), ("next_values", P), ("terminated", P), ("truncated", P),
        ("horizon", I), ("num_envs", I), ("gamma", F), ("gae_lambda", F), ("current_timeout_bootstrap", I),
        ("advantages", P), ("returns", P),
    ]


class PPOGatherArgs(ctypes.Structure):
    """``rl2_ppo_gather_args`` (include/rl2.h)."""

    _fields_ = [
        ("indices", P), ("offset", I), ("rows", I), ("obs_dim", I), ("act_dim", I),
        ("observations", P), ("actions", P), ("means", P), ("stds", P), ("log_probs", P), ("values", P),
        ("advantages", P), ("returns", P), ("obs_plane", Plane), ("batch_actions", P), ("batch_means", P),
        ("batch_stds", P), ("batch_log_probs", P), ("batch_values", P), ("batch_advantages", P),
        ("batch_returns", P),
    ]


class PPOLossArgs(ctypes.Structure):
    """``rl2_ppo_loss_args`` (include/rl2.h)."""

    _fields_ = [
        ("head", P), ("ld_head", LL), ("head_twin_stride", LL), ("std_param", P), ("rows", I), ("act", I),
        ("actions", P), ("old_log_probs", P), ("old_values", P), ("advantages", P), ("returns", P),
        ("clip_ratio", F), ("value_coefficient", F), ("entropy_coefficient", F), ("value_loss_scale", F),
        ("clip_value", I), ("std_type", I), ("std_min", F), ("std_max", F),
        ("loss", P), ("metrics", P), ("d_head", P), ("ld_d_head", LL), ("d_head_twin_stride", LL),
        ("d_plane", Plane), ("d_bias_actor", P), ("d_bias_critic", P), ("d_std_param", P),
        ("partials", P), ("counter", P),
    ]


SIGNATURES.update({
    "rl2_ppo_gae": ([ctypes.POINTER(PPOGaeArgs), P], I),
    "rl2_ppo_normalize_advantages": ([P, I, I, P, P, P, P], I),
    "rl2_ppo_partials": ([I], I),
    "rl2_ppo_permutation": ([ctypes.c_ulonglong, P, I, P, P, P], I),
    "rl2_ppo_gather": ([ctypes.POINTER(PPOGatherArgs), P], I),
    "rl2_ppo_loss": ([ctypes.POINTER(PPOLossArgs), P], I),
    "rl2_ppo_loss_partials": ([I, I], I),
    "rl2_ppo_kl": ([P, LL, P, P, P, I, I, I, F, F, F, P, P, P, P, P], I),
    "rl2_ppo_clip_gradients": ([P, LL, LL, LL, I, F, P, P, P, P], I),
})


class PPOSampleArgs(ctypes.Structure):
    """``rl2_ppo_sample_args`` (include/rl2.h)."""

    _fields_ = [
        ("head", P), ("ld_head", LL), ("head_twin_stride", LL), ("std_param", P), ("std_type", I),
        ("std_min", F), ("std_max", F), ("noise", P), ("rows", I), ("act", I), ("actions", P), ("log_probs", P),
        ("values", P), ("sampled_std", P),
    ]


class PPOStoreArgs(ctypes.Structure):
    """``rl2_ppo_store_args`` (include/rl2.h)."""

    _fields_ = [
        ("step", I), ("num_envs", I), ("obs_dim", I), ("act", I), ("observations", P), ("actions", P),
        ("log_probs", P), ("values", P), ("rewards", P), ("terminated", P), ("truncated", P), ("mean", P),
        ("ld_mean", LL), ("next_values", P), ("next_values_stride", LL), ("sampled_std", P),
        ("r_observations", P), ("r_actions", P), ("r_log_probs", P), ("r_values", P), ("r_rewards", P),
        ("r_terminated", P), ("r_truncated", P), ("r_next_values", P), ("r_means", P), ("r_stds", P),
    ]


SIGNATURES.update({
    "rl2_ppo_sample": ([ctypes.POINTER(PPOSampleArgs), P], I),
    "rl2_ppo_store": ([ctypes.POINTER(PPOStoreArgs), P], I),
})

SIGNATURES["rl2_normal_noise_rows"] = ([ctypes.c_ulonglong, P, LL, I, I, P, LL, P], I)

SIGNATURES.update({
    "rl2_bn_finalize_ranked": ([P, P, LL, I, LL, I, I, I, P, P, P, P, F, F, I, P], I),
    "rl2_bn_backward_finalize_ranked": ([P, P, LL, I, LL, I, I, I, P, P, LL, I, P, P, P], I),
})


class PeerReduceArgs(ctypes.Structure):
    """``rl2_peer_reduce_args`` (include/rl2.h)."""

    _fields_ = [("mean", P), ("n_mean", I), ("max", P), ("n_max", I), ("max_int", P), ("n_max_int", I)]


class SyncBNExchange(ctypes.Structure):
    """``rl2_syncbn_exchange`` (include/rl2.h)."""

    _fields_ = [("peer_data", P), ("peer_flags", P), ("epoch", P), ("world", I), ("rank", I), ("health", P),
                ("timeout_s", F)]


SIGNATURES.update({
    "rl2_syncbn_forward": ([P, P, LL, I, I, I, I, P, P, P, P, F, F, I, ctypes.POINTER(SyncBNExchange), P], I),
    "rl2_syncbn_backward": ([P, P, LL, I, I, I, P, P, LL, P, P, ctypes.POINTER(SyncBNExchange), P], I),
    "rl2_peer_reduce": ([ctypes.POINTER(PeerReduceArgs), ctypes.POINTER(SyncBNExchange), P], I),
    "rl2_syncbn_slot_data_bytes": ([I, I, I], LL),
    "rl2_syncbn_slot_flag_bytes": ([I, I, I], LL),
    "rl2_peer_mean": ([LL, ctypes.POINTER(SyncBNExchange), P], I),
    "rl2_peer_mean_flag_bytes": ([I], LL),
})
