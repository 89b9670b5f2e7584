"""ctypes binding of ``libf16env.so`` (the sm_100a kernels behind the C ABI in include/f16env.h).

The library is built in-tree by ``build.py``.  There is no fallback: if the library is
missing or cannot be loaded, importing the GPU entry points raises, so a GPU run can never
silently take a CPU path.
"""
import ctypes as C
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "libf16env.so"

STATE_N = 101
OBS17_N = 17
IC_N = 12
LAYOUT_SOA = 0
LAYOUT_AOS = 1

_P = C.c_void_p
_I64 = C.c_int64


class Recon(C.Structure):
    """f16_recon: device pointers to the reconstruction buffers (include/f16env.h)."""
    _fields_ = [(n, C.c_void_p) for n in ("hp", "fuel", "t_sec", "prev_att", "prev_valid", "pqr", "dmg_dealt",
                                          "dmg_taken", "hp_loss", "act_hist", "prev_x", "prev_x_valid",
                                          "prev_alt_log")]


class RewardCfg(C.Structure):
    _fields_ = [(n, C.c_double) for n in ("dt", "min_alt", "max_time", "own_damage_weight", "damage_scale",
                                          "shaping_reward_scale", "win_reward", "loss_reward",
                                          "timeout_win_reward", "timeout_loss_reward", "timeout_draw_reward",
                                          "alt_hunt_coef")] + [("reward_mode", C.c_int32), ("reserved", C.c_int32)]


class Origin(C.Structure):
    _fields_ = [(n, C.c_double) for n in ("ox", "oy", "oz", "slat", "clat", "slon", "clon")]


class FdmIO(C.Structure):
    """f16_fdm_io (include/f16env.h)."""
    _fields_ = [("cmd", C.c_void_p), ("bins", C.c_void_p), ("grid_host", C.c_void_p), ("num_bins", C.c_int),
                ("obs17", C.c_void_p), ("finite", C.c_void_p)]


class RecordArgs(C.Structure):
    """f16_record_args (include/f16env.h)."""
    _fields_ = [("reward", C.c_void_p), ("done", C.c_void_p), ("terminal_hp", C.c_void_p),
                ("terminal_alt", C.c_void_p), ("opp_row", C.c_void_p), ("n_opp", C.c_int), ("min_alt", C.c_double),
                ("finite", C.c_void_p), ("b_rew", C.c_void_p), ("next_done", C.c_void_p), ("ep_ret", C.c_void_p),
                ("ep_len", C.c_void_p), ("stats", C.c_void_p)]


class PayoffArgs(C.Structure):
    """f16_payoff_args (include/f16env.h)."""
    _fields_ = [("done", C.c_void_p), ("terminal_hp", C.c_void_p), ("terminal_alt", C.c_void_p),
                ("finite", C.c_void_p), ("reward", C.c_void_p), ("left_slot", C.c_void_p), ("lanes", C.c_int64),
                ("min_alt", C.c_double), ("step", C.c_int32), ("finished", C.c_void_p), ("scores", C.c_void_p),
                ("own_crash", C.c_void_p), ("opp_crash", C.c_void_p), ("finished_count", C.c_void_p),
                ("final_step", C.c_void_p), ("nonfinite", C.c_void_p), ("step_dev", C.c_void_p)]


_PR = C.POINTER(Recon)
_PC = C.POINTER(RewardCfg)
_PO = C.POINTER(Origin)

# name -> (argtypes, restype); keep in step with include/f16env.h
_SIGS = {
    "f16_obs_init_reward": ([_P, C.c_int, _I64, _I64, _P, _PR, _PO, _P], C.c_int),
    "f16_obs_advance": ([_P, C.c_int, _I64, _I64, _P, _PR, _PC, _PO, _P, _P, _P, _P], C.c_int),
    "f16_obs_build": ([_P, C.c_int, _I64, _I64, _P, _PR, _PO, _P, _P, _P], C.c_int),
    "f16_obs_step": ([_P, C.c_int, _I64, _I64, _P, _PR, _PC, _PO, _P, _P, _P, _P, _P, _P], C.c_int),
    "f16_env_post_step": ([_P, C.c_int, _I64, _I64, _P, _PR, _PC, _PO, _P, _I64, _P, _P, _P, _P, _P, _P, _P, _P,
                           _P, _P, _P], C.c_int),
    "f16_state9": ([_P, C.c_int, _I64, _I64, _PO, _P, _P], C.c_int),
    "f16_external_accel": ([_P, C.c_int, _I64, _I64, _P, _P, _P, _PO, C.c_double, _P], C.c_int),
    "f16_external_obs": ([_P, C.c_int, _I64, _I64, _P, _P, _P, _PO, _P], C.c_int),
    "f16_gae": ([_P, _P, _P, _P, _P, C.c_int, _I64, _I64, C.c_double, C.c_double, _P, _P, _P], C.c_int),
    "f16_mlp_set_create": ([_P, C.c_int, _P], C.c_int),
    "f16_mlp_set_destroy": ([_P], C.c_int),
    "f16_policy_forward": ([_P, _P, _P], C.c_int),
    "f16_norm_update": ([_P, _I64, C.c_int, _I64, _P, _P, _P, _P, _I64, _P], C.c_int),
    "f16_norm_scratch_doubles": ([_I64, C.c_int], _I64),
    "f16_norm_sums": ([_P, _I64, C.c_int, _I64, _P, _P, _I64, _P], C.c_int),
    "f16_norm_merge_sums": ([_P, _I64, C.c_int, _P, _P, _P, _P], C.c_int),
    "f16_norm_update_static": ([_P, _I64, C.c_int, _I64, _P, _P, _P, _P], C.c_int),
    "f16_norm_apply": ([_P, _I64, C.c_int, _I64, _P, _P, C.c_double, C.c_double, _P, _I64, _P, _I64, _P],
                       C.c_int),
    "f16_norm_apply_checked": ([_P, _I64, C.c_int, _I64, _P, _P, C.c_double, C.c_double, _P, _I64, _P, _I64, _P,
                                _P], C.c_int),
    "f16_norm_apply_half": ([_P, _I64, C.c_int, _I64, _P, _P, C.c_double, C.c_double, _P, _I64, _P, _I64, C.c_int,
                             _P, _P], C.c_int),
    "f16_norm_apply_scatter": ([_P, _I64, C.c_int, _I64, _P, _P, _P, _P, C.c_int, C.c_double, C.c_double, _P, _I64,
                                C.c_int, _P, _P], C.c_int),
    "f16_fdm_step": ([_P, C.c_int, _I64, _I64, _P, C.c_int, C.c_double, _P, _P], C.c_int),
    "f16_fdm_step_bins": ([_P, C.c_int, _I64, _I64, _P, _P, C.c_int, C.c_int, C.c_double, _P, _P], C.c_int),
    "f16_fdm_step_ex": ([_P, C.c_int, _I64, _I64, C.POINTER(FdmIO), C.c_int, C.c_double, _P], C.c_int),
    "f16_rollout_record": ([_I64, C.POINTER(RecordArgs), _P], C.c_int),
    "f16_payoff_record": ([_I64, C.POINTER(PayoffArgs), _P], C.c_int),
    "f16_split3_bf16": ([_P, _I64, C.c_int, _I64, _P, _I64, C.c_int, _P], C.c_int),
    "f16_bias_act_split": ([_P, _I64, C.c_int, _I64, _P, C.c_int, _P, _I64, C.c_int, _P], C.c_int),
    "f16_act_grad_split": ([_P, _I64, _P, _I64, _I64, C.c_int, C.c_int, _P, _I64, C.c_int, _P, C.c_int, _P],
                           C.c_int),
    "f16_bias_act_value": ([_P, _I64, C.c_int, _I64, _P, C.c_int, _P, _P, _P, _P], C.c_int),
    "f16_act_grad_split_value": ([_P, _P, _P, _I64, _I64, C.c_int, C.c_int, _P, _I64, C.c_int, _P, _P, C.c_int, _P],
                                 C.c_int),
    "f16_categorical_fwd": ([_P, _I64, _I64, C.c_int, C.c_int, _P, C.c_int, _P, _P, _P, _P], C.c_int),
    "f16_categorical_bwd": ([_P, _I64, _I64, C.c_int, C.c_int, _P, C.c_int, _P, _P, _P, _I64, _P], C.c_int),
    "f16_seed_ic": ([_P, _I64, _P, C.c_int, _I64, C.c_double, _P], C.c_int),
    "f16_probe_fp64": ([_P, _I64, C.c_int, C.POINTER(C.c_double), _P], C.c_int),
    "f16_version": ([], C.c_char_p),
    "f16_status_string": ([C.c_int], C.c_char_p),
}

_lib = None


def exported_symbols():
    return list(_SIGS)


def load(path=None):
    """Load (once) and return the library; raises OSError/FileNotFoundError if unavailable."""
    global _lib
    if _lib is None:
        p = Path(path) if path else LIB_PATH
        if not p.exists():
            raise FileNotFoundError(
                f"{p} is missing: build it with `python {HERE.name}/build.py` (no CPU fallback exists)")
        lib = C.CDLL(str(p))
        for name, (args, res) in _SIGS.items():
            fn = getattr(lib, name)
            fn.argtypes = args
            fn.restype = res
        _lib = lib
    return _lib


def check(rc, what):
    if rc != 0:
        msg = load().f16_status_string(int(rc)).decode()
        raise RuntimeError(f"{what} failed: status {rc} ({msg})")


def ptr(t):
    return C.c_void_p(t.data_ptr()) if t is not None else None


def stream_of(t):
    """Raw handle of the torch current stream on the tensor's device."""
    return C.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def require_cuda_tensor(t, dtype, shape, label, device=None):
    """Raise before any launch if a raw-pointer argument is not what the kernel reads
    (same contract as the reference's _kernel_input, R/cuda_fdm/obs_reward.py:391-401)."""
    if not torch.is_tensor(t) or t.dtype not in (dtype if isinstance(dtype, tuple) else (dtype,)):
        raise TypeError(f"{label} requires dtype {dtype}; no implicit pointer cast")
    if shape is not None and tuple(t.shape) != tuple(shape):
        raise ValueError(f"{label} shape {tuple(t.shape)} != {tuple(shape)}")
    if t.device.type != "cuda" or (device is not None and t.device != device):
        raise ValueError(f"{label} must be a CUDA tensor on {device}")
    return t
