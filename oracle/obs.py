"""ctypes front end of obs_oracle.c -- TEST INFRASTRUCTURE ONLY.

``ObsOracle`` holds the reference's per-aircraft reconstruction buffers (the attributes of
R/cuda_fdm/obs_reward.py BatchObsReward._alloc, :338-353) as numpy arrays and runs the C
restatement of obs_kernel.cu's three kernels over them.  States are (nac,101) AoS rows.
"""
import ctypes as C
import math

import numpy as np

from . import fdm as _fdm

_D = C.POINTER(C.c_double)
_U8 = C.POINTER(C.c_uint8)
_F = C.POINTER(C.c_float)
_bound = False

ORIGIN_LAT_DEG = 37.240778
ORIGIN_LON_DEG = 131.869556


def origin7():
    """Official-origin constants the reference passes to its kernels (obs_reward.py:376-383)."""
    olat, olon = math.radians(ORIGIN_LAT_DEG), math.radians(ORIGIN_LON_DEG)
    slat, clat, slon, clon = math.sin(olat), math.cos(olat), math.sin(olon), math.cos(olon)
    A, E2 = 6378137.0, 0.0066943799901411
    Nr = A / math.sqrt(1.0 - E2 * slat * slat)
    return np.array([Nr * clat * clon, Nr * clat * slon, Nr * (1.0 - E2) * slat, slat, clat, slon, clon])


def _lib():
    global _bound
    lb = _fdm.lib()
    if not _bound:
        lb.oracle_obs_init_reward.argtypes = [_D, _U8, _D, _U8, _D, _D, C.c_long, _D]
        lb.oracle_obs_advance.argtypes = [_D, _D, _D, _D, _D, _D, _U8, _D, _D, _D, _D, _D, _D, _U8, _D, _D, _U8,
                                          _U8, C.c_long, _D, _D, C.c_int]
        lb.oracle_obs_build.argtypes = [_D, _U8, _D, _D, _D, _D, _D, _D, _D, _F, C.c_long, _D, _D]
        lb.oracle_kin9.argtypes = [_D, C.c_long, _D, _D]
        lb.oracle_external_accel.argtypes = [_D, _U8, _D, _D, C.c_long, _D, C.c_double]
        lb.oracle_external_obs.argtypes = [_D, _D, _F, _F, C.c_long, _D]
        for f in ("oracle_obs_init_reward", "oracle_obs_advance", "oracle_obs_build", "oracle_kin9",
                  "oracle_external_accel", "oracle_external_obs"):
            getattr(lb, f).restype = None
        _bound = True
    return lb


def _p(a, t):
    return a.ctypes.data_as(t) if a is not None else None


# reward parameters in the order obs_oracle.c expects (R/cuda_fdm/obs_reward.py:410-438 defaults,
# MY_REWARD_CONFIG values of R/claude_code/my_reward.py:45-104)
DEFAULT_REWARD = dict(dt=0.1, min_alt=304.8, max_time=200.0, own_w=1.0, damage_scale=10.0,
                      shaping_reward_scale=0.0001, win_reward=5.0, loss_reward=-5.0, timeout_win_reward=5.0,
                      timeout_loss_reward=-5.0, timeout_draw_reward=-4.0, alt_hunt_coef=5.0)
_RP_ORDER = ("dt", "min_alt", "max_time", "own_w", "damage_scale", "shaping_reward_scale", "win_reward",
             "loss_reward", "timeout_win_reward", "timeout_loss_reward", "timeout_draw_reward", "alt_hunt_coef")


class ObsOracle:
    KEYS = ("hp", "fuel", "t_sec", "prev_att", "prev_valid", "pqr", "last_dmg_dealt", "last_dmg_taken", "hp_loss",
            "act_hist", "prev_x", "prev_x_valid", "prev_alt_log")

    def __init__(self, nenv):
        self.nenv, self.nac = nenv, 2 * nenv
        n = self.nac
        self.hp = np.ones(n)
        self.fuel = np.ones(n)
        self.t_sec = np.zeros(nenv)
        self.prev_att = np.zeros((n, 3))
        self.prev_valid = np.zeros(n, np.uint8)
        self.pqr = np.zeros((n, 3))
        self.last_dmg_dealt = np.zeros(n)
        self.last_dmg_taken = np.zeros(n)
        self.hp_loss = np.zeros(n)
        self.act_hist = np.zeros((n, 5, 4))
        self.prev_x = np.zeros(n)
        self.prev_x_valid = np.zeros(n, np.uint8)
        self.prev_alt_log = np.zeros(n)
        self.aux = None
        self.origin = origin7()

    def copy_from(self, other):
        for k in self.KEYS:
            setattr(self, k, np.array(getattr(other, k), copy=True))

    def init_reward(self, states, env_mask=None):
        st = np.ascontiguousarray(states, np.float64)
        m = None if env_mask is None else np.ascontiguousarray(env_mask, np.uint8)
        _lib().oracle_obs_init_reward(_p(st, _D), _p(m, _U8), _p(self.prev_x, _D), _p(self.prev_x_valid, _U8),
                                      _p(self.prev_alt_log, _D), _p(self.t_sec, _D), self.nenv,
                                      _p(self.origin, _D))

    def advance(self, states, actions, mode=0, **cfg):
        p = dict(DEFAULT_REWARD, **cfg)
        rp = np.array([p[k] for k in _RP_ORDER], dtype=np.float64)
        st = np.ascontiguousarray(states, np.float64)
        ac = np.ascontiguousarray(actions, np.float64)
        reward = np.zeros(self.nac)
        term = np.zeros(self.nenv, np.uint8)
        trunc = np.zeros(self.nenv, np.uint8)
        _lib().oracle_obs_advance(
            _p(st, _D), _p(ac, _D), _p(self.hp, _D), _p(self.fuel, _D), _p(self.t_sec, _D), _p(self.prev_att, _D),
            _p(self.prev_valid, _U8), _p(self.pqr, _D), _p(self.last_dmg_dealt, _D), _p(self.last_dmg_taken, _D),
            _p(self.hp_loss, _D), _p(self.act_hist, _D), _p(self.prev_x, _D), _p(self.prev_x_valid, _U8),
            _p(self.prev_alt_log, _D), _p(reward, _D), _p(term, _U8), _p(trunc, _U8), self.nenv, _p(self.origin, _D),
            _p(rp, _D), int(mode))
        return reward, term, trunc

    def build_obs(self, states, env_mask=None, obs=None, aux=False):
        st = np.ascontiguousarray(states, np.float64)
        out = np.zeros((self.nac, 184), np.float32) if obs is None else obs
        m = None if env_mask is None else np.ascontiguousarray(env_mask, np.uint8)
        ax = np.zeros((self.nenv, 21)) if aux else None
        _lib().oracle_obs_build(_p(st, _D), _p(m, _U8), _p(self.hp, _D), _p(self.fuel, _D), _p(self.t_sec, _D),
                                _p(self.pqr, _D), _p(self.last_dmg_dealt, _D), _p(self.last_dmg_taken, _D),
                                _p(self.act_hist, _D), out.ctypes.data_as(_F), self.nac, _p(self.origin, _D),
                                _p(ax, _D))
        return (out, ax) if aux else out

    def kin9(self, states):
        st = np.ascontiguousarray(states, np.float64)
        out = np.zeros((st.shape[0], 9))
        _lib().oracle_kin9(_p(st, _D), st.shape[0], _p(self.origin, _D), _p(out, _D))
        return out


def external_accel(states, valid, previous, accel, dt=0.1):
    """oracle_external_accel over (nac,101) states; previous / accel (nac,3) updated in place."""
    st = np.ascontiguousarray(states, dtype=np.float64)
    o7 = origin7()
    _lib().oracle_external_accel(_p(st, _D), _p(np.ascontiguousarray(valid, dtype=np.uint8), _U8),
                                 _p(previous, _D), _p(accel, _D), st.shape[0], _p(o7, _D), float(dt))


def external_obs(states, accel, obs184):
    """oracle_external_obs: (nac,214) float32 rows from (nac,101) states, (nac,3) accelerations
    and the (nac,184) observation rows."""
    st = np.ascontiguousarray(states, dtype=np.float64)
    acc = np.ascontiguousarray(accel, dtype=np.float64)
    orig = np.ascontiguousarray(obs184, dtype=np.float32)
    out = np.zeros((st.shape[0], 214), dtype=np.float32)
    o7 = origin7()
    _lib().oracle_external_obs(_p(st, _D), _p(acc, _D), _p(orig, _F), _p(out, _F), st.shape[0], _p(o7, _D))
    return out


_REF = None


def ref_available():
    from pathlib import Path
    return (Path(__file__).resolve().parent / "_ref" / "libobsref.so").exists()


def _ref():
    """The reference's own obs_kernel.cu + external_observation.cu, host-compiled (oracle/_ref)."""
    global _REF
    if _REF is None:
        from pathlib import Path
        lb = C.CDLL(str(Path(__file__).resolve().parent / "_ref" / "libobsref.so"))
        lb.ref_obs_init_reward.argtypes = [_D, _U8, _D, _U8, _D, _D, C.c_int, _D]
        lb.ref_obs_advance.argtypes = [_D, _D, _D, _D, _D, _D, _U8, _D, _D, _D, _D, _D, _D, _U8, _D, _D, _U8, _U8,
                                       C.c_int, _D, _D, C.c_int]
        lb.ref_obs_build.argtypes = [_D, _U8, _D, _D, _D, _D, _D, _D, _D, _F, C.c_int, _D, _D]
        lb.ref_external_accel.argtypes = [_D, _U8, _D, _D, C.c_int, _D, C.c_double]
        lb.ref_external_obs.argtypes = [_D, _D, _F, _F, C.c_int, _D]
        for f in ("ref_obs_init_reward", "ref_obs_advance", "ref_obs_build", "ref_external_accel",
                  "ref_external_obs"):
            getattr(lb, f).restype = None
        _REF = lb
    return _REF


class ObsRef(ObsOracle):
    """Same buffers and calls as ObsOracle, run through the reference's own kernels."""

    def init_reward(self, states, env_mask=None):
        st = np.ascontiguousarray(states, np.float64)
        m = np.ones(self.nenv, np.uint8) if env_mask is None else np.ascontiguousarray(env_mask, np.uint8)
        _ref().ref_obs_init_reward(_p(st, _D), _p(m, _U8), _p(self.prev_x, _D), _p(self.prev_x_valid, _U8),
                                   _p(self.prev_alt_log, _D), _p(self.t_sec, _D), self.nenv, _p(self.origin, _D))

    def advance(self, states, actions, mode=0, **cfg):
        p = dict(DEFAULT_REWARD, **cfg)
        rp = np.array([p[k] for k in _RP_ORDER], dtype=np.float64)
        st = np.ascontiguousarray(states, np.float64)
        ac = np.ascontiguousarray(actions, np.float64)
        reward = np.zeros(self.nac)
        term = np.zeros(self.nenv, np.uint8)
        trunc = np.zeros(self.nenv, np.uint8)
        _ref().ref_obs_advance(
            _p(st, _D), _p(ac, _D), _p(self.hp, _D), _p(self.fuel, _D), _p(self.t_sec, _D), _p(self.prev_att, _D),
            _p(self.prev_valid, _U8), _p(self.pqr, _D), _p(self.last_dmg_dealt, _D), _p(self.last_dmg_taken, _D),
            _p(self.hp_loss, _D), _p(self.act_hist, _D), _p(self.prev_x, _D), _p(self.prev_x_valid, _U8),
            _p(self.prev_alt_log, _D), _p(reward, _D), _p(term, _U8), _p(trunc, _U8), self.nenv, _p(self.origin, _D),
            _p(rp, _D), int(mode))
        return reward, term, trunc

    def build_obs(self, states, env_mask=None, obs=None, aux=False):
        st = np.ascontiguousarray(states, np.float64)
        out = np.zeros((self.nac, 184), np.float32) if obs is None else obs
        m = np.ones(self.nenv, np.uint8) if env_mask is None else np.ascontiguousarray(env_mask, np.uint8)
        ax = np.zeros((self.nenv, 21)) if aux else None
        _ref().ref_obs_build(_p(st, _D), _p(m, _U8), _p(self.hp, _D), _p(self.fuel, _D), _p(self.t_sec, _D),
                             _p(self.pqr, _D), _p(self.last_dmg_dealt, _D), _p(self.last_dmg_taken, _D),
                             _p(self.act_hist, _D), out.ctypes.data_as(_F), self.nac, _p(self.origin, _D),
                             _p(ax, _D))
        return (out, ax) if aux else out


def ref_external_accel(states, valid, previous, accel, dt=0.1):
    st = np.ascontiguousarray(states, dtype=np.float64)
    o7 = origin7()
    _ref().ref_external_accel(_p(st, _D), _p(np.ascontiguousarray(valid, dtype=np.uint8), _U8), _p(previous, _D),
                              _p(accel, _D), st.shape[0], _p(o7, _D), float(dt))


def ref_external_obs(states, accel, obs184):
    st = np.ascontiguousarray(states, dtype=np.float64)
    acc = np.ascontiguousarray(accel, dtype=np.float64)
    orig = np.ascontiguousarray(obs184, dtype=np.float32)
    out = np.zeros((st.shape[0], 214), dtype=np.float32)
    o7 = origin7()
    _ref().ref_external_obs(_p(st, _D), _p(acc, _D), _p(orig, _F), _p(out, _F), st.shape[0], _p(o7, _D))
    return out
