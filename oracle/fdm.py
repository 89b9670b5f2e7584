"""ctypes front end of the FDM parity checkers -- TEST INFRASTRUCTURE ONLY.

``oracle_step`` / ``oracle_seed`` run fdm_oracle.c (our restatement of cuda_fdm/gen/fdm.cuh
and cuda_fdm/ic.py); ``ref_step`` runs the reference's own fdm.cuh compiled into
oracle/_ref (see oracle/build.py).  Arrays are numpy float64, states in the reference's
(nac,101) AoS order.
"""
import ctypes as C
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
_P = C.POINTER(C.c_double)
_lib = None
_ref = {}


def _ptr(a):
    return a.ctypes.data_as(_P)


def lib():
    global _lib
    if _lib is None:
        path = HERE / "liboracle.so"
        if not path.exists():
            from . import build
            build.build_oracle()
        _lib = C.CDLL(str(path))
        _lib.oracle_fdm_step.argtypes = [_P, _P, C.c_long, C.c_int, C.c_double, _P]
        _lib.oracle_fdm_step.restype = C.c_int
        _lib.oracle_seed_ic.argtypes = [_P, C.c_double, _P]
        _lib.oracle_seed_ic.restype = C.c_int
    return _lib


def ref_lib(lineage="root"):
    """The reference's own fdm.cuh; lineage 'root' (FCS dt 1/120) or 'r36' (1/60)."""
    if lineage not in _ref:
        path = HERE / "_ref" / f"libf16ref_{lineage}.so"
        if not path.exists():
            from . import build
            build.build_ref()
        if not path.exists():
            raise FileNotFoundError(f"{path} missing (needs the reference tree to build)")
        lb = C.CDLL(str(path))
        lb.f16ref_step.argtypes = [_P, _P, C.c_long, C.c_int, _P, C.c_int]
        lb.f16ref_step.restype = C.c_int
        lb.f16ref_fcs_dt.restype = C.c_double
        lb.f16ref_max_threads.restype = C.c_int
        _ref[lineage] = lb
    return _ref[lineage]


def ref_available(lineage="root"):
    try:
        ref_lib(lineage)
        return True
    except (FileNotFoundError, OSError):
        return False


def _prep(states, cmd):
    states = np.ascontiguousarray(states, dtype=np.float64)
    cmd = np.ascontiguousarray(cmd, dtype=np.float64)
    assert states.ndim == 2 and states.shape[1] == 101, states.shape
    assert cmd.shape == (states.shape[0], 4), cmd.shape
    return states, cmd


def oracle_step(states, cmd, substeps=1, fcs_dt=1.0 / 120.0, with_obs=True):
    """Advance copies of ``states`` by ``substeps`` frames; returns (states, obs17 or None)."""
    st, cm = _prep(states, cmd)
    st = st.copy()
    obs = np.zeros((st.shape[0], 17)) if with_obs else None
    rc = lib().oracle_fdm_step(_ptr(st), _ptr(cm), st.shape[0], int(substeps), float(fcs_dt),
                               _ptr(obs) if obs is not None else None)
    assert rc == 0
    return st, obs


def ref_step(states, cmd, substeps=1, lineage="root", with_obs=True, nthreads=0):
    st, cm = _prep(states, cmd)
    st = st.copy()
    obs = np.zeros((st.shape[0], 17)) if with_obs else None
    rc = ref_lib(lineage).f16ref_step(_ptr(st), _ptr(cm), st.shape[0], int(substeps),
                                      _ptr(obs) if obs is not None else None, int(nthreads))
    assert rc == 0
    return st, obs


def oracle_seed(ic_rows, fcs_dt=1.0 / 120.0):
    """ic_rows (n, 12) in include/f16env.h F16_IC_* column order -> (n, 101) seed rows."""
    ic = np.ascontiguousarray(np.atleast_2d(ic_rows), dtype=np.float64)
    out = np.zeros((ic.shape[0], 101))
    for i in range(ic.shape[0]):
        row = np.ascontiguousarray(ic[i])
        o = np.zeros(101)
        assert lib().oracle_seed_ic(_ptr(row), float(fcs_dt), _ptr(o)) == 0
        out[i] = o
    return out


# Physical floor (in each column's own unit) below which a state value counts as zero for the
# relative-error test: 1 ft, 1 ft/s, 1 ft/s^2, 1 lb, 1 kt, 1 % rpm, 1 pph for dimensional
# columns; 1e-3 for angles, rates, quaternion components, load factors and normalised values.
def _state_floor():
    f = np.full(101, 1e-3)
    f[0:6] = 1.0          # eci_pos ft, eci_vel ft/s
    f[14] = 1.0           # fuel lb
    f[15:18] = 1.0        # ECI acceleration ft/s^2
    f[46:64] = 1.0        # position / acceleration integrator histories
    f[64:67] = 1.0        # previous body acceleration ft/s^2
    f[75] = 1.0           # vc kts
    f[76] = 1.0           # vg ft/s
    f[82:84] = 1.0        # N1, N2 %
    f[85] = 1.0           # fuel flow pph
    return f


STATE_FLOOR = _state_floor()
# obs17: eci_pos ft, eci_vel ft/s, euler rad, uvw ft/s, alpha, beta rad, mach, Vt ft/s, alt ft
OBS17_FLOOR = np.array([1, 1, 1, 1, 1, 1, 1e-3, 1e-3, 1e-3, 1, 1, 1, 1e-3, 1e-3, 1e-3, 1, 1], dtype=np.float64)


def state_rel_err(got, exp, floor=STATE_FLOOR):
    """|got - exp| / max(|exp|, floor[column]) elementwise (the parity-tolerance metric)."""
    got = np.asarray(got, dtype=np.float64)
    exp = np.asarray(exp, dtype=np.float64)
    return np.abs(got - exp) / np.maximum(np.abs(exp), floor[None, :])
