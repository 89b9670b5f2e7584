"""The observation / reward oracle (oracle/obs_oracle.c) against the reference's OWN kernels,
host-compiled from research/competition_36500/runtime/cuda_fdm/gen/obs_kernel.cu and
external_observation.cu (oracle/_ref/libobsref.so, built by oracle/build.py) -- CPU only.

Both run in lockstep over FDM trajectories that reach damage, hard-deck and HP terminations:
states from the C FDM oracle, identical inputs every step, all four reward modes.  Bound: every
fp64 output within 1e-12 relative (floor 1), observations and flags identical (both are C
restatements of the same fp64 expressions compiled with contraction off).  The external 214-D
observation and its acceleration state are compared the same way.  Skipped where the reference
tree was not available to build libobsref.so.
"""
import numpy as np
import pytest

from conftest import GOLDEN
from oracle import fdm as ofdm
from oracle import obs as oobs

pytestmark = pytest.mark.skipif(not oobs.ref_available(), reason="oracle/_ref/libobsref.so not built")


def close(a, b, tol=1e-12):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.max(np.abs(a - b) / np.maximum(1.0, np.abs(b)))) if a.size else 0.0


@pytest.mark.parametrize("mode", [0, 1, 2, 3])
def test_oracle_equals_reference_kernels(mode):
    g = np.load(GOLDEN / "obs_traj.npz")
    nenv = g["seeds"].shape[0] // 2
    mine, ref = oobs.ObsOracle(nenv), oobs.ObsRef(nenv)
    for o in (mine, ref):
        o.hp[:] = g["hp0"]; o.fuel[:] = g["fuel0"]; o.t_sec[:] = g["t0"]
        o.init_reward(g["seeds"])
    for k in oobs.ObsOracle.KEYS:
        assert close(getattr(mine, k), getattr(ref, k)) <= 1e-12, k
    rng = np.random.default_rng(40 + mode)
    states = g["seeds"]
    prev_m, acc_m = np.zeros((2 * nenv, 3)), np.zeros((2 * nenv, 3))
    prev_r, acc_r = np.zeros((2 * nenv, 3)), np.zeros((2 * nenv, 3))
    nterm = 0
    for step in range(40):
        acts = g["actions"][step] if step < g["actions"].shape[0] else np.clip(
            rng.normal(0.0, 0.6, (2 * nenv, 4)), -1.0, 1.0) * np.array([1, 1, 1, 0.5]) + np.array([0, 0, 0, 0.5])
        states, _ = ofdm.oracle_step(states, acts, 6, 1.0 / 60.0, with_obs=False)
        # the external acceleration runs before the advance (obs_reward.py:417-420)
        oobs.external_accel(states, mine.prev_valid, prev_m, acc_m)
        oobs.ref_external_accel(states, ref.prev_valid, prev_r, acc_r)
        assert close(acc_m, acc_r) <= 1e-12 and close(prev_m, prev_r) <= 1e-12, f"step {step} external accel"
        rm, tm, cm = mine.advance(states, acts, mode)
        rr, tr, cr = ref.advance(states, acts, mode)
        np.testing.assert_array_equal(tm, tr)
        np.testing.assert_array_equal(cm, cr)
        assert close(rm, rr) <= 1e-12, f"step {step} reward"
        for k in oobs.ObsOracle.KEYS:
            assert close(getattr(mine, k), getattr(ref, k)) <= 1e-12, f"step {step} {k}"
        om, am = mine.build_obs(states, aux=True)
        orr, ar = ref.build_obs(states, aux=True)
        np.testing.assert_array_equal(om, orr)
        assert close(am, ar) <= 1e-12
        np.testing.assert_array_equal(oobs.external_obs(states, acc_m, om), oobs.ref_external_obs(states, acc_r, orr))
        nterm += int(tm.sum())
    assert nterm > 0, "the trajectory should reach terminations"
