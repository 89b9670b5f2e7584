"""The observation / reward oracle (oracle/obs_oracle.c) pinned against the reference's own torch
path (R/cuda_fdm/obs_reward.py BatchObsReward, enable_kernel=False) recorded in
tests/golden/obs_traj.npz -- CPU only.

Tolerances: BASELINE's obs/reward bound |a - b| <= 1e-5 * max(1, |b|); termination and
truncation flags bit-exact; HP / fuel / time exact to 1e-12 (the reference's own kernel-vs-
torch check, R/cuda_fdm/tests/obs_reward_val.py:164-218, bounds obs 5e-4, reward 5e-3,
hp 1e-9, pqr 1e-6).  The oracle follows the fused kernel's kin9 (epa rotation + closed-form
geodetic) while the torch path goes through kinematics_state, so they agree to ~1e-9, not bit
for bit.
"""
import numpy as np
import pytest

from conftest import GOLDEN
from oracle import fdm as ofdm
from oracle.obs import ObsOracle


def within(a, b, tol):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return np.max(np.abs(a - b) / np.maximum(1.0, np.abs(b))) <= tol


@pytest.fixture(scope="module")
def g():
    return np.load(GOLDEN / "obs_traj.npz")


def replay(g):
    nenv = g["seeds"].shape[0] // 2
    o = ObsOracle(nenv)
    o.hp[:] = g["hp0"]
    o.fuel[:] = g["fuel0"]
    o.t_sec[:] = g["t0"]
    o.init_reward(g["seeds"])
    yield "init", o, None
    states = g["seeds"]
    for k in range(g["actions"].shape[0]):
        states, _ = ofdm.oracle_step(states, g["actions"][k], 6, 1.0 / 60.0, with_obs=False)
        reward, term, trunc = o.advance(states, g["actions"][k])
        obs = o.build_obs(states)
        yield k, o, (states, reward, term, trunc, obs)


def test_kin9_matches_reference_state9(g):
    o = ObsOracle(g["seeds"].shape[0] // 2)
    states = g["seeds"]
    for k in range(2):
        states, _ = ofdm.oracle_step(states, g["actions"][k], 6, 1.0 / 60.0, with_obs=False)
    s9 = o.kin9(states)
    ref = g["s9"][1]
    np.testing.assert_allclose(s9[:, :3], ref[:, :3], rtol=0, atol=1e-6)       # metres
    d = np.abs(s9[:, 3:6] - ref[:, 3:6])
    d = np.minimum(d, 360.0 - d)
    assert d.max() < 1e-9                                                         # degrees
    np.testing.assert_allclose(s9[:, 6:], ref[:, 6:], rtol=0, atol=1e-9)        # m/s


def test_oracle_matches_reference_torch_path(g):
    for k, o, out in replay(g):
        if k == "init":
            assert within(o.prev_x, g["init_prev_x"], 1e-9)
            np.testing.assert_array_equal(o.prev_x_valid, g["init_prev_x_valid"].astype(np.uint8))
            assert within(o.prev_alt_log, g["init_prev_alt_log"], 1e-12)
            continue
        states, reward, term, trunc, obs = out
        np.testing.assert_array_equal(term.astype(bool), g["term"][k])
        np.testing.assert_array_equal(trunc.astype(bool), g["trunc"][k])
        assert within(obs, g["obs"][k], 1e-5), f"step {k} obs"
        assert within(reward, g["reward"][k], 1e-5), f"step {k} reward"
        for key, mine in (("hp", o.hp), ("fuel", o.fuel), ("t_sec", o.t_sec), ("hp_loss", o.hp_loss),
                          ("dealt", o.last_dmg_dealt), ("taken", o.last_dmg_taken)):
            assert within(mine, g[key][k], 1e-9), f"step {k} {key}"
        assert within(o.pqr, g["pqr"][k], 1e-6), f"step {k} pqr"
        assert within(o.prev_x, g["prev_x"][k], 1e-9), f"step {k} prev_x"
        assert within(o.prev_alt_log, g["prev_alt_log"][k], 1e-9), f"step {k} prev_alt_log"
        np.testing.assert_array_equal(o.act_hist, g["act_hist"][k])


def test_fixture_exercises_the_contract(g):
    """The fixture must contain damage, HP and altitude terminations and time-limit truncation."""
    assert g["dealt"].max() > 0
    assert g["term"].any() and g["trunc"].any()
    assert (g["hp"] <= 0).any()
    assert (-g["s9"][..., 2] < 304.8).any()
