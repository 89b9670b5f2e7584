"""External 214-D observation (f16_external_accel / f16_external_obs through
BatchObsReward.enable_external_observations / build_external_obs) vs the C oracle, which is
itself pinned to the reference's own external_observation.cu (tests/test_oracle_obs_ref.py) --
needs a B200.

Trajectory: the golden observation scenario (tests/golden/obs_traj.npz) stepped by the FDM
oracle; per step the acceleration state is updated before the advance, as kernel_advance does,
and the 214-D rows are built.  Bounds: accelerations within 1e-9 relative (floor 1 m/s^2),
observation rows within BASELINE's 1e-5 * max(1, |b|); the 164 + 20 copied columns equal the
184-D rows exactly.
"""
import numpy as np
import pytest
import torch

from conftest import GOLDEN, pkg_module
from oracle import fdm as ofdm
from oracle import obs as oobs

pytestmark = pytest.mark.gpu


def within(a, b, tol):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.max(np.abs(a - b) / np.maximum(1.0, np.abs(b))))


def test_external_rows_match_oracle(cuda):
    OR = pkg_module("obs_reward")
    g = np.load(GOLDEN / "obs_traj.npz")
    nenv = g["seeds"].shape[0] // 2
    b = OR.BatchObsReward(nenv, device=cuda)
    b.enable_external_observations()
    o = oobs.ObsOracle(nenv)
    b.hp.copy_(torch.as_tensor(g["hp0"])); b.fuel.copy_(torch.as_tensor(g["fuel0"]))
    b.t_sec.copy_(torch.as_tensor(g["t0"]))
    o.hp[:] = g["hp0"]; o.fuel[:] = g["fuel0"]; o.t_sec[:] = g["t0"]
    st = torch.as_tensor(g["seeds"], device=cuda)
    b.kernel_init_reward_state(st)
    o.init_reward(g["seeds"])
    prev, acc = np.zeros((2 * nenv, 3)), np.zeros((2 * nenv, 3))
    states = g["seeds"]
    for k in range(g["actions"].shape[0]):
        states, _ = ofdm.oracle_step(states, g["actions"][k], 6, 1.0 / 60.0, with_obs=False)
        st = torch.as_tensor(states, device=cuda)
        act = torch.as_tensor(g["actions"][k], device=cuda)
        b.kernel_advance(st, act)
        ext = b.build_external_obs(st)
        oobs.external_accel(states, o.prev_valid, prev, acc)
        o.advance(states, g["actions"][k])
        obs184 = o.build_obs(states)
        exp = oobs.external_obs(states, acc, obs184)
        torch.cuda.synchronize()
        assert within(b.external_accel.cpu().numpy(), acc, 0) <= 1e-9, f"step {k} accel"
        got = ext.cpu().numpy()
        assert within(got, exp, 0) <= 1e-5, f"step {k} 214-D rows"
        mine184 = b.obs_buf.cpu().numpy()
        np.testing.assert_array_equal(got[:, :164], mine184[:, :164])
        np.testing.assert_array_equal(got[:, 194:], mine184[:, 164:])
    assert float(np.abs(acc).max()) > 0.0
