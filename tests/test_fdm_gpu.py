"""FDM + FCS kernel (f16_fdm_step) and GPU IC seeder vs the oracle -- needs a B200.

Tolerances: one-frame state error <= 1e-9 relative, where relative
means |got - exp| <= 1e-9 * max(|exp|, floor) with the per-column physical floor of
oracle.fdm.STATE_FLOOR (1 ft, 1 ft/s, 1 ft/s^2, ... for dimensional columns, 1e-3 for
angles, rates and normalised values), so columns that are zero up to rounding noise (e.g.
the lateral body acceleration of a wings-level seed) are not compared relative to that
noise; 600-frame divergence is reported as RMS position / attitude error, bounded loosely.
"""
import numpy as np
import pytest
import torch

from conftest import GOLDEN, pkg_module
from oracle import fdm as ofdm

pytestmark = pytest.mark.gpu

TOL_FRAME = 1e-9


def scaled_err(got, exp):
    floor = ofdm.OBS17_FLOOR if np.shape(exp)[-1] == 17 else ofdm.STATE_FLOOR
    return ofdm.state_rel_err(got, exp, floor)


@pytest.fixture(scope="module")
def cfg1():
    return np.load(GOLDEN / "fdm_cfg1.npz")


@pytest.fixture(scope="module")
def mods():
    return pkg_module("gpu_env"), pkg_module("ic")


def cmds(ic, bins):
    return ic.bins_to_commands(torch.as_tensor(bins)).double().numpy()


def make_sim(mods, nenv, seeds, fcs_dt, cuda):
    ge, _ = mods
    sim = ge.GpuDogfight(nenv, substeps=6, fcs_dt=fcs_dt, device=cuda)
    sim.load_seed(torch.as_tensor(seeds))
    return sim


def test_one_frame_parity(cfg1, mods, cuda):
    _, ic = mods
    c = cmds(ic, cfg1["bins"][0])
    sim = make_sim(mods, 64, cfg1["seeds"], float(cfg1["fcs_dt"]), cuda)
    obs = sim.step(torch.as_tensor(c), substeps=1)
    got = sim.states.cpu().numpy()
    exp, exp_obs = ofdm.oracle_step(cfg1["seeds"], c, 1, float(cfg1["fcs_dt"]))
    err = scaled_err(got, exp)
    assert err.max() <= TOL_FRAME, f"max scaled err {err.max():.3e} at col {np.argmax(err.max(0))}"
    oerr = scaled_err(obs.reshape(-1, 17).cpu().numpy(), exp_obs)
    assert oerr.max() <= TOL_FRAME, f"obs17 err {oerr.max():.3e}"


def test_one_decision_parity_and_history_slots(cfg1, mods, cuda):
    """6 frames in one launch (only the surviving history slots are stored) vs the oracle."""
    _, ic = mods
    c = cmds(ic, cfg1["bins"][0])
    sim = make_sim(mods, 64, cfg1["seeds"], float(cfg1["fcs_dt"]), cuda)
    sim.step(torch.as_tensor(c))
    exp, _ = ofdm.oracle_step(cfg1["seeds"], c, 6, float(cfg1["fcs_dt"]))
    err = scaled_err(sim.states.cpu().numpy(), exp)
    assert err.max() <= 1e-9, f"max scaled err {err.max():.3e} at col {np.argmax(err.max(0))}"


@pytest.mark.parametrize("ss", [1, 2, 3, 4])
def test_substep_split_matches(cfg1, mods, cuda, ss):
    """k launches of ss frames == oracle over k*ss frames (history shifting for ss < 3)."""
    _, ic = mods
    c = cmds(ic, cfg1["bins"][1])
    sim = make_sim(mods, 64, cfg1["seeds"], float(cfg1["fcs_dt"]), cuda)
    for _ in range(12 // ss):
        sim.step(torch.as_tensor(c), substeps=ss)
    exp, _ = ofdm.oracle_step(cfg1["seeds"], c, 12, float(cfg1["fcs_dt"]))
    err = scaled_err(sim.states.cpu().numpy(), exp)
    assert err.max() <= 1e-8, f"ss={ss}: max scaled err {err.max():.3e}"


def test_600_frame_trajectory_drift(cfg1, mods, cuda):
    """100 decisions x 6 frames; RMS position (ft) and attitude (rad) drift vs the oracle."""
    _, ic = mods
    sim = make_sim(mods, 64, cfg1["seeds"], float(cfg1["fcs_dt"]), cuda)
    for d in range(100):
        obs = sim.step(torch.as_tensor(cmds(ic, cfg1["bins"][d])))
    got = obs.reshape(-1, 17).cpu().numpy()
    exp = cfg1["obs17_f600"]          # the reference's own fdm.cuh (oracle/_ref), bit-equal to the oracle
    pos_rms = np.sqrt(np.mean(np.sum((got[:, 0:3] - exp[:, 0:3]) ** 2, axis=1)))
    d_att = np.angle(np.exp(1j * (got[:, 6:9] - exp[:, 6:9])))
    att_rms = np.sqrt(np.mean(d_att ** 2))
    print(f"600-frame drift: RMS position {pos_rms:.3e} ft, RMS attitude {att_rms:.3e} rad")
    assert pos_rms < 1.0 and att_rms < 1e-3


def test_layouts_and_bins_agree(cfg1, mods, cuda):
    """SoA vs AoS state and fp64 commands vs in-kernel action bins give identical states."""
    ge, ic = mods
    lib = pkg_module("_lib")
    L = lib.load()
    bins = torch.as_tensor(cfg1["bins"][2]).to(cuda)
    c = ic.bins_to_commands(bins).double().contiguous()
    a = make_sim(mods, 64, cfg1["seeds"], float(cfg1["fcs_dt"]), cuda)
    a.step(c)
    b = make_sim(mods, 64, cfg1["seeds"], float(cfg1["fcs_dt"]), cuda)
    b.step_bins(bins.contiguous())
    torch.testing.assert_close(a.states, b.states, rtol=0, atol=0)
    aos = torch.as_tensor(cfg1["seeds"]).to(cuda).contiguous()
    obs = torch.zeros(128, 17, dtype=torch.float64, device=cuda)
    lib.check(L.f16_fdm_step(lib.ptr(aos), lib.LAYOUT_AOS, 101, 128, lib.ptr(c), 6, float(cfg1["fcs_dt"]),
                             lib.ptr(obs), lib.stream_of(aos)), "aos step")
    torch.testing.assert_close(aos, a.states, rtol=0, atol=0)


def test_gpu_seeder_matches_oracle(cfg1, mods, cuda):
    ge, ic = mods
    sim = ge.GpuDogfight(64, substeps=6, fcs_dt=float(cfg1["fcs_dt"]), device=cuda)
    sim.reset_ic_rows(cfg1["ic"])
    got = sim.states.cpu().numpy()
    exp = ofdm.oracle_seed(cfg1["ic"], float(cfg1["fcs_dt"]))
    err = scaled_err(got, exp)
    assert err.max() <= 1e-9, f"seed err {err.max():.3e} at col {np.argmax(err.max(0))}"


def test_reset_ic_dicts(cfg1, mods, cuda):
    ge, ic = mods
    rows = cfg1["ic"][:4]
    dicts = [dict(lat_deg=r[0], lon_deg=r[1], alt_ft=r[2], vt_fps=r[3], phi_deg=r[4], theta_deg=r[5],
                  psi_deg=r[6], alpha_deg=r[7], beta_deg=r[8], fuel_lbs=r[9], throttle=0.8) for r in rows]
    sim = ge.GpuDogfight(2, fcs_dt=float(cfg1["fcs_dt"]), device=cuda)
    sim.reset_ic(dicts)
    exp = ofdm.oracle_seed(rows, float(cfg1["fcs_dt"]))
    assert scaled_err(sim.states.cpu().numpy(), exp).max() <= 1e-9


def test_step_host_matches_step(cfg1, mods, cuda):
    """The host-driven, slice-pipelined step gives step()'s states and obs17 bit for bit."""
    ge, ic = mods
    fcs_dt = float(cfg1["fcs_dt"])
    a = make_sim(mods, 64, cfg1["seeds"], fcs_dt, cuda)
    b = make_sim(mods, 64, cfg1["seeds"], fcs_dt, cuda)
    out = torch.empty(128, 17, dtype=torch.float64).pin_memory()
    for k in range(3):
        c = ic.bins_to_commands(torch.as_tensor(cfg1["bins"][k]).to(cuda)).double().contiguous()
        oa = a.step(c).reshape(128, 17).clone()
        ob = b.step_host(c.cpu().pin_memory(), out, chunks=3)
        torch.cuda.synchronize()
        torch.testing.assert_close(a.states, b.states, rtol=0, atol=0)
        torch.testing.assert_close(oa.cpu(), ob.reshape(128, 17), rtol=0, atol=0)


def envelope_ics(n, seed):
    """IC rows spread over the flight envelope's edges: 300 ft to 80,000 ft (troposphere,
    tropopause and both stratosphere layers), 150 to 1,900 ft/s (subsonic through Mach ~1.9,
    which runs the supersonic calibrated-airspeed iteration), alpha -15..45 deg, beta +-20 deg,
    rolled / inverted / steep attitudes, nearly empty to full tanks."""
    rng = np.random.default_rng(seed)
    rows = np.zeros((n, 12))
    rows[:, 0] = 37.24 + rng.uniform(-1.0, 1.0, n)
    rows[:, 1] = 131.87 + rng.uniform(-1.0, 1.0, n)
    rows[:, 2] = rng.choice([300.0, 5000.0, 36089.0, 45000.0, 65000.0, 80000.0], n)
    rows[:, 3] = rng.choice([150.0, 400.0, 900.0, 1300.0, 1900.0], n)
    rows[:, 4] = rng.choice([0.0, 90.0, -170.0], n)
    rows[:, 5] = rng.choice([-80.0, 0.0, 60.0], n)
    rows[:, 6] = rng.uniform(0.0, 360.0, n)
    rows[:, 7] = rng.choice([-15.0, 0.0, 25.0, 45.0], n)
    rows[:, 8] = rng.choice([-20.0, 0.0, 15.0], n)
    rows[:, 9] = rng.choice([50.0, 3000.0, 6000.0], n)
    return rows


@pytest.mark.parametrize("fcs_dt", [1.0 / 120.0, 1.0 / 60.0])
def test_envelope_edges_and_edge_commands(mods, cuda, fcs_dt):
    """Extreme states under full-deflection / afterburner / idle / zero commands, 1, 2, 3 and 7
    frames per launch: GPU vs oracle within the one-frame tolerance for one frame and within
    1e-8 (scaled) over several, with non-finite values (if any) in the same places."""
    ge, _ = mods
    n = 256
    rows = envelope_ics(n, 20260108)
    seeds = ofdm.oracle_seed(rows, fcs_dt)
    assert np.isfinite(seeds).all()
    cmds_ = [np.tile([1.0, -1.0, 1.0, 1.0], (n, 1)), np.tile([-1.0, 1.0, -1.0, 0.0], (n, 1)),
             np.zeros((n, 4)), np.tile([0.3, 0.44, -0.2, 0.55], (n, 1))]
    worst = {}
    for ci, c in enumerate(cmds_):
        for ss in (1, 2, 3, 7):
            sim = ge.GpuDogfight(n // 2, substeps=ss, fcs_dt=fcs_dt, device=cuda)
            sim.load_seed(torch.as_tensor(seeds))
            obs = sim.step(torch.as_tensor(c).to(cuda), substeps=ss).reshape(n, 17).cpu().numpy()
            got = sim.states.cpu().numpy()
            exp, exp_obs = ofdm.oracle_step(seeds, c, ss, fcs_dt)
            fin = np.isfinite(exp)
            assert np.array_equal(np.isfinite(got), fin), f"cmd {ci} ss {ss}: non-finite pattern differs"
            rows_ok = fin.all(axis=1)
            err = scaled_err(got[rows_ok], exp[rows_ok]).max()
            oerr = scaled_err(obs[rows_ok], exp_obs[rows_ok]).max()
            worst[(ci, ss)] = (err, oerr)
            bound = TOL_FRAME if ss == 1 else 1e-8
            assert err <= bound and oerr <= bound, f"cmd {ci} ss {ss}: state {err:.3e} obs17 {oerr:.3e}"
    print("worst scaled error per (command, frames):",
          {k: f"{v[0]:.1e}/{v[1]:.1e}" for k, v in worst.items()})
