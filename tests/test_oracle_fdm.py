"""The FDM oracle (oracle/fdm_oracle.c) pinned against the reference itself (CPU only).

* seeds: the oracle's IC seeder must reproduce the reference's Python build_seed_vector rows
  stored in tests/golden (bit for bit: same libm, same operation order);
* frames: the oracle must reproduce the reference's own fdm.cuh (host-compiled, oracle/_ref)
  trajectories stored in tests/golden, bit for bit, for both FCS-dt lineages.
"""
import sys
from pathlib import Path

import numpy as np
import pytest

from conftest import GOLDEN
from oracle import fdm as ofdm


@pytest.fixture(scope="module")
def cfg1():
    return np.load(GOLDEN / "fdm_cfg1.npz")


@pytest.fixture(scope="module")
def r36():
    return np.load(GOLDEN / "fdm_r36.npz")


def bins_to_cmd(bins):
    import torch
    from conftest import pkg_module
    return pkg_module("ic").bins_to_commands(torch.as_tensor(bins)).double().numpy()


def test_oracle_seed_matches_reference_python(cfg1, r36):
    # The reference's Python atmosphere / air-data helpers evaluate a few expressions in a
    # different order than its fdm.cuh (which the oracle follows), so the seed rows agree to
    # ~1e-14 relative rather than bit for bit.
    for g in (cfg1, r36):
        mine = ofdm.oracle_seed(g["ic"], float(g["fcs_dt"]))
        np.testing.assert_allclose(mine, g["seeds"], rtol=1e-12, atol=1e-12)


def test_oracle_one_frame_and_one_decision_bit_exact(cfg1):
    cmd = bins_to_cmd(cfg1["bins"][0])
    s1, _ = ofdm.oracle_step(cfg1["seeds"], cmd, 1, float(cfg1["fcs_dt"]))
    np.testing.assert_array_equal(s1, cfg1["state_f1"])
    s6, _ = ofdm.oracle_step(cfg1["seeds"], cmd, 6, float(cfg1["fcs_dt"]))
    np.testing.assert_array_equal(s6, cfg1["state_f6"])


def test_oracle_600_frames_bit_exact(cfg1):
    s = cfg1["seeds"]
    obs = None
    for d in range(cfg1["bins"].shape[0]):
        s, obs = ofdm.oracle_step(s, bins_to_cmd(cfg1["bins"][d]), 6, float(cfg1["fcs_dt"]))
    np.testing.assert_array_equal(s, cfg1["state_f600"])
    np.testing.assert_array_equal(obs, cfg1["obs17_f600"])


def test_oracle_r36_lineage_bit_exact(r36):
    s = r36["seeds"]
    for d in range(r36["bins"].shape[0]):
        s, obs = ofdm.oracle_step(s, bins_to_cmd(r36["bins"][d]), 6, float(r36["fcs_dt"]))
    np.testing.assert_array_equal(s, r36["state_f60"])
    np.testing.assert_array_equal(obs, r36["obs17_f60"])


@pytest.mark.skipif(not ofdm.ref_available("root"), reason="oracle/_ref not built (needs the reference tree)")
def test_oracle_matches_ref_on_edge_commands(cfg1):
    """Full-deflection, afterburner and zero commands, odd substep counts."""
    seeds = cfg1["seeds"][:16]
    cmds = [np.tile([1.0, -1.0, 1.0, 1.0], (16, 1)), np.tile([-1.0, 1.0, -1.0, 0.0], (16, 1)),
            np.zeros((16, 4)), np.tile([0.3, 0.44, -0.2, 0.55], (16, 1))]
    for c in cmds:
        for ss in (1, 2, 3, 7):
            a, oa = ofdm.oracle_step(seeds, c, ss, 1.0 / 120.0)
            b, ob = ofdm.ref_step(seeds, c, ss, "root")
            np.testing.assert_array_equal(a, b)
            np.testing.assert_array_equal(oa, ob)


@pytest.mark.skipif(not (ofdm.ref_available("root") and ofdm.ref_available("r36")),
                    reason="oracle/_ref not built (needs the reference tree)")
def test_oracle_matches_ref_at_envelope_edges():
    """The envelope-edge ICs of the GPU test (300-80,000 ft, up to Mach ~1.9, extreme attitudes)
    under edge commands: the oracle equals the reference's fdm.cuh bit for bit, both lineages."""
    sys.path.insert(0, str(Path(__file__).resolve().parent))
    from test_fdm_gpu import envelope_ics
    rows = envelope_ics(256, 20260108)
    for lineage, dt in (("root", 1.0 / 120.0), ("r36", 1.0 / 60.0)):
        seeds = ofdm.oracle_seed(rows, dt)
        for c in ([1.0, -1.0, 1.0, 1.0], [-1.0, 1.0, -1.0, 0.0], [0.0] * 4, [0.3, 0.44, -0.2, 0.55]):
            cm = np.tile(c, (256, 1))
            for ss in (1, 7):
                a, oa = ofdm.oracle_step(seeds, cm, ss, dt)
                b, ob = ofdm.ref_step(seeds, cm, ss, lineage)
                np.testing.assert_array_equal(a, b)
                np.testing.assert_array_equal(oa, ob)
