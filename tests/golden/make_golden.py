#!/usr/bin/env python3
"""Regenerate the golden fixtures in tests/golden/ from the reference itself.

Run only where the reference tree is available (``F16_REFERENCE`` or /root/reference); the
GPU box never runs this.  What each fixture pins:

fdm_cfg1.npz  BASELINE configs[0]: 64 envs x 2 F-16s, seeded ICs (altitude U(6,9) km, Mach
              U(0.6,0.9), head-on 10 km apart, heading offsets U(-30,30) deg, fuel 6000 lb)
              whose seed rows come from the reference's Python ``cuda_fdm.ic.build_seed_vector``;
              random 4x21-bin actions held 6 frames, 100 decisions; states after 1, 6 and 600
              frames and obs17 after 600 frames from the reference's own fdm.cuh (oracle/_ref,
              repository-root lineage, FCS dt 1/120).
fdm_r36.npz   the same ICs (first 16 envs) through the research/competition_36500 lineage
              (FCS dt 1/60) seed builder and fdm.cuh, 60 frames.
"""
import importlib
import os
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
REF = Path(os.environ.get("F16_REFERENCE", "/root/reference"))
OUT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

from oracle import fdm as ofdm  # noqa: E402

pkg = importlib.import_module("2026_ai_pilot_challenge-1st_solution_b200")
ic_mod = importlib.import_module(pkg.__name__ + ".ic")

SEED_CFG1 = 20260101
NENV_CFG1 = 64


def ref_seed_rows(ic_rows, lineage_root):
    """Seed rows through the reference's Python build_seed_vector of one lineage."""
    for k in list(sys.modules):
        if k == "cuda_fdm" or k.startswith("cuda_fdm."):
            del sys.modules[k]
    sys.path.insert(0, str(lineage_root))
    try:
        from cuda_fdm.ic import build_seed_vector
        out = []
        for r in ic_rows:
            out.append(build_seed_vector(lat_deg=r[0], lon_deg=r[1], alt_ft=r[2], vt_fps=r[3], phi_deg=r[4],
                                         theta_deg=r[5], psi_deg=r[6], alpha_deg=r[7], beta_deg=r[8],
                                         fuel_lbs=r[9], throttle=0.8))
        return np.array(out)
    finally:
        sys.path.remove(str(lineage_root))


def bins_to_cmd_np(bins):
    """Reference action_to_env in float32 (R/cuda_fdm/ppo_gpu.py:361-369), widened to float64."""
    import torch
    return ic_mod.bins_to_commands(torch.as_tensor(bins)).double().numpy()


def main():
    ics = ic_mod.baseline_ics(NENV_CFG1, SEED_CFG1)
    rng = np.random.default_rng(SEED_CFG1 + 1)
    bins = rng.integers(0, 21, size=(100, 2 * NENV_CFG1, 4), dtype=np.uint8)
    seeds = ref_seed_rows(ics, REF)
    s = seeds.copy()
    snaps = {}
    obs600 = None
    for dcs in range(100):
        cmd = bins_to_cmd_np(bins[dcs])
        if dcs == 0:
            s1, _ = ofdm.ref_step(s, cmd, 1, "root")
            snaps["state_f1"] = s1
        s, obs = ofdm.ref_step(s, cmd, 6, "root")
        if dcs == 0:
            snaps["state_f6"] = s.copy()
        obs600 = obs
    np.savez_compressed(OUT / "fdm_cfg1.npz", ic=ics, seeds=seeds, bins=bins, state_f1=snaps["state_f1"],
                        state_f6=snaps["state_f6"], state_f600=s, obs17_f600=obs600,
                        fcs_dt=np.array(1.0 / 120.0))
    print("fdm_cfg1.npz", seeds.shape)

    r36 = REF / "research" / "competition_36500" / "runtime"
    ics16 = ics[:32]
    seeds16 = ref_seed_rows(ics16, r36)
    s = seeds16.copy()
    for dcs in range(10):
        s, obs = ofdm.ref_step(s, bins_to_cmd_np(bins[dcs, :32]), 6, "r36")
    np.savez_compressed(OUT / "fdm_r36.npz", ic=ics16, seeds=seeds16, bins=bins[:10, :32], state_f60=s,
                        obs17_f60=obs, fcs_dt=np.array(1.0 / 60.0))
    print("fdm_r36.npz", seeds16.shape)


if __name__ == "__main__":
    main()
