"""GAE / RunningNorm oracles (oracle/gae.py) pinned against the reference (CPU only).

gae.npz holds the reference trainer's own GAE loop run with torch fp32 (bit-exact target) and
the reference test's independent numpy reference _ref_gae (fp64; its own bound is 1e-5,
R/.. cuda_fdm/tests/ppo_gpu_val.py:94).  norm.npz holds the reference RunningNorm's state after
three updates and a normalize; inputs are regenerated from the stored seed.
"""
import numpy as np
import torch

from conftest import GOLDEN
from oracle import gae as og


def norm_inputs(seed):
    g = torch.Generator().manual_seed(int(seed))
    xs = [torch.randn(B, 184, generator=g) * torch.linspace(0.1, 3.0, 184) + torch.linspace(-2, 2, 184)
          for B in (512, 1000, 37)]
    xs.append(torch.randn(24, 184, generator=g) * 40.0)
    return [x.numpy() for x in xs]


def test_gae_oracle_bit_exact_vs_reference_loop():
    g = np.load(GOLDEN / "gae.npz")
    for tag in ("ref", "cfg4"):
        gamma, lam = g[f"{tag}_gamma_lam"]
        adv, ret = og.gae(g[f"{tag}_rew"], g[f"{tag}_val"], g[f"{tag}_done"], g[f"{tag}_last_val"],
                          g[f"{tag}_next_done"], float(gamma), float(lam))
        np.testing.assert_array_equal(adv, g[f"{tag}_adv"])
        np.testing.assert_array_equal(ret, g[f"{tag}_ret"])
        assert np.abs(adv - g[f"{tag}_ref64"]).max() < 1e-4 * max(1.0, np.abs(g[f"{tag}_ref64"]).max())


def test_running_norm_oracle_vs_reference():
    g = np.load(GOLDEN / "norm.npz")
    xs = norm_inputs(g["seed"])
    mean, var, count = np.zeros(184, np.float32), np.ones(184, np.float32), np.float32(1e-4)
    for i in range(3):
        mean, var, count = og.running_norm_update(mean, var, count, xs[i])
        np.testing.assert_allclose(mean, g[f"mean{i}"], rtol=1e-5, atol=1e-6)
        np.testing.assert_allclose(var, g[f"var{i}"], rtol=1e-5, atol=1e-6)
        assert abs(count - g[f"count{i}"]) <= 1e-6 * count
    y = og.running_norm_apply(xs[3], mean, var)
    np.testing.assert_allclose(y, g["yt"], rtol=1e-5, atol=1e-5)
