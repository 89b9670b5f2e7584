"""GAE and RunningNorm kernels vs the reference (golden) and the oracle -- needs a B200.

GAE must be bit-exact (each op rounded as torch rounds it); RunningNorm statistics and
normalised observations within 1e-5 relative (fp64 reduction vs torch's fp32 reduction).
"""
import numpy as np
import pytest
import torch

from conftest import GOLDEN, pkg_module
from oracle import gae as og
from test_oracle_rollout import norm_inputs

pytestmark = pytest.mark.gpu


def test_gae_bit_exact_vs_reference_loop(cuda):
    ro = pkg_module("rollout")
    g = np.load(GOLDEN / "gae.npz")
    for tag in ("ref", "cfg4"):
        gamma, lam = g[f"{tag}_gamma_lam"]
        t = lambda k: torch.as_tensor(g[f"{tag}_{k}"]).to(cuda)
        adv, ret = ro.gae(t("rew"), t("val"), t("done"), t("last_val"), t("next_done"), float(gamma), float(lam))
        np.testing.assert_array_equal(adv.cpu().numpy(), g[f"{tag}_adv"])
        np.testing.assert_array_equal(ret.cpu().numpy(), g[f"{tag}_ret"])


def test_gae_full_size_vs_oracle(cuda):
    """BASELINE cfg4 buffer: T = 64, 131,072 envs."""
    ro = pkg_module("rollout")
    T, n = 64, 131072
    gen = torch.Generator(device=cuda).manual_seed(3)
    rew = torch.randn(T, n, device=cuda, generator=gen)
    val = torch.randn(T, n, device=cuda, generator=gen)
    done = (torch.rand(T, n, device=cuda, generator=gen) < 0.02).float()
    lv = torch.randn(n, device=cuda, generator=gen)
    nd = (torch.rand(n, device=cuda, generator=gen) < 0.02).float()
    adv, ret = ro.gae(rew, val, done, lv, nd, 0.99, 0.95)
    cols = slice(0, 4096)
    eadv, eret = og.gae(rew[:, cols].cpu().numpy(), val[:, cols].cpu().numpy(), done[:, cols].cpu().numpy(),
                        lv[cols].cpu().numpy(), nd[cols].cpu().numpy(), 0.99, 0.95)
    np.testing.assert_array_equal(adv[:, cols].cpu().numpy(), eadv)
    np.testing.assert_array_equal(ret[:, cols].cpu().numpy(), eret)


def test_running_norm_vs_reference(cuda):
    ro = pkg_module("rollout")
    g = np.load(GOLDEN / "norm.npz")
    xs = [torch.as_tensor(x).to(cuda) for x in norm_inputs(g["seed"])]
    rn = ro.RunningNorm(184, cuda)
    for i in range(3):
        rn.update(xs[i])
        np.testing.assert_allclose(rn.mean.cpu().numpy(), g[f"mean{i}"], rtol=1e-5, atol=1e-6)
        np.testing.assert_allclose(rn.var.cpu().numpy(), g[f"var{i}"], rtol=1e-5, atol=1e-6)
        assert abs(float(rn.count) - float(g[f"count{i}"])) <= 1e-6 * float(g[f"count{i}"])
    y = rn.normalize(xs[3])
    np.testing.assert_allclose(y.cpu().numpy(), g["yt"], rtol=1e-5, atol=1e-5)
    yf = torch.empty_like(y)
    yb = rn.normalize_bf16(xs[3], out_f32=yf)
    assert yb.shape == (24, 192)
    assert torch.equal(yb[:, :184], yf.to(torch.bfloat16)) and bool((yb[:, 184:] == 0).all())
    assert torch.equal(yf, y)
