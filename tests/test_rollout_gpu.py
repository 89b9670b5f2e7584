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


def test_checked_normalise_cast_and_nonfinite_count(cuda):
    """f16_norm_apply_checked: normalise equals f16_norm_apply bit for bit (fp32 and bf16 rows,
    strided input); mean = var = NULL casts the rows unchanged into the zero-padded bf16 layout;
    the counter stays 0 on finite data and counts a planted NaN row."""
    ro = pkg_module("rollout")
    rn = ro.RunningNorm(184, cuda)
    g = torch.Generator(device=cuda).manual_seed(11)
    src = torch.randn(3000, 368, device=cuda, generator=g) * 4.0
    x = src[:, :184]                                      # ldx 368, as the env's (nenv, 2, 184) view
    rn.update(x)
    y1, y2 = torch.empty(3000, 184, device=cuda), torch.empty(3000, 184, device=cuda)
    b1 = torch.full((3000, 192), 7.0, device=cuda).to(torch.bfloat16)
    b2 = b1.clone()
    L = pkg_module("_lib")
    lib = L.load()
    L.check(lib.f16_norm_apply(L.ptr(x), 3000, 184, 368, L.ptr(rn.mean), L.ptr(rn.var), rn.eps, rn.clip, L.ptr(y1),
                               184, L.ptr(b1), 192, L.stream_of(x)), "apply")
    cnt = torch.zeros(1, dtype=torch.int32, device=cuda)
    rn.normalize_bf16(x, out_f32=y2, out_bf16=b2, nonfinite=cnt)
    torch.cuda.synchronize()
    assert torch.equal(y1, y2) and torch.equal(b1, b2) and int(cnt) == 0
    assert bool((b2[:, 184:] == 0).all())
    ref = ((x - rn.mean) / torch.sqrt(rn.var + rn.eps)).clamp(-rn.clip, rn.clip)
    assert torch.equal(y2, ref)
    # pass-through cast
    c = torch.full((3000, 192), 5.0, device=cuda).to(torch.bfloat16)
    ro.cast_bf16(x, c)
    torch.cuda.synchronize()
    assert torch.equal(c[:, :184], x.to(torch.bfloat16)) and bool((c[:, 184:] == 0).all())
    # a NaN in the input is counted
    src[17, 5] = float("nan")
    rn.normalize_bf16(x, out_f32=y2, out_bf16=b2, nonfinite=cnt)
    torch.cuda.synchronize()
    assert int(cnt) >= 1 and bool(torch.isnan(y2[17, 5]))


@pytest.mark.parametrize("rows,dim", [(131_072, 184), (5_000, 184), (777, 12), (4_096, 1_024), (333, 7)])
def test_sums_then_merge_equals_update(cuda, rows, dim):
    """The data-parallel form of the norm update (per-feature fp64 sums, then a merge of the
    summed pairs: f16_norm_sums + f16_norm_merge_sums, what each rank runs around its
    all-reduce) gives f16_norm_update's mean, var and count bit for bit on one rank, over three
    updates; the partial sums of both come from the same kernel in the same order."""
    ro = pkg_module("rollout")
    L = pkg_module("_lib")
    lib = L.load()
    g = torch.Generator(device=cuda).manual_seed(rows + dim)
    a, b = ro.RunningNorm(dim, cuda), ro.RunningNorm(dim, cuda)
    scratch = torch.empty(int(lib.f16_norm_scratch_doubles(rows, dim)), dtype=torch.float64, device=cuda)
    sums = torch.empty(2 * dim, dtype=torch.float64, device=cuda)
    for i in range(3):
        x = torch.randn(rows, dim, device=cuda, generator=g) * (1.0 + i) + 0.25 * i
        a.update(x)
        s = L.stream_of(x)
        L.check(lib.f16_norm_sums(L.ptr(x), rows, dim, x.stride(0), L.ptr(sums), L.ptr(scratch), scratch.numel(), s),
                "sums")
        L.check(lib.f16_norm_merge_sums(L.ptr(sums), rows, dim, L.ptr(b.mean), L.ptr(b.var), L.ptr(b.count), s),
                "merge_sums")
        torch.cuda.synchronize()
        assert torch.equal(a.mean, b.mean) and torch.equal(a.var, b.var) and torch.equal(a.count, b.count)


@pytest.mark.parametrize("rows", [131_075, 70_001])
def test_normalise_rollout_batch_bit_exact(cuda, rows):
    """At rollout sizes (each block then takes more than the minimum row share, and the last block
    a ragged remainder) the fp32 rows equal torch's (x - mean) / sqrt(var + eps) clamped, bit for
    bit, and the 16-bit rows are those values rounded, with zero padding, for both operands."""
    ro = pkg_module("rollout")
    g = torch.Generator(device=cuda).manual_seed(rows)
    src = torch.randn(rows, 368, device=cuda, generator=g) * 3.0 + 0.5
    x = src[:, 184:]                                      # the opponent half of a (nenv, 2, 184) view
    rn = ro.RunningNorm(184, cuda)
    rn.update(x)
    ref = ((x - rn.mean) / torch.sqrt(rn.var + rn.eps)).clamp(-rn.clip, rn.clip)
    for dtype in (torch.float16, torch.bfloat16):
        yf = torch.full((rows, 184), 3.0, device=cuda)
        yh = rn.normalize_half(x, out_f32=yf, dtype=dtype)
        torch.cuda.synchronize()
        assert torch.equal(yf, ref)
        assert torch.equal(yh[:, :184], ref.to(dtype)) and bool((yh[:, 184:] == 0).all())
        c = torch.full((rows, 192), 5.0, device=cuda).to(dtype)        # the cast without a normaliser
        ro.cast_half(x, c)
        torch.cuda.synchronize()
        assert torch.equal(c[:, :184], x.to(dtype)) and bool((c[:, 184:] == 0).all())


def test_norm_apply_half_fp16(cuda):
    """f16_norm_apply_half with the fp16 operand: the fp16 rows are the fp32 rows rounded to
    nearest (zero padding beyond the features), values past fp16's range saturate at +-65504,
    and the bf16 operand reproduces f16_norm_apply_checked bit for bit."""
    ro = pkg_module("rollout")
    g = torch.Generator(device=cuda).manual_seed(4)
    x = torch.randn(3000, 184, device=cuda, generator=g) * 3.0
    rn = ro.RunningNorm(184, cuda)
    rn.update(x)
    yf = torch.zeros(3000, 184, device=cuda)
    yh = rn.normalize_half(x, out_f32=yf, dtype=torch.float16)
    assert yh.dtype == torch.float16
    assert torch.equal(yh[:, :184], yf.to(torch.float16)) and bool((yh[:, 184:] == 0).all())
    yb = rn.normalize_half(x, dtype=torch.bfloat16)
    assert torch.equal(yb, rn.normalize_bf16(x))
    big = torch.tensor([[1e6, -1e6, 70000.0, 1.5] + [0.0] * 180], device=cuda)
    c = torch.full((1, 192), 9.0, device=cuda).to(torch.float16)
    ro.cast_half(big, c)
    assert c[0, :4].tolist() == [65504.0, -65504.0, 65504.0, 1.5] and bool((c[0, 184:] == 0).all())
