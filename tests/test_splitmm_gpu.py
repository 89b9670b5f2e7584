"""fp32-accurate split products (splitmm) on a B200.

* f16_split3_bf16: hi + lo + mid reproduces every fp32 input to within 2^-24 relative.
* SplitLinear forward, input gradient and weight gradient against fp64 references: errors no
  larger than 4x those of fp32 SGEMM on the same operands (and below 5e-6 of the largest
  output; TF32 products are near 1e-3), for the update's layer shapes (184 -> 512, 512 -> 512)
  with 65,536 rows -- the weight gradient's reduction over the rows accumulates in the tensor
  cores' fp32 adders, measured at 2-3.5x SGEMM's error.
* A PPO update on the GPU with split products and one with plain fp32 matmuls give the same
  statistics within 1e-4 and parameters within 1e-5 relative.
"""
import pytest
import torch

from conftest import pkg_module

pytestmark = pytest.mark.gpu


def rel(a, ref):
    return float((a.double() - ref).abs().max() / ref.abs().max())


def test_split3_reconstructs(cuda):
    sm = pkg_module("splitmm")
    g = torch.Generator(device=cuda).manual_seed(1)
    x = torch.randn(1000, 184, device=cuda, generator=g) * torch.exp(torch.randn(1000, 184, device=cuda, generator=g) * 5)
    s = sm.split3(x)
    back = s[:, :184].double() + s[:, 184:368].double() + s[:, 368:].double()
    assert float(((back - x.double()).abs() / x.double().abs().clamp_min(1e-30)).max()) <= 2.0 ** -24


@pytest.mark.parametrize("k,n", [(184, 512), (512, 512)])
def test_split_linear_matches_fp64(cuda, k, n):
    sm = pkg_module("splitmm")
    torch.backends.cuda.matmul.allow_tf32 = False
    g = torch.Generator(device=cuda).manual_seed(k + n)
    m = 65536
    x = torch.randn(m, k, device=cuda, generator=g).requires_grad_(True)
    w = (torch.randn(n, k, device=cuda, generator=g) / k ** 0.5).requires_grad_(True)
    b = torch.randn(n, device=cuda, generator=g).requires_grad_(True)
    gy = torch.randn(m, n, device=cuda, generator=g)
    y = sm.SplitLinear.apply(x, w, b)
    y.backward(gy)
    xd, wd, gd = x.detach().double(), w.detach().double(), gy.double()
    ry = xd @ wd.t() + b.detach().double()
    rgx, rgw = gd @ wd, gd.t() @ xd
    y32 = x.detach() @ w.detach().t() + b.detach()
    gx32, gw32 = gy @ w.detach(), gy.t() @ x.detach()
    for got, ref, base in ((y.detach(), ry, y32), (x.grad, rgx, gx32), (w.grad, rgw, gw32)):
        e, e32 = rel(got, ref), rel(base, ref)
        assert e <= max(4.0 * e32, 1e-7) and e <= 5e-6, (e, e32)


def test_ppo_update_split_vs_fp32(cuda):
    tr = pkg_module("trainer")
    torch.backends.cuda.matmul.allow_tf32 = False
    T, n = 4, 2048
    g = torch.Generator(device=cuda).manual_seed(7)
    obs = torch.randn(T, n, 184, device=cuda, generator=g)
    act = torch.randint(0, 21, (T, n, 4), device=cuda, generator=g).to(torch.uint8)
    old_logp = -torch.rand(T, n, device=cuda, generator=g) * 12
    b_val = torch.randn(T, n, device=cuda, generator=g)
    adv = torch.randn(T, n, device=cuda, generator=g)
    ret = b_val + adv
    res, params = [], []
    for split in (True, False):
        torch.manual_seed(3)
        model = tr.MLPActorCritic(hidden=(512, 512), activation="relu").to(cuda)
        cfg = tr.PPOConfig(update_epochs=2, num_minibatches=4, target_kl=None, hidden=(512, 512), activation="relu")
        a_opt = torch.optim.Adam(model.actor_parameters(), lr=cfg.lr, eps=1e-5)
        c_opt = torch.optim.Adam(model.critic_parameters(), lr=cfg.lr, eps=1e-5)
        gen = torch.Generator(device=cuda).manual_seed(11)
        r = tr.ppo_update(model, a_opt, c_opt, cfg, obs, act, old_logp, b_val, adv, ret, generator=gen,
                          split_products=split)
        res.append(r)
        params.append([p.detach().clone() for p in model.parameters()])
    for key in ("pl", "vl", "ent", "kl"):
        a, b = float(res[0][key]), float(res[1][key])
        assert abs(a - b) <= 1e-4 * max(1.0, abs(b)), (key, a, b)
    for p, q in zip(*params):
        assert float((p - q).abs().max()) <= 1e-5 * max(1.0, float(q.abs().max()))
