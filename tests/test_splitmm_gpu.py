"""fp32-accurate split products (splitmm) on a B200.

* f16_split3_bf16: the parts are [mid | lo | hi] with hi = bf16(v), and mid + lo + hi reproduces
  every fp32 input to within 2^-24 relative; a width that is not a multiple of 8 gets zero pad
  columns in each part; the six-part layout repeats [lo | hi | hi].
* f16_bias_act_split: act(y + b) equal to torch's F.linear bias add followed by nn.ReLU /
  nn.Identity (bit for bit, NaN kept by relu) or nn.Tanh (within 1 ulp), and its split.
* f16_act_grad_split: torch's threshold_backward / tanh_backward / identity, its split, and the
  bias gradient (the column sums) against fp64 sums.
* A SplitBlock product (forward, input gradient, weight gradient) against fp64 references: errors
  no larger than 2.5x those of fp32 SGEMM on the same operands and below 2e-6 of the largest
  output (measured: 0.2-1.7x SGEMM's at 65,536 rows, below SGEMM's at the update's 524,288;
  TF32 products are 2e-4..1.4e-3), for the update's layer shapes (184 -> 512, 512 -> 512,
  512 -> 84 with zero-padded parts) with 65,536 rows, and 512 -> 512 at the update's 524,288-row
  minibatch (pytest -s prints the errors).
* A whole actor tower (84 logits) and critic tower (the value head fused into the last hidden
  layer) through run_tower against the same tower in fp64: output within 1e-5 relative, every
  parameter gradient within 1e-5 for tanh towers; for relu towers within 3x the error of torch's
  own fp32 tower (ReLU mask flips at pre-activations within rounding of zero move whole
  gradient rows in any fp32 evaluation); the reference's final shape (three 384-wide tanh
  layers) within 1e-5 for both towers.
* The fused categorical head against torch.distributions.Categorical: log-prob, entropy and the
  logits gradient within 1e-5, infinite logits included; NaN logits and out-of-range actions
  raise ValueError as torch's argument validation does.
* A PPO update on the GPU with split products and one with plain fp32 matmuls give the same
  statistics within 1e-4 and parameters within 1e-5 relative.
"""
import pytest
import torch

from conftest import pkg_module

pytestmark = pytest.mark.gpu


def rel(a, ref):
    return float((a.double() - ref).abs().max() / ref.abs().max())


def recon(s, cols):
    p = (cols + 7) & ~7
    return s[:, :cols].double() + s[:, p:p + cols].double() + s[:, 2 * p:2 * p + cols].double()


def test_split3_reconstructs(cuda):
    sm = pkg_module("splitmm")
    g = torch.Generator(device=cuda).manual_seed(1)
    x = torch.randn(1000, 184, device=cuda, generator=g) * torch.exp(torch.randn(1000, 184, device=cuda, generator=g) * 5)
    s = sm.split3(x)
    hi = x.bfloat16()                                   # the terms restated with torch's RN casts
    r1 = x - hi.float()
    lo = r1.bfloat16()
    mid = (r1 - lo.float()).bfloat16()
    bits = lambda t: t.contiguous().view(torch.int16)
    assert torch.equal(bits(s[:, 368:]), bits(hi)) and torch.equal(bits(s[:, 184:368]), bits(lo))
    assert torch.equal(bits(s[:, :184]), bits(mid))
    back = recon(s, 184)
    assert float(((back - x.double()).abs() / x.double().abs().clamp_min(1e-30)).max()) <= 2.0 ** -24


def test_split3_pads_parts(cuda):
    sm = pkg_module("splitmm")
    g = torch.Generator(device=cuda).manual_seed(2)
    x = torch.randn(333, 84, device=cuda, generator=g)
    s = sm.split3(x)
    assert s.shape == (333, 264)
    for j in range(3):
        assert bool((s[:, 88 * j + 84:88 * (j + 1)] == 0).all())
    back = recon(s, 84)
    assert float(((back - x.double()).abs() / x.double().abs().clamp_min(1e-30)).max()) <= 2.0 ** -24


def test_split3_six_parts(cuda):
    sm = pkg_module("splitmm")
    g = torch.Generator(device=cuda).manual_seed(9)
    x = torch.randn(777, 84, device=cuda, generator=g)
    s3, s6 = sm.split3(x), sm.split3(x, 6)
    assert s6.shape == (777, 528) and torch.equal(s6[:, :264], s3)
    lo, hi = s3[:, 88:176], s3[:, 176:264]
    assert torch.equal(s6[:, 264:352], lo) and torch.equal(s6[:, 352:440], hi) and torch.equal(s6[:, 440:], hi)
    assert sm.parts_for(512, 184) == 6 and sm.parts_for(88, 512) == 3


@pytest.mark.parametrize("act", ["none", "relu", "tanh"])
def test_bias_act_split(cuda, act):
    sm = pkg_module("splitmm")
    code = {"none": sm.ACT_NONE, "relu": sm.ACT_RELU, "tanh": sm.ACT_TANH}[act]
    g = torch.Generator(device=cuda).manual_seed(3)
    rows, cols = 4099, 84
    y = torch.randn(rows, cols, device=cuda, generator=g) * 3
    y[5, 7] = float("nan")
    b = torch.randn(cols, device=cuda, generator=g)
    pre = y + b
    ref = {"none": pre, "relu": torch.relu(pre), "tanh": torch.tanh(pre)}[act]
    yk = y.clone()
    hs = sm.bias_act_split(yk, b, code, 3)
    assert bool(torch.isnan(yk[5, 7]))
    fin = torch.isfinite(ref)
    if act == "tanh":
        ulp = (yk[fin].view(torch.int32) - ref[fin].view(torch.int32)).abs().max()
        assert int(ulp) <= 1
    else:
        assert torch.equal(yk[fin], ref[fin])
    back = recon(hs, cols)
    keep = torch.isfinite(back)
    assert bool(keep.sum() == fin.sum())
    assert float(((back - yk.double())[keep].abs() / yk.double()[keep].abs().clamp_min(1e-30)).max()) <= 2.0 ** -24
    assert sm.bias_act_split(y.clone(), b, code, 0) is None
    y6 = y.clone()
    hs6 = sm.bias_act_split(y6, b, code, 6)
    bits, bits6 = hs.view(torch.int16), hs6.view(torch.int16)     # bitwise: the planted NaN included
    assert torch.equal(y6[fin], yk[fin]) and torch.equal(bits6[:, :264], bits)
    assert torch.equal(bits6[:, 264:352], bits[:, 88:176]) and torch.equal(bits6[:, 352:440], bits[:, 176:264])
    assert torch.equal(bits6[:, 440:528], bits[:, 176:264])


@pytest.mark.parametrize("act", ["none", "relu", "tanh"])
def test_act_grad_split(cuda, act):
    sm = pkg_module("splitmm")
    code = {"none": sm.ACT_NONE, "relu": sm.ACT_RELU, "tanh": sm.ACT_TANH}[act]
    g = torch.Generator(device=cuda).manual_seed(4)
    rows, cols = 70001, 512
    gh = torch.randn(rows, cols, device=cuda, generator=g)
    pre = torch.randn(rows, cols, device=cuda, generator=g)
    h = {"none": pre, "relu": torch.relu(pre), "tanh": torch.tanh(pre)}[act]
    if act == "relu":
        ref = torch.ops.aten.threshold_backward(gh, h, 0.0)
    elif act == "tanh":
        ref = torch.ops.aten.tanh_backward(gh, h)
    else:
        ref = gh
    gys, gb = sm.act_grad_split(gh, h, code)
    back = recon(gys, cols)
    err = (back - ref.double()).abs() / ref.double().abs().clamp_min(1e-30)
    assert float(err.max()) <= 2.0 ** -24
    want = ref.double().sum(0)
    scale = ref.double().abs().sum(0)
    assert float(((gb.double() - want).abs() / scale).max()) <= 1e-6


@pytest.mark.parametrize("k,n,m", [(184, 512, 65536), (512, 512, 65536), (512, 84, 65536), (512, 512, 524288)])
def test_split_linear_matches_fp64(cuda, k, n, m):
    sm = pkg_module("splitmm")
    torch.backends.cuda.matmul.allow_tf32 = False
    g = torch.Generator(device=cuda).manual_seed(k + n)
    x = torch.randn(m, k, device=cuda, generator=g).requires_grad_(True)
    w = (torch.randn(n, k, device=cuda, generator=g) / k ** 0.5).requires_grad_(True)
    b = torch.randn(n, device=cuda, generator=g).requires_grad_(True)
    gy = torch.randn(m, n, device=cuda, generator=g)
    y = sm.split_linear(x, w, b)
    y.backward(gy)
    xd, wd, gd = x.detach().double(), w.detach().double(), gy.double()
    ry = xd @ wd.t() + b.detach().double()
    rgx, rgw = gd @ wd, gd.t() @ xd
    y32 = x.detach() @ w.detach().t() + b.detach()
    gx32, gw32 = gy @ w.detach(), gy.t() @ x.detach()
    for what, got, ref, base in (("y", y.detach(), ry, y32), ("dx", x.grad, rgx, gx32), ("dW", w.grad, rgw, gw32)):
        e, e32 = rel(got, ref), rel(base, ref)
        print(f"{m} x {k} -> {n} {what}: split {e:.2g}, SGEMM {e32:.2g} (relative to the largest |fp64|)")
        assert e <= max(2.5 * e32, 1e-7) and e <= 2e-6, (e, e32)
    assert rel(b.grad, gd.sum(0)) <= 1e-6


@pytest.mark.parametrize("activation", ["relu", "tanh"])
@pytest.mark.parametrize("out_dim", [84, 1])
def test_tower_matches_fp64(cuda, activation, out_dim):
    sm = pkg_module("splitmm")
    tr = pkg_module("trainer")
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.manual_seed(5)
    net = tr.mlp(184, (512, 512), out_dim, activation).to(cuda)
    with torch.no_grad():
        for mod in net:
            if isinstance(mod, torch.nn.Linear):
                mod.bias.normal_(0.0, 0.1)
    ref_net = tr.mlp(184, (512, 512), out_dim, activation).double().to(cuda)
    ref_net.load_state_dict({k: v.double() for k, v in net.state_dict().items()})
    g = torch.Generator(device=cuda).manual_seed(6)
    x = torch.randn(20000, 184, device=cuda, generator=g)
    gout = torch.randn(20000, out_dim, device=cuda, generator=g)
    n32 = tr.mlp(184, (512, 512), out_dim, activation).to(cuda)
    n32.load_state_dict(net.state_dict())
    out = sm.run_tower(net, x)
    out.backward(gout)
    o32 = n32(x)
    o32.backward(gout)
    ref = ref_net(x.double())
    ref.backward(gout.double())
    assert rel(out.detach(), ref.detach()) <= 1e-5
    for p, q, r in zip(net.parameters(), n32.parameters(), ref_net.parameters()):
        e, e32 = rel(p.grad, r.grad), rel(q.grad, r.grad)
        if activation == "tanh":
            assert e <= 1e-5, (e, e32)
        else:
            # relu: a pre-activation within rounding of zero takes the other side of the mask in
            # any fp32 evaluation, moving a whole weight-gradient row; torch's own fp32 tower
            # shows the same (or larger) gradient errors, measured at 1e-4..1e-2 against fp64
            assert e <= max(3.0 * e32, 1e-5), (e, e32)


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


def _torch_head(z, a, A=4, B=21):
    dist = torch.distributions.Categorical(logits=z.view(-1, A, B))
    return dist.log_prob(a.long()).sum(-1), dist.entropy().sum(-1)


@pytest.mark.parametrize("adtype,A,B", [(torch.uint8, 4, 21), (torch.int64, 4, 21), (torch.uint8, 3, 13)])
def test_categorical_head_matches_torch(cuda, adtype, A, B):
    cat = pkg_module("categorical")
    g = torch.Generator(device=cuda).manual_seed(8)
    m, W = 30001, A * B
    z = (torch.randn(m, W, device=cuda, generator=g) * 4).requires_grad_(True)
    with torch.no_grad():
        z[3, 0:B] = -float("inf")
        z[3, 5] = 2.0
        z[7, B + 9] = 1e30
    a = torch.randint(0, B, (m, A), device=cuda, generator=g).to(adtype)
    a[3, 0] = 5
    g_lp = torch.randn(m, device=cuda, generator=g)
    # the update's upstream entropy gradient is -ent_coef / rows, far below 1: torch clamps -inf
    # logits at -FLT_MAX, so on a row with -inf logits an entropy gradient above 1 in magnitude
    # overflows inside its softmax backward (inf * 0 = NaN) where the kernel returns the limit 0
    g_ent = torch.randn(m, device=cuda, generator=g) * 1e-2
    lp, ent = cat.logp_entropy(z, a, A, B)
    (lp * g_lp + ent * g_ent).sum().backward()
    gz = z.grad.clone()
    z.grad = None
    rlp, rent = _torch_head(z, a, A, B)
    (rlp * g_lp + rent * g_ent).sum().backward()
    for got, ref in ((lp, rlp), (ent, rent), (gz, z.grad)):
        got, ref = got.detach(), ref.detach()
        assert bool(torch.isfinite(got).all())
        assert float((got - ref).abs().max()) <= 1e-5 * max(1.0, float(ref.abs().max()))
    # log-prob only (the entropy unused): its gradient path alone
    z.grad = None
    lp, _ = cat.logp_entropy(z, a, A, B)
    lp.sum().backward()
    gz = z.grad.clone()
    z.grad = None
    _torch_head(z, a, A, B)[0].sum().backward()
    # p enters as exp(z - logsumexp) in torch's logsumexp backward and as the softmax of the
    # normalised logits here: a few ulps apart
    assert float((gz - z.grad).abs().max()) <= 1e-5 * max(1.0, float(z.grad.abs().max()))


def test_categorical_head_validates(cuda):
    cat = pkg_module("categorical")
    z = torch.randn(100, 84, device=cuda)
    a = torch.randint(0, 21, (100, 4), device=cuda).to(torch.uint8)
    lp, ent = cat.logp_entropy(z, a, 4, 21)
    assert lp.shape == (100,) and ent.shape == (100,)
    bad = a.clone()
    bad[9, 2] = 21
    with pytest.raises(ValueError, match="support"):
        cat.logp_entropy(z, bad, 4, 21)
    with pytest.raises(ValueError):
        _torch_head(z, bad)
    zn = z.clone()
    zn[4, 50] = float("nan")
    with pytest.raises(ValueError, match="constraint"):
        cat.logp_entropy(zn, a, 4, 21)
    with pytest.raises(ValueError):
        _torch_head(zn, a)


def test_tower_input_split_reused_and_invalidated(cuda):
    sm = pkg_module("splitmm")
    tr = pkg_module("trainer")
    torch.manual_seed(12)
    actor = tr.mlp(184, (512, 512), 84, "relu").to(cuda)
    critic = tr.mlp(184, (512, 512), 1, "relu").to(cuda)
    y = torch.randn(4096, 184, device=cuda)
    sm.run_tower(actor, y)
    assert not hasattr(y, "_f16_split")              # unmarked inputs keep nothing
    x = torch.randn(4096, 184, device=cuda)
    setattr(x, sm.SHARE_SPLIT, True)
    a1 = sm.run_tower(actor, x)
    xs = x._f16_split[2]
    v1 = sm.run_tower(critic, x)
    assert x._f16_split[2] is xs                     # the critic reused the actor's split
    ref = sm.run_tower(critic, x.clone())
    assert torch.equal(v1, ref)
    x.mul_(2.0)                                      # in place: the cached split is stale
    v2 = sm.run_tower(critic, x)
    assert x._f16_split[2] is not xs
    assert torch.equal(v2, sm.run_tower(critic, x.clone()))
    assert torch.equal(a1, sm.run_tower(actor, (x / 2.0).clone()))


@pytest.mark.parametrize("out_dim", [84, 1])
def test_tower_reference_final_shape(cuda, out_dim):
    """The reference's final model shape (three 384-wide tanh layers): actor and critic towers
    through run_tower within 1e-5 of fp64, output and every parameter gradient."""
    sm = pkg_module("splitmm")
    tr = pkg_module("trainer")
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.manual_seed(13)
    net = tr.mlp(184, (384, 384, 384), out_dim, "tanh").to(cuda)
    with torch.no_grad():
        for mod in net:
            if isinstance(mod, torch.nn.Linear):
                mod.bias.normal_(0.0, 0.1)
    ref_net = tr.mlp(184, (384, 384, 384), out_dim, "tanh").double().to(cuda)
    ref_net.load_state_dict({k: v.double() for k, v in net.state_dict().items()})
    g = torch.Generator(device=cuda).manual_seed(14)
    x = torch.randn(30000, 184, device=cuda, generator=g)
    gout = torch.randn(30000, out_dim, device=cuda, generator=g)
    out = sm.run_tower(net, x)
    out.backward(gout)
    ref = ref_net(x.double())
    ref.backward(gout.double())
    assert rel(out.detach(), ref.detach()) <= 1e-5
    for p, q in zip(net.parameters(), ref_net.parameters()):
        assert rel(p.grad, q.grad) <= 1e-5
