"""Host logic of the PPO update's split-product path (no GPU needed).

* part_width / parts_for: 16-byte part alignment and the layout choice (six parts -- one GEMM --
  only where the two fp32 read-modify-write passes it saves outweigh the extra parts written).
* run_tower off the GPU is the module's own forward: CPU tensors never reach the C ABI, so the
  reference's CPU update keeps plain fp32 torch arithmetic (and its golden test holds).
* The fused categorical head only takes CUDA fp32 (M, A*B) logits within its size limits; the
  actor's evaluate_actions on CPU is torch.distributions.Categorical's.
* The split's arithmetic (restated with torch's round-to-nearest casts on the CPU): both
  differences x - hi and (x - hi) - lo are exact in fp32, so mid + lo + hi is within 2^-24 of x
  across the whole normal range (the kernel's parts are pinned to this restatement on the GPU).
"""
import torch

from conftest import pkg_module


def test_part_width_and_layout_choice():
    sm = pkg_module("splitmm")
    assert [sm.part_width(c) for c in (4, 8, 84, 88, 184, 512)] == [8, 8, 88, 88, 184, 512]
    # forward of the hidden layers: 512 outputs from 184 / 512 inputs -> one GEMM
    assert sm.parts_for(512, 184) == 6 and sm.parts_for(512, 512) == 6
    # the 84 logits from 512 inputs: three GEMMs move fewer bytes
    assert sm.parts_for(84, 512) == 3
    # input gradient of the logits layer: 512 outputs from the 88-column gradient parts
    assert sm.parts_for(512, 88) == 6


def test_run_tower_on_cpu_is_the_module():
    sm = pkg_module("splitmm")
    tr = pkg_module("trainer")
    torch.manual_seed(1)
    for out_dim, act in ((84, "relu"), (1, "tanh")):
        net = tr.mlp(184, (512, 512), out_dim, act)
        x = torch.randn(37, 184, requires_grad=True)
        y = sm.run_tower(net, x)
        assert torch.equal(y, net(x))
        y.sum().backward()
        assert x.grad is not None and torch.isfinite(x.grad).all()


def test_layer_eligibility():
    sm = pkg_module("splitmm")
    lin = torch.nn.Linear
    x_cpu = torch.zeros(4, 184)
    assert not sm.usable(lin(184, 512), x_cpu)                   # CPU input: plain path
    assert sm._dims_ok(lin(184, 512)) and sm._dims_ok(lin(512, 84))
    assert not sm._dims_ok(lin(512, 1))                          # value head: folded, not split
    assert not sm._dims_ok(lin(186, 512))                        # input width off the 16-byte grid
    assert not sm._dims_ok(lin(512, 2048))                       # wider than the prologue kernel takes


def test_categorical_head_eligibility_and_cpu_path():
    cat = pkg_module("categorical")
    tr = pkg_module("trainer")
    assert not cat.usable(torch.zeros(8, 84), 4, 21)            # CPU logits
    torch.manual_seed(2)
    model = tr.MLPActorCritic(hidden=(64, 64), activation="tanh")
    model.split_products = True                                  # no effect on CPU tensors
    obs = torch.randn(16, 184)
    act = torch.randint(0, 21, (16, 4), dtype=torch.uint8)
    lp, ent = model.evaluate_actions(obs, act)
    dist = torch.distributions.Categorical(logits=model.actor_logits(obs).view(-1, 4, 21))
    assert torch.equal(lp, dist.log_prob(act.long()).sum(-1))
    assert torch.equal(ent, dist.entropy().sum(-1))


def test_split_arithmetic_is_exact_in_fp32():
    g = torch.Generator().manual_seed(3)
    x = torch.randn(200000, generator=g) * torch.exp(torch.randn(200000, generator=g) * 20)
    x = x[torch.isfinite(x) & (x.abs() > 1e-30) & (x.abs() < 1e30)]
    hi = x.bfloat16()
    r1 = x - hi.float()
    lo = r1.bfloat16()
    r2 = r1 - lo.float()
    mid = r2.bfloat16()
    xd = x.double()
    assert torch.equal(r1.double(), xd - hi.double())                      # exact differences
    assert torch.equal(r2.double(), xd - hi.double() - lo.double())
    back = hi.double() + lo.double() + mid.double()
    assert float(((back - xd).abs() / xd.abs()).max()) <= 2.0 ** -24
