"""Host side of the policy kernel's network descriptors (no GPU): the fp32 value-head row a critic
carries, its refresh by load_from, and the descriptor fields that point at it."""
import torch
import torch.nn as nn

from conftest import pkg_module


def _seq(hidden, out, seed):
    g = torch.Generator().manual_seed(seed)
    layers, last = [], 184
    for h in hidden:
        layers += [nn.Linear(last, h), nn.ReLU()]
        last = h
    layers.append(nn.Linear(last, out))
    seq = nn.Sequential(*layers)
    with torch.no_grad():
        for p in seq.parameters():
            p.copy_(torch.randn(p.shape, generator=g) * 0.05)
    return seq


def test_value_head_row_in_fp32_and_refreshed():
    P = pkg_module("policy")
    critic = _seq((512, 512), 1, 1)
    w = P.MlpWeights.from_sequential(critic, P.HEAD_VALUE, torch.device("cpu"), operand="fp16")
    assert w.head_w32 is not None and w.head_w32.dtype == torch.float32
    assert torch.equal(w.head_w32, critic[-1].weight.detach())           # the fp32 row itself, not rounded
    d = w.desc()
    assert d.head_weight_f32 == w.head_w32.data_ptr() and d.operand == P.OPERANDS["fp16"][0]
    # an optimiser step in place, then load_from: the 16-bit copies and the fp32 row both follow
    with torch.no_grad():
        for p in critic.parameters():
            p.add_(0.01)
    ptr = w.head_w32.data_ptr()
    w.load_from(critic)
    assert w.head_w32.data_ptr() == ptr                                   # same buffer: the set stays valid
    assert torch.equal(w.head_w32, critic[-1].weight.detach())
    assert torch.equal(w.weights[-1], critic[-1].weight.detach().to(torch.float16))


def test_no_fp32_row_for_actors_or_a_single_layer_critic():
    P = pkg_module("policy")
    actor = _seq((512, 512), 84, 2)
    a = P.MlpWeights.from_sequential(actor, P.HEAD_CATEGORICAL, torch.device("cpu"), operand="bf16")
    assert a.head_w32 is None and not a.desc().head_weight_f32
    lone = nn.Sequential(nn.Linear(184, 1))
    c = P.MlpWeights.from_sequential(lone, P.HEAD_VALUE, torch.device("cpu"), operand="fp16")
    assert c.head_w32 is None and not c.desc().head_weight_f32
