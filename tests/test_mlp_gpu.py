"""tcgen05 policy / value MLP vs torch -- needs a B200.

References: (a) a torch emulation of the kernel's numerics (16-bit weights and inputs, fp32
accumulation, bias + activation in fp32, hidden activations rounded to the operand type):
logits / values within 1e-2 absolute + 1e-2 relative (accumulation order can flip single
roundings of hidden units); (b) the plain fp32 nn.Sequential of the reference architecture
(R/claude_code/model.py _mlp, :34-44) and torch.distributions.Categorical on its logits (the
reference's actor_step, ppo_gpu.py:273-285), the contract of the parity table:
  fp16 operands: logits within 1e-3 * max|logit|, summed log-prob of the sampled bins within
                 1e-3 relative, argmax equal to fp32 torch's on every row whose top-two logit gap
                 exceeds twice the logit bound;
  bf16 operands: the same checks at 1e-2 (bf16 keeps 8 significant bits; measured about 4e-3 of
                 max|logit| and 5e-3 relative log-prob, so 1e-3 is out of its reach).
Sampling: log-prob equals the summed log-softmax of the kernel's own logits at the sampled
bins; sampled frequencies pass a chi-square test against the softmax probabilities.
"""
import math

import numpy as np
import pytest
import torch
import torch.nn as nn

from conftest import pkg_module

pytestmark = pytest.mark.gpu


def make_seq(in_dim, hidden, out, act, seed, device):
    g = torch.Generator().manual_seed(seed)
    layers, last = [], in_dim
    for h in hidden:
        layers += [nn.Linear(last, h), nn.ReLU() if act == "relu" else nn.Tanh()]
        last = h
    layers.append(nn.Linear(last, out))
    seq = nn.Sequential(*layers)
    with torch.no_grad():
        for m in seq:
            if isinstance(m, nn.Linear):
                w = torch.randn(m.weight.shape, generator=g)
                q, _ = torch.linalg.qr(w.T if w.shape[0] < w.shape[1] else w)
                m.weight.copy_((q.T if w.shape[0] < w.shape[1] else q)[:m.weight.shape[0], :m.weight.shape[1]]
                               * math.sqrt(2))
                m.bias.copy_(torch.rand(m.bias.shape, generator=g) * 0.2 - 0.1)
    return seq.to(device)


def emulate(seq, xb, head_w32=True):
    """The kernel's numerics in torch: weights in xb's 16-bit type, fp32 accumulation, hidden
    activations rounded to that type -- except a width-1 value head after a hidden layer, which
    takes the last hidden layer's fp32 activations and its fp32 weight row (the 16-bit row
    widened when the descriptor carries no fp32 copy, head_w32=False)."""
    dt = xb.dtype
    lin = [m for m in seq if isinstance(m, nn.Linear)]
    act = [m for m in seq if not isinstance(m, nn.Linear)]
    fold = lin[-1].out_features == 1 and len(lin) >= 2
    h = xb.float()
    for i, l in enumerate(lin):
        last = i == len(lin) - 1
        w = l.weight.detach()
        w = w.float() if (last and fold and head_w32) else w.to(dt).float()
        h = h @ w.T + l.bias.detach().float()
        if not last:
            h = act[i](h)
            if not (fold and i == len(lin) - 2):
                h = h.to(dt).float()
    return h


def make_x(rows, device, seed=0, pad=192, dtype=torch.bfloat16):
    g = torch.Generator(device=device).manual_seed(seed)
    x = (torch.randn(rows, 184, device=device, generator=g) * 1.5).clamp(-10, 10)
    xb = torch.zeros(rows, pad, dtype=dtype, device=device)
    xb[:, :184] = x.to(dtype)
    return x, xb


@pytest.fixture(scope="module")
def P():
    return pkg_module("policy")


def check_close(got, ref, atol, rtol, what):
    d = (got - ref).abs()
    bad = d > atol + rtol * ref.abs()
    print(f"{what}: max abs err {d.max().item():.3e}, max |ref| {ref.abs().max().item():.3e}")
    assert not bool(bad.any()), f"{what}: {int(bad.sum())} elements out of tolerance"


def test_actor_and_critic_logits_and_value(P, cuda):
    actor = make_seq(184, (512, 512), 84, "relu", 1, cuda)
    critic = make_seq(184, (512, 512), 1, "relu", 2, cuda)
    ps = P.PolicySet([P.MlpWeights.from_sequential(actor, P.HEAD_CATEGORICAL, cuda),
                      P.MlpWeights.from_sequential(critic, P.HEAD_VALUE, cuda)])
    rows = 1000                                      # 7 full tiles + a partial one
    x, xb = make_x(rows, cuda)
    logits = torch.full((rows, 84), float("nan"), device=cuda)
    logp = torch.zeros(rows, device=cuda)
    bins = torch.zeros(rows, 4, dtype=torch.uint8, device=cuda)
    ps.forward(xb, [(rows, [0])], logits=logits, logp=logp, bins=bins, seed=5, step=1)
    value = torch.zeros(rows, device=cuda)
    ps.forward(xb, [(rows, [1])], value=value)
    torch.cuda.synchronize()
    ps.check_error()
    ref_l = emulate(actor, xb[:, :184])
    ref_v = emulate(critic, xb[:, :184])[:, 0]
    check_close(logits, ref_l, 1e-2, 1e-2, "actor logits vs bf16 emulation")
    check_close(value, ref_v, 1e-2, 1e-2, "critic value vs bf16 emulation")
    with torch.no_grad():
        f32_l = actor(x)
        f32_v = critic(x)[:, 0]
    check_close(logits, f32_l, 1e-2 * f32_l.abs().max().item(), 0.0, "actor logits vs fp32 torch")
    check_close(value, f32_v, 1e-2 * f32_v.abs().max().item(), 0.0, "critic value vs fp32 torch")
    # log-prob of the sampled bins from the kernel's own logits
    lsm = torch.log_softmax(logits.view(rows, 4, 21), -1)
    exp_logp = lsm.gather(-1, bins.long().unsqueeze(-1)).squeeze(-1).sum(-1)
    check_close(logp, exp_logp, 1e-4, 1e-5, "summed log-prob")
    # fused actor + critic in one launch equals the separate launches
    logp2 = torch.zeros(rows, device=cuda)
    value2 = torch.zeros(rows, device=cuda)
    bins2 = torch.zeros(rows, 4, dtype=torch.uint8, device=cuda)
    ps.forward(xb, [(rows, [0, 1])], nets_per_group=2, logp=logp2, value=value2, bins=bins2, seed=5, step=1)
    torch.cuda.synchronize()
    assert torch.equal(bins2, bins) and torch.equal(logp2, logp) and torch.equal(value2, value)


def test_deterministic_is_argmax(P, cuda):
    actor = make_seq(184, (512, 512), 84, "relu", 3, cuda)
    ps = P.PolicySet([P.MlpWeights.from_sequential(actor, P.HEAD_CATEGORICAL, cuda)])
    rows = 512
    _, xb = make_x(rows, cuda, seed=4)
    logits = torch.zeros(rows, 84, device=cuda)
    act = torch.zeros(rows, 4, dtype=torch.int32, device=cuda)
    ps.forward(xb, [(rows, [0])], logits=logits, act_idx=act, deterministic=True)
    torch.cuda.synchronize()
    assert torch.equal(act.long(), logits.view(rows, 4, 21).argmax(-1))


def test_grouped_opponents_and_interleaved_bins(P, cuda):
    """8 frozen actors on contiguous 256-row blocks, bins written to the odd (opponent) slots."""
    nets = [make_seq(184, (512, 512), 84, "relu", 10 + i, cuda) for i in range(8)]
    ps = P.PolicySet([P.MlpWeights.from_sequential(n, P.HEAD_CATEGORICAL, cuda) for n in nets])
    rows = 8 * 256
    _, xb = make_x(rows, cuda, seed=6)
    logits = torch.zeros(rows, 84, device=cuda)
    bins = torch.full((2 * rows, 4), 255, dtype=torch.uint8, device=cuda)
    ps.forward(xb, [(256 * (i + 1), [i]) for i in range(8)], logits=logits, bins=bins, bins_stride=8,
               bins_offset=4, deterministic=True)
    torch.cuda.synchronize()
    for i in range(8):
        r = slice(256 * i, 256 * (i + 1))
        check_close(logits[r], emulate(nets[i], xb[r, :184]), 1e-2, 1e-2, f"opponent {i}")
    assert bool((bins[0::2] == 255).all())
    assert torch.equal(bins[1::2].long(), logits.view(rows, 4, 21).argmax(-1))


def test_tanh_384x3(P, cuda):
    """The final lineage's shape (research/competition_36500/README.md:10): 384x3 tanh."""
    actor = make_seq(184, (384, 384, 384), 84, "tanh", 21, cuda)
    critic = make_seq(184, (384, 384, 384), 1, "tanh", 22, cuda)
    ps = P.PolicySet([P.MlpWeights.from_sequential(actor, P.HEAD_CATEGORICAL, cuda),
                      P.MlpWeights.from_sequential(critic, P.HEAD_VALUE, cuda)])
    rows = 640
    _, xb = make_x(rows, cuda, seed=7)
    logits = torch.zeros(rows, 84, device=cuda)
    value = torch.zeros(rows, device=cuda)
    ps.forward(xb, [(rows, [0])], logits=logits, deterministic=True)
    ps.forward(xb, [(rows, [1])], value=value)
    torch.cuda.synchronize()
    check_close(logits, emulate(actor, xb[:, :184]), 1e-2, 1e-2, "tanh actor")
    check_close(value, emulate(critic, xb[:, :184])[:, 0], 1e-2, 1e-2, "tanh critic")


def test_sampling_frequencies_chi_square(P, cuda):
    """One observation repeated 2^17 times: per-channel bin counts vs softmax probabilities."""
    actor = make_seq(184, (512, 512), 84, "relu", 31, cuda)
    with torch.no_grad():
        actor[-1].weight.mul_(0.05)          # moderate logits so many bins have mass
    ps = P.PolicySet([P.MlpWeights.from_sequential(actor, P.HEAD_CATEGORICAL, cuda)])
    rows = 1 << 17
    _, xb1 = make_x(1, cuda, seed=8)
    xb = xb1.expand(rows, -1).contiguous()
    logits = torch.zeros(rows, 84, device=cuda)
    act = torch.zeros(rows, 4, dtype=torch.int32, device=cuda)
    ps.forward(xb, [(rows, [0])], logits=logits, act_idx=act, seed=12345, step=7)
    torch.cuda.synchronize()
    probs = torch.softmax(logits[0].view(4, 21).double(), -1).cpu().numpy()
    from scipy.stats import chisquare
    for c in range(4):
        counts = np.bincount(act[:, c].cpu().numpy(), minlength=21).astype(np.float64)
        exp = probs[c] * rows
        keep = exp >= 5
        obs_k = np.append(counts[keep], counts[~keep].sum())
        exp_k = np.append(exp[keep], exp[~keep].sum())
        if exp_k[-1] == 0:
            obs_k, exp_k = obs_k[:-1], exp_k[:-1]
        p = chisquare(obs_k, exp_k * obs_k.sum() / exp_k.sum()).pvalue
        print(f"channel {c}: chi-square p = {p:.3f}")
        assert p > 1e-4


def test_other_head_shape(P, cuda):
    """A categorical head other than 4 x 21 (3 channels x 11 bins) takes the generic epilogue."""
    actor = make_seq(184, (256, 256), 33, "relu", 41, cuda)
    ps = P.PolicySet([P.MlpWeights.from_sequential(actor, P.HEAD_CATEGORICAL, cuda, act_dim=3, num_bins=11)])
    rows = 384
    _, xb = make_x(rows, cuda, seed=9)
    logits = torch.zeros(rows, 33, device=cuda)
    act = torch.zeros(rows, 3, dtype=torch.int32, device=cuda)
    logp = torch.zeros(rows, device=cuda)
    ps.forward(xb, [(rows, [0])], logits=logits, act_idx=act, logp=logp, seed=3, step=2)
    torch.cuda.synchronize()
    check_close(logits, emulate(actor, xb[:, :184]), 1e-2, 1e-2, "3x11 logits")
    lsm = torch.log_softmax(logits.view(rows, 3, 11), -1)
    exp_logp = lsm.gather(-1, act.long().unsqueeze(-1)).squeeze(-1).sum(-1)
    check_close(logp, exp_logp, 1e-4, 1e-5, "3x11 summed log-prob")
    ps.forward(xb, [(rows, [0])], logits=logits, act_idx=act, deterministic=True)
    torch.cuda.synchronize()
    assert torch.equal(act.long(), logits.view(rows, 3, 11).argmax(-1))


# contract bound per operand type: logits (fraction of max |logit|) and summed log-prob (relative)
CONTRACT = {"fp16": 1e-3, "bf16": 1e-2}


@pytest.mark.parametrize("operand", ["fp16", "bf16"])
@pytest.mark.parametrize("fp32_row", [True, False])
def test_value_head_against_fp32_torch(P, cuda, operand, fp32_row):
    """The critic's width-1 head runs in the last hidden layer's epilogue in fp32: values against
    the fp32 network within the operand's contract bound (fraction of max |value|), against the
    kernel-numerics emulation within a quarter of it, with the descriptor's fp32 weight row and
    without it (the 16-bit row widened); a partial last tile, tanh and a 384-wide hidden layer
    (not split into accumulator halves) included."""
    bound = CONTRACT[operand]
    dt = torch.float16 if operand == "fp16" else torch.bfloat16
    for hidden, act, seed in (((512, 512), "relu", 41), ((384, 384, 384), "tanh", 42), ((512,), "relu", 43)):
        critic = make_seq(184, hidden, 1, act, seed, cuda)
        net = P.MlpWeights.from_sequential(critic, P.HEAD_VALUE, cuda, operand=operand)
        if not fp32_row:
            net.head_w32 = None
        actor = make_seq(184, (512, 512), 84, "relu", seed + 100, cuda)
        ps = P.PolicySet([P.MlpWeights.from_sequential(actor, P.HEAD_CATEGORICAL, cuda, operand=operand), net])
        rows = 3000                                  # 23 full tiles + a partial one
        x, xb = make_x(rows, cuda, seed=seed, dtype=dt)
        value = torch.full((rows,), float("nan"), device=cuda)
        ps.forward(xb, [(rows, [1])], value=value)
        # fused with the actor (the rollout's launch) the values are the same bits
        value2 = torch.full((rows,), float("nan"), device=cuda)
        logp = torch.zeros(rows, device=cuda)
        ps.forward(xb, [(rows, [0, 1])], nets_per_group=2, value=value2, logp=logp, seed=3, step=1)
        torch.cuda.synchronize()
        ps.check_error()
        assert torch.equal(value, value2)
        with torch.no_grad():
            f32 = critic(x)[:, 0]
        em = emulate(critic, xb[:, :184], head_w32=fp32_row)[:, 0]
        scale = f32.abs().max().item()
        err = (value - f32).abs().max().item() / scale
        em_err = (value - em).abs().max().item() / em.abs().max().item()
        print(f"{operand} {hidden} {act} fp32 row {fp32_row}: value {err:.2e} of max |value| vs fp32 torch, "
              f"{em_err:.2e} vs emulation")
        assert err <= bound
        # the emulation rounds the 16-bit hidden layers as the kernel does, but its fp32 sums run in
        # another order (and tanh is not the kernel's fast tanh), so a few 16-bit roundings differ
        assert em_err <= bound / 4


@pytest.mark.parametrize("operand", ["fp16", "bf16"])
@pytest.mark.parametrize("seed", [1, 3])
def test_policy_against_fp32_torch(P, cuda, operand, seed):
    """Rows a10 / a11 against the fp32 reference network (not the kernel's own logits): logits,
    the summed log-prob of the kernel's sampled bins under torch.distributions.Categorical of the
    fp32 logits, and deterministic argmax bins against fp32 argmax away from near-ties."""
    bound = CONTRACT[operand]
    dt = torch.float16 if operand == "fp16" else torch.bfloat16
    actor = make_seq(184, (512, 512), 84, "relu", seed, cuda)
    ps = P.PolicySet([P.MlpWeights.from_sequential(actor, P.HEAD_CATEGORICAL, cuda, operand=operand)])
    rows = 4096
    x, xb = make_x(rows, cuda, seed=seed + 10, dtype=dt)
    logits = torch.zeros(rows, 84, device=cuda)
    logp = torch.zeros(rows, device=cuda)
    bins = torch.zeros(rows, 4, dtype=torch.uint8, device=cuda)
    ps.forward(xb, [(rows, [0])], logits=logits, logp=logp, bins=bins, seed=9, step=2)
    det = torch.zeros(rows, 4, dtype=torch.int32, device=cuda)
    ps.forward(xb, [(rows, [0])], act_idx=det, deterministic=True)
    torch.cuda.synchronize()
    ps.check_error()
    with torch.no_grad():
        ref = actor(x)
    scale = ref.abs().max().item()
    lerr = (logits - ref).abs().max().item() / scale
    dist = torch.distributions.Categorical(logits=ref.view(rows, 4, 21))
    ref_lp = dist.log_prob(bins.long()).sum(-1)
    lp_rel = ((logp - ref_lp).abs() / ref_lp.abs().clamp_min(1e-6)).max().item()
    top2 = ref.view(rows, 4, 21).topk(2, dim=-1).values
    clear = (top2[..., 0] - top2[..., 1]) > 2 * bound * scale
    agree = det.long() == ref.view(rows, 4, 21).argmax(-1)
    print(f"{operand} seed {seed}: logits {lerr:.2e} of max |logit| ({scale:.2f}), summed log-prob "
          f"{lp_rel:.2e} relative, argmax compared on {int(clear.sum())} of {clear.numel()} channel rows "
          f"({int((agree | ~clear).logical_not().sum())} disagree; {int((~agree).sum())} differ overall)")
    assert lerr <= bound
    assert lp_rel <= bound
    assert bool(agree[clear].all())
