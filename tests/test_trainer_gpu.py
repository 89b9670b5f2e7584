"""PPOTrainer rollout + update on a B200 (trainer.py).

A short rollout through the real env and kernels, checked against torch on the rollout buffers:
* log-probs of the sampled bins and values vs an emulation of the actor / critic in the trainer's
  16-bit operand type (fp16 by default: 16-bit weights and inputs, fp32 accumulation): within
  5e-2 (sum of four channel log-probs) and 1e-2 + 1e-2 relative;
* the env commands of the last step equal the reference action_to_env of the stored bins
  exactly (main, even aircraft) and of the argmax of the assigned opponent's emulated logits
  (deterministic opponents, odd aircraft; >= 99 % of rows, the rest are near-ties);
* advantages / returns equal the reference GAE loop (ppo_gpu.py:1983-1995) on the buffers
  bit for bit;
* after ``update`` the kernel's weights are refreshed (logits follow the new parameters).
"""
import pytest
import torch
import torch.nn as nn

from conftest import pkg_module

pytestmark = pytest.mark.gpu


def emulate(seq, xb):
    """The policy kernel's numerics in torch, in xb's 16-bit type."""
    dt = xb.dtype
    lin = [m for m in seq if isinstance(m, nn.Linear)]
    act = [m for m in seq if not isinstance(m, nn.Linear)]
    h = xb.float()
    for i, l in enumerate(lin):
        h = h @ l.weight.detach().to(dt).float().T + l.bias.detach().float()
        if i < len(lin) - 1:
            h = act[i](h).to(dt).float()
    return h


def ref_gae(b_rew, b_val, b_done, last_value, next_done, gamma, lam):
    T = b_rew.shape[0]
    adv = torch.zeros_like(b_rew)
    lastgae = torch.zeros(b_rew.shape[1], device=b_rew.device)
    for t in reversed(range(T)):
        if t == T - 1:
            nnt = 1.0 - next_done
            nv = last_value
        else:
            nnt = 1.0 - b_done[t + 1]
            nv = b_val[t + 1]
        delta = b_rew[t] + gamma * nv * nnt - b_val[t]
        lastgae = delta + gamma * lam * nnt * lastgae
        adv[t] = lastgae
    return adv, adv + b_val


def action_to_env(idx, grid):
    cont = grid[idx.long()]
    ctrl = cont.clone()
    ctrl[:, 3] = 0.5 * cont[:, 3] + 0.5
    return ctrl.double()


def make_trainer(cuda, nenv, n_opp, opp_mode, seed):
    rl_env = pkg_module("rl_env")
    tr = pkg_module("trainer")
    ro = pkg_module("rollout")
    env = rl_env.GpuDogfightVecEnv(nenv, substeps=6, seed=seed)
    torch.manual_seed(seed)
    cfg = tr.PPOConfig(rollout_steps=4, gamma=0.99, gae_lambda=0.95, hidden=(512, 512), activation="relu",
                       opp_sample=False, seed=seed, update_epochs=1, num_minibatches=2)
    opps = []
    for i in range(n_opp):
        net = tr.MLPActorCritic(hidden=(512, 512), activation="relu").to(cuda)
        norm = None
        if i == 1:                                   # one opponent with its own normaliser
            norm = ro.RunningNorm(184, cuda)
            norm.update(torch.randn(4096, 184, device=cuda) * 2.0 + 0.5)
        opps.append(tr.Opponent(net, norm))
    weights = torch.linspace(1.0, 2.0, n_opp) if opp_mode == "pool" else None
    return tr.PPOTrainer(env, cfg, opponents=opps, opp_mode=opp_mode, opp_weights=weights), tr


def check_rollout(t, adv, ret):
    cfg = t.cfg
    model = t.model
    grid = t.grid
    for s in range(cfg.rollout_steps):
        xb = t.b_obs[s].to(t.policy.dtype)
        lg = emulate(model.actor_logits, xb).view(-1, 4, 21)
        lsm = torch.log_softmax(lg, -1)
        exp_logp = lsm.gather(-1, t.b_act[s].long().unsqueeze(-1)).squeeze(-1).sum(-1)
        d = (t.b_logp[s] - exp_logp).abs().max().item()
        assert d < 5e-2, f"step {s}: log-prob error {d}"
        ev = emulate(model.critic, xb)[:, 0]
        assert bool(((t.b_val[s] - ev).abs() <= 1e-2 + 1e-2 * ev.abs()).all()), f"step {s}: values"
    cmd = t.env.action_buffer.view(t.nenv, 2, 4)
    assert torch.equal(cmd[:, 0], action_to_env(t.b_act[-1], grid)), "main commands != action_to_env(bins)"
    a2, r2 = ref_gae(t.b_rew, t.b_val, t.b_done, t.last_value, t._next_done, cfg.gamma, cfg.gae_lambda)
    assert torch.equal(adv, a2) and torch.equal(ret, r2), "GAE differs from the reference loop"


def test_rollout_blocks_and_update(cuda):
    t, tr = make_trainer(cuda, 640, 2, "blocks", 3)
    t.reset(stagger=False)
    adv, ret, stats = t.collect_rollout()
    torch.cuda.synchronize()
    check_rollout(t, adv, ret)
    assert abs(float(t.norm.count) - (1e-4 + 4 * 640)) < 1.0
    # opponents: deterministic argmax of each block's own actor on its (normalised) input
    cmd = t.env.action_buffer.view(t.nenv, 2, 4)
    agree = 0
    for g, (a, b) in enumerate(t._blocks):
        lg = emulate(t.opponents[g].actor, t.x_opp[a:b, :184]).view(-1, 4, 21)
        agree += int((cmd[a:b, 1] == action_to_env(lg.argmax(-1), t.grid)).all(-1).sum())
    assert agree >= 0.99 * t.nenv, f"opponent commands agree on {agree}/{t.nenv} rows"
    assert float(stats["ep_count"]) >= 0
    # update, then the kernel uses the new parameters
    before = [p.detach().clone() for p in t.model.actor_parameters()]
    res = t.update(adv, ret)
    assert res["optimizer_steps"] >= 1
    assert any(float((p.detach() - q).abs().max()) > 0 for p, q in zip(t.model.actor_parameters(), before))
    logits = torch.zeros(t.nenv, 84, device=cuda)
    t.policy.forward(t.x_main, [(t.nenv, [0])], logits=logits, deterministic=True)
    torch.cuda.synchronize()
    ref = emulate(t.model.actor_logits, t.x_main[:, :184])
    assert float((logits - ref).abs().max()) <= 1e-2 + 1e-2 * float(ref.abs().max())


def test_rollout_pool_assignment(cuda):
    """Pool mode: a decision's opponent path (assignment resampling at episode ends, device-side
    grouping, grouped normalise, grouped policy launch, command scatter) and env step run without
    a host synchronisation (torch's sync debug mode raises on any; the rollout's once-per-rollout
    finiteness check stays outside), and each env's opponent command is its assigned opponent's
    argmax on its (normalised) input, grouped in tile-aligned blocks as the reference's
    argsort + split."""
    t, tr = make_trainer(cuda, 512, 3, "pool", 4)
    t.reset(stagger=False)
    t.collect_rollout()                      # first use of every buffer, outside the check
    torch.cuda.synchronize()
    cmd = t.env.action_buffer
    torch.cuda.set_sync_debug_mode("error")
    try:
        for _ in range(3):
            sampled = t._sample_opp(t.nenv)
            t.opp_assign = torch.where(t._next_done.bool(), sampled, t.opp_assign)
            t._opponents_act(cmd)
            obs, _, done, _ = t.env.step(cmd)
            t._next_opp_obs = obs[:, 1, :]
            t._next_done.copy_(done)
    finally:
        torch.cuda.set_sync_debug_mode("default")
    adv, ret, _ = t.collect_rollout()
    torch.cuda.synchronize()
    check_rollout(t, adv, ret)
    rows = t.opp_assign
    counts = torch.bincount(rows, minlength=3).tolist()
    order = torch.argsort(rows, stable=True)
    cmd = t.env.action_buffer.view(t.nenv, 2, 4)
    off = c0 = agree = 0
    for g, c in enumerate(counts):
        if c == 0:
            continue
        lanes = order[c0:c0 + c]
        c0 += c
        lg = emulate(t.opponents[g].actor, t.x_opp[off:off + c, :184]).view(-1, 4, 21)
        agree += int((cmd[lanes, 1] == action_to_env(lg.argmax(-1), t.grid)).all(-1).sum())
        off += -(-c // 128) * 128
    assert agree >= 0.99 * t.nenv, f"opponent commands agree on {agree}/{t.nenv} rows"
    # the assignment follows opp_weights (1 : 1.5 : 2 over three opponents, 512 envs resampled)
    freq = torch.bincount(t._sample_opp(200_000), minlength=3).float() / 200_000
    assert torch.allclose(freq.cpu(), torch.tensor([1.0, 1.5, 2.0]) / 4.5, atol=0.01)


@pytest.mark.parametrize("opp_mode,n_opp", [("blocks", 2), ("pool", 3)])
def test_side_stream_rollout_bit_identical(cuda, opp_mode, n_opp):
    """The opponents' input prepared on a side stream gives the single-stream rollout's buffers,
    advantages and commands bit for bit (two rollouts, so the second starts from the first's
    end state; one opponent has its own normaliser)."""
    out = []
    for side in (False, True):
        t, tr = make_trainer(cuda, 768, n_opp, opp_mode, 9)
        t.side_stream_opponents = side
        t.reset(stagger=False)
        t.collect_rollout()
        adv, ret, stats = t.collect_rollout()
        torch.cuda.synchronize()
        out.append([t.b_obs.clone(), t.b_act.clone(), t.b_logp.clone(), t.b_val.clone(), t.b_rew.clone(),
                    t.b_done.clone(), adv, ret, t.env.action_buffer.clone(), t.x_opp.clone(), t.opp_assign.clone(),
                    stats["ep_count"].clone()])
        del t
    for i, (a, b) in enumerate(zip(*out)):
        assert torch.equal(a, b), f"buffer {i} differs between the side-stream and single-stream rollouts"
