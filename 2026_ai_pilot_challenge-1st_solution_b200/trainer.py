"""PPO rollout collection and update of the feed-forward lineage on the sm_100a kernels.

Mirrors ``PPOGPUTrainer`` of the reference (R/cuda_fdm/ppo_gpu.py) for the MLP actor/critic:

* ``collect_rollout`` (:1856-2017): per decision step RunningNorm update + normalise (one
  kernel writes the fp32 rollout row and the bf16 policy input), ONE tcgen05 launch for actor
  sample + log-prob + critic value that also writes the env commands (action_to_env fused),
  one grouped launch for the frozen opponents, then the env step (FDM kernel + fused
  post-step kernel).  The episode statistics are the reference's torch expressions.  After T
  steps: bootstrap value (critic launch) and the bit-exact GAE kernel.
* ``update`` (:2020-2144): the reference's clipped-PPO minibatch loop in torch (fp32), with
  the data-parallel additions of a multi-GPU run: gradients all-reduced (mean, one flat bucket
  per optimiser) before the norm clip, minibatch advantage statistics and approx-KL reduced
  over ranks, so every rank applies the same optimiser step.
* ``MLPActorCritic``: the reference architecture (R/claude_code/model.py:34-44 ``_mlp``,
  :162-241 ``MLPDiscreteActorCritic``; ppo_gpu.py:248-290), same parameter names, so
  checkpoints load unchanged.

Opponents: ``opp_mode="blocks"`` gives opponent g the contiguous environment block g (the
benchmark configuration); ``opp_mode="pool"`` keeps a per-environment assignment resampled at
episode ends from ``opp_weights`` (``_sample_opp``, :1306-1309) and regroups the rows each step
on the device -- counts, tile-padded group ends and destination rows from torch ops, one
normalise-and-scatter launch with each opponent's own normaliser, one grouped policy launch that
reads the group ends from device memory -- so, unlike ``ActiveLeaguePool.act``'s
``bincount().cpu()`` (:879-880), a step never waits on the host.
"""
import ctypes as C
import dataclasses
from typing import Optional

import numpy as np
import torch
import torch.nn as nn

from . import _lib
from . import categorical
from . import splitmm
from .policy import HEAD_CATEGORICAL, HEAD_VALUE, MlpWeights, PolicySet
from .rollout import RunningNorm, cast_half, gae, half_operand, make_action_grid

OBS_DIM = 184
ACT_DIM = 4
ACTION_BINS = 21
IN_PAD = 192            # 16-bit policy input row: 184 features + zero padding to a 64-byte multiple
TILE_ROWS = 128         # MLP kernel row tile; opponent groups start on a multiple of it
NORM_CLIP, NORM_EPS = 10.0, 1e-8    # RunningNorm's clip and eps (ppo_gpu.py:184-222)

_ACTIVATIONS = {"tanh": nn.Tanh, "relu": nn.ReLU}


def mlp(in_dim, hidden, out_dim, activation):
    """Linear -> act -> ... -> Linear (model.py:34-44)."""
    layers, last = [], in_dim
    for h in hidden:
        layers += [nn.Linear(last, h), _ACTIVATIONS[activation]()]
        last = h
    layers.append(nn.Linear(last, out_dim))
    return nn.Sequential(*layers)


class MLPActorCritic(nn.Module):
    """Independent categorical actor (act_dim x num_bins logits) and value critic."""

    is_recurrent = False
    state_size = 1

    def __init__(self, obs_dim=OBS_DIM, act_dim=ACT_DIM, num_bins=ACTION_BINS, hidden=(512, 512, 512),
                 activation="tanh", critic_hidden=None, critic_activation=None):
        super().__init__()
        self.obs_dim, self.act_dim, self.num_bins = int(obs_dim), int(act_dim), int(num_bins)
        self.hidden = list(hidden)
        self.activation = activation
        self.critic_hidden = list(critic_hidden) if critic_hidden is not None else list(hidden)
        self.critic_activation = critic_activation or activation
        self.actor_logits = mlp(obs_dim, hidden, self.act_dim * self.num_bins, activation)
        self.critic = mlp(obs_dim, self.critic_hidden, 1, self.critic_activation)
        self.apply(self._init_weights)

    @staticmethod
    def _init_weights(module):
        # orthogonal(gain sqrt 2) weights, zero biases (model.py:87-90)
        if isinstance(module, nn.Linear):
            nn.init.orthogonal_(module.weight, gain=np.sqrt(2))
            nn.init.zeros_(module.bias)

    def actor_parameters(self):
        return list(self.actor_logits.parameters())

    def critic_parameters(self):
        return list(self.critic.parameters())

    # set by the PPO update on CUDA: linear layers through splitmm (fp32-accurate products on the
    # bf16 tensor cores) instead of SGEMM and the categorical head through its fused kernels; the
    # modules and their parameters are the same
    split_products = False

    def _run(self, seq, x):
        if not self.split_products:
            return seq(x)
        return splitmm.run_tower(seq, x)

    def _dist(self, obs):
        return torch.distributions.Categorical(logits=self._run(self.actor_logits, obs).view(-1, self.act_dim,
                                                                                              self.num_bins))

    def get_value(self, obs):
        return self._run(self.critic, obs).squeeze(-1)

    def evaluate_actions(self, obs, action):
        """(summed log-prob, summed entropy) of category indices under the current actor."""
        if self.split_products and obs.dim() == 2:
            logits = self._run(self.actor_logits, obs)
            if categorical.usable(logits, self.act_dim, self.num_bins):
                return categorical.logp_entropy(logits, action, self.act_dim, self.num_bins)
            dist = torch.distributions.Categorical(logits=logits.view(-1, self.act_dim, self.num_bins))
            return dist.log_prob(action.long()).sum(-1), dist.entropy().sum(-1)
        dist = self._dist(obs)
        action = action.long()
        return dist.log_prob(action).sum(-1), dist.entropy().sum(-1)


@dataclasses.dataclass
class PPOConfig:
    """The PPOGPUConfig fields (ppo_gpu.py:950-980) that the MLP rollout and update read."""
    rollout_steps: int = 32
    gamma: float = 0.997
    gae_lambda: float = 0.95
    clip_coef: float = 0.2
    update_epochs: int = 4
    num_minibatches: int = 8
    lr: float = 3e-4
    critic_lr: Optional[float] = None
    ent_coef: float = 0.0
    vf_coef: float = 0.5
    max_grad_norm: float = 0.5
    target_kl: Optional[float] = 0.03
    num_bins: int = ACTION_BINS
    hidden: tuple = (512, 512, 512)
    activation: str = "tanh"
    normalize_obs: bool = True
    norm_adv: bool = True
    opp_sample: bool = True
    seed: int = 0
    # 16-bit operand type of the rollout-time policy kernel: "fp16" keeps logits / log-probs
    # within 1e-3 of the fp32 networks at the same tensor rate as "bf16" (about 4e-3)
    policy_operand: str = "fp16"


class Opponent:
    """A frozen actor (an ``MLPActorCritic`` or a bare logits ``nn.Sequential``) with its own
    optional observation normaliser, as a pool entry's ``net`` / ``norm``."""

    def __init__(self, net, norm=None):
        self.actor = net.actor_logits if hasattr(net, "actor_logits") else net
        self.norm = norm


def _mix64(x):
    x = (x + 0x9E3779B97F4A7C15) & 0xFFFFFFFFFFFFFFFF
    x = ((x ^ (x >> 30)) * 0xBF58476D1CE4E5B9) & 0xFFFFFFFFFFFFFFFF
    x = ((x ^ (x >> 27)) * 0x94D049BB133111EB) & 0xFFFFFFFFFFFFFFFF
    return x ^ (x >> 31)


def _world(group):
    if group is None:
        return 1
    import torch.distributed as dist
    return dist.get_world_size(group)


def _allreduce_mean_(tensors, group, world):
    """All-reduce the gradients of ``tensors`` as one flat bucket and divide by the world size."""
    if world == 1:
        return
    import torch.distributed as dist
    grads = [p.grad for p in tensors if p.grad is not None]
    flat = torch.cat([g.reshape(-1) for g in grads])
    dist.all_reduce(flat, group=group)
    flat.div_(world)
    off = 0
    for g in grads:
        n = g.numel()
        g.copy_(flat[off:off + n].view_as(g))
        off += n


def ppo_update(model, actor_opt, critic_opt, cfg, obs, act, old_logp, b_val, adv, ret, group=None, generator=None,
               split_products=None):
    """Clipped PPO over one rollout (ppo_gpu.py:2020-2144, ``aux_pred`` off).

    obs (T, n, 184) fp32, act (T, n, 4) indices (any integer dtype), old_logp / b_val / adv / ret
    (T, n) fp32.  Single rank: the reference's arithmetic op for op.  With a process group of W
    ranks, each rank permutes its own shard; gradients are averaged over ranks before the norm
    clip, and the minibatch advantage mean / std and the epoch approx-KL are those of the union
    of the ranks' minibatches, so all ranks take identical optimiser steps and the update equals
    a single-rank update whose minibatch is the concatenation of the ranks' minibatches.
    """
    world = _world(group)
    dev = obs.device
    # fp32-accurate split products on the tensor cores for the CUDA update (splitmm); the CPU
    # path (and split_products=False) multiplies in plain fp32
    prev_split = model.split_products
    model.split_products = (dev.type == "cuda") if split_products is None else bool(split_products)
    try:
        return _ppo_update(model, actor_opt, critic_opt, cfg, obs, act, old_logp, b_val, adv, ret, group, generator)
    finally:
        model.split_products = prev_split


def _ppo_update(model, actor_opt, critic_opt, cfg, obs, act, old_logp, b_val, adv, ret, group, generator):
    world = _world(group)
    dev = obs.device
    obs_f = obs.flatten(0, 1)
    act_f = act.flatten(0, 1)
    old_logp_f = old_logp.flatten()
    advantages, returns = adv.flatten(), ret.flatten()
    count = int(obs_f.shape[0])
    if count == 0 or cfg.update_epochs < 1 or cfg.num_minibatches < 1:
        raise ValueError("MLP PPO requires nonempty rollout, positive epochs and minibatches")
    if tuple(adv.shape) != tuple(b_val.shape) or tuple(ret.shape) != tuple(b_val.shape):
        raise ValueError("advantage/return shape must match the rollout values")
    mb_size = (count + cfg.num_minibatches - 1) // cfg.num_minibatches
    clip = cfg.clip_coef
    zero = torch.zeros((), device=dev)
    last_pl = last_vl = last_ent = last_kl = last_cf = zero
    last_actor_grad = last_critic_grad = zero
    early = False
    epoch = 0
    optimizer_steps = 0
    if world > 1:
        import torch.distributed as dist
    for epoch in range(cfg.update_epochs):
        perm = torch.randperm(count, device=dev, generator=generator)
        kls = []
        for s in range(0, count, mb_size):
            mb = perm[s:s + mb_size]
            mb_obs = obs_f.index_select(0, mb)
            setattr(mb_obs, splitmm.SHARE_SPLIT, True)   # actor and critic share its split
            new_logp, entropy = model.evaluate_actions(mb_obs, act_f.index_select(0, mb))
            log_ratio = new_logp - old_logp_f.index_select(0, mb)
            ratio = log_ratio.exp()
            mb_adv = advantages.index_select(0, mb)
            if world == 1:
                if cfg.norm_adv and mb_adv.numel() > 1:
                    mb_adv = (mb_adv - mb_adv.mean()) / (mb_adv.std() + 1e-8)
            elif cfg.norm_adv:
                # mean and sample std of the union of the ranks' minibatches (two passes; the
                # union has at least `world` >= 2 rows, so the sample std is always defined)
                st = torch.stack([mb_adv.sum(), mb_adv.new_full((), float(mb_adv.numel()))])
                dist.all_reduce(st, group=group)
                mean = st[0] / st[1]
                sq = ((mb_adv - mean) ** 2).sum()
                dist.all_reduce(sq, group=group)
                mb_adv = (mb_adv - mean) / (torch.sqrt(sq / (st[1] - 1)) + 1e-8)
            pg1 = -mb_adv * ratio
            pg2 = -mb_adv * torch.clamp(ratio, 1 - clip, 1 + clip)
            policy_loss = torch.max(pg1, pg2).mean()
            ent = entropy.mean()

            actor_opt.zero_grad(set_to_none=True)
            actor_loss = policy_loss - cfg.ent_coef * ent
            actor_loss.backward()
            _allreduce_mean_(model.actor_parameters(), group, world)
            last_actor_grad = nn.utils.clip_grad_norm_(model.actor_parameters(), cfg.max_grad_norm)
            actor_opt.step()

            new_value = model.get_value(mb_obs)
            value_loss = 0.5 * ((new_value - returns.index_select(0, mb)) ** 2).mean()
            critic_opt.zero_grad(set_to_none=True)
            critic_loss = cfg.vf_coef * value_loss
            critic_loss.backward()
            _allreduce_mean_(model.critic_parameters(), group, world)
            last_critic_grad = nn.utils.clip_grad_norm_(model.critic_parameters(), cfg.max_grad_norm)
            critic_opt.step()
            optimizer_steps += 1

            with torch.no_grad():
                kls.append(((ratio - 1.0) - log_ratio).mean())
                clipfrac = ((ratio - 1.0).abs() > clip).float().mean()
            last_pl = policy_loss.detach(); last_vl = value_loss.detach()
            last_ent = ent.detach(); last_cf = clipfrac
        last_kl = torch.stack(kls).mean()
        if world > 1:
            dist.all_reduce(last_kl, group=group)
            last_kl = last_kl / world
        if cfg.target_kl is not None and float(last_kl) > cfg.target_kl:
            early = True
            break

    b_ret = ret.reshape(-1)
    b_v = b_val.reshape(-1)
    var_y = b_ret.var() if count > 1 else torch.zeros((), device=dev)
    ev = torch.where(var_y == 0, torch.zeros((), device=dev),
                     1.0 - (b_ret - b_v).var(correction=1 if count > 1 else 0) / (var_y + 1e-8))
    return {"pl": last_pl, "vl": last_vl, "ent": last_ent, "kl": last_kl, "cf": last_cf, "ev": ev,
            "epochs": epoch + 1, "early": early, "actor_grad_norm": last_actor_grad.detach(),
            "critic_grad_norm": last_critic_grad.detach(), "optimizer_steps": optimizer_steps}


class PPOTrainer:
    """Rollout + update driver over a ``GpuDogfightVecEnv``.

    env        : rl_env.GpuDogfightVecEnv (this rank's environments)
    opponents  : list of ``Opponent`` (at most 18: the kernel registers 20 networks)
    opp_mode   : "blocks" or "pool" (module docstring)
    group      : torch.distributed process group for data-parallel training, or None
    """

    # True: collect_rollout prepares the opponents' input on a side stream (overlapping the
    # learner's normalise and forward); False: everything on the current stream.
    side_stream_opponents = True

    def __init__(self, env, cfg=None, model=None, opponents=(), opp_mode="blocks", opp_weights=None, group=None,
                 keep_terminal_obs=False):
        self.env = env
        self.cfg = cfg = cfg or PPOConfig()
        self.device = dev = env.device
        self.nenv, self.nac = env.nenv, env.nac
        self.group = group
        self.world = _world(group)
        self.rank = 0
        if self.world > 1:
            import torch.distributed as dist
            self.rank = dist.get_rank(group)
        self.model = (model or MLPActorCritic(OBS_DIM, ACT_DIM, cfg.num_bins, cfg.hidden, cfg.activation)).to(dev)
        if self.world > 1:
            import torch.distributed as dist
            for p in self.model.parameters():        # identical start on every rank
                dist.broadcast(p.data, src=dist.get_global_rank(group, 0) if group is not None else 0,
                               group=group)
        self.norm = RunningNorm(OBS_DIM, dev) if cfg.normalize_obs else None
        clr = cfg.lr if cfg.critic_lr is None else cfg.critic_lr
        self.actor_opt = torch.optim.Adam(self.model.actor_parameters(), lr=cfg.lr, eps=1e-5)
        self.critic_opt = torch.optim.Adam(self.model.critic_parameters(), lr=clr, eps=1e-5)
        self.grid = make_action_grid(cfg.num_bins, device=dev)
        if not keep_terminal_obs:
            env.terminal_obs_enabled = False      # collect_rollout never reads info["terminal_obs"]

        self.opponents = list(opponents)
        if len(self.opponents) > 18:
            raise ValueError("at most 18 frozen opponents (20 registered networks incl. actor and critic)")
        if opp_mode not in ("blocks", "pool"):
            raise ValueError("opp_mode must be 'blocks' or 'pool'")
        if not self.opponents:
            raise ValueError("at least one opponent is required")
        self.opp_mode = opp_mode
        op = cfg.policy_operand
        self._main_w = [MlpWeights.from_sequential(self.model.actor_logits, HEAD_CATEGORICAL, dev, ACT_DIM,
                                                   cfg.num_bins, operand=op),
                        MlpWeights.from_sequential(self.model.critic, HEAD_VALUE, dev, operand=op)]
        self._opp_w = [MlpWeights.from_sequential(o.actor, HEAD_CATEGORICAL, dev, ACT_DIM, cfg.num_bins, operand=op)
                       for o in self.opponents]
        self.policy = PolicySet(self._main_w + self._opp_w)
        P = len(self.opponents)
        if opp_weights is None:
            opp_weights = torch.full((P,), 1.0 / P)
        self.opp_weights = torch.as_tensor(opp_weights, dtype=torch.float32, device=dev)
        blk = -(-self.nenv // P)
        blk = -(-blk // TILE_ROWS) * TILE_ROWS
        self._blocks = [(g * blk, min((g + 1) * blk, self.nenv)) for g in range(P) if g * blk < self.nenv]
        self.opp_assign = torch.zeros(self.nenv, dtype=torch.long, device=dev)
        for g, (a, b) in enumerate(self._blocks):
            self.opp_assign[a:b] = g

        T, n = cfg.rollout_steps, self.nenv
        self.b_obs = torch.zeros(T, n, OBS_DIM, device=dev)
        self.b_act = torch.zeros(T, n, ACT_DIM, dtype=torch.uint8, device=dev)
        self.b_logp = torch.zeros(T, n, device=dev)
        self.b_val = torch.zeros(T, n, device=dev)
        self.b_rew = torch.zeros(T, n, device=dev)
        self.b_done = torch.zeros(T, n, device=dev)
        self.x_main = torch.zeros(n, IN_PAD, dtype=self.policy.dtype, device=dev)
        pad_rows = n + P * TILE_ROWS
        self.x_opp = torch.zeros(pad_rows, IN_PAD, dtype=self.policy.dtype, device=dev)
        self._opp_cmd = torch.zeros(pad_rows, ACT_DIM, dtype=torch.float64, device=dev) if opp_mode == "pool" else None
        if opp_mode == "pool":
            # device-side grouping buffers and each opponent's normaliser statistics (NULL: none)
            self._pool_counts = torch.zeros(P, dtype=torch.int64, device=dev)
            self._pool_ends = torch.zeros(P, dtype=torch.int64, device=dev)
            self._pool_ones = torch.ones(n, dtype=torch.int64, device=dev)
            self._pool_iota = torch.arange(n, dtype=torch.int64, device=dev)
            self._pool_rank = torch.zeros(n, dtype=torch.int64, device=dev)
            for o in self.opponents:
                if o.norm is not None and (o.norm.clip != NORM_CLIP or o.norm.eps != NORM_EPS):
                    raise ValueError("pool-mode opponent normalisers must use the trainer's clip and eps")
            self._pool_mean_ptrs = torch.tensor([o.norm.mean.data_ptr() if o.norm is not None else 0
                                                 for o in self.opponents], dtype=torch.int64, device=dev)
            self._pool_var_ptrs = torch.tensor([o.norm.var.data_ptr() if o.norm is not None else 0
                                                for o in self.opponents], dtype=torch.int64, device=dev)
        self.last_value = torch.zeros(n, device=dev)
        self.ep_ret = torch.zeros(n, device=dev)
        self.ep_len = torch.zeros(n, device=dev)
        self._stats = torch.zeros(8 + 3 * P, dtype=torch.float64, device=dev)
        self._nonfinite = torch.zeros(1, dtype=torch.int32, device=dev)
        self._lib = _lib.load()
        self.global_step = 0
        self.decisions = 0
        self._key_main = _mix64((cfg.seed << 8) ^ (self.rank << 1))
        self._key_opp = _mix64((cfg.seed << 8) ^ (self.rank << 1) ^ 1)
        self.min_alt = env.min_altitude_m
        self._next_obs = self._next_opp_obs = None
        self._side_stream = self._opp_ready = None
        self._next_done = torch.zeros(n, device=dev)
        self._rec = _lib.RecordArgs(n_opp=P, min_alt=float(self.min_alt), next_done=self._next_done.data_ptr(),
                                    ep_ret=self.ep_ret.data_ptr(), ep_len=self.ep_len.data_ptr(),
                                    stats=self._stats.data_ptr())

    # ---- weights ----
    def refresh_policy(self):
        """Copy the learner's parameters into the kernel's 16-bit buffers (after ``update``)."""
        self._main_w[0].load_from(self.model.actor_logits)
        self._main_w[1].load_from(self.model.critic)

    # ---- env ----
    def reset(self, stagger=True):
        obs = self.env.reset(stagger=bool(stagger))
        self._next_obs = obs[:, 0, :]
        self._next_opp_obs = obs[:, 1, :]
        self._next_done.zero_()
        self.ep_ret.zero_(); self.ep_len.zero_()
        if self.opp_mode == "pool":
            self.opp_assign = self._sample_opp(self.nenv)

    def _sample_opp(self, n):
        """n opponent indices drawn with probabilities proportional to ``opp_weights`` (the
        reference's multinomial with replacement, :1306-1309), as an inverse-CDF lookup of
        uniform draws so no step waits on the host."""
        cdf = torch.cumsum(self.opp_weights, 0)
        u = torch.rand(n, device=self.device) * cdf[-1]
        return torch.searchsorted(cdf, u, right=True).clamp_(max=len(self.opponents) - 1)

    def _normalize_into(self, norm, x, out_half, out_f32=None, nonfinite=None):
        if norm is not None:
            norm.normalize_half(x, out_f32=out_f32, out_half=out_half, pad_to=IN_PAD, nonfinite=nonfinite)
        else:
            cast_half(x, out_half, out_f32=out_f32, nonfinite=nonfinite)

    def _opponents_prepare(self):
        """The opponents' 16-bit policy input ``x_opp`` from their observation rows: each block's
        own normaliser or a plain cast ("blocks"); in "pool" mode the rows grouped by assigned
        opponent on the device and normalised into their group slots.  Returns what
        ``_opponents_forward`` launches with (the block groups, or each env's grouped row)."""
        opp_obs = self._next_opp_obs
        if self.opp_mode == "blocks":
            groups = []
            run = None                                  # consecutive blocks without a normaliser
            for g, (a, b) in enumerate(self._blocks):
                if self.opponents[g].norm is None:
                    run = (run[0] if run else a, b)
                else:
                    if run:
                        cast_half(opp_obs[run[0]:run[1]], self.x_opp[run[0]:run[1]])
                        run = None
                    self._normalize_into(self.opponents[g].norm, opp_obs[a:b], self.x_opp[a:b])
                groups.append((b, [2 + g]))
            if run:
                cast_half(opp_obs[run[0]:run[1]], self.x_opp[run[0]:run[1]])
            return groups
        # pool: rows grouped by assigned opponent on the device (no host round trip): per-group
        # counts, tile-padded cumulative ends, and each env's destination row (its rank within
        # its group after a stable sort, as the reference's argsort + split, ppo_gpu.py:877-898)
        rows = self.opp_assign
        P = len(self.opponents)
        counts = self._pool_counts.zero_().index_add_(0, rows, self._pool_ones)
        padded = (counts + (TILE_ROWS - 1)) // TILE_ROWS * TILE_ROWS
        torch.cumsum(padded, 0, out=self._pool_ends)
        order = torch.argsort(rows, stable=True)
        self._pool_rank.index_copy_(0, order, self._pool_iota)
        first = torch.cumsum(counts, 0) - counts                  # sorted position of each group's first row
        dst = (self._pool_ends - padded).index_select(0, rows) + self._pool_rank - first.index_select(0, rows)
        _lib.check(self._lib.f16_norm_apply_scatter(
            _lib.ptr(opp_obs), self.nenv, OBS_DIM, opp_obs.stride(0), _lib.ptr(rows), _lib.ptr(dst),
            _lib.ptr(self._pool_mean_ptrs), _lib.ptr(self._pool_var_ptrs), P, NORM_EPS, NORM_CLIP,
            _lib.ptr(self.x_opp), self.x_opp.stride(0), half_operand(self.x_opp), None,
            _lib.stream_of(self.x_opp)), "f16_norm_apply_scatter")
        return dst

    def _opponents_forward(self, cmd, prep):
        """Opponent commands into the odd aircraft rows of ``cmd`` (nac, 4) from the input that
        ``_opponents_prepare`` wrote (``prep``: its return value)."""
        cfg = self.cfg
        kw = dict(seed=self._key_opp, step=self.decisions, deterministic=not cfg.opp_sample, grid=self.grid)
        if self.opp_mode == "blocks":
            self.policy.forward(self.x_opp[:self.nenv], prep, cmd=cmd, cmd_stride=2 * ACT_DIM, cmd_offset=ACT_DIM,
                                **kw)
            return
        P = len(self.opponents)
        self.policy.forward(self.x_opp, [(0, [2 + g]) for g in range(P)], group_end_dev=self._pool_ends,
                            cmd=self._opp_cmd, cmd_stride=ACT_DIM, cmd_offset=0, **kw)
        cmd.view(self.nenv, 2 * ACT_DIM)[:, ACT_DIM:].copy_(self._opp_cmd.index_select(0, prep))

    def _opponents_act(self, cmd):
        """Opponent commands into the odd aircraft rows of ``cmd`` (nac, 4), on the current stream."""
        self._opponents_forward(cmd, self._opponents_prepare())

    # ---- rollout (ppo_gpu.py:1856-2017) ----
    @torch.no_grad()
    def collect_rollout(self, update_norm=True):
        cfg = self.cfg
        T, dev, nenv = cfg.rollout_steps, self.device, self.nenv
        if self._next_obs is None:
            self.reset()
        P = len(self.opponents)
        self._stats.zero_()
        self._nonfinite.zero_()
        rec = self._rec
        cmd = self.env.action_buffer
        # The opponents' input is prepared on a side stream while the learner's normalise and
        # forward run on the current one: the two read different observation rows and write
        # different inputs, and the opponents' forward waits for it (-1.2% per rollout; the
        # buffers are the single-stream rollout's bit for bit).
        cur = torch.cuda.current_stream(dev)
        use_side = self.side_stream_opponents
        if use_side and self._side_stream is None:
            self._side_stream, self._opp_ready = torch.cuda.Stream(dev), torch.cuda.Event()
        side, ready = self._side_stream, self._opp_ready

        for t in range(T):
            if self.opp_mode == "pool":
                sampled = self._sample_opp(nenv)
                self.opp_assign = torch.where(self._next_done.bool(), sampled, self.opp_assign)
            if use_side:
                side.wait_stream(cur)       # this decision's observations, the last forward's reads done
                with torch.cuda.stream(side):
                    prep = self._opponents_prepare()
                ready.record(side)
                if self.opp_mode == "pool":
                    prep.record_stream(cur)  # each env's grouped row, read again on this stream
            else:
                prep = self._opponents_prepare()
            main_obs = self._next_obs
            if self.norm is not None and update_norm:
                self.norm.update(main_obs, self.group)
            self._normalize_into(self.norm, main_obs, self.x_main, out_f32=self.b_obs[t], nonfinite=self._nonfinite)
            self.b_done[t].copy_(self._next_done)
            # actor sample + log-prob + env commands (even aircraft) and critic value, one launch
            self.policy.forward(self.x_main, [(nenv, [0, 1])], nets_per_group=2, bins=self.b_act[t],
                                bins_stride=ACT_DIM, logp=self.b_logp[t], value=self.b_val[t],
                                seed=self._key_main, step=self.decisions, cmd=cmd, cmd_stride=2 * ACT_DIM,
                                cmd_offset=0, grid=self.grid)
            if use_side:
                cur.wait_event(ready)
            self._opponents_forward(cmd, prep)
            self.decisions += 1
            obs, reward, done, info = self.env.step(cmd)
            self._next_obs = obs[:, 0, :]
            self._next_opp_obs = obs[:, 1, :]
            self.global_step += nenv
            # reward row, next-done, episode return / length and the win / loss statistics of
            # ppo_gpu.py:1914-1960 in one kernel (f16_rollout_record)
            th, ta, fin = info["terminal_hp"], info["terminal_alt_m"], info["terminal_state_finite"]
            rec.reward, rec.done = reward.data_ptr(), done.data_ptr()
            rec.terminal_hp, rec.terminal_alt, rec.finite = th.data_ptr(), ta.data_ptr(), fin.data_ptr()
            rec.opp_row = self.opp_assign.data_ptr()
            rec.b_rew = self.b_rew[t].data_ptr()
            _lib.check(self._lib.f16_rollout_record(nenv, C.byref(rec), _lib.stream_of(self.b_rew)),
                       "f16_rollout_record")

        self._normalize_into(self.norm, self._next_obs, self.x_main)
        self.policy.forward(self.x_main, [(nenv, [1])], value=self.last_value)
        adv, ret = gae(self.b_rew, self.b_val, self.b_done, self.last_value, self._next_done, cfg.gamma,
                       cfg.gae_lambda)

        st = self._stats.float()
        # every b_obs row came out of the checked normalise / cast kernel, whose counter stands
        # in for torch.isfinite(b_obs).all() (one pass over the 6 GB buffer saved per rollout)
        finite_checks = [st[7] == 0, self._nonfinite[0] == 0]
        finite_checks.extend(torch.isfinite(x).all() for x in (self.b_rew, self.b_val, self.b_logp, adv, ret))
        if not bool(torch.stack(finite_checks).all()):
            raise FloatingPointError("non-finite physical trajectory or PPO rollout; update refused")
        self.policy.check_error()
        names = ("ret_sum", "len_sum", "ep_count", "win_sum", "loss_sum", "alt_loss_sum", "opponent_alt_loss_sum")
        stats = {k: st[i] for i, k in enumerate(names)}
        stats["win_by_opp"] = st[8:8 + P]
        stats["loss_by_opp"] = st[8 + P:8 + 2 * P]
        stats["ep_by_opp"] = st[8 + 2 * P:8 + 3 * P]
        return adv, ret, stats

    def reduce_stats(self, stats):
        """Sum the rollout statistics over the ranks (league EMA inputs); no-op on one rank."""
        if self.world == 1:
            return stats
        import torch.distributed as dist
        keys = sorted(stats)
        flat = torch.cat([stats[k].reshape(-1).float() for k in keys])
        dist.all_reduce(flat, group=self.group)
        out, off = {}, 0
        for k in keys:
            n = stats[k].numel()
            out[k] = flat[off:off + n].view_as(stats[k])
            off += n
        return out

    # ---- update (ppo_gpu.py:2020-2144) ----
    # None: fp32-accurate split products on CUDA (splitmm); False: plain fp32 matmuls (then TF32
    # when torch.backends.cuda.matmul.allow_tf32 is set)
    split_products = None

    def update(self, adv, ret, generator=None):
        res = ppo_update(self.model, self.actor_opt, self.critic_opt, self.cfg, self.b_obs, self.b_act, self.b_logp,
                         self.b_val, adv, ret, group=self.group, generator=generator,
                         split_products=self.split_products)
        self.refresh_policy()
        return res

    def iteration(self):
        adv, ret, stats = self.collect_rollout()
        return self.update(adv, ret), self.reduce_stats(stats)
