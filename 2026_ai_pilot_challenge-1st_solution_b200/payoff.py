"""Batched payoff evaluation on the rollout kernels (R/cuda_fdm/batched_payoff.py; the
single-matchup evaluator R/cuda_fdm/ppo_gpu.py:1386-1575).

One left policy plays up to ``capacity`` right policies at once.  Matchup i owns the
``lanes = 2 * per_order`` consecutive environments ``[i * lanes, (i + 1) * lanes)`` of one
``GpuDogfightVecEnv``, each loaded with the same mirrored evaluation bank: in the first
``per_order`` lanes the left policy flies aircraft 0, in the rest aircraft 1, over byte-identical
initial conditions.  Every lane's first finished game is scored for the left policy.

Per step, on the device and without a host synchronisation:
  * one gather of every policy's observation rows (row groups: the left policy's rows for all
    matchups, then each right policy's rows, every group starting on a 128-row tile);
  * one normalise / 16-bit cast per policy (its own RunningNorm, or none);
  * ONE grouped ``f16_policy_forward`` launch for all policies -- each group with its own
    frozen weights -- sampling the 4 x 21-bin actions (Gumbel-max) and writing the env
    commands (action_to_env) in the epilogue;
  * one scatter of the commands into the env's command buffer, the fused env step, and
    ``f16_payoff_record`` (per-lane first-game scoring, matchup completion step, non-finite
    count).
The whole decision is captured once as a CUDA graph and replayed (the reference replays a
graph of its 128-row forwards); the RNG step and the scoring step come from a device counter
the graph advances.  The host reads completion and the non-finite count every ``check_every``
decisions (the reference reads them every decision); finished lanes are frozen, so the extra
decisions change no result.

Sampling is the kernel's counter-based Gumbel-max stream keyed by the evaluation seed, the
step and the row: replayable for a given seed, not torch.multinomial's stream (the
reference's per-matchup torch generators).  The league's bootstrap interval over paired
blocks (league.py paired_score_interval) is league statistics and stays with the caller:
``summarize_pair`` returns the ``paired_scores`` it is computed from.
"""
import math

import numpy as np
import torch

from . import _lib
from .policy import HEAD_CATEGORICAL, MlpWeights, PolicySet
from .rl_env import GpuDogfightVecEnv
from .rollout import cast_half, make_action_grid

TILE_ROWS = 128
MAX_POLICIES = 20            # networks one registered policy set can hold


class EvalPolicy:
    """A frozen policy: an actor logits network (an ``nn.Sequential`` or a module with
    ``actor_logits``) and its optional observation normaliser -- the reference's
    ``(net, norm, _)`` tuple.  ``obs_dim`` 184 or 214 (the external observation)."""

    def __init__(self, net, norm=None):
        self.actor = net.actor_logits if hasattr(net, "actor_logits") else net
        self.norm = norm
        linears = [m for m in self.actor if isinstance(m, torch.nn.Linear)]
        self.obs_dim = int(linears[0].in_features)
        if self.obs_dim not in (184, 214):
            raise ValueError("evaluation policies take the 184-D or the 214-D observation")


def outcome_summary(scores, altitude_losses):
    """PPOGPUTrainer._outcome_summary (ppo_gpu.py:1410-1418)."""
    scores = np.asarray(scores, dtype=np.float64)
    altitude_losses = np.asarray(altitude_losses, dtype=np.bool_)
    wins = int(np.count_nonzero(scores == 1.0))
    losses = int(np.count_nonzero(scores == 0.0))
    return {"score": float(scores.mean()), "games": int(scores.size), "wins": wins,
            "draws": int(scores.size - wins - losses), "losses": losses,
            "alt_loss_rate": float(altitude_losses.mean())}


def summarize_pair(scores, left_alt_loss, right_alt_loss, per_order, final_step, seed_block=0, eval_seed=0):
    """The fields of PPOGPUTrainer._summarize_clean_pair (ppo_gpu.py:1517-1575) that the
    evaluation itself determines; every value is from the left policy's perspective."""
    s = np.asarray(scores, dtype=np.float64)
    la = np.asarray(left_alt_loss, dtype=np.bool_)
    ra = np.asarray(right_alt_loss, dtype=np.bool_)
    fwd_s, swp_s = s[:per_order], s[per_order:]
    forward = outcome_summary(fwd_s, la[:per_order])
    reverse = outcome_summary(1.0 - swp_s, ra[per_order:])
    agg = outcome_summary(s, la)
    opp_losses = int(np.count_nonzero(ra))
    wins_by_opp_alt = int(np.count_nonzero((s == 1.0) & ra))
    own_losses = int(np.count_nonzero(la))
    losses_by_own_alt = int(np.count_nonzero((s == 0.0) & la))
    agg.update({
        "opponent_alt_loss_rate": float(ra.mean()),
        "opponent_alt_loss_count": opp_losses,
        "wins_by_opponent_altitude": wins_by_opp_alt,
        "wins_by_opponent_altitude_rate": float(wins_by_opp_alt / s.size),
        "wins_by_opponent_altitude_share": float(wins_by_opp_alt / agg["wins"]) if agg["wins"] else 0.0,
        "own_alt_loss_count": own_losses,
        "losses_by_own_altitude": losses_by_own_alt,
        "losses_by_own_altitude_rate": float(losses_by_own_alt / s.size),
        "altitude_diagnostic_protocol": "mirrored_terminal_cause_observability_v2",
        "forward": forward, "reverse": reverse, "paired_blocks": int(per_order), "seed_block": int(seed_block),
        "paired_scores": (0.5 * (fwd_s + swp_s)).tolist(), "deterministic": False, "stochastic": True,
        "policy_rng_seed": int(eval_seed), "steps": int(final_step)})
    return agg


class BatchedPayoff:
    """Batched evaluator of ``capacity`` matchups with ``per_order`` games per policy ordering
    (R/cuda_fdm/batched_payoff.py evaluate_chunk / evaluate_row)."""

    def __init__(self, per_order, capacity=16, *, substeps=6, seed=0, device="cuda", min_altitude_m=304.8,
                 max_engage_time_s=200.0, reward_cfg=None, alt_hunt_coef=5.0, num_bins=21, operand="fp16"):
        per_order = int(per_order)
        if per_order < 4 or per_order % 4:
            raise ValueError("per_order must be a positive multiple of 4 (ppo_gpu.py:1388)")
        if not 1 <= int(capacity) < MAX_POLICIES:
            raise ValueError(f"capacity must be between 1 and {MAX_POLICIES - 1}")
        self.per_order, self.capacity, self.lanes = per_order, int(capacity), 2 * per_order
        self.seed, self.num_bins = int(seed), int(num_bins)
        self.operand = operand                      # 16-bit operand type of the policy kernel
        kw = dict(substeps=substeps, seed=seed, device=device, min_altitude_m=min_altitude_m,
                  max_engage_time_s=max_engage_time_s, reward_cfg=reward_cfg, reward_mode=0,
                  alt_hunt_coef=alt_hunt_coef)
        # the bank of one matchup (the reference's template evaluation env), and the batch
        self.template = GpuDogfightVecEnv(self.lanes, **kw)
        self.env = GpuDogfightVecEnv(self.capacity * self.lanes, **kw)
        self.env.ic_pool_size = min(128, self.lanes)          # ppo_gpu.py:1405
        self.env.terminal_obs_enabled = False
        dev = self.device = self.env.device
        n = self.env.nenv
        lane = torch.arange(n, device=dev) % self.lanes
        self.left_slot = (lane >= per_order).to(torch.uint8)
        self.grid = make_action_grid(self.num_bins, device=dev)
        self.finished = torch.zeros(n, dtype=torch.uint8, device=dev)
        self.scores = torch.zeros(n, dtype=torch.float32, device=dev)
        self.own_crash = torch.zeros(n, dtype=torch.uint8, device=dev)
        self.opp_crash = torch.zeros(n, dtype=torch.uint8, device=dev)
        self.counts = torch.zeros(self.capacity + 1, dtype=torch.int32, device=dev)   # [nonfinite, per matchup]
        self.final_step = torch.zeros(self.capacity, dtype=torch.int32, device=dev)
        self.lib = _lib.load()

    # ---- row layout of one grouped policy launch ----
    def _layout(self, n_match):
        lanes, dev = self.lanes, self.device
        used = n_match * lanes
        tile = lambda r: -(-r // TILE_ROWS) * TILE_ROWS
        env = torch.arange(used, device=dev)
        ls = self.left_slot[:used].long()
        left_air = 2 * env + ls
        right_air = 2 * env + 1 - ls
        lpad, rpad = tile(used), tile(lanes)
        total = lpad + n_match * rpad
        src = torch.zeros(total, dtype=torch.long, device=dev)
        src[:used] = left_air
        groups, spans, valid = [(lpad, [0])], [(0, used)], [torch.arange(used, device=dev)]
        for i in range(n_match):
            b = lpad + i * rpad
            src[b:b + lanes] = right_air[i * lanes:(i + 1) * lanes]
            groups.append((b + rpad, [1 + i]))
            spans.append((b, b + lanes))
            valid.append(torch.arange(b, b + lanes, device=dev))
        valid = torch.cat(valid)
        return src, groups, spans, valid, src[valid].clone()

    @torch.no_grad()
    def evaluate(self, left, rights, *, seed_block=0, sample=True, check_every=8, use_graph=True):
        """One summary dict per right policy (the reference's evaluate_chunk).  With ``use_graph``
        the per-decision launches (gather, normalise, policy, scatter, env step, scoring) are
        one CUDA graph replayed every decision, like the reference's captured forwards."""
        rights = list(rights)
        if not 1 <= len(rights) <= self.capacity:
            raise ValueError("matchup count must be between one and batch capacity")
        env, dev, lanes = self.env, self.device, self.lanes
        n_match = len(rights)
        used = n_match * lanes
        pols = [left] + rights
        external = any(p.obs_dim == 214 for p in pols)
        # one launch shares one input layout: with a 214-D policy every first layer is widened
        # to 216 zero-padded columns
        nets = [MlpWeights.from_sequential(p.actor, HEAD_CATEGORICAL, dev, 4, self.num_bins,
                                           in_width=216 if external else None, operand=self.operand) for p in pols]
        pset = PolicySet(nets)
        if external:
            env.obr.enable_external_observations()
        in_pad = 256 if external else 192
        src, groups, spans, valid, dst = self._layout(n_match)
        total = src.numel()
        x184 = torch.zeros(total, 184, device=dev)
        x214 = torch.zeros(total, 214, device=dev) if external else None
        xb = torch.zeros(total, in_pad, dtype=pset.dtype, device=dev)
        cmd_rows = torch.zeros(total, 4, dtype=torch.float64, device=dev)

        # the mirrored bank of one matchup, repeated per matchup (batched_payoff.py:82-89)
        self.template.reset_evaluation(paired=True, seed_block=int(seed_block))
        bank = self.template._evaluation_seed_bank.view(lanes, 2, -1)
        env.sim.load_seed(bank.repeat(self.capacity, 1, 1))
        env.obr.reset_all()
        env.obr.kernel_init_reward_state(env.sim.states)
        env.obr.kernel_build_obs(env.sim.states)
        cmd = env.action_buffer
        cmd.zero_()
        self.finished.zero_()
        self.finished[used:] = 1
        self.scores.fill_(float("nan"))
        self.own_crash.zero_(); self.opp_crash.zero_()
        self.counts.zero_(); self.final_step.zero_()
        eval_seed = (self.seed * 1_000_003 + int(seed_block) * 97_409 + self.per_order * 193) % (2 ** 31 - 1)
        max_steps = math.ceil(float(env.max_engage_time_s) / float(env.obr.dt)) + 4
        args = _lib.PayoffArgs(left_slot=self.left_slot.data_ptr(), lanes=lanes, min_alt=float(env.min_altitude_m),
                               finished=self.finished.data_ptr(), scores=self.scores.data_ptr(),
                               own_crash=self.own_crash.data_ptr(), opp_crash=self.opp_crash.data_ptr(),
                               finished_count=self.counts[1:].data_ptr(), final_step=self.final_step.data_ptr(),
                               nonfinite=self.counts[:1].data_ptr())
        counter = torch.zeros(1, dtype=torch.int64, device=dev)     # decisions taken before this one
        args.step, args.step_dev = 1, counter.data_ptr()
        keep = {}

        def decision():
            obs = env.obr.obs_buf.view(env.nac, 184)
            torch.index_select(obs, 0, src, out=x184)
            if external:
                torch.index_select(env.obr.build_external_obs(env.sim.states), 0, src, out=x214)
            for p, (a, b) in zip(pols, spans):
                x = (x214 if p.obs_dim == 214 else x184)[a:b]
                if p.norm is not None:
                    p.norm.normalize_half(x, out_half=xb[a:b], pad_to=in_pad)
                else:
                    cast_half(x, xb[a:b])
            pset.forward(xb, groups, seed=eval_seed, step=1, step_dev=counter, deterministic=not sample,
                         cmd=cmd_rows, cmd_stride=4, cmd_offset=0, grid=self.grid)
            cmd.index_copy_(0, dst, cmd_rows.index_select(0, valid))
            _, _, _, info = env.step(cmd)
            keep["finite"] = info["terminal_state_finite"].to(torch.uint8)
            args.done = env._done.data_ptr()
            args.terminal_hp, args.terminal_alt = env._terminal_hp.data_ptr(), env._terminal_alt.data_ptr()
            args.finite = keep["finite"].data_ptr()
            args.reward = env.obr.reward_buf.data_ptr()
            _lib.check(self.lib.f16_payoff_record(env.nenv, args, _lib.stream_of(self.scores)), "f16_payoff_record")
            counter.add_(1)

        # the first decision runs eagerly (it also initialises every lazily built buffer); the
        # rest replay one captured CUDA graph of it, the step counter advancing on the device
        decision()
        graph = None
        if use_graph:
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                decision()
        complete = False
        for step in range(1, max_steps + 1):
            if step > 1:
                if graph is not None:
                    graph.replay()
                else:
                    decision()
            if step % int(check_every) == 0 or step == max_steps:
                c = self.counts[:1 + n_match].tolist()
                if c[0]:
                    raise FloatingPointError("non-finite batched league evaluation trajectory")
                if all(v == lanes for v in c[1:]):
                    complete = True
                    break
        del graph
        pset.check_error()
        s = self.scores[:used].view(n_match, lanes).cpu().numpy()
        oc = self.own_crash[:used].view(n_match, lanes).cpu().numpy().astype(bool)
        pc = self.opp_crash[:used].view(n_match, lanes).cpu().numpy().astype(bool)
        steps = self.final_step[:n_match].tolist()
        if not complete or not np.isfinite(s).all():
            raise RuntimeError("batched evaluation did not complete every required game")
        pset.close()
        return [summarize_pair(s[i], oc[i], pc[i], self.per_order, steps[i], seed_block, eval_seed)
                for i in range(n_match)]
