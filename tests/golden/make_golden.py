#!/usr/bin/env python3
"""Regenerate the golden fixtures in tests/golden/ from the reference itself.

Run only where the reference tree is available (the ``F16_REFERENCE`` directory or the default local checkout); the
GPU box never runs this.  What each fixture pins:

fdm_cfg1.npz  BASELINE configs[0]: 64 envs x 2 F-16s, seeded ICs (altitude U(6,9) km, Mach
              U(0.6,0.9), head-on 10 km apart, heading offsets U(-30,30) deg, fuel 6000 lb)
              whose seed rows come from the reference's Python ``cuda_fdm.ic.build_seed_vector``;
              random 4x21-bin actions held 6 frames, 100 decisions; states after 1, 6 and 600
              frames and obs17 after 600 frames from the reference's own fdm.cuh (oracle/_ref,
              repository-root lineage, FCS dt 1/120).
fdm_r36.npz   the same ICs (first 16 envs) through the research/competition_36500 lineage
              (FCS dt 1/60) seed builder and fdm.cuh, 60 frames.
obs_traj.npz, gae.npz, norm.npz, ppo_update.npz, payoff.npz: see make_obs_golden,
              make_gae_golden, make_norm_golden, make_ppo_golden and make_payoff_golden below.
"""
import importlib
import os
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
REF = Path(os.environ.get("F16_REFERENCE") or ROOT.parent / "reference")
OUT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(OUT))

from oracle import fdm as ofdm  # noqa: E402

pkg = importlib.import_module("2026_ai_pilot_challenge-1st_solution_b200")
ic_mod = importlib.import_module(pkg.__name__ + ".ic")

SEED_CFG1 = 20260101
NENV_CFG1 = 64


def ref_seed_rows(ic_rows, lineage_root):
    """Seed rows through the reference's Python build_seed_vector of one lineage."""
    for k in list(sys.modules):
        if k == "cuda_fdm" or k.startswith("cuda_fdm."):
            del sys.modules[k]
    sys.path.insert(0, str(lineage_root))
    try:
        from cuda_fdm.ic import build_seed_vector
        out = []
        for r in ic_rows:
            out.append(build_seed_vector(lat_deg=r[0], lon_deg=r[1], alt_ft=r[2], vt_fps=r[3], phi_deg=r[4],
                                         theta_deg=r[5], psi_deg=r[6], alpha_deg=r[7], beta_deg=r[8],
                                         fuel_lbs=r[9], throttle=0.8))
        return np.array(out)
    finally:
        sys.path.remove(str(lineage_root))


def bins_to_cmd_np(bins):
    """Reference action_to_env in float32 (R/cuda_fdm/ppo_gpu.py:361-369), widened to float64."""
    import torch
    return ic_mod.bins_to_commands(torch.as_tensor(bins)).double().numpy()


def main():
    ics = ic_mod.baseline_ics(NENV_CFG1, SEED_CFG1)
    rng = np.random.default_rng(SEED_CFG1 + 1)
    bins = rng.integers(0, 21, size=(100, 2 * NENV_CFG1, 4), dtype=np.uint8)
    seeds = ref_seed_rows(ics, REF)
    s = seeds.copy()
    snaps = {}
    obs600 = None
    for dcs in range(100):
        cmd = bins_to_cmd_np(bins[dcs])
        if dcs == 0:
            s1, _ = ofdm.ref_step(s, cmd, 1, "root")
            snaps["state_f1"] = s1
        s, obs = ofdm.ref_step(s, cmd, 6, "root")
        if dcs == 0:
            snaps["state_f6"] = s.copy()
        obs600 = obs
    np.savez_compressed(OUT / "fdm_cfg1.npz", ic=ics, seeds=seeds, bins=bins, state_f1=snaps["state_f1"],
                        state_f6=snaps["state_f6"], state_f600=s, obs17_f600=obs600,
                        fcs_dt=np.array(1.0 / 120.0))
    print("fdm_cfg1.npz", seeds.shape)

    r36 = REF / "research" / "competition_36500" / "runtime"
    ics16 = ics[:32]
    seeds16 = ref_seed_rows(ics16, r36)
    s = seeds16.copy()
    for dcs in range(10):
        s, obs = ofdm.ref_step(s, bins_to_cmd_np(bins[dcs, :32]), 6, "r36")
    np.savez_compressed(OUT / "fdm_r36.npz", ic=ics16, seeds=seeds16, bins=bins[:10, :32], state_f60=s,
                        obs17_f60=obs, fcs_dt=np.array(1.0 / 60.0))
    print("fdm_r36.npz", seeds16.shape)


def obs_scenario_ics(nenv, seed):
    """IC rows (2*nenv, 12) for the observation/reward fixtures: a third 'engaged' pairs (target
    on the ownship's nose at 150-1300 m, inside the damage cones), a third random cfg3-like
    pairs (+-20 km, 1-12 km altitude, 150-350 m/s, any attitude), the rest near the 1000 ft hard
    deck (altitude exits).  Fuel 3000 lb (R/cuda_fdm/rl_env.py:327)."""
    rng = np.random.default_rng(seed)
    rows = np.zeros((2 * nenv, 12))
    d2r = np.pi / 180.0
    for e in range(nenv):
        kind = e * 3 // nenv
        roll, pitch, yaw = rng.uniform(-60, 60), rng.uniform(-20, 20), rng.uniform(0, 360)
        if kind == 0:
            n0, e0, alt = rng.uniform(-3000, 3000), rng.uniform(-3000, 3000), rng.uniform(2000, 8000)
            fwd = np.array([np.cos(pitch * d2r) * np.cos(yaw * d2r), np.cos(pitch * d2r) * np.sin(yaw * d2r),
                            -np.sin(pitch * d2r)])
            dist = rng.uniform(150, 1300)
            side = np.cross(fwd, [0, 0, 1.0])
            side /= np.linalg.norm(side)
            p1 = np.array([n0, e0, -alt]) + dist * fwd + side * dist * np.tan(rng.uniform(-0.8, 0.8) * d2r)
            own = (n0, e0, -alt, roll, pitch, yaw)
            tgt = (p1[0], p1[1], p1[2], rng.uniform(-60, 60), rng.uniform(-20, 20), rng.uniform(0, 360))
        elif kind == 1:
            own = (rng.uniform(-2e4, 2e4), rng.uniform(-2e4, 2e4), -rng.uniform(1000, 12000),
                   rng.uniform(-180, 180), rng.uniform(-85, 85), rng.uniform(0, 360))
            tgt = (rng.uniform(-2e4, 2e4), rng.uniform(-2e4, 2e4), -rng.uniform(1000, 12000),
                   rng.uniform(-180, 180), rng.uniform(-85, 85), rng.uniform(0, 360))
        else:
            a0 = rng.choice([200.0, 320.0, 2000.0])
            own = (rng.uniform(-1000, 1000), 0.0, -a0, roll, pitch, yaw)
            tgt = (rng.uniform(-1000, 1000), 500.0, -rng.choice([200.0, 2000.0]), 0.0, 0.0, rng.uniform(0, 360))
        for k, s in enumerate((own, tgt)):
            lat, lon, alt_ft = ic_mod.official_seed_latlon(np.array([s[0]]), np.array([s[1]]), np.array([s[2]]))
            r = rows[2 * e + k]
            r[0], r[1], r[2] = lat[0], lon[0], alt_ft[0]
            r[3] = rng.uniform(150, 350) / 0.3048
            r[4], r[5], r[6] = s[3], s[4], s[5] % 360.0
            r[7], r[8] = rng.uniform(-4, 8), rng.uniform(-3, 3)
            r[9] = 3000.0
    return rows


def make_obs_golden(nenv=24, steps=8, seed=20260103):
    """obs_traj.npz: the reference's torch observation / reward path
    (R/cuda_fdm/obs_reward.py BatchObsReward(enable_kernel=False): push_actions, advance,
    build_obs, compute_reward; termination by R/cuda_fdm/rl_env.py:481-496) over an FDM
    trajectory (R/ lineage, FCS dt 1/60) from obs_scenario_ics, with randomised reconstruction
    buffers (HP, fuel, time incl. 100/150 s cone tiers and the 200 s limit)."""
    import torch
    r36 = REF / "research" / "competition_36500" / "runtime"
    for k in list(sys.modules):
        if k == "cuda_fdm" or k.startswith("cuda_fdm.") or k in ("my_observation", "my_reward"):
            del sys.modules[k]
    sys.path.insert(0, str(r36))
    sys.path.insert(0, str(REF / "src"))
    from cuda_fdm import obs_reward as OR
    from cuda_fdm.rl_env import kinematics_state, ned_from_ecef_altasl, FT2M, R2D
    from claude_code.my_reward import MY_REWARD_CONFIG
    from dogfight.envs.termination import time_limit_reached

    rows = obs_scenario_ics(nenv, seed)
    seeds = ofdm.oracle_seed(rows, 1.0 / 60.0)
    rng = np.random.default_rng(seed + 1)
    nac = 2 * nenv
    ref = OR.BatchObsReward(nenv, device="cpu", enable_kernel=False)
    hp0 = rng.uniform(0.2, 1.0, nac)
    hp0[rng.choice(nac, 4, replace=False)] = 0.004          # a hit in the cone ends the match on HP
    fuel0 = rng.uniform(0.3, 1.0, nac)
    t0 = rng.choice([0.0, 37.3, 99.95, 120.0, 149.95, 170.0, 199.85, 199.95], nenv)
    ref.hp.copy_(torch.as_tensor(hp0))
    ref.fuel.copy_(torch.as_tensor(fuel0))
    ref.t_sec.copy_(torch.as_tensor(t0))

    def state9(st):
        ecef_m, euler, vuvw, alt_ft = kinematics_state(torch.as_tensor(st))
        n, e, d = ned_from_ecef_altasl(ecef_m, alt_ft * FT2M)
        return torch.cat([torch.stack([n, e, d], 1), euler * R2D, vuvw * FT2M], 1)

    s9 = state9(seeds)
    ref.initialize_reward_state(s9, cfg=MY_REWARD_CONFIG)
    init = {k: getattr(ref, k).clone().numpy() for k in ("prev_x", "prev_x_valid", "prev_alt_log")}
    states = seeds.copy()
    acts = np.zeros((steps, nac, 4))
    out = {k: [] for k in ("obs", "reward", "term", "trunc", "hp", "fuel", "t_sec", "pqr", "prev_att", "dealt",
                           "taken", "hp_loss", "prev_x", "prev_alt_log", "act_hist", "s9")}
    for k in range(steps):
        a = np.zeros((nac, 4))
        a[:, 0:3] = rng.uniform(-0.4, 0.4, (nac, 3))
        a[:, 3] = rng.uniform(0.5, 0.95, nac)
        acts[k] = a
        states, _ = ofdm.oracle_step(states, a, 6, 1.0 / 60.0, with_obs=False)
        s9 = state9(states)
        at = torch.as_tensor(a)
        ref.push_actions(at)
        ref.advance(s9)
        obs = ref.build_obs(s9)
        v = s9.view(nenv, 2, 9)
        alt = -v[:, :, 2]
        fin = torch.isfinite(v).all(dim=2)
        hp = ref.hp.view(nenv, 2)
        term = (alt < 304.8).any(1) | (hp <= 0.0).any(1) | (~fin).any(1)
        trunc = time_limit_reached(ref.t_sec, 200.0) & (~term)
        rew = ref.compute_reward(s9, term, cfg=MY_REWARD_CONFIG, truncated_env=trunc)
        for key, val in (("obs", obs), ("reward", rew), ("term", term), ("trunc", trunc), ("hp", ref.hp),
                         ("fuel", ref.fuel), ("t_sec", ref.t_sec), ("pqr", ref.pqr), ("prev_att", ref.prev_att),
                         ("dealt", ref.last_dmg_dealt), ("taken", ref.last_dmg_taken), ("hp_loss", ref.hp_loss),
                         ("prev_x", ref.prev_x), ("prev_alt_log", ref.prev_alt_log), ("act_hist", ref.act_hist),
                         ("s9", s9)):
            out[key].append(val.clone().numpy())
    np.savez_compressed(OUT / "obs_traj.npz", ic=rows, seeds=seeds, actions=acts, hp0=hp0, fuel0=fuel0, t0=t0,
                        init_prev_x=init["prev_x"], init_prev_x_valid=init["prev_x_valid"],
                        init_prev_alt_log=init["prev_alt_log"],
                        **{k: np.stack(v) for k, v in out.items()})
    print("obs_traj.npz", nenv, steps, "terminations per step:", np.stack(out["term"]).sum(1),
          "truncations:", np.stack(out["trunc"]).sum(1), "nonzero damage:", int((np.stack(out["dealt"]) > 0).sum()))


def make_gae_golden(T=24, n=96, seed=20260104):
    """gae.npz: the trainer's own GAE loop (R/cuda_fdm/ppo_gpu.py:1983-1995, as exercised by
    cuda_fdm/tests/ppo_gpu_val.py:62-95) run with torch fp32 on CPU, plus that test's independent
    numpy reference ``_ref_gae`` (fp64), on random rewards / values / done flags, for the
    reference default (gamma 0.997, lambda 0.95) and BASELINE cfg4's (0.99, 0.95)."""
    import importlib.util
    import torch
    spec = importlib.util.spec_from_file_location("ppo_gpu_val", REF / "cuda_fdm" / "tests" / "ppo_gpu_val.py")
    sys.path.insert(0, str(REF))
    sys.path.insert(0, str(REF / "src"))
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    g = torch.Generator().manual_seed(seed)
    out = {}
    for tag, gamma, lam in (("ref", 0.997, 0.95), ("cfg4", 0.99, 0.95)):
        rew = torch.randn(T, n, generator=g) * 3
        val = torch.randn(T, n, generator=g) * 5
        done = (torch.rand(T, n, generator=g) < 0.1).float()
        last_val = torch.randn(n, generator=g) * 5
        next_done = (torch.rand(n, generator=g) < 0.1).float()
        adv = torch.zeros_like(rew)
        lastgae = torch.zeros(n)
        for t in reversed(range(T)):
            if t == T - 1:
                next_nonterminal = 1.0 - next_done
                next_values = last_val
            else:
                next_nonterminal = 1.0 - done[t + 1]
                next_values = val[t + 1]
            delta = rew[t] + gamma * next_values * next_nonterminal - val[t]
            lastgae = delta + gamma * lam * next_nonterminal * lastgae
            adv[t] = lastgae
        ret = adv + val
        ref64 = m._ref_gae(rew.numpy().astype(np.float64), val.numpy().astype(np.float64),
                           done.numpy().astype(np.float64), last_val.numpy().astype(np.float64),
                           next_done.numpy().astype(np.float64), gamma, lam)
        for k, v in (("rew", rew), ("val", val), ("done", done), ("last_val", last_val), ("next_done", next_done),
                     ("adv", adv), ("ret", ret)):
            out[f"{tag}_{k}"] = v.numpy()
        out[f"{tag}_ref64"] = ref64
        out[f"{tag}_gamma_lam"] = np.array([gamma, lam])
    np.savez_compressed(OUT / "gae.npz", **out)
    print("gae.npz", T, n)


def make_norm_golden(seed=20260105):
    """norm.npz: the reference's RunningNorm (R/cuda_fdm/ppo_gpu.py:184-222) on CPU: three
    batch updates of 184-feature observation-like rows, then normalize of a fourth batch."""
    import torch
    r36 = REF / "research" / "competition_36500" / "runtime"
    for k in list(sys.modules):
        if k == "cuda_fdm" or k.startswith("cuda_fdm."):
            del sys.modules[k]
    sys.path.insert(0, str(r36))
    sys.path.insert(0, str(REF / "src"))
    from cuda_fdm.ppo_gpu import RunningNorm
    rn = RunningNorm(184, "cpu")
    out = {"seed": np.array(seed)}
    xs = norm_inputs(seed)
    for i, x in enumerate(xs[:-1]):
        rn.update(x)
        out[f"mean{i}"] = rn.mean.numpy().copy()
        out[f"var{i}"] = rn.var.numpy().copy()
        out[f"count{i}"] = rn.count.numpy().copy()
    out["yt"] = rn.normalize(xs[-1].clone()).numpy()
    np.savez_compressed(OUT / "norm.npz", **out)
    print("norm.npz")


def norm_inputs(seed):
    """Deterministic inputs of norm.npz (regenerated by the tests from the stored seed)."""
    import torch
    g = torch.Generator().manual_seed(int(seed))
    xs = [torch.randn(B, 184, generator=g) * torch.linspace(0.1, 3.0, 184) + torch.linspace(-2, 2, 184)
          for B in (512, 1000, 37)]
    xs.append(torch.randn(24, 184, generator=g) * 40.0)
    return xs


def make_ppo_golden(seed=20260106):
    """ppo_update.npz: the reference's own PPOGPUTrainer.update (R/cuda_fdm/ppo_gpu.py:2020-2144,
    MLP path, aux_pred off) run on CPU over a seeded 4 x 48 rollout of a (32, 32) tanh
    MLPActorCritic; stores the parameters after the update and the returned statistics."""
    import types
    import torch
    r36 = REF / "research" / "competition_36500" / "runtime"
    for k in list(sys.modules):
        if k == "cuda_fdm" or k.startswith("cuda_fdm.") or k == "claude_code" or k.startswith("claude_code."):
            del sys.modules[k]
    sys.path.insert(0, str(r36))
    import cuda_fdm.ppo_gpu as P
    from ppo_case import PPO_CFG, PPO_HIDDEN, ppo_inputs
    torch.manual_seed(seed)
    model = P.MLPActorCritic(184, 4, 21, hidden=PPO_HIDDEN, activation="tanh")
    init = torch.cat([p.detach().reshape(-1) for p in model.parameters()]).double()
    obs, act, old_logp, b_val, adv, ret = ppo_inputs(model, seed)
    cfg = P.PPOGPUConfig(device="cpu", aux_pred=False, hidden=PPO_HIDDEN, activation="tanh", **PPO_CFG)
    fake = types.SimpleNamespace(cfg=cfg, model=model, b_obs=obs, b_act=act, b_logp=old_logp, b_val=b_val,
                                 actor_opt=torch.optim.Adam(model.actor_parameters(), lr=cfg.lr, eps=1e-5),
                                 critic_opt=torch.optim.Adam(model.critic_parameters(), lr=cfg.lr, eps=1e-5))
    torch.manual_seed(seed + 1)
    res = P.PPOGPUTrainer.update(fake, adv, ret)
    out = {"seed": np.array(seed), "init_sum": np.array([float(init.sum()), float(init.abs().sum())]),
           "params": torch.cat([p.detach().reshape(-1) for p in model.parameters()]).numpy()}
    for k in ("pl", "vl", "ent", "kl", "cf", "ev", "actor_grad_norm", "critic_grad_norm"):
        out[k] = np.array(float(res[k]))
    out["epochs"] = np.array(res["epochs"]); out["early"] = np.array(bool(res["early"]))
    out["optimizer_steps"] = np.array(res["optimizer_steps"])
    np.savez_compressed(OUT / "ppo_update.npz", **out)
    print("ppo_update.npz", res["epochs"], res["early"], res["optimizer_steps"])


def make_payoff_golden(seed=20260107, per_order=4, capacity=3, nright=3, nsteps=14):
    """payoff.npz: the reference's own batched payoff loop (R/cuda_fdm/batched_payoff.py
    evaluate_chunk, scoring :131-156, summaries via PPOGPUTrainer._summarize_clean_pair,
    ppo_gpu.py:1517-1575) run on CPU with a scripted environment whose step returns the
    payoff_case.payoff_steps() terminal values; stores each matchup's scores, crash flags,
    completion step and summary (without the bootstrap interval, which is league statistics)."""
    import json
    import types
    import torch
    from payoff_case import payoff_steps
    r36 = REF / "research" / "competition_36500" / "runtime"
    for k in list(sys.modules):
        if k == "cuda_fdm" or k.startswith("cuda_fdm.") or k == "claude_code" or k.startswith("claude_code."):
            del sys.modules[k]
    sys.path.insert(0, str(r36))
    sys.path.insert(0, str(REF / "src"))
    import cuda_fdm.batched_payoff as BP
    import cuda_fdm.ppo_gpu as P
    lanes = 2 * per_order
    nenv = lanes * capacity
    script = payoff_steps(seed, nenv, nsteps)

    class Obr:
        dt = 0.1

        def reset_all(self):
            pass

        def kernel_init_reward_state(self, states, env_mask=None):
            pass

        def kernel_build_obs(self, states, env_mask=None):
            return torch.zeros(2 * nenv, 184)

    class Env:
        OBS_SIZE = 184
        max_engage_time_s = (nsteps - 4) * 0.1
        min_altitude_m = 304.8
        ic_pool_size = 16

        def __init__(self):
            self.nenv = nenv
            self.obr = Obr()
            self.sim = types.SimpleNamespace(states=torch.zeros(2 * nenv, 101), load_seed=lambda t: None)
            self.k = 0

        def step(self, controls, reset_indices=None):
            d = script[self.k]
            self.k += 1
            info = {"terminal_hp": torch.as_tensor(d["hp"]), "terminal_alt_m": torch.as_tensor(d["alt"]),
                    "terminal_state_finite": torch.as_tensor(d["finite"])}
            return (torch.zeros(nenv, 2, 184), torch.as_tensor(d["reward"]), torch.as_tensor(d["done"]), info)

    class Template:
        ic_pool, ic_pool_size = torch.zeros(16, 2, 101), 16
        _evaluation_seed_bank = torch.zeros(lanes * 2, 101)

        def reset_evaluation(self, paired=True, seed_block=0):
            pass

        def _ensure_ic_pool(self):
            pass

    class Net:
        num_bins = 21

        def actor_logits(self, x):
            return torch.zeros(x.shape[0], 84)

    recorded = []
    trainer = types.SimpleNamespace(cfg=types.SimpleNamespace(seed=5, device="cpu", num_bins=21),
                                    grid=P.make_action_grid(21, "cpu"), _batch_captured_actions=False,
                                    _outcome_summary=P.PPOGPUTrainer._outcome_summary)
    trainer._league_eval_env = lambda blocks: (Template(), per_order)
    trainer._batched_payoff_env = ((capacity, per_order), Env())

    def summarize(*a):
        recorded.append([np.asarray(x.detach().cpu().numpy()) if torch.is_tensor(x) else x for x in a])
        return P.PPOGPUTrainer._summarize_clean_pair(trainer, *a)
    trainer._summarize_clean_pair = summarize
    pol = (Net(), None, None)
    res = BP.evaluate_chunk(trainer, pol, [pol] * nright, lanes, 0, capacity)
    out = {"seed": np.array(seed), "per_order": np.array(per_order), "capacity": np.array(capacity),
           "nright": np.array(nright), "nsteps": np.array(nsteps), "min_alt": np.array(Env.min_altitude_m)}
    for i, (r, rec) in enumerate(zip(res, recorded)):
        scores, own, opp, po, sb, es, st = rec
        out[f"scores{i}"] = scores.astype(np.float32)
        out[f"own{i}"] = own.astype(np.uint8)
        out[f"opp{i}"] = opp.astype(np.uint8)
        out[f"final_step{i}"] = np.array(st)
        r = {k: v for k, v in r.items() if k not in ("lcb95", "ucb95")}
        out[f"summary{i}"] = np.array(json.dumps(r, sort_keys=True))
    np.savez_compressed(OUT / "payoff.npz", **out)
    print("payoff.npz", [int(out[f"final_step{i}"]) for i in range(nright)])


if __name__ == "__main__":
    main()
    make_obs_golden()
    make_gae_golden()
    make_norm_golden()
    make_ppo_golden()
    make_payoff_golden()
