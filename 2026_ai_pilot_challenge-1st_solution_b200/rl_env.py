"""``GpuDogfightVecEnv``: drop-in for the reference's vectorised 1-v-1 environment
(R/cuda_fdm/rl_env.py:177-570) on the sm_100a kernels.

Same constructor, ``reset`` / ``reset_evaluation`` / ``step`` / ``state9_flat`` / ``state9``
contract and return values.  Differences in *how*, not *what*:

* IC pairs are drawn vectorised (same distributions as ``_sample_ic_pair``, :224-252) and
  seeded on the GPU (f16_seed_ic) instead of a per-aircraft CPU ``build_seed_vector``;
* ``step`` runs the FDM kernel (no obs17; it also flags non-finite aircraft, replacing a
  torch.isfinite pass over the whole state) and then ONE fused kernel
  (f16_env_post_step) for advance + terminal observation + autoreset, instead of ~10 torch
  launches and a full clone; like the reference it never synchronises the host.
"""
import ctypes as C
import math

import numpy as np
import torch

from . import _lib
from .gpu_env import GpuDogfight, STATE_N, FCS_DT_R36
from .ic import official_seed_latlon, seed_states
from .obs_reward import BatchObsReward, OBS_SIZE, REWARD_CONFIG, validate_reward_mode

ORIGIN_LAT_DEG = 37.240778
ORIGIN_LON_DEG = 131.869556
FT2M = 0.3048
M2FT = 1.0 / FT2M
HARD_DECK_FT = 1000.0
HARD_DECK_M = HARD_DECK_FT * FT2M
S9 = dict(N=0, E=1, D=2, roll=3, pitch=4, yaw=5, u=6, v=7, w=8)
SEA_LEVEL_RADIUS_FT = 20925646.32546


class GpuDogfightVecEnv:
    """nenv engagements of 2 aircraft (ownship = 2e, opponent = 2e+1)."""

    OBS_SIZE = OBS_SIZE

    def __init__(self, nenv, substeps=6, precision="fp64", block=128, seed=None, device="cuda",
                 min_altitude_m=HARD_DECK_M, max_engage_time_s=200.0, reward_cfg=None, reward_mode=0,
                 alt_hunt_coef=5.0, fcs_dt=FCS_DT_R36):
        if precision != "fp64":
            raise ValueError("GpuDogfightVecEnv supports precision='fp64' only: fused observation/reward "
                             "kernels require float64 state and action buffers.")
        self.sim = GpuDogfight(nenv, substeps=substeps, planes_per_env=2, precision=precision, block=block,
                               fcs_dt=fcs_dt, device=device)
        self.device = self.sim.device
        self.lib = _lib.load()
        self.nenv = int(nenv)
        self.nac = self.sim.nac
        self.substeps = int(substeps)
        self.seed = 0 if seed is None else int(seed)
        self.rng = np.random.default_rng(seed)
        # official IC distribution (rl_env.py:199-207)
        self.center_n = 3500.0
        self.center_e = 0.0
        self.alt_ft_range = (2000.0, 30000.0)
        self.speed_mps_range = (200.0, 300.0)
        self.distA_ft_choices = (2000.0, 2500.0, 3000.0)
        self.dist_headon_ft = 5539.0 / FT2M
        self.scenario_b_prob = 0.0
        self.min_altitude_m = min_altitude_m
        self.max_engage_time_s = max_engage_time_s
        self.reward_cfg = dict(REWARD_CONFIG if reward_cfg is None else reward_cfg)
        self.reward_mode = validate_reward_mode(reward_mode, alt_hunt_coef)
        self.alt_hunt_coef = float(alt_hunt_coef)
        self.obr = BatchObsReward(nenv, device=self.device)
        self.ic_pool = None
        self.ic_pool_size = 4096
        self._evaluation_seed_bank = None
        self._evaluation_seed_bank_key = None
        self._evaluation_seed_metadata = None
        dev = self.device
        self._reward = torch.zeros(self.nac, dtype=torch.float64, device=dev)
        self._done = torch.zeros(self.nenv, dtype=torch.uint8, device=dev)
        self._terminal_obs = torch.zeros(self.nac, OBS_SIZE, dtype=torch.float32, device=dev)
        self._terminal_hp = torch.zeros(self.nac, dtype=torch.float64, device=dev)
        self._terminal_alt = torch.zeros(self.nac, dtype=torch.float64, device=dev)
        self._actions = torch.zeros(self.nac, 4, dtype=torch.float64, device=dev)
        self._s9 = torch.zeros(self.nac, 9, dtype=torch.float64, device=dev)
        self._finite = torch.ones(self.nac, dtype=torch.uint8, device=dev)
        self.terminal_obs_enabled = True
        # warm-up command range per channel (lower end, width), kept on the device
        self._warm_lo = torch.tensor([-0.2, -0.2, -0.2, 0.6], dtype=torch.float64, device=dev)
        self._warm_span = torch.tensor([0.4, 0.4, 0.4, 0.3], dtype=torch.float64, device=dev)

    # ---- IC sampling (rl_env.py:224-252), vectorised ----
    def _sample_ic_rows(self, n, rng=None, alt_ft=None, speed=None, side_swap=None, head_swap=None, dist_ft=None):
        """(2n, 12) IC rows for n engagements drawn from the official distribution."""
        rng = self.rng if rng is None else rng
        alt_ft = rng.uniform(*self.alt_ft_range, n) if alt_ft is None else np.broadcast_to(alt_ft, (n,))
        speed = rng.uniform(*self.speed_mps_range, n) if speed is None else np.broadcast_to(speed, (n,))
        side = (rng.integers(0, 2, n) if side_swap is None else np.broadcast_to(side_swap, (n,))).astype(bool)
        scen_b = rng.random(n) < self.scenario_b_prob
        head = (rng.integers(0, 2, n) if head_swap is None else np.broadcast_to(head_swap, (n,))).astype(bool)
        dist = (rng.choice(np.asarray(self.distA_ft_choices), n) if dist_ft is None
                else np.broadcast_to(dist_ft, (n,)))
        half = np.where(scen_b, 0.5 * self.dist_headon_ft * FT2M, 0.5 * dist * FT2M)
        own_n = self.center_n + np.where(side, -half, half)
        tgt_n = self.center_n + np.where(side, half, -half)
        own_h = np.where(scen_b, np.where(side, 0.0, 180.0), np.where(head, 270.0, 90.0))
        tgt_h = np.where(scen_b, np.where(side, 180.0, 0.0), np.where(head, 90.0, 270.0))
        d = -alt_ft * FT2M
        rows = np.zeros((2 * n, _lib.IC_N))
        for k, (nn, hh) in enumerate(((own_n, own_h), (tgt_n, tgt_h))):
            lat, lon, altf = official_seed_latlon(nn, np.full(n, self.center_e), d)
            r = rows[k::2]
            r[:, 0], r[:, 1], r[:, 2] = lat, lon, altf
            r[:, 3] = speed * M2FT
            r[:, 6] = hh
            r[:, 9] = 3000.0            # fuel (rl_env.py:327)
        return rows

    def _initialize_physical_seeds(self, ic_rows):
        """GPU-seed the rows, then exactly one neutral 60 Hz tick (rl_env.py:329-341)."""
        st = seed_states(ic_rows, self.sim.fcs_dt, device=self.device)          # (101, n) SoA
        n = st.shape[1]
        cmd = torch.zeros(n, 4, dtype=torch.float64, device=self.device)
        cmd[:, 3] = 1.0
        _lib.check(self.lib.f16_fdm_step(_lib.ptr(st), _lib.LAYOUT_SOA, n, n, _lib.ptr(cmd), 1, self.sim.fcs_dt,
                                         None, _lib.stream_of(st)), "f16_fdm_step")
        return st.t()                                                            # (n, 101) view

    def _build_all_seeds(self):
        return self._initialize_physical_seeds(self._sample_ic_rows(self.nenv))

    def _ensure_ic_pool(self):
        """(pool, 2, 101) autoreset pool, built once on the GPU (rl_env.py:353-365)."""
        if self.ic_pool is not None:
            return
        rows = self._initialize_physical_seeds(self._sample_ic_rows(self.ic_pool_size))
        self.ic_pool = rows.contiguous().view(self.ic_pool_size, 2, STATE_N)

    def _build_evaluation_seed_bank(self, *, paired=False, seed_block=0):
        """Deterministic stratified clean ICs (rl_env.py:254-305)."""
        paired = bool(paired)
        if paired and self.nenv % 8:
            raise ValueError("mirrored 3:1 evaluation requires nenv divisible by 8")
        base = self.nenv // 2 if paired else self.nenv
        rng = np.random.default_rng((self.seed + 19_870_331 + int(seed_block) * 1_000_003) % (2 ** 63 - 1))
        alt_order = rng.permutation(base)
        spd_order = rng.permutation(base)
        idx = np.arange(base)
        alt = self.alt_ft_range[0] + (alt_order + 0.5) / base * (self.alt_ft_range[1] - self.alt_ft_range[0])
        spd = self.speed_mps_range[0] + (spd_order + 0.5) / base * (self.speed_mps_range[1] - self.speed_mps_range[0])
        dist = np.asarray(self.distA_ft_choices)[idx % len(self.distA_ft_choices)]
        rows = self._sample_ic_rows(base, rng=np.random.default_rng(0), alt_ft=alt, speed=spd,
                                    side_swap=(idx % 2) == 1, head_swap=((idx // 2) % 2) == 1, dist_ft=dist)
        counts = {str(int(d)): int((dist == d).sum()) for d in self.distA_ft_choices}
        if paired:
            rows = np.concatenate([rows, rows], 0)
        self._evaluation_seed_metadata = {"paired": paired, "seed_block": int(seed_block), "base_count": int(base),
                                          "three_nine": int(base), "headon": 0,
                                          "three_nine_distance_counts": counts}
        return self._initialize_physical_seeds(rows).contiguous()

    def reset_evaluation(self, *, paired=False, seed_block=0):
        key = (bool(paired), int(seed_block))
        if self._evaluation_seed_bank is None or self._evaluation_seed_bank_key != key:
            self._evaluation_seed_bank = self._build_evaluation_seed_bank(paired=paired, seed_block=seed_block)
            self._evaluation_seed_bank_key = key
        self.sim.load_seed(self._evaluation_seed_bank)
        self.obr.reset_all()
        self.obr.kernel_init_reward_state(self.sim.states)
        return self.obr.kernel_build_obs(self.sim.states).view(self.nenv, 2, self.OBS_SIZE)

    # ---- reset (rl_env.py:368-441) ----
    def reset(self, stagger=True, max_stagger_steps=256, warmup_action_fn=None):
        """Fresh ICs for every env; with ``stagger`` each env is then advanced a random number of
        valid steps in [0, max_stagger_steps) (the reference's staggered start, rl_env.py:386-441),
        entirely on the device: departed envs are re-seeded from the IC pool and the host is
        never synchronised inside the warm-up."""
        seeds = self._build_all_seeds()
        if not bool(torch.isfinite(seeds).all()):
            raise FloatingPointError("non-finite initial physical states")
        self.sim.states.copy_(seeds)
        self.obr.reset_all()
        self.obr.kernel_init_reward_state(self.sim.states)
        if stagger and max_stagger_steps > 0:
            self._staggered_warmup_device(max_stagger_steps, warmup_action_fn)
        return self.obr.kernel_build_obs(self.sim.states).view(self.nenv, 2, self.OBS_SIZE)

    def _staggered_warmup_device(self, max_steps, action_fn, check_every=0):
        """The staggered warm-up with every decision on the device: per env a target phase in
        [0, max_steps); each step the physics kernel, the advance kernel and the departure test
        run for all envs; departed, not yet captured envs are re-seeded from the IC pool (the
        autoreset pool, same IC distribution) and restart their count; envs reaching their target
        are captured with masked copies (torch.where, no boolean indexing).  The only host reads
        are the final finiteness check and, when ``check_every`` > 0, an all-captured test every
        that many steps for an early exit."""
        self._ensure_ic_pool()
        targ = torch.as_tensor(self.rng.integers(0, max_steps, size=self.nenv), device=self.device)
        captured, obr_buf, warm_finite = self._warmup_loop_device(max_steps, action_fn, targ, check_every)
        if not bool(warm_finite):
            raise FloatingPointError("non-finite physical trajectory during staggered initialization")
        self.sim.states.copy_(captured)
        self.obr.restore(obr_buf)
        self.obr.kernel_init_reward_state(self.sim.states)

    def _warmup_loop_device(self, max_steps, action_fn, targ, check_every=0, pool_picks=None):
        """Loop of _staggered_warmup_device; returns (captured states, captured reconstruction
        buffers, finite flag), all on the device.  ``pool_picks`` optionally fixes the IC-pool row
        each env would be re-seeded from: a (max_steps + 1, nenv) int64 device tensor, row i used
        at step i and the last row for the envs never captured (default: uniform draws on the
        device)."""
        dev = self.device
        age = torch.zeros(self.nenv, dtype=torch.long, device=dev)
        captured_mask = targ == 0
        captured = self.sim.states.clone()
        obr_buf = self.obr.clone_state()
        warm_finite = torch.ones((), dtype=torch.bool, device=dev)
        st3 = self.sim.states.view(self.nenv, 2, STATE_N)

        def reseed(mask, i):
            pick = (pool_picks[i] if pool_picks is not None
                    else torch.randint(0, self.ic_pool_size, (self.nenv,), device=dev))
            st3.copy_(torch.where(mask.view(-1, 1, 1), self.ic_pool[pick], st3))
            self.obr.reset_envs(mask)
            self.obr.kernel_init_reward_state(self.sim.states, mask)

        for i in range(max_steps):
            if action_fn is None:
                a = self._random_actions()
            else:
                a = action_fn(self.obr.kernel_build_obs(self.sim.states)).to(torch.float64).reshape(self.nac, 4)
            self.sim.step(a, substeps=self.substeps)
            fin = torch.isfinite(st3).all(dim=2).all(dim=1)
            warm_finite.logical_and_((fin | captured_mask).all())
            self.obr.kernel_advance(self.sim.states, a.contiguous(), cfg=self.reward_cfg,
                                    min_alt=self.min_altitude_m, max_time=self.max_engage_time_s)
            dep = self._departed_envs(self.state9_flat()) & (~captured_mask)
            reseed(dep, i)
            age = torch.where(dep, torch.zeros_like(age), age) + (~captured_mask).long()
            hit = (~captured_mask) & (age == targ)
            captured.copy_(torch.where(hit.repeat_interleave(2).view(-1, 1), self.sim.states, captured))
            self.obr.capture_where(obr_buf, hit)
            captured_mask = captured_mask | hit
            if check_every > 0 and (i + 1) % check_every == 0 and bool(captured_mask.all()):
                break
        rest = ~captured_mask                                   # still short of their phase
        reseed(rest, max_steps)
        captured.copy_(torch.where(rest.repeat_interleave(2).view(-1, 1), self.sim.states, captured))
        self.obr.capture_where(obr_buf, rest)
        return captured, obr_buf, warm_finite

    def _departed_envs(self, s9_flat=None, floor_m=100.0):
        """Per env: True when either aircraft is below ``floor_m`` of MSL altitude or has a
        non-finite 9-DoF state (the warm-up's departure test)."""
        s9 = self.state9() if s9_flat is None else s9_flat.view(self.nenv, 2, 9)
        ok = torch.isfinite(s9).all(dim=2) & (s9[:, :, S9["D"]] <= -floor_m)
        return ~ok.all(dim=1)

    def _random_actions(self):
        """Warm-up commands (rl_env.py:468-473): the three sticks uniform in [-0.2, 0.2], throttle
        uniform in [0.6, 0.9], one row per aircraft."""
        a = torch.rand(self.nac, 4, dtype=torch.float64, device=self.device)
        return a.mul_(self._warm_span).add_(self._warm_lo)

    def _to_nac4(self, actions):
        a = torch.as_tensor(actions, dtype=torch.float64, device=self.device)
        return a.reshape(self.nac, 4)

    def _termination(self, s9_flat):
        """(terminated, truncated) per env from a 9-DoF state (rl_env.py:481-496)."""
        s9 = s9_flat.view(self.nenv, 2, 9)
        alt = -s9[:, :, S9["D"]]
        finite = torch.isfinite(s9).all(dim=2)
        hp = self.obr.hp.view(self.nenv, 2)
        term = (alt < self.min_altitude_m).any(dim=1) | (hp <= 0.0).any(dim=1) | (~finite).any(dim=1)
        trunc = (self.obr.t_sec >= self.max_engage_time_s - 1.0e-8) & (~term)
        return term, trunc

    # ---- step (rl_env.py:499-555) ----
    @property
    def action_buffer(self):
        """The (nac, 4) fp64 command buffer ``step`` reads; a policy may write commands into it
        directly (f16_policy_forward's cmd output) and pass it back to ``step`` uncopied."""
        return self._actions

    def step(self, actions, *, reset_indices=None):
        if actions is not self._actions:
            self._actions.copy_(self._to_nac4(actions))
        if self.ic_pool is None:
            self._ensure_ic_pool()
        sim = self.sim
        sh = _lib.stream_of(sim.states_soa)
        # physics; the same launch flags aircraft whose 101 state values are all finite
        io = _lib.FdmIO(cmd=self._actions.data_ptr(), finite=self._finite.data_ptr())
        _lib.check(self.lib.f16_fdm_step_ex(_lib.ptr(sim.states_soa), _lib.LAYOUT_SOA, self.nac, self.nac,
                                            C.byref(io), self.substeps, sim.fcs_dt, sh), "f16_fdm_step_ex")
        terminal_state_finite = self._finite.view(torch.bool).view(self.nenv, 2).all(dim=1)
        if reset_indices is None:
            pick = torch.randint(0, self.ic_pool_size, (self.nenv,), device=self.device)
        else:
            if (reset_indices.shape != (self.nenv,) or reset_indices.dtype != torch.long
                    or reset_indices.device != self.device):
                raise ValueError("reset indices must be one device int64 index per environment")
            pick = reset_indices
        obr = self.obr
        rc = obr._reward_cfg(self.reward_cfg, self.min_altitude_m, self.max_engage_time_s, self.reward_mode,
                             self.alt_hunt_coef)
        aux = obr.aux_features.data_ptr() if obr.aux_features is not None else None
        term_obs = self._terminal_obs.data_ptr() if self.terminal_obs_enabled else None
        obr._external_advance(_lib.ptr(sim.states_soa), _lib.LAYOUT_SOA, self.nac)
        _lib.check(self.lib.f16_env_post_step(
            _lib.ptr(sim.states_soa), _lib.LAYOUT_SOA, self.nac, self.nenv, _lib.ptr(self._actions), obr._recon(), rc,
            obr._origin, _lib.ptr(self.ic_pool), self.ic_pool_size, _lib.ptr(pick), _lib.ptr(obr.reward_buf),
            _lib.ptr(obr.term_buf), _lib.ptr(obr.trunc_buf), _lib.ptr(self._done), _lib.ptr(obr.obs_buf), term_obs,
            _lib.ptr(self._terminal_hp), _lib.ptr(self._terminal_alt), aux, sh), "f16_env_post_step")
        term = obr.term_buf.bool()
        trunc = obr.trunc_buf.bool()
        done = self._done.bool()
        if hasattr(obr, "external_accel"):                  # autoreset clears the external state too
            d1 = done.repeat_interleave(2).unsqueeze(1)
            obr.external_accel.masked_fill_(d1, 0.0)
            obr.external_previous_velocity.masked_fill_(d1, 0.0)
        reward = obr.reward_buf.view(self.nenv, 2).clone()
        obs = obr.obs_buf.view(self.nenv, 2, self.OBS_SIZE)
        info = {"terminated": term, "truncated": trunc,
                "terminal_obs": self._terminal_obs.view(self.nenv, 2, self.OBS_SIZE).clone()
                if self.terminal_obs_enabled else None,
                "terminal_hp": self._terminal_hp.view(self.nenv, 2).clone(),
                "terminal_alt_m": self._terminal_alt.view(self.nenv, 2).clone(), "done": done,
                "terminal_state_finite": terminal_state_finite}
        return obs, reward, done, info

    # ---- state export ----
    def state9_flat(self):
        """Official 9-DoF (nac, 9): N/E/D m, roll/pitch/yaw deg, body u/v/w m/s."""
        _lib.check(self.lib.f16_state9(_lib.ptr(self.sim.states_soa), _lib.LAYOUT_SOA, self.nac, self.nac,
                                       self.obr._origin, _lib.ptr(self._s9), _lib.stream_of(self._s9)), "f16_state9")
        return self._s9.clone()

    def state9(self):
        return self.state9_flat().view(self.nenv, 2, 9)
