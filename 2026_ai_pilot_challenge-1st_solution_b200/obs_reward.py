"""``BatchObsReward``: drop-in for the reference's batched 184-D observation / reward state
(R/cuda_fdm/obs_reward.py:319-560), backed by the sm_100a kernels of obs_kernels.cu.

Same buffers (names, shapes, dtypes, per-aircraft layout), same kernel methods
(``kernel_advance``, ``kernel_init_reward_state``, ``kernel_build_obs``) and the same state
bookkeeping (``reset_all``, ``reset_envs``, ``clone_state``, ``capture_into``, ``restore``,
``push_actions``, ``enable_aux_capture``).  The FDM state argument may be the reference's
contiguous (nac,101) tensor or GpuDogfight's (nac,101) view of its (101,nac) SoA storage; the
latter is read in place with coalesced loads.  ``kernel_step`` fuses advance and build_obs.
"""
import math

import torch

from . import _lib

OBS_SIZE = 184           # 50 scalars + 38x3 frame-projected vectors + 5x4 action history
ACT_LEN = 5
ACT_DIM = 4
DT_PER_STEP = 6 / 60     # STEP_RATIO / SIM_HZ (R/claude_code/my_observation.py:105)
AUX_FEATURE_DIM = 21     # R/cuda_fdm/future_aux.py

STANDARD_REWARD, ALTITUDE_HUNT_REWARD, ATTACK_REWARD, DEFENSE_REWARD = 0, 1, 2, 3

# Reward constants the fused kernel reads (R/claude_code/my_reward.py:45-104, MY_REWARD_CONFIG).
REWARD_CONFIG = {
    "win_reward": 5.0, "loss_reward": -5.0,
    "timeout_win_reward": 5.0, "timeout_loss_reward": -5.0, "timeout_draw_reward": -4.0,
    "damage_scale": 10.0, "own_damage_weight": 1.0,
    "geometry_episode_budget": 5.0, "geometry_reference_duration_sec": 200.0,
    "shaping_reward_scale": 0.0001,
}

ORIGIN_LAT_DEG = 37.240778
ORIGIN_LON_DEG = 131.869556


def validate_reward_mode(mode, coefficient=5.0):
    """Reference contract (R/cuda_fdm/reward_modes.py validate_reward_mode)."""
    if mode not in (STANDARD_REWARD, ALTITUDE_HUNT_REWARD, ATTACK_REWARD, DEFENSE_REWARD):
        raise ValueError(f"unknown reward mode: {mode!r}")
    if not math.isfinite(coefficient) or coefficient < 0:
        raise ValueError("altitude-hunt coefficient must be finite and nonnegative")
    return int(mode)


def official_origin():
    """ECEF (m) of the official BaseLat/BaseLon and its sin/cos (obs_reward.py:376-383)."""
    olat, olon = math.radians(ORIGIN_LAT_DEG), math.radians(ORIGIN_LON_DEG)
    slat, clat, slon, clon = math.sin(olat), math.cos(olat), math.sin(olon), math.cos(olon)
    A, E2 = 6378137.0, 0.0066943799901411
    Nr = A / math.sqrt(1.0 - E2 * slat * slat)
    return _lib.Origin(Nr * clat * clon, Nr * clat * slon, Nr * (1.0 - E2) * slat, slat, clat, slon, clon)


class BatchObsReward:
    """Observation / reward state of nac = 2*nenv aircraft; partner(a) = a ^ 1."""

    _AC_KEYS = ("hp", "fuel", "prev_att", "prev_valid", "pqr", "last_dmg_dealt", "last_dmg_taken", "hp_loss",
                "act_hist", "prev_x", "prev_x_valid", "prev_alt_log")
    _ENV_KEYS = ("t_sec",)

    def __init__(self, nenv, device="cuda", dtype=torch.float64, enable_kernel=True):
        if dtype != torch.float64:
            raise ValueError("the fused observation / reward kernels work on float64 state")
        self.nenv = int(nenv)
        self.nac = 2 * self.nenv
        self.device = torch.device(device)
        if self.device.type == "cuda" and self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.dtype = dtype
        self.dt = DT_PER_STEP
        idx = torch.arange(self.nac, device=self.device)
        self.partner = idx ^ 1
        self.env_of = idx // 2
        self._alloc()
        self.reset_all()
        self.kernel_ready = False
        if enable_kernel:
            self._init_kernels()

    def _alloc(self):
        n, ne, dev, dt = self.nac, self.nenv, self.device, self.dtype
        self.hp = torch.ones(n, device=dev, dtype=dt)
        self.fuel = torch.ones(n, device=dev, dtype=dt)
        self.t_sec = torch.zeros(ne, device=dev, dtype=dt)
        self.prev_att = torch.zeros(n, 3, device=dev, dtype=dt)
        self.prev_valid = torch.zeros(n, device=dev, dtype=torch.bool)
        self.pqr = torch.zeros(n, 3, device=dev, dtype=dt)
        self.last_dmg_dealt = torch.zeros(n, device=dev, dtype=dt)
        self.last_dmg_taken = torch.zeros(n, device=dev, dtype=dt)
        self.hp_loss = torch.zeros(n, device=dev, dtype=dt)
        self.act_hist = torch.zeros(n, ACT_LEN, ACT_DIM, device=dev, dtype=dt)
        self.prev_x = torch.zeros(n, device=dev, dtype=dt)
        self.prev_x_valid = torch.zeros(n, device=dev, dtype=torch.bool)
        self.prev_alt_log = torch.zeros(n, device=dev, dtype=dt)
        self.aux_features = None

    def enable_aux_capture(self):
        if self.aux_features is None:
            self.aux_features = torch.zeros(self.nenv, AUX_FEATURE_DIM, dtype=torch.float64, device=self.device)

    # ---- kernels ----
    def _init_kernels(self):
        if self.device.type != "cuda":
            raise RuntimeError("the observation / reward kernels need a CUDA device")
        self.lib = _lib.load()
        self.obs_buf = torch.zeros(self.nac, OBS_SIZE, dtype=torch.float32, device=self.device)
        self.reward_buf = torch.zeros(self.nac, dtype=torch.float64, device=self.device)
        self.term_buf = torch.zeros(self.nenv, dtype=torch.uint8, device=self.device)
        self.trunc_buf = torch.zeros(self.nenv, dtype=torch.uint8, device=self.device)
        self._origin = official_origin()
        self.kernel_ready = True

    def _recon(self):
        # rebuilt per call: reset/restore may have replaced a buffer object
        p = lambda t: t.data_ptr()
        return _lib.Recon(p(self.hp), p(self.fuel), p(self.t_sec), p(self.prev_att), p(self.prev_valid), p(self.pqr),
                          p(self.last_dmg_dealt), p(self.last_dmg_taken), p(self.hp_loss), p(self.act_hist),
                          p(self.prev_x), p(self.prev_x_valid), p(self.prev_alt_log))

    def _require_ready(self):
        if not self.kernel_ready:
            raise ValueError("FP64 CUDA observation/reward kernels are not initialized")

    def _kernel_states(self, states):
        """(ptr, layout, ld, keepalive) of a (nac,101) float64 FDM state tensor on this device."""
        self._require_ready()
        _lib.require_cuda_tensor(states, torch.float64, (self.nac, _lib.STATE_N), "FDM states", self.device)
        if states.stride() == (1, states.shape[0]) or (states.stride(0) == 1 and states.stride(1) >= self.nac):
            return states.data_ptr(), _lib.LAYOUT_SOA, states.stride(1), states
        st = states.contiguous()
        return st.data_ptr(), _lib.LAYOUT_AOS, _lib.STATE_N, st

    def _kernel_mask(self, mask):
        if mask is None:
            return None, None
        _lib.require_cuda_tensor(mask, (torch.bool, torch.uint8), (self.nenv,), "environment mask", self.device)
        m = mask.contiguous()
        return m.data_ptr(), m

    def _reward_cfg(self, cfg, min_alt, max_time, reward_mode, alt_hunt_coef):
        cfg = REWARD_CONFIG if cfg is None else cfg
        mode = validate_reward_mode(reward_mode, alt_hunt_coef)
        return _lib.RewardCfg(self.dt, float(min_alt), float(max_time), float(cfg.get("own_damage_weight", 0.5)),
                              float(cfg["damage_scale"]), float(cfg["shaping_reward_scale"]), float(cfg["win_reward"]),
                              float(cfg["loss_reward"]), float(cfg["timeout_win_reward"]),
                              float(cfg["timeout_loss_reward"]), float(cfg["timeout_draw_reward"]),
                              float(alt_hunt_coef), mode, 0)

    def _actions(self, actions):
        _lib.require_cuda_tensor(actions, torch.float64, (self.nac, 4), "actions", self.device)
        return actions.contiguous()

    def kernel_advance(self, states, actions, cfg=None, min_alt=304.8, max_time=200.0, reward_mode=0,
                       alt_hunt_coef=5.0):
        """Fused advance + reward (one thread per env); call after the physics step.
        Returns (reward (nac,), term (nenv,) uint8, trunc (nenv,) uint8)."""
        rc = self._reward_cfg(cfg, min_alt, max_time, reward_mode, alt_hunt_coef)
        sp, lay, ld, keep = self._kernel_states(states)
        ac = self._actions(actions)
        recon = self._recon()
        self._external_advance(sp, lay, ld)
        _lib.check(self.lib.f16_obs_advance(sp, lay, ld, self.nenv, ac.data_ptr(), recon, rc, self._origin,
                                            self.reward_buf.data_ptr(), self.term_buf.data_ptr(),
                                            self.trunc_buf.data_ptr(), _lib.stream_of(self.hp)), "f16_obs_advance")
        return self.reward_buf, self.term_buf, self.trunc_buf

    def kernel_init_reward_state(self, states, env_mask=None):
        sp, lay, ld, keep = self._kernel_states(states)
        mp, mkeep = self._kernel_mask(env_mask)
        _lib.check(self.lib.f16_obs_init_reward(sp, lay, ld, self.nenv, mp, self._recon(), self._origin,
                                                _lib.stream_of(self.hp)), "f16_obs_init_reward")

    def kernel_build_obs(self, states, env_mask=None):
        """obs (nac,184) fp32 of the masked envs (all if None); other rows keep their values."""
        sp, lay, ld, keep = self._kernel_states(states)
        mp, mkeep = self._kernel_mask(env_mask)
        aux = self.aux_features.data_ptr() if self.aux_features is not None else None
        _lib.check(self.lib.f16_obs_build(sp, lay, ld, self.nenv, mp, self._recon(), self._origin,
                                          self.obs_buf.data_ptr(), aux, _lib.stream_of(self.hp)), "f16_obs_build")
        return self.obs_buf

    def kernel_step(self, states, actions, cfg=None, min_alt=304.8, max_time=200.0, reward_mode=0,
                    alt_hunt_coef=5.0):
        """kernel_advance followed by kernel_build_obs of every env, fused in one launch."""
        rc = self._reward_cfg(cfg, min_alt, max_time, reward_mode, alt_hunt_coef)
        sp, lay, ld, keep = self._kernel_states(states)
        ac = self._actions(actions)
        aux = self.aux_features.data_ptr() if self.aux_features is not None else None
        self._external_advance(sp, lay, ld)
        _lib.check(self.lib.f16_obs_step(sp, lay, ld, self.nenv, ac.data_ptr(), self._recon(), rc, self._origin,
                                         self.reward_buf.data_ptr(), self.term_buf.data_ptr(),
                                         self.trunc_buf.data_ptr(), self.obs_buf.data_ptr(), aux,
                                         _lib.stream_of(self.hp)), "f16_obs_step")
        return self.obs_buf, self.reward_buf, self.term_buf, self.trunc_buf

    # ---- external 214-D observation (obs_reward.py:471-496, external_observation.cu) ----
    def enable_external_observations(self):
        """Optional extra state for frozen 214-D opponents; never changes the 184-D rows or the
        reward."""
        if hasattr(self, "external_accel"):
            return
        n, dev = self.nac, self.device
        self.external_previous_velocity = torch.zeros(n, 3, device=dev, dtype=self.dtype)
        self.external_accel = torch.zeros_like(self.external_previous_velocity)
        self.external_obs = torch.zeros(n, 214, device=dev, dtype=torch.float32)
        self._AC_KEYS = self._AC_KEYS + ("external_previous_velocity", "external_accel")

    def _external_advance(self, sp, lay, ld):
        """The acceleration update that precedes the advance when external rows are enabled."""
        if not hasattr(self, "external_accel"):
            return
        _lib.check(self.lib.f16_external_accel(sp, lay, ld, self.nac, self.prev_valid.data_ptr(),
                                               self.external_previous_velocity.data_ptr(),
                                               self.external_accel.data_ptr(), self._origin, float(self.dt),
                                               _lib.stream_of(self.hp)), "f16_external_accel")

    def build_external_obs(self, states):
        """(nac, 214) rows: the 184-D rows rebuilt from `states` with the 30 acceleration features
        inserted before the action history."""
        self.enable_external_observations()
        self.kernel_build_obs(states)
        sp, lay, ld, keep = self._kernel_states(states)
        _lib.check(self.lib.f16_external_obs(sp, lay, ld, self.nac, self.external_accel.data_ptr(),
                                             self.obs_buf.data_ptr(), self.external_obs.data_ptr(), self._origin,
                                             _lib.stream_of(self.hp)), "f16_external_obs")
        return self.external_obs

    # ---- state bookkeeping (obs_reward.py:498-562) ----
    def reset_all(self):
        self.hp.fill_(1.0); self.fuel.fill_(1.0); self.t_sec.zero_()
        self.prev_att.zero_(); self.prev_valid.zero_(); self.pqr.zero_()
        self.last_dmg_dealt.zero_(); self.last_dmg_taken.zero_(); self.hp_loss.zero_()
        self.act_hist.zero_(); self.prev_x.zero_(); self.prev_x_valid.zero_()
        self.prev_alt_log.zero_()
        if hasattr(self, "external_accel"):
            self.external_accel.zero_(); self.external_previous_velocity.zero_()

    def reset_envs(self, env_mask):
        """Reset the reconstruction state of the masked envs in place, without a host sync."""
        ac = env_mask.repeat_interleave(2)
        ac1 = ac.unsqueeze(1)
        if hasattr(self, "external_accel"):
            self.external_accel.masked_fill_(ac1, 0.0)
            self.external_previous_velocity.masked_fill_(ac1, 0.0)
        self.hp.masked_fill_(ac, 1.0)
        self.fuel.masked_fill_(ac, 1.0)
        self.t_sec.masked_fill_(env_mask, 0.0)
        self.prev_att.masked_fill_(ac1, 0.0)
        self.prev_valid.masked_fill_(ac, False)
        self.pqr.masked_fill_(ac1, 0.0)
        self.last_dmg_dealt.masked_fill_(ac, 0.0)
        self.last_dmg_taken.masked_fill_(ac, 0.0)
        self.hp_loss.masked_fill_(ac, 0.0)
        self.act_hist.masked_fill_(ac.view(-1, 1, 1), 0.0)
        self.prev_x.masked_fill_(ac, 0.0)
        self.prev_x_valid.masked_fill_(ac, False)
        self.prev_alt_log.masked_fill_(ac, 0.0)

    def clone_state(self):
        buf = {k: getattr(self, k).clone() for k in self._AC_KEYS + self._ENV_KEYS}
        if self.aux_features is not None:
            buf["aux_features"] = self.aux_features.clone()
        return buf

    def capture_into(self, buf, env_mask):
        ac = env_mask.repeat_interleave(2)
        for k in self._AC_KEYS:
            buf[k][ac] = getattr(self, k)[ac]
        for k in self._ENV_KEYS:
            buf[k][env_mask] = getattr(self, k)[env_mask]
        if self.aux_features is not None:
            buf["aux_features"][env_mask] = self.aux_features[env_mask]

    def capture_where(self, buf, env_mask):
        """capture_into without boolean indexing: buf[k] = where(mask, current, buf[k]) for every
        reconstruction buffer, so no host synchronisation is needed."""
        ac = env_mask.repeat_interleave(2)
        for k in self._AC_KEYS:
            cur = getattr(self, k)
            m = ac.view(-1, *([1] * (cur.dim() - 1)))
            buf[k].copy_(torch.where(m, cur, buf[k]))
        for k in self._ENV_KEYS:
            buf[k].copy_(torch.where(env_mask, getattr(self, k), buf[k]))
        if self.aux_features is not None:
            buf["aux_features"].copy_(torch.where(env_mask.view(-1, 1), self.aux_features, buf["aux_features"]))

    def restore(self, buf):
        for k in self._AC_KEYS + self._ENV_KEYS:
            getattr(self, k).copy_(buf[k])
        if self.aux_features is not None:
            self.aux_features.copy_(buf["aux_features"])

    def push_actions(self, actions_nac4):
        """Newest action into row 0 of the 5-deep history (obs_reward.py:559-562)."""
        a = actions_nac4.to(self.dtype)
        self.act_hist.copy_(torch.roll(self.act_hist, 1, dims=1))
        self.act_hist[:, 0, :] = a[:, :ACT_DIM]
