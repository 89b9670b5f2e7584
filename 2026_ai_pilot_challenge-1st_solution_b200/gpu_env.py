"""``GpuDogfight``: drop-in for the reference's batched F-16 physics object (cuda_fdm/gpu_env.py:25-112).

Same constructor, attributes and methods (``states (nac,101)``, ``obs (nac,17)``, ``actions
(nac,4)``, ``load_seed``, ``reset_ic``, ``step``, ``get_state``, ``get_obs``), backed by the
AOT-built sm_100a kernel ``f16_fdm_step`` instead of an NVRTC compile.

Memory layout: the state lives in a (101, nac) structure-of-arrays buffer so every column is
read and written with coalesced accesses; ``states`` is the (nac, 101) transposed *view* of
it, so the reference's indexing (``states[:, 0:3]``, ``torch.where(mask, rows, states)``,
``states[idx] = rows``, ``.view(nenv, 2, 101)``) works unchanged on the same memory.
"""
import numpy as np
import torch

from . import _lib
from .ic import ic_rows, seed_states

STATE_N = _lib.STATE_N
OBS_N = _lib.OBS17_N
# obs17 columns (cuda_fdm/gpu_env.py:19-22)
OBS = dict(eci_pos=slice(0, 3), eci_vel=slice(3, 6), euler=slice(6, 9),
           vUVW=slice(9, 12), alpha=12, beta=13, mach=14, Vt=15, alt_asl=16)

FCS_DT_ROOT = 1.0 / 120.0     # cuda_fdm/gen/fdm.cuh:23 (golden contract)
FCS_DT_R36 = 1.0 / 60.0       # research/competition_36500 lineage (184-D env)


class GpuDogfight:
    """nenv one-vs-one engagements, planes_per_env aircraft each (a = ppe*e + k)."""

    def __init__(self, nenv, substeps=1, planes_per_env=2, block=128, precision="fp64",
                 max_registers="auto", fcs_dt=FCS_DT_ROOT, device="cuda"):
        if precision != "fp64":
            raise NotImplementedError("only precision='fp64' is implemented on the B200 path")
        if not torch.cuda.is_available():
            raise RuntimeError("GpuDogfight needs a CUDA device")
        self.lib = _lib.load()
        self.nenv = int(nenv)
        self.ppe = int(planes_per_env)
        self.nac = self.nenv * self.ppe
        self.substeps = int(substeps)
        self.block = block                 # accepted for API parity; launch shape is chosen by the library
        self.max_registers = max_registers
        self.precision = precision
        self.dtype = torch.float64
        self.fcs_dt = float(fcs_dt)
        self.device = torch.device(device) if not isinstance(device, torch.device) else device
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.states_soa = torch.zeros(STATE_N, self.nac, dtype=torch.float64, device=self.device)
        self.states = self.states_soa.t()              # (nac, 101) view, stride (1, nac)
        self.obs = torch.zeros(self.nac, OBS_N, dtype=torch.float64, device=self.device)
        self.actions = torch.zeros(self.nac, 4, dtype=torch.float64, device=self.device)
        self._grid_cache = {}

    # ---- reset ----
    def load_seed(self, seed):
        """seed: (nac,101), (101,) broadcast, (ppe,101) per-plane, or (nenv,ppe,101)."""
        t = torch.as_tensor(seed, dtype=torch.float64)
        if t.ndim == 1:
            t = t.unsqueeze(0).expand(self.nac, -1)
        elif t.ndim == 3:
            t = t.reshape(self.nac, STATE_N)
        elif t.shape[0] != self.nac:
            t = t.unsqueeze(0).expand(self.nenv, -1, -1).reshape(self.nac, STATE_N)
        self.states.copy_(t.to(self.device))

    def reset_ic(self, ic_list):
        """ic_list: nac IC dicts (or (nenv, ppe) nested), keyword names of cuda_fdm/ic.py
        build_seed_vector.  Seeds are built on the GPU (f16_seed_ic)."""
        flat = []
        for item in ic_list:
            if isinstance(item, dict):
                flat.append(item)
            else:
                flat.extend(item)
        if len(flat) != self.nac:
            raise ValueError(f"{len(flat)} != nac {self.nac}")
        seed_states(ic_rows(flat), self.fcs_dt, device=self.device, out=self.states_soa)

    def reset_ic_rows(self, rows):
        """(nac, 12) IC rows (include/f16env.h F16_IC_* columns) -> seeded states, on the GPU."""
        rows = np.asarray(rows, dtype=np.float64) if not torch.is_tensor(rows) else rows
        if rows.shape[0] != self.nac:
            raise ValueError(f"{rows.shape[0]} != nac {self.nac}")
        seed_states(rows, self.fcs_dt, device=self.device, out=self.states_soa)

    # ---- step ----
    def step(self, actions, substeps=None):
        """actions: (nac,4) or (nenv,ppe,4) [aileron, elevator, rudder, throttle].
        Returns obs (nenv, ppe, 17), a view of self.obs."""
        ss = self.substeps if substeps is None else int(substeps)
        a = torch.as_tensor(actions, dtype=torch.float64, device=self.device).reshape(self.nac, 4)
        self.actions.copy_(a)
        _lib.check(self.lib.f16_fdm_step(_lib.ptr(self.states_soa), _lib.LAYOUT_SOA, self.nac, self.nac,
                                         _lib.ptr(self.actions), ss, self.fcs_dt, _lib.ptr(self.obs),
                                         _lib.stream_of(self.states_soa)), "f16_fdm_step")
        return self.obs.view(self.nenv, self.ppe, OBS_N)

    def step_host(self, actions, obs_out=None, substeps=None, chunks=4):
        """step() driven from host memory: ``actions`` (nac, 4) fp64 on the host (pinned, so the
        copies are asynchronous) and obs17 written into ``obs_out`` (nac, 17) fp64 host memory
        (pinned; allocated once when omitted).  The aircraft are split into ``chunks`` slices
        whose host-to-device copy, FDM launch and device-to-host copy run on a stream of their
        own, so the copies of one slice overlap the physics of the others; the caller's
        current stream waits for all of it.  Results are step()'s bit for bit (aircraft are
        independent).  Returns ``obs_out`` viewed (nenv, ppe, 17)."""
        ss = self.substeps if substeps is None else int(substeps)
        a = torch.as_tensor(actions, dtype=torch.float64)
        if a.device.type != "cpu":
            raise ValueError("step_host takes host actions; use step() for device tensors")
        a = a.reshape(self.nac, 4).contiguous()
        if obs_out is None:
            if getattr(self, "_host_obs", None) is None:
                self._host_obs = torch.empty(self.nac, OBS_N, dtype=torch.float64).pin_memory()
            obs_out = self._host_obs
        if obs_out.device.type != "cpu" or obs_out.dtype != torch.float64 or obs_out.numel() != self.nac * OBS_N:
            raise ValueError("obs_out must be a (nac, 17) float64 host tensor")
        out = obs_out.view(self.nac, OBS_N)
        n, chunks = self.nac, max(1, min(int(chunks), self.nac))
        if getattr(self, "_side_streams", None) is None:
            self._side_streams = []
        while len(self._side_streams) < chunks:            # one stream per slice
            self._side_streams.append(torch.cuda.Stream(self.device))
        cur = torch.cuda.current_stream(self.device)
        start = torch.cuda.Event()
        start.record(cur)
        st, act, obs = self.states_soa.data_ptr(), self.actions.data_ptr(), self.obs.data_ptr()
        for i in range(chunks):
            lo, hi = n * i // chunks, n * (i + 1) // chunks
            if hi == lo:
                continue
            s = self._side_streams[i]
            s.wait_event(start)
            with torch.cuda.stream(s):
                self.actions[lo:hi].copy_(a[lo:hi], non_blocking=True)
                _lib.check(self.lib.f16_fdm_step(st + 8 * lo, _lib.LAYOUT_SOA, self.nac, hi - lo, act + 32 * lo, ss,
                                                 self.fcs_dt, obs + 8 * OBS_N * lo, s.cuda_stream), "f16_fdm_step")
                out[lo:hi].copy_(self.obs[lo:hi], non_blocking=True)
        for s in self._side_streams[:chunks]:
            cur.wait_stream(s)
        return out.view(self.nenv, self.ppe, OBS_N)

    def step_bins(self, bins, num_bins=21, substeps=None, write_obs=True, grid=None):
        """Fused action mapping: bins (nac,4) uint8 -> reference action_to_env grid -> FDM.
        grid: the float32 action grid (default: torch.linspace(-1, 1, num_bins) evaluated on
        this device, as the reference trainer builds it, R/cuda_fdm/ppo_gpu.py:1134)."""
        ss = self.substeps if substeps is None else int(substeps)
        _lib.require_cuda_tensor(bins, torch.uint8, (self.nac, 4), "action bins", self.device)
        b = bins.contiguous()
        if grid is None:
            grid = self._grid_cache.get(num_bins)
            if grid is None:
                grid = torch.linspace(-1.0, 1.0, int(num_bins), device=self.device).cpu().contiguous()
                self._grid_cache[num_bins] = grid
        g = torch.as_tensor(grid, dtype=torch.float32).cpu().contiguous()
        if g.numel() != num_bins:
            raise ValueError("grid must hold num_bins values")
        _lib.check(self.lib.f16_fdm_step_bins(_lib.ptr(self.states_soa), _lib.LAYOUT_SOA, self.nac, self.nac,
                                              _lib.ptr(b), _lib.ptr(g), int(num_bins), ss, self.fcs_dt,
                                              _lib.ptr(self.obs) if write_obs else None,
                                              _lib.stream_of(self.states_soa)), "f16_fdm_step_bins")
        return self.obs.view(self.nenv, self.ppe, OBS_N)

    def get_state(self):
        return self.states.view(self.nenv, self.ppe, STATE_N)

    def get_obs(self):
        return self.obs.view(self.nenv, self.ppe, OBS_N)
