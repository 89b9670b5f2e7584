#!/usr/bin/env python3
"""Record the environment contract of the reference trainer (dropin_trace.json).

Runs the reference's own PPOGPUTrainer (research/competition_36500/runtime/cuda_fdm/ppo_gpu.py:
__init__ :1099-1180 with _reset_env_state :1315-1328, collect_rollout :1856-2017, and the
checkpoint pair _runtime_state / _restore_runtime :2859-2920) on CPU against a traced stand-in
environment, and writes every attribute read, attribute write and method call the trainer makes on
the environment (its ``sim`` and ``obr`` members included) with the type / shape / dtype of
each argument and result.  tests/test_dropin_gpu.py replays the trace against this package's
GpuDogfightVecEnv on a GPU: every read must exist with the recorded type, shape and dtype, every
call must accept the recorded arguments and return the recorded structure.

The stand-in restates the reference environment's interface, not its physics: step returns
obs (nenv,2,184) float32, reward (nenv,2) float64, done (nenv,) bool and the info dict of
rl_env.py:499-555; the reconstruction buffers are BatchObsReward's (obs_reward.py:338-353); the
simulator holds states (nac,101), obs (nac,17), actions (nac,4) float64 (gpu_env.py:60-62).
Run only where the reference tree is available; the GPU box replays the committed JSON.
"""
import json
import os
import sys
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
REF = Path(os.environ.get("F16_REFERENCE") or ROOT.parent / "reference")
OUT = Path(__file__).resolve().parent / "dropin_trace.json"
NENV, T = 8, 3


def spec(v):
    """JSON description of a value (tensors by shape and dtype)."""
    if torch.is_tensor(v):
        return {"tensor": list(v.shape), "dtype": str(v.dtype).replace("torch.", "")}
    if isinstance(v, (bool, np.bool_)):
        return {"bool": bool(v)}
    if isinstance(v, (int, np.integer)):
        return {"int": int(v)}
    if isinstance(v, (float, np.floating)):
        return {"float": float(v)}
    if isinstance(v, str):
        return {"str": v}
    if v is None:
        return {"none": True}
    if isinstance(v, dict):
        return {"dict": {str(k): spec(x) for k, x in v.items()}}
    if isinstance(v, (tuple, list)):
        return {"seq": [spec(x) for x in v]}
    if isinstance(v, np.random.Generator):
        return {"numpy_generator": True}
    return {"object": type(v).__name__}


class TracedDict(dict):
    """A returned dict that records which keys the trainer reads."""

    def __init__(self, d, path, log):
        super().__init__(d)
        self._path, self._log = path, log

    def __getitem__(self, k):
        v = super().__getitem__(k)
        self._log.append({"op": "item", "path": f"{self._path}[{k!r}]", "value": spec(v)})
        return v


class Traced:
    """Proxy of the stand-in: records attribute reads / writes and calls by dotted path."""

    SUB = ("sim", "obr")

    def __init__(self, target, path, log):
        object.__setattr__(self, "_t", target)
        object.__setattr__(self, "_path", path)
        object.__setattr__(self, "_log", log)

    def __getattr__(self, name):
        v = getattr(self._t, name)
        p = f"{self._path}.{name}"
        if callable(v) and not torch.is_tensor(v):
            def call(*a, **k):
                r = v(*a, **k)
                self._log.append({"op": "call", "path": p, "args": [spec(x) for x in a],
                                  "kwargs": {kk: spec(x) for kk, x in k.items()}, "ret": spec(r)})
                if isinstance(r, tuple) and len(r) == 4 and isinstance(r[3], dict):
                    r = r[:3] + (TracedDict(r[3], p + "()[3]", self._log),)
                return r
            return call
        self._log.append({"op": "get", "path": p, "value": spec(v)})
        if name in self.SUB:
            return Traced(v, p, self._log)
        return v

    def __setattr__(self, name, value):
        self._log.append({"op": "set", "path": f"{self._path}.{name}", "value": spec(value)})
        setattr(self._t, name, value)


def stand_in(nenv):
    """The reference environment's interface with placeholder values."""
    import types
    nac = 2 * nenv
    f64 = torch.float64
    keys = dict(hp=(nac,), fuel=(nac,), prev_att=(nac, 3), pqr=(nac, 3), last_dmg_dealt=(nac,),
                last_dmg_taken=(nac,), hp_loss=(nac,), act_hist=(nac, 5, 4), prev_x=(nac,), prev_alt_log=(nac,))

    class Obr:
        dt = 0.1
        aux_features = None

        def __init__(self):
            for k, s in keys.items():
                setattr(self, k, torch.ones(s, dtype=f64))
            self.prev_valid = torch.zeros(nac, dtype=torch.bool)
            self.prev_x_valid = torch.zeros(nac, dtype=torch.bool)
            self.t_sec = torch.zeros(nenv, dtype=f64)

        def clone_state(self):
            return {k: getattr(self, k).clone() for k in list(keys) + ["prev_valid", "prev_x_valid", "t_sec"]}

        def restore(self, buf):
            for k, v in buf.items():
                getattr(self, k).copy_(v)

    class Env:
        OBS_SIZE = 184
        substeps = 6
        min_altitude_m = 304.8
        max_engage_time_s = 200.0
        reward_mode = 0
        alt_hunt_coef = 5.0

        def __init__(self):
            self.nenv, self.nac = nenv, nac
            self.obr = Obr()
            self.sim = types.SimpleNamespace(states=torch.zeros(nac, 101, dtype=f64), obs=torch.zeros(nac, 17, dtype=f64),
                                             actions=torch.zeros(nac, 4, dtype=f64))
            self.ic_pool = torch.zeros(4096, 2, 101, dtype=f64)      # rl_env.py ic_pool_size 4096
            self.ic_pool_size = 4096
            self.rng = np.random.default_rng(0)
            self.reward_cfg = {"shaping_reward_scale": 0.0001}

        def reset(self, stagger=True, max_stagger_steps=256, warmup_action_fn=None):
            return torch.zeros(nenv, 2, 184)

        def step(self, actions, *, reset_indices=None):
            info = {"terminated": torch.zeros(nenv, dtype=torch.bool), "truncated": torch.zeros(nenv, dtype=torch.bool),
                    "terminal_obs": torch.zeros(nenv, 2, 184), "terminal_hp": torch.ones(nenv, 2, dtype=f64),
                    "terminal_alt_m": torch.full((nenv, 2), 5000.0, dtype=f64),
                    "done": torch.zeros(nenv, dtype=torch.bool),
                    "terminal_state_finite": torch.ones(nenv, dtype=torch.bool)}
            return (torch.zeros(nenv, 2, 184), torch.zeros(nenv, 2, dtype=f64), torch.zeros(nenv, dtype=torch.bool),
                    info)

    return Env()


def main():
    r36 = REF / "research" / "competition_36500" / "runtime"
    for k in list(sys.modules):
        if k.split(".")[0] in ("cuda_fdm", "claude_code"):
            del sys.modules[k]
    sys.path.insert(0, str(r36))
    sys.path.insert(0, str(REF / "src"))
    import cuda_fdm.ppo_gpu as P
    log = []
    env = Traced(stand_in(NENV), "env", log)
    cfg = P.PPOGPUConfig(device="cpu", rollout_steps=T, hidden=(32, 32), activation="tanh", league_enabled=False,
                         aux_pred=False, seed=3)
    phases = {}
    trainer = P.PPOGPUTrainer(env, cfg)
    phases["init"] = len(log)
    trainer.collect_rollout()
    phases["collect_rollout"] = len(log)
    state = trainer._runtime_state()
    phases["runtime_state"] = len(log)
    trainer._restore_runtime(state)
    phases["restore_runtime"] = len(log)
    out = {"nenv": NENV, "rollout_steps": T, "phases": phases, "ops": log,
           "source": "research/competition_36500/runtime/cuda_fdm/ppo_gpu.py PPOGPUTrainer on CPU"}
    OUT.write_text(json.dumps(out, indent=1) + "\n")
    print(OUT, len(log), "operations", phases)


if __name__ == "__main__":
    main()
