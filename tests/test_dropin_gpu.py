"""Drop-in proof at the trainer boundary: the reference trainer's environment contract replayed
against this package's GpuDogfightVecEnv -- needs a B200.

tests/golden/dropin_trace.json was recorded by running the reference's own PPOGPUTrainer
(research/competition_36500/runtime/cuda_fdm/ppo_gpu.py: construction with its first reset,
collect_rollout :1856-2017, and the checkpoint pair _runtime_state / _restore_runtime
:2859-2920) on CPU against a traced stand-in of its environment (make_dropin_trace.py): every
attribute read and write and every call the trainer makes on ``env``, ``env.sim`` and
``env.obr``, with the type / shape / dtype of each argument and result, and the info keys it
reads.  Here each operation is replayed in order on GpuDogfightVecEnv: every attribute must
exist with the recorded type, shape, dtype and (for integers and the reward configuration)
value, every call must accept the recorded arguments and return the recorded structure, every
written attribute must be writable.  Devices are not compared (the trace ran on CPU).
"""
import json

import numpy as np
import pytest
import torch

from conftest import GOLDEN, pkg_module

pytestmark = pytest.mark.gpu


def conforms(v, s, where):
    if "tensor" in s:
        assert torch.is_tensor(v), f"{where}: expected a tensor, got {type(v).__name__}"
        assert list(v.shape) == s["tensor"], f"{where}: shape {list(v.shape)} != {s['tensor']}"
        assert str(v.dtype).replace("torch.", "") == s["dtype"], f"{where}: dtype {v.dtype} != {s['dtype']}"
    elif "bool" in s:
        assert isinstance(v, (bool, np.bool_)), f"{where}: expected bool"
    elif "int" in s:
        assert isinstance(v, (int, np.integer)) and not isinstance(v, bool), f"{where}: expected int"
        assert int(v) == s["int"], f"{where}: {v} != {s['int']}"
    elif "float" in s:
        assert isinstance(v, (float, int, np.floating)), f"{where}: expected a number"
        assert float(v) == s["float"], f"{where}: {v} != {s['float']}"
    elif "none" in s:
        assert v is None, f"{where}: expected None"
    elif "dict" in s:
        assert isinstance(v, dict), f"{where}: expected a dict"
        for k, sub in s["dict"].items():
            assert k in v, f"{where}: key {k!r} missing"
            conforms(v[k], sub, f"{where}[{k!r}]")
    elif "seq" in s:
        assert isinstance(v, (tuple, list)) and len(v) == len(s["seq"]), f"{where}: expected {len(s['seq'])} items"
        for i, (x, sub) in enumerate(zip(v, s["seq"])):
            conforms(x, sub, f"{where}[{i}]")
    elif "numpy_generator" in s:
        assert isinstance(v, np.random.Generator), f"{where}: expected a numpy Generator"
    else:
        assert v is not None, f"{where}: missing"


def make(s, dev):
    """An argument of the recorded spec (tensors zero-filled on the GPU)."""
    if "tensor" in s:
        return torch.zeros(s["tensor"], dtype=getattr(torch, s["dtype"]), device=dev)
    if "dict" in s:
        return {k: make(x, dev) for k, x in s["dict"].items()}
    if "seq" in s:
        return [make(x, dev) for x in s["seq"]]
    for k in ("int", "float", "bool", "str"):
        if k in s:
            return s[k]
    return None


def resolve(root, path):
    """(owner, attribute name) of a dotted path below ``env``."""
    parts = path.split(".")
    assert parts[0] == "env"
    obj = root
    for p in parts[1:-1]:
        obj = getattr(obj, p)
    return obj, parts[-1]


def test_reference_trainer_contract_replays_on_gpu_env(cuda):
    rl_env = pkg_module("rl_env")
    trace = json.loads((GOLDEN / "dropin_trace.json").read_text())
    env = rl_env.GpuDogfightVecEnv(trace["nenv"], seed=3, device=cuda)
    last = {}
    counts = {}
    for i, e in enumerate(trace["ops"]):
        where = f"op {i} {e['op']} {e['path']}"
        counts[e["op"]] = counts.get(e["op"], 0) + 1
        if e["op"] == "item":
            base, key = e["path"].split("()[3][")
            info = last[base][3]
            conforms(info[key[1:-2]], e["value"], where)
            continue
        owner, name = resolve(env, e["path"])
        assert hasattr(owner, name), f"{where}: attribute missing"
        if e["op"] == "get":
            conforms(getattr(owner, name), e["value"], where)
        elif e["op"] == "set":
            cur = getattr(owner, name)
            conforms(cur, e["value"], where)
            setattr(owner, name, cur)                     # writable
        else:
            fn = getattr(owner, name)
            args = [make(a, cuda) for a in e["args"]]
            kwargs = {k: make(a, cuda) for k, a in e["kwargs"].items()}
            r = fn(*args, **kwargs)
            conforms(r, e["ret"], where)
            last[e["path"]] = r
    torch.cuda.synchronize()
    print("replayed", counts)
    assert counts.get("call", 0) >= 5 and counts.get("item", 0) >= 9
