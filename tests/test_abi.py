"""The C-ABI library loads without a GPU and exports every entry point include/f16env.h declares."""
import ctypes
import re
from pathlib import Path

from conftest import ROOT, pkg_module

HEADER = ROOT / "include" / "f16env.h"


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\*?\s+\**(f16_\w+)\s*\(", text, flags=re.M)))


def test_header_declares_entry_points():
    names = declared_functions()
    assert "f16_fdm_step" in names and "f16_seed_ic" in names
    assert len(names) >= 5


def test_library_exports_every_declared_symbol():
    _lib = pkg_module("_lib")
    lib = _lib.load()
    for name in declared_functions():
        assert hasattr(lib, name), f"{name} declared in f16env.h but not exported"
        assert name in _lib.exported_symbols(), f"{name} has no ctypes signature in _lib.py"
    for name in _lib.exported_symbols():
        assert name in declared_functions(), f"{name} bound in _lib.py but not declared"


def test_library_reports_version_and_status_without_gpu():
    lib = pkg_module("_lib").load()
    assert b"sm_100a" in lib.f16_version()
    assert lib.f16_status_string(1) == b"invalid argument"


def test_entry_points_reject_bad_arguments_before_any_launch():
    """Null / negative-size arguments return F16_ERR_ARG without touching a device."""
    lib = pkg_module("_lib").load()
    assert lib.f16_fdm_step(None, 0, 1, 1, None, 6, 1 / 60, None, None) == 1
    assert lib.f16_fdm_step_bins(None, 0, 1, 1, None, None, 21, 6, 1 / 60, None, None) == 1
    buf = (ctypes.c_double * 202)()
    assert lib.f16_fdm_step(ctypes.cast(buf, ctypes.c_void_p), 0, 1, 2, None, 6, 1 / 60, None, None) == 1
    assert lib.f16_fdm_step(ctypes.cast(buf, ctypes.c_void_p), 7, 2, 2, ctypes.cast(buf, ctypes.c_void_p),
                            6, 1 / 60, None, None) == 1
    assert lib.f16_seed_ic(None, 4, None, 0, 4, 1 / 60, None) == 1


def test_update_entry_points_reject_bad_arguments_before_any_launch():
    """The PPO-update kernels' entry points check shapes, part counts, activation codes and the
    categorical head's limits on the host (F16_ERR_ARG = 1) before any launch."""
    lib = pkg_module("_lib").load()
    buf = (ctypes.c_float * 4096)()
    p = ctypes.cast(buf, ctypes.c_void_p)
    assert lib.f16_split3_bf16(None, 4, 8, 8, p, 24, 3, None) == 1
    assert lib.f16_split3_bf16(p, 4, 6, 8, p, 24, 3, None) == 1          # cols not a multiple of 4
    assert lib.f16_split3_bf16(p, 4, 8, 8, p, 24, 5, None) == 1          # parts must be 3 or 6
    assert lib.f16_split3_bf16(p, 4, 8, 8, p, 40, 6, None) == 1          # row stride below 6 parts
    assert lib.f16_bias_act_split(p, 4, 8, 8, p, 3, None, 0, 3, None) == 1   # unknown activation
    assert lib.f16_bias_act_split(p, 4, 8, 8, p, 1, p, 16, 3, None) == 1     # split row stride too small
    assert lib.f16_act_grad_split(p, 8, None, 8, 4, 8, 1, p, 24, 3, p, 1, None) == 1   # relu without h
    assert lib.f16_act_grad_split(p, 2048, p, 2048, 4, 2048, 0, p, 6144, 3, p, 1, None) == 1  # > 1024 cols
    assert lib.f16_bias_act_value(p, 4, 8, 8, p, 1, None, p, p, None) == 1            # no head weight
    assert lib.f16_act_grad_split_value(p, p, p, 8, 4, 8, 1, p, 24, 3, p, p, 0, None) == 1   # nblk 0
    assert lib.f16_categorical_fwd(p, 84, 4, 4, 33, p, 1, p, p, p, None) == 1      # B > 32
    assert lib.f16_categorical_fwd(p, 84, 4, 4, 21, p, 2, p, p, p, None) == 1      # action bytes 2
    assert lib.f16_categorical_bwd(p, 84, 4, 4, 21, p, 1, None, None, p, 80, None) == 1   # ldg < A*B


def test_dropin_trace_fixture_covers_the_trainer_contract():
    """The recorded reference-trainer contract (tests/golden/dropin_trace.json, replayed on the
    GPU by test_dropin_gpu.py) holds the reset, one step per rollout step with the three info
    keys the trainer reads, and the checkpoint reads / writes."""
    import json
    from conftest import GOLDEN
    t = json.loads((GOLDEN / "dropin_trace.json").read_text())
    calls = [e["path"] for e in t["ops"] if e["op"] == "call"]
    assert calls.count("env.step") == t["rollout_steps"] and "env.reset" in calls
    assert {"env.obr.clone_state", "env.obr.restore"} <= set(calls)
    items = {e["path"].split("[")[-1] for e in t["ops"] if e["op"] == "item"}
    assert items == {"'terminal_state_finite']", "'terminal_hp']", "'terminal_alt_m']"}
    sets = {e["path"] for e in t["ops"] if e["op"] == "set"}
    assert {"env.reward_mode", "env.alt_hunt_coef", "env.ic_pool"} <= sets
