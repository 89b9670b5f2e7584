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
