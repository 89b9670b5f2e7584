"""The ctypes mirrors of the C-ABI structs (``_lib.py``, ``policy.py``) have the C header's layout:
same size and the same offset for every field, as a C compiler lays out include/f16env.h."""
import ctypes
import shutil
import subprocess

import pytest

from conftest import ROOT, pkg_module

PAIRS = [("f16_fdm_io", "_lib", "FdmIO"), ("f16_recon", "_lib", "Recon"), ("f16_reward_cfg", "_lib", "RewardCfg"),
         ("f16_origin", "_lib", "Origin"), ("f16_record_args", "_lib", "RecordArgs"),
         ("f16_payoff_args", "_lib", "PayoffArgs"), ("f16_mlp_desc", "policy", "MlpDesc"),
         ("f16_policy_args", "policy", "PolicyArgs")]


@pytest.fixture(scope="module")
def c_layout(tmp_path_factory):
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    lines = ['#include <stddef.h>', '#include <stdio.h>', '#include "f16env.h"', "int main(void) {"]
    for cname, mod, cls in PAIRS:
        py = getattr(pkg_module(mod), cls)
        lines.append(f'  printf("{cname} size %zu\\n", sizeof({cname}));')
        for field in py._fields_:
            lines.append(f'  printf("{cname} {field[0]} %zu\\n", offsetof({cname}, {field[0]}));')
    lines += ["  return 0;", "}"]
    d = tmp_path_factory.mktemp("abi")
    src, exe = d / "layout.c", d / "layout"
    src.write_text("\n".join(lines) + "\n")
    subprocess.run([cc, "-std=c99", "-I", str(ROOT / "include"), str(src), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout
    table = {}
    for ln in out.splitlines():
        struct, key, val = ln.split()
        table[(struct, key)] = int(val)
    return table


@pytest.mark.parametrize("cname,mod,cls", PAIRS)
def test_struct_layout_matches_header(c_layout, cname, mod, cls):
    py = getattr(pkg_module(mod), cls)
    assert ctypes.sizeof(py) == c_layout[(cname, "size")], f"{cls} size differs from {cname}"
    for field in py._fields_:
        off = getattr(py, field[0]).offset
        assert off == c_layout[(cname, field[0])], f"{cls}.{field[0]} at {off}, {cname} at {c_layout[(cname, field[0])]}"
