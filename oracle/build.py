#!/usr/bin/env python3
"""Build the parity checkers (TEST INFRASTRUCTURE ONLY).

* ``oracle/liboracle.so``          -- our C restatement of the reference FDM (fdm_oracle.c).
* ``oracle/_ref/libf16ref_root.so`` -- the reference's own fdm.cuh (repository root lineage,
  FCS dt 1/120), host-compiled from where it lies under the reference tree.
* ``oracle/_ref/libf16ref_r36.so``  -- the same for research/competition_36500/runtime
  (FCS dt 1/60, the 184-D lineage).
* ``oracle/_ref/libobsref.so``      -- the reference's own observation / reward kernels
  (research/competition_36500/runtime/cuda_fdm/gen/obs_kernel.cu with external_observation.cu),
  host-compiled through ref_obs_driver.cpp.

The ``_ref`` builds need the reference tree (``$F16_REFERENCE``, else a ``reference`` directory beside this repository); on a
machine without it they are skipped and the previously built files are used as they are.
Flags follow the reference's own host validation: ``-O2 -ffp-contract=off``.
"""
import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
# The reference checkout: $F16_REFERENCE, else a "reference" directory beside this repository;
# where neither exists the _ref builds are skipped.
REF = Path(os.environ.get("F16_REFERENCE") or HERE.parent.parent / "reference")
CFLAGS = ["-O2", "-ffp-contract=off", "-fPIC", "-shared"]
REF_LINEAGES = {
    "root": REF / "cuda_fdm" / "gen",
    "r36": REF / "research" / "competition_36500" / "runtime" / "cuda_fdm" / "gen",
}


def _run(cmd):
    print(" ".join(str(c) for c in cmd), flush=True)
    subprocess.run([str(c) for c in cmd], check=True)


def build_oracle(force=False):
    out = HERE / "liboracle.so"
    srcs = [HERE / "fdm_oracle.c", HERE / "obs_oracle.c"]
    deps = srcs + [HERE.parent / "include" / "f16env.h",
                   HERE.parent / "2026_ai_pilot_challenge-1st_solution_b200" / "csrc" / "f16_tables.h"]
    if force or not out.exists() or any(d.stat().st_mtime > out.stat().st_mtime for d in deps):
        _run(["gcc", "-std=c99", *CFLAGS, *srcs, "-o", out, "-lm"])
    return out


def build_ref(force=False):
    outdir = HERE / "_ref"
    outdir.mkdir(exist_ok=True)
    built = {}
    for name, gen in REF_LINEAGES.items():
        out = outdir / f"libf16ref_{name}.so"
        if (gen / "fdm.cuh").exists():
            if force or not out.exists() or (HERE / "ref_driver.cpp").stat().st_mtime > out.stat().st_mtime:
                _run(["g++", "-std=c++14", *CFLAGS, "-fopenmp", "-I", gen, HERE / "ref_driver.cpp",
                      "-o", out, "-lm"])
        if out.exists():
            built[name] = out
    # the reference's own observation / reward kernels (184-D lineage), host-compiled
    r36 = REF_LINEAGES["r36"]
    out = outdir / "libobsref.so"
    if (r36 / "obs_kernel.cu").exists():
        drv = HERE / "ref_obs_driver.cpp"
        if force or not out.exists() or drv.stat().st_mtime > out.stat().st_mtime:
            _run(["g++", "-std=c++14", *CFLAGS, "-I", r36, "-I", r36.parent, drv, "-o", out, "-lm"])
    if out.exists():
        built["obs"] = out
    return built


def main():
    force = "--force" in sys.argv
    build_oracle(force)
    print("reference builds:", build_ref(force))


if __name__ == "__main__":
    main()
