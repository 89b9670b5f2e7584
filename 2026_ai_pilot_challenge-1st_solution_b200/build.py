"""Build ``libf16env.so`` (all CUDA kernels + the C ABI) in-tree for sm_100a.

Every ``csrc/*.cu`` file is compiled with nvcc for ``sm_100a`` only (no PTX, no other
architectures) and linked into one shared library next to this file.  The library is
what ``_lib.py`` loads; it travels with the source tree (it is git-ignored, not copied into
site-packages).
"""
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
OUT = HERE / "libf16env.so"
OBJ = HERE / "_build"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
              "-Xptxas", "-warn-spills"]


def nvcc():
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise FileNotFoundError("nvcc not found (set NVCC)")


def _deps(src):
    return [src] + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + [HERE.parent / "include" / "f16env.h"]


def _stale(target, deps):
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.exists() and d.stat().st_mtime > t for d in deps)


def build(force=False, verbose=False):
    """Compile stale objects and relink. Returns the library path."""
    OBJ.mkdir(exist_ok=True)
    srcs = sorted(CSRC.glob("*.cu"))
    cc = nvcc()
    jobs = []
    for s in srcs:
        o = OBJ / (s.stem + ".o")
        if force or _stale(o, _deps(s)):
            jobs.append([cc, *ARCH, *NVCC_FLAGS, "-I", str(CSRC), "-c", str(s), "-o", str(o)])

    def run(cmd):
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed:\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
        if verbose and (r.stdout or r.stderr):
            print(r.stdout + r.stderr)
        return r

    with ThreadPoolExecutor(max_workers=max(1, min(len(jobs), os.cpu_count() or 4))) as ex:
        list(ex.map(run, jobs))
    objs = [OBJ / (s.stem + ".o") for s in srcs]
    if force or jobs or _stale(OUT, objs):
        run([cc, *ARCH, "-shared", "-o", str(OUT), *map(str, objs), "-lcuda"])
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
