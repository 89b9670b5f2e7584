"""bench.py run exactly as the round-end driver runs it (N=1, 20 timed steps, 5 warm-up
steps): it must exit 0 and print one parsable JSON line carrying the contract's keys.  The
CPU tests cover the helpers that need no GPU."""
import json
import subprocess
import sys

import pytest

from conftest import ROOT


def _bench():
    sys.path.insert(0, str(ROOT))
    import bench
    return bench


def test_host_cores_counts_the_affinity_set():
    import os
    b = _bench()
    assert b.host_cores() == len(os.sched_getaffinity(0))


def test_profile_traffic_refuses_a_stale_summary(tmp_path, monkeypatch):
    b = _bench()
    prof = tmp_path / "profiles"
    prof.mkdir()
    name = "fdm_step_cfg2.md"
    monkeypatch.setattr(b, "ROOT", tmp_path)
    (tmp_path / b.PKG).mkdir()
    (tmp_path / b.PKG / "csrc").symlink_to(ROOT / b.PKG / "csrc")
    cur = b.kernel_source_sha16(name)
    (prof / name).write_text(f"traffic_bytes_per_launch: 123\nkernel_source_sha16: {cur}\n")
    assert b.profile_traffic(name)[0] == 123.0
    (prof / name).write_text("traffic_bytes_per_launch: 123\nkernel_source_sha16: 0000000000000000\n")
    v, why = b.profile_traffic(name)
    assert v is None and "predates" in why


def test_reference_arm_sampler_steps_the_reference():
    """The --impl reference arm's sampler: the reference's fdm.cuh compiled here (or, where
    that build is absent, the C restatement on one core) steps a bounded sample and reports a
    rate; with the reference present every host core of the affinity set is used."""
    b = _bench()
    run, threads, n, kind = b.cpu_reference_sampler(nsample_per_thread=8)
    rate, reps = run(0.2)
    assert rate > 0 and reps >= 1 and n >= 64
    assert (kind, threads) == ("port", 1) or (kind == "reference" and threads == b.host_cores())


@pytest.mark.gpu
def test_driver_command_line_prints_the_contract_line(cuda):
    r = subprocess.run([sys.executable, "bench.py", "--gpus", "1", "--steps", "20", "--warmup", "5"],
                       cwd=ROOT, capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stderr[-4000:]
    line = json.loads(r.stdout.strip().splitlines()[-1])
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
              "scaling", "dtype", "config", "roofline", "e2e", "gpu_launches", "clocks", "cpu_baseline"):
        assert k in line, k
    assert line["steps"] == 20 and line["warmup"] == 5 and line["n_gpus"] == 1
    assert line["value"] > 0 and line["e2e"]["value"] > 0 and line["roofline"]["frac"] > 0
    assert line["cpu_baseline"]["value"] > 0 and line["cpu_baseline"]["cores"] >= 1
