"""bench.py's reference arm on the CPU: one JSON line with the contract's
keys from rank 0, nothing (and exit status 0) from any other rank."""

from __future__ import annotations

import json
import os
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def _run(env_extra):
    env = dict(os.environ, **env_extra)
    cmd = [sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--workload", "decode8_int8",
           "--steps", "1", "--warmup", "0"]
    return subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=300)


def test_reference_arm_prints_one_contract_line():
    p = _run({"RANK": "0"})
    assert p.returncode == 0, p.stderr[-2000:]
    lines = [ln for ln in p.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1
    line = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["impl"] == "reference" and line["value"] > 0 and line["higher_is_better"] is True
    # the reference itself when its package is installed beside the bench, else the oracle port
    want = "reference" if (ROOT / "baseline" / "_ref" / "expertrelay").is_dir() else "port"
    assert line["cpu_baseline"]["kind"] == want and line["cpu_baseline"]["cores"] >= 1
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["value"] == line["value"]
    assert line["config"]["workload"] == "decode8_int8"


def test_reference_arm_other_ranks_exit_quietly():
    p = _run({"RANK": "1"})
    assert p.returncode == 0, p.stderr[-2000:]
    assert p.stdout.strip() == ""


def test_reference_arm_uses_every_core_under_a_launcher_limit():
    """torchrun sets OMP_NUM_THREADS=1 on every rank; the reference arm still
    gives BLAS and numba all of this host's cores and says so."""
    p = _run({"RANK": "0", "OMP_NUM_THREADS": "1"})
    assert p.returncode == 0, p.stderr[-2000:]
    line = json.loads(p.stdout.strip().splitlines()[-1])
    cores = line["cpu_baseline"]["cores"]
    assert cores == len(os.sched_getaffinity(0))
    assert line["cpu_baseline"]["threads"]["blas"] == cores


def test_expert_parallel_microbatch_sizes():
    """Microbatches of the expert-parallel layer: half a rank's tokens within
    4096..16384, a power of two that divides the rank's share, unless
    --ep-microbatch names one."""
    import argparse

    sys.path.insert(0, str(ROOT))
    import bench

    args = argparse.Namespace(ep_tokens=65536, ep_microbatch=0)
    assert [bench.ep_microbatch(args, w) for w in (1, 2, 4, 8)] == [16384, 16384, 8192, 4096]
    for w in (1, 2, 4, 8):
        assert (65536 // w) % bench.ep_microbatch(args, w) == 0
    assert bench.ep_microbatch(argparse.Namespace(ep_tokens=65536, ep_microbatch=2048), 2) == 2048


def test_roofline_traffic_comes_from_the_profiles():
    """The DRAM traffic a bench line carries is the per-launch figure of an
    ncu capture summarised under profiles/, named with the file it came from."""
    sys.path.insert(0, str(ROOT))
    import bench

    for workload in ("prefill4096_int8_zipf", "decode8_int8"):
        value, src = bench.traffic_from_profiles(workload, "gate_up")
        assert value and value > 1e8 and src.startswith("profiles/")
        assert f"traffic_per_launch_bytes[{workload}/gate_up]" in (ROOT / src).read_text()
    assert bench.traffic_from_profiles("no_such_workload", "gate_up") == (None, None)
