"""The bench.py output contract, checked on the CPU through its reference arm.

`bench.py --impl reference` times the reference's own CPU matmul (oracle/_ref, built
from the tensor.cx sources) on the GPU arm's metric and config. Its stdout must be
exactly one JSON line with the keys a benchmark driver reads; under a multi-rank launch
only rank 0 prints and the other ranks exit 0 without work. The GPU arm shares the
line's layout and needs a B200, so only its argument parsing is checked here.
"""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BENCH = os.path.join(ROOT, "bench.py")


def _run(args, env_extra=None, timeout=300):
    env = dict(os.environ)
    for k in ("RANK", "WORLD_SIZE", "LOCAL_RANK"):
        env.pop(k, None)
    env.update(env_extra or {})
    return subprocess.run([sys.executable, BENCH, *args], capture_output=True, text=True, cwd=ROOT, env=env,
                          timeout=timeout)


def test_help_lists_the_driver_flags():
    r = _run(["--help"])
    assert r.returncode == 0, r.stderr
    for flag in ("--gpus", "--steps", "--warmup", "--impl"):
        assert flag in r.stdout


def test_reference_arm_prints_one_contract_line():
    from oracle.oracle import Reference
    r = _run(["--impl", "reference", "--steps", "2", "--warmup", "1", "--size", "512"])
    assert r.returncode == 0, r.stderr
    lines = [ln for ln in r.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1, r.stdout
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    if not Reference.available():
        assert "unavailable" in d
        pytest.skip("oracle/_ref/libtcx_ref.so not built: the arm reports itself unavailable")
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["steps"] == 2 and d["warmup"] == 1 and d["n_gpus"] == 1
    assert d["unit"] == "TFLOP/s" and d["higher_is_better"] is True and d["scaling"] == "weak"
    assert d["value"] > 0 and d["ms_per_step"] > 0
    assert "workload" in d["config"]
    cb = d["cpu_baseline"]
    assert cb["kind"] == "reference" and cb["cores"] >= 1 and cb["value"] == d["value"] and cb["sample"]
    e2e = d["e2e"]
    assert e2e["value"] == d["value"] and e2e["unit"] == d["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0


def test_reference_arm_other_ranks_exit_quietly():
    r = _run(["--impl", "reference", "--gpus", "2", "--steps", "1", "--warmup", "1", "--size", "512"],
             {"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"})
    assert r.returncode == 0, r.stderr
    assert r.stdout.strip() == ""
