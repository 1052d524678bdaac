"""bench.py's reference arm on the CPU, at a small size.

The driver runs `bench.py --impl reference` beside the library's own arm and
compares the two lines, so the reference line must carry the contract's keys
and the same `config` dict as the library's arm.  The arm runs the
reference's own CPU path (oracle/_ref, built from the reference sources) on
inputs the oracle's generator rebuilds on the CPU; it must not load the
library (hillserve_b200/_lib/libhsb.so).  Runs in a few seconds."""
from __future__ import annotations

import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
ARGS = ["--impl", "reference", "--tokens", "1024", "--batch", "4", "--steps", "1", "--warmup", "1"]


@pytest.fixture(scope="module")
def line():
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    # The child prints the JSON line, then the shared objects it mapped.
    code = ("import runpy, sys; sys.argv = ['bench.py'] + sys.argv[1:]; "
            "runpy.run_path('bench.py', run_name='__main__'); "
            "print('MAPS ' + ' '.join(sorted({l.split()[-1] for l in open('/proc/self/maps') "
            "if l.rstrip().endswith('.so')})))")
    r = subprocess.run([sys.executable, "-c", code, *ARGS], cwd=ROOT, env=env, capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    maps = [ln for ln in r.stdout.splitlines() if ln.startswith("MAPS ")]
    assert len(lines) == 1 and len(maps) == 1, r.stdout[-2000:]
    return json.loads(lines[0]), maps[0].split()[1:]


def test_reference_line_keeps_the_contract(line):
    d, _ = line
    if "unavailable" in d:
        pytest.skip(d["unavailable"])
    assert d["impl"] == "reference"
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["value"] > 0 and d["unit"] == "layer-steps/s" and d["higher_is_better"] is True
    assert d["cpu_baseline"]["kind"] == "reference" and d["cpu_baseline"]["value"] == d["value"]
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    assert d["steps"] == 1 and d["warmup"] >= 3


def test_reference_line_config_equals_the_library_arms(line):
    d, _ = line
    if "unavailable" in d:
        pytest.skip(d["unavailable"])
    sys.path.insert(0, str(ROOT))
    import bench

    saved = sys.argv
    try:
        sys.argv = ["bench.py", *ARGS]
        args = bench.parse()
    finally:
        sys.argv = saved
    assert d["config"] == json.loads(json.dumps(bench.shard_config(args, 1)))
    assert d["metric"] == bench.METRIC


def test_reference_arm_does_not_load_the_library(line):
    d, maps = line
    if "unavailable" in d:
        pytest.skip(d["unavailable"])
    assert not [m for m in maps if m.endswith("libhsb.so") or m.endswith("libhsb_compat.so")], maps
    assert any(m.endswith("libhs_ref.so") for m in maps), maps
