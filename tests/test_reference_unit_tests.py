"""The reference's own unit tests, run against the reference build in
oracle/_ref.

That build -- compiled from the reference's sources by oracle/Makefile --
produces the golden fixtures under tests/golden and times the CPU baseline,
so its own tests must pass on it: scorer bit patterns
(tests/full_gqa_cpu_tests.cpp), the selector's semantics
(tests/gqa_policy_tests.cpp, tests/quality_alpha_tests.cpp), pack and union
(tests/gqa_pack_tests.cpp), the V3 pipeline markers
(kernels/full_gqa_pipeline/kernel_check.cpp) and the V2 kernel with N from 1
(tests/full_gqa_kernel_check.cpp), the binary16 helpers
(tests/policy_tests.cpp), the payload cover (tests/full_gqa_prefetch_tests.cpp),
H2O residency and the read plan.  Each program exits 0 on success.  Skipped
where the reference sources were absent at build time.  CPU only, a few
seconds."""
from __future__ import annotations

import subprocess
from pathlib import Path

import pytest

REF = Path(__file__).resolve().parents[1] / "oracle" / "_ref"
PROGRAMS = ["policy_tests", "full_gqa_cpu_tests", "gqa_policy_tests", "gqa_pack_tests", "qk_pipeline_check",
            "h2o_residency_tests", "kv_read_plan_tests", "full_gqa_prefetch_tests", "quality_alpha_tests",
            "full_gqa_kernel_check"]


@pytest.mark.parametrize("program", PROGRAMS)
def test_reference_program_passes(program, tmp_path):
    exe = REF / program
    if not exe.exists():
        pytest.skip(f"{program} not built (reference sources absent at build time)")
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300, cwd=tmp_path)
    assert r.returncode == 0, (r.stdout[-2000:], r.stderr[-2000:])
    assert "passed" in r.stdout + r.stderr
