"""The drop-in's argument checks against the reference's, class and message.

tests/cpp/host_checks.cpp calls the path's C++ interfaces (FullGqaCpuScorer,
score_full_gqa_legacy_cpu, select_gqa_scores, gqa_physical_union,
pack_gqa_workspace) with 37 sets of arguments each must reject before doing
any work -- one bad argument at a time, and pairs that show which check comes
first -- and prints the exception's class and message per case.  Built
against the drop-in headers and libhsb_compat, its output must equal
tests/golden/host_checks_reference.txt, the same program built against the
reference's own headers and sources (tests/golden/make_golden.py
--only host_checks).  Where the reference tree is present the fixture itself
is reproduced.  No GPU is touched: CPU only."""
from __future__ import annotations

import shutil
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
FIXTURE = ROOT / "tests" / "golden" / "host_checks_reference.txt"
sys.path.insert(0, str(ROOT / "tests" / "golden"))
import make_golden as mg  # noqa: E402


def _run(exe: Path) -> str:
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    return r.stdout


@pytest.fixture(scope="module")
def gxx():
    if shutil.which("g++") is None:
        pytest.skip("g++ absent")


def test_dropin_rejects_like_the_reference(gxx, tmp_path):
    from hillserve_b200 import build

    if not build.COMPAT_LIB.exists():
        build.build()
    got = _run(mg.build_host_checks(tmp_path / "host_checks_dropin", "dropin"))
    want = FIXTURE.read_text()
    assert got.splitlines()[-1] == "cases|37"
    assert got == want


def test_fixture_reproduces_from_the_reference(gxx, tmp_path):
    if not (mg.REFERENCE / "policy" / "full_gqa_cpu.cpp").exists():
        pytest.skip("reference tree absent")
    assert _run(mg.build_host_checks(tmp_path / "host_checks_ref", "reference")) == FIXTURE.read_text()
