"""The drop-in headers under hillserve_b200/compat against the reference's own
translation units.

A maintainer swaps the path onto the B200 by putting hillserve_b200/compat
first on the include path.  Every reference source that includes one of the
replaced headers and stays in the build must then still compile: the
runtime policy and the no-SSD policy (the path's callers), the scorer's and
the half helpers' own sources, the V3 pipeline check, and the reference's
unit tests of the path.  Each is compiled here with `g++ -fsyntax-only`,
the drop-in directory before the reference tree, exactly as the swap would
compile it.  Sources that need headers absent from this machine (llama.cpp,
ggml) are not listed.  Skipped where the reference tree is absent.  CPU
only."""
from __future__ import annotations

import os
import shutil
import subprocess
import sysconfig
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
REFERENCE = Path(os.environ.get("HILLSERVE_REFERENCE", "/root/reference"))
SOURCES = [
    "policy/full_gqa_runtime.cpp",
    "runtime/no_ssd_policy.cpp",
    "policy/full_gqa_cpu.cpp",
    "policy/host_policy.cpp",
    "kernels/full_gqa_pipeline/kernel_check.cpp",
    "tests/full_gqa_cpu_tests.cpp",
    "tests/gqa_pack_tests.cpp",
    "tests/policy_tests.cpp",
    "tests/full_gqa_prefetch_tests.cpp",
    "tests/quality_alpha_tests.cpp",
    "tests/full_gqa_runtime_tests.cpp",
    "tests/no_ssd_policy_tests.cpp",
]


def _nlohmann() -> str | None:
    # The runtime policy includes nlohmann/json.hpp, which the reference does
    # not vendor; a copy ships with the cuDNN frontend headers.
    p = Path(sysconfig.get_paths()["purelib"]) / "include" / "cudnn_frontend" / "thirdparty"
    return str(p) if (p / "nlohmann" / "json.hpp").exists() else None


def _compile(src: str):
    cmd = ["g++", "-std=c++17", "-fsyntax-only", f"-I{ROOT / 'hillserve_b200' / 'compat'}", f"-I{ROOT / 'include'}",
           f"-I{REFERENCE}"]
    nl = _nlohmann()
    if nl:
        cmd.append(f"-I{nl}")
    r = subprocess.run([*cmd, str(REFERENCE / src)], capture_output=True, text=True, timeout=300)
    return src, r.returncode, r.stderr


@pytest.fixture(scope="module")
def results():
    if not (REFERENCE / "policy" / "full_gqa_cpu.cpp").exists():
        pytest.skip("reference tree absent")
    if shutil.which("g++") is None:
        pytest.skip("g++ absent")
    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        return {src: (rc, err) for src, rc, err in ex.map(_compile, SOURCES)}


@pytest.mark.parametrize("src", SOURCES)
def test_reference_source_compiles_against_dropin(results, src):
    if src.startswith("policy/full_gqa_runtime") or src.endswith("runtime_tests.cpp") or \
            src.endswith("prefetch_tests.cpp") or src.endswith("quality_alpha_tests.cpp"):
        if _nlohmann() is None:
            pytest.skip("nlohmann/json.hpp absent")
    rc, err = results[src]
    assert rc == 0, err[-3000:]
