"""The C++ drop-in layer on the GPU: tests/cpp/compat_tests.cpp includes the
reference's own header paths (policy/full_gqa_cpu.hpp, policy/gqa_policy.hpp,
runtime/gqa_pack.hpp, runtime/gqa_prefetch_cuda.hpp, runtime/gqa_delivery.hpp)
from hillserve_b200/compat and runs the reference unit tests' checks against
the B200 implementation."""
from __future__ import annotations

import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
pytestmark = pytest.mark.gpu


def build_compat_tests() -> Path:
    from hillserve_b200 import build

    build.build()
    out = ROOT / "tests" / "cpp" / "_build" / "compat_tests"
    src = ROOT / "tests" / "cpp" / "compat_tests.cpp"
    lib = build.LIBDIR
    if not out.exists() or out.stat().st_mtime < max(src.stat().st_mtime, build.COMPAT_LIB.stat().st_mtime):
        out.parent.mkdir(parents=True, exist_ok=True)
        subprocess.run([build.nvcc_path(), "-std=c++17", "-O2", "-x", "cu", *build.ARCH,
                        f"-I{ROOT / 'hillserve_b200' / 'compat'}", f"-I{ROOT / 'include'}", str(src), "-o", str(out),
                        f"-L{lib}", "-lhsb_compat", "-lhsb", "--cudart", "shared", f"-Xlinker=-rpath,{lib}",
                        f"-Xlinker=-rpath,{build.CUDA_LIB}"], check=True)
    return out


def test_reference_interfaces_on_b200(cuda):
    exe = build_compat_tests()
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr + r.stdout
    assert '"status":"passed"' in r.stdout


@pytest.mark.parametrize("program", ["full_gqa_cpu_tests", "gqa_pack_tests", "quality_alpha_tests",
                                     "full_gqa_prefetch_tests", "no_ssd_policy_tests"])
def test_reference_unit_test_program_on_b200(cuda, program, tmp_path):
    """The reference's own test programs, compiled unmodified against the
    drop-in headers and linked to libhsb_compat (oracle/Makefile), run on the
    library's kernels:

    - tests/full_gqa_cpu_tests.cpp: the scorer, bit-exact against the test's
      independent oracle (ragged and non-contiguous views, subnormals,
      overflow, signed zero, the rounding-mode rejection);
    - tests/gqa_pack_tests.cpp: union and pack layout;
    - tests/quality_alpha_tests.cpp and tests/full_gqa_prefetch_tests.cpp:
      the reference's FullGqaRuntimePolicy (built from its own sources) with
      its scorer and selector taken from the drop-in -- exact k and counts per
      alpha, the live runtime against its scalar oracle, and the payload
      cover containing the final selections;
    - tests/no_ssd_policy_tests.cpp: the reference's no-SSD policy
      (runtime/no_ssd_policy.cpp) on the drop-in scorer and selector."""
    exe = ROOT / "oracle" / "_ref" / f"{program}_b200"
    if not exe.exists():
        pytest.skip("built only where the reference sources were present")
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300, cwd=tmp_path)
    assert r.returncode == 0, r.stderr + r.stdout
    assert "pass" in r.stdout.lower()
