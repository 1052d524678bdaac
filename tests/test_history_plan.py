"""The decode history's hot placement (hsb_history_plan_slots) against the
reference's plan_full_gqa_runtime (runtime/full_gqa_contract.hpp, compiled
from its source into oracle/_ref where it exists) and the fixture made from
it; and the planner's rejections.  CPU only."""
from __future__ import annotations

import ctypes as C
from pathlib import Path

import numpy as np
import pytest

import inputs
from oracle import binding as ob

GOLDEN = Path(__file__).resolve().parent / "golden" / "history_plans.npz"


def _plan(lib, cap, prompt, gen, beta, partial):
    out = np.zeros(cap, dtype=np.int64)
    hot = C.c_size_t(0)
    rc = lib.hsb_history_plan_slots(prompt, gen, cap, beta, int(partial), out.ctypes.data, C.byref(hot))
    return rc, out, hot.value


@pytest.fixture(scope="module")
def lib():
    from hillserve_b200 import _capi

    return _capi.lib()


def test_plan_matches_fixture(lib):
    import importlib.util
    import sys

    spec = importlib.util.spec_from_file_location("make_golden", GOLDEN.parent / "make_golden.py")
    mg = importlib.util.module_from_spec(spec)
    sys.modules.setdefault("make_golden", mg)
    spec.loader.exec_module(mg)
    g = np.load(GOLDEN)
    for i, case in enumerate(mg.PLAN_CASES):
        rc, slots, hot = _plan(lib, *case)
        assert rc == 0
        assert inputs.digest(slots) == str(g["slots_digest"][i]), case
        assert hot == int(g["hot_tokens"][i])


@pytest.mark.skipif(not ob.reference_available(), reason="reference sources not built here")
def test_plan_matches_reference_randomised(lib):
    rng = np.random.default_rng(8)
    for _ in range(60):
        prompt = int(rng.integers(128, 20000))
        partial = bool(prompt % 64) or bool(rng.integers(0, 2))
        gen = int(rng.integers(1, 513))
        cap = (prompt + gen + 63) // 64 * 64 + 64 * int(rng.integers(0, 3))
        beta = float(rng.choice([0.0, 0.1, 0.5, 1.0, 2.0, 9.0, np.inf]))
        rc, slots, hot = _plan(lib, cap, prompt, gen, beta, partial)
        ref, ref_hot = ob.ref_plan_hot_slots(cap, prompt, gen, beta, partial)
        assert rc == 0 and np.array_equal(slots, ref) and hot == ref_hot


def test_plan_rejections(lib):
    assert _plan(lib, 4096, 100, 16, 1.0, True)[0] == 101        # prompt < 128
    assert _plan(lib, 4096, 4000, 16, 1.0, False)[0] == 101      # partial tail without hot-tail mode
    assert _plan(lib, 4096, 3968, 0, 1.0, False)[0] == 101       # generated 0
    assert _plan(lib, 4096, 3968, 513, 1.0, False)[0] == 101
    assert _plan(lib, 4000, 3840, 16, 1.0, False)[0] == 101      # capacity not 64-aligned
    assert _plan(lib, 4096, 3968, 16, -1.0, False)[0] == 101
    assert _plan(lib, 4096, 3968, 16, float("nan"), False)[0] == 101
