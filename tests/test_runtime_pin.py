"""The payload cover and the decode selection pinned to the reference's own
FullGqaRuntimePolicy (policy/full_gqa_runtime.cpp:299-344 prefetch_payload,
:549-585 select), run by tests/golden/make_golden.py --only runtime through
oracle/_ref/libhs_ref_runtime.so (compiled from the reference sources) on
seeded prompts and rehearsal queries.  The fixture tests/golden/
runtime_decode.npz holds, per decode step, the cover's per-head bound and
lists, its sorted physical IDs with the reference's hot/cold placement, and
the final per-head selections.

CPU: the oracle's cover (orc_prefetch_cover) and selection chain reproduce
them bit for bit.  Where the reference runtime library is built, the fixture
itself is reproduced live."""
from __future__ import annotations

import sys
import tempfile
from pathlib import Path

import numpy as np
import pytest

import inputs

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT / "tests" / "golden"))
import make_golden as mg  # noqa: E402

FIXTURE = ROOT / "tests" / "golden" / "runtime_decode.npz"


def load():
    return np.load(FIXTURE, allow_pickle=False)


def case(i):
    seed, cap, prompt, steps, layer, beta, alpha = mg.RUNTIME_CASES[i]
    return int(seed), int(cap), int(prompt), int(steps), int(layer), float(beta), float(alpha)


@pytest.mark.parametrize("i", range(len(mg.RUNTIME_CASES)))
def test_oracle_cover_and_selection_match_reference_runtime(ob, i):
    fx = load()
    seed, cap, prompt, steps, layer, beta, alpha = case(i)
    rows = mg.runtime_rows(seed, cap)
    q = mg.runtime_queries(seed, steps)
    assert str(fx[f"c{i}_input_digest"]) == inputs.digest(rows, q)
    for s in range(steps):
        pos = prompt + s
        q16 = q[s].astype(np.float16).view(np.uint16)  # F16-exact: the runtime's query_f16
        raw = np.zeros((32, cap), dtype=np.uint16)
        raw[:, :pos] = ob.score(q16, rows[:pos, :1024].reshape(-1), pos, 1024)
        per_head, physical = ob.prefetch_cover(raw, cap, pos, alpha)
        bound = int(fx[f"c{i}_bound"][s])
        assert per_head.shape[1] == bound
        assert np.array_equal(per_head.astype(np.uint32), fx[f"c{i}_cover"][s][:, :bound])
        nphys = int(fx[f"c{i}_nphysical"][s])
        assert np.array_equal(physical.astype(np.uint32), fx[f"c{i}_physical"][s][:nphys])
        raw[:, :pos + 1] = ob.score(q16, rows[:pos + 1, :1024].reshape(-1), pos + 1, 1024)
        ids, counts, k, tied = ob.select(ob.scale(raw), 32, cap, pos + 1, alpha, 0.2)
        assert k == int(fx[f"c{i}_k"][s])
        assert np.array_equal(ids.astype(np.uint32), fx[f"c{i}_final"][s][:, :k])


def test_placement_matches_reference_runtime(ob):
    """The cold flags the reference runtime reported for the cover's rows
    equal the library's placement rule (hsb_history_plan_slots restates
    plan_full_gqa_runtime; pinned in test_history_plan.py)."""
    fx = load()
    for i in range(len(mg.RUNTIME_CASES)):
        seed, cap, prompt, steps, layer, beta, alpha = case(i)
        if not ob.reference_available():
            pytest.skip("reference placement library not built")
        slots, _ = ob.ref_plan_hot_slots(cap, prompt, steps, beta)
        for s in range(steps):
            n = int(fx[f"c{i}_nphysical"][s])
            phys = fx[f"c{i}_physical"][s][:n].astype(np.int64)
            assert np.array_equal(fx[f"c{i}_cold"][s][:n].astype(bool), slots[phys] < 0)


@pytest.mark.skipif(not (ROOT / "oracle" / "_ref" / "libhs_ref_runtime.so").exists(),
                    reason="reference runtime library not built (reference sources absent)")
def test_fixture_reproduces_live(ob):
    fx = load()
    for i in (0, 2):
        seed, cap, prompt, steps, layer, beta, alpha = case(i)
        with tempfile.TemporaryDirectory() as d:
            r = ob.ref_runtime_decode(mg.runtime_rows(seed, cap), cap, prompt, steps, layer, beta, alpha,
                                      mg.runtime_queries(seed, steps), d)
        assert np.array_equal(r["bound"], fx[f"c{i}_bound"]) and np.array_equal(r["k"], fx[f"c{i}_k"])
        kmax = int(r["k"].max())
        assert np.array_equal(r["final"][:, :, :kmax].astype(np.uint32), fx[f"c{i}_final"])
