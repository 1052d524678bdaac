"""The host-side parts of the Python mirror (hillserve_b200/__init__.py) on the
CPU: the FullGqaCpuScorer mirror's argument checks and accessors, and the
host-only wrappers (the segment file header, the read plan and its
validation groups, the history's hot placement) against the C ABI and the
golden fixtures made from the reference.  No call here reaches a kernel."""
from __future__ import annotations

import ctypes as C
import importlib.util
import sys
from pathlib import Path

import numpy as np
import pytest

import inputs

GOLDEN = Path(__file__).resolve().parent / "golden"


def _make_golden():
    spec = importlib.util.spec_from_file_location("make_golden", GOLDEN / "make_golden.py")
    mg = importlib.util.module_from_spec(spec)
    sys.modules.setdefault("make_golden", mg)
    spec.loader.exec_module(mg)
    return mg


@pytest.fixture(scope="module")
def hsb():
    pytest.importorskip("torch")
    import hillserve_b200

    return hillserve_b200


def test_scorer_mirror_checks_like_the_reference(hsb):
    # policy/full_gqa_cpu.cpp:153-163: threads 1..128, a known implementation.
    for threads in (0, 129):
        with pytest.raises(hsb.InvalidArgument, match="full GQA CPU threads must be 1..128"):
            hsb.FullGqaScorer(threads)
    with pytest.raises(hsb.InvalidArgument, match="unknown full GQA CPU implementation"):
        hsb.FullGqaScorer(4, "avx512")
    s = hsb.FullGqaScorer(7, "scalar")
    assert s.threads() == 7 and s.implementation_name() == "sm100a_ordered_fp32"


@pytest.mark.parametrize("case", [0, 1, 2])
def test_segment_header_wrapper_matches_the_reference_file(hsb, ob, case):
    mg = _make_golden()
    request, layers, positions, nbytes, payloads = mg.record_case(case)
    img = inputs.segment_image(request, layers, positions, nbytes, payloads, ob.records_encode)
    assert inputs.digest(img) == str(np.load(GOLDEN / "records_vectors.npz")[f"file{case}_digest"])
    assert hsb.segment_header(request, layers, positions, nbytes) == img[:4096].tobytes()
    assert hsb.segment_extent_bytes(layers, positions, nbytes) == img.nbytes


def test_segment_header_wrapper_raises_on_bad_geometry(hsb):
    with pytest.raises(hsb.HsbError):
        hsb.segment_header(1, 0, 10, 4096)


def test_read_plan_wrappers_match_the_c_abi(hsb):
    from hillserve_b200 import _capi

    lib = _capi.lib()
    rng = np.random.default_rng(2)
    stride, positions = 4128, 32768
    ids = np.sort(rng.choice(positions, 500, replace=False))
    offs = [4096 + int(i) * stride for i in ids]
    extent = hsb.segment_extent_bytes(1, positions, 4096)
    plan = hsb.kv_read_plan(offs, stride, extent)
    arr = (C.c_uint64 * len(offs))(*offs)
    wins = (hsb.KVReadWindow * len(offs))()
    n = C.c_size_t(0)
    assert lib.hsb_kv_read_plan(arr, len(offs), stride, extent, 1 << 20, 16 << 10, 1500, wins, len(wins),
                                C.byref(n)) == 0
    assert plan == [(w.begin, w.end, w.required_page_bytes, w.first_record, w.end_record) for w in wins[:n.value]]
    assert plan[0][3] == 0 and plan[-1][4] == len(offs)
    groups = hsb.kv_read_groups(plan, len(offs))
    assert len(groups) == len(offs) and min(groups) >= 0


def test_hot_placement_wrapper_matches_the_fixture(hsb):
    mg = _make_golden()
    g = np.load(GOLDEN / "history_plans.npz")
    for i, (cap, prompt, gen, beta, partial) in enumerate(mg.PLAN_CASES):
        slots, hot = hsb.plan_hot_slots(prompt, gen, cap, beta, partial)
        assert inputs.digest(slots) == str(g["slots_digest"][i]), (cap, prompt, gen, beta, partial)
        assert hot == int(g["hot_tokens"][i])
