"""Generates the golden fixtures in tests/golden/ by running the REFERENCE's
own CPU code (oracle/_ref/libhs_ref.so, compiled from the HillServe sources by
oracle/Makefile) on seeded inputs.  Run here, where the reference sources
exist:

    make -C oracle && python tests/golden/make_golden.py [--only h2o|records|history|runtime|host_checks]

Inputs are regenerated bit-exactly from their seeds by tests/inputs.py, so
the fixtures hold only input digests and the reference's outputs.
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tests"))

from oracle import binding as ob  # noqa: E402
import inputs  # noqa: E402

OUT = Path(__file__).resolve().parent
ALPHAS = (0.1, 5.0, 10.0, 20.0, 50.0)


def ref_scores(q, k, n, stride, threads=8):
    scorer = ob.RefScorer(threads, 0)
    return scorer.score(q, [(k, 0, n, stride)])


def scorer_vectors():
    """The reference scorer test's own vectors (full_gqa_cpu_tests.cpp:76-86)."""
    rng = inputs.XorShift32(0x7F123451)
    out = {}
    for n in (1, 2, 7, 8, 9, 17, 65, 129):
        for stride in (1024, 2048):
            q, data = inputs.cpu_test_case(rng, n, stride)
            s = ref_scores(q, data, n, stride)
            out[f"n{n}_s{stride}"] = (inputs.digest(q, data), inputs.digest(s))
            if n >= 9:  # mixed views: tokens 7-8, 0-2, 1
                views = [(data, 7 * stride, 2, stride), (data, 0, 3, stride), (data, stride, 1, stride)]
                mv = ob.RefScorer(2, 0).score(q, views)
                out[f"n{n}_s{stride}_views"] = (inputs.digest(q, data), inputs.digest(mv))
    return out


# (first, queries) blocks of the H2O fixture; keys = first + queries.
H2O_BLOCKS = ((0, 1), (0, 3), (0, 7), (0, 16), (0, 17), (0, 64), (0, 129),
              (3, 2), (5, 1), (63, 1), (100, 17), (255, 1), (200, 56), (511, 4))


def h2o_reference_importance(seed: int, first: int, queries: int) -> np.ndarray:
    """The reference H2OResidency's importance after observing, through its
    own CPU observe_attention (policy/h2o_residency.cpp:60-80), a one-hot
    block on key 0 for queries 0..first-1 and then the seeded block
    (first, queries).  Keys >= 1 hold exactly that block's group sums."""
    keys = first + queries
    r = ob.RefH2O(prompt_tokens=keys)
    if first:
        prior = np.zeros((32, first, first), dtype=np.float32)
        prior[:, :, 0] = 1.0
        r.observe_attention(0, 0, first, first, prior)
    r.observe_attention(0, first, queries, keys, inputs.h2o_probabilities(seed, first, queries, keys))
    return r.importance(0, keys)


def h2o_vectors() -> None:
    names, digests, heads = [], [], []
    for i, (first, queries) in enumerate(H2O_BLOCKS):
        imp = h2o_reference_importance(1000 + i, first, queries)
        names.append(f"f{first}_q{queries}")
        digests.append(inputs.digest(imp))
        heads.append(imp[:, :8] if imp.shape[1] >= 8 else np.pad(imp, ((0, 0), (0, 8 - imp.shape[1]))))
    np.savez_compressed(OUT / "h2o_vectors.npz", names=np.array(names), blocks=np.array(H2O_BLOCKS),
                        importance_digest=np.array(digests), importance_head=np.stack(heads))


# (request, layers, positions, record_bytes, rows per layer) of the record fixture
RECORD_CASES = ((991, 3, 70, 4096, (70, 33, 0)), (765, 2, 37, 100, (37, 5)), (7, 1, 9, 4128, (9,)))


def record_case(i: int):
    request, layers, positions, nbytes, rows = RECORD_CASES[i]
    payloads = [inputs.record_payload(100 * i + l, r, nbytes) for l, r in enumerate(rows)]
    return request, layers, positions, nbytes, payloads


def plan_case(seed: int):
    """Seeded sorted record offsets of one layer of a 32 x 4096-position store
    (stride 4128) and read limits, in the shape of kv_read_plan_tests.cpp."""
    rng = np.random.default_rng(seed)
    capacity, stride = 4096, 4128
    extent = (4096 + 32 * capacity * stride + 4095) // 4096 * 4096
    layer = int(rng.integers(0, 32))
    n = int(rng.integers(1, 600))
    ids = np.sort(rng.choice(capacity, size=n, replace=False))
    offsets = (4096 + (layer * capacity + ids) * stride).astype(np.uint64)
    window = int(rng.choice([12288, 65536, 1 << 20]))
    gap = int(rng.choice([0, 4096, 16384, 65536]))
    amp = int(rng.choice([1000, 1250, 1500, 2000]))
    return offsets, stride, extent, window, gap, amp


def records_vectors() -> None:
    import tempfile

    fields = {}
    # checksum_four over the reference reader test's bytes (direct_read_batch_tests.cpp:17-19)
    i = np.arange(4 * 65536, dtype=np.uint64)
    data = ((i // 4096 * 31 + i * 17) % 251).astype(np.uint8)
    rows = [data[j * 65536:(j + 1) * 65536] for j in range(4)]
    four = []
    for length in (0, 1, 17, 4096, 65536):
        for n in range(1, 5):
            four.append(ob.ref_checksum_four(rows[:n], length) + [0] * (4 - n))
    fields["checksum_four"] = np.array(four, dtype=np.uint64)
    # whole store files written by the reference SegmentedKVStore
    with tempfile.TemporaryDirectory() as tmp:
        for c in range(len(RECORD_CASES)):
            request, layers, positions, nbytes, payloads = record_case(c)
            path = f"{tmp}/store{c}"
            ob.ref_segment_roundtrip(path, request, layers, positions, nbytes, 9 << 30, payloads)
            fields[f"file{c}_digest"] = inputs.digest(np.fromfile(path, dtype=np.uint8))
    # read plans
    plans = []
    for seed in range(24):
        offsets, stride, extent, window, gap, amp = plan_case(seed)
        plans.append(inputs.digest(ob.ref_read_plan(offsets, stride, extent, window, gap, amp)))
    fields["plan_digest"] = np.array(plans)
    np.savez_compressed(OUT / "records_vectors.npz", **fields)


# (capacity, prompt, generated, beta, allow_partial) of the placement fixture
PLAN_CASES = ((4096, 3968, 128, 1.0, False), (4096, 4000, 16, 1.0, True), (32832, 32768, 64, 1.0, False),
              (32832, 32768, 64, 0.25, False), (8192, 8000, 100, float("inf"), True), (192, 128, 1, 1.0, False),
              (49152, 48000, 512, 3.0, False), (4096, 2048, 512, 0.0, False), (16384, 16000, 200, 7.5, True))


def history_plans() -> None:
    digests, hots = [], []
    for cap, prompt, gen, beta, partial in PLAN_CASES:
        slots, hot = ob.ref_plan_hot_slots(cap, prompt, gen, beta, partial)
        digests.append(inputs.digest(slots))
        hots.append(hot)
    np.savez_compressed(OUT / "history_plans.npz", slots_digest=np.array(digests), hot_tokens=np.array(hots))


# Decode cases run through the reference's own FullGqaRuntimePolicy:
# (seed, capacity, prompt, steps, layer, beta, alpha).  Alphas are chosen so
# that no step selects nothing (the runtime throws there) and some steps stay
# below the 20 % cap.
RUNTIME_CASES = ((5, 192, 128, 3, 3, 1.0, 4.0), (6, 1088, 1024, 4, 2, 0.25, 3.0), (7, 4160, 4096, 2, 7, 1.0, 3.0),
                 (8, 640, 576, 3, 5, 0.5, 4.0), (9, 2112, 2048, 3, 4, 1.0, 6.0))


def runtime_rows(seed: int, capacity: int) -> np.ndarray:
    """K||V rows [capacity][2048] (F16 bits) of a runtime case: K ~ N(0,1)
    with heavy rows x4, V ~ N(0,1) (tests/inputs.py streams)."""
    k = inputs.normals(seed, capacity * 1024, stream=2).reshape(capacity, 1024)
    k[inputs.heavy_rows(seed, capacity)] *= 4.0
    rows = np.empty((capacity, 2048), dtype=np.uint16)
    rows[:, :1024] = inputs.f16_bits(k)
    rows[:, 1024:] = inputs.values(seed, capacity).reshape(capacity, 1024)
    return rows


def runtime_queries(seed: int, steps: int) -> np.ndarray:
    """F16-exact F32 rehearsal queries [steps][4096] of a runtime case."""
    return np.stack([inputs.f16_bits(inputs.normals(seed * 100 + s, 4096, stream=1)).view(np.float16)
                     .astype(np.float32) for s in range(steps)])


def runtime_vectors() -> None:
    import tempfile

    assert ob.ref_runtime_available(), "build oracle/_ref/libhs_ref_runtime.so first (make -C oracle)"
    fields = {"cases": np.array(RUNTIME_CASES, dtype=np.float64)}
    for i, (seed, cap, prompt, steps, layer, beta, alpha) in enumerate(RUNTIME_CASES):
        rows = runtime_rows(seed, cap)
        q = runtime_queries(seed, steps)
        with tempfile.TemporaryDirectory() as d:
            r = ob.ref_runtime_decode(rows, cap, prompt, steps, layer, beta, alpha, q, d)
        b = int(r["bound"].max())
        kmax = int(r["k"].max())
        fields[f"c{i}_input_digest"] = np.array(inputs.digest(rows, q))
        fields[f"c{i}_bound"] = r["bound"]
        fields[f"c{i}_cover"] = r["cover"][:, :, :b].astype(np.uint32)
        fields[f"c{i}_nphysical"] = r["nphysical"]
        fields[f"c{i}_physical"] = r["physical"][:, :int(r["nphysical"].max())].astype(np.uint32)
        fields[f"c{i}_cold"] = r["cold"][:, :int(r["nphysical"].max())]
        fields[f"c{i}_k"] = r["k"]
        fields[f"c{i}_final"] = r["final"][:, :, :kmax].astype(np.uint32)
        print("runtime case", i, "bound", r["bound"].tolist(), "k", r["k"].tolist(), "physical",
              r["nphysical"].tolist())
    np.savez_compressed(OUT / "runtime_decode.npz", **fields)


REFERENCE = Path(__import__("os").environ.get("HILLSERVE_REFERENCE", "/root/reference"))
HOST_CHECKS = ROOT / "tests" / "cpp" / "host_checks.cpp"


def build_host_checks(out: Path, against: str) -> Path:
    """tests/cpp/host_checks.cpp built against the reference's own headers and
    sources (against="reference") or against the drop-in headers and
    libhsb_compat (against="dropin")."""
    import subprocess

    cmd = ["g++", "-std=c++17", "-O1", "-ffp-contract=off", "-pthread"]
    if against == "reference":
        srcs = [REFERENCE / f for f in ("policy/full_gqa_cpu.cpp", "policy/gqa_policy.cpp", "policy/host_policy.cpp",
                                        "smartssd/adapter.cpp")]
        cmd += [f"-I{REFERENCE}", str(HOST_CHECKS), *map(str, srcs)]
    else:
        lib = ROOT / "hillserve_b200" / "_lib"
        cmd += [f"-I{ROOT / 'hillserve_b200' / 'compat'}", f"-I{ROOT / 'include'}", str(HOST_CHECKS), f"-L{lib}",
                "-lhsb_compat", "-lhsb", f"-Wl,-rpath,{lib}"]
    subprocess.run([*cmd, "-o", str(out)], check=True)
    return out


def host_checks() -> None:
    """The reference's exception class and message for each rejected call of
    tests/cpp/host_checks.cpp (host_checks_reference.txt)."""
    import subprocess
    import tempfile

    with tempfile.TemporaryDirectory() as d:
        exe = build_host_checks(Path(d) / "host_checks_ref", "reference")
        text = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout
    (OUT / "host_checks_reference.txt").write_text(text)


def main() -> None:
    assert ob.reference_available(), "build oracle/_ref first (make -C oracle)"
    if sys.argv[1:] == ["--only", "host_checks"]:
        host_checks()
        print("host-check fixture written to", OUT)
        return
    if sys.argv[1:] == ["--only", "runtime"]:
        runtime_vectors()
        print("runtime fixture written to", OUT)
        return
    if sys.argv[1:] == ["--only", "history"]:
        history_plans()
        print("history fixture written to", OUT)
        return
    if sys.argv[1:] == ["--only", "h2o"]:
        h2o_vectors()
        print("h2o fixture written to", OUT)
        return
    if sys.argv[1:] == ["--only", "records"]:
        records_vectors()
        print("records fixture written to", OUT)
        return
    records_vectors()
    history_plans()
    host_checks()
    if ob.ref_runtime_available():
        runtime_vectors()
    # ---- 0. H2O group sums through the reference's CPU policy
    h2o_vectors()
    # ---- 1. reference scorer test vectors
    vec = scorer_vectors()
    names = sorted(vec)
    np.savez_compressed(OUT / "scorer_vectors.npz", names=np.array(names),
                        input_digest=np.array([vec[n][0] for n in names]),
                        score_digest=np.array([vec[n][1] for n in names]))

    # ---- 2. config 1 (N=4096, seed 0) + alpha sweep, and config-3 lengths
    for n in (64, 1024, 4096, 16384):
        q, k, heavy = inputs.config1(n, seed=0)
        raw = ref_scores(q, k, n, 1024)
        scaled = ob.ref_scale(raw)
        fields = dict(n=n, input_digest=inputs.digest(q, k), raw_digest=inputs.digest(raw),
                      scaled_digest=inputs.digest(scaled), alphas=np.array(ALPHAS, dtype=np.float32))
        if n <= 1024:
            fields["raw"] = raw  # small enough to keep verbatim
        for a in ALPHAS:
            ids, counts, kk, tied = ob.ref_select(scaled, 32, n, n, a, 0.2)
            tag = f"a{a:g}".replace(".", "p")
            fields[f"{tag}_k"] = kk
            fields[f"{tag}_tied"] = tied
            fields[f"{tag}_counts"] = counts
            fields[f"{tag}_ids_digest"] = inputs.digest(ids.astype(np.uint32))
            fields[f"{tag}_ids_head"] = ids[:, : min(kk, 64)].astype(np.uint32)
        np.savez_compressed(OUT / f"config1_n{n}.npz", **fields)
        print("config1", n, {a: int(fields[f"a{a:g}".replace('.', 'p') + '_k']) for a in ALPHAS})

    # ---- 3. random selector trials (structure of gqa_policy_tests.cpp:49-59)
    rng = inputs.XorShift32(1741)
    sel = {}
    for trial in range(24):
        heads, n, stride = 32, 257, 288
        x = np.full(heads * stride, inputs.f16_bits(np.float32(1000.0)), dtype=np.uint16)
        for h in range(heads):
            for t in range(n):
                if t % 17 == 0:
                    x[h * stride + t] = 0 if t % 2 else 0x8000
                else:
                    x[h * stride + t] = inputs.f16_bits(np.float32((int(rng() % 97) - 48) / 2))
        ids, counts, kk, tied = ob.ref_select(x, heads, stride, n, 10.0, 0.2)
        sel[f"t{trial}"] = (inputs.digest(x), kk, tied, inputs.digest(ids.astype(np.uint64)), inputs.digest(counts))
    names = sorted(sel)
    np.savez_compressed(OUT / "select_trials.npz", names=np.array(names),
                        input_digest=np.array([sel[n][0] for n in names]),
                        k=np.array([sel[n][1] for n in names]), tied=np.array([sel[n][2] for n in names]),
                        ids_digest=np.array([sel[n][3] for n in names]),
                        counts_digest=np.array([sel[n][4] for n in names]))

    # ---- 4. pack / union trials (structure of gqa_pack_tests.cpp:15-39)
    pk = {}
    for trial in range(16):
        case = pack_case(trial)
        ids, sizes, positions, rows, payload, slots = case
        k, v, mask = ob.ref_pack(ids, sizes, positions, rows, payload, slots)
        u = ob.ref_union(ids, sizes, len(rows))
        pk[f"t{trial:02d}"] = (inputs.digest(ids, sizes, positions, rows, payload), inputs.digest(k), inputs.digest(v),
                               inputs.digest(mask), inputs.digest(u))
    names = sorted(pk)
    np.savez_compressed(OUT / "pack_trials.npz", names=np.array(names),
                        input_digest=np.array([pk[n][0] for n in names]),
                        k_digest=np.array([pk[n][1] for n in names]), v_digest=np.array([pk[n][2] for n in names]),
                        mask_digest=np.array([pk[n][3] for n in names]),
                        union_digest=np.array([pk[n][4] for n in names]))
    print("fixtures written to", OUT)


def pack_case(trial: int):
    """A seeded pack case: n rows in shuffled physical order, per-head
    shuffled selections (full or truncated), two query positions."""
    rng = inputs.XorShift32(781 + 7919 * trial)
    n = 65 + trial * 4
    slots = (n + 31) // 32 * 32
    rows = np.arange(n, dtype=np.uint64)
    for i in range(n - 1, 0, -1):  # Fisher-Yates with the xorshift stream
        j = rng() % (i + 1)
        rows[i], rows[j] = rows[j], rows[i]
    payload = np.array([rng() & 0xFF for _ in range(n * 4096)], dtype=np.uint8)
    ids = np.zeros((32, n), dtype=np.uint64)
    sizes = np.zeros(32, dtype=np.uint64)
    for h in range(32):
        head = rows.copy()
        for i in range(n - 1, 0, -1):
            j = rng() % (i + 1)
            head[i], head[j] = head[j], head[i]
        size = n if trial % 2 == 0 else 1 + rng() % n
        ids[h, :size] = head[:size]
        sizes[h] = size
    positions = np.array([n // 2, n - 1], dtype=np.uint64)
    return ids, sizes, positions, rows, payload, slots


if __name__ == "__main__":
    main()
