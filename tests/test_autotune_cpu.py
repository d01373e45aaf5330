"""The `.tune` v2 store and the candidate search, on CPU with fake candidates.

Mirrors projects/titan-autotune/src/lib.rs:13-88 (TuneKey/TuneEntry/TuneBudget defaults,
Autotuner open/get/insert/flush, `# titan.tune version=2` header) and the rules of
docs/architecture/autotune-v2.md (exact keys, rejection records, median then p95 within
2%, provisional on budget exhaustion, checksummed canonical JSONL, locked atomic writes)."""
import json
import multiprocessing as mp

import numpy as np
import pytest

from titan_rs_b200 import autotune as A


def key(op="gemm", shape="[8,8],[8,8]->[8,8]"):
    return A.TuneKey(operator=op, device="B200/sm_100/148sm", shape=shape, dtype="BF16,BF16->BF16",
                     layout="[8,1];[8,1]->[8,1];transpose_rhs=1", artifact="abc")


def entry(c="k1", med=100):
    return A.TuneEntry(candidate=c, median_ns=med, p95_ns=med + 5, correctness_hash="h", provisional=False)


def test_budget_defaults_match_the_reference():
    b = A.TuneBudget()
    assert (b.max_candidates, b.warmups, b.samples, b.wall_time) == (32, 3, 9, 2.0)


def test_round_trip_and_canonical_file(tmp_path):
    t = A.Autotuner.open(tmp_path / "kernels")
    assert t.path.name == "kernels.tune"
    t.insert(key(shape="b"), entry("kb", 20))
    t.insert(key(shape="a"), entry("ka", 10))
    t.flush()
    lines = t.path.read_text().splitlines()
    assert lines[0] == A.HEADER
    assert lines[1:] == sorted(lines[1:])
    rec = json.loads(lines[1])
    assert set(rec) == {"key", "entry", "checksum"}
    u = A.Autotuner(tmp_path / "kernels.tune")
    assert u.get(key(shape="a")) == entry("ka", 10)
    assert u.get(key(shape="b")) == entry("kb", 20)
    assert u.get(key(shape="c")) is None
    # Keys are exact: a different artifact identity is a different decision.
    other = A.TuneKey(**{**key(shape="a").__dict__, "artifact": "def"})
    assert u.get(other) is None


def test_tampered_malformed_and_old_version_lines_are_ignored(tmp_path):
    t = A.Autotuner(tmp_path / "x")
    t.insert(key(shape="a"), entry("ka"))
    t.insert(key(shape="b"), entry("kb"))
    t.flush()
    lines = t.path.read_text().splitlines()
    bad = json.loads(lines[1])
    bad["entry"]["candidate"] = "evil"
    lines[1] = json.dumps(bad)
    lines.append("{not json")
    t.path.write_text("\n".join(lines) + "\n")
    u = A.Autotuner(tmp_path / "x")
    assert len(u.entries) == 1 and u.ignored_lines == 2
    t.path.write_text("# titan.tune version=1\n" + "\n".join(lines[1:]) + "\n")
    assert A.Autotuner(tmp_path / "x").entries == {}


def _writer(path, shape, cand):
    t = A.Autotuner(path)
    t.insert(key(shape=shape), entry(cand))
    t.flush()


def test_concurrent_flushes_merge_under_the_lock(tmp_path):
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_writer, args=(str(tmp_path / "m"), f"s{i}", f"k{i}")) for i in range(6)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(30)
        assert p.exitcode == 0
    u = A.Autotuner(tmp_path / "m")
    assert {k.shape: e.candidate for k, e in u.entries.items()} == {f"s{i}": f"k{i}" for i in range(6)}
    assert not (tmp_path / "m.tune.tmp").exists()


def test_selection_median_then_p95_within_two_percent():
    ms = [A.Measured("a", 100, 150, "h"), A.Measured("b", 101, 110, "h"), A.Measured("c", 90, 200, "h")]
    assert A.select(ms).candidate == "c"  # 100 and 101 are not within 2% of 90
    ms = [A.Measured("a", 100, 150, "h"), A.Measured("b", 101, 110, "h"), A.Measured("c", 120, 100, "h")]
    assert A.select(ms).candidate == "b"
    ms = [A.Measured("a", 100, 110, "h", workspace_bytes=64), A.Measured("b", 100, 110, "h", workspace_bytes=0)]
    assert A.select(ms).candidate == "b"


class FakeProblem:
    """Candidates with fixed outputs and timings; 'unsupported' ones raise."""

    def __init__(self, outputs, times, unsupported=()):
        self.outputs, self.times, self.unsupported = outputs, times, set(unsupported)
        self.current = None
        self.timed = []

    def run(self, c):
        if c in self.unsupported:
            raise A.CandidateUnsupported(f"{c} does not take this shape")
        self.current = c

    def read(self):
        return self.outputs[self.current]

    def time_ns(self, c, warmups, samples):
        self.timed.append(c)
        return [self.times[c]] * samples


def test_tune_rejects_with_records_and_picks_the_fastest(tmp_path):
    ref = np.linspace(-1, 1, 64).astype(np.float32)
    fp = FakeProblem({"a": ref, "b": ref + 1e-4, "c": ref + 0.5, "g": ref},
                     {"a": 300, "b": 200, "c": 100, "g": 50}, unsupported={"u"})
    t = A.Autotuner(tmp_path / "t")
    res = t.tune(key(), ["u", "a", "b", "c"], ["g"], fp.run, fp.read, fp.time_ns, 1e-2)
    assert res.entry.candidate == "b" and not res.entry.provisional
    stages = {r.candidate: r.stage for r in res.rejections}
    assert stages == {"u": "capability", "c": "correctness", "g": "selection", "a": "selection"}
    assert "g" not in fp.timed  # the fallback is not timed when a primary candidate takes the problem
    assert t.get(key()) == res.entry and t.tunings == 1


def test_fallback_runs_only_when_no_primary_is_capable(tmp_path):
    ref = np.ones(8, np.float32)
    fp = FakeProblem({"g": ref}, {"g": 10}, unsupported={"a", "b"})
    res = A.Autotuner(tmp_path / "t").tune(key(), ["a", "b"], ["g"], fp.run, fp.read, fp.time_ns, 1e-2)
    assert res.entry.candidate == "g"
    fp = FakeProblem({}, {}, unsupported={"a", "g"})
    with pytest.raises(A.CandidateUnsupported, match="no candidate"):
        A.Autotuner(tmp_path / "t").tune(key(), ["a"], ["g"], fp.run, fp.read, fp.time_ns, 1e-2)


def test_wall_time_budget_marks_the_winner_provisional(tmp_path):
    ref = np.ones(8, np.float32)
    fp = FakeProblem({c: ref for c in "abc"}, {"a": 30, "b": 20, "c": 10})
    res = A.Autotuner(tmp_path / "t").tune(key(), ["a", "b", "c"], [], fp.run, fp.read, fp.time_ns, 1e-2,
                                           A.TuneBudget(wall_time=0.0))
    assert res.entry.provisional and res.entry.candidate == "a"
    assert {r.candidate: r.stage for r in res.rejections} == {"b": "budget", "c": "budget"}


def test_non_finite_output_is_a_correctness_rejection(tmp_path):
    ref = np.ones(4, np.float32)
    fp = FakeProblem({"a": ref, "b": np.array([1, np.nan, 1, 1], np.float32)}, {"a": 5, "b": 1})
    res = A.Autotuner(tmp_path / "t").tune(key(), ["a", "b"], [], fp.run, fp.read, fp.time_ns, 1e-2)
    assert res.entry.candidate == "a"
    assert [(r.candidate, r.stage) for r in res.rejections] == [("b", "correctness")]


def test_every_registered_candidate_is_a_native_kernel_its_operator_accepts():
    """The registry names only kernels that exist in the sm_100a sources and that the
    operator's C entry recognises as a candidate (a typo would surface as a rejection
    at tuning time, never as a wrong kernel)."""
    import pathlib
    import re
    root = pathlib.Path(A.__file__).resolve().parent / "csrc"
    kernels = "\n".join(f.read_text() for f in (root / "kernels").glob("*.cu"))
    # Entries a macro builds by token pasting (e.g. softmax_f32_warp##NV), by invocation.
    pasted = set()
    for macro, param, prefix in re.findall(r"#define (\w+)\((\w+)\)[^\n]*\\\n[^\n]*?(\w+)##\2", kernels):
        pasted.update(prefix + arg for arg in re.findall(rf"^{macro}\((\w+)\)", kernels, re.M))
    host = {"gemm": "op_gemm.cpp", "gemm.bias_act": "op_gemm.cpp", "softmax": "op_softmax.cpp",
            "scaled_dot_product_attention": "op_sdpa.cpp", "conv2d": "op_conv2d.cpp"}
    for (op, _dtype), (primary, fallback) in A.CANDIDATES.items():
        source = (root / "host" / host[op]).read_text()
        for name in primary + fallback:
            assert f'"{name}"' in source, (op, name)
            for kernel in A.COMPOSED.get(name, (name,)):
                assert kernel in pasted or re.search(rf"\b{re.escape(kernel)}\s*[(,]", kernels), (op, name, kernel)
