"""The native `.tune` version 2 store (tb_tune_* in libtitan_b200.so), on CPU.

The file rules follow projects/titan-autotune/src/lib.rs:46-82 and
docs/architecture/autotune-v2.md:9. Python's hashlib and json modules are the oracles
for the store's SHA-256 and canonical JSON: a file written by either side must be
byte-identical to what the other would write."""
import hashlib
import json
import math
import random

import pytest
from hypothesis import given, settings
from hypothesis import strategies as st

from titan_rs_b200 import _native as N
from titan_rs_b200 import autotune as A


def py_canonical(obj) -> str:
    return json.dumps(obj, sort_keys=True, separators=(",", ":"))


def py_row(key: dict, entry: dict) -> str:
    """One record line as the v2 rules define it, written with the standard library."""
    body = {"key": key, "entry": entry}
    return py_canonical({**body, "checksum": hashlib.sha256(py_canonical(body).encode()).hexdigest()})


@pytest.mark.parametrize("n", [0, 1, 3, 55, 56, 57, 63, 64, 65, 119, 120, 127, 128, 129, 1000])
def test_sha256_matches_hashlib(n):
    data = bytes(random.Random(n).getrandbits(8) for _ in range(n))
    assert N.sha256_hex(data) == hashlib.sha256(data).hexdigest()


def test_sha256_of_a_megabyte():
    data = random.Random(7).randbytes(1 << 20)
    assert N.sha256_hex(data) == hashlib.sha256(data).hexdigest()


json_scalars = (st.none() | st.booleans() | st.integers(min_value=-(10 ** 30), max_value=10 ** 30)
                | st.floats(allow_nan=True, allow_infinity=True) | st.text())
json_values = st.recursive(json_scalars, lambda inner: st.lists(inner, max_size=4)
                           | st.dictionaries(st.text(), inner, max_size=4), max_leaves=20)


@settings(max_examples=400, deadline=None)
@given(json_values, st.sampled_from([None, 1, 2]), st.booleans())
def test_canonical_json_matches_python(value, indent, ascii_only):
    text = json.dumps(value, indent=indent, ensure_ascii=ascii_only)
    assert N.canonical_json(text) == py_canonical(json.loads(text))


@pytest.mark.parametrize("x", [0.0, -0.0, 1.0, 0.1, 1e-4, 1e-5, 123456789012345.6, 1234567890123456.0, 1e16,
                               1e22, 5e-324, 1.7976931348623157e308, 2.5e-7, 100.0, 3.14159])
def test_float_repr_matches_python(x):
    assert N.canonical_json(json.dumps([x, -x])) == py_canonical([x, -x])


def test_random_doubles_match_python_repr():
    rng = random.Random(3)
    xs = [rng.uniform(-1, 1) * 10 ** rng.randint(-320, 308) for _ in range(3000)]
    xs = [x for x in xs if math.isfinite(x)]
    assert N.canonical_json(json.dumps(xs)) == py_canonical(xs)


@pytest.mark.parametrize("text", ['"\\ud800"', '"\\ud83d\\ude00"', '"\\ud83d\\u0041"', '"a\\/b"', '-0', '1E5',
                                  '{"b":1,"a":{"d":[],"c":{}},"b":2}', ' [ 1 , 2 ] ', '"\\u00e9\x7f"',
                                  'NaN', '-Infinity', '"tab\\there"'])
def test_canonical_edge_cases_match_python(text):
    assert N.canonical_json(text) == py_canonical(json.loads(text))


@pytest.mark.parametrize("text", ['', '{', '[1,]', '{"a" 1}', '01', '1.', '"\x01"', '"\\x"', '"\\u12"', 'nul',
                                  '{"a":1} x', "'a'", '\ufeff{}', '[1e]'])
def test_canonical_rejects_what_python_rejects(text):
    with pytest.raises(json.JSONDecodeError):
        json.loads(text)
    with pytest.raises(ValueError):
        N.canonical_json(text)


def test_file_written_by_the_standard_library_is_read_and_rewritten_identically(tmp_path):
    path = tmp_path / "k.tune"
    keys = [{"operator": "gemm", "shape": f"[{i}]", "device": "B200 \u00b5", "n": i} for i in range(5)]
    entries = [{"candidate": f"c{i}", "median_ns": 10 * i, "provisional": i % 2 == 0, "ratio": i / 7} for i in range(5)]
    rows = sorted(py_row(k, e) for k, e in zip(keys, entries))
    text = A.HEADER + "\n" + "\n".join(rows) + "\n"
    path.write_text(text)
    store = N.TuneStore(path)
    assert store.stats() == (5, 0)
    assert json.loads(store.get(json.dumps(keys[3], indent=1))) == entries[3]
    assert store.get('{"operator":"softmax"}') is None
    store.flush()
    assert path.read_text() == text
    assert not (tmp_path / "k.tune.tmp").exists()


def test_store_merges_with_disk_and_its_own_records_win(tmp_path):
    path = tmp_path / "m.tune"
    a, b = N.TuneStore(path), N.TuneStore(path)
    a.insert('{"k":1}', '{"v":"a1"}')
    a.insert('{"k":2}', '{"v":"a2"}')
    a.flush()
    b.insert('{"k":2}', '{"v":"b2"}')
    b.insert('{"k":3}', '{"v":"b3"}')
    b.flush()
    assert dict(b.records()) == {'{"k":1}': '{"v":"a1"}', '{"k":2}': '{"v":"b2"}', '{"k":3}': '{"v":"b3"}'}
    lines = path.read_text().splitlines()
    assert lines[0] == A.HEADER and lines[1:] == sorted(lines[1:])
    for line in lines[1:]:
        rec = json.loads(line)
        assert line == py_row(rec["key"], rec["entry"])


def test_rejected_lines_are_counted_and_dropped(tmp_path):
    path = tmp_path / "r.tune"
    good = py_row({"k": 1}, {"v": 1})
    tampered = json.loads(py_row({"k": 2}, {"v": 2}))
    tampered["entry"]["v"] = 3
    lines = [A.HEADER, good, json.dumps(tampered), "{not json", "[1, 2]", '{"key": {"k": 4}, "entry": {}}',
             json.dumps({"key": [4], "entry": {}, "checksum": "0" * 64}), "   ", ""]
    path.write_text("\n".join(lines) + "\n")
    store = N.TuneStore(path)
    assert store.stats() == (1, 5)
    store.flush()
    assert path.read_text() == A.HEADER + "\n" + good + "\n"
    assert store.stats() == (1, 5)  # the count is of the file as last read


def test_other_headers_and_non_utf8_files_contribute_nothing(tmp_path):
    path = tmp_path / "h.tune"
    row = py_row({"k": 1}, {"v": 1})
    path.write_text("# titan.tune version=1\n" + row + "\n")
    assert N.TuneStore(path).stats() == (0, 2)
    path.write_bytes((A.HEADER + "\n" + row + "\n").encode() + b"\xff\n")
    assert N.TuneStore(path).stats() == (0, 0)
    path.write_text("\r\n".join([" " + A.HEADER + "\t", row]))  # CRLF and padded header still read
    assert N.TuneStore(path).stats() == (1, 0)


def test_records_of_another_schema_survive_a_python_flush(tmp_path):
    """A record with fields TuneKey does not know is ignored by the Python host but kept."""
    path = tmp_path / "s.tune"
    foreign = py_row({"operator": "gemm", "tile": [2, 1]}, {"candidate": "x"})
    path.write_text(A.HEADER + "\n" + foreign + "\n")
    t = A.Autotuner(path)
    assert t.entries == {} and t.ignored_lines == 1
    k = A.TuneKey(operator="gemm", device="d", shape="s", dtype="BF16", layout="l")
    t.insert(k, A.TuneEntry("c", 1, 2, "h", False))
    t.flush()
    assert foreign in path.read_text().splitlines()
    assert A.Autotuner(path).get(k) == A.TuneEntry("c", 1, 2, "h", False)


def test_flush_reports_file_system_errors(tmp_path):
    (tmp_path / "file").write_text("x")
    store = N.TuneStore(tmp_path / "file" / "sub" / "t.tune")
    store.insert("{}", "{}")
    with pytest.raises(OSError, match="create directory"):
        store.flush()


def test_arguments_must_be_json_objects(tmp_path):
    store = N.TuneStore(tmp_path / "a.tune")
    with pytest.raises(ValueError, match="key is not a JSON object"):
        store.insert("[1]", "{}")
    with pytest.raises(ValueError, match="entry is not a JSON object"):
        store.insert("{}", "{oops")


@settings(max_examples=300, deadline=None)
@given(st.lists(st.tuples(st.sampled_from(["a", "b", "c", "gemm_bf16_tn", "gemm_bf16_tn_2sm"]),
                          st.integers(1, 200), st.integers(1, 300), st.sampled_from([0, 64, 4096])),
                min_size=1, max_size=8))
def test_native_selection_rule_matches_its_statement(rows):
    """tb_tune_select against the rule written out: lowest median; within 2% of it the
    lower p95, then the smaller workspace, then the name."""
    ms = [A.Measured(c, med, p95, "h", ws) for c, med, p95, ws in rows]
    best = min(m.median_ns for m in ms)
    want = min((m for m in ms if m.median_ns <= best * 1.02), key=lambda m: (m.p95_ns, m.workspace_bytes, m.candidate))
    got = A.select(ms)
    assert (got.candidate, got.median_ns, got.p95_ns, got.workspace_bytes) == \
        (want.candidate, want.median_ns, want.p95_ns, want.workspace_bytes)
