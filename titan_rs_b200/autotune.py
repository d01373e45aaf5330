"""Operator tuning: exact-shape keys, candidate evaluation, and the versioned `.tune` store.

Mirrors projects/titan-autotune/src/lib.rs:13-88 (`TuneKey`, `TuneEntry`, `TuneBudget`,
`Autotuner::{open, get, insert, flush}`, `measure`) and follows the v2 rules of
docs/architecture/autotune-v2.md that the reference specifies but does not implement:

* keys are exact: operator, device fingerprint, shapes, strides, dtypes, layout and
  semantic attributes, strategy version, workspace policy, precision, determinism and
  the identity of the kernel library;
* candidates go through capability -> workspace -> correctness -> benchmark ->
  selection in that order, and every candidate that fails a stage leaves a
  `Rejection` record (no silent fallback);
* kernels are timed with CUDA events on the launching stream after warm-ups, so
  module loads, uploads, downloads and device synchronisation are not counted;
* the winner has the lowest median; within 2% of it the lower p95, then the smaller
  workspace, then the name decide. When the wall-time budget runs out, the best
  verified candidate so far wins and is marked provisional;
* the file is a `# titan.tune version=2` header plus canonical JSON lines, each with
  a SHA-256 checksum of its record; writes take an exclusive lock, merge with the
  records on disk, go to a temporary file that is fsynced, are renamed atomically,
  and fsync the directory. Malformed, tampered or old-version lines are ignored.
  A cache hit neither compiles nor benchmarks. The store itself is native
  (tb_tune_* in libtitan_b200.so), so Rust and C hosts share the same file.
"""
from __future__ import annotations

import ctypes
import hashlib
import json
import math
import pathlib
import time
from dataclasses import asdict, dataclass, field
from typing import Callable, Iterable, Optional, Sequence

import numpy as np

from . import _native

HEADER = "# titan.tune version=2"
STRATEGY_VERSION = 1

# Registered kernels per operator and input dtype, in preference order: the first
# capable one is the correctness baseline. Fallbacks are only tried when no direct
# tensor-core candidate takes the problem (they are slower by design, and timing them
# on large problems would spend the tuning budget for nothing): the staged GEMM (operands
# copied K-major, then the tensor cores) and the CUDA-core kernels.
CANDIDATES = {
    ("gemm", "BF16"): (["gemm_bf16_tn_2sm", "gemm_bf16_tn", "gemm_bf16_tn_splitk", "gemm_bf16_nn_2sm",
                        "gemm_bf16_ta_2sm", "gemm_bf16_ta_nn_2sm"], ["gemm_bf16_staged", "gemm_bf16_generic"]),
    ("gemm", "F32"): (["gemm_f32_tiled"], []),
    ("softmax", "F32"): (["softmax_f32_warp1", "softmax_f32_warp2", "softmax_f32_warp4", "softmax_f32_warp8",
                          "softmax_f32_warp16", "softmax_f32_warp32", "softmax_f32_stream"], []),
    ("scaled_dot_product_attention", "BF16"): (["sdpa_fwd_bf16_d128_pair", "sdpa_fwd_bf16_d128_bn64",
                                                 "sdpa_fwd_bf16_d128"], ["sdpa_bf16_generic"]),
    ("softmax", "BF16"): (["softmax_bf16_rows"], []),
    ("conv2d", "BF16"): (["conv2d_fprop_bf16_nhwc_2sm", "conv2d_fprop_bf16_nhwc"], ["conv2d_bf16_nhwc_generic"]),
    ("conv2d", "F32"): (["conv2d_f32"], []),
    ("gemm.bias_act", "BF16"): (["gemm_bf16_tn_bias_act_2sm", "gemm_bf16_tn_bias_act", "gemm_bf16_nn_2sm",
                                 "gemm_bf16_ta_2sm", "gemm_bf16_ta_nn_2sm"], ["gemm_bf16_staged"]),
}

# Candidates that are a sequence of launches rather than one kernel, with their kernels.
COMPOSED = {
    "gemm_bf16_staged": ("stage_bf16_pad_rows", "unstage_bf16_rows", "gemm_bf16_tn_2sm", "gemm_bf16_tn",
                         "gemm_bf16_nn_2sm", "gemm_bf16_ta_2sm", "gemm_bf16_ta_nn_2sm", "gemm_bf16_tn_bias_act_2sm",
                         "gemm_bf16_tn_bias_act"),
}

# Correctness bar against the baseline candidate: |got - ref| <= tol * max|ref|.
TOLERANCE = {"BF16": 1e-2, "F32": 1e-5}


@dataclass(frozen=True)
class TuneKey:
    """Exact identity of an operator tuning decision (TuneKey, lib.rs:13-21, plus the v2 fields)."""
    operator: str
    device: str
    shape: str
    dtype: str
    layout: str
    strategy_version: int = STRATEGY_VERSION
    precision: str = "fp32-accumulate"
    determinism: str = "bitwise-repeatable"
    workspace_policy: str = "stream-scratch"
    artifact: str = ""


@dataclass
class TuneEntry:
    """Persisted winner and evidence (TuneEntry, lib.rs:23-31)."""
    candidate: str
    median_ns: int
    p95_ns: int
    correctness_hash: str
    provisional: bool
    workspace_bytes: int = 0


@dataclass(frozen=True)
class TuneBudget:
    """Bounded synchronous tuning budget (TuneBudget, lib.rs:33-45; same defaults)."""
    max_candidates: int = 32
    warmups: int = 3
    samples: int = 9
    wall_time: float = 2.0


@dataclass
class Rejection:
    candidate: str
    stage: str   # capability | workspace | correctness | benchmark | budget | selection
    reason: str


@dataclass
class Measured:
    candidate: str
    median_ns: int
    p95_ns: int
    correctness_hash: str
    workspace_bytes: int = 0


@dataclass
class TuneResult:
    entry: TuneEntry
    rejections: list = field(default_factory=list)
    measured: list = field(default_factory=list)


def measure(operation: Callable[[], None]) -> float:
    """Host wall time of a synchronous operation in seconds (measure, lib.rs:84-88)."""
    t0 = time.perf_counter()
    operation()
    return time.perf_counter() - t0


def _canonical(obj) -> str:
    return json.dumps(obj, sort_keys=True, separators=(",", ":"))


def _percentile(sorted_vals: Sequence[float], q: float) -> float:
    """Nearest-rank percentile of an ascending sequence."""
    k = max(0, min(len(sorted_vals) - 1, math.ceil(q * len(sorted_vals)) - 1))
    return sorted_vals[k]


def select(measured: Sequence[Measured]) -> Measured:
    """Lowest median; within 2% of it: lower p95, then smaller workspace, then name
    (the native rule, tb_tune_select)."""
    names = [m.candidate.encode() for m in measured]
    arr = (_native.TuneMeasurement * len(measured))(
        *[_native.TuneMeasurement(nm, int(m.median_ns), int(m.p95_ns), int(m.workspace_bytes))
          for nm, m in zip(names, measured)])
    w = ctypes.c_size_t(0)
    if _native.lib().tb_tune_select(arr, len(measured), ctypes.byref(w)) != _native.TB_OK:
        raise ValueError(_native.last_error()[1])
    return measured[w.value]


class Autotuner:
    """Version 2 `.tune` store (Autotuner, lib.rs:46-82) over the native store (tb_tune_*).

    The native library owns the file: parsing, checksums, canonical JSON, the lock, the
    merge and the atomic write. This class maps its canonical records to `TuneKey` and
    `TuneEntry`; a record that passed the native checks but whose fields these classes do
    not take is counted in `ignored_lines` and left in the file for the host that wrote it."""

    def __init__(self, path):
        p = pathlib.Path(path)
        self.path = p.with_suffix(".tune")
        self.tunings = 0  # candidate searches run by this object (a cache hit runs none)
        self._store = _native.TuneStore(self.path)
        self._foreign = 0
        self.entries: dict[TuneKey, TuneEntry] = self._decode()

    @classmethod
    def open(cls, path) -> "Autotuner":
        return cls(path)

    # ---- persistence ----
    @property
    def ignored_lines(self) -> int:
        """Lines the last read of the file skipped, plus records of another schema."""
        return self._store.stats()[1] + self._foreign

    def _decode(self) -> dict:
        entries: dict[TuneKey, TuneEntry] = {}
        self._foreign = 0
        for k, e in self._store.records():
            try:
                entries[TuneKey(**json.loads(k))] = TuneEntry(**json.loads(e))
            except TypeError:
                self._foreign += 1
        return entries

    def get(self, key: TuneKey) -> Optional[TuneEntry]:
        return self.entries.get(key)

    def insert(self, key: TuneKey, entry: TuneEntry) -> None:
        self.entries[key] = entry
        self._store.insert(_canonical(asdict(key)), _canonical(asdict(entry)))

    def flush(self) -> None:
        """Merges with the file under an exclusive lock and replaces it atomically."""
        for k, e in self.entries.items():
            self._store.insert(_canonical(asdict(k)), _canonical(asdict(e)))
        self._store.flush()
        self.entries = self._decode()

    # ---- search ----
    def tune(self, key: TuneKey, primary: Sequence[str], fallback: Sequence[str],
             run: Callable[[str], None], read_output: Callable[[], np.ndarray],
             time_ns: Callable[[str, int, int], list], tolerance: float,
             budget: TuneBudget = TuneBudget(), workspace_bytes: Callable[[str], int] = lambda c: 0) -> TuneResult:
        """Evaluates candidates and records the winner.

        run(c) launches candidate c once (raising `CandidateUnsupported` when the kernel
        does not take the problem); read_output() returns the output as float32 after the
        last run; time_ns(c, warmups, samples) returns per-launch device times in ns."""
        self.tunings += 1
        t0 = time.perf_counter()
        result = TuneResult(entry=None)
        baseline = None
        out_of_time = False

        def evaluate(names: Iterable[str]) -> None:
            nonlocal baseline, out_of_time
            for name in names:
                if len(result.measured) >= budget.max_candidates:
                    result.rejections.append(Rejection(name, "budget", "max_candidates reached"))
                    continue
                if out_of_time:
                    result.rejections.append(Rejection(name, "budget", "wall-time budget exhausted"))
                    continue
                try:
                    run(name)
                except CandidateUnsupported as e:
                    result.rejections.append(Rejection(name, "capability", str(e)))
                    continue
                ws = workspace_bytes(name)
                out = np.asarray(read_output(), dtype=np.float32)
                digest = hashlib.sha256(out.tobytes()).hexdigest()
                if not np.isfinite(out).all():
                    result.rejections.append(Rejection(name, "correctness", "non-finite output"))
                    continue
                if baseline is None:
                    baseline = out
                else:
                    scale = float(np.max(np.abs(baseline))) or 1.0
                    err = float(np.max(np.abs(out - baseline))) / scale
                    if err > tolerance:
                        result.rejections.append(
                            Rejection(name, "correctness", f"max|err| {err:.3e} x max|ref| > {tolerance:g}"))
                        continue
                times = sorted(time_ns(name, budget.warmups, budget.samples))
                result.measured.append(Measured(name, int(_percentile(times, 0.5)), int(_percentile(times, 0.95)),
                                                digest, ws))
                if time.perf_counter() - t0 > budget.wall_time:
                    out_of_time = True

        evaluate(primary)
        if not result.measured:
            evaluate(fallback)
        else:
            for name in fallback:
                result.rejections.append(Rejection(name, "selection", "CUDA-core fallback; a tensor-core "
                                                                       "candidate takes this problem"))
        if not result.measured:
            raise CandidateUnsupported(f"no candidate takes {key.operator} {key.shape}: "
                                       + "; ".join(f"{r.candidate}: {r.reason}" for r in result.rejections))
        win = select(result.measured)
        for m in result.measured:
            if m is not win:
                result.rejections.append(Rejection(m.candidate, "selection",
                                                   f"median {m.median_ns} ns vs {win.median_ns} ns"))
        result.entry = TuneEntry(win.candidate, win.median_ns, win.p95_ns, win.correctness_hash,
                                 provisional=out_of_time, workspace_bytes=win.workspace_bytes)
        self.insert(key, result.entry)
        return result


class CandidateUnsupported(RuntimeError):
    """A candidate kernel does not take the problem (TB_ERR_UNSUPPORTED from the operator)."""


def library_identity() -> str:
    """SHA-256 prefix of the loaded kernel library (the artifact a tune decision belongs to)."""
    from . import _native as N
    path = N.LIB_PATH
    if not path.exists():
        return "unknown"
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for chunk in iter(lambda: f.read(1 << 20), b""):
            h.update(chunk)
    return h.hexdigest()[:16]


__all__ = ["HEADER", "STRATEGY_VERSION", "CANDIDATES", "TOLERANCE", "TuneKey", "TuneEntry", "TuneBudget",
           "Rejection", "Measured", "TuneResult", "Autotuner", "CandidateUnsupported", "measure", "select",
           "library_identity"]
