"""Benchmark of the titan.rs operator hot path on B200 (one process per GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--op gemm|softmax|sdpa|conv2d] [--impl ours|reference]

Prints ONE JSON line (rank 0). Workloads are the BASELINE.json configurations:
  gemm    C3  bf16 A[8192,8192] row-major x B column-major, fp32 accumulate, bf16 C (TFLOP/s);
              N>1: B is N-sharded and C re-assembled with an all-gather (strong scaling).
  softmax C2  fp32 [32768, 4096] row softmax, N(0, 2^2), seed 1 (GB/s; replicas at N>1).
  sdpa    C4  causal bf16 B8 H32 S4096 D128 (TFLOP/s, causal-halved FLOPs); B*H-sharded at N>1.
  conv2d  C5  bf16 NHWC 64x56x56x256 -> 256, 3x3 s1 p1 (TFLOP/s); batch-sharded at N>1.
Inputs are seeded synthetic data (no dataset exists for this path).

`value` is the device-timed whole-job throughput with inputs resident in HBM;
`e2e` is the same metric through the public API with pinned-host inputs copied in and
the result copied out inside every timed step: at N=1 the GEMM and attention through
titan_rs_b200.streaming (blocks uploaded, computed and downloaded overlapped), otherwise
whole-tensor copies around the operator with steps pipelined over two streams (one
step's upload overlaps the previous step's download); `e2e.path` names which.
`--impl reference` times the CPU
restatement of the reference's scalar operator (oracle/) on the host cores; it never
loads the product library (its inputs come from the oracle's copy of the generator).

The headline line is `--op` (default gemm, C3). With `--ops` (default: the other three
configs when `--op` is gemm) the same run measures C2, C4 and C5 the same way and
reports them under "ops", each with value, ms_per_step, roofline, e2e and, at N=1,
cpu_baseline; "ops" also holds C1, the reference's own CPU configuration (f32 256^3),
timed on the host at one thread and at all threads beside the f32 kernel on the GPU
(launched from the host, and replayed from a CUDA graph).
"""
from __future__ import annotations

import argparse
import json
import math
import os
import pathlib
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

PEAK_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def load_peaks() -> tuple[dict, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return json.loads(p.read_text()), "measured"
        except Exception:
            pass
    return dict(PEAK_FALLBACK), "fallback"


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    """Samples nvidia-smi during the timed region (SM clock, max clock, throttle reasons)."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu_index = gpu_index
        self.proc = None
        self.lines: list[str] = []
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu_index}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (FileNotFoundError, OSError):
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        sm, smax, power, reasons = [], [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            try:
                power.append(float(parts[3]))
            except ValueError:
                pass
            for name, flag in zip(names, parts[5:9]):
                if flag.lower() == "active":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(smax), "reasons": sorted(reasons),
                "samples": len(sm), "power_w": statistics.median(power) if power else None}


# ----------------------------------------------------------------------------- workloads
def workload_config(op: str, world: int, small: bool = False) -> dict:
    """The `config` object of a bench line; both arms print the same dict for the same run."""
    if op == "softmax":
        rows = 16384 if small else 32768
        return {"workload": "C2 row softmax fp32 [32768,4096], x~N(0,2^2) seed 1", "rows": rows, "cols": 4096,
                "parallelism": f"replicas{world}", "l2": f"inputs {rows * 4096 * 4 // 2**20} MiB > 126 MB L2"}
    if op == "gemm":
        m = 4096 if small else 8192
        cfg = {"workload": f"C3 bf16 GEMM M=N=K={m}, A row-major N(0,1), B column-major N(0,1/K), seed 2",
               "M": m, "N": m, "K": m, "parallelism": f"N-shard{world}" if world > 1 else "single",
               "l2": f"inputs {2 * m * m * 2 // 2**20} MiB > 126 MB L2"}
        if world > 1:
            p2p = os.environ.get("TITAN_B200_ALLGATHER", "p2p") == "p2p"
            cfg["allgather"] = ("fused GEMM + all-gather kernel: NVLink peer stores into registered C (CTA pairs "
                                "with push warps; from 4 ranks, dedicated pusher CTAs: gemm_bf16_tn_allgather_2sm_push)"
                                if p2p else "NCCL all-gather + re-layout kernel")
        return cfg
    if op == "sdpa":
        b = 2 if small else 8
        return {"workload": f"C4 causal SDPA fwd bf16 B{b} H32 S4096 D128, N(0,1) seed 3, "
                            "scale 1/sqrt(128), FLOPs = 4*B*H*S^2*D/2",
                "B": b, "H": 32, "S": 4096, "D": 128,
                "parallelism": f"bh-shard{world}" if world > 1 else "single",
                "l2": f"inputs {3 * b * 32 * 4096 * 128 * 2 // world // 2**20} MiB per GPU vs 126 MB L2"}
    if op == "conv2d":
        n = 16 if small else 64
        return {"workload": f"C5 conv2d fwd bf16 NHWC N{n} 56x56 Cin256 Cout256 3x3 s1 p1, "
                            "x N(0,1), w N(0,2/2304), seed 4",
                "N": n, "H": 56, "W": 56, "Cin": 256, "Cout": 256, "R": 3, "S": 3,
                "parallelism": f"batch-shard{world}" if world > 1 else "single",
                "l2": f"3 rotating input/output pairs ({3 * 2 * n * 56 * 56 * 256 * 2 // world // 2**20} MiB "
                      "working set per GPU > 126 MB L2)"}
    raise ValueError(op)


class Workload:
    """One hot-path op at one configuration, on one rank."""
    name = ""
    metric = ""
    unit = ""
    dtype = ""
    scaling = "weak"
    bound = "hbm"
    flush_l2 = False

    def __init__(self, tb, session, stream, rank: int, world: int, comm=None, small: bool = False):
        self.tb, self.s, self.st, self.rank, self.world, self.comm = tb, session, stream, rank, world, comm
        self.small = small

    # work per step on this rank, in the metric's unit base (bytes or FLOPs)
    def units_per_step(self) -> float:
        raise NotImplementedError

    def job_units_per_step(self) -> float:
        return self.units_per_step() * self.world

    def step(self):
        raise NotImplementedError

    def e2e_upload(self, stream):
        raise NotImplementedError

    def e2e_download(self, stream):
        raise NotImplementedError

    # A workload whose public API streams host operands through the GPU (upload,
    # compute and download overlapped inside a step) sets this to a callable
    # (stream, after_event_or_None) -> None that enqueues one such step.
    e2e_streamed = None

    def h2d_bytes(self) -> int:
        raise NotImplementedError

    def d2h_bytes(self) -> int:
        raise NotImplementedError

    def config(self) -> dict:
        raise NotImplementedError

    def cpu_sample(self, budget_s: float) -> dict:
        raise NotImplementedError


def _tensor(tb, buf, dtype, shape):
    from titan_rs_b200.runtime import c_tensor, contiguous_strides
    return c_tensor(buf, dtype, shape, contiguous_strides(shape))


class SoftmaxWorkload(Workload):
    name = "softmax"
    metric = "row softmax fp32 [32768,4096] HBM throughput per B200"
    unit = "GB/s"
    dtype = "f32"
    scaling = "weak"
    bound = "hbm"
    rows, cols = 32768, 4096

    def __init__(self, *a, **k):
        super().__init__(*a, **k)
        import ctypes
        from titan_rs_b200 import _native as N
        from titan_rs_b200.kernel_abi import DType
        self.N, self.ctypes, self.DType = N, ctypes, DType
        if self.small:
            self.rows = 16384  # 256 MiB input: still larger than L2, for ncu captures
        n = self.rows * self.cols
        self.nbytes = n * 4
        self.host_in = self.s.host_alloc(self.nbytes)
        self.host_out = self.s.host_alloc(self.nbytes)
        x = self.host_in.array(np.float32, (self.rows, self.cols))
        x[:] = self.tb.fill_normal(n, seed=1, mean=0.0, std=2.0).reshape(self.rows, self.cols)
        self.x_host = x
        self.din = self.s.allocate(self.nbytes)
        self.dout = self.s.allocate(self.nbytes)
        self.s.upload_pinned(self.st, self.din, self.host_in)
        self.s.synchronize(self.st)
        self.tin = _tensor(self.tb, self.din, DType.F32, (self.rows, self.cols))
        self.tout = _tensor(self.tb, self.dout, DType.F32, (self.rows, self.cols))
        self.kernel = "softmax_f32_warp32"

    def units_per_step(self):
        return 2.0 * self.nbytes  # read x once, write y once

    def step(self):
        rc = self.N.lib().tb_op_softmax(self.s.ptr, self.st.ptr, self.ctypes.byref(self.tin),
                                        self.ctypes.byref(self.tout), None, 0, None)
        if rc:
            raise RuntimeError(self.N.last_error())

    def e2e_upload(self, stream):
        self.s.upload_pinned(stream, self.din, self.host_in)

    def e2e_download(self, stream):
        self.s.download_pinned(stream, self.dout, self.host_out)

    def h2d_bytes(self):
        return self.nbytes

    def d2h_bytes(self):
        return self.nbytes

    def config(self):
        return workload_config(self.name, self.world, self.small)

    def cpu_sample(self, budget_s, threads=0):
        import oracle
        threads = threads or oracle.cpu_count()
        rows = 256
        t0 = time.perf_counter()
        done = 0
        while True:
            r0 = (done * rows) % self.rows
            oracle.softmax_rows_mt(self.x_host[r0:r0 + rows], threads)
            done += 1
            if time.perf_counter() - t0 > budget_s:
                break
        dt = time.perf_counter() - t0
        gbs = done * rows * self.cols * 8 / dt / 1e9
        return {"value": gbs, "unit": "GB/s", "cores": threads, "kind": "port",
                "sample": f"{done * rows} rows of the [32768,4096] tensor ({done} x {rows}-row chunks), "
                          f"{dt:.1f} s on {threads} threads"}


def tensor_seed(config_seed: int, index: int) -> int:
    """Seed of the index-th input tensor of a configuration (A=0, B=1; Q=0, K=1, V=2; x=0, w=1)."""
    return config_seed * 16 + index


class GemmWorkload(Workload):
    name = "gemm"
    metric = "bf16 GEMM 8192^3 (A row-major x B column-major, fp32 accumulate) TFLOP/s per B200"
    unit = "TFLOP/s"
    dtype = "bf16"
    scaling = "strong"
    bound = "tensor"
    M = N = K = 8192

    def __init__(self, *a, **k):
        super().__init__(*a, **k)
        import ctypes
        from titan_rs_b200 import _native as N
        from titan_rs_b200.kernel_abi import DType
        self.Nn, self.ctypes, self.DType = N, ctypes, DType
        if self.small:
            self.M = self.N = self.K = 4096
        M, Nn, K = self.M, self.N, self.K
        from titan_rs_b200.distributed import even_shard
        from titan_rs_b200.runtime import TensorHandle, contiguous_strides
        lo, hi = even_shard(Nn, self.world, self.rank)  # this rank's output columns / rows of B's [N,K] storage
        self.n_local = hi - lo
        self.a_bytes, self.b_bytes, self.c_bytes = M * K * 2, self.n_local * K * 2, M * Nn * 2
        self.host_a = self.s.host_alloc(self.a_bytes)
        self.host_b = self.s.host_alloc(self.b_bytes)
        self.host_c = self.s.host_alloc(self.c_bytes)
        self.a_bits = self.host_a.array(np.uint16, (M, K))
        self.b_bits = self.host_b.array(np.uint16, (self.n_local, K))
        self.a_bits[:] = self.tb.fill_normal(M * K, seed=tensor_seed(2, 0), std=1.0, dtype=DType.BF16).reshape(M, K)
        self.b_bits[:] = self.tb.fill_normal(hi * K, seed=tensor_seed(2, 1), std=1.0 / math.sqrt(K),
                                             dtype=DType.BF16)[lo * K:].reshape(self.n_local, K)
        self.da = self.s.allocate(self.a_bytes)
        self.db = self.s.allocate(self.b_bytes)
        self.dc = self.s.allocate(self.c_bytes)
        self.s.upload_pinned(self.st, self.da, self.host_a)
        self.s.upload_pinned(self.st, self.db, self.host_b)
        self.s.synchronize(self.st)
        self.ta = _tensor(self.tb, self.da, DType.BF16, (M, K))
        self.tbm = _tensor(self.tb, self.db, DType.BF16, (self.n_local, K))
        self.tc = _tensor(self.tb, self.dc, DType.BF16, (M, Nn))
        # N > 1: "p2p" (default) = one fused kernel storing this rank's columns into every
        # rank's registered C over NVLink; "nccl" = GEMM into slot `rank` of a [p][M][N/p]
        # gather buffer, NCCL all-gather, re-layout kernel.
        self.allgather = os.environ.get("TITAN_B200_ALLGATHER", "p2p")
        if self.allgather not in ("p2p", "nccl"):
            raise SystemExit("TITAN_B200_ALLGATHER must be p2p or nccl")
        if self.world > 1:
            self.dws = self.s.allocate(self.c_bytes) if self.allgather == "nccl" else None
            self.dc_local = self.s.allocate(M * self.n_local * 2)
            self.tc_local = _tensor(self.tb, self.dc_local, DType.BF16, (M, self.n_local))
            self.h_a = TensorHandle(self.s, self.da, DType.BF16, (M, K), contiguous_strides((M, K)))
            self.h_b = TensorHandle(self.s, self.db, DType.BF16, (self.n_local, K),
                                    contiguous_strides((self.n_local, K)))
            self.h_c = TensorHandle(self.s, self.dc, DType.BF16, (M, Nn), contiguous_strides((M, Nn)))
            if self.allgather == "p2p":
                self.comm.register_buffer(self.st, self.dc)  # collective: every rank maps every rank's C
        # Optional kernel choice for the single-GPU GEMM (an operator candidate name);
        # unset, the operator picks its default kernel.
        cand = os.environ.get("TITAN_B200_GEMM_CANDIDATE", "")
        self.attrs = (N.Attr * 2)()
        self.n_attrs = 2 if cand else 1
        self._key, self._ckey, self._cval = b"transpose_rhs", b"candidate", cand.encode()
        self.attrs[0].key = self._key
        self.attrs[0].value = 1
        self.attrs[1].key = self._ckey
        self.attrs[1].str = self._cval
        self.kernel = cand or "gemm_bf16_tn_2sm"  # the operator's choice at 8192^3

    def units_per_step(self):
        return 2.0 * self.M * self.n_local * self.K

    def _local_gemm(self, out_tensor):
        rc = self.Nn.lib().tb_op_gemm(self.s.ptr, self.st.ptr, self.ctypes.byref(self.ta), self.ctypes.byref(self.tbm),
                                      self.ctypes.byref(out_tensor), self.attrs, self.n_attrs, None)
        if rc:
            raise RuntimeError(self.Nn.last_error())

    def step(self):
        if self.world == 1:
            self._local_gemm(self.tc)
        else:
            self.comm.sharded_gemm(self.st, self.h_a, self.h_b, self.h_c, self.dws)

    def dominant_kernel_ms(self, session, stream, steps):
        """Average duration of the GEMM kernel alone (the compute phase of a step)."""
        if self.world == 1:
            return None
        for _ in range(3):
            self._local_gemm(self.tc_local)
        e0 = session.record(stream)
        for _ in range(steps):
            self._local_gemm(self.tc_local)
        e1 = session.record(stream)
        session.synchronize(stream)
        return session.elapsed_ms(e0, e1) / steps

    def e2e_upload(self, stream):
        self.s.upload_pinned(stream, self.da, self.host_a)
        self.s.upload_pinned(stream, self.db, self.host_b)

    def e2e_download(self, stream):
        self.s.download_pinned(stream, self.dc, self.host_c)

    def _streamed_step(self, stream, after):
        if self._streamer is None:
            from titan_rs_b200.streaming import StreamedGemm
            self._streamer = StreamedGemm(self.s, self.M, self.N, self.K)
        self._streamer.run(stream, self.host_a, self.host_b, self.host_c, after=after)

    @property
    def e2e_streamed(self):
        # One GPU: the host-operand GEMM of titan_rs_b200.streaming (B, then A in row
        # blocks, each block's GEMM and download overlapping the later blocks' uploads).
        if self.world != 1 or os.environ.get("TITAN_B200_E2E", "streamed") != "streamed":
            return None
        return self._streamed_step

    _streamer = None

    def h2d_bytes(self):
        return self.a_bytes + self.b_bytes

    def d2h_bytes(self):
        return self.c_bytes

    def config(self):
        return workload_config(self.name, self.world, self.small)

    def cpu_sample(self, budget_s, threads=0):
        import oracle
        threads = threads or oracle.cpu_count()
        rng = np.random.default_rng(0)
        pts = 0
        t0 = time.perf_counter()
        while time.perf_counter() - t0 < budget_s:
            rows = rng.integers(0, self.M, 2048)
            cols = rng.integers(0, self.N, 2048)
            oracle.gemm_bf16_points(self.a_bits, self.b_bits, True, self.M, self.N, self.K, rows, cols, threads)
            pts += 2048
        dt = time.perf_counter() - t0
        return {"value": 2.0 * self.K * pts / dt / 1e12, "unit": "TFLOP/s", "cores": threads, "kind": "port",
                "sample": f"{pts} random C elements (full {self.K}-long dot products, reference loop order) "
                          f"in {dt:.1f} s on {threads} threads; rate extrapolated per element"}


class SdpaWorkload(Workload):
    name = "sdpa"
    metric = "causal SDPA fwd bf16 B8 H32 S4096 D128 TFLOP/s per B200 (causal-halved FLOPs)"
    unit = "TFLOP/s"
    dtype = "bf16"
    scaling = "strong"
    bound = "tensor"
    B, H, S, D = 8, 32, 4096, 128

    def __init__(self, *a, **k):
        super().__init__(*a, **k)
        import ctypes
        from titan_rs_b200 import _native as N
        from titan_rs_b200.kernel_abi import DType
        self.Nn, self.ctypes = N, ctypes
        if self.small:
            self.B = 2
        total_bh = self.B * self.H
        if total_bh % self.world:
            raise SystemExit(f"B*H={total_bh} does not split over {self.world} GPUs")
        self.bh_local = total_bh // self.world  # batch*heads shard of this rank: no communication
        S, D = self.S, self.D
        n = self.bh_local * S * D
        self.nbytes = n * 2
        self.hosts = [self.s.host_alloc(self.nbytes) for _ in range(3)]
        self.host_o = self.s.host_alloc(self.nbytes)
        self.bits = []
        for i, host in enumerate(self.hosts):
            arr = host.array(np.uint16, (self.bh_local, S, D))
            full_offset = self.rank * n  # this rank's slice of the seeded tensor (counter-based generator)
            arr[:] = self.tb.fill_normal(full_offset + n, seed=tensor_seed(3, i),
                                         dtype=DType.BF16)[full_offset:].reshape(self.bh_local, S, D)
            self.bits.append(arr)
        self.dev = [self.s.allocate(self.nbytes) for _ in range(3)]
        self.do = self.s.allocate(self.nbytes)
        for h, d in zip(self.hosts, self.dev):
            self.s.upload_pinned(self.st, d, h)
        self.s.synchronize(self.st)
        shape = (1, self.bh_local, S, D)
        self.tq, self.tk, self.tv = (_tensor(self.tb, d, DType.BF16, shape) for d in self.dev)
        self.to = _tensor(self.tb, self.do, DType.BF16, shape)
        cand = os.environ.get("TITAN_B200_SDPA_CANDIDATE", "sdpa_fwd_bf16_d128_pair")
        self.attrs = (N.Attr * 2)()
        self._key, self._ckey, self._cval = b"causal", b"candidate", cand.encode()
        self.attrs[0].key = self._key
        self.attrs[0].value = 1
        self.attrs[1].key = self._ckey
        self.attrs[1].str = self._cval
        self.kernel = cand

    def units_per_step(self):
        return 4.0 * self.bh_local * self.S * self.S * self.D / 2.0

    def step(self):
        c = self.ctypes
        rc = self.Nn.lib().tb_op_sdpa(self.s.ptr, self.st.ptr, c.byref(self.tq), c.byref(self.tk), c.byref(self.tv),
                                      c.byref(self.to), self.attrs, 2, None)
        if rc:
            raise RuntimeError(self.Nn.last_error())

    def e2e_upload(self, stream):
        for h, d in zip(self.hosts, self.dev):
            self.s.upload_pinned(stream, d, h)

    _streamer = None

    def _streamed_step(self, stream, after):
        if self._streamer is None:
            from titan_rs_b200.kernel_abi import DType
            from titan_rs_b200.streaming import StreamedBatchOp
            # [B*H, 1, S, D]: the same (batch, head) problems, blocked over the leading dimension.
            spec = (DType.BF16, (self.bh_local, 1, self.S, self.D), True)
            self._streamer = StreamedBatchOp(self.s, "scaled_dot_product_attention", [spec, spec, spec],
                                             (DType.BF16, (self.bh_local, 1, self.S, self.D)),
                                             {"causal": 1, "candidate": self._cval.decode()})
        self._streamer.run(stream, self.hosts, self.host_o, after=after)

    @property
    def e2e_streamed(self):
        # One GPU: titan_rs_b200.streaming.StreamedBatchOp over (batch, head) blocks.
        if self.world != 1 or os.environ.get("TITAN_B200_E2E", "streamed") != "streamed":
            return None
        return self._streamed_step

    def e2e_download(self, stream):
        self.s.download_pinned(stream, self.do, self.host_o)

    def h2d_bytes(self):
        return 3 * self.nbytes

    def d2h_bytes(self):
        return self.nbytes

    def config(self):
        return workload_config(self.name, self.world, self.small)

    def cpu_sample(self, budget_s, threads=0):
        import oracle
        threads = threads or oracle.cpu_count()
        S, D = self.S, self.D
        rng = np.random.default_rng(0)
        macs = 0.0
        rows_done = 0
        t0 = time.perf_counter()
        q, k, v = (b.reshape(-1) for b in self.bits)
        while time.perf_counter() - t0 < budget_s:
            ids = np.sort(rng.integers(0, self.bh_local * S, 256))
            oracle.sdpa_bf16_rows(q, k, v, 1, self.bh_local, S, S, D, True, ids, threads=threads)
            macs += float(np.sum((ids % S) + 1)) * 2 * D  # QK^T and PV per visible key
            rows_done += ids.size
        dt = time.perf_counter() - t0
        return {"value": 2.0 * macs / dt / 1e12, "unit": "TFLOP/s", "cores": threads, "kind": "port",
                "sample": f"{rows_done} random causal query rows (reference loop order) in {dt:.1f} s on "
                          f"{threads} threads; FLOP/s of the rows computed"}


class ConvWorkload(Workload):
    name = "conv2d"
    metric = "conv2d fwd bf16 NHWC 64x56x56x256->256 3x3 s1 p1 (implicit GEMM) TFLOP/s per B200"
    unit = "TFLOP/s"
    dtype = "bf16"
    scaling = "strong"
    bound = "tensor"
    N, H, W, C, K, R, S = 64, 56, 56, 256, 256, 3, 3
    ROTATE = 3  # input/output pairs cycled so each step reads an input evicted from L2

    def __init__(self, *a, **k):
        super().__init__(*a, **k)
        import ctypes
        from titan_rs_b200 import _native as N
        from titan_rs_b200.kernel_abi import DType
        self.Nn, self.ctypes = N, ctypes
        if self.small:
            self.N = 16
        if self.N % self.world:
            raise SystemExit(f"batch {self.N} does not split over {self.world} GPUs")
        self.n_local = self.N // self.world  # batch shard of this rank: no communication
        H, W, C, K = self.H, self.W, self.C, self.K
        nx = self.n_local * H * W * C
        self.x_bytes = nx * 2
        self.w_bytes = K * self.R * self.S * C * 2
        self.y_bytes = self.n_local * H * W * K * 2
        self.host_x = self.s.host_alloc(self.x_bytes)
        self.host_w = self.s.host_alloc(self.w_bytes)
        self.host_y = self.s.host_alloc(self.y_bytes)
        off = self.rank * nx
        self.x_bits = self.host_x.array(np.uint16, (self.n_local, H, W, C))
        self.x_bits[:] = self.tb.fill_normal(off + nx, seed=tensor_seed(4, 0), dtype=DType.BF16)[off:].reshape(
            self.x_bits.shape)
        self.w_bits = self.host_w.array(np.uint16, (K, self.R, self.S, C))
        self.w_bits[:] = self.tb.fill_normal(K * self.R * self.S * C, seed=tensor_seed(4, 1),
                                             std=math.sqrt(2.0 / (self.R * self.S * C)),
                                             dtype=DType.BF16).reshape(self.w_bits.shape)
        self.dx = [self.s.allocate(self.x_bytes) for _ in range(self.ROTATE)]
        self.dy = [self.s.allocate(self.y_bytes) for _ in range(self.ROTATE)]
        self.dw = self.s.allocate(self.w_bytes)
        for d in self.dx:
            self.s.upload_pinned(self.st, d, self.host_x)
        self.s.upload_pinned(self.st, self.dw, self.host_w)
        self.s.synchronize(self.st)
        self.tx = [_tensor(self.tb, d, DType.BF16, (self.n_local, H, W, C)) for d in self.dx]
        self.ty = [_tensor(self.tb, d, DType.BF16, (self.n_local, H, W, K)) for d in self.dy]
        self.tw = _tensor(self.tb, self.dw, DType.BF16, (K, self.R, self.S, C))
        names = ["stride_h", "stride_w", "pad_h", "pad_w", "dilation_h", "dilation_w", "groups", "layout"]
        vals = [1, 1, 1, 1, 1, 1, 1, b"NHWC"]
        # Optional kernel choice (an operator candidate name); unset, the operator picks.
        cand = os.environ.get("TITAN_B200_CONV_CANDIDATE", "")
        if cand:
            names.append("candidate")
            vals.append(cand.encode())
        self._keys = [n.encode() for n in names]
        self._strs = [v for v in vals if isinstance(v, bytes)]  # kept alive for the C strings
        self.attr_dict = {n: (v.decode() if isinstance(v, bytes) else v) for n, v in zip(names, vals)}
        self.attrs = (N.Attr * len(names))()
        for i, (key, v) in enumerate(zip(self._keys, vals)):
            self.attrs[i].key = key
            if isinstance(v, bytes):
                self.attrs[i].str = v
            else:
                self.attrs[i].value = v
        self.i = 0
        # The operator's choice at C5 (and at every batch shard of up to 8 GPUs).
        self.kernel = cand or "conv2d_fprop_bf16_nhwc_2sm"

    def units_per_step(self):
        return 2.0 * self.n_local * self.H * self.W * self.K * self.C * self.R * self.S

    def step(self):
        c = self.ctypes
        j = self.i % self.ROTATE
        self.i += 1
        rc = self.Nn.lib().tb_op_conv2d(self.s.ptr, self.st.ptr, c.byref(self.tx[j]), c.byref(self.tw), None,
                                        c.byref(self.ty[j]), self.attrs, len(self._keys), None)
        if rc:
            raise RuntimeError(self.Nn.last_error())

    def e2e_upload(self, stream):
        self.s.upload_pinned(stream, self.dx[0], self.host_x)
        self.s.upload_pinned(stream, self.dw, self.host_w)
        self.i = 0  # the next step() uses input/output pair 0

    _streamer = None

    def _streamed_step(self, stream, after):
        if self._streamer is None:
            from titan_rs_b200.kernel_abi import DType
            from titan_rs_b200.streaming import StreamedBatchOp
            attrs = self.attr_dict
            H, W, C, K = self.H, self.W, self.C, self.K
            self._streamer = StreamedBatchOp(
                self.s, "conv2d", [(DType.BF16, (self.n_local, H, W, C), True),
                                   (DType.BF16, (K, self.R, self.S, C), False)],
                (DType.BF16, (self.n_local, H, W, K)), attrs)
        self._streamer.run(stream, [self.host_x, self.host_w], self.host_y, after=after)

    @property
    def e2e_streamed(self):
        # titan_rs_b200.streaming.StreamedBatchOp over image blocks (weights once per call) on
        # request only: the conv's uploads (99 MB) dwarf its 0.16 ms of compute, and the
        # blocks measured no faster (97.5 against 98.6 TFLOP/s end to end).
        if self.world != 1 or os.environ.get("TITAN_B200_E2E", "") != "streamed":
            return None
        return self._streamed_step

    def e2e_download(self, stream):
        self.s.download_pinned(stream, self.dy[0], self.host_y)

    def h2d_bytes(self):
        return self.x_bytes + self.w_bytes

    def d2h_bytes(self):
        return self.y_bytes

    def config(self):
        return workload_config(self.name, self.world, self.small)

    def cpu_sample(self, budget_s, threads=0):
        import oracle
        threads = threads or oracle.cpu_count()
        rng = np.random.default_rng(0)
        pts = 0
        t0 = time.perf_counter()
        total = self.n_local * self.H * self.W * self.K
        while time.perf_counter() - t0 < budget_s:
            idx = rng.integers(0, total, 2048)
            oracle.conv2d_nhwc_bf16_points(self.x_bits, self.w_bits, None, self.n_local, self.H, self.W, self.C,
                                           self.K, self.R, self.S, (1, 1), (1, 1), (1, 1), self.H, self.W, idx,
                                           threads)
            pts += 2048
        dt = time.perf_counter() - t0
        return {"value": 2.0 * self.C * self.R * self.S * pts / dt / 1e12, "unit": "TFLOP/s", "cores": threads,
                "kind": "port", "sample": f"{pts} random output elements (reference loop order) in {dt:.1f} s on "
                                          f"{threads} threads; rate extrapolated per element (border taps counted)"}


WORKLOADS = {"softmax": SoftmaxWorkload, "gemm": GemmWorkload, "sdpa": SdpaWorkload, "conv2d": ConvWorkload}
DEFAULT_OP = "gemm"


# ----------------------------------------------------------------------------- driver
def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    return world, rank, local


def init_dist(world, local):
    if world <= 1:
        return None
    import datetime
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", local))
    return dist


def barrier(dist):
    if dist is not None:
        dist.barrier()


def reduce_max(dist, value: float) -> float:
    if dist is None:
        return value
    import torch
    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def run_reference_arm(args, world, rank):
    """The reference's scalar CPU operators (the oracle's restatement) on all host threads.

    Each step is one bounded sample of the configuration's work (args.ref_step_seconds of
    CPU time); the rate is extrapolated per output element or row. The product library is
    not loaded: the inputs come from the oracle's copy of the seeded generator."""
    if rank != 0:
        return 0
    import oracle
    wl_cls = WORKLOADS[args.op]
    sampler = REFERENCE_SAMPLERS[args.op]
    threads = oracle.cpu_count()  # every core this process may run on (torchrun sets OMP_NUM_THREADS=1)
    inputs = sampler(oracle, None, 0, 0)  # the sample's inputs, made once before the steps
    times = []
    info = None
    for i in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        info = sampler(oracle, inputs, args.ref_step_seconds, threads)
        if i >= args.warmup:
            times.append(time.perf_counter() - t0)
    single = sampler(oracle, inputs, max(args.ref_step_seconds / 2, 0.5), 1)
    cpu = {"value": info["value"], "unit": info["unit"], "cores": threads, "kind": "port",
           "sample": info["sample"] + "; ms_per_step is the wall time of one such bounded sample",
           "single_thread": {"value": single["value"], "cores": 1, "sample": single["sample"]}}
    line = {"impl": "reference", "metric": wl_cls.metric, "value": info["value"], "unit": info["unit"],
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 1000.0 * statistics.mean(times), "higher_is_better": True, "scaling": wl_cls.scaling,
            "vs_baseline": None, "dtype": wl_cls.dtype, "data": "synthetic (seeded, BASELINE.json shapes)",
            "config": workload_config(args.op, world), "op": wl_cls.name, "cpu_baseline": cpu,
            "e2e": {"value": info["value"], "unit": info["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    ops = {}
    for op in parse_ops(args):
        samp = REFERENCE_SAMPLERS[op]
        ins = samp(oracle, None, 0, 0)
        r = samp(oracle, ins, args.ref_step_seconds, threads)
        r1 = samp(oracle, ins, max(args.ref_step_seconds / 2, 0.5), 1)
        ops[OP_LABEL[op]] = {"metric": WORKLOADS[op].metric, "value": r["value"], "unit": r["unit"],
                             "config": workload_config(op, world),
                             "cpu_baseline": {"value": r["value"], "unit": r["unit"], "cores": threads,
                                              "kind": "port", "sample": r["sample"],
                                              "single_thread": {"value": r1["value"], "cores": 1,
                                                                "sample": r1["sample"]}}}
    if parse_ops(args) or args.op == DEFAULT_OP:
        ops["C1"] = c1_cpu(oracle, threads)
    if ops:
        line["ops"] = ops
    if any(m == "titan_rs_b200" or m.startswith("titan_rs_b200.") for m in sys.modules):
        raise SystemExit("the reference arm loaded the product library")
    print(json.dumps(line), flush=True)
    return 0


def _timed(budget_s, fn):
    """Calls fn() until budget_s has passed (at least once); returns (calls, seconds)."""
    n = 0
    t0 = time.perf_counter()
    while True:
        fn()
        n += 1
        if time.perf_counter() - t0 >= budget_s:
            break
    return n, time.perf_counter() - t0


def _ref_softmax(oracle, inputs, budget_s, threads):
    rows, cols = SoftmaxWorkload.rows, SoftmaxWorkload.cols
    chunk = 512
    if inputs is None:  # the first rows of the C2 tensor
        return oracle.fill_normal(chunk * cols, 1, 0.0, 2.0).reshape(chunk, cols)
    n, dt = _timed(budget_s, lambda: oracle.softmax_rows_mt(inputs, threads))
    return {"value": n * chunk * cols * 8 / dt / 1e9, "unit": "GB/s",
            "sample": f"{n} passes over the first {chunk} of the {rows} rows of C2 ({n * chunk} rows) in {dt:.1f} s "
                      f"on {threads} threads; bytes = 8 per element (read x, write y)"}


def _ref_gemm(oracle, inputs, budget_s, threads):
    K = GemmWorkload.K
    rows_needed = 512
    if inputs is None:  # the first 512 rows of A and of B's [N,K] storage: the sample draws only from those
        return (oracle.fill_normal(rows_needed * K, tensor_seed(2, 0), bf16=True).reshape(rows_needed, K),
                oracle.fill_normal(rows_needed * K, tensor_seed(2, 1), 0.0, 1.0 / math.sqrt(K),
                                   bf16=True).reshape(rows_needed, K))
    a, b = inputs
    rng = np.random.default_rng(0)

    def one():
        oracle.gemm_bf16_points(a, b, True, rows_needed, rows_needed, K, rng.integers(0, rows_needed, 2048),
                                rng.integers(0, rows_needed, 2048), threads)

    n, dt = _timed(budget_s, one)
    pts = n * 2048
    return {"value": 2.0 * K * pts / dt / 1e12, "unit": "TFLOP/s",
            "sample": f"{pts} C elements of C3 ({K}-long dot products in the reference loop order) in {dt:.1f} s "
                      f"on {threads} threads; rate extrapolated per element"}


def _ref_sdpa(oracle, inputs, budget_s, threads):
    S, D = SdpaWorkload.S, SdpaWorkload.D
    heads = 2  # the first two (b, h) pairs of C4
    if inputs is None:
        return [oracle.fill_normal(heads * S * D, tensor_seed(3, i), bf16=True) for i in range(3)]
    q, k, v = inputs
    rng = np.random.default_rng(0)
    acc = {"macs": 0.0, "rows": 0}

    def one():
        ids = np.sort(rng.integers(0, heads * S, 256))
        oracle.sdpa_bf16_rows(q, k, v, 1, heads, S, S, D, True, ids, threads=threads)
        acc["macs"] += float(np.sum((ids % S) + 1)) * 2 * D
        acc["rows"] += ids.size

    n, dt = _timed(budget_s, one)
    return {"value": 2.0 * acc["macs"] / dt / 1e12, "unit": "TFLOP/s",
            "sample": f"{acc['rows']} causal query rows of the first 2 heads of C4 in {dt:.1f} s on {threads} "
                      "threads; FLOP/s of the rows computed"}


def _ref_conv2d(oracle, inputs, budget_s, threads):
    wl = ConvWorkload
    imgs = 2  # the first two images of C5
    if inputs is None:
        return (oracle.fill_normal(imgs * wl.H * wl.W * wl.C, tensor_seed(4, 0), bf16=True),
                oracle.fill_normal(wl.K * wl.R * wl.S * wl.C, tensor_seed(4, 1), 0.0,
                                   math.sqrt(2.0 / (wl.R * wl.S * wl.C)), bf16=True))
    x, w = inputs
    rng = np.random.default_rng(0)

    def one():
        idx = rng.integers(0, imgs * wl.H * wl.W * wl.K, 2048)
        oracle.conv2d_nhwc_bf16_points(x, w, None, imgs, wl.H, wl.W, wl.C, wl.K, wl.R, wl.S, (1, 1), (1, 1), (1, 1),
                                       wl.H, wl.W, idx, threads)

    n, dt = _timed(budget_s, one)
    pts = n * 2048
    return {"value": 2.0 * wl.C * wl.R * wl.S * pts / dt / 1e12, "unit": "TFLOP/s",
            "sample": f"{pts} output elements of the first 2 images of C5 in {dt:.1f} s on {threads} threads; "
                      "rate extrapolated per element (border taps counted)"}


REFERENCE_SAMPLERS = {"softmax": _ref_softmax, "gemm": _ref_gemm, "sdpa": _ref_sdpa, "conv2d": _ref_conv2d}
OP_LABEL = {"softmax": "C2", "gemm": "C3", "sdpa": "C4", "conv2d": "C5"}
C1_FLOP = 2.0 * 256 ** 3


def c1_inputs(oracle):
    """C1: A, B f32 [256, 256] row-major, U[-1, 1), seed 0 (A = seed 0, B = seed 1)."""
    a = oracle.fill_uniform(256 * 256, tensor_seed(0, 0), -1.0, 1.0).reshape(256, 256)
    b = oracle.fill_uniform(256 * 256, tensor_seed(0, 1), -1.0, 1.0).reshape(256, 256)
    return a, b


def c1_cpu(oracle, threads, budget_s=1.0):
    """The reference's scalar gemm (rt:955-989) on the whole of C1, one thread and all threads."""
    a, b = c1_inputs(oracle)
    n1, dt1 = _timed(budget_s, lambda: oracle.gemm(a, b))
    nt, dtt = _timed(budget_s, lambda: oracle.gemm_mt(a, b, threads))
    return {"metric": "CPU scalar-reference MatMul f32 C[256,256] = A[256,256] B[256,256] GFLOP/s",
            "unit": "GFLOP/s",
            "config": {"workload": "C1 f32 GEMM M=N=K=256 row-major, A,B ~ U[-1,1) seed 0", "M": 256, "N": 256,
                       "K": 256},
            "cpu_baseline": {"value": nt * C1_FLOP / dtt / 1e9, "unit": "GFLOP/s", "cores": threads, "kind": "port",
                             "sample": f"{nt} full 256^3 products in {dtt:.2f} s on {threads} threads (rows split)",
                             "single_thread": {"value": n1 * C1_FLOP / dt1 / 1e9, "cores": 1,
                                               "sample": f"{n1} full 256^3 products in {dt1:.2f} s, one thread, "
                                                         "the reference's loop order"}}}


def parse_ops(args) -> list:
    """The extra configurations measured in the same run (never the headline op itself)."""
    if args.ops == "default":
        names = ["softmax", "sdpa", "conv2d"] if args.op == DEFAULT_OP else []
    elif args.ops in ("", "none"):
        names = []
    else:
        names = [o.strip() for o in args.ops.split(",") if o.strip()]
        for o in names:
            if o not in WORKLOADS:
                raise SystemExit(f"--ops: unknown op {o}")
    return [o for o in names if o != args.op]


def roofline_of(wl, per_launch_ms, peaks, peak_src, small):
    scale = 1e9 if wl.unit == "GB/s" else 1e12
    achieved = wl.units_per_step() / (per_launch_ms / 1e3) / scale
    if wl.bound == "hbm":
        peak, r_unit = float(peaks.get("hbm_gbs", PEAK_FALLBACK["hbm_gbs"])), "GB/s"
    else:
        peak, r_unit = float(peaks.get("bf16_tflops", PEAK_FALLBACK["bf16_tflops"])), "TFLOP/s"
    line = {"bound": wl.bound, "kernel": wl.kernel, "achieved": achieved, "peak": peak, "unit": r_unit,
            "frac": achieved / peak, "peak_source": "measured burst figure (MEASURED_PEAKS.json)"
            if peak_src == "measured" else "fallback", "ms_per_launch": per_launch_ms,
            "algorithmic_units_per_launch": wl.units_per_step()}
    if wl.bound == "tensor":
        # The bench times its steps after a power soak, between the burst and the
        # seconds-long sustained regime of the measured cuBLAS figures: both are given.
        sustained = float(peaks.get("bf16_tflops_sustained", PEAK_FALLBACK["bf16_tflops_sustained"]))
        line.update({"peak_sustained": sustained, "frac_of_sustained": achieved / sustained})
    line.update(traffic_of(wl.kernel, wl.world == 1 and not small))
    return line


def measure(wl, args, session, stream, dist, peaks, peak_src, tb, N) -> dict:
    """Warm-up, a clock soak, K device-timed steps (max over ranks), the kernel's roofline and
    the end-to-end figure through the C ABI with host buffers, for one workload."""
    w0 = session.record(stream)
    for _ in range(args.warmup):
        wl.step()
    w1 = session.record(stream)
    session.synchronize(stream)
    # The kernel the operator actually launched for this workload (the roofline names it).
    wl.kernel = N.lib().tb_last_candidate().decode()
    est_ms = max(session.elapsed_ms(w0, w1) / args.warmup, 1e-3)

    # nvidia-smi samples every 50 ms: keep the GPU busy with untimed steps for
    # ~0.3 s first so the clock record covers the load the timed steps run under.
    clocks = ClockSampler(int(os.environ.get("LOCAL_RANK", "0")))
    clocks.start()
    soak = 0 if args.small or args.soak_ms <= 0 else int(
        reduce_max(dist, float(min(max(args.soak_ms / est_ms, 1), 20000))))
    for _ in range(soak):
        wl.step()

    # Device-timed region: K back-to-back steps between one event pair on the
    # launching stream (the host enqueues faster than the kernels run), bracketed
    # by a barrier and a synchronize on both sides; max over ranks.
    barrier(dist)
    session.synchronize(stream)
    launches0 = int(N.lib().tb_launch_count())
    e0 = session.record(stream)
    for _ in range(args.steps):
        wl.step()
    e1 = session.record(stream)
    session.synchronize(stream)
    launches = int(N.lib().tb_launch_count()) - launches0
    barrier(dist)
    clock_info = clocks.stop()
    local_ms = session.elapsed_ms(e0, e1)
    total_ms = reduce_max(dist, local_ms)
    ms_step = total_ms / args.steps
    units_step = wl.job_units_per_step()
    scale = 1e9 if wl.unit == "GB/s" else 1e12
    value = units_step / (ms_step / 1e3) / scale

    # Roofline of the dominant kernel: its algorithmic units per launch / its average
    # launch duration on the launching stream. With a collective in the step (sharded
    # GEMM) the GEMM kernel is also timed alone: that is the compute phase, reported
    # beside the end-to-end value.
    kernel_ms = wl.dominant_kernel_ms(session, stream, args.steps) if hasattr(wl, "dominant_kernel_ms") else None
    compute_phase = None
    if kernel_ms is not None:
        step_kernel = wl.kernel
        wl.kernel = N.lib().tb_last_candidate().decode()
        kernel_ms_max = reduce_max(dist, kernel_ms)
        compute_phase = {"ms_per_step": kernel_ms_max, "value": units_step / (kernel_ms_max / 1e3) / scale,
                         "kernel": wl.kernel, "step_kernel": step_kernel,
                         "note": "GEMM kernel alone on this rank's shard, max over ranks (no all-gather); the step "
                                 "itself is bound by the all-gather's NVLink traffic"}
    per_launch_ms = kernel_ms if kernel_ms is not None else local_ms / args.steps
    roofline = roofline_of(wl, per_launch_ms, peaks, peak_src, args.small)

    # End to end through the C ABI with pinned host buffers: every step copies its inputs
    # in and its result out. Steps are pipelined as a server would run them: uploads and
    # the operator on the main stream, downloads on a second stream, so step i+1's upload
    # overlaps step i's download (PCIe is full duplex); the operator of step i+1 waits
    # for step i's download, since it overwrites the result buffer.
    e2e = None
    if not args.small:
        out_stream = session.create_stream()

        streamed = wl.e2e_streamed

        def e2e_run(steps, start=None):
            if streamed is not None:
                # Every step's uploads, operator and downloads are enqueued by the
                # public call; the first step's uploads wait for the start event.
                for i in range(steps):
                    streamed(stream, start if i == 0 else None)
                return
            prev_download = None
            for _ in range(steps):
                wl.e2e_upload(stream)
                if prev_download is not None:
                    session.wait_event(stream, prev_download)
                wl.step()
                session.wait_event(out_stream, session.record(stream))
                wl.e2e_download(out_stream)
                prev_download = session.record(out_stream)

        e2e_run(2)
        session.synchronize(stream)
        session.synchronize(out_stream)
        barrier(dist)
        session.synchronize(stream)
        e0 = session.record(stream)
        e2e_steps = max(3, min(args.steps, 10))
        e2e_run(e2e_steps, e0)
        if streamed is None:
            e1 = session.record(out_stream)
        else:
            e1 = session.record(stream)  # the call's stream waits for its last download
        session.synchronize(out_stream)
        session.synchronize(stream)
        e2e_ms = reduce_max(dist, session.elapsed_ms(e0, e1)) / e2e_steps
        e2e = {"value": units_step / (e2e_ms / 1e3) / scale, "unit": wl.unit, "h2d_bytes_per_step": wl.h2d_bytes(),
               "d2h_bytes_per_step": wl.d2h_bytes(), "ms_per_step": e2e_ms,
               "path": (f"titan_rs_b200.streaming.{type(wl._streamer).__name__}.run (blocks: upload, operator and "
                        "download overlapped)" if streamed is not None else
                        "tb_upload_pinned + operator + tb_download_pinned, steps pipelined over two streams")}
    out = {"metric": wl.metric, "value": value, "unit": wl.unit, "ms_per_step": ms_step, "scaling": wl.scaling,
           "dtype": wl.dtype, "config": wl.config(), "op": wl.name, "roofline": roofline, "e2e": e2e,
           "gpu_launches": launches, "clocks": clock_info}
    if compute_phase is not None:
        out["compute_phase"] = compute_phase
    return out


def cpu_baseline_of(wl, budget_s):
    """All host threads on a bounded sample, then one thread on a shorter one."""
    cpu = wl.cpu_sample(budget_s)
    one = wl.cpu_sample(max(budget_s / 4, 0.5), threads=1)
    cpu["single_thread"] = {"value": one["value"], "cores": 1, "sample": one["sample"]}
    return cpu


def c1_gpu(tb, N, session, stream, steps):
    """The f32 reference-ABI GEMM on the GPU over C1's inputs (device-timed, launch-bound)."""
    import ctypes
    from titan_rs_b200.kernel_abi import DType
    a = tb.fill_uniform(256 * 256, seed=tensor_seed(0, 0), low=-1.0, high=1.0).reshape(256, 256)
    b = tb.fill_uniform(256 * 256, seed=tensor_seed(0, 1), low=-1.0, high=1.0).reshape(256, 256)
    bufs = [session.allocate(256 * 256 * 4) for _ in range(3)]
    session.upload(stream, bufs[0], a)
    session.upload(stream, bufs[1], b)
    ta, tbm, tc = (_tensor(tb, buf, DType.F32, (256, 256)) for buf in bufs)

    def step():
        rc = N.lib().tb_op_gemm(session.ptr, stream.ptr, ctypes.byref(ta), ctypes.byref(tbm), ctypes.byref(tc), None,
                                0, None)
        if rc:
            raise RuntimeError(N.last_error())

    for _ in range(3):
        step()
    session.synchronize(stream)
    kernel = N.lib().tb_last_candidate().decode()
    e0 = session.record(stream)
    for _ in range(steps):
        step()
    e1 = session.record(stream)
    session.synchronize(stream)
    ms = session.elapsed_ms(e0, e1) / steps
    # The same launches captured once into a CUDA graph and replayed with one launch
    # (tb_capture_begin/end, tb_graph_exec_launch): the host's per-launch work leaves
    # the timed region, which at this size is most of it.
    session.capture_begin(stream)
    for _ in range(steps):
        step()
    graph = session.capture_end(stream)
    graph.launch(stream)  # warm-up replay
    session.synchronize(stream)
    g0 = session.record(stream)
    graph.launch(stream)
    g1 = session.record(stream)
    session.synchronize(stream)
    gms = session.elapsed_ms(g0, g1) / steps
    graph.release()
    return {"value": C1_FLOP / (ms / 1e3) / 1e9, "unit": "GFLOP/s", "ms_per_step": ms, "kernel": kernel,
            "note": "f32 reference ABI on CUDA cores (bit-identical to the scalar reference); launch-bound at this size",
            "graph_replay": {"value": C1_FLOP / (gms / 1e3) / 1e9, "unit": "GFLOP/s", "ms_per_step": gms,
                             "note": f"{steps} launches captured into one CUDA graph, replayed with one launch"}}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--op", default=DEFAULT_OP, choices=sorted(WORKLOADS))
    ap.add_argument("--ops", default="default",
                    help="extra configs measured in the same run: comma list of ops, 'none', or 'default' "
                         "(softmax,sdpa,conv2d when --op is gemm)")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=8.0, help="CPU baseline sample budget (rank 0, N=1)")
    ap.add_argument("--ops-cpu-seconds", type=float, default=4.0, help="CPU baseline budget of each extra config")
    ap.add_argument("--ref-step-seconds", type=float, default=2.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--soak-ms", type=float, default=300.0,
                    help="untimed steps run before the timed ones so the clocks settle under load (0: none)")
    ap.add_argument("--small", action="store_true",
                    help="reduced problem (still larger than L2) for profiler captures; not a bench line")
    args = ap.parse_args(argv)
    if args.warmup < 3:
        args.warmup = 3
    world, rank, local = dist_env()
    if args.impl == "reference":
        return run_reference_arm(args, world, rank)

    import gc

    import titan_rs_b200 as tb
    from titan_rs_b200 import _native as N
    dist = init_dist(world, local)
    session = tb.Session(local)
    stream = session.create_stream()
    comm = None
    if world > 1 and args.op == "gemm":
        from titan_rs_b200 import distributed as D
        comm = D.NcclCollective(session, D.broadcast_comm_id(rank), world, rank, timeout_ms=60000)
    peaks, peak_src = load_peaks()
    cpu_leg = rank == 0 and world == 1 and not args.no_cpu_baseline and not args.small

    wl = WORKLOADS[args.op](tb, session, stream, rank, world, comm=comm, small=args.small)
    head = measure(wl, args, session, stream, dist, peaks, peak_src, tb, N)
    cpu = cpu_baseline_of(wl, args.cpu_seconds) if cpu_leg else None
    del wl
    gc.collect()

    ops = {}
    for op in parse_ops(args):
        w = WORKLOADS[op](tb, session, stream, rank, world, small=args.small)
        r = measure(w, args, session, stream, dist, peaks, peak_src, tb, N)
        r["cpu_baseline"] = cpu_baseline_of(w, args.ops_cpu_seconds) if cpu_leg else None
        ops[OP_LABEL[op]] = r
        del w
        gc.collect()
    if ops and not args.small:
        c1 = {"gpu": c1_gpu(tb, N, session, stream, args.steps)}
        if cpu_leg:
            import oracle
            c1.update(c1_cpu(oracle, oracle.cpu_count()))
        ops["C1"] = c1

    if rank == 0:
        line = {
            "metric": head["metric"], "value": head["value"], "unit": head["unit"], "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": head["ms_per_step"], "higher_is_better": True,
            "scaling": head["scaling"], "vs_baseline": None, "dtype": head["dtype"],
            "data": "synthetic (seeded, BASELINE.json shapes)", "config": head["config"], "op": head["op"],
            "roofline": head["roofline"], "cpu_baseline": cpu, "e2e": head["e2e"],
            "gpu_launches": head["gpu_launches"], "clocks": head["clocks"],
        }
        if "compute_phase" in head:
            line["compute_phase"] = head["compute_phase"]
        if ops:
            line["ops"] = ops
        print(json.dumps(line), flush=True)
    if dist is not None:
        session.synchronize(stream)
        dist.barrier()
        if comm is not None:
            comm.close()
        dist.destroy_process_group()
    return 0


# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of one full-size launch of
# each kernel at N=1, from 1-pass ncu captures of bench.py. Each figure carries the
# SHA-256 prefix of the kernel's sources (its .cu file, every shared .cuh and the tile
# configuration header) at capture time; when the sources differ now, the figure
# belongs to another build of the kernel and the bench prints null instead.
_TRAFFIC_CAPTURE = ("ncu --metrics dram__bytes_read.sum,dram__bytes_write.sum,gpu__time_duration.sum "
                    "--clock-control none -k regex:{kernel} -s 3 -c 1 python bench.py --op {op} --ops none "
                    "--steps 5 --warmup 3 --no-cpu-baseline --soak-ms 0")
TRAFFIC_PER_LAUNCH: dict = {
    "gemm_bf16_tn_2sm": {"read": 1044584704, "write": 126917888, "source_sha16": "a1c6ceac6de8b7b5",
                         "capture": _TRAFFIC_CAPTURE.format(kernel="gemm_bf16_tn_2sm", op="gemm")},
    "softmax_f32_warp32": {"read": 536921856, "write": 481277184, "source_sha16": "d9c1e674e4ee55f3",
                           "capture": _TRAFFIC_CAPTURE.format(kernel="softmax_f32_warp32", op="softmax")},
    "sdpa_fwd_bf16_d128_pair": {"read": 817332224, "write": 250097664, "source_sha16": "634d5518b8f1f1b4",
                                "capture": _TRAFFIC_CAPTURE.format(kernel="sdpa_fwd_bf16_d128_pair", op="sdpa")},
    "conv2d_fprop_bf16_nhwc_2sm": {"read": 103998464, "write": 55198720, "source_sha16": "b42c3a7b52ea5292",
                                   "capture": _TRAFFIC_CAPTURE.format(kernel="conv2d_fprop_bf16_nhwc_2sm",
                                                                      op="conv2d")},
}

KERNEL_SOURCE = {"softmax_f32_warp": "softmax.cu", "gemm_bf16_tn": "gemm_bf16.cu", "gemm_bf16_nn": "gemm_bf16.cu",
                 "gemm_bf16_ta": "gemm_bf16.cu", "sdpa_fwd_bf16_d128_pair": "sdpa_bf16_pair.cu",
                 "sdpa_fwd_bf16_d128_bn64": "sdpa_bf16_bn64.cu", "sdpa_fwd_bf16_d128": "sdpa_bf16.cu",
                 "conv2d_fprop_bf16_nhwc": "conv2d_bf16.cu"}


def kernel_source_digest(kernel: str):
    import hashlib
    kdir = ROOT / "titan_rs_b200" / "csrc" / "kernels"
    src = next((f for prefix, f in sorted(KERNEL_SOURCE.items(), key=lambda kv: -len(kv[0]))
                if kernel.startswith(prefix)), None)
    if src is None:
        return None
    h = hashlib.sha256()
    for path in [kdir / src] + sorted(kdir.glob("*.cuh")) + [kdir / "kernel_configs.h"]:
        h.update(path.name.encode())
        h.update(path.read_bytes())
    return h.hexdigest()[:16]


def traffic_of(kernel: str, full_size_single_gpu: bool) -> dict:
    entry = TRAFFIC_PER_LAUNCH.get(kernel)
    if not full_size_single_gpu or entry is None:
        return {"traffic": None, "traffic_note": "no ncu capture of this kernel at this configuration"}
    if entry["source_sha16"] != kernel_source_digest(kernel):
        return {"traffic": None, "traffic_note": "the ncu capture was of another build of this kernel"}
    return {"traffic": entry["read"] + entry["write"], "traffic_read": entry["read"], "traffic_write": entry["write"],
            "traffic_note": f"ncu dram__bytes_read.sum + dram__bytes_write.sum per launch ({entry['capture']})"}


if __name__ == "__main__":
    sys.exit(main())
