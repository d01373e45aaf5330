"""bench.py's reference arm on the CPU: it runs the oracle only (the product library is
never imported), and its line carries the same config dicts as the product arm's."""
import json
import os
import pathlib
import subprocess
import sys

import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

import bench  # noqa: E402


def test_reference_arm_runs_without_the_product_library():
    proc = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1", "--warmup",
                           "3", "--ref-step-seconds", "0.05"], capture_output=True, text=True, timeout=600,
                          cwd=str(ROOT))
    assert proc.returncode == 0, proc.stderr
    line = json.loads(proc.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["op"] == "gemm"
    assert line["config"] == bench.workload_config("gemm", 1)
    assert set(line["ops"]) == {"C1", "C2", "C4", "C5"}
    for label, op in [("C2", "softmax"), ("C4", "sdpa"), ("C5", "conv2d")]:
        assert line["ops"][label]["config"] == bench.workload_config(op, 1)
        assert line["ops"][label]["cpu_baseline"]["single_thread"]["cores"] == 1
    assert line["cpu_baseline"]["single_thread"]["value"] > 0
    assert line["ops"]["C1"]["cpu_baseline"]["single_thread"]["value"] > 0
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["value"] == line["value"]


@pytest.mark.parametrize("op", ["softmax", "sdpa", "conv2d"])
def test_reference_arm_single_op(op):
    # torchrun starts every rank with OMP_NUM_THREADS=1; the reference arm still uses every
    # core the process may run on.
    env = dict(os.environ, OMP_NUM_THREADS="1")
    proc = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--op", op, "--steps", "1",
                           "--warmup", "3", "--ref-step-seconds", "0.05"], capture_output=True, text=True,
                          timeout=600, cwd=str(ROOT), env=env)
    assert proc.returncode == 0, proc.stderr
    line = json.loads(proc.stdout.strip().splitlines()[-1])
    assert line["config"] == bench.workload_config(op, 1) and "ops" not in line
    assert line["cpu_baseline"]["cores"] == len(os.sched_getaffinity(0))


def test_configs_name_the_shard_at_n_gpus():
    assert bench.workload_config("gemm", 8)["parallelism"] == "N-shard8"
    assert bench.workload_config("sdpa", 4)["parallelism"] == "bh-shard4"
    assert bench.workload_config("conv2d", 2)["parallelism"] == "batch-shard2"
    assert bench.workload_config("softmax", 2)["parallelism"] == "replicas2"


def test_traffic_figure_needs_the_captured_build():
    """A traffic figure is printed only for the kernel build it was captured on."""
    saved = dict(bench.TRAFFIC_PER_LAUNCH)
    try:
        bench.TRAFFIC_PER_LAUNCH["gemm_bf16_tn_2sm"] = {"read": 1.0, "write": 2.0, "source_sha16": "0" * 16,
                                                       "capture": "test"}
        assert bench.traffic_of("gemm_bf16_tn_2sm", True)["traffic"] is None
        bench.TRAFFIC_PER_LAUNCH["gemm_bf16_tn_2sm"]["source_sha16"] = bench.kernel_source_digest("gemm_bf16_tn_2sm")
        assert bench.traffic_of("gemm_bf16_tn_2sm", True)["traffic"] == 3.0
        assert bench.traffic_of("gemm_bf16_tn_2sm", False)["traffic"] is None
        assert bench.traffic_of("unlisted_kernel", True)["traffic"] is None
    finally:
        bench.TRAFFIC_PER_LAUNCH.clear()
        bench.TRAFFIC_PER_LAUNCH.update(saved)
