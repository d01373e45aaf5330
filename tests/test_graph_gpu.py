"""bf16 graphs through the compiled plan on the B200: a two-layer MLP
(gemm -> broadcast.add -> gelu -> gemm -> broadcast.add) compiles to two
gemm.bias_act nodes, runs without host waits between nodes, and matches the oracle
(the reference's gemm, bias add and gelu in f32, with the bf16 hidden layer); an
attention chain (gemm -> softmax -> gemm) compiles to one flash-attention launch."""
import math

import numpy as np
import pytest

import oracle
import titan_rs_b200 as tb
from titan_rs_b200 import graph as G
from titan_rs_b200.kernel_abi import DType
from titan_rs_b200.runtime import TensorSpec

from gpu_util import max_rel_err

pytestmark = pytest.mark.gpu


def test_bf16_mlp_graph_fuses_and_matches_oracle():
    s = tb.Session(0)
    rt = tb.Runtime(s)
    m, d_in, d_hid, d_out = 256, 512, 768, 384
    x = tb.fill_normal(m * d_in, seed=301, dtype=DType.BF16).reshape(m, d_in)
    w1 = tb.fill_normal(d_hid * d_in, seed=302, std=1 / math.sqrt(d_in), dtype=DType.BF16).reshape(d_hid, d_in)
    b1 = tb.fill_normal(d_hid, seed=303, std=0.5)
    w2 = tb.fill_normal(d_out * d_hid, seed=304, std=1 / math.sqrt(d_hid), dtype=DType.BF16).reshape(d_out, d_hid)
    b2 = tb.fill_normal(d_out, seed=305, std=0.5)
    values = {0: TensorSpec(DType.BF16, (m, d_in)), 1: TensorSpec(DType.BF16, (d_hid, d_in)),
              2: TensorSpec(DType.F32, (d_hid,)), 3: TensorSpec(DType.BF16, (m, d_hid)),
              4: TensorSpec(DType.BF16, (m, d_hid)), 5: TensorSpec(DType.BF16, (m, d_hid)),
              6: TensorSpec(DType.BF16, (d_out, d_hid)), 7: TensorSpec(DType.F32, (d_out,)),
              8: TensorSpec(DType.BF16, (m, d_out)), 9: TensorSpec(DType.BF16, (m, d_out))}
    nodes = [G.GraphNode(10, "gemm", [0, 1], [3], {"transpose_rhs": True}),
             G.GraphNode(11, "broadcast.add", [3, 2], [4]),
             G.GraphNode(12, "gelu", [4], [5]),
             G.GraphNode(13, "gemm", [5, 6], [8], {"transpose_rhs": True}),
             G.GraphNode(14, "broadcast.add", [8, 7], [9])]
    plan = G.compile(G.Graph([0, 1, 2, 6, 7], [9], values, nodes))
    assert [n.operator for n in plan.graph.nodes] == ["gemm.bias_act", "gemm.bias_act"]
    bind = {0: tb.TensorHandle.from_numpy(s, x, DType.BF16), 1: tb.TensorHandle.from_numpy(s, w1, DType.BF16),
            2: tb.TensorHandle.from_numpy(s, b1), 6: tb.TensorHandle.from_numpy(s, w2, DType.BF16),
            7: tb.TensorHandle.from_numpy(s, b2)}
    h = plan.execute(rt, bind).wait()
    assert h.kernel == "graph.plan"
    got = h.outputs[0].to_f32()

    rows, cols = np.divmod(np.arange(m * d_hid), d_hid)
    hid = oracle.gelu(oracle.gemm_bf16_points(x, w1, True, m, d_hid, d_in, rows, cols).reshape(m, d_hid) + b1)
    hid_bits = tb.f32_to_bf16_bits(hid)  # the hidden layer is a bf16 tensor between the two nodes
    rows, cols = np.divmod(np.arange(m * d_out), d_out)
    ref = oracle.gemm_bf16_points(hid_bits, w2, True, m, d_out, d_hid, rows, cols).reshape(m, d_out) + b2
    assert np.isfinite(got).all()
    assert max_rel_err(got, ref) <= 1e-2, max_rel_err(got, ref)
    s.close()


def test_attention_chain_fuses_into_one_flash_attention_launch():
    s = tb.Session(0)
    rt = tb.Runtime(s)
    tq, tk, d = 256, 384, 128
    std = d ** -0.25  # scores of unit variance, as with pre-scaled queries
    q = tb.fill_normal(tq * d, seed=311, std=std, dtype=DType.BF16).reshape(tq, d)
    k = tb.fill_normal(tk * d, seed=312, std=std, dtype=DType.BF16).reshape(tk, d)
    v = tb.fill_normal(tk * d, seed=313, dtype=DType.BF16).reshape(tk, d)
    values = {0: TensorSpec(DType.BF16, (tq, d)), 1: TensorSpec(DType.BF16, (tk, d)),
              2: TensorSpec(DType.BF16, (tk, d)), 3: TensorSpec(DType.BF16, (tq, tk)),
              4: TensorSpec(DType.BF16, (tq, tk)), 5: TensorSpec(DType.BF16, (tq, d))}
    nodes = [G.GraphNode(10, "gemm", [0, 1], [3], {"transpose_rhs": True}),
             G.GraphNode(11, "softmax", [3], [4], {"axis": 1}),
             G.GraphNode(12, "gemm", [4, 2], [5])]
    graph = G.Graph([0, 1, 2], [5], values, nodes)
    plan = G.compile(graph)
    assert [n.operator for n in plan.graph.nodes] == ["attention.fused"]
    binds = {i: tb.TensorHandle.from_numpy(s, a, DType.BF16, rt.stream) for i, a in enumerate((q, k, v))}
    before = tb.launch_count()
    fused = plan.execute(rt, binds).wait().outputs[0]
    assert tb.launch_count() - before == 1 and tb.last_candidate() == "sdpa_fwd_bf16_d128_pair"
    assert fused.shape == (tq, d)
    # The same graph unfused: three kernels, S and P rounded to bf16 in memory.
    before = tb.launch_count()
    unfused = G.ExecutionPlan(graph, []).execute(rt, binds).wait().outputs[0]
    assert tb.launch_count() - before == 3
    ref = oracle.sdpa_bf16_rows(q.reshape(1, 1, tq, d), k.reshape(1, 1, tk, d), v.reshape(1, 1, tk, d), 1, 1, tq, tk,
                                d, False, np.arange(tq), scale=1.0)
    assert max_rel_err(fused.to_f32(), ref) <= 1e-2
    assert max_rel_err(unfused.to_f32(), ref) <= 3e-2
    s.close()


def test_compiled_plan_captured_as_a_cuda_graph_replays_on_new_inputs():
    """ExecutionPlan.capture: the MLP's two fused nodes as one CUDA graph. Each replay,
    after new contents are uploaded into the bound input, must equal an eager run of
    the plan on the same input, bit for bit (same kernels, same buffers)."""
    s = tb.Session(0)
    rt = tb.Runtime(s)
    m, d_in, d_hid, d_out = 256, 512, 768, 384
    w1 = tb.fill_normal(d_hid * d_in, seed=402, std=1 / math.sqrt(d_in), dtype=DType.BF16).reshape(d_hid, d_in)
    b1 = tb.fill_normal(d_hid, seed=403, std=0.5)
    w2 = tb.fill_normal(d_out * d_hid, seed=404, std=1 / math.sqrt(d_hid), dtype=DType.BF16).reshape(d_out, d_hid)
    b2 = tb.fill_normal(d_out, seed=405, std=0.5)
    values = {0: TensorSpec(DType.BF16, (m, d_in)), 1: TensorSpec(DType.BF16, (d_hid, d_in)),
              2: TensorSpec(DType.F32, (d_hid,)), 3: TensorSpec(DType.BF16, (m, d_hid)),
              4: TensorSpec(DType.BF16, (m, d_hid)), 5: TensorSpec(DType.BF16, (m, d_hid)),
              6: TensorSpec(DType.BF16, (d_out, d_hid)), 7: TensorSpec(DType.F32, (d_out,)),
              8: TensorSpec(DType.BF16, (m, d_out)), 9: TensorSpec(DType.BF16, (m, d_out))}
    nodes = [G.GraphNode(10, "gemm", [0, 1], [3], {"transpose_rhs": True}),
             G.GraphNode(11, "broadcast.add", [3, 2], [4]),
             G.GraphNode(12, "gelu", [4], [5]),
             G.GraphNode(13, "gemm", [5, 6], [8], {"transpose_rhs": True}),
             G.GraphNode(14, "broadcast.add", [8, 7], [9])]
    plan = G.compile(G.Graph([0, 1, 2, 6, 7], [9], values, nodes))
    x0 = tb.fill_normal(m * d_in, seed=400, dtype=DType.BF16).reshape(m, d_in)
    x_t = tb.TensorHandle.from_numpy(s, x0, DType.BF16)
    bind = {0: x_t, 1: tb.TensorHandle.from_numpy(s, w1, DType.BF16), 2: tb.TensorHandle.from_numpy(s, b1),
            6: tb.TensorHandle.from_numpy(s, w2, DType.BF16), 7: tb.TensorHandle.from_numpy(s, b2)}
    captured = plan.capture(rt, bind)
    for seed in (410, 420):
        x = tb.fill_normal(m * d_in, seed=seed, dtype=DType.BF16).reshape(m, d_in)
        s.wait(s.upload(rt.stream, x_t.buffer, x))
        captured.launch()
        s.synchronize(rt.stream)
        got = captured.outputs[0].to_numpy(rt.stream)
        want = plan.execute(rt, bind).wait().outputs[0].to_numpy(rt.stream)
        np.testing.assert_array_equal(got, want)
        assert np.isfinite(tb.bf16_bits_to_f32(got)).all()
    captured.graph.release()
    s.close()
