"""A bf16 graph through the compiled plan on the B200: a two-layer MLP
(gemm -> broadcast.add -> gelu -> gemm -> broadcast.add) compiles to two
gemm.bias_act nodes, runs without host waits between nodes, and matches the oracle
(the reference's gemm, bias add and gelu in f32, with the bf16 hidden layer)."""
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
