"""Graph compile passes and binding errors (no GPU): the ExecutionPlan mirror of
projects/titan-runtime/src/lib.rs:176-276, 3472-3483 and the gemm-epilogue fusion."""
import pytest

from titan_rs_b200 import graph as G
from titan_rs_b200.kernel_abi import DType
from titan_rs_b200.runtime import ExecutionError, TensorSpec


def spec(dtype, *shape):
    return TensorSpec(dtype, tuple(shape))


def mlp_graph(act="gelu", bias_dtype=DType.F32, output_intermediate=False, transpose_rhs=True):
    # x[8,16] W1[32,16] b1[32] -> gemm -> add -> act -> h[8,32]; W2[4,32] b2[4] -> gemm -> add -> y[8,4]
    values = {0: spec(DType.BF16, 8, 16), 1: spec(DType.BF16, 32, 16), 2: spec(bias_dtype, 32),
              3: spec(DType.BF16, 8, 32), 4: spec(DType.BF16, 8, 32), 5: spec(DType.BF16, 8, 32),
              6: spec(DType.BF16, 4, 32), 7: spec(DType.F32, 4), 8: spec(DType.BF16, 8, 4), 9: spec(DType.BF16, 8, 4)}
    nodes = [G.GraphNode(10, "gemm", [0, 1], [3], {"transpose_rhs": transpose_rhs}),
             G.GraphNode(11, "broadcast.add", [3, 2], [4]),
             G.GraphNode(12, act, [4], [5]),
             G.GraphNode(13, "gemm", [5, 6], [8], {"transpose_rhs": True}),
             G.GraphNode(14, "broadcast.add", [7, 8], [9])]
    outputs = [9] + ([4] if output_intermediate else [])
    return G.Graph([0, 1, 2, 6, 7], outputs, values, nodes)


def test_fusion_turns_each_gemm_chain_into_one_node():
    plan = G.compile(mlp_graph())
    ops = [(n.operator, n.inputs, n.outputs, n.attrs) for n in plan.graph.nodes]
    assert ops == [("gemm.bias_act", [0, 1, 2], [5], {"transpose_rhs": True, "activation": "gelu"}),
                   ("gemm.bias_act", [5, 6, 7], [9], {"transpose_rhs": True, "activation": "none"})]
    assert 3 not in plan.graph.values and 4 not in plan.graph.values and 8 not in plan.graph.values
    fusion = [r for r in plan.reports if r.name == "fusion.gemm_epilogue"][0]
    assert fusion.changed and len(fusion.notes) == 2


def test_fusion_keeps_what_it_cannot_absorb():
    # A visible intermediate stops the chain at that value.
    g = G.compile(mlp_graph(output_intermediate=True)).graph
    assert [n.operator for n in g.nodes] == ["gemm.bias_act", "gelu", "gemm.bias_act"]
    assert g.nodes[0].attrs["activation"] == "none" and g.nodes[0].outputs == [4]
    # A bf16 bias or an untransposed B is left alone.
    assert [n.operator for n in G.compile(mlp_graph(bias_dtype=DType.BF16)).graph.nodes][:3] == \
        ["gemm", "broadcast.add", "gelu"]
    assert G.compile(mlp_graph(act="silu")).graph.nodes[0].attrs["activation"] == "silu"


def test_fusion_covers_every_storage_order_and_extent():
    def chain(k, n, attrs):
        # x[8, k] times W (stored [k, n], or [n, k] with transpose_rhs) -> + b[n] -> gelu
        w_shape = (n, k) if attrs.get("transpose_rhs") else (k, n)
        values = {0: spec(DType.BF16, 8, k), 1: spec(DType.BF16, *w_shape), 2: spec(DType.F32, n),
                  3: spec(DType.BF16, 8, n), 4: spec(DType.BF16, 8, n), 5: spec(DType.BF16, 8, n)}
        nodes = [G.GraphNode(10, "gemm", [0, 1], [3], attrs), G.GraphNode(11, "broadcast.add", [3, 2], [4]),
                 G.GraphNode(12, "gelu", [4], [5])]
        return G.compile(G.Graph([0, 1, 2], [5], values, nodes)).graph.nodes
    fused = chain(16, 24, {})  # B stored [K, N]: the N-contiguous kernel takes it
    assert [n.operator for n in fused] == ["gemm.bias_act"] and fused[0].attrs == {"activation": "gelu"}
    # Extents the tensor maps cannot read directly run staged inside gemm.bias_act.
    assert [n.operator for n in chain(12, 24, {})] == ["gemm.bias_act"]  # K % 8 != 0
    assert [n.operator for n in chain(16, 20, {})] == ["gemm.bias_act"]  # N % 8 != 0 with B [K, N]
    assert [n.operator for n in chain(16, 20, {"transpose_rhs": True})] == ["gemm.bias_act"]


def test_dead_code_and_empty_graph():
    g = mlp_graph()
    g.outputs = [5]  # the second layer is dead
    plan = G.compile(g)
    assert [n.id for n in plan.graph.nodes] == [10]
    assert [r.changed for r in plan.reports if r.name == "dce"] == [True]
    empty = G.Graph([0], [0], {0: spec(DType.F32, 4)}, [G.GraphNode(1, "softmax", [0], [1])])
    empty.values[1] = spec(DType.F32, 4)
    with pytest.raises(ExecutionError) as e:
        G.compile(empty)
    assert e.value.phase == "compile" and "no nodes" in e.value.message


def test_validation_and_binding_errors():
    g = mlp_graph()
    g.nodes[0].inputs = [0, 99]
    with pytest.raises(ExecutionError, match="before it is produced"):
        G.compile(g)
    plan = G.compile(mlp_graph())
    with pytest.raises(ExecutionError) as e:
        plan.execute(runtime=None, bindings={0: object()})
    assert e.value.phase == "bind" and "missing binding for input value 1" in e.value.message


def attention_graph(tq=64, tk=96, d=128, dtype=DType.BF16, axis=1, p_is_output=False, s_users=1, v_shape=None,
                    transpose_rhs=True):
    # Q[tq,d] K[tk,d] V[tk,d] -> S = gemm(Q, K^T) -> P = softmax(S) -> O = gemm(P, V)
    values = {0: spec(dtype, tq, d), 1: spec(dtype, tk, d), 2: spec(dtype, *(v_shape or (tk, d))),
              3: spec(dtype, tq, tk), 4: spec(dtype, tq, tk), 5: spec(dtype, tq, d)}
    attrs = {"axis": axis} if axis is not None else {}
    nodes = [G.GraphNode(10, "gemm", [0, 1], [3], {"transpose_rhs": transpose_rhs}),
             G.GraphNode(11, "softmax", [3], [4], attrs),
             G.GraphNode(12, "gemm", [4, 2], [5])]
    outputs = [5] + ([4] if p_is_output else [])
    if s_users == 2:
        values[6] = spec(dtype, tq, tk)
        nodes.append(G.GraphNode(13, "softmax", [3], [6], {"axis": 1}))
        outputs.append(6)
    return G.Graph([0, 1, 2], outputs, values, nodes)


def test_attention_fusion_replaces_the_chain():
    plan = G.compile(attention_graph())
    assert [(n.operator, n.inputs, n.outputs, n.attrs) for n in plan.graph.nodes] == \
        [("attention.fused", [0, 1, 2], [5], {"scale": 1.0})]
    assert 3 not in plan.graph.values and 4 not in plan.graph.values
    rep = [r for r in plan.reports if r.name == "fusion.attention"][0]
    assert rep.changed and "attention.fused [64x96, D=128]" in rep.notes[0]
    # The default axis (none given) is the last one too.
    assert G.compile(attention_graph(axis=None)).graph.nodes[0].operator == "attention.fused"


def test_attention_fusion_leaves_other_chains_alone():
    def ops(g):
        return [n.operator for n in G.compile(g).graph.nodes]
    unfused = ["gemm", "softmax", "gemm"]
    assert ops(attention_graph(dtype=DType.F32)) == unfused          # f32 keeps the reference kernels
    assert ops(attention_graph(axis=0)) == unfused                   # softmax over the query axis
    assert ops(attention_graph(p_is_output=True)) == unfused         # P is visible
    assert ops(attention_graph(s_users=2)) == ["gemm", "softmax", "gemm", "softmax"]  # S has another reader
    assert ops(attention_graph(transpose_rhs=False, tk=128)) == unfused  # K not stored [Tk, D]


def test_fused_attention_node_reaches_the_runtime_as_one_request():
    """The plan hands attention.fused to the runtime as one request on the bound [T, D]
    tensors with scale 1.0 (the router views them as [1, 1, T, D]; that view is checked
    in test_native_cpu) and binds the [Tq, D] result."""
    from types import SimpleNamespace

    from titan_rs_b200.runtime import ExecutionHandle, TensorHandle, contiguous_strides

    class FakeRuntime:
        def __init__(self):
            self.requests = []

        def execute(self, req):
            self.requests.append(req)
            spec = req.outputs[0]
            out = TensorHandle("session", "out-buffer", spec.dtype, tuple(spec.shape), contiguous_strides(spec.shape))
            return ExecutionHandle([out], "sdpa_fwd_bf16_d128_pair", "kernel", SimpleNamespace(name="event"))

    def handle(name, shape):
        return TensorHandle("session", name, DType.BF16, shape, contiguous_strides(shape))

    plan = G.compile(attention_graph(tq=64, tk=96, d=128))
    rt = FakeRuntime()
    res = plan.execute(rt, {0: handle("q", (64, 128)), 1: handle("k", (96, 128)), 2: handle("v", (96, 128))})
    (req,) = rt.requests
    assert req.operator == "attention.fused" and req.attrs == {"scale": 1.0}
    assert [(t.buffer, t.shape) for t in req.inputs] == [("q", (64, 128)), ("k", (96, 128)), ("v", (96, 128))]
    assert tuple(req.outputs[0].shape) == (64, 128)
    out = res.outputs[0]
    assert (out.buffer, out.shape, out.strides) == ("out-buffer", (64, 128), (128, 1))
