"""The native graph compiler (tb_graph_compile) against a Python statement of the same
passes, on generated graphs (no GPU).

`Oracle` below is test infrastructure: the passes written as plain Python over the
GraphNode / Graph dataclasses (validate, dead-code elimination, the GEMM-epilogue fusion
and the attention fusion, as the Runtime::compile mirror defines them). The generator
builds graphs from fusable templates (gemm -> bias -> activation, gemm -> softmax -> gemm)
and perturbs them: other dtypes and shapes, extra consumers, visible intermediates, other
softmax axes and attributes, dead nodes, reads of values not yet produced."""
import random

import pytest
from hypothesis import given, settings
from hypothesis import strategies as st

from titan_rs_b200 import graph as G
from titan_rs_b200.graph import Graph, GraphNode, PassReport
from titan_rs_b200.kernel_abi import DType
from titan_rs_b200.runtime import ExecutionError, TensorSpec


class Oracle:
    @staticmethod
    def validate(graph: Graph) -> None:
        if not graph.outputs:
            raise ExecutionError("graph.validate", "compile", "graph must declare at least one output")
        for v in list(graph.inputs) + list(graph.outputs):
            if v not in graph.values:
                raise ExecutionError("graph.validate", "compile", f"value {v} has no TensorSpec")
        seen = set()
        for node in graph.nodes:
            if node.id in seen:
                raise ExecutionError("graph.validate", "compile", f"duplicate node id {node.id}")
            seen.add(node.id)
        produced = set(graph.inputs)
        for node in graph.nodes:
            for v in node.inputs:
                if v not in produced:
                    raise ExecutionError(node.operator, "compile", f"node {node.id} reads value {v} before it is produced")
            for v in node.outputs:
                if v not in graph.values:
                    raise ExecutionError(node.operator, "compile", f"missing TensorSpec for value {v}")
                produced.add(v)


    @staticmethod
    def dead_code_eliminate(graph: Graph) -> tuple[Graph, bool]:
        live = set(graph.outputs)
        kept = []
        for node in reversed(graph.nodes):
            if any(o in live for o in node.outputs):
                kept.append(node)
                live.update(node.inputs)
        kept.reverse()
        return Graph(list(graph.inputs), list(graph.outputs), dict(graph.values), kept), len(kept) != len(graph.nodes)


    @staticmethod
    def _consumers(graph: Graph, value: int) -> list:
        return [n for n in graph.nodes if value in n.inputs]


    @staticmethod
    def fuse_gemm_epilogues(graph: Graph) -> tuple[Graph, list]:
        """gemm -> [broadcast.add(bias fp32 [N])] -> [gelu | silu]  =>  gemm.bias_act."""
        notes = []
        nodes = list(graph.nodes)
        values = dict(graph.values)
        outputs = set(graph.outputs)
        changed = True
        while changed:
            changed = False
            current = Graph(graph.inputs, graph.outputs, values, nodes)
            for g in nodes:
                if g.operator != "gemm" or len(g.outputs) != 1 or len(g.inputs) != 2:
                    continue
                out = g.outputs[0]
                spec = values[out]
                if spec.dtype != DType.BF16 or len(spec.shape) != 2:
                    continue
                absorbed, bias, act, tail = [], None, "none", out
                users = Oracle._consumers(current, tail)
                if tail not in outputs and len(users) == 1 and users[0].operator == "broadcast.add" and \
                        len(users[0].inputs) == 2:
                    add = users[0]
                    other = add.inputs[1] if add.inputs[0] == tail else add.inputs[0]
                    bspec = values.get(other)
                    if bspec is not None and bspec.dtype == DType.F32 and tuple(bspec.shape) == (spec.shape[1],) and \
                            values[add.outputs[0]].dtype == DType.BF16:
                        absorbed.append(add)
                        bias, tail = other, add.outputs[0]
                        users = Oracle._consumers(current, tail)
                if tail not in outputs and len(users) == 1 and users[0].operator in ("gelu", "silu") and \
                        values[users[0].outputs[0]].dtype == DType.BF16:
                    absorbed.append(users[0])
                    act, tail = users[0].operator, users[0].outputs[0]
                if not absorbed:
                    continue
                layout = {key: bool(g.attrs[key]) for key in ("transpose_lhs", "transpose_rhs") if key in g.attrs}
                fused = GraphNode(g.id, "gemm.bias_act", list(g.inputs) + ([bias] if bias is not None else []), [tail],
                                  {**layout, "activation": act})
                # The fused node sits where the chain's last node was.
                gone = [g] + absorbed[:-1]
                nodes = [fused if n is absorbed[-1] else n for n in nodes if not any(n is x for x in gone)]
                for n in [g] + absorbed[:-1]:
                    values.pop(n.outputs[0], None)
                notes.append(f"fused node {g.id} (gemm) with " + ", ".join(f"node {n.id} ({n.operator})" for n in absorbed)
                             + " into gemm.bias_act")
                changed = True
                break
        return Graph(list(graph.inputs), list(graph.outputs), values, nodes), notes


    @staticmethod
    def _is_last_axis_softmax(node: GraphNode, rank: int) -> bool:
        axis = node.attrs.get("axis", rank - 1)
        return isinstance(axis, int) and not isinstance(axis, bool) and axis == rank - 1 and \
            set(node.attrs) <= {"axis"}


    @staticmethod
    def fuse_attention(graph: Graph) -> tuple[Graph, list]:
        """gemm(Q, K; transpose_rhs) -> softmax(last axis) -> gemm(P, V)  =>  attention.fused(Q, K, V)."""
        notes = []
        nodes = list(graph.nodes)
        values = dict(graph.values)
        outputs = set(graph.outputs)
        changed = True
        while changed:
            changed = False
            current = Graph(graph.inputs, graph.outputs, values, nodes)
            for g in nodes:
                if g.operator != "gemm" or len(g.inputs) != 2 or len(g.outputs) != 1 or \
                        not g.attrs.get("transpose_rhs") or g.attrs.get("transpose_lhs"):
                    continue
                q, k = g.inputs
                s_val = g.outputs[0]
                specs = [values.get(v) for v in (q, k, s_val)]
                if any(sp is None or sp.dtype != DType.BF16 or len(sp.shape) != 2 for sp in specs):
                    continue
                (tq, d), (tk, dk), _ = (tuple(sp.shape) for sp in specs)
                users = Oracle._consumers(current, s_val)
                if s_val in outputs or len(users) != 1 or users[0].operator != "softmax" or \
                        not Oracle._is_last_axis_softmax(users[0], 2):
                    continue
                sm = users[0]
                p_val = sm.outputs[0]
                p_spec = values.get(p_val)
                if p_spec is None or p_spec.dtype != DType.BF16 or tuple(p_spec.shape) != (tq, tk):
                    continue
                users = Oracle._consumers(current, p_val)
                if p_val in outputs or len(users) != 1 or users[0].operator != "gemm" or \
                        users[0].inputs[0] != p_val or len(users[0].inputs) != 2 or \
                        users[0].attrs.get("transpose_lhs") or users[0].attrs.get("transpose_rhs"):
                    continue
                pv = users[0]
                v = pv.inputs[1]
                v_spec, o_spec = values.get(v), values.get(pv.outputs[0])
                if v_spec is None or o_spec is None or v_spec.dtype != DType.BF16 or o_spec.dtype != DType.BF16 or \
                        tuple(v_spec.shape) != (tk, d) or tuple(o_spec.shape) != (tq, d) or dk != d:
                    continue
                # The fused node sits where P V was: Q, K and V are all produced by then.
                fused = GraphNode(pv.id, "attention.fused", [q, k, v], [pv.outputs[0]], {"scale": 1.0})
                nodes = [fused if n is pv else n for n in nodes if n is not g and n is not sm]
                values.pop(s_val, None)
                values.pop(p_val, None)
                notes.append(f"fused node {g.id} (gemm), node {sm.id} (softmax) and node {pv.id} (gemm) into "
                             f"attention.fused [{tq}x{tk}, D={d}]")
                changed = True
                break
        return Graph(list(graph.inputs), list(graph.outputs), values, nodes), notes


    @staticmethod
    def compile(graph: Graph):
        reports = []
        Oracle.validate(graph)
        reports.append(PassReport("validate", False, ["schema and constraints ok"]))
        graph, changed = Oracle.dead_code_eliminate(graph)
        reports.append(PassReport("dce", changed, ["removed unreachable pure nodes"]))
        graph, notes = Oracle.fuse_gemm_epilogues(graph)
        reports.append(PassReport("fusion.gemm_epilogue", bool(notes), notes))
        graph, notes = Oracle.fuse_attention(graph)
        reports.append(PassReport("fusion.attention", bool(notes), notes))
        Oracle.validate(graph)
        if not graph.nodes:
            raise ExecutionError("graph.empty", "compile", "graph has no nodes after passes")
        return graph, reports


BF, F32 = DType.BF16, DType.F32


@st.composite
def graphs(draw):
    """A graph of fusable templates with random perturbations."""
    values, nodes, inputs = {}, [], []
    ids = iter(range(1000, 100000))
    vid = iter(range(0, 1000))

    def value(dtype, *shape, graph_input=False):
        v = next(vid)
        values[v] = TensorSpec(dtype, tuple(shape))
        if graph_input:
            inputs.append(v)
        return v

    rnd = random.Random(draw(st.integers(0, 2 ** 32 - 1)))  # uniform perturbation rates

    def maybe(p=0.15):
        return rnd.random() < p

    def flip(dtype):
        return (F32 if dtype == BF else BF) if maybe(0.1) else dtype

    produced = []
    for _ in range(draw(st.integers(1, 5))):
        kind = draw(st.sampled_from(["mlp", "attn", "extra"]))
        if kind == "mlp" or (kind == "extra" and not produced):
            m, k, n = draw(st.sampled_from([4, 8, 12])), draw(st.sampled_from([8, 16, 12])), draw(st.sampled_from([8, 16, 20]))
            tr = draw(st.sampled_from([True, False, 1, 0, None]))
            x = produced[-1] if produced and maybe(0.3) and len(values[produced[-1]].shape) == 2 else value(BF, m, k, graph_input=True)
            m, k = values[x].shape
            w = value(BF, *((n, k) if tr else (k, n)), graph_input=True)
            y = value(flip(BF), m, n)
            attrs = {} if tr is None else {"transpose_rhs": tr}
            if maybe(0.1):
                attrs["transpose_lhs"] = False
            nodes.append(GraphNode(next(ids), "gemm", [x, w], [y], attrs))
            produced.append(y)
            if not maybe(0.3):
                if maybe(0.2):  # a bias produced by a node between the gemm and the add
                    b0 = value(F32, n, graph_input=True)
                    b = value(flip(F32), n if not maybe(0.1) else n + 1)
                    nodes.append(GraphNode(next(ids), "silu", [b0], [b]))
                else:
                    b = value(flip(F32), n if not maybe(0.1) else n + 1, graph_input=True)
                z = value(flip(BF), m, n)
                nodes.append(GraphNode(next(ids), "broadcast.add", [y, b] if maybe(0.7) else [b, y], [z]))
                produced.append(z)
                y = z
            if not maybe(0.4):
                a = value(flip(BF), m, n)
                nodes.append(GraphNode(next(ids), draw(st.sampled_from(["gelu", "silu"])), [y], [a]))
                produced.append(a)
        elif kind == "attn":
            tq, tk, d = draw(st.sampled_from([4, 8])), draw(st.sampled_from([4, 8, 16])), draw(st.sampled_from([8, 16]))
            q, k, v = value(BF, tq, d, graph_input=True), value(flip(BF), tk, d, graph_input=True), value(BF, tk, d if not maybe(0.1) else d + 8, graph_input=True)
            s = value(BF, tq, tk)
            nodes.append(GraphNode(next(ids), "gemm", [q, k], [s], {"transpose_rhs": True} if not maybe(0.1) else {}))
            p = value(flip(BF), tq, tk)
            sm_attrs = rnd.choice([{}, {"axis": 1}, {}, {"axis": 1}, {}, {"axis": 0}, {"axis": True}, {"axis": 1, "t": 2}])
            nodes.append(GraphNode(next(ids), "softmax", [s], [p], sm_attrs))
            o = value(flip(BF), tq, d)
            nodes.append(GraphNode(next(ids), "gemm", [p, v], [o], {} if not maybe(0.1) else {"transpose_rhs": True}))
            produced += [s, p, o]
        else:
            src = draw(st.sampled_from(produced))
            out = value(values[src].dtype, *values[src].shape)
            nodes.append(GraphNode(next(ids), draw(st.sampled_from(["gelu", "softmax", "silu"])), [src], [out]))
            produced.append(out)
    outputs = [produced[-1]] + [v for v in produced[:-1] if maybe(0.15)]
    if maybe(0.05):
        outputs.append(max(values) + 1)  # an output without a spec
    if maybe(0.05) and len(nodes) > 1:
        nodes.insert(0, nodes.pop())  # a node that reads values before they exist
    if maybe(0.04) and len(nodes) > 1:
        nodes[-1].id = nodes[0].id  # two nodes with one id
    if maybe(0.02):
        outputs = []
    return Graph(inputs, outputs, values, nodes)


def shape_of(graph):
    return ([(n.id, n.operator, list(n.inputs), list(n.outputs), n.attrs) for n in graph.nodes], sorted(graph.values))


@settings(max_examples=500, deadline=None)
@given(graphs())
def test_native_compiler_matches_the_python_passes(graph):
    try:
        want, want_reports = Oracle.compile(graph)
    except ExecutionError as e:
        with pytest.raises(ExecutionError) as got:
            G.compile(graph)
        assert (got.value.operator, got.value.phase, got.value.message) == (e.operator, e.phase, e.message)
        return
    plan = G.compile(graph)
    assert shape_of(plan.graph) == shape_of(want)
    assert [(r.name, r.changed, r.notes) for r in plan.reports] == [(r.name, r.changed, r.notes) for r in want_reports]


def test_individual_passes_match():
    values = {0: TensorSpec(BF, (8, 16)), 1: TensorSpec(BF, (32, 16)), 2: TensorSpec(F32, (32,)),
              3: TensorSpec(BF, (8, 32)), 4: TensorSpec(BF, (8, 32)), 5: TensorSpec(BF, (8, 32)), 6: TensorSpec(BF, (8, 32))}
    nodes = [GraphNode(10, "gemm", [0, 1], [3], {"transpose_rhs": 1}), GraphNode(11, "broadcast.add", [3, 2], [4]),
             GraphNode(12, "silu", [4], [5]), GraphNode(13, "gelu", [3], [6])]
    g = Graph([0, 1, 2], [5], values, nodes)
    for native, oracle in [(G.dead_code_eliminate, Oracle.dead_code_eliminate),
                           (G.fuse_gemm_epilogues, Oracle.fuse_gemm_epilogues), (G.fuse_attention, Oracle.fuse_attention)]:
        (a, ra), (b, rb) = native(g), oracle(g)
        assert shape_of(a) == shape_of(b) and ra == rb
    dce, _ = G.dead_code_eliminate(g)
    fused, notes = G.fuse_gemm_epilogues(dce)
    assert [n.operator for n in fused.nodes] == ["gemm.bias_act"] and fused.nodes[0].attrs == {
        "transpose_rhs": True, "activation": "silu"}
    assert notes == ["fused node 10 (gemm) with node 11 (broadcast.add), node 12 (silu) into gemm.bias_act"]


def test_serde_shaped_graph_with_tagged_attributes():
    """A graph as serde_json writes the reference's Graph (graph.rs:72-105, AttrValue
    externally tagged, titan-types/src/lib.rs:140-147): extra fields are ignored, tagged
    attributes are read, and the fused nodes carry tagged attributes back."""
    import ctypes
    import json
    import struct
    from titan_rs_b200 import _native as N

    def spec(dtype, *shape):
        return {"dtype": dtype, "shape": list(shape), "strides": [], "layout": "Contiguous", "alias": "NoAlias"}

    def node(i, op, ins, outs, attrs):
        return {"id": i, "operator": op, "inputs": ins, "outputs": outs, "attrs": attrs,
                "effects": {"kind": "pure"}, "source": {"file": "g", "line": 1, "column": 1}}

    graph = {"schema": 1, "inputs": [0, 1, 2, 6, 7, 8], "outputs": [5, 11], "constraints": [],
             "values": {"0": spec("BF16", 8, 16), "1": spec("BF16", 32, 16), "2": spec("F32", 32),
                        "3": spec("BF16", 8, 32), "4": spec("BF16", 8, 32), "5": spec("BF16", 8, 32),
                        "6": spec("BF16", 4, 16), "7": spec("BF16", 4, 16), "8": spec("BF16", 4, 16),
                        "9": spec("BF16", 4, 4), "10": spec("BF16", 4, 4), "11": spec("BF16", 4, 16)},
             "nodes": [node(20, "gemm", [0, 1], [3], {"transpose_rhs": {"Bool": True}}),
                       node(21, "broadcast.add", [3, 2], [4], {}),
                       node(22, "gelu", [4], [5], {}),
                       node(23, "gemm", [6, 7], [9], {"transpose_rhs": {"Int": 1}}),
                       node(24, "softmax", [9], [10], {"axis": {"Int": 1}}),
                       node(25, "gemm", [10, 8], [11], {})]}
    buf = ctypes.create_string_buffer(1 << 16)
    n = ctypes.c_size_t(0)
    assert N.lib().tb_graph_compile(json.dumps(graph).encode(), b"compile", buf, len(buf), ctypes.byref(n)) == N.TB_OK
    out = json.loads(buf.raw[:n.value])
    nodes = {x["id"]: x for x in out["graph"]["nodes"]}
    assert nodes[20]["operator"] == "gemm.bias_act" and nodes[20]["inputs"] == [0, 1, 2] and nodes[20]["outputs"] == [5]
    assert nodes[20]["attrs"] == {"transpose_rhs": {"Bool": True}, "activation": {"String": "gelu"}}
    one = struct.unpack("<Q", struct.pack("<d", 1.0))[0]
    assert nodes[25]["operator"] == "attention.fused" and nodes[25]["inputs"] == [6, 7, 8]
    assert nodes[25]["attrs"] == {"scale": {"Float": one}}
    assert sorted(nodes) == [20, 25]


def test_numpy_attribute_values_compile_like_python_ones():
    import numpy as np
    values = {0: TensorSpec(BF, (8, 16)), 1: TensorSpec(BF, (32, 16)), 3: TensorSpec(BF, (8, 32)),
              5: TensorSpec(BF, (8, 32))}
    nodes = [GraphNode(10, "gemm", [0, 1], [3], {"transpose_rhs": np.bool_(True), "tag": object()}),
             GraphNode(12, "gelu", [3], [5], {"weight": np.float32(0.5), "dims": np.arange(2)})]
    plan = G.compile(Graph([0, 1], [5], values, nodes))
    assert [(n.operator, n.attrs) for n in plan.graph.nodes] == [
        ("gemm.bias_act", {"transpose_rhs": True, "activation": "gelu"})]


def test_bias_produced_after_the_gemm_fuses_at_the_add():
    """gemm (10) -> silu making the bias (11) -> broadcast.add (12): the fused node takes the
    add's position, after the bias exists, and the compiled graph validates."""
    values = {0: TensorSpec(BF, (8, 16)), 1: TensorSpec(BF, (32, 16)), 2: TensorSpec(F32, (32,)),
              3: TensorSpec(BF, (8, 32)), 4: TensorSpec(F32, (32,)), 5: TensorSpec(BF, (8, 32))}
    nodes = [GraphNode(10, "gemm", [0, 1], [3], {"transpose_rhs": True}), GraphNode(11, "silu", [2], [4]),
             GraphNode(12, "broadcast.add", [3, 4], [5])]
    g = Graph([0, 1, 2], [5], values, nodes)
    plan = G.compile(g)
    assert [(n.id, n.operator, n.inputs, n.outputs) for n in plan.graph.nodes] == [
        (11, "silu", [2], [4]), (10, "gemm.bias_act", [0, 1, 4], [5])]
    want, _ = Oracle.compile(g)
    assert shape_of(plan.graph) == shape_of(want)


def test_validate_rejects_duplicate_node_ids_and_graphs_without_outputs():
    values = {0: TensorSpec(F32, (4,)), 1: TensorSpec(F32, (4,)), 2: TensorSpec(F32, (4,))}
    dup = Graph([0], [2], values, [GraphNode(7, "softmax", [0], [1]), GraphNode(7, "softmax", [1], [2])])
    with pytest.raises(ExecutionError) as e:
        G.compile(dup)
    assert (e.value.operator, e.value.message) == ("graph.validate", "duplicate node id 7")
    none = Graph([0], [], values, [GraphNode(7, "softmax", [0], [1])])
    with pytest.raises(ExecutionError) as e:
        G.compile(none)
    assert (e.value.operator, e.value.message) == ("graph.validate", "graph must declare at least one output")

