"""Graph execution for the hot-path operators.

Mirrors titan.rs's `ExecutionPlan` (projects/titan-runtime/src/lib.rs:176-276) and
`Runtime::compile` (:3472-3483) over the Graph IR (projects/titan-graph/src/graph.rs:72-105):
values map to `TensorSpec`s, nodes run in construction order as `OpRequest`s through
`Runtime.execute`, and intermediate tensors live in a binding environment. Values of
any dtype the operators take (bf16 included) flow between nodes unchanged.

Two differences, both for the B200:

* Nodes are only enqueued: every node runs on the runtime's stream, so each one
  starts after its producers without a host wait, and the plan waits once, on the
  last node's event. The reference waits after every node (`handle.wait()`, :235).
* `compile` runs fusion passes beside validation and dead-code elimination (the
  reference's core pipeline, projects/titan-graph/src/optimize.rs:23-60):
  - a bf16 `gemm` (any storage order and extents; storage the tensor maps cannot read
    is staged K-major inside the fused node) whose only consumer
    is `broadcast.add` of an fp32 [N] bias and/or `gelu` / `silu` becomes one
    `gemm.bias_act` node, i.e. one
    tensor-core kernel whose epilogue applies the bias and the activation to the
    fp32 accumulator (the chain's intermediate bf16 roundings disappear);
  - softmax into its attention consumer: S = gemm(Q, K, transpose_rhs),
    P = softmax(S, last axis), O = gemm(P, V) on bf16 [T, D] values, with S and P
    used only inside the chain, becomes one `attention.fused` node, run as the
    flash-attention kernel (scores, softmax and P V in one pass; the [Tq, Tk] S
    and P never reach memory). The chain has no 1/sqrt(D) factor, so the node
    calls `scaled_dot_product_attention` with scale 1.0 on [1, 1, T, D] views of
    the same buffers.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Optional

from . import _native as N
from .kernel_abi import DType
from .runtime import (ExecutionError, ExecutionHandle, OpRequest, Runtime, TensorHandle, TensorSpec,
                      contiguous_strides)


@dataclass
class GraphNode:
    """GraphNode (graph.rs:72-87): id, operator, input/output value ids, attributes."""
    id: int
    operator: str
    inputs: list
    outputs: list
    attrs: dict = field(default_factory=dict)


@dataclass
class Graph:
    """Graph (graph.rs:91-105): inputs, outputs, value table, nodes in construction order."""
    inputs: list
    outputs: list
    values: dict
    nodes: list


@dataclass
class PassReport:
    """PassReport (optimize.rs:10-20)."""
    name: str
    changed: bool
    notes: list


def validate(graph: Graph) -> None:
    for v in list(graph.inputs) + list(graph.outputs):
        if v not in graph.values:
            raise ExecutionError("graph.validate", "compile", f"value {v} has no TensorSpec")
    produced = set(graph.inputs)
    for node in graph.nodes:
        for v in node.inputs:
            if v not in produced:
                raise ExecutionError(node.operator, "compile", f"node {node.id} reads value {v} before it is produced")
        for v in node.outputs:
            if v not in graph.values:
                raise ExecutionError(node.operator, "compile", f"missing TensorSpec for value {v}")
            produced.add(v)


def dead_code_eliminate(graph: Graph) -> tuple[Graph, bool]:
    live = set(graph.outputs)
    kept = []
    for node in reversed(graph.nodes):
        if any(o in live for o in node.outputs):
            kept.append(node)
            live.update(node.inputs)
    kept.reverse()
    return Graph(list(graph.inputs), list(graph.outputs), dict(graph.values), kept), len(kept) != len(graph.nodes)


def _consumers(graph: Graph, value: int) -> list:
    return [n for n in graph.nodes if value in n.inputs]


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
            users = _consumers(current, tail)
            if tail not in outputs and len(users) == 1 and users[0].operator == "broadcast.add" and \
                    len(users[0].inputs) == 2:
                add = users[0]
                other = add.inputs[1] if add.inputs[0] == tail else add.inputs[0]
                bspec = values.get(other)
                if bspec is not None and bspec.dtype == DType.F32 and tuple(bspec.shape) == (spec.shape[1],) and \
                        values[add.outputs[0]].dtype == DType.BF16:
                    absorbed.append(add)
                    bias, tail = other, add.outputs[0]
                    users = _consumers(current, tail)
            if tail not in outputs and len(users) == 1 and users[0].operator in ("gelu", "silu") and \
                    values[users[0].outputs[0]].dtype == DType.BF16:
                absorbed.append(users[0])
                act, tail = users[0].operator, users[0].outputs[0]
            if not absorbed:
                continue
            layout = {key: bool(g.attrs[key]) for key in ("transpose_lhs", "transpose_rhs") if key in g.attrs}
            fused = GraphNode(g.id, "gemm.bias_act", list(g.inputs) + ([bias] if bias is not None else []), [tail],
                              {**layout, "activation": act})
            gone = {n.id for n in absorbed}
            nodes = [fused if n is g else n for n in nodes if n.id not in gone]
            for n in [g] + absorbed[:-1]:
                values.pop(n.outputs[0], None)
            notes.append(f"fused node {g.id} (gemm) with " + ", ".join(f"node {n.id} ({n.operator})" for n in absorbed)
                         + " into gemm.bias_act")
            changed = True
            break
    return Graph(list(graph.inputs), list(graph.outputs), values, nodes), notes


def _is_last_axis_softmax(node: GraphNode, rank: int) -> bool:
    axis = node.attrs.get("axis", rank - 1)
    return isinstance(axis, int) and not isinstance(axis, bool) and axis == rank - 1 and \
        set(node.attrs) <= {"axis"}


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
            users = _consumers(current, s_val)
            if s_val in outputs or len(users) != 1 or users[0].operator != "softmax" or \
                    not _is_last_axis_softmax(users[0], 2):
                continue
            sm = users[0]
            p_val = sm.outputs[0]
            p_spec = values.get(p_val)
            if p_spec is None or p_spec.dtype != DType.BF16 or tuple(p_spec.shape) != (tq, tk):
                continue
            users = _consumers(current, p_val)
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


def _view(t: TensorHandle, shape: tuple) -> TensorHandle:
    """The same contiguous buffer under another shape (a reshape without a copy)."""
    if tuple(t.strides) != contiguous_strides(t.shape):
        raise ExecutionError("attention.fused", "bind", "fused attention requires contiguous Q, K and V")
    return TensorHandle(t.session, t.buffer, t.dtype, tuple(shape), contiguous_strides(shape))


class ExecutionPlan:
    """ExecutionPlan (lib.rs:176-276): the optimised graph and its pass reports."""

    def __init__(self, graph: Graph, reports: list):
        self.graph = graph
        self.reports = reports

    def node_count(self) -> int:
        return len(self.graph.nodes)

    def execute(self, runtime: Runtime, bindings: dict) -> ExecutionHandle:
        env = dict(bindings)
        for v in self.graph.inputs:
            if v not in env:
                raise ExecutionError("graph.bind", "bind", f"missing binding for input value {v}")
        last: Optional[ExecutionHandle] = None
        for node in self.graph.nodes:
            inputs = []
            for v in node.inputs:
                if v not in env:
                    raise ExecutionError(node.operator, "bind", f"missing tensor for value {v}")
                inputs.append(env[v])
            specs = []
            for v in node.outputs:
                if v not in self.graph.values:
                    raise ExecutionError(node.operator, "bind", f"missing TensorSpec for value {v}")
                specs.append(self.graph.values[v])
            if node.operator == "attention.fused":
                # [T, D] values as [1, 1, T, D] views for the BHTD attention operator.
                (tq, d), (tk, _) = inputs[0].shape, inputs[1].shape
                views = [_view(inputs[0], (1, 1, tq, d)), _view(inputs[1], (1, 1, tk, d)),
                         _view(inputs[2], (1, 1, tk, d))]
                handle = runtime.execute(OpRequest("scaled_dot_product_attention", views,
                                                   [TensorSpec(DType.BF16, (1, 1, tq, d))], dict(node.attrs)))
                handle = ExecutionHandle([_view(handle.outputs[0], (tq, d))], handle.candidate, handle.kernel,
                                         handle.event)
            else:
                handle = runtime.execute(OpRequest(node.operator, inputs, specs, dict(node.attrs)))
            if len(handle.outputs) != len(node.outputs):
                raise ExecutionError(node.operator, "execute", f"node {node.id} produced {len(handle.outputs)} "
                                                               f"outputs, expected {len(node.outputs)}")
            for v, t in zip(node.outputs, handle.outputs):
                env[v] = t
            last = handle
        outs = []
        for v in self.graph.outputs:
            if v not in env:
                raise ExecutionError("graph.output", "bind", f"missing output value {v}")
            outs.append(env[v])
        if not outs and last is not None:
            outs = last.outputs
        # Every node ran on the runtime's stream: the last node's event covers them all.
        return ExecutionHandle(outs, "b200/graph", "graph.plan", last.event if last else None)


def compile(graph: Graph) -> ExecutionPlan:
    """Runtime::compile (lib.rs:3472-3483): validate, DCE, fusion; an empty result is an error."""
    reports = []
    validate(graph)
    reports.append(PassReport("validate", False, ["schema and constraints ok"]))
    graph, changed = dead_code_eliminate(graph)
    reports.append(PassReport("dce", changed, ["removed unreachable pure nodes"]))
    graph, notes = fuse_gemm_epilogues(graph)
    reports.append(PassReport("fusion.gemm_epilogue", bool(notes), notes))
    graph, notes = fuse_attention(graph)
    reports.append(PassReport("fusion.attention", bool(notes), notes))
    validate(graph)
    if not graph.nodes:
        raise ExecutionError("graph.empty", "compile", "graph has no nodes after passes", N.TB_ERR_INVALID)
    return ExecutionPlan(graph, reports)


__all__ = ["GraphNode", "Graph", "PassReport", "ExecutionPlan", "compile", "validate", "dead_code_eliminate",
           "fuse_gemm_epilogues", "fuse_attention"]
