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

import ctypes
import json
from dataclasses import dataclass, field
from typing import Optional

import numpy as np

from . import _native as N
from .runtime import ExecutionError, ExecutionHandle, OpRequest, Runtime


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


def _json_attr(value):
    """Attribute values json does not know: numpy scalars by kind, anything else by repr
    (the compiler only reads bools, ints, floats and strings; other values pass through on
    the Python side untouched)."""
    if isinstance(value, np.bool_):
        return bool(value)
    if isinstance(value, np.integer):
        return int(value)
    if isinstance(value, np.floating):
        return float(value)
    if isinstance(value, (tuple, np.ndarray)):
        return list(value.tolist() if isinstance(value, np.ndarray) else value)
    return repr(value)


def _graph_json(graph: Graph) -> str:
    values = {str(k): {"dtype": v.dtype.name, "shape": [int(x) for x in v.shape]} for k, v in graph.values.items()}
    nodes = [{"id": n.id, "operator": n.operator, "inputs": list(n.inputs), "outputs": list(n.outputs),
              "attrs": dict(n.attrs)} for n in graph.nodes]
    return json.dumps({"inputs": [int(v) for v in graph.inputs], "outputs": [int(v) for v in graph.outputs],
                       "values": values, "nodes": nodes}, default=_json_attr)


def _run_passes(graph: Graph, passes: str) -> tuple[Graph, list]:
    """Runs passes of the native compiler (tb_graph_compile) and maps the result back:
    unchanged nodes keep their objects, value specs come from this graph."""
    L = N.lib()
    text = _graph_json(graph).encode()
    cap = 1 << 16
    n = ctypes.c_size_t(0)
    while True:
        buf = ctypes.create_string_buffer(cap)
        L.tb_graph_compile(text, passes.encode(), buf, cap, ctypes.byref(n))
        if n.value < cap:
            break
        cap = n.value + 1
    res = json.loads(buf.raw[:n.value].decode())
    if "error" in res:
        e = res["error"]
        raise ExecutionError(e["operator"], e["phase"], e["message"], N.TB_ERR_INVALID)
    out = res["graph"]
    originals = {(n.id, n.operator, tuple(n.inputs), tuple(n.outputs)): n for n in graph.nodes}
    nodes = [originals.get((j["id"], j["operator"], tuple(j["inputs"]), tuple(j["outputs"])))
             or GraphNode(j["id"], j["operator"], j["inputs"], j["outputs"], j["attrs"]) for j in out["nodes"]]
    values = {v: graph.values[v] for v in out["values"]}
    reports = [PassReport(r["name"], r["changed"], r["notes"]) for r in res["reports"]]
    return Graph(list(graph.inputs), list(graph.outputs), values, nodes), reports


def validate(graph: Graph) -> None:
    """Every graph input/output has a spec; every node reads only produced values."""
    _run_passes(graph, "check")


def dead_code_eliminate(graph: Graph) -> tuple[Graph, bool]:
    g, reports = _run_passes(graph, "dce")
    return g, reports[0].changed


def fuse_gemm_epilogues(graph: Graph) -> tuple[Graph, list]:
    """gemm -> [broadcast.add(bias fp32 [N])] -> [gelu | silu]  =>  gemm.bias_act."""
    g, reports = _run_passes(graph, "fusion.gemm_epilogue")
    return g, reports[0].notes


def fuse_attention(graph: Graph) -> tuple[Graph, list]:
    """gemm(Q, K; transpose_rhs) -> softmax(last axis) -> gemm(P, V)  =>  attention.fused(Q, K, V)."""
    g, reports = _run_passes(graph, "fusion.attention")
    return g, reports[0].notes


class ExecutionPlan:
    """ExecutionPlan (lib.rs:176-276): the optimised graph and its pass reports."""

    def __init__(self, graph: Graph, reports: list):
        self.graph = graph
        self.reports = reports

    def node_count(self) -> int:
        return len(self.graph.nodes)

    def execute(self, runtime: Runtime, bindings: dict, _outputs: Optional[dict] = None) -> ExecutionHandle:
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
            # Fused nodes ("gemm.bias_act", "attention.fused") are operators of the router too.
            request = OpRequest(node.operator, inputs, specs, dict(node.attrs))
            out = _outputs.get(node.outputs[0]) if _outputs else None
            handle = runtime.execute(request) if out is None else runtime.execute(request, output=out)
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
        handle = ExecutionHandle(outs, "b200/graph", "graph.plan", last.event if last else None)
        handle.values = env
        return handle

    def capture(self, runtime: Runtime, bindings: dict) -> "CapturedPlan":
        """The plan as a CUDA graph: one eager run allocates every node's output (and any
        per-stream scratch its operators use), then the same nodes, writing into those
        outputs, are captured on the runtime's stream. CapturedPlan.launch() replays them
        with one launch, on the bound input tensors (upload new contents to replay on new
        data) and into the same output tensors."""
        eager = self.execute(runtime, bindings)
        eager.wait()
        produced = {v: t for v, t in eager.values.items() if v not in bindings}
        runtime.session.capture_begin(runtime.stream)
        try:
            self.execute(runtime, bindings, _outputs=produced)
        finally:
            graph = runtime.session.capture_end(runtime.stream)
        return CapturedPlan(runtime, graph, eager.outputs)


class CapturedPlan:
    """A compiled plan captured as a CUDA graph (ExecutionPlan.capture)."""

    def __init__(self, runtime: Runtime, graph, outputs: list):
        self.runtime, self.graph, self.outputs = runtime, graph, outputs

    def launch(self) -> None:
        """Enqueues one replay on the runtime's stream."""
        self.graph.launch(self.runtime.stream)


def compile(graph: Graph) -> ExecutionPlan:
    """Runtime::compile (lib.rs:3472-3483): validate, DCE, fusion; an empty result is an error.
    The passes run in the native library (tb_graph_compile)."""
    g, reports = _run_passes(graph, "compile")
    return ExecutionPlan(g, reports)


__all__ = ["GraphNode", "Graph", "PassReport", "ExecutionPlan", "CapturedPlan", "compile", "validate",
           "dead_code_eliminate",
           "fuse_gemm_epilogues", "fuse_attention"]
