// Graph compilation for the hot-path operators: Runtime::compile
// (projects/titan-runtime/src/lib.rs:3472-3483) over the Graph IR
// (projects/titan-graph/src/graph.rs:72-105), with the core pipeline's shape
// (projects/titan-graph/src/optimize.rs:23-60: validate, dead-code elimination, fusion,
// validate) and two fusions for the B200 kernels in place of the reference's
// elementwise -> relu annotation:
//
//   fusion.gemm_epilogue  a bf16 rank-2 `gemm` whose only consumer is `broadcast.add` of
//                         an F32 [N] bias and/or `gelu` / `silu` (each intermediate used
//                         once and not a graph output) becomes one `gemm.bias_act` node
//                         with the gemm's id, attributes transpose_lhs / transpose_rhs
//                         (as bools, when given) and `activation`;
//   fusion.attention      S = gemm(Q, K; transpose_rhs), P = softmax(S; last axis),
//                         O = gemm(P, V) on bf16 [T, D] values, S and P used only in the
//                         chain and not outputs, becomes `attention.fused(Q, K, V)` with
//                         the id of the P V gemm and attribute scale = 1.0.
//
// Each fusion scans the nodes once in order and rewrites in place, which finds the same
// chains as rewriting one at a time and rescanning (see Index below); a graph of a few
// thousand nodes compiles in milliseconds. The graph crosses the C ABI as JSON:
//   {"inputs": [ids], "outputs": [ids], "values": {"<id>": {"dtype": "BF16", "shape": [..]}},
//    "nodes": [{"id": n, "operator": "gemm", "inputs": [ids], "outputs": [ids], "attrs": {..}}]}
// Attribute values may be plain JSON or serde's externally tagged AttrValue (a serde_json
// dump of the reference's Graph); nodes the passes create are written in the same form,
// kept nodes exactly as given. The result comes back as
// {"graph": {... "values": [ids still present] ...}, "reports":
// [{"name", "changed", "notes"}]}, or {"error": {"operator", "phase", "message"}}.
#include <algorithm>
#include <set>
#include <unordered_map>
#include <unordered_set>

#include "internal.hpp"
#include "json.hpp"

namespace {

using tb::json::Json;

struct Spec {
  std::string dtype;
  std::vector<long long> shape;
};

struct Node {
  long long id = 0;
  std::string op;
  std::vector<long long> in, out;
  Json attrs;      // an object of plain values, what the passes read
  Json raw_attrs;  // the attributes as given, written back for nodes the passes keep
  bool rewritten = false;
};

struct Graph {
  std::vector<long long> inputs, outputs;
  std::map<long long, Spec> values;
  std::vector<Node> nodes;
  bool tagged = false;  // attributes arrive as serde's externally tagged AttrValue
};

struct Report {
  std::string name;
  bool changed = false;
  std::vector<std::string> notes;
};

// A compile failure: ExecutionError{operator, phase: "compile", message}.
struct Failure {
  std::string op, message;
};

bool to_int(const Json& v, long long& out) {
  if (v.kind != Json::Int) return false;
  char* end = nullptr;
  errno = 0;
  out = strtoll(v.text.c_str(), &end, 10);
  return errno == 0 && end && *end == '\0';
}

bool int_list(const Json& v, std::vector<long long>& out) {
  if (v.kind != Json::Array) return false;
  out.clear();
  for (const Json& x : v.items) {
    long long i;
    if (!to_int(x, i)) return false;
    out.push_back(i);
  }
  return true;
}

const Json* member(const Json& obj, const char* key) {
  auto it = obj.members.find(key);
  return it == obj.members.end() ? nullptr : &it->second;
}

// Python truthiness of an attribute value (absent is false).
bool truthy(const Json* v) {
  if (!v) return false;
  switch (v->kind) {
    case Json::Null: return false;
    case Json::Bool: return v->flag;
    case Json::Int: return v->text != "0";
    case Json::Float: return v->number != 0.0;
    case Json::String: return !v->text.empty();
    case Json::Array: return !v->items.empty();
    case Json::Object: return !v->members.empty();
  }
  return false;
}

// titan_types::AttrValue (titan-types/src/lib.rs:140-147) as serde_json writes it:
// {"Bool": b}, {"Int": i}, {"Float": f64 bits as u64}, {"String": s}, {"Ints": [..]},
// {"Strings": [..]}. Such a value becomes the plain JSON value; anything else is kept.
bool untag(const Json& v, Json& plain) {
  if (v.kind != Json::Object || v.members.size() != 1) return false;
  const std::string& tag = v.members.begin()->first;
  const Json& x = v.members.begin()->second;
  if ((tag == "Bool" && x.kind == Json::Bool) || (tag == "Int" && x.kind == Json::Int) ||
      (tag == "String" && x.kind == Json::String) || ((tag == "Ints" || tag == "Strings") && x.kind == Json::Array)) {
    plain = x;
    return true;
  }
  if (tag == "Float" && x.kind == Json::Int) {
    unsigned long long bits = strtoull(x.text.c_str(), nullptr, 10);
    double d;
    memcpy(&d, &bits, sizeof d);
    plain = Json();
    plain.kind = Json::Float;
    plain.number = d;
    return true;
  }
  return false;
}

// A plain attribute value in the form the input used.
Json attr_out(const Json& plain, bool tagged) {
  if (!tagged) return plain;
  Json x = plain, w;
  w.kind = Json::Object;
  const char* tag = plain.kind == Json::Bool ? "Bool" : plain.kind == Json::Int ? "Int" : "String";
  if (plain.kind == Json::Float) {
    unsigned long long bits;
    memcpy(&bits, &plain.number, sizeof bits);
    x = Json();
    x.kind = Json::Int;
    x.text = std::to_string(bits);
    tag = "Float";
  }
  w.members[tag] = x;
  return w;
}

bool parse_graph(const Json& j, Graph& g, std::string& err) {
  if (j.kind != Json::Object) return err = "graph must be an object", false;
  const Json *in = member(j, "inputs"), *out = member(j, "outputs"), *vals = member(j, "values"),
             *nodes = member(j, "nodes");
  if (!in || !int_list(*in, g.inputs)) return err = "inputs must be a list of integer value ids", false;
  if (!out || !int_list(*out, g.outputs)) return err = "outputs must be a list of integer value ids", false;
  if (!vals || vals->kind != Json::Object) return err = "values must map value ids to specs", false;
  for (const auto& kv : vals->members) {
    char* end = nullptr;
    long long id = strtoll(kv.first.c_str(), &end, 10);
    if (kv.first.empty() || *end != '\0') return err = "value id " + kv.first + " is not an integer", false;
    const Json *dt = member(kv.second, "dtype"), *shape = member(kv.second, "shape");
    Spec sp;
    if (kv.second.kind != Json::Object || !dt || dt->kind != Json::String || !shape || !int_list(*shape, sp.shape))
      return err = "value " + kv.first + " needs a dtype string and an integer shape", false;
    sp.dtype = dt->text;
    g.values[id] = sp;
  }
  if (!nodes || nodes->kind != Json::Array) return err = "nodes must be a list", false;
  for (const Json& n : nodes->items) {
    Node node;
    const Json *id = member(n, "id"), *op = member(n, "operator"), *ni = member(n, "inputs"),
               *no = member(n, "outputs"), *at = member(n, "attrs");
    if (n.kind != Json::Object || !id || !to_int(*id, node.id) || !op || op->kind != Json::String || !ni ||
        !int_list(*ni, node.in) || !no || !int_list(*no, node.out))
      return err = "every node needs an integer id, an operator string and integer input/output lists", false;
    node.op = op->text;
    if (at && at->kind != Json::Object) return err = "node attrs must be an object", false;
    node.attrs.kind = Json::Object;
    node.raw_attrs.kind = Json::Object;
    if (at) {
      node.raw_attrs = *at;
      for (const auto& kv : at->members) {
        Json plain;
        const bool t = untag(kv.second, plain);
        g.tagged = g.tagged || t;
        node.attrs.members[kv.first] = t ? plain : kv.second;
      }
    }
    g.nodes.push_back(std::move(node));
  }
  return true;
}

bool contains(const std::vector<long long>& v, long long x) { return std::find(v.begin(), v.end(), x) != v.end(); }

// Graph::validate (titan-graph/src/graph.rs:185-214): at least one output, a spec for
// every graph input and output, unique node ids; then every node reads only values
// produced before it and writes values that have a spec.
bool validate(const Graph& g, Failure& f) {
  if (g.outputs.empty()) return f = {"graph.validate", "graph must declare at least one output"}, false;
  for (const auto* list : {&g.inputs, &g.outputs})
    for (long long v : *list)
      if (!g.values.count(v)) return f = {"graph.validate", "value " + std::to_string(v) + " has no TensorSpec"}, false;
  std::set<long long> ids;
  for (const Node& n : g.nodes)
    if (!ids.insert(n.id).second) return f = {"graph.validate", "duplicate node id " + std::to_string(n.id)}, false;
  std::set<long long> produced(g.inputs.begin(), g.inputs.end());
  for (const Node& n : g.nodes) {
    for (long long v : n.in)
      if (!produced.count(v))
        return f = {n.op, "node " + std::to_string(n.id) + " reads value " + std::to_string(v) +
                              " before it is produced"},
               false;
    for (long long v : n.out) {
      if (!g.values.count(v)) return f = {n.op, "missing TensorSpec for value " + std::to_string(v)}, false;
      produced.insert(v);
    }
  }
  return true;
}

bool dead_code_eliminate(Graph& g) {
  std::set<long long> live(g.outputs.begin(), g.outputs.end());
  std::vector<Node> kept;
  for (auto it = g.nodes.rbegin(); it != g.nodes.rend(); ++it) {
    bool used = false;
    for (long long o : it->out) used = used || live.count(o);
    if (used) {
      kept.push_back(*it);
      live.insert(it->in.begin(), it->in.end());
    }
  }
  std::reverse(kept.begin(), kept.end());
  const bool changed = kept.size() != g.nodes.size();
  g.nodes = std::move(kept);
  return changed;
}

// The fusions rewrite in place: a fused node takes the position of the last node of its
// chain (where every value it reads has been produced, a bias made between the gemm and
// the add included) and the other nodes of the chain are marked dead, so positions stay
// valid. The index
// holds the consumers of each value (live positions; a node once however often it reads
// the value) and is updated with each rewrite.
//
// Both fusions scan the nodes once, in order. Rescanning from the first node after each
// rewrite (the plain statement of "one rewrite, then rescan") finds nothing more: a
// rewrite keeps every surviving value's consumer count (the fused node reads what the
// chain read from outside it, at one position), and the only consumers that change
// operator name are chain nodes, which no earlier chain could have matched (they are
// gemm / broadcast.add / gelu / silu / softmax nodes whose inputs an earlier gemm would
// have needed as its own single consumer).
struct Index {
  std::unordered_map<long long, std::vector<size_t>> users;
  std::unordered_set<long long> outputs;
  std::vector<bool> dead;
  explicit Index(const Graph& g) : outputs(g.outputs.begin(), g.outputs.end()), dead(g.nodes.size(), false) {
    for (size_t i = 0; i < g.nodes.size(); ++i)
      for (long long v : g.nodes[i].in) add(v, i);
  }
  void add(long long v, size_t i) {
    std::vector<size_t>& u = users[v];
    if (std::find(u.begin(), u.end(), i) == u.end()) u.push_back(i);
  }
  std::vector<size_t> consumers(long long v) const {
    std::vector<size_t> out;
    auto it = users.find(v);
    if (it != users.end())
      for (size_t i : it->second)
        if (!dead[i]) out.push_back(i);
    std::sort(out.begin(), out.end());
    return out;
  }
};

const Spec* spec_of(const Graph& g, long long v) {
  auto it = g.values.find(v);
  return it == g.values.end() ? nullptr : &it->second;
}

void drop_dead(Graph& g, const Index& ix) {
  std::vector<Node> nodes;
  nodes.reserve(g.nodes.size());
  for (size_t i = 0; i < g.nodes.size(); ++i)
    if (!ix.dead[i]) nodes.push_back(std::move(g.nodes[i]));
  g.nodes = std::move(nodes);
}

// gemm -> [broadcast.add(bias F32 [N])] -> [gelu | silu]  =>  gemm.bias_act
std::vector<std::string> fuse_gemm_epilogues(Graph& g) {
  std::vector<std::string> notes;
  Index ix(g);
  for (size_t gi = 0; gi < g.nodes.size(); ++gi) {
    if (ix.dead[gi]) continue;
    const Node& gm = g.nodes[gi];
    if (gm.op != "gemm" || gm.out.size() != 1 || gm.in.size() != 2) continue;
    const Spec* spec = spec_of(g, gm.out[0]);
    if (!spec || spec->dtype != "BF16" || spec->shape.size() != 2) continue;
    std::vector<size_t> absorbed;
    long long tail = gm.out[0], bias = 0;
    bool has_bias = false;
    std::string act = "none";
    std::vector<size_t> users = ix.consumers(tail);
    if (!ix.outputs.count(tail) && users.size() == 1 && g.nodes[users[0]].op == "broadcast.add" &&
        g.nodes[users[0]].in.size() == 2 && g.nodes[users[0]].out.size() == 1) {
      const Node& add = g.nodes[users[0]];
      const long long other = add.in[0] == tail ? add.in[1] : add.in[0];
      const Spec *bspec = spec_of(g, other), *aspec = spec_of(g, add.out[0]);
      if (bspec && aspec && bspec->dtype == "F32" && bspec->shape == std::vector<long long>{spec->shape[1]} &&
          aspec->dtype == "BF16") {
        absorbed.push_back(users[0]);
        bias = other;
        has_bias = true;
        tail = add.out[0];
        users = ix.consumers(tail);
      }
    }
    if (!ix.outputs.count(tail) && users.size() == 1 &&
        (g.nodes[users[0]].op == "gelu" || g.nodes[users[0]].op == "silu") && g.nodes[users[0]].out.size() == 1) {
      const Spec* ospec = spec_of(g, g.nodes[users[0]].out[0]);
      if (ospec && ospec->dtype == "BF16") {
        absorbed.push_back(users[0]);
        act = g.nodes[users[0]].op;
        tail = g.nodes[users[0]].out[0];
      }
    }
    if (absorbed.empty()) continue;
    Node fused;
    fused.id = gm.id;
    fused.op = "gemm.bias_act";
    fused.rewritten = true;
    fused.in = gm.in;
    if (has_bias) fused.in.push_back(bias);
    fused.out = {tail};
    fused.attrs.kind = Json::Object;
    for (const char* key : {"transpose_lhs", "transpose_rhs"}) {
      const Json* v = member(gm.attrs, key);
      if (!v) continue;
      Json b;
      b.kind = Json::Bool;
      b.flag = truthy(v);
      fused.attrs.members[key] = b;
    }
    Json a;
    a.kind = Json::String;
    a.text = act;
    fused.attrs.members["activation"] = a;
    std::string note = "fused node " + std::to_string(gm.id) + " (gemm) with ";
    for (size_t i = 0; i < absorbed.size(); ++i) {
      const Node& n = g.nodes[absorbed[i]];
      note += (i ? ", " : "") + std::string("node ") + std::to_string(n.id) + " (" + n.op + ")";
    }
    notes.push_back(note + " into gemm.bias_act");
    // Values that only lived inside the chain: the gemm's output and every absorbed
    // node's output but the last.
    g.values.erase(gm.out[0]);
    for (size_t i = 0; i + 1 < absorbed.size(); ++i) g.values.erase(g.nodes[absorbed[i]].out[0]);
    // The fused node replaces the chain's last node; the gemm and the other absorbed
    // nodes go.
    const size_t last = absorbed.back();
    ix.dead[gi] = true;
    for (size_t i = 0; i + 1 < absorbed.size(); ++i) ix.dead[absorbed[i]] = true;
    for (long long v : fused.in) ix.add(v, last);
    g.nodes[last] = std::move(fused);
  }
  drop_dead(g, ix);
  return notes;
}

bool last_axis_softmax(const Node& n, long long rank) {
  for (const auto& kv : n.attrs.members)
    if (kv.first != "axis") return false;
  const Json* axis = member(n.attrs, "axis");
  if (!axis) return true;
  long long a;
  return to_int(*axis, a) && a == rank - 1;
}

// gemm(Q, K; transpose_rhs) -> softmax(last axis) -> gemm(P, V)  =>  attention.fused(Q, K, V)
std::vector<std::string> fuse_attention(Graph& g) {
  std::vector<std::string> notes;
  auto bf16_2d = [&](long long v) {
    const Spec* s = spec_of(g, v);
    return s && s->dtype == "BF16" && s->shape.size() == 2 ? s : nullptr;
  };
  Index ix(g);
  for (size_t gi = 0; gi < g.nodes.size(); ++gi) {
    if (ix.dead[gi]) continue;
    const Node& gm = g.nodes[gi];
    if (gm.op != "gemm" || gm.in.size() != 2 || gm.out.size() != 1 || !truthy(member(gm.attrs, "transpose_rhs")) ||
        truthy(member(gm.attrs, "transpose_lhs")))
      continue;
    const long long q = gm.in[0], k = gm.in[1], s_val = gm.out[0];
    const Spec *qs = bf16_2d(q), *ks = bf16_2d(k), *ss = bf16_2d(s_val);
    if (!qs || !ks || !ss) continue;
    const long long tq = qs->shape[0], d = qs->shape[1], tk = ks->shape[0], dk = ks->shape[1];
    std::vector<size_t> users = ix.consumers(s_val);
    if (ix.outputs.count(s_val) || users.size() != 1 || g.nodes[users[0]].op != "softmax" ||
        !last_axis_softmax(g.nodes[users[0]], 2) || g.nodes[users[0]].out.empty())
      continue;
    const size_t si = users[0];
    const long long p_val = g.nodes[si].out[0];
    const Spec* ps = spec_of(g, p_val);
    if (!ps || ps->dtype != "BF16" || ps->shape != std::vector<long long>{tq, tk}) continue;
    users = ix.consumers(p_val);
    if (ix.outputs.count(p_val) || users.size() != 1) continue;
    const size_t pi = users[0];
    const Node& pv = g.nodes[pi];
    if (pv.op != "gemm" || pv.in[0] != p_val || pv.in.size() != 2 || truthy(member(pv.attrs, "transpose_lhs")) ||
        truthy(member(pv.attrs, "transpose_rhs")) || pv.out.empty())
      continue;
    const long long v = pv.in[1];
    const Spec *vs = spec_of(g, v), *os = spec_of(g, pv.out[0]);
    if (!vs || !os || vs->dtype != "BF16" || os->dtype != "BF16" || vs->shape != std::vector<long long>{tk, d} ||
        os->shape != std::vector<long long>{tq, d} || dk != d)
      continue;
    // The fused node sits where P V was: Q, K and V are all produced by then.
    Node fused;
    fused.id = pv.id;
    fused.op = "attention.fused";
    fused.rewritten = true;
    fused.in = {q, k, v};
    fused.out = {pv.out[0]};
    fused.attrs.kind = Json::Object;
    Json scale;
    scale.kind = Json::Float;
    scale.number = 1.0;
    fused.attrs.members["scale"] = scale;
    notes.push_back("fused node " + std::to_string(gm.id) + " (gemm), node " + std::to_string(g.nodes[si].id) +
                    " (softmax) and node " + std::to_string(pv.id) + " (gemm) into attention.fused [" +
                    std::to_string(tq) + "x" + std::to_string(tk) + ", D=" + std::to_string(d) + "]");
    g.values.erase(s_val);
    g.values.erase(p_val);
    ix.dead[gi] = ix.dead[si] = true;
    ix.add(q, pi);
    ix.add(k, pi);
    g.nodes[pi] = std::move(fused);
  }
  drop_dead(g, ix);
  return notes;
}

Json int_array(const std::vector<long long>& v) {
  Json a;
  a.kind = Json::Array;
  for (long long x : v) {
    Json i;
    i.kind = Json::Int;
    i.text = std::to_string(x);
    a.items.push_back(i);
  }
  return a;
}

Json str(const std::string& s) {
  Json j;
  j.kind = Json::String;
  j.text = s;
  return j;
}

std::string result_json(const Graph& g, const std::vector<Report>& reports) {
  Json graph, out, reps;
  graph.kind = out.kind = Json::Object;
  reps.kind = Json::Array;
  graph.members["inputs"] = int_array(g.inputs);
  graph.members["outputs"] = int_array(g.outputs);
  std::vector<long long> ids;
  for (const auto& kv : g.values) ids.push_back(kv.first);
  graph.members["values"] = int_array(ids);
  Json nodes;
  nodes.kind = Json::Array;
  for (const Node& n : g.nodes) {
    Json j;
    j.kind = Json::Object;
    Json id;
    id.kind = Json::Int;
    id.text = std::to_string(n.id);
    j.members["id"] = id;
    j.members["operator"] = str(n.op);
    j.members["inputs"] = int_array(n.in);
    j.members["outputs"] = int_array(n.out);
    if (n.rewritten) {
      Json attrs;
      attrs.kind = Json::Object;
      for (const auto& kv : n.attrs.members) attrs.members[kv.first] = attr_out(kv.second, g.tagged);
      j.members["attrs"] = attrs;
    } else {
      j.members["attrs"] = n.raw_attrs;
    }
    nodes.items.push_back(j);
  }
  graph.members["nodes"] = nodes;
  for (const Report& r : reports) {
    Json j, notes, changed;
    j.kind = Json::Object;
    notes.kind = Json::Array;
    for (const auto& s : r.notes) notes.items.push_back(str(s));
    changed.kind = Json::Bool;
    changed.flag = r.changed;
    j.members["name"] = str(r.name);
    j.members["changed"] = changed;
    j.members["notes"] = notes;
    reps.items.push_back(j);
  }
  out.members["graph"] = graph;
  out.members["reports"] = reps;
  std::string text;
  tb::json::emit(text, out);
  return text;
}

std::string error_json(const Failure& f) {
  Json e, o;
  e.kind = o.kind = Json::Object;
  e.members["operator"] = str(f.op);
  e.members["phase"] = str("compile");
  e.members["message"] = str(f.message);
  o.members["error"] = e;
  std::string text;
  tb::json::emit(text, o);
  return text;
}

tb_status give(const std::string& text, char* out, size_t cap, size_t* len, tb_status status) {
  if (len) *len = text.size();
  if (!out || cap <= text.size())
    return tb::set_error(TB_ERR_INVALID, "compile",
                         "output buffer too small: " + std::to_string(text.size() + 1) + " bytes needed");
  memcpy(out, text.data(), text.size());
  out[text.size()] = '\0';
  return status;
}

}  // namespace

extern "C" tb_status tb_graph_compile(const char* graph_json, const char* passes, char* out, size_t cap,
                                      size_t* len) {
  Failure f;
  auto fail = [&](const Failure& failure) {
    std::string text = error_json(failure);
    tb_status st = give(text, out, cap, len, TB_ERR_INVALID);
    if (st == TB_ERR_INVALID && len && *len < cap)  // the error object fits: report the compile failure itself
      tb::set_error(TB_ERR_INVALID, "compile", failure.op + ": " + failure.message);
    return st;
  };
  if (!graph_json) return fail({"graph", "graph JSON is null"});
  Json j;
  std::string err;
  const std::string text = graph_json;
  if (!tb::json::valid_utf8(text)) return fail({"graph", "graph JSON: not valid UTF-8"});
  if (!tb::json::Parser(text).parse(j, err)) return fail({"graph", "graph JSON: " + err});
  Graph g;
  if (!parse_graph(j, g, err)) return fail({"graph", err});
  const std::string list = passes && *passes ? passes : "compile";
  std::vector<std::string> steps;
  for (size_t b = 0; b <= list.size();) {
    size_t e = list.find(',', b);
    if (e == std::string::npos) e = list.size();
    steps.push_back(list.substr(b, e - b));
    b = e + 1;
  }
  if (steps.size() == 1 && steps[0] == "compile")
    steps = {"validate", "dce", "fusion.gemm_epilogue", "fusion.attention", "check", "nonempty"};
  std::vector<Report> reports;
  for (const std::string& step : steps) {
    if (step == "validate" || step == "check") {
      if (!validate(g, f)) return fail(f);
      if (step == "validate") reports.push_back({"validate", false, {"schema and constraints ok"}});
    } else if (step == "dce") {
      reports.push_back({"dce", dead_code_eliminate(g), {"removed unreachable pure nodes"}});
    } else if (step == "fusion.gemm_epilogue" || step == "fusion.attention") {
      std::vector<std::string> notes = step == "fusion.attention" ? fuse_attention(g) : fuse_gemm_epilogues(g);
      reports.push_back({step, !notes.empty(), notes});
    } else if (step == "nonempty") {
      if (g.nodes.empty()) return fail({"graph.empty", "graph has no nodes after passes"});
    } else {
      return fail({"graph", "unknown pass " + step});
    }
  }
  return give(result_json(g, reports), out, cap, len, TB_OK);
}
