// CUDA graphs over a session stream: the device work enqueued on a stream between
// tb_capture_begin and tb_capture_end (operators, device-to-device copies, memsets,
// event records) becomes one graph that tb_graph_exec_launch replays with a single
// launch. No counterpart in the reference, whose runtime launches every kernel from
// the host (titan-backend-cuda/src/lib.rs:1413-1507); here it serves launch-bound
// sequences of small operators.
//
// Capture is per thread (CU_STREAM_CAPTURE_MODE_THREAD_LOCAL): other host threads keep
// using the session meanwhile. Work that is not stream-ordered device work invalidates
// the capture and tb_capture_end reports it: host-staged uploads and downloads (their
// host side runs at enqueue time), waits on the host, and an operator's first use of
// per-stream scratch memory (it allocates), so such an operator runs once before capture.
// A replay reads and writes the same device buffers the captured work named.
#include "internal.hpp"

namespace tb {

struct GraphExec : RefCounted {
  Session* session = nullptr;
  CUgraphExec exec = nullptr;
};

}  // namespace tb

using namespace tb;

extern "C" {

tb_status tb_capture_begin(tb_session* session, tb_stream* stream) {
  Session* s = reinterpret_cast<Session*>(session);
  if (!s) return set_error(TB_ERR_INVALID, "capture", "null session");
  Stream* st = nullptr;
  tb_status rc = check_stream(s, stream, &st);
  if (rc) return rc;
  rc = activate(s);
  if (rc) return rc;
  TB_CU("cuStreamBeginCapture", driver()->cuStreamBeginCapture_v2(st->raw, CU_STREAM_CAPTURE_MODE_THREAD_LOCAL));
  return TB_OK;
}

tb_status tb_capture_end(tb_session* session, tb_stream* stream, tb_graph_exec** out) {
  Session* s = reinterpret_cast<Session*>(session);
  if (!s || !out) return set_error(TB_ERR_INVALID, "capture", "null argument");
  *out = nullptr;
  Stream* st = nullptr;
  tb_status rc = check_stream(s, stream, &st);
  if (rc) return rc;
  rc = activate(s);
  if (rc) return rc;
  const DriverApi* d = driver();
  CUgraph graph = nullptr;
  // Ends the capture in every case; an invalidated capture (a call that cannot be
  // captured ran meanwhile) reports the driver's error and yields no graph.
  TB_CU("cuStreamEndCapture", d->cuStreamEndCapture(st->raw, &graph));
  if (!graph) return set_error(TB_ERR_INVALID, "capture", "nothing was captured");
  CUgraphExec exec = nullptr;
  const CUresult r = d->cuGraphInstantiateWithFlags(&exec, graph, 0);
  d->cuGraphDestroy(graph);
  if (r != CUDA_SUCCESS) return cu_error("cuGraphInstantiate", r);
  GraphExec* g = new GraphExec();
  g->session = s;
  g->exec = exec;
  s->refs.fetch_add(1);
  *out = reinterpret_cast<tb_graph_exec*>(g);
  return TB_OK;
}

tb_status tb_graph_exec_launch(tb_session* session, tb_graph_exec* graph, tb_stream* stream) {
  Session* s = reinterpret_cast<Session*>(session);
  GraphExec* g = reinterpret_cast<GraphExec*>(graph);
  if (!s || !g) return set_error(TB_ERR_INVALID, "launch", "null argument");
  if (g->session != s) return set_error(TB_ERR_INVALID, "launch", "graph belongs to another session");
  Stream* st = nullptr;
  tb_status rc = check_stream(s, stream, &st);
  if (rc) return rc;
  rc = activate(s);
  if (rc) return rc;
  TB_CU("cuGraphLaunch", driver()->cuGraphLaunch(g->exec, st->raw));
  return TB_OK;
}

void tb_graph_exec_release(tb_graph_exec* graph) {
  GraphExec* g = reinterpret_cast<GraphExec*>(graph);
  if (!g || g->refs.fetch_sub(1) != 1) return;
  Session* s = g->session;
  const DriverApi* d = driver();
  if (d && g->exec) {
    d->cuCtxSetCurrent(s->context);
    d->cuGraphExecDestroy(g->exec);  // a replay still in flight completes; the driver frees it then
  }
  delete g;
  tb_session_release(reinterpret_cast<tb_session*>(s));
}

}  // extern "C"
