// HAL session layer of libtitan_b200: driver discovery, sessions, buffers,
// streams, events, module load and ABI-payload launch.
//
// Behaviour follows the titan.rs CUDA backend (titan-backend-cuda/src/lib.rs):
// the same ownership rules, the same rejection messages and the same
// upload/download completion semantics, over the Driver API. Differences that
// are deliberate: modules are cached per session by content (the reference
// JITs on every execute, lib.rs:1339), `load` accepts sm_100a cubins as well
// as PTX, and buffers are freed when their last handle is released.
#include <dlfcn.h>

#include <cinttypes>
#include <cstdio>
#include <cstdlib>

#include "internal.hpp"

namespace tb {

// ---------------------------------------------------------------- errors
namespace {
thread_local std::string g_op;
thread_local std::string g_detail;
thread_local std::string g_candidate;
thread_local uint64_t g_launches = 0;
std::atomic<uint64_t> g_next_identity{1};
}  // namespace

tb_status set_error(tb_status status, const char* operation, const std::string& detail) {
  g_op = operation ? operation : "";
  g_detail = detail;
  return status;
}

tb_status cu_error(const char* operation, CUresult result) {
  const DriverApi* d = driver();
  const char* name = nullptr;
  const char* text = nullptr;
  if (d && d->cuGetErrorName) d->cuGetErrorName(result, &name);
  if (d && d->cuGetErrorString) d->cuGetErrorString(result, &text);
  char buf[256];
  snprintf(buf, sizeof buf, "CUDA driver status %d (%s: %s)", (int)result, name ? name : "?", text ? text : "?");
  tb_status st = TB_ERR_CUDA;
  if (result == CUDA_ERROR_OUT_OF_MEMORY) st = TB_ERR_OUT_OF_MEMORY;
  if (result == CUDA_ERROR_NO_DEVICE || result == CUDA_ERROR_NOT_INITIALIZED) st = TB_ERR_DRIVER_UNAVAILABLE;
  return set_error(st, operation, buf);
}

void note_launch(const char* candidate) {
  g_candidate = candidate ? candidate : "";
  ++g_launches;
}

void note_candidate(const char* candidate) { g_candidate = candidate ? candidate : ""; }

// ---------------------------------------------------------------- driver
namespace {
std::once_flag g_driver_once;
DriverApi g_driver;
bool g_driver_ok = false;
std::string g_driver_op, g_driver_detail;

void open_driver() {
  void* h = dlopen("libcuda.so.1", RTLD_NOW | RTLD_LOCAL);
  if (!h) {
    g_driver_op = "load_driver";
    const char* e = dlerror();
    g_driver_detail = e ? e : "libcuda.so.1 not found";
    return;
  }
  g_driver.handle = h;
#define TB_RESOLVE(name)                                                   \
  g_driver.name = reinterpret_cast<decltype(g_driver.name)>(dlsym(h, #name)); \
  if (!g_driver.name) {                                                    \
    g_driver_op = "load_driver";                                           \
    g_driver_detail = "missing driver symbol " #name;                      \
    return;                                                                \
  }
  TB_CU_FUNCS(TB_RESOLVE)
#undef TB_RESOLVE
  CUresult r = g_driver.cuInit(0);
  if (r != CUDA_SUCCESS) {
    g_driver_op = "cuInit";
    g_driver_detail = "CUDA driver status " + std::to_string((int)r);
    return;
  }
  int count = 0;
  r = g_driver.cuDeviceGetCount(&count);
  if (r != CUDA_SUCCESS) {
    g_driver_op = "cuDeviceGetCount";
    g_driver_detail = "CUDA driver status " + std::to_string((int)r);
    return;
  }
  g_driver_ok = true;
}
}  // namespace

const DriverApi* driver() {
  std::call_once(g_driver_once, open_driver);
  if (!g_driver_ok) {
    set_error(TB_ERR_DRIVER_UNAVAILABLE, g_driver_op.c_str(), g_driver_detail);
    return nullptr;
  }
  return &g_driver;
}

tb_status activate(Session* s) {
  const DriverApi* d = driver();
  if (!d) return TB_ERR_DRIVER_UNAVAILABLE;
  TB_CU("cuCtxSetCurrent", d->cuCtxSetCurrent(s->context));
  return TB_OK;
}

// ---------------------------------------------------------------- registries
tb_status check_buffer(Session* s, tb_buffer* handle, Buffer** out) {
  Buffer* b = reinterpret_cast<Buffer*>(handle);
  if (!b) return set_error(TB_ERR_INVALID, "buffer", "null buffer");
  std::lock_guard<std::mutex> lock(s->mu);
  if (!s->buffers.count(b)) {
    // A buffer of another session: cross-device when the ordinal differs
    // (titan-backend-cuda/src/lib.rs:1179-1181), otherwise foreign (:1183-1189).
    bool other_device = false;
    if (b->session && b->session != s && b->session->ordinal != s->ordinal) other_device = true;
    return set_error(TB_ERR_FOREIGN, "buffer", other_device ? "cross-device buffer" : "foreign buffer");
  }
  *out = b;
  return TB_OK;
}

tb_status check_stream(Session* s, tb_stream* handle, Stream** out) {
  Stream* st = reinterpret_cast<Stream*>(handle);
  if (!st) return set_error(TB_ERR_INVALID, "stream", "null stream");
  std::lock_guard<std::mutex> lock(s->mu);
  if (!s->streams.count(st)) return set_error(TB_ERR_FOREIGN, "stream", "foreign stream");
  *out = st;
  return TB_OK;
}

tb_status check_event(Session* s, tb_event* handle, Event** out) {
  Event* e = reinterpret_cast<Event*>(handle);
  if (!e) return set_error(TB_ERR_INVALID, "event", "null event");
  std::lock_guard<std::mutex> lock(s->mu);
  if (!s->events.count(e)) return set_error(TB_ERR_FOREIGN, "event", "foreign event");
  *out = e;
  return TB_OK;
}

tb_status consume_device_status(Session* s) {
  if (!s->status.host) return TB_OK;
  uint32_t code = *s->status.host;
  if (code == 0) return TB_OK;
  *s->status.host = 0;
  char buf[160];
  snprintf(buf, sizeof buf,
           "a kernel gave up a bounded device-side wait (code 0x%08x); its output is invalid, the context is usable",
           code);
  return set_error(TB_ERR_TIMEOUT, "wait", buf);
}

namespace {

void session_destroy(Session* s) {
  const DriverApi* d = driver();
  if (d) d->cuCtxSetCurrent(s->context);
  for (Kernel* k : s->kernels) delete k;
  s->module_cache.clear();
  if (d) {
    for (auto& kv : s->builtin_modules)
      if (kv.second && kv.second->raw) d->cuModuleUnload(kv.second->raw);
  }
  for (Event* e : s->events) {
    if (d && e->raw) d->cuEventDestroy_v2(e->raw);
    delete e;
  }
  for (Stream* st : s->streams) {
    if (d && st->raw) {
      d->cuStreamSynchronize(st->raw);
      if (st->scratch) d->cuMemFree_v2(st->scratch);
      d->cuStreamDestroy_v2(st->raw);
    }
    delete st;
  }
  for (Buffer* b : s->buffers) {
    if (d && b->owned && b->ptr) d->cuMemFree_v2(b->ptr);
    delete b;
  }
  for (void* p : s->pinned)
    if (d) d->cuMemFreeHost(p);
  if (d && s->status.host) d->cuMemFreeHost((void*)s->status.host);
  if (d && s->context) d->cuDevicePrimaryCtxRelease_v2(s->device);
  delete s;
}

void session_unref(Session* s) {
  if (s && s->refs.fetch_sub(1) == 1) session_destroy(s);
}

bool fill_fingerprint(const DriverApi* d, uint32_t ordinal, tb_fingerprint* fp) {
  CUdevice dev;
  if (d->cuDeviceGet(&dev, (int)ordinal) != CUDA_SUCCESS) return false;
  memset(fp, 0, sizeof *fp);
  fp->ordinal = ordinal;
  d->cuDeviceGetName(fp->model, sizeof fp->model - 1, dev);
  int version = 0;
  d->cuDriverGetVersion(&version);
  snprintf(fp->driver, sizeof fp->driver, "%d.%d", version / 1000, (version % 1000) / 10);
  int major = 0, minor = 0, sms = 0;
  d->cuDeviceGetAttribute(&major, CU_DEVICE_ATTRIBUTE_COMPUTE_CAPABILITY_MAJOR, dev);
  d->cuDeviceGetAttribute(&minor, CU_DEVICE_ATTRIBUTE_COMPUTE_CAPABILITY_MINOR, dev);
  d->cuDeviceGetAttribute(&sms, CU_DEVICE_ATTRIBUTE_MULTIPROCESSOR_COUNT, dev);
  snprintf(fp->capability_revision, sizeof fp->capability_revision, "sm_%d%d", major, minor);
  fp->sm_count = (uint32_t)sms;
  size_t total = 0;
  d->cuDeviceTotalMem_v2(&total, dev);
  fp->total_memory = total;
  return true;
}

uint64_t fnv1a(const void* data, size_t len) {
  const unsigned char* p = static_cast<const unsigned char*>(data);
  uint64_t h = 1469598103934665603ull;
  for (size_t i = 0; i < len; ++i) {
    h ^= p[i];
    h *= 1099511628211ull;
  }
  return h;
}

}  // namespace

tb_status record_event(Session* s, Stream* stream, std::shared_ptr<std::vector<uint8_t>> staging, tb_event** out) {
  const DriverApi* d = driver();
  CUevent raw = nullptr;
  TB_CU("cuEventCreate", d->cuEventCreate(&raw, CU_EVENT_DEFAULT));
  CUresult r = d->cuEventRecord(raw, stream->raw);
  if (r != CUDA_SUCCESS) {
    d->cuEventDestroy_v2(raw);
    // A failed record must not release staging still read by an async copy
    // (titan-backend-cuda/src/lib.rs:1279-1286).
    if (staging) d->cuStreamSynchronize(stream->raw);
    return cu_error("cuEventRecord", r);
  }
  if (!out) {
    if (staging) {
      // Nobody holds the event: the staging must outlive the copy, so wait here.
      d->cuEventSynchronize(raw);
    }
    d->cuEventDestroy_v2(raw);
    return TB_OK;
  }
  Event* e = new Event();
  e->session = s;
  e->raw = raw;
  e->staging = std::move(staging);
  s->refs.fetch_add(1);
  {
    std::lock_guard<std::mutex> lock(s->mu);
    s->events.insert(e);
  }
  *out = reinterpret_cast<tb_event*>(e);
  return TB_OK;
}

bool stream_capturing(Stream* st) {
  CUstreamCaptureStatus status = CU_STREAM_CAPTURE_STATUS_NONE;
  return driver()->cuStreamIsCapturing(st->raw, &status) == CUDA_SUCCESS && status != CU_STREAM_CAPTURE_STATUS_NONE;
}

tb_status stream_scratch(Session* s, Stream* st, size_t bytes, CUdeviceptr* out) {
  if (st->scratch_bytes >= bytes) {
    *out = st->scratch;
    return TB_OK;
  }
  if (stream_capturing(st))
    return set_error(TB_ERR_INVALID, "capture",
                     "first use of the stream's scratch memory inside a graph capture: run the operator once before");
  const DriverApi* d = driver();
  if (st->scratch) {
    // Earlier kernels on this stream may still read the old scratch.
    TB_CU("cuStreamSynchronize", d->cuStreamSynchronize(st->raw));
    d->cuMemFree_v2(st->scratch);
    st->scratch = 0;
    st->scratch_bytes = 0;
  }
  CUdeviceptr p = 0;
  TB_CU("allocate", d->cuMemAlloc_v2(&p, bytes));
  st->scratch = p;
  st->scratch_bytes = bytes;
  (void)s;
  *out = p;
  return TB_OK;
}

tb_status builtin_function(Session* s, const char* module, const char* entry, CUfunction* out) {
  std::string key = std::string(module) + ":" + entry;
  {
    std::lock_guard<std::mutex> lock(s->mu);
    auto it = s->builtin_functions.find(key);
    if (it != s->builtin_functions.end()) {
      *out = it->second;
      return TB_OK;
    }
  }
  const DriverApi* d = driver();
  std::shared_ptr<Module> mod;
  {
    std::lock_guard<std::mutex> lock(s->mu);
    auto it = s->builtin_modules.find(module);
    if (it != s->builtin_modules.end()) mod = it->second;
  }
  if (!mod) {
    size_t n = 0;
    const EmbeddedCubin* cubins = embedded_cubins(&n);
    const EmbeddedCubin* found = nullptr;
    for (size_t i = 0; i < n; ++i)
      if (strcmp(cubins[i].name, module) == 0) found = &cubins[i];
    if (!found) return set_error(TB_ERR_UNSUPPORTED, "load", std::string("no embedded module ") + module);
    mod = std::make_shared<Module>();
    TB_CU("cuModuleLoadData", d->cuModuleLoadData(&mod->raw, found->data));
    std::lock_guard<std::mutex> lock(s->mu);
    s->builtin_modules[module] = mod;
  }
  CUfunction fn = nullptr;
  TB_CU("cuModuleGetFunction", d->cuModuleGetFunction(&fn, mod->raw, entry));
  std::lock_guard<std::mutex> lock(s->mu);
  s->builtin_functions[key] = fn;
  *out = fn;
  return TB_OK;
}

}  // namespace tb

using namespace tb;

extern "C" {

const char* tb_last_error_operation(void) { return tb::g_op.c_str(); }
const char* tb_last_error_detail(void) { return tb::g_detail.c_str(); }
const char* tb_version(void) { return "titan_b200 1 (sm_100a)"; }
const char* tb_last_candidate(void) { return tb::g_candidate.c_str(); }
uint64_t tb_launch_count(void) { return tb::g_launches; }

tb_status tb_driver_open(void) { return driver() ? TB_OK : TB_ERR_DRIVER_UNAVAILABLE; }

tb_status tb_driver_enumerate(tb_fingerprint* out, uint32_t capacity, uint32_t* count) {
  const DriverApi* d = driver();
  if (!d) return TB_ERR_DRIVER_UNAVAILABLE;
  int n = 0;
  TB_CU("cuDeviceGetCount", d->cuDeviceGetCount(&n));
  if (count) *count = (uint32_t)n;
  for (int i = 0; i < n && (uint32_t)i < capacity && out; ++i) {
    if (!fill_fingerprint(d, (uint32_t)i, &out[i])) return set_error(TB_ERR_CUDA, "enumerate", "cuDeviceGet failed");
  }
  return TB_OK;
}

tb_status tb_session_open(uint32_t ordinal, tb_session** out) {
  if (!out) return set_error(TB_ERR_INVALID, "open", "null output");
  const DriverApi* d = driver();
  if (!d) return TB_ERR_DRIVER_UNAVAILABLE;
  int n = 0;
  TB_CU("cuDeviceGetCount", d->cuDeviceGetCount(&n));
  if ((int)ordinal >= n) return set_error(TB_ERR_INVALID, "open", "CUDA device ordinal is unavailable");
  Session* s = new Session();
  s->ordinal = ordinal;
  CUresult r = d->cuDeviceGet(&s->device, (int)ordinal);
  if (r == CUDA_SUCCESS) r = d->cuDevicePrimaryCtxRetain(&s->context, s->device);
  if (r != CUDA_SUCCESS) {
    delete s;
    return cu_error("open_primary_context", r);
  }
  if (d->cuCtxSetCurrent(s->context) != CUDA_SUCCESS || !fill_fingerprint(d, ordinal, &s->fingerprint)) {
    d->cuDevicePrimaryCtxRelease_v2(s->device);
    delete s;
    return set_error(TB_ERR_CUDA, "open", "cannot activate the primary context");
  }
  d->cuDeviceGetAttribute(&s->sm_count, CU_DEVICE_ATTRIBUTE_MULTIPROCESSOR_COUNT, s->device);
  d->cuDeviceGetAttribute(&s->max_smem_optin, CU_DEVICE_ATTRIBUTE_MAX_SHARED_MEMORY_PER_BLOCK_OPTIN, s->device);
  void* host = nullptr;
  r = d->cuMemHostAlloc(&host, 64, CU_MEMHOSTALLOC_DEVICEMAP | CU_MEMHOSTALLOC_PORTABLE);
  if (r == CUDA_SUCCESS) r = d->cuMemHostGetDevicePointer_v2(&s->status.device, host, 0);
  if (r != CUDA_SUCCESS) {
    if (host) d->cuMemFreeHost(host);
    d->cuDevicePrimaryCtxRelease_v2(s->device);
    delete s;
    return cu_error("cuMemHostAlloc", r);
  }
  memset(host, 0, 64);
  s->status.host = static_cast<volatile uint32_t*>(host);
  *out = reinterpret_cast<tb_session*>(s);
  return TB_OK;
}

void tb_session_retain(tb_session* session) {
  if (session) reinterpret_cast<Session*>(session)->refs.fetch_add(1);
}

void tb_session_release(tb_session* session) { session_unref(reinterpret_cast<Session*>(session)); }

tb_status tb_session_fingerprint(const tb_session* session, tb_fingerprint* out) {
  if (!session || !out) return set_error(TB_ERR_INVALID, "fingerprint", "null argument");
  *out = reinterpret_cast<const Session*>(session)->fingerprint;
  return TB_OK;
}

// ---------------------------------------------------------------- buffers
tb_status tb_allocate(tb_session* session, size_t bytes, size_t alignment, tb_buffer** out) {
  Session* s = reinterpret_cast<Session*>(session);
  if (!s || !out) return set_error(TB_ERR_INVALID, "allocate", "null argument");
  // As CudaContext::allocate (titan-backend-cuda/src/lib.rs:122-125).
  if (bytes == 0) return set_error(TB_ERR_INVALID, "allocate", "zero-byte CUDA allocations are unsupported");
  // cuMemAlloc returns 256-byte aligned memory; larger alignments are not offered.
  if (alignment > 256 || (alignment & (alignment - 1)) != 0)
    return set_error(TB_ERR_INVALID, "allocate", "alignment must be a power of two no larger than 256");
  tb_status st = activate(s);
  if (st) return st;
  const DriverApi* d = driver();
  CUdeviceptr p = 0;
  TB_CU("allocate", d->cuMemAlloc_v2(&p, bytes));
  Buffer* b = new Buffer();
  b->session = s;
  b->identity = g_next_identity.fetch_add(1);
  b->ptr = p;
  b->bytes = bytes;
  b->owned = true;
  s->refs.fetch_add(1);
  {
    std::lock_guard<std::mutex> lock(s->mu);
    s->buffers.insert(b);
  }
  *out = reinterpret_cast<tb_buffer*>(b);
  return TB_OK;
}

tb_status tb_buffer_wrap(tb_session* session, uint64_t device_ptr, size_t bytes, tb_buffer** out) {
  Session* s = reinterpret_cast<Session*>(session);
  if (!s || !out) return set_error(TB_ERR_INVALID, "buffer", "null argument");
  if (device_ptr == 0 && bytes != 0) return set_error(TB_ERR_INVALID, "buffer", "null device pointer");
  Buffer* b = new Buffer();
  b->session = s;
  b->identity = g_next_identity.fetch_add(1);
  b->ptr = (CUdeviceptr)device_ptr;
  b->bytes = bytes;
  b->owned = false;
  s->refs.fetch_add(1);
  {
    std::lock_guard<std::mutex> lock(s->mu);
    s->buffers.insert(b);
  }
  *out = reinterpret_cast<tb_buffer*>(b);
  return TB_OK;
}

void tb_buffer_retain(tb_buffer* buffer) {
  if (buffer) reinterpret_cast<Buffer*>(buffer)->refs.fetch_add(1);
}

void tb_buffer_release(tb_buffer* buffer) {
  Buffer* b = reinterpret_cast<Buffer*>(buffer);
  if (!b || b->refs.fetch_sub(1) != 1) return;
  Session* s = b->session;
  {
    std::lock_guard<std::mutex> lock(s->mu);
    s->buffers.erase(b);
  }
  const DriverApi* d = driver();
  if (d && b->owned && b->ptr) {
    d->cuCtxSetCurrent(s->context);
    d->cuMemFree_v2(b->ptr);
  }
  delete b;
  session_unref(s);
}

size_t tb_buffer_byte_len(const tb_buffer* buffer) {
  return buffer ? reinterpret_cast<const Buffer*>(buffer)->bytes : 0;
}
uint64_t tb_buffer_identity(const tb_buffer* buffer) {
  return buffer ? reinterpret_cast<const Buffer*>(buffer)->identity : 0;
}
uint64_t tb_buffer_device_ptr(const tb_buffer* buffer) {
  return buffer ? (uint64_t)reinterpret_cast<const Buffer*>(buffer)->ptr : 0;
}

// ---------------------------------------------------------------- streams / events
tb_status tb_create_stream(tb_session* session, tb_stream** out) {
  Session* s = reinterpret_cast<Session*>(session);
  if (!s || !out) return set_error(TB_ERR_INVALID, "create_stream", "null argument");
  tb_status st = activate(s);
  if (st) return st;
  CUstream raw = nullptr;
  TB_CU("cuStreamCreate", driver()->cuStreamCreate(&raw, CU_STREAM_NON_BLOCKING));
  Stream* x = new Stream();
  x->session = s;
  x->raw = raw;
  s->refs.fetch_add(1);
  {
    std::lock_guard<std::mutex> lock(s->mu);
    s->streams.insert(x);
  }
  *out = reinterpret_cast<tb_stream*>(x);
  return TB_OK;
}

void tb_stream_release(tb_stream* stream) {
  Stream* x = reinterpret_cast<Stream*>(stream);
  if (!x || x->refs.fetch_sub(1) != 1) return;
  Session* s = x->session;
  {
    std::lock_guard<std::mutex> lock(s->mu);
    s->streams.erase(x);
  }
  const DriverApi* d = driver();
  if (d && x->raw) {
    d->cuCtxSetCurrent(s->context);
    if (x->scratch) {
      d->cuStreamSynchronize(x->raw);
      d->cuMemFree_v2(x->scratch);
    }
    d->cuStreamDestroy_v2(x->raw);
  }
  delete x;
  session_unref(s);
}

uint64_t tb_stream_handle(const tb_stream* stream) {
  return stream ? (uint64_t)(uintptr_t)reinterpret_cast<const Stream*>(stream)->raw : 0;
}

tb_status tb_create_event(tb_session* session, tb_event** out) {
  Session* s = reinterpret_cast<Session*>(session);
  if (!s || !out) return set_error(TB_ERR_INVALID, "create_event", "null argument");
  tb_status st = activate(s);
  if (st) return st;
  CUevent raw = nullptr;
  TB_CU("cuEventCreate", driver()->cuEventCreate(&raw, CU_EVENT_DEFAULT));
  Event* e = new Event();
  e->session = s;
  e->raw = raw;
  s->refs.fetch_add(1);
  {
    std::lock_guard<std::mutex> lock(s->mu);
    s->events.insert(e);
  }
  *out = reinterpret_cast<tb_event*>(e);
  return TB_OK;
}

void tb_event_release(tb_event* event) {
  Event* e = reinterpret_cast<Event*>(event);
  if (!e || e->refs.fetch_sub(1) != 1) return;
  Session* s = e->session;
  {
    std::lock_guard<std::mutex> lock(s->mu);
    s->events.erase(e);
  }
  const DriverApi* d = driver();
  if (d && e->raw) {
    d->cuCtxSetCurrent(s->context);
    // Staging must outlive the copy that reads it: wait before dropping it.
    if (e->staging) d->cuEventSynchronize(e->raw);
    d->cuEventDestroy_v2(e->raw);
  }
  delete e;
  session_unref(s);
}

tb_status tb_record(tb_session* session, tb_stream* stream, tb_event** out) {
  Session* s = reinterpret_cast<Session*>(session);
  if (!s) return set_error(TB_ERR_INVALID, "event", "null session");
  Stream* st = nullptr;
  tb_status rc = check_stream(s, stream, &st);
  if (rc) return rc;
  rc = activate(s);
  if (rc) return rc;
  return record_event(s, st, nullptr, out);
}

tb_status tb_event_elapsed_ms(tb_session* session, tb_event* start, tb_event* end, float* ms) {
  Session* s = reinterpret_cast<Session*>(session);
  if (!s || !ms) return set_error(TB_ERR_INVALID, "event", "null argument");
  Event *a = nullptr, *b = nullptr;
  tb_status rc = check_event(s, start, &a);
  if (rc) return rc;
  rc = check_event(s, end, &b);
  if (rc) return rc;
  rc = activate(s);
  if (rc) return rc;
  TB_CU("cuEventElapsedTime", driver()->cuEventElapsedTime(ms, a->raw, b->raw));
  return TB_OK;
}

tb_status tb_stream_synchronize(tb_session* session, tb_stream* stream) {
  Session* s = reinterpret_cast<Session*>(session);
  if (!s) return set_error(TB_ERR_INVALID, "wait", "null session");
  Stream* st = nullptr;
  tb_status rc = check_stream(s, stream, &st);
  if (rc) return rc;
  rc = activate(s);
  if (rc) return rc;
  TB_CU("cuStreamSynchronize", driver()->cuStreamSynchronize(st->raw));
  return consume_device_status(s);
}

// ---------------------------------------------------------------- copies
tb_status tb_upload(tb_session* session, tb_stream* stream, tb_buffer* dst, const void* src, size_t len,
                    tb_event** out) {
  Session* s = reinterpret_cast<Session*>(session);
  if (!s) return set_error(TB_ERR_INVALID, "upload", "null session");
  Stream* st = nullptr;
  Buffer* b = nullptr;
  tb_status rc = check_stream(s, stream, &st);
  if (rc) return rc;
  rc = check_buffer(s, dst, &b);
  if (rc) return rc;
  if (len > b->bytes) return set_error(TB_ERR_INVALID, "upload", "source exceeds allocation");
  if (len && !src) return set_error(TB_ERR_INVALID, "upload", "null source");
  rc = activate(s);
  if (rc) return rc;
  if (stream_capturing(st))
    return set_error(TB_ERR_INVALID, "upload", "staged upload inside a graph capture (use tb_upload_pinned)");
  auto staging = std::make_shared<std::vector<uint8_t>>(static_cast<const uint8_t*>(src),
                                                        static_cast<const uint8_t*>(src) + len);
  if (len) TB_CU("cuMemcpyHtoDAsync", driver()->cuMemcpyHtoDAsync_v2(b->ptr, staging->data(), len, st->raw));
  return record_event(s, st, staging, out);
}

tb_status tb_download(tb_session* session, tb_stream* stream, tb_buffer* src, void* dst, size_t len,
                      tb_event** out) {
  Session* s = reinterpret_cast<Session*>(session);
  if (!s) return set_error(TB_ERR_INVALID, "download", "null session");
  Stream* st = nullptr;
  Buffer* b = nullptr;
  tb_status rc = check_stream(s, stream, &st);
  if (rc) return rc;
  rc = check_buffer(s, src, &b);
  if (rc) return rc;
  if (len > b->bytes) return set_error(TB_ERR_INVALID, "download", "destination exceeds allocation");
  if (len && !dst) return set_error(TB_ERR_INVALID, "download", "null destination");
  rc = activate(s);
  if (rc) return rc;
  if (stream_capturing(st))
    return set_error(TB_ERR_INVALID, "download", "download inside a graph capture (use tb_download_pinned)");
  const DriverApi* d = driver();
  if (len) TB_CU("cuMemcpyDtoHAsync", d->cuMemcpyDtoHAsync_v2(dst, b->ptr, len, st->raw));
  // The borrowed host destination cannot outlive this call (lib.rs:1300-1304).
  TB_CU("cuStreamSynchronize", d->cuStreamSynchronize(st->raw));
  rc = consume_device_status(s);
  if (rc) return rc;
  return record_event(s, st, nullptr, out);
}

tb_status tb_copy(tb_session* session, tb_stream* stream, tb_buffer* dst, tb_buffer* src, size_t bytes,
                  tb_event** out) {
  Session* s = reinterpret_cast<Session*>(session);
  if (!s) return set_error(TB_ERR_INVALID, "copy", "null session");
  Stream* st = nullptr;
  Buffer *bd = nullptr, *bs = nullptr;
  tb_status rc = check_stream(s, stream, &st);
  if (rc) return rc;
  rc = check_buffer(s, dst, &bd);
  if (rc) return rc;
  rc = check_buffer(s, src, &bs);
  if (rc) return rc;
  if (bytes > bs->bytes || bytes > bd->bytes) return set_error(TB_ERR_INVALID, "copy", "transfer exceeds allocation");
  rc = activate(s);
  if (rc) return rc;
  if (bytes) TB_CU("cuMemcpyDtoDAsync", driver()->cuMemcpyDtoDAsync_v2(bd->ptr, bs->ptr, bytes, st->raw));
  return record_event(s, st, nullptr, out);
}

tb_status tb_host_alloc(tb_session* session, size_t bytes, void** out) {
  Session* s = reinterpret_cast<Session*>(session);
  if (!s || !out) return set_error(TB_ERR_INVALID, "allocate", "null argument");
  tb_status rc = activate(s);
  if (rc) return rc;
  void* p = nullptr;
  TB_CU("cuMemHostAlloc", driver()->cuMemHostAlloc(&p, bytes ? bytes : 1, CU_MEMHOSTALLOC_PORTABLE));
  std::lock_guard<std::mutex> lock(s->mu);
  s->pinned.insert(p);
  *out = p;
  return TB_OK;
}

tb_status tb_host_free(tb_session* session, void* ptr) {
  Session* s = reinterpret_cast<Session*>(session);
  if (!s) return set_error(TB_ERR_INVALID, "allocate", "null session");
  {
    std::lock_guard<std::mutex> lock(s->mu);
    if (!s->pinned.erase(ptr)) return set_error(TB_ERR_FOREIGN, "allocate", "foreign host allocation");
  }
  tb_status rc = activate(s);
  if (rc) return rc;
  TB_CU("cuMemFreeHost", driver()->cuMemFreeHost(ptr));
  return TB_OK;
}

tb_status tb_upload_pinned(tb_session* session, tb_stream* stream, tb_buffer* dst, size_t dst_offset,
                           const void* src, size_t len, tb_event** out) {
  Session* s = reinterpret_cast<Session*>(session);
  if (!s) return set_error(TB_ERR_INVALID, "upload", "null session");
  Stream* st = nullptr;
  Buffer* b = nullptr;
  tb_status rc = check_stream(s, stream, &st);
  if (rc) return rc;
  rc = check_buffer(s, dst, &b);
  if (rc) return rc;
  if (dst_offset > b->bytes || len > b->bytes - dst_offset)
    return set_error(TB_ERR_INVALID, "upload", "source exceeds allocation");
  rc = activate(s);
  if (rc) return rc;
  if (len) TB_CU("cuMemcpyHtoDAsync", driver()->cuMemcpyHtoDAsync_v2(b->ptr + dst_offset, src, len, st->raw));
  if (!out) return TB_OK;
  return record_event(s, st, nullptr, out);
}

tb_status tb_download_pinned(tb_session* session, tb_stream* stream, tb_buffer* src, size_t src_offset, void* dst,
                             size_t len, tb_event** out) {
  Session* s = reinterpret_cast<Session*>(session);
  if (!s) return set_error(TB_ERR_INVALID, "download", "null session");
  Stream* st = nullptr;
  Buffer* b = nullptr;
  tb_status rc = check_stream(s, stream, &st);
  if (rc) return rc;
  rc = check_buffer(s, src, &b);
  if (rc) return rc;
  if (src_offset > b->bytes || len > b->bytes - src_offset)
    return set_error(TB_ERR_INVALID, "download", "destination exceeds allocation");
  rc = activate(s);
  if (rc) return rc;
  if (len) TB_CU("cuMemcpyDtoHAsync", driver()->cuMemcpyDtoHAsync_v2(dst, b->ptr + src_offset, len, st->raw));
  if (!out) return TB_OK;
  return record_event(s, st, nullptr, out);
}

// ---------------------------------------------------------------- poll / wait
tb_status tb_poll(tb_session* session, tb_event* event, int* ready) {
  Session* s = reinterpret_cast<Session*>(session);
  if (!s || !ready) return set_error(TB_ERR_INVALID, "event", "null argument");
  Event* e = nullptr;
  tb_status rc = check_event(s, event, &e);
  if (rc) return rc;
  rc = activate(s);
  if (rc) return rc;
  CUresult r = driver()->cuEventQuery(e->raw);
  if (r == CUDA_SUCCESS) {
    *ready = 1;
    return consume_device_status(s);
  }
  if (r == CUDA_ERROR_NOT_READY) {
    *ready = 0;
    return TB_OK;
  }
  return cu_error("cuEventQuery", r);
}

tb_status tb_wait(tb_session* session, tb_event* event) {
  Session* s = reinterpret_cast<Session*>(session);
  if (!s) return set_error(TB_ERR_INVALID, "wait", "null session");
  Event* e = nullptr;
  tb_status rc = check_event(s, event, &e);
  if (rc) return rc;
  rc = activate(s);
  if (rc) return rc;
  TB_CU("cuEventSynchronize", driver()->cuEventSynchronize(e->raw));
  return consume_device_status(s);
}

tb_status tb_wait_event(tb_session* session, tb_stream* stream, tb_event* event) {
  Session* s = reinterpret_cast<Session*>(session);
  if (!s) return set_error(TB_ERR_INVALID, "wait_event", "null session");
  Stream* st = nullptr;
  Event* e = nullptr;
  tb_status rc = check_stream(s, stream, &st);
  if (rc) return rc;
  rc = check_event(s, event, &e);
  if (rc) return rc;
  rc = activate(s);
  if (rc) return rc;
  TB_CU("cuStreamWaitEvent", driver()->cuStreamWaitEvent(st->raw, e->raw, 0));
  return TB_OK;
}

// ---------------------------------------------------------------- load / launch
tb_status tb_load(tb_session* session, const void* artifact, size_t len, const char* abi_hash,
                  const tb_launch_metadata* metadata, tb_kernel** out) {
  Session* s = reinterpret_cast<Session*>(session);
  if (!s || !out || !metadata || !abi_hash) return set_error(TB_ERR_INVALID, "load", "null argument");
  if (!artifact || len == 0) return set_error(TB_ERR_INVALID, "load", "empty artifact");
  if (!metadata->entry || !metadata->entry[0]) return set_error(TB_ERR_INVALID, "load", "missing kernel entry");
  for (uint32_t i = 0; i < metadata->num_arguments; ++i) {
    uint32_t kind = metadata->arguments[i].kind;
    if (kind > TB_ARG_SHAPE) return set_error(TB_ERR_INVALID, "load", "unknown launch argument kind");
  }
  const unsigned char* bytes = static_cast<const unsigned char*>(artifact);
  bool is_elf = len >= 4 && bytes[0] == 0x7f && bytes[1] == 'E' && bytes[2] == 'L' && bytes[3] == 'F';
  std::vector<unsigned char> text;
  const void* image = artifact;
  if (!is_elf) {
    // PTX text (the reference's only artifact form, titan-backend-cuda/src/ptx/mod.rs:21-37).
    std::string str(reinterpret_cast<const char*>(bytes), strnlen(reinterpret_cast<const char*>(bytes), len));
    if (str.find(".version") == std::string::npos || str.find(".target") == std::string::npos)
      return set_error(TB_ERR_INVALID, "load", "artifact is neither a cubin nor PTX text with .version/.target");
    text.assign(str.begin(), str.end());
    text.push_back(0);
    image = text.data();
  }
  tb_status rc = activate(s);
  if (rc) return rc;
  const DriverApi* d = driver();
  char keybuf[64];
  snprintf(keybuf, sizeof keybuf, "%016" PRIx64 ":%zu", fnv1a(artifact, len), len);
  std::shared_ptr<Module> mod;
  {
    std::lock_guard<std::mutex> lock(s->mu);
    auto it = s->module_cache.find(keybuf);
    if (it != s->module_cache.end()) mod = it->second;
  }
  if (!mod) {
    auto fresh = std::shared_ptr<Module>(new Module(), [d](Module* m) {
      if (m->raw) d->cuModuleUnload(m->raw);
      delete m;
    });
    TB_CU("cuModuleLoadData", d->cuModuleLoadData(&fresh->raw, image));
    std::lock_guard<std::mutex> lock(s->mu);
    s->module_cache[keybuf] = fresh;
    mod = fresh;
  }
  CUfunction fn = nullptr;
  TB_CU("cuModuleGetFunction", d->cuModuleGetFunction(&fn, mod->raw, metadata->entry));
  Kernel* k = new Kernel();
  k->session = s;
  k->module = mod;
  k->function = fn;
  k->abi_hash = abi_hash;
  k->entry = metadata->entry;
  k->arguments.assign(metadata->arguments, metadata->arguments + metadata->num_arguments);
  memcpy(k->block, metadata->block, sizeof k->block);
  k->shared_bytes = metadata->shared_bytes;
  s->refs.fetch_add(1);
  {
    std::lock_guard<std::mutex> lock(s->mu);
    s->kernels.insert(k);
  }
  *out = reinterpret_cast<tb_kernel*>(k);
  return TB_OK;
}

tb_status tb_builtin_cubin(const char* module, const void** data, size_t* len) {
  if (!module || !data || !len) return set_error(TB_ERR_INVALID, "load", "null argument");
  size_t n = 0;
  const EmbeddedCubin* cubins = embedded_cubins(&n);
  for (size_t i = 0; i < n; ++i) {
    if (strcmp(cubins[i].name, module) == 0) {
      *data = cubins[i].data;
      *len = cubins[i].size;
      return TB_OK;
    }
  }
  return set_error(TB_ERR_UNSUPPORTED, "load", std::string("no embedded module ") + module);
}

void tb_kernel_release(tb_kernel* kernel) {
  Kernel* k = reinterpret_cast<Kernel*>(kernel);
  if (!k || k->refs.fetch_sub(1) != 1) return;
  Session* s = k->session;
  {
    std::lock_guard<std::mutex> lock(s->mu);
    s->kernels.erase(k);
  }
  delete k;
  session_unref(s);
}

tb_status tb_launch(tb_session* session, tb_stream* stream, tb_kernel* kernel, const tb_encoded_args* args,
                    const tb_launch_geometry* geometry, tb_event** out) {
  Session* s = reinterpret_cast<Session*>(session);
  if (!s || !args || !geometry) return set_error(TB_ERR_INVALID, "launch", "null argument");
  Stream* st = nullptr;
  tb_status rc = check_stream(s, stream, &st);
  if (rc) return rc;
  Kernel* k = reinterpret_cast<Kernel*>(kernel);
  if (!k) return set_error(TB_ERR_INVALID, "launch", "null kernel");
  bool known = false;
  {
    std::lock_guard<std::mutex> lock(s->mu);
    known = s->kernels.count(k) != 0;
  }
  if (!known) {
    if (k->session && k->session->ordinal != s->ordinal)
      return set_error(TB_ERR_FOREIGN, "launch", "cross-device kernel");
    return set_error(TB_ERR_FOREIGN, "launch", "kernel belongs to another CUDA session");
  }
  if (args->canonical_abi_len != k->abi_hash.size() ||
      (args->canonical_abi_len && memcmp(args->canonical_abi, k->abi_hash.data(), k->abi_hash.size()) != 0))
    return set_error(TB_ERR_INVALID, "launch", "encoded arguments do not match kernel ABI");
  // EncodedLaunchArgs::try_new rejects duplicate slots (titan-hal/src/lib.rs:153-165).
  for (uint32_t i = 0; i < args->num_bindings; ++i)
    for (uint32_t j = i + 1; j < args->num_bindings; ++j)
      if (args->bindings[i].slot == args->bindings[j].slot)
        return set_error(TB_ERR_INVALID, "encode", "duplicate buffer binding slot");

  const uint8_t* p = args->payload;
  size_t n = args->payload_len, cursor = 0;
  std::vector<std::vector<uint8_t>> values;
  std::vector<uint32_t> required;
  values.reserve(k->arguments.size());
  for (const tb_launch_arg& a : k->arguments) {
    if (a.kind == TB_ARG_BUFFER) {
      if (n - cursor < 4) return set_error(TB_ERR_INVALID, "launch", "truncated buffer slot");
      uint32_t slot;
      memcpy(&slot, p + cursor, 4);
      cursor += 4;
      required.push_back(slot);
      const tb_binding* found = nullptr;
      for (uint32_t i = 0; i < args->num_bindings; ++i)
        if (args->bindings[i].slot == slot) found = &args->bindings[i];
      if (!found) return set_error(TB_ERR_INVALID, "launch", "missing buffer binding for slot " + std::to_string(slot));
      Buffer* b = nullptr;
      rc = check_buffer(s, found->buffer, &b);
      if (rc) return rc;
      std::vector<uint8_t> v(sizeof(CUdeviceptr));
      memcpy(v.data(), &b->ptr, sizeof(CUdeviceptr));
      values.push_back(std::move(v));
    } else if (a.kind == TB_ARG_SCALAR) {
      if (n - cursor < 4) return set_error(TB_ERR_INVALID, "launch", "truncated scalar length");
      uint32_t len;
      memcpy(&len, p + cursor, 4);
      cursor += 4;
      if (len != a.width) return set_error(TB_ERR_INVALID, "launch", "scalar width disagrees with ABI");
      if (n - cursor < len) return set_error(TB_ERR_INVALID, "launch", "truncated scalar");
      values.emplace_back(p + cursor, p + cursor + len);
      cursor += len;
    } else {
      size_t len = (size_t)a.width * 8;
      if (n - cursor < len) return set_error(TB_ERR_INVALID, "launch", "truncated shape");
      values.emplace_back(p + cursor, p + cursor + len);
      cursor += len;
    }
  }
  if (cursor != n) return set_error(TB_ERR_INVALID, "launch", "trailing ABI bytes");
  // EncodedLaunchArgs::validate_for (titan-hal/src/lib.rs:168-189).
  for (uint32_t slot : required) {
    const tb_binding* found = nullptr;
    for (uint32_t i = 0; i < args->num_bindings; ++i)
      if (args->bindings[i].slot == slot) found = &args->bindings[i];
    if (!found)
      return set_error(TB_ERR_INVALID, "validate_bindings", "missing buffer binding for slot " + std::to_string(slot));
    if (found->owner != reinterpret_cast<const tb_session*>(s))
      return set_error(TB_ERR_FOREIGN, "validate_bindings",
                       "cross-session buffer binding for slot " + std::to_string(slot));
  }
  std::vector<void*> params;
  params.reserve(values.size());
  for (auto& v : values) params.push_back(v.data());
  rc = activate(s);
  if (rc) return rc;
  const DriverApi* d = driver();
  if (geometry->shared_bytes > 48 * 1024)
    TB_CU("cuFuncSetAttribute",
          d->cuFuncSetAttribute(k->function, CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES,
                                (int)geometry->shared_bytes));
  TB_CU("cuLaunchKernel",
        d->cuLaunchKernel(k->function, geometry->grid[0], geometry->grid[1], geometry->grid[2], geometry->block[0],
                          geometry->block[1], geometry->block[2], geometry->shared_bytes, st->raw, params.data(),
                          nullptr));
  note_launch(k->entry.c_str());
  return record_event(s, st, nullptr, out);
}

}  // extern "C"
