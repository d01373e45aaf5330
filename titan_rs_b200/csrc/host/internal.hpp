// Internal state of libtitan_b200: sessions and their handle registries.
//
// Mirrors the CUDA backend's CudaSession (titan-backend-cuda/src/lib.rs:1170-1244):
// every buffer, stream and event is registered with the session that created
// it, and a handle presented to another session is rejected as foreign. Handles
// are reference counted so that an event can keep its upload staging alive
// (the reference's `CudaEvent{staging}`), exactly as the Arc-based reference does.
#pragma once

#include <atomic>
#include <cstdint>
#include <cstring>
#include <memory>
#include <mutex>
#include <string>
#include <unordered_map>
#include <unordered_set>
#include <vector>

#include "../../../include/titan_b200.h"
#include "driver.hpp"

namespace tb {

// ---- error reporting (HalError{operation, detail}) ----
tb_status set_error(tb_status status, const char* operation, const std::string& detail);
tb_status cu_error(const char* operation, CUresult result);
#define TB_CU(op, call)                         \
  do {                                          \
    CUresult tb_r__ = (call);                   \
    if (tb_r__ != CUDA_SUCCESS) return ::tb::cu_error(op, tb_r__); \
  } while (0)

struct Session;

struct RefCounted {
  std::atomic<int> refs{1};
};

struct Buffer : RefCounted {
  Session* session = nullptr;
  uint64_t identity = 0;
  CUdeviceptr ptr = 0;
  size_t bytes = 0;
  bool owned = true;
};

struct Stream : RefCounted {
  Session* session = nullptr;
  CUstream raw = nullptr;
  // Scratch device memory for kernels launched on this stream (split-K partials).
  // Stream order serialises its users; it grows on demand and is freed with the stream.
  CUdeviceptr scratch = 0;
  size_t scratch_bytes = 0;
};

struct Event : RefCounted {
  Session* session = nullptr;
  CUevent raw = nullptr;
  std::shared_ptr<std::vector<uint8_t>> staging;  // kept alive until the event is released
};

struct Module {
  CUmodule raw = nullptr;
};

struct Kernel : RefCounted {
  Session* session = nullptr;
  std::shared_ptr<Module> module;
  CUfunction function = nullptr;
  std::string abi_hash;
  std::string entry;
  std::vector<tb_launch_arg> arguments;
  uint32_t block[3] = {1, 1, 1};
  uint32_t shared_bytes = 0;
};

// Device-side status word: kernels that give up a bounded wait write a nonzero
// code here (host-mapped pinned memory, so the host reads it without a copy).
struct StatusWord {
  volatile uint32_t* host = nullptr;
  CUdeviceptr device = 0;
};

struct Session : RefCounted {
  uint32_t ordinal = 0;
  CUdevice device = 0;
  CUcontext context = nullptr;
  tb_fingerprint fingerprint{};
  std::mutex mu;
  std::unordered_set<Buffer*> buffers;
  std::unordered_set<Stream*> streams;
  std::unordered_set<Event*> events;
  std::unordered_set<Kernel*> kernels;
  std::unordered_map<std::string, std::shared_ptr<Module>> module_cache;  // by artifact content hash
  std::unordered_map<std::string, CUfunction> builtin_functions;        // embedded cubin entries
  std::unordered_map<std::string, std::shared_ptr<Module>> builtin_modules;
  std::unordered_map<CUfunction, int> pair_occupancy;  // resident CTA pairs of a built-in pair kernel
  std::unordered_set<void*> pinned;
  StatusWord status;
  int sm_count = 0;
  int max_smem_optin = 0;
};

// Makes the session's context current on this thread (the reference re-activates
// before every driver call, titan-backend-cuda/src/lib.rs:1576-1579).
tb_status activate(Session* s);

// Registry lookups: they fail with the reference's messages ("foreign buffer", ...).
tb_status check_buffer(Session* s, tb_buffer* b, Buffer** out);
tb_status check_stream(Session* s, tb_stream* st, Stream** out);
tb_status check_event(Session* s, tb_event* e, Event** out);

// At least `bytes` of the stream's scratch memory (allocating or growing it).
tb_status stream_scratch(Session* s, Stream* st, size_t bytes, CUdeviceptr* out);

// Whether `st` is being captured into a CUDA graph (tb_capture_begin): host-staged
// copies and allocations are refused then, since a replay would run them on memory
// the call no longer owns.
bool stream_capturing(Stream* st);

// Records an event on `stream` and hands it to the caller (or drops it if out is null).
tb_status record_event(Session* s, Stream* stream, std::shared_ptr<std::vector<uint8_t>> staging, tb_event** out);

// Resolves an entry point of one of the embedded sm_100a cubins (loaded once per session).
tb_status builtin_function(Session* s, const char* module, const char* entry, CUfunction* out);

// Reads and clears the device status word; returns TB_ERR_TIMEOUT if a kernel gave up a wait.
tb_status consume_device_status(Session* s);

// Counts kernel launches made by this thread (the bench's gpu_launches figure).
void note_launch(const char* candidate);
// Names the candidate an operator ran when it took several launches (no launch counted).
void note_candidate(const char* candidate);

// Embedded cubins (generated at build time).
struct EmbeddedCubin {
  const char* name;
  const unsigned char* data;
  size_t size;
};
const EmbeddedCubin* embedded_cubins(size_t* count);

}  // namespace tb
