// Collective over NVLink/NVSwitch: the titan.rs `Collective` trait's all_gather
// (projects/titan-distributed/src/lib.rs:95-99, LocalRing :129-134) on device
// buffers through NCCL, plus the N-sharded GEMM that uses it.
//
// The sharded GEMM has two forms. With an output buffer registered on every rank
// (tb_comm_register_buffer: CUDA IPC mappings of each rank's buffer, and of a small
// signal block, in every other rank), one fused kernel computes this rank's column
// block and stores each output chunk straight into every rank's row-major C over
// NVLink; the ranks meet through flags in the signal blocks at the kernel's start
// and end, so the call is a single launch.
// Otherwise the GEMM writes a [p][M][N/p] workspace slot, NCCL all-gathers it in
// place and a layout kernel writes the row-major C.
//
// NCCL is opened with dlopen like the CUDA driver, so the library still loads
// where NCCL is absent. Communicators are non-blocking (ncclConfig_t.blocking = 0).
// A watchdog thread per communicator watches the event recorded after each
// collective: if it has not completed `timeout_ms` after it was enqueued, or
// NCCL reports an asynchronous error, the watchdog aborts the communicator, so
// the stuck collective kernel returns and later calls fail with TB_ERR_NCCL
// instead of hanging on a peer that died.
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <condition_variable>
#include <thread>

#include "../kernels/kernel_configs.h"
#include "ops_common.hpp"

namespace tb {

tb_status launch_gemm_bf16_default(Session* s, Stream* st, CUdeviceptr a, CUdeviceptr b, CUdeviceptr c, int M, int N,
                                   int K, long long ldc);
tb_status launch_gemm_bf16_tn_allgather(Session* s, Stream* st, CUdeviceptr a, CUdeviceptr b, const CUdeviceptr* outs,
                                        const CUdeviceptr* signals, int ranks, int self, uint32_t epoch, int M, int N,
                                        int K, long long ldc, long long col0, CUdeviceptr ready, size_t ready_count);

namespace {

struct NcclApi {
  decltype(&::ncclGetUniqueId) GetUniqueId = nullptr;
  decltype(&::ncclCommInitRankConfig) CommInitRankConfig = nullptr;
  decltype(&::ncclCommDestroy) CommDestroy = nullptr;
  decltype(&::ncclCommAbort) CommAbort = nullptr;
  decltype(&::ncclCommGetAsyncError) CommGetAsyncError = nullptr;
  decltype(&::ncclAllGather) AllGather = nullptr;
  decltype(&::ncclAllReduce) AllReduce = nullptr;
  decltype(&::ncclGetErrorString) GetErrorString = nullptr;
  bool ok = false;
  std::string error;
};

NcclApi& nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
      api.error = dlerror() ? dlerror() : "libnccl.so.2 not found";
      return;
    }
#define TB_NCCL(field, sym)                                               \
  api.field = reinterpret_cast<decltype(api.field)>(dlsym(h, #sym));      \
  if (!api.field) {                                                       \
    api.error = "missing NCCL symbol " #sym;                              \
    return;                                                               \
  }
    TB_NCCL(GetUniqueId, ncclGetUniqueId)
    TB_NCCL(CommInitRankConfig, ncclCommInitRankConfig)
    TB_NCCL(CommDestroy, ncclCommDestroy)
    TB_NCCL(CommAbort, ncclCommAbort)
    TB_NCCL(CommGetAsyncError, ncclCommGetAsyncError)
    TB_NCCL(AllGather, ncclAllGather)
    TB_NCCL(AllReduce, ncclAllReduce)
    TB_NCCL(GetErrorString, ncclGetErrorString)
#undef TB_NCCL
    api.ok = true;
  });
  return api;
}

tb_status nccl_error(const char* op, ncclResult_t r) {
  NcclApi& n = nccl();
  return set_error(TB_ERR_NCCL, op, std::string("NCCL status ") + std::to_string((int)r) + " (" +
                                        (n.GetErrorString ? n.GetErrorString(r) : "?") + ")");
}

}  // namespace

// A buffer registered on every rank: where each rank's copy, and each rank's signal
// block (TB_SIGNAL_BLOCK_BYTES of flags, see kernels/peer_signal.cuh), are mapped here.
struct PeerMapping {
  Buffer* local = nullptr;             // retained while registered
  std::vector<CUdeviceptr> base;       // per rank; this rank's entry is local->ptr
  std::vector<uint64_t> bytes;         // per rank
  std::vector<CUdeviceptr> opened;     // per rank: IPC mapping to close (0 for this rank)
  CUdeviceptr signal_local = 0;        // this rank's signal block (owned)
  std::vector<CUdeviceptr> signal;     // per rank
  std::vector<CUdeviceptr> signal_opened;
  uint32_t epoch = 0;                  // fused calls made with this buffer (same on every rank)
  CUdeviceptr ready = 0;               // per-tile counters of the pusher-CTA kernel (owned)
  size_t ready_count = 0;
};

struct Comm {
  Session* session = nullptr;
  ncclComm_t comm = nullptr;
  int rank = 0, size = 0;
  uint32_t timeout_ms = 0;
  CUdeviceptr barrier_word = 0;
  // Watchdog state.
  std::mutex mu;
  std::condition_variable cv;
  std::thread watchdog;
  bool stop = false;
  bool aborted = false;
  std::string abort_reason;
  std::vector<std::pair<CUevent, std::chrono::steady_clock::time_point>> pending;
  std::vector<PeerMapping> mappings;  // registered buffers (caller's thread only)
};

namespace {

// Waits for a non-blocking NCCL call to leave ncclInProgress (bounded by the comm timeout).
tb_status settle(Comm* c, const char* op) {
  NcclApi& n = nccl();
  const auto deadline = std::chrono::steady_clock::now() + std::chrono::milliseconds(c->timeout_ms);
  while (true) {
    ncclResult_t st = ncclSuccess;
    ncclResult_t r = n.CommGetAsyncError(c->comm, &st);
    if (r != ncclSuccess) return nccl_error(op, r);
    if (st == ncclSuccess) return TB_OK;
    if (st != ncclInProgress) return nccl_error(op, st);
    if (std::chrono::steady_clock::now() > deadline) {
      n.CommAbort(c->comm);
      c->comm = nullptr;
      return set_error(TB_ERR_NCCL, op, "NCCL operation did not complete before the communicator timeout; aborted");
    }
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

void watchdog_loop(Comm* c) {
  const DriverApi* d = driver();
  NcclApi& n = nccl();
  std::unique_lock<std::mutex> lock(c->mu);
  while (!c->stop) {
    c->cv.wait_for(lock, std::chrono::milliseconds(10));
    if (c->stop || c->aborted || !c->comm) continue;
    d->cuCtxSetCurrent(c->session->context);
    // Drop completed collectives; abort when the oldest one is overdue.
    while (!c->pending.empty() && d->cuEventQuery(c->pending.front().first) == CUDA_SUCCESS) {
      d->cuEventDestroy_v2(c->pending.front().first);
      c->pending.erase(c->pending.begin());
    }
    ncclResult_t async = ncclSuccess;
    n.CommGetAsyncError(c->comm, &async);
    const bool overdue = !c->pending.empty() &&
                         std::chrono::steady_clock::now() - c->pending.front().second >
                             std::chrono::milliseconds(c->timeout_ms);
    if ((async != ncclSuccess && async != ncclInProgress) || overdue) {
      c->abort_reason = overdue ? "a collective made no progress within the communicator timeout (peer lost?)"
                                : std::string("NCCL asynchronous error ") + std::to_string((int)async);
      n.CommAbort(c->comm);
      c->comm = nullptr;
      c->aborted = true;
    }
  }
}

tb_status track(Comm* c, Stream* st) {
  const DriverApi* d = driver();
  CUevent ev = nullptr;
  TB_CU("cuEventCreate", d->cuEventCreate(&ev, CU_EVENT_DISABLE_TIMING));
  TB_CU("cuEventRecord", d->cuEventRecord(ev, st->raw));
  std::lock_guard<std::mutex> lock(c->mu);
  c->pending.emplace_back(ev, std::chrono::steady_clock::now());
  return TB_OK;
}

tb_status usable(Comm* c, const char* op) {
  if (!c) return set_error(TB_ERR_INVALID, op, "null communicator");
  std::lock_guard<std::mutex> lock(c->mu);
  if (c->aborted || !c->comm)
    return set_error(TB_ERR_NCCL, op, "communicator was aborted: " + c->abort_reason);
  return TB_OK;
}

// Stream-ordered barrier: a one-element NCCL all-reduce.
tb_status enqueue_barrier(Comm* c, Stream* st) {
  void* p = reinterpret_cast<void*>(c->barrier_word);
  ncclResult_t r = nccl().AllReduce(p, p, 1, ncclInt32, ncclSum, c->comm, st->raw);
  if (r != ncclSuccess && r != ncclInProgress) return nccl_error("ncclAllReduce", r);
  tb_status rc = settle(c, "ncclAllReduce");
  if (rc) return rc;
  return track(c, st);
}

void unmap(PeerMapping& m) {
  const DriverApi* d = driver();
  for (CUdeviceptr p : m.opened)
    if (p && d) d->cuIpcCloseMemHandle(p);
  m.opened.clear();
  for (CUdeviceptr p : m.signal_opened)
    if (p && d) d->cuIpcCloseMemHandle(p);
  m.signal_opened.clear();
  if (m.signal_local && d) d->cuMemFree_v2(m.signal_local);
  m.signal_local = 0;
  if (m.ready && d) d->cuMemFree_v2(m.ready);
  m.ready = 0;
  if (m.local) tb_buffer_release(reinterpret_cast<tb_buffer*>(m.local));
  m.local = nullptr;
}

PeerMapping* find_mapping(Comm* c, const Buffer* b) {
  for (PeerMapping& m : c->mappings)
    if (m.local == b) return &m;
  return nullptr;
}

// What one rank publishes about its registered buffer.
struct MappingRecord {
  CUipcMemHandle handle;         // the buffer's allocation
  CUipcMemHandle signal_handle;  // the rank's signal block
  uint64_t offset;               // of the buffer inside its allocation
  uint64_t bytes;
  int32_t pci_domain, pci_bus, pci_device, pad;
};

}  // namespace
}  // namespace tb

using namespace tb;

extern "C" {

tb_status tb_comm_unique_id(uint8_t id[TB_COMM_ID_BYTES]) {
  NcclApi& n = nccl();
  if (!n.ok) return set_error(TB_ERR_NCCL, "load_nccl", n.error);
  static_assert(sizeof(ncclUniqueId) == TB_COMM_ID_BYTES, "ncclUniqueId size");
  ncclUniqueId uid;
  ncclResult_t r = n.GetUniqueId(&uid);
  if (r != ncclSuccess) return nccl_error("ncclGetUniqueId", r);
  memcpy(id, &uid, TB_COMM_ID_BYTES);
  return TB_OK;
}

tb_status tb_comm_init(tb_session* session, const uint8_t id[TB_COMM_ID_BYTES], int nranks, int rank,
                       uint32_t timeout_ms, tb_comm** out) {
  Session* s = reinterpret_cast<Session*>(session);
  if (!s || !id || !out) return set_error(TB_ERR_INVALID, "comm_init", "null argument");
  if (nranks < 1 || rank < 0 || rank >= nranks) return set_error(TB_ERR_INVALID, "comm_init", "bad rank or size");
  NcclApi& n = nccl();
  if (!n.ok) return set_error(TB_ERR_NCCL, "load_nccl", n.error);
  tb_status rc = activate(s);
  if (rc) return rc;
  Comm* c = new Comm();
  c->session = s;
  c->rank = rank;
  c->size = nranks;
  c->timeout_ms = timeout_ms ? timeout_ms : 60000;
  ncclUniqueId uid;
  memcpy(&uid, id, TB_COMM_ID_BYTES);
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  ncclResult_t r = n.CommInitRankConfig(&c->comm, nranks, uid, rank, &cfg);
  if (r != ncclSuccess && r != ncclInProgress) {
    delete c;
    return nccl_error("ncclCommInitRankConfig", r);
  }
  rc = settle(c, "ncclCommInitRankConfig");
  if (rc) {
    if (c->comm) n.CommAbort(c->comm);
    delete c;
    return rc;
  }
  CUresult cr = driver()->cuMemAlloc_v2(&c->barrier_word, 64);
  if (cr != CUDA_SUCCESS) {
    n.CommAbort(c->comm);
    delete c;
    return cu_error("allocate", cr);
  }
  s->refs.fetch_add(1);
  c->watchdog = std::thread(watchdog_loop, c);
  *out = reinterpret_cast<tb_comm*>(c);
  return TB_OK;
}

void tb_comm_release(tb_comm* comm) {
  Comm* c = reinterpret_cast<Comm*>(comm);
  if (!c) return;
  {
    std::lock_guard<std::mutex> lock(c->mu);
    c->stop = true;
  }
  c->cv.notify_all();
  if (c->watchdog.joinable()) c->watchdog.join();
  const DriverApi* d = driver();
  NcclApi& n = nccl();
  if (d) d->cuCtxSetCurrent(c->session->context);
  for (auto& p : c->pending) {
    if (d) {
      // Bounded: the watchdog is gone, so abort rather than wait on a collective that never finishes.
      if (d->cuEventQuery(p.first) != CUDA_SUCCESS && c->comm) {
        n.CommAbort(c->comm);
        c->comm = nullptr;
      }
      d->cuEventDestroy_v2(p.first);
    }
  }
  for (PeerMapping& m : c->mappings) unmap(m);
  if (c->comm) n.CommDestroy(c->comm);
  if (d && c->barrier_word) d->cuMemFree_v2(c->barrier_word);
  Session* s = c->session;
  delete c;
  tb_session_release(reinterpret_cast<tb_session*>(s));
}

int tb_comm_rank(const tb_comm* comm) { return comm ? reinterpret_cast<const Comm*>(comm)->rank : -1; }
int tb_comm_size(const tb_comm* comm) { return comm ? reinterpret_cast<const Comm*>(comm)->size : 0; }

tb_status tb_comm_all_gather(tb_comm* comm, tb_stream* stream, tb_buffer* send, tb_buffer* recv,
                             size_t bytes_per_rank, tb_event** out) {
  Comm* c = reinterpret_cast<Comm*>(comm);
  tb_status rc = usable(c, "all_gather");
  if (rc) return rc;
  Session* s = c->session;
  Stream* st = nullptr;
  Buffer *bs = nullptr, *br = nullptr;
  if ((rc = check_stream(s, stream, &st)) || (rc = check_buffer(s, send, &bs)) || (rc = check_buffer(s, recv, &br)))
    return rc;
  if (bytes_per_rank > bs->bytes || bytes_per_rank * (size_t)c->size > br->bytes)
    return set_error(TB_ERR_INVALID, "all_gather", "transfer exceeds allocation");
  rc = activate(s);
  if (rc) return rc;
  ncclResult_t r = nccl().AllGather(reinterpret_cast<const void*>(bs->ptr), reinterpret_cast<void*>(br->ptr),
                                    bytes_per_rank, ncclUint8, c->comm, st->raw);
  if (r != ncclSuccess && r != ncclInProgress) return nccl_error("ncclAllGather", r);
  if ((rc = settle(c, "ncclAllGather")) || (rc = track(c, st))) return rc;
  return record_event(s, st, nullptr, out);
}

tb_status tb_comm_barrier(tb_comm* comm, tb_stream* stream) {
  Comm* c = reinterpret_cast<Comm*>(comm);
  tb_status rc = usable(c, "barrier");
  if (rc) return rc;
  Stream* st = nullptr;
  if ((rc = check_stream(c->session, stream, &st))) return rc;
  rc = activate(c->session);
  if (rc) return rc;
  return enqueue_barrier(c, st);
}

tb_status tb_comm_register_buffer(tb_comm* comm, tb_stream* stream, tb_buffer* buffer) {
  Comm* c = reinterpret_cast<Comm*>(comm);
  tb_status rc = usable(c, "register");
  if (rc) return rc;
  Session* s = c->session;
  Stream* st = nullptr;
  Buffer* b = nullptr;
  if ((rc = check_stream(s, stream, &st)) || (rc = check_buffer(s, buffer, &b))) return rc;
  if (find_mapping(c, b)) return set_error(TB_ERR_INVALID, "register", "buffer is already registered with this communicator");
  rc = activate(s);
  if (rc) return rc;
  const DriverApi* d = driver();
  const int p = c->size;
  PeerMapping m;
  m.base.assign(p, 0);
  m.bytes.assign(p, 0);
  m.opened.assign(p, 0);
  m.base[c->rank] = b->ptr;
  m.bytes[c->rank] = b->bytes;
  m.signal.assign(p, 0);
  m.signal_opened.assign(p, 0);
  TB_CU("allocate", d->cuMemAlloc_v2(&m.signal_local, TB_SIGNAL_BLOCK_BYTES));
  m.signal[c->rank] = m.signal_local;
  // Tile counters for the pusher-CTA kernel (two per 256x256 tile of a rank's column
  // block): one per 16 KB of the buffer, at least 1024. A call that needs more, or a
  // failed allocation, runs the kernel with in-CTA push warps instead.
  m.ready_count = b->bytes / 16384 > 1024 ? b->bytes / 16384 : 1024;
  if (d->cuMemAlloc_v2(&m.ready, m.ready_count * sizeof(uint32_t)) != CUDA_SUCCESS) {
    m.ready = 0;
    m.ready_count = 0;
  }
  CUresult zr = d->cuMemsetD32Async(m.signal_local, 0, TB_SIGNAL_BLOCK_BYTES / 4, st->raw);
  if (zr == CUDA_SUCCESS) zr = d->cuStreamSynchronize(st->raw);
  if (zr != CUDA_SUCCESS) {
    unmap(m);
    return cu_error("register", zr);
  }
  if (p > 1) {
    // Publish (IPC handle of the allocation, offset, size) and gather everyone's.
    CUdeviceptr alloc_base = 0;
    size_t alloc_size = 0;
    TB_CU("cuMemGetAddressRange", d->cuMemGetAddressRange_v2(&alloc_base, &alloc_size, b->ptr));
    MappingRecord mine{};
    CUresult hr = d->cuIpcGetMemHandle(&mine.handle, alloc_base);
    if (hr == CUDA_SUCCESS) hr = d->cuIpcGetMemHandle(&mine.signal_handle, m.signal_local);
    if (hr == CUDA_SUCCESS) hr = d->cuDeviceGetAttribute(&mine.pci_domain, CU_DEVICE_ATTRIBUTE_PCI_DOMAIN_ID, s->device);
    if (hr == CUDA_SUCCESS) hr = d->cuDeviceGetAttribute(&mine.pci_bus, CU_DEVICE_ATTRIBUTE_PCI_BUS_ID, s->device);
    if (hr == CUDA_SUCCESS) hr = d->cuDeviceGetAttribute(&mine.pci_device, CU_DEVICE_ATTRIBUTE_PCI_DEVICE_ID, s->device);
    if (hr != CUDA_SUCCESS) {
      unmap(m);
      return cu_error("register", hr);
    }
    mine.offset = b->ptr - alloc_base;
    mine.bytes = b->bytes;
    std::vector<MappingRecord> all(p);
    CUdeviceptr dev = 0;
    TB_CU("allocate", d->cuMemAlloc_v2(&dev, sizeof(MappingRecord) * p));
    const CUdeviceptr slot = dev + sizeof(MappingRecord) * c->rank;
    CUresult cr = d->cuMemcpyHtoDAsync_v2(slot, &mine, sizeof(mine), st->raw);
    ncclResult_t r = ncclSuccess;
    if (cr == CUDA_SUCCESS) {
      r = nccl().AllGather(reinterpret_cast<const void*>(slot), reinterpret_cast<void*>(dev), sizeof(MappingRecord),
                           ncclUint8, c->comm, st->raw);
      if (r == ncclSuccess || r == ncclInProgress) rc = settle(c, "ncclAllGather");
      if ((r == ncclSuccess || r == ncclInProgress) && rc == TB_OK)
        cr = d->cuMemcpyDtoHAsync_v2(all.data(), dev, sizeof(MappingRecord) * p, st->raw);
      if (cr == CUDA_SUCCESS) cr = d->cuStreamSynchronize(st->raw);
    }
    d->cuMemFree_v2(dev);
    if (cr != CUDA_SUCCESS || (r != ncclSuccess && r != ncclInProgress) || rc) {
      unmap(m);
      if (cr != CUDA_SUCCESS) return cu_error("register", cr);
      if (r != ncclSuccess && r != ncclInProgress) return nccl_error("ncclAllGather", r);
      return rc;
    }
    // The fused kernels of different ranks wait on each other's flags, which is only
    // safe when every rank has its own GPU.
    for (int i = 0; i < p; ++i)
      for (int j = i + 1; j < p; ++j)
        if (all[i].pci_domain == all[j].pci_domain && all[i].pci_bus == all[j].pci_bus &&
            all[i].pci_device == all[j].pci_device) {
          unmap(m);
          return set_error(TB_ERR_UNSUPPORTED, "register",
                           "ranks " + std::to_string(i) + " and " + std::to_string(j) +
                               " share a GPU; peer-store collectives need one GPU per rank");
        }
    for (int j = 0; j < p; ++j) {
      if (j == c->rank) continue;
      CUdeviceptr peer = 0, peer_signal = 0;
      cr = d->cuIpcOpenMemHandle_v2(&peer, all[j].handle, CU_IPC_MEM_LAZY_ENABLE_PEER_ACCESS);
      if (cr == CUDA_SUCCESS) {
        m.opened[j] = peer;
        cr = d->cuIpcOpenMemHandle_v2(&peer_signal, all[j].signal_handle, CU_IPC_MEM_LAZY_ENABLE_PEER_ACCESS);
      }
      if (cr != CUDA_SUCCESS) {
        unmap(m);
        return cu_error("cuIpcOpenMemHandle", cr);
      }
      m.signal_opened[j] = peer_signal;
      m.signal[j] = peer_signal;
      m.base[j] = peer + all[j].offset;
      m.bytes[j] = all[j].bytes;
    }
  }
  tb_buffer_retain(buffer);
  m.local = b;
  c->mappings.push_back(std::move(m));
  return TB_OK;
}

tb_status tb_comm_deregister_buffer(tb_comm* comm, tb_buffer* buffer) {
  Comm* c = reinterpret_cast<Comm*>(comm);
  if (!c) return set_error(TB_ERR_INVALID, "deregister", "null communicator");
  Buffer* b = nullptr;
  tb_status rc = check_buffer(c->session, buffer, &b);
  if (rc) return rc;
  for (size_t i = 0; i < c->mappings.size(); ++i) {
    if (c->mappings[i].local != b) continue;
    activate(c->session);
    unmap(c->mappings[i]);
    c->mappings.erase(c->mappings.begin() + (long)i);
    return TB_OK;
  }
  return set_error(TB_ERR_INVALID, "deregister", "buffer is not registered with this communicator");
}

tb_status tb_op_gemm_sharded(tb_comm* comm, tb_stream* stream, const tb_tensor* lhs, const tb_tensor* rhs_shard,
                             const tb_tensor* output, tb_buffer* workspace, tb_event** out) {
  Comm* c = reinterpret_cast<Comm*>(comm);
  tb_status rc = usable(c, "contract");
  if (rc) return rc;
  Session* s = c->session;
  if (!lhs || !rhs_shard || !output) return contract("sharded GEMM requires A, a B shard and an output");
  if (lhs->dtype != TB_BF16 || rhs_shard->dtype != TB_BF16 || output->dtype != TB_BF16)
    return contract("sharded GEMM requires BF16 A, B shard and C");
  if (lhs->rank != 2 || rhs_shard->rank != 2 || output->rank != 2 || !is_contiguous(lhs) ||
      !is_contiguous(rhs_shard) || !is_contiguous(output))
    return contract("sharded GEMM requires contiguous rank-2 tensors");
  const uint64_t M = lhs->shape[0], K = lhs->shape[1], Np = rhs_shard->shape[0], p = (uint64_t)c->size;
  if (rhs_shard->shape[1] != K) return contract("gemm inner dimensions must match");
  if (output->shape[0] != M || output->shape[1] != Np * p) return contract("gemm output shape mismatch");
  if (K % 8 != 0 || Np % 8 != 0) return unsupported("sharded GEMM needs K and N/p to be multiples of 8");
  Stream* st = nullptr;
  Buffer *ba = nullptr, *bb = nullptr, *bc = nullptr, *bw = nullptr;
  if ((rc = check_stream(s, stream, &st)) || (rc = tensor_buffer(s, lhs, "gemm lhs", &ba)) ||
      (rc = tensor_buffer(s, rhs_shard, "gemm rhs", &bb)) || (rc = tensor_buffer(s, output, "gemm output", &bc)))
    return rc;
  PeerMapping* mapping = find_mapping(c, bc);
  if (mapping) {
    // Fused: every rank's C is mapped here; this rank's column block goes to all of them.
    for (int j = 0; j < (int)p; ++j)
      if (mapping->bytes[j] < M * Np * p * 2) return contract("a rank's registered output is smaller than C");
    if (p > TB_MAX_RANKS) return unsupported("fused all-gather supports at most 8 ranks");
    rc = activate(s);
    if (rc) return rc;
    rc = launch_gemm_bf16_tn_allgather(s, st, ba->ptr, bb->ptr, mapping->base.data(), mapping->signal.data(), (int)p,
                                       c->rank, mapping->epoch + 1, (int)M, (int)Np, (int)K, (long long)(Np * p),
                                       (long long)(Np * (uint64_t)c->rank), mapping->ready, mapping->ready_count);
    if (rc) return rc;
    ++mapping->epoch;
    return record_event(s, st, nullptr, out);
  }
  if ((rc = check_buffer(s, workspace, &bw))) return rc;
  const size_t shard_bytes = M * Np * 2;
  if (bw->bytes < shard_bytes * p) return contract("sharded GEMM workspace holds fewer than p*M*(N/p) elements");
  rc = activate(s);
  if (rc) return rc;
  // 1. This rank's columns straight into its slot of the gather layout [p][M][N/p].
  const CUdeviceptr slot = bw->ptr + (CUdeviceptr)c->rank * shard_bytes;
  rc = launch_gemm_bf16_default(s, st, ba->ptr, bb->ptr, slot, (int)M, (int)Np, (int)K, (long long)Np);
  if (rc) return rc;
  // 2. In-place all-gather of the shards over NVLink.
  if (p > 1) {
    ncclResult_t r = nccl().AllGather(reinterpret_cast<const void*>(slot), reinterpret_cast<void*>(bw->ptr),
                                      shard_bytes, ncclUint8, c->comm, st->raw);
    if (r != ncclSuccess && r != ncclInProgress) return nccl_error("ncclAllGather", r);
    if ((rc = settle(c, "ncclAllGather")) || (rc = track(c, st))) return rc;
  }
  // 3. Column blocks -> row-major C[M, N].
  CUfunction fn = nullptr;
  rc = builtin_function(s, "layout", "gather_column_blocks_bf16", &fn);
  if (rc) return rc;
  CUdeviceptr src = bw->ptr, dst = bc->ptr;
  int m = (int)M, np = (int)Np, parts = (int)p;
  void* params[] = {&src, &dst, &m, &np, &parts};
  const uint64_t vecs = M * Np * p / 8;
  uint64_t grid = (vecs + 255) / 256;
  if (grid > (uint64_t)s->sm_count * 16) grid = (uint64_t)s->sm_count * 16;
  rc = launch_builtin(s, st, fn, (unsigned)grid, 1, 1, 256, 0, params, "gather_column_blocks_bf16");
  if (rc) return rc;
  return record_event(s, st, nullptr, out);
}

}  // extern "C"
