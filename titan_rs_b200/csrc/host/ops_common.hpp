// Helpers shared by the operator entry points: contract checks with the
// runtime's messages, attribute lookup, tensor-map encoding and launches.
#pragma once

#include <string>

#include "internal.hpp"

namespace tb {

inline size_t dtype_size(uint32_t dt) {
  switch (dt) {
    case TB_F32:
    case TB_I32:
      return 4;
    case TB_F16:
    case TB_BF16:
      return 2;
    case TB_I64:
      return 8;
    default:
      return 0;
  }
}

inline const char* dtype_name(uint32_t dt) {
  switch (dt) {
    case TB_F32: return "F32";
    case TB_F16: return "F16";
    case TB_BF16: return "BF16";
    case TB_I32: return "I32";
    case TB_I64: return "I64";
    default: return "?";
  }
}

// Row-major strides for `shape` (contiguous_strides, titan-runtime/src/lib.rs:485-493).
inline bool is_contiguous(const tb_tensor* t) {
  int64_t step = 1;
  for (int a = (int)t->rank - 1; a >= 0; --a) {
    if (t->strides[a] != step) return false;
    step *= (int64_t)t->shape[a];
  }
  return true;
}

inline uint64_t numel(const tb_tensor* t) {
  uint64_t n = 1;
  for (uint32_t a = 0; a < t->rank; ++a) n *= t->shape[a];
  return n;
}

inline tb_status contract(const std::string& msg) { return set_error(TB_ERR_INVALID, "contract", msg); }
inline tb_status unsupported(const std::string& msg) { return set_error(TB_ERR_UNSUPPORTED, "contract", msg); }

inline const tb_attr* find_attr(const tb_attr* attrs, uint32_t n, const char* key) {
  for (uint32_t i = 0; i < n; ++i)
    if (attrs[i].key && strcmp(attrs[i].key, key) == 0) return &attrs[i];
  return nullptr;
}

// `int` attribute helper (titan-runtime/src/lib.rs:521-527).
inline tb_status int_attr(const tb_attr* attrs, uint32_t n, const char* key, const int64_t* dflt, int64_t* out) {
  const tb_attr* a = find_attr(attrs, n, key);
  if (!a) {
    if (!dflt) return contract(std::string("missing integer attribute ") + key);
    *out = *dflt;
    return TB_OK;
  }
  if (a->str) return contract(std::string(key) + " must be an integer");
  if (a->value < 0) return contract(std::string(key) + " must be non-negative");
  *out = a->value;
  return TB_OK;
}

// Resolves a tensor's buffer in this session and checks it holds the tensor.
inline tb_status tensor_buffer(Session* s, const tb_tensor* t, const char* what, Buffer** out) {
  tb_status rc = check_buffer(s, t->buffer, out);
  if (rc) return rc;
  uint64_t need = numel(t) * dtype_size(t->dtype);
  if ((*out)->bytes < need)
    return contract(std::string(what) + " buffer holds " + std::to_string((*out)->bytes) + " bytes, needs " +
                    std::to_string(need));
  return TB_OK;
}

// Launches a built-in kernel on a session stream and counts it.
inline tb_status launch_builtin(Session* s, Stream* st, CUfunction fn, unsigned gx, unsigned gy, unsigned gz,
                                unsigned bx, unsigned shared_bytes, void** params, const char* candidate,
                                unsigned cluster_x = 1) {
  const DriverApi* d = driver();
  if (shared_bytes > 48 * 1024)
    TB_CU("cuFuncSetAttribute",
          d->cuFuncSetAttribute(fn, CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES, (int)shared_bytes));
  if (cluster_x > 1) {
    CUlaunchConfig cfg{};
    cfg.gridDimX = gx;
    cfg.gridDimY = gy;
    cfg.gridDimZ = gz;
    cfg.blockDimX = bx;
    cfg.blockDimY = 1;
    cfg.blockDimZ = 1;
    cfg.sharedMemBytes = shared_bytes;
    cfg.hStream = st->raw;
    CUlaunchAttribute attr{};
    attr.id = CU_LAUNCH_ATTRIBUTE_CLUSTER_DIMENSION;
    attr.value.clusterDim.x = cluster_x;
    attr.value.clusterDim.y = 1;
    attr.value.clusterDim.z = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    TB_CU("cuLaunchKernelEx", d->cuLaunchKernelEx(&cfg, fn, params, nullptr));
  } else {
    TB_CU("cuLaunchKernel", d->cuLaunchKernel(fn, gx, gy, gz, bx, 1, 1, shared_bytes, st->raw, params, nullptr));
  }
  note_launch(candidate);
  return TB_OK;
}

// CTA pairs (clusters of two along x) of a built-in pair kernel that can be resident at
// once. The driver is asked once per kernel and session (each built-in pair kernel is
// always launched with the same block and shared-memory size).
inline tb_status pair_occupancy(Session* s, Stream* st, CUfunction fn, unsigned bx, unsigned shared_bytes,
                                const char* candidate, int* out) {
  int clusters = 0;
  {
    std::lock_guard<std::mutex> lock(s->mu);
    auto it = s->pair_occupancy.find(fn);
    if (it != s->pair_occupancy.end()) clusters = it->second;
  }
  if (clusters == 0) {
    const DriverApi* d = driver();
    TB_CU("cuFuncSetAttribute",
          d->cuFuncSetAttribute(fn, CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES, (int)shared_bytes));
    CUlaunchConfig cfg{};
    cfg.gridDimX = (unsigned)s->sm_count & ~1u;
    cfg.gridDimY = cfg.gridDimZ = 1;
    cfg.blockDimX = bx;
    cfg.blockDimY = cfg.blockDimZ = 1;
    cfg.sharedMemBytes = shared_bytes;
    cfg.hStream = st->raw;
    CUlaunchAttribute attr{};
    attr.id = CU_LAUNCH_ATTRIBUTE_CLUSTER_DIMENSION;
    attr.value.clusterDim.x = 2;
    attr.value.clusterDim.y = 1;
    attr.value.clusterDim.z = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    TB_CU("cuOccupancyMaxActiveClusters", d->cuOccupancyMaxActiveClusters(&clusters, fn, &cfg));
    if (clusters < 1) return unsupported(std::string("no CTA pair of ") + candidate + " fits on this device");
    std::lock_guard<std::mutex> lock(s->mu);
    s->pair_occupancy[fn] = clusters;
  }
  *out = clusters;
  return TB_OK;
}

// Launches a persistent kernel built on the 2-SM pipeline: as many pairs as can be
// resident at once, at most `pair_tiles`.
inline tb_status launch_builtin_pairs(Session* s, Stream* st, CUfunction fn, long long pair_tiles, unsigned bx,
                                      unsigned shared_bytes, void** params, const char* candidate) {
  int clusters = 0;
  tb_status rc = pair_occupancy(s, st, fn, bx, shared_bytes, candidate, &clusters);
  if (rc) return rc;
  const unsigned pairs = (unsigned)(pair_tiles < clusters ? pair_tiles : clusters);
  return launch_builtin(s, st, fn, 2 * pairs, 1, 1, bx, shared_bytes, params, candidate, 2);
}

// 2-D bf16 tensor map over a row-major [rows, cols] matrix with leading
// dimension `ld` elements; box = [box_rows, box_cols] with 128-byte swizzle.
inline tb_status tmap_bf16_2d(CUtensorMap* map, CUdeviceptr base, uint64_t rows, uint64_t cols, uint64_t ld,
                              uint32_t box_rows, uint32_t box_cols, CUtensorMapSwizzle swizzle,
                              CUtensorMapL2promotion promo = CU_TENSOR_MAP_L2_PROMOTION_L2_256B) {
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {ld * 2};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t elem[2] = {1, 1};
  TB_CU("cuTensorMapEncodeTiled",
        driver()->cuTensorMapEncodeTiled(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, reinterpret_cast<void*>(base), dims,
                                         strides, box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, promo,
                                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE));
  return TB_OK;
}

}  // namespace tb
