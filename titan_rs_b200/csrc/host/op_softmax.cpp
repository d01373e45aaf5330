// "softmax" operator entry: the contract of execute_cuda_softmax
// (titan-runtime/src/lib.rs:1504-1596), then the B200 kernel choice. Besides the
// reference's `axis`, the operator takes `candidate` (a registered kernel name:
// softmax_f32_warp{1,2,4,8,16,32} for rows of at most that many x 128 columns, or
// softmax_f32_stream), which the autotuner uses. BF16 input and output (an extension
// for bf16 graphs) take softmax_bf16_rows: fp32 arithmetic, one rounding.
#include "ops_common.hpp"

using namespace tb;

extern "C" tb_status tb_op_softmax(tb_session* session, tb_stream* stream, const tb_tensor* input,
                                   const tb_tensor* output, const tb_attr* attrs, uint32_t num_attrs, tb_event** out) {
  Session* s = reinterpret_cast<Session*>(session);
  if (!s) return set_error(TB_ERR_INVALID, "contract", "null session");
  if (!input || !output) return contract("CUDA softmax requires exactly one input and one output");
  const char* candidate = nullptr;
  for (uint32_t i = 0; i < num_attrs; ++i) {
    if (attrs[i].key && strcmp(attrs[i].key, "candidate") == 0) {
      if (!attrs[i].str) return contract("softmax candidate must be a string");
      candidate = attrs[i].str;
      continue;
    }
    if (!attrs[i].key || strcmp(attrs[i].key, "axis") != 0)
      return contract("CUDA softmax only accepts the axis attribute");
  }
  const bool bf16 = input->dtype == TB_BF16 && output->dtype == TB_BF16;
  if (!bf16 && (input->dtype != TB_F32 || output->dtype != TB_F32))
    return contract("CUDA softmax requires F32 input and output (or BF16 input and output)");
  if (input->rank == 0 || input->rank > TB_MAX_RANK) return contract("CUDA softmax requires a non-scalar input");
  if (!is_contiguous(input)) return contract("CUDA softmax requires a contiguous input");
  int64_t last = (int64_t)input->rank - 1, axis = 0;
  tb_status rc = int_attr(attrs, num_attrs, "axis", &last, &axis);
  if (rc) return rc;
  if (axis != last) return contract("CUDA softmax only supports the last axis");
  bool same = output->rank == input->rank;
  for (uint32_t a = 0; same && a < input->rank; ++a) same = output->shape[a] == input->shape[a];
  if (!same || !is_contiguous(output))
    return contract("CUDA softmax requires a contiguous output with the same shape as the input");
  uint64_t cols = input->shape[input->rank - 1];
  uint64_t rows = 1;
  for (uint32_t a = 0; a + 1 < input->rank; ++a) rows *= input->shape[a];
  if (rows == 0 || cols == 0) return contract("CUDA softmax requires non-zero dimensions");
  if (rows > 0x7fffffffull) return contract("CUDA softmax row count exceeds i32 ABI");
  if (cols > 0x7fffffffull) return contract("CUDA softmax axis length exceeds i32 ABI");
  Stream* st = nullptr;
  rc = check_stream(s, stream, &st);
  if (rc) return rc;
  Buffer *bin = nullptr, *bout = nullptr;
  rc = tensor_buffer(s, input, "softmax input", &bin);
  if (rc) return rc;
  rc = tensor_buffer(s, output, "softmax output", &bout);
  if (rc) return rc;
  rc = activate(s);
  if (rc) return rc;

  int r = (int)rows, c = (int)cols;
  CUdeviceptr pin = bin->ptr, pout = bout->ptr;
  void* params[] = {&pin, &pout, &r, &c};
  if (bf16) {
    if (candidate && strcmp(candidate, "softmax_bf16_rows") != 0)
      return contract(std::string("unknown BF16 softmax candidate ") + candidate);
    CUfunction fn = nullptr;
    rc = builtin_function(s, "softmax", "softmax_bf16_rows", &fn);
    if (rc) return rc;
    uint64_t grid = (rows + 7) / 8;  // 8 rows (warps) per 256-thread CTA
    if (grid > (uint64_t)s->sm_count * 32) grid = (uint64_t)s->sm_count * 32;
    rc = launch_builtin(s, st, fn, (unsigned)grid, 1, 1, 256, 0, params, "softmax_bf16_rows");
    if (rc) return rc;
    return record_event(s, st, nullptr, out);
  }
  const bool aligned = ((pin | pout) & 15u) == 0;
  const bool reg_ok = aligned && cols % 4 == 0 && cols <= 4096;
  // Register-path variants: one warp per row, up to `nv` x 128 columns.
  static const struct {
    const char* name;
    uint64_t nv;
  } kWarp[] = {{"softmax_f32_warp1", 1},  {"softmax_f32_warp2", 2},   {"softmax_f32_warp4", 4},
               {"softmax_f32_warp8", 8},  {"softmax_f32_warp16", 16}, {"softmax_f32_warp32", 32}};
  const char* entry = nullptr;  // a register-path variant, or null for the streaming kernel
  if (candidate) {
    bool known = strcmp(candidate, "softmax_f32_stream") == 0;
    for (const auto& w : kWarp) {
      if (strcmp(candidate, w.name) != 0) continue;
      known = true;
      if (!reg_ok || cols > 128 * w.nv)
        return unsupported(std::string("candidate ") + candidate + " does not take this shape or alignment");
      entry = w.name;
    }
    if (!known) return contract(std::string("unknown softmax candidate ") + candidate);
  } else if (reg_ok) {
    entry = cols <= 128    ? "softmax_f32_warp1"
            : cols <= 256  ? "softmax_f32_warp2"
            : cols <= 512  ? "softmax_f32_warp4"
            : cols <= 1024 ? "softmax_f32_warp8"
            : cols <= 2048 ? "softmax_f32_warp16"
                           : "softmax_f32_warp32";
  }
  CUfunction fn = nullptr;
  if (entry) {
    rc = builtin_function(s, "softmax", entry, &fn);
    if (rc) return rc;
    // 4 rows (warps) per 128-thread CTA; one CTA per 4 rows.
    uint64_t grid = (rows + 3) / 4;
    rc = launch_builtin(s, st, fn, (unsigned)grid, 1, 1, 128, 0, params, entry);
  } else {
    rc = builtin_function(s, "softmax", "softmax_f32_stream", &fn);
    if (rc) return rc;
    unsigned block = cols >= 8192 ? 512 : 256;
    uint64_t grid = rows < (uint64_t)s->sm_count * 16 ? rows : (uint64_t)s->sm_count * 16;
    rc = launch_builtin(s, st, fn, (unsigned)grid, 1, 1, block, 0, params, "softmax_f32_stream");
  }
  if (rc) return rc;
  return record_event(s, st, nullptr, out);
}
