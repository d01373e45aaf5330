// "scaled_dot_product_attention" operator entry: the contract of
// execute_cuda_attention and the CPU reference (titan-runtime/src/lib.rs:2575-2705,
// 1090-1151), then the kernel choice:
//   BF16, D == 128, 16-byte aligned  -> sdpa_fwd_bf16_d128_pair (tcgen05, TMA, TMEM; two query
//                                       tiles per CTA); causal optional. Candidates
//                                       sdpa_fwd_bf16_d128 (one query tile, P through shared
//                                       memory) and sdpa_fwd_bf16_d128_bn64 (64-key tiles, two
//                                       CTAs per SM) take the same inputs
//   BF16, other head dims            -> sdpa_bf16_generic (CUDA cores)
//   F32                              -> scaled_dot_product_attention_f32 (reference ABI kernel);
//                                       mask/causal rejected as the reference does
// BF16 also takes `scale` (a decimal string, > 0): the factor applied to Q K^T in place
// of the reference's fixed 1/sqrt(D). The graph compiler's attention fusion uses it for
// gemm -> softmax -> gemm chains, which carry no scale.
#include <cmath>
#include <cstdlib>

#include "../kernels/kernel_configs.h"
#include "ops_common.hpp"

namespace tb {

tb_status tmap_bhtd(CUtensorMap* map, CUdeviceptr base, uint64_t bh, uint64_t t, uint64_t d, uint32_t box_rows = 128) {
  cuuint64_t dims[3] = {d, t, bh};
  cuuint64_t strides[2] = {d * 2, t * d * 2};
  cuuint32_t box[3] = {64, box_rows, 1};
  cuuint32_t elem[3] = {1, 1, 1};
  TB_CU("cuTensorMapEncodeTiled",
        driver()->cuTensorMapEncodeTiled(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, reinterpret_cast<void*>(base), dims,
                                         strides, box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                         CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE));
  return TB_OK;
}

tb_status launch_sdpa_bf16_d128(Session* s, Stream* st, CUdeviceptr q, CUdeviceptr k, CUdeviceptr v, CUdeviceptr o,
                                int bh, int tq, int tk, int causal, float scale) {
  CUtensorMap mq, mk, mv;
  tb_status rc;
  if ((rc = tmap_bhtd(&mq, q, bh, tq, TB_SDPA_HD)) || (rc = tmap_bhtd(&mk, k, bh, tk, TB_SDPA_HD)) ||
      (rc = tmap_bhtd(&mv, v, bh, tk, TB_SDPA_HD)))
    return rc;
  CUfunction fn = nullptr;
  rc = builtin_function(s, "sdpa_bf16", "sdpa_fwd_bf16_d128", &fn);
  if (rc) return rc;
  float scale_log2 = (float)(1.4426950408889634 * (double)scale);  // the kernels exponentiate base 2
  CUdeviceptr status = s->status.device;
  void* params[] = {&mq, &mk, &mv, &o, &tq, &tk, &causal, &scale_log2, &status};
  const unsigned long long qtiles = (unsigned long long)((tq + TB_SDPA_BM - 1) / TB_SDPA_BM);
  if (qtiles * (unsigned long long)bh > 0x7fffffffull) return contract("CUDA attention grid exceeds 2^31 CTAs");
  return launch_builtin(s, st, fn, (unsigned)(qtiles * bh), 1, 1, TB_SDPA_THREADS, TB_SDPA_SMEM_BYTES, params,
                        "sdpa_fwd_bf16_d128");
}

tb_status launch_sdpa_bf16_d128_pair(Session* s, Stream* st, CUdeviceptr q, CUdeviceptr k, CUdeviceptr v,
                                     CUdeviceptr o, int bh, int tq, int tk, int causal, float scale) {
  CUtensorMap mq, mk, mv;
  tb_status rc;
  if ((rc = tmap_bhtd(&mq, q, bh, tq, TB_SDPA_HD)) || (rc = tmap_bhtd(&mk, k, bh, tk, TB_SDPA_HD)) ||
      (rc = tmap_bhtd(&mv, v, bh, tk, TB_SDPA_HD)))
    return rc;
  CUfunction fn = nullptr;
  rc = builtin_function(s, "sdpa_bf16_pair", "sdpa_fwd_bf16_d128_pair", &fn);
  if (rc) return rc;
  // The kernel's warpgroups re-divide the registers the CTA was launched with; a launch
  // with fewer than it assumes would leave the softmax warpgroups waiting for registers.
  int regs = 0;
  TB_CU("cuFuncGetAttribute", driver()->cuFuncGetAttribute(&regs, CU_FUNC_ATTRIBUTE_NUM_REGS, fn));
  if (regs < TB_SDPA2_PAIR_LAUNCH_REGS)
    return unsupported("sdpa_fwd_bf16_d128_pair was built with fewer registers than its warpgroups share");
  float scale_log2 = (float)(1.4426950408889634 * (double)scale);  // the kernels exponentiate base 2
  CUdeviceptr status = s->status.device;
  void* params[] = {&mq, &mk, &mv, &o, &tq, &tk, &causal, &scale_log2, &status};
  const unsigned long long pairs = (unsigned long long)((tq + 2 * TB_SDPA_BM - 1) / (2 * TB_SDPA_BM));
  if (pairs * (unsigned long long)bh > 0x7fffffffull) return contract("CUDA attention grid exceeds 2^31 CTAs");
  return launch_builtin(s, st, fn, (unsigned)(pairs * bh), 1, 1, TB_SDPA2_PAIR_THREADS, TB_SDPA2_SMEM_BYTES, params,
                        "sdpa_fwd_bf16_d128_pair");
}

// The pair pipeline on persistent CTAs (one per SM) walking every (batch*head, pair)
// item; the kernel's own schedule, so the grid is just the SM count (or fewer items).
tb_status launch_sdpa_bf16_d128_persist(Session* s, Stream* st, CUdeviceptr q, CUdeviceptr k, CUdeviceptr v,
                                        CUdeviceptr o, int bh, int tq, int tk, int causal, float scale) {
  CUtensorMap mq, mk, mv;
  tb_status rc;
  if ((rc = tmap_bhtd(&mq, q, bh, tq, TB_SDPA_HD)) || (rc = tmap_bhtd(&mk, k, bh, tk, TB_SDPA_HD)) ||
      (rc = tmap_bhtd(&mv, v, bh, tk, TB_SDPA_HD)))
    return rc;
  CUfunction fn = nullptr;
  rc = builtin_function(s, "sdpa_bf16_persist", "sdpa_fwd_bf16_d128_persist", &fn);
  if (rc) return rc;
  // Same register split as the pair kernel.
  int regs = 0;
  TB_CU("cuFuncGetAttribute", driver()->cuFuncGetAttribute(&regs, CU_FUNC_ATTRIBUTE_NUM_REGS, fn));
  if (regs < TB_SDPA2_PAIR_LAUNCH_REGS)
    return unsupported("sdpa_fwd_bf16_d128_persist was built with fewer registers than its warpgroups share");
  float scale_log2 = (float)(1.4426950408889634 * (double)scale);  // the kernels exponentiate base 2
  CUdeviceptr status = s->status.device;
  const unsigned long long items =
      (unsigned long long)((tq + 2 * TB_SDPA_BM - 1) / (2 * TB_SDPA_BM)) * (unsigned long long)bh;
  if (items > 0x7fffffffull) return contract("CUDA attention work list exceeds 2^31 items");
  const unsigned grid = (unsigned)std::min<unsigned long long>(items, (unsigned long long)s->sm_count);
  // The work-item counter the CTAs draw from, zeroed in stream order before the launch.
  CUdeviceptr next_item = 0;
  if ((rc = stream_scratch(s, st, sizeof(uint32_t), &next_item))) return rc;
  TB_CU("cuMemsetD32Async", driver()->cuMemsetD32Async(next_item, 0, 1, st->raw));
  void* params[] = {&mq, &mk, &mv, &o, &bh, &tq, &tk, &causal, &scale_log2, &next_item, &status};
  return launch_builtin(s, st, fn, grid, 1, 1, TB_SDPA2_PAIR_THREADS, TB_SDPA2_SMEM_BYTES, params,
                        "sdpa_fwd_bf16_d128_persist");
}

tb_status launch_sdpa_bf16_d128_bn64(Session* s, Stream* st, CUdeviceptr q, CUdeviceptr k, CUdeviceptr v,
                                     CUdeviceptr o, int bh, int tq, int tk, int causal, float scale) {
  CUtensorMap mq, mk, mv;
  tb_status rc;
  if ((rc = tmap_bhtd(&mq, q, bh, tq, TB_SDPA_HD, 128)) || (rc = tmap_bhtd(&mk, k, bh, tk, TB_SDPA_HD, TB_SDPA3_BN)) ||
      (rc = tmap_bhtd(&mv, v, bh, tk, TB_SDPA_HD, TB_SDPA3_BN)))
    return rc;
  CUfunction fn = nullptr;
  rc = builtin_function(s, "sdpa_bf16_bn64", "sdpa_fwd_bf16_d128_bn64", &fn);
  if (rc) return rc;
  float scale_log2 = (float)(1.4426950408889634 * (double)scale);  // the kernels exponentiate base 2
  CUdeviceptr status = s->status.device;
  void* params[] = {&mq, &mk, &mv, &o, &tq, &tk, &causal, &scale_log2, &status};
  const unsigned long long qtiles = (unsigned long long)((tq + TB_SDPA_BM - 1) / TB_SDPA_BM);
  if (qtiles * (unsigned long long)bh > 0x7fffffffull) return contract("CUDA attention grid exceeds 2^31 CTAs");
  return launch_builtin(s, st, fn, (unsigned)(qtiles * bh), 1, 1, TB_SDPA3_THREADS, TB_SDPA3_SMEM_BYTES, params,
                        "sdpa_fwd_bf16_d128_bn64");
}

}  // namespace tb

using namespace tb;

extern "C" tb_status tb_op_sdpa(tb_session* session, tb_stream* stream, const tb_tensor* q, const tb_tensor* k,
                                const tb_tensor* v, const tb_tensor* output, const tb_attr* attrs, uint32_t num_attrs,
                                tb_event** out) {
  Session* s = reinterpret_cast<Session*>(session);
  if (!s) return set_error(TB_ERR_INVALID, "contract", "null session");
  if (!q || !k || !v || !output)
    return contract("scaled dot-product attention requires exactly three rank-4 BHTD inputs");
  const uint32_t dt = q->dtype;
  bool causal = false;
  const char* candidate = nullptr;  // optional: name of a registered kernel to run (autotuning / tests)
  double scale = 0.0;               // optional score scale (a decimal string); 0 = the reference's 1/sqrt(D)
  if (dt == TB_F32) {
    if (num_attrs)
      return unsupported("CUDA scaled dot-product attention does not implement mask, causal, or other attributes");
  } else {
    for (uint32_t i = 0; i < num_attrs; ++i) {
      if (attrs[i].key && strcmp(attrs[i].key, "causal") == 0 && !attrs[i].str && attrs[i].value >= 0 &&
          attrs[i].value <= 1) {
        causal = attrs[i].value != 0;
        continue;
      }
      if (attrs[i].key && strcmp(attrs[i].key, "candidate") == 0 && attrs[i].str) {
        candidate = attrs[i].str;
        continue;
      }
      if (attrs[i].key && strcmp(attrs[i].key, "scale") == 0) {
        char* end = nullptr;
        scale = attrs[i].str ? strtod(attrs[i].str, &end) : 0.0;
        if (!attrs[i].str || end == attrs[i].str || *end != '\0' || !std::isfinite(scale) || !(scale > 0.0))
          return contract("scaled dot-product attention scale must be a positive finite number (decimal string)");
        continue;
      }
      return unsupported(
          "CUDA scaled dot-product attention does not implement mask or attributes other than causal and scale");
    }
  }
  if (!(dt == TB_F32 || dt == TB_BF16) || k->dtype != dt || v->dtype != dt || output->dtype != dt)
    return contract("CUDA scaled dot-product attention requires F32 (or BF16) Q, K, V, and output of one dtype");
  if (q->rank != 4 || k->rank != 4 || v->rank != 4)
    return contract("scaled dot-product attention requires exactly three rank-4 BHTD inputs");
  if (!is_contiguous(q) || !is_contiguous(k) || !is_contiguous(v))
    return contract("CUDA scaled dot-product attention requires contiguous rank-4 BHTD Q, K, and V");
  if (output->rank != 4 || !is_contiguous(output))
    return contract("CUDA scaled dot-product attention requires a contiguous rank-4 output");
  const uint64_t B = q->shape[0], H = q->shape[1], Tq = q->shape[2], D = q->shape[3];
  const uint64_t Tk = k->shape[2];
  if (k->shape[0] != B || v->shape[0] != B || k->shape[1] != H || v->shape[1] != H || k->shape[3] != D ||
      v->shape[3] != D || v->shape[2] != Tk)
    return contract("scaled dot-product attention B, H, D, and K/V sequence dimensions must match");
  if (Tq == 0 || Tk == 0 || D == 0)
    return contract("scaled dot-product attention requires non-zero Tq, Tk, and D dimensions");
  if (B == 0 || H == 0) return contract("CUDA attention B, H, Tq, Tk, and D must be non-zero");
  if (output->shape[0] != B || output->shape[1] != H || output->shape[2] != Tq || output->shape[3] != D)
    return contract("scaled dot-product attention output shape mismatch");
  if (B * H > 0x7fffffffull || Tq > 0x7fffffffull || Tk > 0x7fffffffull)
    return contract("CUDA attention shape exceeds u32 ABI");
  if (D > 256) return unsupported("CUDA scaled dot-product attention does not implement head dimensions above 256");
  Stream* st = nullptr;
  tb_status rc = check_stream(s, stream, &st);
  if (rc) return rc;
  Buffer *bq = nullptr, *bk = nullptr, *bv = nullptr, *bo = nullptr;
  if ((rc = tensor_buffer(s, q, "attention Q", &bq)) || (rc = tensor_buffer(s, k, "attention K", &bk)) ||
      (rc = tensor_buffer(s, v, "attention V", &bv)) || (rc = tensor_buffer(s, output, "attention output", &bo)))
    return rc;
  rc = activate(s);
  if (rc) return rc;
  CUdeviceptr pq = bq->ptr, pk = bk->ptr, pv = bv->ptr, po = bo->ptr;
  int b = (int)B, h = (int)H, tq = (int)Tq, tk = (int)Tk, d = (int)D, c = causal ? 1 : 0;
  float sc = (float)(scale > 0.0 ? scale : 1.0 / std::sqrt((double)D));
  const bool tc_ok = dt == TB_BF16 && D == TB_SDPA_HD && ((pq | pk | pv | po) & 15) == 0;
  if (candidate && strcmp(candidate, "sdpa_fwd_bf16_d128_pair") != 0 && strcmp(candidate, "sdpa_fwd_bf16_d128") != 0 &&
      strcmp(candidate, "sdpa_fwd_bf16_d128_bn64") != 0 && strcmp(candidate, "sdpa_fwd_bf16_d128_persist") != 0 &&
      strcmp(candidate, "sdpa_bf16_generic") != 0)
    return contract(std::string("unknown attention candidate ") + candidate);
  if (candidate && !tc_ok && strcmp(candidate, "sdpa_bf16_generic") != 0)
    return unsupported(std::string("candidate ") + candidate + " does not take this shape or alignment");
  if (tc_ok && (!candidate || strcmp(candidate, "sdpa_fwd_bf16_d128_pair") == 0)) {
    rc = launch_sdpa_bf16_d128_pair(s, st, pq, pk, pv, po, b * h, tq, tk, c, sc);
  } else if (tc_ok && strcmp(candidate, "sdpa_fwd_bf16_d128_persist") == 0) {
    rc = launch_sdpa_bf16_d128_persist(s, st, pq, pk, pv, po, b * h, tq, tk, c, sc);
  } else if (tc_ok && strcmp(candidate, "sdpa_fwd_bf16_d128_bn64") == 0) {
    rc = launch_sdpa_bf16_d128_bn64(s, st, pq, pk, pv, po, b * h, tq, tk, c, sc);
  } else if (tc_ok && strcmp(candidate, "sdpa_fwd_bf16_d128") == 0) {
    rc = launch_sdpa_bf16_d128(s, st, pq, pk, pv, po, b * h, tq, tk, c, sc);
  } else {
    const bool bf = dt == TB_BF16;
    CUfunction fn = nullptr;
    rc = builtin_function(s, "compat", bf ? "sdpa_bf16_generic" : "scaled_dot_product_attention_f32", &fn);
    if (rc) return rc;
    uint64_t rows = B * H * Tq;
    uint64_t grid = (rows + 7) / 8;
    if (grid > (uint64_t)s->sm_count * 64) grid = (uint64_t)s->sm_count * 64;
    if (bf) {
      void* params[] = {&pq, &pk, &pv, &po, &b, &h, &tq, &tk, &d, &c, &sc};
      rc = launch_builtin(s, st, fn, (unsigned)grid, 1, 1, 256, 0, params, "sdpa_bf16_generic");
    } else {
      void* params[] = {&pq, &pk, &pv, &po, &b, &h, &tq, &tk, &d};
      rc = launch_builtin(s, st, fn, (unsigned)grid, 1, 1, 256, 0, params, "scaled_dot_product_attention_f32");
    }
  }
  if (rc) return rc;
  return record_event(s, st, nullptr, out);
}
