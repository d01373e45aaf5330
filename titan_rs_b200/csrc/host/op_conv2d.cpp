// "conv2d" operator entry: the contract of execute_cuda_conv2d and the CPU
// conv2d (titan-runtime/src/lib.rs:2406-2573, 991-1088), then the kernel choice:
//   F32 (NCHW input, OIHW weight)        -> conv2d_f32 (reference ABI kernel, bit-exact)
//   BF16 with layout="NHWC" (KRSC weight):
//     groups 1, Cin % 8 == 0, Cout % 8 == 0, stride <= 8, 16-byte aligned
//                                          -> conv2d_fprop_bf16_nhwc_2sm (tcgen05 implicit GEMM on
//                                             CTA pairs) when the output fills the SMs, else
//                                             conv2d_fprop_bf16_nhwc (one SM per tile)
//     otherwise                            -> conv2d_bf16_nhwc_generic (CUDA cores)
// A `candidate` attribute (not a reference attribute; the autotuner's) names one of
// these kernels; a kernel that does not take the problem is TB_ERR_UNSUPPORTED.
#include "../kernels/kernel_configs.h"
#include "ops_common.hpp"

namespace tb {

// pairs: -1 = choose (CTA pairs once the output holds a full wave of 128x256 tiles),
// 0 = conv2d_fprop_bf16_nhwc, 1 = conv2d_fprop_bf16_nhwc_2sm.
tb_status launch_conv2d_bf16(Session* s, Stream* st, CUdeviceptr x, CUdeviceptr w, CUdeviceptr bias, CUdeviceptr y,
                             int batch, int H, int W, int C, int Cout, int R, int S, int Ho, int Wo, int sh, int sw,
                             int ph, int pw, int dh, int dw, int pairs) {
  const long long m_tiles = (long long)((batch + 1) / 2) * ((Ho + 7) / 8) * ((Wo + 7) / 8);
  const long long n_tiles = (Cout + TB_GEMM_BN - 1) / TB_GEMM_BN;
  const long long tiles = m_tiles * n_tiles;
  if (pairs < 0) pairs = (m_tiles >= 2 && tiles >= s->sm_count) ? 1 : 0;
  CUtensorMap tx, tw;
  {
    cuuint64_t dims[4] = {(cuuint64_t)C, (cuuint64_t)W, (cuuint64_t)H, (cuuint64_t)batch};
    cuuint64_t strides[3] = {(cuuint64_t)C * 2, (cuuint64_t)W * C * 2, (cuuint64_t)H * W * C * 2};
    cuuint32_t box[4] = {64, (cuuint32_t)(8 * sw), (cuuint32_t)(8 * sh), 2};
    cuuint32_t elem[4] = {1, (cuuint32_t)sw, (cuuint32_t)sh, 1};
    TB_CU("cuTensorMapEncodeTiled",
          driver()->cuTensorMapEncodeTiled(&tx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, reinterpret_cast<void*>(x), dims,
                                           strides, box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                           CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE));
  }
  {
    cuuint64_t dims[3] = {(cuuint64_t)C, (cuuint64_t)R * S, (cuuint64_t)Cout};
    cuuint64_t strides[2] = {(cuuint64_t)C * 2, (cuuint64_t)R * S * C * 2};
    cuuint32_t box[3] = {64, 1, pairs ? 128u : (cuuint32_t)TB_GEMM_BN};
    cuuint32_t elem[3] = {1, 1, 1};
    TB_CU("cuTensorMapEncodeTiled",
          driver()->cuTensorMapEncodeTiled(&tw, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, reinterpret_cast<void*>(w), dims,
                                           strides, box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                           CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE));
  }
  CUfunction fn = nullptr;
  const char* name = pairs ? "conv2d_fprop_bf16_nhwc_2sm" : "conv2d_fprop_bf16_nhwc";
  tb_status rc = builtin_function(s, "conv2d_bf16", name, &fn);
  if (rc) return rc;
  CUdeviceptr status = s->status.device;
  void* params[] = {&tx, &tw, &y, &bias, &batch, &C, &Cout, &R, &S, &Ho, &Wo, &sh, &sw, &ph, &pw, &dh, &dw, &status};
  if (pairs)
    return launch_builtin_pairs(s, st, fn, (m_tiles + 1) / 2 * n_tiles, TB_GEMM_THREADS, TB_GEMM2_SMEM_BYTES, params,
                                name);
  const unsigned grid = (unsigned)(tiles < s->sm_count ? tiles : s->sm_count);
  return launch_builtin(s, st, fn, grid, 1, 1, TB_GEMM_THREADS, TB_GEMM_SMEM_BYTES, params, name);
}

}  // namespace tb

using namespace tb;

extern "C" tb_status tb_op_conv2d(tb_session* session, tb_stream* stream, const tb_tensor* input,
                                  const tb_tensor* weight, const tb_tensor* bias, const tb_tensor* output,
                                  const tb_attr* attrs, uint32_t num_attrs, tb_event** out) {
  Session* s = reinterpret_cast<Session*>(session);
  if (!s) return set_error(TB_ERR_INVALID, "contract", "null session");
  if (!input || !weight || !output)
    return contract("CUDA Conv2D requires input, weight, optional bias, and one output");
  static const char* kKnown[] = {"stride_h", "stride_w", "pad_h", "pad_w", "dilation_h", "dilation_w", "groups",
                                 "layout",   "candidate"};
  const char* layout = nullptr;
  const char* candidate = nullptr;  // optional registered kernel name (autotuner)
  for (uint32_t i = 0; i < num_attrs; ++i) {
    bool known = false;
    for (const char* k : kKnown) known = known || (attrs[i].key && strcmp(attrs[i].key, k) == 0);
    if (!known) return contract("CUDA Conv2D received unsupported attributes");
    if (strcmp(attrs[i].key, "layout") == 0) {
      if (!attrs[i].str) return contract("conv2d layout must be a string");
      layout = attrs[i].str;
    }
    if (strcmp(attrs[i].key, "candidate") == 0) {
      if (!attrs[i].str) return contract("conv2d candidate must be a string");
      candidate = attrs[i].str;
    }
  }
  if (candidate && strcmp(candidate, "conv2d_fprop_bf16_nhwc") != 0 &&
      strcmp(candidate, "conv2d_fprop_bf16_nhwc_2sm") != 0 && strcmp(candidate, "conv2d_bf16_nhwc_generic") != 0 &&
      strcmp(candidate, "conv2d_f32") != 0)
    return contract(std::string("unknown conv2d candidate ") + candidate);
  const bool nhwc = layout && strcmp(layout, "NHWC") == 0;
  if (layout && !nhwc && strcmp(layout, "NCHW") != 0) return contract("conv2d layout must be NCHW or NHWC");
  const uint32_t dt = input->dtype;
  const bool f32 = dt == TB_F32 && weight->dtype == TB_F32 && output->dtype == TB_F32 && (!bias || bias->dtype == TB_F32);
  const bool bf16 = dt == TB_BF16 && weight->dtype == TB_BF16 && output->dtype == TB_BF16 &&
                    (!bias || bias->dtype == TB_F32);
  if (!f32 && !bf16)
    return contract("CUDA Conv2D requires F32 input, weight, optional bias, and output (or BF16 with an F32 bias)");
  if (bf16 && !nhwc) return unsupported("CUDA Conv2D does not implement BF16 NCHW; pass layout=NHWC");
  if (f32 && nhwc) return unsupported("CUDA Conv2D does not implement F32 NHWC");
  if (input->rank != 4 || weight->rank != 4 || (bias && bias->rank != 1))
    return contract("conv2d requires rank-4 NCHW input, rank-4 OIHW weight, and optional bias");
  if (!is_contiguous(input) || !is_contiguous(weight) || (bias && !is_contiguous(bias)))
    return contract("CUDA Conv2D requires contiguous NCHW input, OIHW weight, and optional rank-1 bias");
  if (output->rank != 4 || !is_contiguous(output)) return contract("CUDA Conv2D requires a contiguous rank-4 output");
  // Conv2dF32Descriptor::validate (titan-backend-cuda/src/lib.rs:815-825): every input and weight extent first.
  for (int i = 0; i < 4; ++i)
    if (input->shape[i] == 0 || weight->shape[i] == 0) return contract("CUDA Conv2D dimensions must be non-zero");
  int64_t sh, sw, ph, pw, dh, dw, groups;
  tb_status rc;
  if ((rc = int_attr(attrs, num_attrs, "stride_h", nullptr, &sh)) ||
      (rc = int_attr(attrs, num_attrs, "stride_w", nullptr, &sw)) ||
      (rc = int_attr(attrs, num_attrs, "pad_h", nullptr, &ph)) || (rc = int_attr(attrs, num_attrs, "pad_w", nullptr, &pw)) ||
      (rc = int_attr(attrs, num_attrs, "dilation_h", nullptr, &dh)) ||
      (rc = int_attr(attrs, num_attrs, "dilation_w", nullptr, &dw)) ||
      (rc = int_attr(attrs, num_attrs, "groups", nullptr, &groups)))
    return rc;
  if (sh == 0 || sw == 0 || dh == 0 || dw == 0 || groups == 0)
    return contract("conv2d stride, dilation, and groups must be non-zero");
  // Logical dims: NCHW/OIHW for F32, NHWC/KRSC for BF16.
  const uint64_t batch = input->shape[0];
  const uint64_t cin = nhwc ? input->shape[3] : input->shape[1];
  const uint64_t h = nhwc ? input->shape[1] : input->shape[2];
  const uint64_t wd = nhwc ? input->shape[2] : input->shape[3];
  const uint64_t cout = weight->shape[0];
  const uint64_t wcin = nhwc ? weight->shape[3] : weight->shape[1];
  const uint64_t kh = nhwc ? weight->shape[1] : weight->shape[2];
  const uint64_t kw = nhwc ? weight->shape[2] : weight->shape[3];
  const uint64_t g = (uint64_t)groups;
  if (cin == 0 || h == 0 || wd == 0 || cout == 0 || kh == 0 || kw == 0 || cin % g != 0 || cout % g != 0 ||
      wcin != cin / g)
    return contract("conv2d channels, groups, and kernel dimensions are invalid");
  if (bias && bias->shape[0] != cout) return contract("conv2d bias must have shape [output_channels]");
  const uint64_t eff_h = (uint64_t)dh * (kh - 1) + 1, eff_w = (uint64_t)dw * (kw - 1) + 1;
  const uint64_t padded_h = h + 2 * (uint64_t)ph, padded_w = wd + 2 * (uint64_t)pw;
  if (eff_h > padded_h || eff_w > padded_w) return contract("conv2d kernel geometry exceeds padded input");
  const uint64_t ho = (padded_h - eff_h) / (uint64_t)sh + 1, wo = (padded_w - eff_w) / (uint64_t)sw + 1;
  const uint64_t o0 = output->shape[0], o1 = output->shape[1], o2 = output->shape[2], o3 = output->shape[3];
  const bool shape_ok = nhwc ? (o0 == batch && o1 == ho && o2 == wo && o3 == cout)
                             : (o0 == batch && o1 == cout && o2 == ho && o3 == wo);
  if (!shape_ok) return contract("conv2d output shape mismatch");
  if (batch * cin * h * wd > (1ull << 40) || batch > 0x7fffffffull)
    return contract("CUDA Conv2D shape exceeds the i32 ABI");
  Stream* st = nullptr;
  rc = check_stream(s, stream, &st);
  if (rc) return rc;
  Buffer *bx = nullptr, *bw = nullptr, *bb = nullptr, *by = nullptr;
  if ((rc = tensor_buffer(s, input, "conv2d input", &bx)) || (rc = tensor_buffer(s, weight, "conv2d weight", &bw)) ||
      (bias && (rc = tensor_buffer(s, bias, "conv2d bias", &bb))) ||
      (rc = tensor_buffer(s, output, "conv2d output", &by)))
    return rc;
  rc = activate(s);
  if (rc) return rc;
  CUdeviceptr px = bx->ptr, pw_ = bw->ptr, pb = bb ? bb->ptr : 0, py = by->ptr;
  int N = (int)batch, C = (int)cin, H = (int)h, Wd = (int)wd, K = (int)cout, R = (int)kh, S = (int)kw;
  int Ho = (int)ho, Wo = (int)wo, SH = (int)sh, SW = (int)sw, PH = (int)ph, PW = (int)pw, DH = (int)dh, DW = (int)dw;
  int G = (int)groups, has_bias = bias ? 1 : 0;
  uint64_t total = batch * ho * wo * cout;
  uint64_t grid = (total + 255) / 256;
  if (grid > (uint64_t)s->sm_count * 32) grid = (uint64_t)s->sm_count * 32;
  CUfunction fn = nullptr;
  if (candidate && (f32 != (strcmp(candidate, "conv2d_f32") == 0)))
    return unsupported(std::string("candidate ") + candidate + " does not take this dtype");
  if (f32) {
    rc = builtin_function(s, "compat", "conv2d_f32", &fn);
    if (rc) return rc;
    void* params[] = {&px, &pw_, &pb, &py, &N, &C, &H, &Wd, &K, &R, &S, &Ho, &Wo, &SH, &SW, &PH, &PW, &DH, &DW, &G,
                      &has_bias};
    rc = launch_builtin(s, st, fn, (unsigned)grid, 1, 1, 256, 0, params, "conv2d_f32");
  } else {
    // Strides reach the kernel as TMA traversal strides, which must be at most 8.
    const bool tc_ok = G == 1 && C % 8 == 0 && K % 8 == 0 && SH >= 1 && SH <= 8 && SW >= 1 && SW <= 8 &&
                       ((px | pw_ | py) & 15) == 0;
    const bool want_generic = candidate && strcmp(candidate, "conv2d_bf16_nhwc_generic") == 0;
    if (candidate && !want_generic && !tc_ok)
      return unsupported(std::string("candidate ") + candidate + " does not take this shape, stride or alignment");
    if (tc_ok && !want_generic) {
      const int pairs = !candidate ? -1 : strcmp(candidate, "conv2d_fprop_bf16_nhwc_2sm") == 0 ? 1 : 0;
      rc = launch_conv2d_bf16(s, st, px, pw_, pb, py, N, H, Wd, C, K, R, S, Ho, Wo, SH, SW, PH, PW, DH, DW, pairs);
    } else {
      rc = builtin_function(s, "compat", "conv2d_bf16_nhwc_generic", &fn);
      if (rc) return rc;
      void* params[] = {&px, &pw_, &pb, &py, &N, &H, &Wd, &C, &K, &R, &S, &Ho, &Wo, &SH, &SW, &PH, &PW, &DH, &DW, &G};
      rc = launch_builtin(s, st, fn, (unsigned)grid, 1, 1, 256, 0, params, "conv2d_bf16_nhwc_generic");
    }
  }
  if (rc) return rc;
  return record_event(s, st, nullptr, out);
}
