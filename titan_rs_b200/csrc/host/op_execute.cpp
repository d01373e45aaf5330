// Runtime::execute by operator name (projects/titan-runtime/src/lib.rs:1171-1256).
//
// The reference routes an OpRequest on `operator.0` and the first input's backend to
// execute_cuda_{gemm,conv2d,attention,softmax}; a name it has no route for fails in
// the contract phase. Here the request arrives as tensors and attributes, each name is
// checked for its input count, and the per-operator entries do the rest. The route list
// adds the graph compiler's fused nodes ("gemm.bias_act", "attention.fused"), so every
// node of a compiled plan runs through this one entry.
#include <cstring>

#include "ops_common.hpp"

namespace {

struct Route {
  const char* name;
  uint32_t min_inputs, max_inputs;
  const char* arity;  // the runtime's message for a wrong input count
};

const Route kRoutes[] = {
    {"softmax", 1, 1, "CUDA softmax requires exactly one input and one output"},
    {"gemm", 2, 2, "gemm requires exactly two rank-2 inputs"},
    {"scaled_dot_product_attention", 3, 3, "scaled dot-product attention requires exactly three rank-4 BHTD inputs"},
    {"conv2d", 2, 3, "conv2d requires rank-4 NCHW input, rank-4 OIHW weight, and optional bias"},
    {"gemm.bias_act", 2, 3, "gemm.bias_act requires two rank-2 inputs, an optional bias and one output"},
    {"attention.fused", 3, 3, "attention.fused requires Q, K and V"},
};

// A contiguous rank-2 [T, D] tensor as the [1, 1, T, D] view of the same buffer.
bool as_bhtd(const tb_tensor& t, tb_tensor& view) {
  if (t.rank != 2 || t.strides[1] != 1 || t.strides[0] != (int64_t)t.shape[1]) return false;
  const uint64_t rows = t.shape[0], cols = t.shape[1];
  view = t;
  view.rank = 4;
  view.shape[0] = view.shape[1] = 1;
  view.shape[2] = rows;
  view.shape[3] = cols;
  view.strides[0] = view.strides[1] = (int64_t)(rows * cols);
  view.strides[2] = (int64_t)cols;
  view.strides[3] = 1;
  return true;
}

}  // namespace

extern "C" tb_status tb_execute(tb_session* session, tb_stream* stream, const char* op, const tb_tensor* inputs,
                                uint32_t num_inputs, const tb_tensor* output, const tb_attr* attrs,
                                uint32_t num_attrs, tb_event** out) {
  using tb::contract;
  if (!op) return contract("operator name is null");
  const Route* route = nullptr;
  for (const Route& r : kRoutes)
    if (strcmp(op, r.name) == 0) route = &r;
  if (!route)
    return tb::unsupported(std::string("operator ") + op + " is not on the B200 hot path (does not implement)");
  if (num_inputs < route->min_inputs || num_inputs > route->max_inputs || !inputs || !output)
    return contract(route->arity);
  const tb_tensor* third = num_inputs > 2 ? &inputs[2] : nullptr;
  switch (route - kRoutes) {
    case 0: return tb_op_softmax(session, stream, &inputs[0], output, attrs, num_attrs, out);
    case 1: return tb_op_gemm(session, stream, &inputs[0], &inputs[1], output, attrs, num_attrs, out);
    case 2: return tb_op_sdpa(session, stream, &inputs[0], &inputs[1], &inputs[2], output, attrs, num_attrs, out);
    case 3: return tb_op_conv2d(session, stream, &inputs[0], &inputs[1], third, output, attrs, num_attrs, out);
    case 4:
      return tb_op_gemm_bias_act(session, stream, &inputs[0], &inputs[1], third, output, attrs, num_attrs, out);
    default: {
      // The graph compiler's gemm -> softmax -> gemm node: the flash-attention operator on
      // [1, 1, T, D] views (its `scale` attribute is the chain's, 1.0).
      tb_tensor q, k, v, o;
      if (!as_bhtd(inputs[0], q) || !as_bhtd(inputs[1], k) || !as_bhtd(inputs[2], v) || !as_bhtd(*output, o))
        return contract("attention.fused requires contiguous rank-2 [T, D] Q, K, V and output");
      return tb_op_sdpa(session, stream, &q, &k, &v, &o, attrs, num_attrs, out);
    }
  }
}
