// Runtime::execute by operator name (projects/titan-runtime/src/lib.rs:1171-1256).
//
// The reference routes an OpRequest on `operator.0` and the first input's backend to
// execute_cuda_{gemm,conv2d,attention,softmax}; a name it has no route for fails in
// the contract phase. Here the request arrives as tensors and attributes, each name is
// checked for its input count, and the per-operator entries do the rest.
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
};

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
    default:
      return tb_op_gemm_bias_act(session, stream, &inputs[0], &inputs[1], third, output, attrs, num_attrs, out);
  }
}
