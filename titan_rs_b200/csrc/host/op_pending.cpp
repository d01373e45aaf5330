// Entry points whose kernels are not built yet report "does not implement".
#include "ops_common.hpp"

using namespace tb;

extern "C" {

tb_status tb_comm_unique_id(uint8_t*) { return unsupported("collective not built"); }
tb_status tb_comm_init(tb_session*, const uint8_t*, int, int, uint32_t, tb_comm**) {
  return unsupported("collective not built");
}
void tb_comm_release(tb_comm*) {}
int tb_comm_rank(const tb_comm*) { return -1; }
int tb_comm_size(const tb_comm*) { return 0; }
tb_status tb_comm_all_gather(tb_comm*, tb_stream*, tb_buffer*, tb_buffer*, size_t, tb_event**) {
  return unsupported("collective not built");
}
tb_status tb_comm_barrier(tb_comm*, tb_stream*) { return unsupported("collective not built"); }
tb_status tb_op_gemm_sharded(tb_comm*, tb_stream*, const tb_tensor*, const tb_tensor*, const tb_tensor*, tb_buffer*,
                             tb_event**) {
  return unsupported("collective not built");
}

}  // extern "C"
