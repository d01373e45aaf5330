// Split-K bf16 GEMM that allocates no memory.
//
// tb_op_gemm's split-K path keeps its fp32 partial tiles in scratch memory the
// library allocates on the caller's stream. Some callers of this code cannot let
// a library allocate device memory: a serving runtime that has planned every byte of
// HBM up front and forbids ad-hoc allocations on the request path, or code that
// runs where the allocator must not be entered. This entry point gives them the
// same kernels with the scratch in a fixed, file-scope device array instead.
//
// The scratch array (TB_NOALLOC_SCRATCH_FLOATS fp32 values, 32 MiB) exists on every
// GPU that loads this library's module and stays allocated until the process exits.
// In host code its name is only a host-side stand-in, so its device address is
// fetched with cudaGetSymbolAddress once per device (on the first call on that
// device, with that device current) and passed to the kernels. That first call
// therefore does set-up work and should come before any stream capture.
//
// Every call shares the one array and leaves its partials behind: calls that can
// overlap on the GPU (different streams, or different host threads on one
// device) race on it and must be serialised by the caller. Nothing in the array
// needs clearing: every partial the reduction reads is written earlier in the
// same call.
//
// The kernels run asynchronously, so the call itself cannot report a device-side
// failure. Each bounded wait inside the split-K kernel that runs out writes a code
// into a per-device status word (zero when the module loads) and the kernel then
// returns early, which leaves C wrong. The word is sticky: later calls do not clear
// it. tb_gemm_bf16_splitk_noalloc_status synchronises a stream, reads the word and
// clears it, and returns TB_ERR_TIMEOUT with the code when any call on the device
// since the previous query timed out. It allocates nothing either.
#include <cuda_runtime.h>

#include <cstdio>
#include <mutex>

#include "../../../include/titan_b200.h"
#include "../host/internal.hpp"
#include "../kernels/gemm_policies.cuh"

namespace {

constexpr size_t kScratchFloats = (size_t)8 << 20;  // 32 MiB of fp32 partials
constexpr int kMaxDevices = 64;
constexpr uint32_t kFailNoAlloc = 0x4E000000u;

static __device__ __align__(256) float g_partial[kScratchFloats];
static __device__ __align__(256) uint32_t g_status[64];

__global__ void __launch_bounds__(TB_GEMM_THREADS, 1)
    gemm_bf16_tn_splitk_noalloc(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                                float* __restrict__ partial, int M, int N, int K, int splits, int kb_per_split,
                                uint32_t* status) {
  tb::gemm::run_splitk(&tmap_a, &tmap_b, partial, M, N, K, splits, kb_per_split, status, kFailNoAlloc);
}

__global__ void __launch_bounds__(256) splitk_reduce_bf16_noalloc(const float* __restrict__ partial,
                                                                 __nv_bfloat16* __restrict__ c, int M, int N,
                                                                 int splits, long long ldc) {
  tb::gemm::splitk_reduce(partial, c, M, N, splits, ldc);
}

struct DeviceSetup {
  std::once_flag once;
  cudaError_t error = cudaSuccess;
  const char* step = "";
  float* partial = nullptr;
  uint32_t* status = nullptr;
  int sm_count = 0;
};
DeviceSetup g_setup[kMaxDevices];

// Once per device, with that device current: device addresses of the static
// arrays, the kernel's shared-memory opt-in and the SM count.
void setup_device(int dev) {
  DeviceSetup& d = g_setup[dev];
  if ((d.error = cudaGetSymbolAddress(reinterpret_cast<void**>(&d.partial), g_partial)) != cudaSuccess) {
    d.step = "cudaGetSymbolAddress(scratch)";
    return;
  }
  if ((d.error = cudaGetSymbolAddress(reinterpret_cast<void**>(&d.status), g_status)) != cudaSuccess) {
    d.step = "cudaGetSymbolAddress(status)";
    return;
  }
  if ((d.error = cudaFuncSetAttribute(gemm_bf16_tn_splitk_noalloc, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      TB_GEMM_SMEM_BYTES)) != cudaSuccess) {
    d.step = "cudaFuncSetAttribute";
    return;
  }
  if ((d.error = cudaDeviceGetAttribute(&d.sm_count, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess)
    d.step = "cudaDeviceGetAttribute";
}

tb_status rt_error(const char* step, cudaError_t e) {
  return tb::set_error(TB_ERR_CUDA, "launch", std::string(step) + ": " + cudaGetErrorString(e));
}

tb_status encode(CUtensorMap* map, const void* base, uint64_t rows, uint64_t k, uint32_t box_rows) {
  const tb::DriverApi* d = tb::driver();
  if (!d) return TB_ERR_DRIVER_UNAVAILABLE;
  cuuint64_t dims[2] = {k, rows};
  cuuint64_t strides[1] = {k * 2};
  cuuint32_t box[2] = {TB_GEMM_BK, box_rows};
  cuuint32_t elem[2] = {1, 1};
  CUresult r = d->cuTensorMapEncodeTiled(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims,
                                         strides, box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? TB_OK : tb::cu_error("cuTensorMapEncodeTiled", r);
}

}  // namespace

extern "C" tb_status tb_gemm_bf16_splitk_noalloc(uint64_t stream, const void* a, const void* b, void* c, int m, int n,
                                                 int k, int splits) {
  using tb::set_error;
  if (!a || !b || !c) return set_error(TB_ERR_INVALID, "contract", "null A, B or C");
  if (((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b) | reinterpret_cast<uintptr_t>(c)) & 15) != 0)
    return set_error(TB_ERR_INVALID, "contract", "A, B and C must be 16-byte aligned");
  if (m <= 0 || n <= 0 || k <= 0) return set_error(TB_ERR_INVALID, "contract", "M, N and K must be positive");
  if (k % 8 != 0) return set_error(TB_ERR_INVALID, "contract", "K must be a multiple of 8");
  if (splits < 0) return set_error(TB_ERR_INVALID, "contract", "splits must be >= 0 (0 chooses)");
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return rt_error("cudaGetDevice", e);
  if (dev < 0 || dev >= kMaxDevices) return set_error(TB_ERR_INVALID, "contract", "device ordinal out of range");
  DeviceSetup& d = g_setup[dev];
  std::call_once(d.once, setup_device, dev);
  if (d.error != cudaSuccess) return rt_error(d.step, d.error);

  // The split plan tb_op_gemm uses: enough slices to occupy the SMs, at most 32.
  const int tiles = ((m + TB_GEMM_BM - 1) / TB_GEMM_BM) * ((n + TB_GEMM_BN - 1) / TB_GEMM_BN);
  const int num_k = (k + TB_GEMM_BK - 1) / TB_GEMM_BK;
  int want = splits;
  if (want == 0) want = d.sm_count / tiles < 2 ? 2 : d.sm_count / tiles;
  if (want > 32) want = 32;
  if (want > num_k) want = num_k;
  if (want < 1) want = 1;
  const int kb_per_split = (num_k + want - 1) / want;
  const int used = (num_k + kb_per_split - 1) / kb_per_split;  // every slice gets >= 1 k-block
  const unsigned long long need = (unsigned long long)used * (unsigned long long)m * (unsigned long long)n;
  if (need > kScratchFloats)
    return set_error(TB_ERR_INVALID, "contract",
                     "splits*M*N = " + std::to_string(need) + " fp32 partials exceed the static scratch of " +
                         std::to_string(kScratchFloats) + " (32 MiB); use tb_op_gemm, or fewer splits");

  CUtensorMap ta, tbm;
  tb_status rc = encode(&ta, a, (uint64_t)m, (uint64_t)k, TB_GEMM_BM);
  if (rc) return rc;
  rc = encode(&tbm, b, (uint64_t)n, (uint64_t)k, TB_GEMM_BN);
  if (rc) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(static_cast<uintptr_t>(stream));
  const long long units = (long long)tiles * used;
  const unsigned grid = (unsigned)(units < d.sm_count ? units : d.sm_count);
  gemm_bf16_tn_splitk_noalloc<<<grid, TB_GEMM_THREADS, TB_GEMM_SMEM_BYTES, st>>>(ta, tbm, d.partial, m, n, k, used,
                                                                                   kb_per_split, d.status);
  if ((e = cudaGetLastError()) != cudaSuccess) return rt_error("gemm_bf16_tn_splitk_noalloc", e);
  const unsigned long long vecs = ((unsigned long long)m * n + 3) / 4;
  unsigned long long rgrid = (vecs + 255) / 256;
  if (rgrid > (unsigned long long)d.sm_count * 16) rgrid = (unsigned long long)d.sm_count * 16;
  splitk_reduce_bf16_noalloc<<<(unsigned)rgrid, 256, 0, st>>>(d.partial, static_cast<__nv_bfloat16*>(c), m, n, used,
                                                             (long long)n);
  if ((e = cudaGetLastError()) != cudaSuccess) return rt_error("splitk_reduce_bf16_noalloc", e);
  tb::note_launch("gemm_bf16_tn_splitk_noalloc");
  return TB_OK;
}

extern "C" tb_status tb_gemm_bf16_splitk_noalloc_status(uint64_t stream, uint32_t* code) {
  if (code) *code = 0;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return rt_error("cudaGetDevice", e);
  if (dev < 0 || dev >= kMaxDevices) return tb::set_error(TB_ERR_INVALID, "contract", "device ordinal out of range");
  DeviceSetup& d = g_setup[dev];
  std::call_once(d.once, setup_device, dev);
  if (d.error != cudaSuccess) return rt_error(d.step, d.error);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(static_cast<uintptr_t>(stream));
  // Stream order: the copy sees every earlier call on this stream; the clear follows it.
  uint32_t word = 0;
  if ((e = cudaMemcpyAsync(&word, d.status, sizeof(word), cudaMemcpyDeviceToHost, st)) != cudaSuccess)
    return rt_error("cudaMemcpyAsync(status)", e);
  if ((e = cudaMemsetAsync(d.status, 0, sizeof(uint32_t), st)) != cudaSuccess)
    return rt_error("cudaMemsetAsync(status)", e);
  if ((e = cudaStreamSynchronize(st)) != cudaSuccess) return rt_error("cudaStreamSynchronize", e);
  if (code) *code = word;
  if (word != 0) {
    char buf[160];
    snprintf(buf, sizeof buf,
             "a split-K no-alloc kernel gave up a bounded device-side wait (code 0x%08x); its output is invalid",
             word);
    return tb::set_error(TB_ERR_TIMEOUT, "wait", buf);
  }
  return TB_OK;
}
