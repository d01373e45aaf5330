// CUDA Driver API resolved at run time from libcuda.so.1, as the titan.rs CUDA
// backend does (CudaDiscovery::open, titan-backend-cuda/src/lib.rs:190-230).
// Nothing links against libcuda, so the library loads on machines without a
// driver and reports "load_driver" from tb_driver_open instead.
#pragma once

#include <cuda.h>

namespace tb {

#define TB_CU_FUNCS(X)                 \
  X(cuInit)                            \
  X(cuDriverGetVersion)                \
  X(cuDeviceGetCount)                  \
  X(cuDeviceGet)                       \
  X(cuDeviceGetName)                   \
  X(cuDeviceGetAttribute)              \
  X(cuDeviceTotalMem_v2)               \
  X(cuDevicePrimaryCtxRetain)          \
  X(cuDevicePrimaryCtxRelease_v2)      \
  X(cuCtxSetCurrent)                   \
  X(cuCtxGetCurrent)                   \
  X(cuMemAlloc_v2)                     \
  X(cuMemFree_v2)                      \
  X(cuMemGetInfo_v2)                   \
  X(cuMemHostAlloc)                    \
  X(cuMemFreeHost)                     \
  X(cuMemHostGetDevicePointer_v2)      \
  X(cuMemcpyHtoDAsync_v2)              \
  X(cuMemcpyDtoHAsync_v2)              \
  X(cuMemcpyDtoDAsync_v2)              \
  X(cuMemsetD8Async)                   \
  X(cuMemsetD32Async)                  \
  X(cuStreamCreate)                    \
  X(cuStreamDestroy_v2)                \
  X(cuStreamSynchronize)               \
  X(cuStreamWaitEvent)                 \
  X(cuStreamBeginCapture_v2)           \
  X(cuStreamIsCapturing)               \
  X(cuStreamEndCapture)                \
  X(cuGraphInstantiateWithFlags)       \
  X(cuGraphLaunch)                     \
  X(cuGraphExecDestroy)                \
  X(cuGraphDestroy)                    \
  X(cuEventCreate)                     \
  X(cuEventDestroy_v2)                 \
  X(cuEventRecord)                     \
  X(cuEventQuery)                      \
  X(cuEventSynchronize)                \
  X(cuEventElapsedTime)                \
  X(cuModuleLoadData)                  \
  X(cuModuleUnload)                    \
  X(cuModuleGetFunction)               \
  X(cuFuncSetAttribute)                \
  X(cuFuncGetAttribute)                \
  X(cuLaunchKernel)                    \
  X(cuLaunchKernelEx)                  \
  X(cuOccupancyMaxActiveClusters)      \
  X(cuTensorMapEncodeTiled)            \
  X(cuGetErrorString)                  \
  X(cuGetErrorName)                    \
  X(cuPointerGetAttribute)             \
  X(cuMemGetAddressRange_v2)           \
  X(cuIpcGetMemHandle)                 \
  X(cuIpcOpenMemHandle_v2)             \
  X(cuIpcCloseMemHandle)

struct DriverApi {
#define TB_DECLARE(name) decltype(&::name) name = nullptr;
  TB_CU_FUNCS(TB_DECLARE)
#undef TB_DECLARE
  void* handle = nullptr;
};

// Opens libcuda once (thread-safe). Returns nullptr and sets the thread's last
// error ("load_driver" or "cuInit") when no usable driver exists.
const DriverApi* driver();

}  // namespace tb
