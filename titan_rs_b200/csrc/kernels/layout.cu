// Re-layout after the N-sharded GEMM's all-gather: the gathered buffer holds
// rank r's output columns as a contiguous [M, Np] block at offset r*M*Np; the
// result is the row-major C[M, p*Np]. Pure HBM copy: 16-byte loads and stores,
// consecutive threads walk consecutive 8-element groups of one output row.
#include <cuda_bf16.h>
#include <stdint.h>

extern "C" __global__ void __launch_bounds__(256) gather_column_blocks_bf16(const __nv_bfloat16* __restrict__ src,
                                                                           __nv_bfloat16* __restrict__ dst, int M,
                                                                           int Np, int p) {
  const long long row_vecs = (long long)Np * p / 8;  // 8 bf16 per 16-byte vector
  const long long total = row_vecs * M;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long m = i / row_vecs;
    const long long col = (i - m * row_vecs) * 8;
    const long long r = col / Np, j = col - r * Np;
    const uint4 v = __ldcs(reinterpret_cast<const uint4*>(src + (r * M + m) * Np + j));
    __stcs(reinterpret_cast<uint4*>(dst + m * (long long)Np * p + col), v);
  }
}
