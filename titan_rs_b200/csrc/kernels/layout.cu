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

// Operand staging for GEMMs whose storage the TMA cannot describe (a contiguous extent
// that is not a multiple of 8 bf16, i.e. rows that do not start 16-byte aligned).
// dst is the K-major [rows, kp] copy of a [rows, k] operand, kp = k rounded up to 8,
// with columns k..kp-1 zero. Zero columns in both operands add exact zeros to every
// dot product, so the tensor-core GEMM over kp gives the product over k.
//
// Source contiguous along k (element (r, c) at src[r * s_r + c]): row-by-row copy,
// consecutive threads on consecutive columns of one row.
extern "C" __global__ void __launch_bounds__(256) stage_bf16_k_major_rows(const uint16_t* __restrict__ src,
                                                                         uint16_t* __restrict__ dst, int rows, int k,
                                                                         int kp, long long s_r) {
  for (int r = blockIdx.y; r < rows; r += gridDim.y) {
    const uint16_t* in = src + (long long)r * s_r;
    uint16_t* out = dst + (long long)r * kp;
    for (int c = blockIdx.x * 256 + threadIdx.x; c < kp; c += gridDim.x * 256) out[c] = c < k ? in[c] : 0;
  }
}

// Source contiguous along rows (element (r, c) at src[c * s_c + r]): 32 x 32 tiles
// transposed through shared memory, read along rows and written along columns. The
// tile loop depends only on blockIdx, so every thread reaches both barriers.
extern "C" __global__ void __launch_bounds__(256) stage_bf16_k_major_cols(const uint16_t* __restrict__ src,
                                                                         uint16_t* __restrict__ dst, int rows, int k,
                                                                         int kp, long long s_c) {
  __shared__ uint16_t tile[32][34];  // 17-word rows: column reads hit 32 distinct banks
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const long long tiles_c = (kp + 31) / 32, tiles = tiles_c * ((rows + 31) / 32);
  for (long long t = blockIdx.x; t < tiles; t += gridDim.x) {
    const int r0 = (int)(t / tiles_c) * 32, c0 = (int)(t % tiles_c) * 32;
    for (int i = ty; i < 32; i += 8) {
      const int c = c0 + i, r = r0 + tx;
      tile[i][tx] = (c < k && r < rows) ? src[(long long)c * s_c + r] : (uint16_t)0;
    }
    __syncthreads();
    for (int i = ty; i < 32; i += 8) {
      const int r = r0 + i, c = c0 + tx;
      if (r < rows && c < kp) dst[(long long)r * kp + c] = tile[tx][i];
    }
    __syncthreads();
  }
}
