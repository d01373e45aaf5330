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

// Operand staging for GEMMs whose storage the TMA cannot describe: an operand whose
// contiguous extent is not a multiple of 8 bf16 (its rows do not start 16-byte
// aligned) or whose base is not 16-byte aligned. The copy keeps the storage order and
// only pads each row: dst[r * ld_dst + c] = src[r * ld_src + c] for c < cols and 0 for
// cols <= c < ld_dst, with ld_dst % 8 == 0 and dst 16-byte aligned. The GEMM then reads
// the copy with its row pitch, the logical extent unchanged; zero columns of a K-major
// operand add exact zeros to every dot product, and columns past N or M of an MN-major
// operand are never stored.
//
// One thread per 16-byte destination chunk (8 columns). Its 8 source elements lie in
// at most two aligned 16-byte source chunks, which it reads whole (a chunk holding any
// byte of the row lies inside the row's allocation) and shifts into place; consecutive
// threads read consecutive chunks, so the loads are coalesced and the second read of
// each chunk hits L1.
extern "C" __global__ void __launch_bounds__(256) stage_bf16_pad_rows(const uint16_t* __restrict__ src,
                                                                     uint16_t* __restrict__ dst, int rows, int cols,
                                                                     long long ld_src, int ld_dst) {
  const int chunks = ld_dst / 8;
  const long long total = (long long)rows * chunks;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / chunks;
    const int c0 = (int)(i - r * chunks) * 8;
    uint4 out = make_uint4(0u, 0u, 0u, 0u);
    if (c0 < cols) {
      const uint16_t* row = src + r * ld_src;
      const uintptr_t a = reinterpret_cast<uintptr_t>(row + c0);
      const uintptr_t base = a & ~static_cast<uintptr_t>(15);
      const int mis = static_cast<int>(a - base);  // even, 0..14
      const uint4 lo = __ldg(reinterpret_cast<const uint4*>(base));
      uint4 hi = make_uint4(0u, 0u, 0u, 0u);
      if (mis != 0 && base + 16 < reinterpret_cast<uintptr_t>(row + cols))
        hi = __ldg(reinterpret_cast<const uint4*>(base) + 1);
      const uint32_t w[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
      const int q = mis >> 2;          // whole words to skip
      const bool half = (mis & 2) != 0;  // and one more bf16
      uint32_t o[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint32_t x0 = q == 0 ? w[j] : q == 1 ? w[j + 1] : q == 2 ? w[j + 2] : w[j + 3];
        const uint32_t x1 = q == 0 ? w[j + 1] : q == 1 ? w[j + 2] : q == 2 ? w[j + 3] : w[j + 4];
        o[j] = half ? __funnelshift_r(x0, x1, 16) : x0;
      }
      const int valid = cols - c0;  // elements of this chunk inside the row
      if (valid < 8) {
#pragma unroll
        for (int e = 0; e < 8; ++e)
          if (e >= valid) o[e >> 1] &= (e & 1) ? 0x0000FFFFu : 0xFFFF0000u;
      }
      out = make_uint4(o[0], o[1], o[2], o[3]);
    }
    *reinterpret_cast<uint4*>(dst + r * ld_dst + c0) = out;
  }
}

// The inverse copy for a GEMM output whose rows do not start 16-byte aligned (N not a
// multiple of 8, or a misaligned base): the tensor-core kernel writes C into an aligned
// [rows, ld_src] scratch (ld_src % 8 == 0) with vector stores, and this copy moves it to
// dst[r * ld_dst + c], c < cols. One thread per 16-byte-aligned block of a destination
// row: a block wholly inside the row is one 16-byte store of 8 source elements shifted
// out of the (at most two) aligned source chunks that hold them; the partial blocks at
// the row's two ends are written element by element.
extern "C" __global__ void __launch_bounds__(256) unstage_bf16_rows(const uint16_t* __restrict__ src,
                                                                   uint16_t* __restrict__ dst, int rows, int cols,
                                                                   int ld_src, long long ld_dst) {
  const int blocks = cols / 8 + 2;  // an upper bound of the aligned 16-byte blocks a row touches
  const long long total = (long long)rows * blocks;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / blocks;
    const int b = (int)(i - r * blocks);
    uint16_t* drow = dst + r * ld_dst;
    const uint16_t* srow = src + r * (long long)ld_src;
    const uintptr_t d0 = reinterpret_cast<uintptr_t>(drow);
    const uintptr_t blk = (d0 & ~static_cast<uintptr_t>(15)) + 16 * static_cast<uintptr_t>(b);
    const long long e0 = (static_cast<long long>(blk) - static_cast<long long>(d0)) / 2;  // may be < 0 for b = 0
    if (e0 >= cols) continue;
    if (e0 >= 0 && e0 + 8 <= cols) {
      const int mis = static_cast<int>((e0 * 2) & 15);
      const uint4* p = reinterpret_cast<const uint4*>(srow) + ((e0 * 2) >> 4);
      const uint4 lo = __ldg(p);
      const uint4 hi = mis ? __ldg(p + 1) : make_uint4(0u, 0u, 0u, 0u);  // inside the row's ld_src >= cols
      const uint32_t w[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
      const int q = mis >> 2;
      const bool half = (mis & 2) != 0;
      uint32_t o[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint32_t x0 = q == 0 ? w[j] : q == 1 ? w[j + 1] : q == 2 ? w[j + 2] : w[j + 3];
        const uint32_t x1 = q == 0 ? w[j + 1] : q == 1 ? w[j + 2] : q == 2 ? w[j + 3] : w[j + 4];
        o[j] = half ? __funnelshift_r(x0, x1, 16) : x0;
      }
      *reinterpret_cast<uint4*>(blk) = make_uint4(o[0], o[1], o[2], o[3]);
    } else {
      const long long lo_e = e0 < 0 ? 0 : e0, hi_e = e0 + 8 < cols ? e0 + 8 : cols;
      for (long long e = lo_e; e < hi_e; ++e) drow[e] = srow[e];
    }
  }
}
