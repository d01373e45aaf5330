// Problem policies for the tcgen05 GEMM pipeline (umma_pipeline.cuh) and the
// split-K reduction, shared by every translation unit that instantiates them.
//
//   GemmPolicy     C[M,N] bf16 = A[M,K] x B^T, B stored [N,K] (column-major B).
//   SplitKPolicy   fp32 partial tiles of the same product; work unit
//                  t = split * (num_m * num_n) + output tile, each split covering
//                  kb_per_split k-blocks of 64 (the last one possibly fewer, none empty),
//                  written to `partial` laid out [splits][M][N].
//   splitk_reduce  C[m, n] = bf16( sum_{s < splits} partial[s][m][n] ), summed in
//                  split order, so the result is deterministic.
#pragma once

#include "umma_pipeline.cuh"

namespace tb {
namespace gemm {

struct GemmPolicy {
  const CUtensorMap* ta;
  const CUtensorMap* tb;
  __nv_bfloat16* c;
  int M, N, K;
  long long ldc;
  bool vec_ok;
  int num_m, num_n;

  __device__ int num_tiles() const { return num_m * num_n; }
  __device__ void k_blocks(int, int& kb0, int& kb1) const {
    kb0 = 0;
    kb1 = (K + umma::BK - 1) / umma::BK;
  }
  __device__ void prefetch() const {
    tma_prefetch_desc(ta);
    tma_prefetch_desc(tb);
  }
  __device__ void tile(int t, int& m_blk, int& n_blk) const { umma::grouped_tile(t, num_m, num_n, 16, m_blk, n_blk); }
  __device__ void load(uint8_t* a_dst, uint8_t* b_dst, uint64_t* bar, int m_blk, int n_blk, int kb) const {
    tma_load_2d(a_dst, ta, bar, kb * umma::BK, m_blk * umma::BM);
    tma_load_2d(b_dst, tb, bar, kb * umma::BK, n_blk * umma::BN);
  }
  __device__ void store(int row, int, int m_blk, int n_blk, int col, const uint32_t (&r)[32]) const {
    const int gr = m_blk * umma::BM + row;
    const int gc = n_blk * umma::BN + col;
    if (gr >= M || gc >= N) return;
    umma::store_bf16_chunk(c + (long long)gr * ldc + gc, N - gc, vec_ok, r, nullptr);
  }
};

struct SplitKPolicy {
  const CUtensorMap* ta;
  const CUtensorMap* tb;
  float* partial;  // [splits][M][N] fp32
  int M, N, K;
  int num_m, num_n, splits, kb_per_split;
  bool vec_ok;

  __device__ int num_tiles() const { return num_m * num_n * splits; }
  __device__ void k_blocks(int t, int& kb0, int& kb1) const {
    const int s = t / (num_m * num_n);
    const int num_k = (K + umma::BK - 1) / umma::BK;
    kb0 = s * kb_per_split;
    kb1 = min(kb0 + kb_per_split, num_k);
  }
  __device__ void prefetch() const {
    tma_prefetch_desc(ta);
    tma_prefetch_desc(tb);
  }
  __device__ void tile(int t, int& m_blk, int& n_blk) const {
    umma::grouped_tile(t % (num_m * num_n), num_m, num_n, 16, m_blk, n_blk);
  }
  __device__ void load(uint8_t* a_dst, uint8_t* b_dst, uint64_t* bar, int m_blk, int n_blk, int kb) const {
    tma_load_2d(a_dst, ta, bar, kb * umma::BK, m_blk * umma::BM);
    tma_load_2d(b_dst, tb, bar, kb * umma::BK, n_blk * umma::BN);
  }
  __device__ void store(int row, int t, int m_blk, int n_blk, int col, const uint32_t (&r)[32]) const {
    const int s = t / (num_m * num_n);
    const int gr = m_blk * umma::BM + row;
    const int gc = n_blk * umma::BN + col;
    if (gr >= M || gc >= N) return;
    float* dst = partial + ((long long)s * M + gr) * N + gc;
    if (vec_ok && gc + 32 <= N) {
#pragma unroll
      for (int q = 0; q < 8; ++q)
        reinterpret_cast<float4*>(dst)[q] = make_float4(__uint_as_float(r[4 * q]), __uint_as_float(r[4 * q + 1]),
                                                        __uint_as_float(r[4 * q + 2]), __uint_as_float(r[4 * q + 3]));
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (gc + j < N) dst[j] = __uint_as_float(r[j]);
    }
  }
};

__device__ __forceinline__ void run_splitk(const CUtensorMap* ta, const CUtensorMap* tb, float* partial, int M, int N,
                                           int K, int splits, int kb_per_split, uint32_t* status, uint32_t fail) {
  SplitKPolicy p;
  p.ta = ta;
  p.tb = tb;
  p.partial = partial;
  p.M = M;
  p.N = N;
  p.K = K;
  p.num_m = (M + umma::BM - 1) / umma::BM;
  p.num_n = (N + umma::BN - 1) / umma::BN;
  p.splits = splits;
  p.kb_per_split = kb_per_split;
  p.vec_ok = (N % 4) == 0 && (reinterpret_cast<uintptr_t>(partial) & 15) == 0;
  umma::run(p, status, fail);
}

// Four columns per thread (16-byte loads) when N % 4 == 0.
__device__ __forceinline__ void splitk_reduce(const float* __restrict__ partial, __nv_bfloat16* __restrict__ c, int M,
                                              int N, int splits, long long ldc) {
  const long long plane = (long long)M * N;
  if ((N & 3) == 0) {
    const long long total = plane / 4;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
      float4 acc = __ldcs(reinterpret_cast<const float4*>(partial) + i);
      for (int s = 1; s < splits; ++s) {
        const float4 v = __ldcs(reinterpret_cast<const float4*>(partial + s * plane) + i);
        acc.x += v.x;
        acc.y += v.y;
        acc.z += v.z;
        acc.w += v.w;
      }
      const long long e = i * 4;
      const long long m = e / N, n = e % N;
      uint2 packed = make_uint2(pack_bf16x2(acc.x, acc.y), pack_bf16x2(acc.z, acc.w));
      if ((ldc & 3) == 0) {
        *reinterpret_cast<uint2*>(c + m * ldc + n) = packed;
      } else {
        __nv_bfloat162* d = reinterpret_cast<__nv_bfloat162*>(&packed);
        c[m * ldc + n] = d[0].x;
        c[m * ldc + n + 1] = d[0].y;
        c[m * ldc + n + 2] = d[1].x;
        c[m * ldc + n + 3] = d[1].y;
      }
    }
  } else {
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < plane;
         i += (long long)gridDim.x * blockDim.x) {
      float acc = partial[i];
      for (int s = 1; s < splits; ++s) acc += partial[s * plane + i];
      c[(i / N) * ldc + (i % N)] = __float2bfloat16_rn(acc);
    }
  }
}

}  // namespace gemm
}  // namespace tb
