// bf16 GEMM with fp32 accumulation on the 5th-generation tensor cores.
//
//   C[M,N] (bf16, row-major, leading dimension ldc) = A[M,K] (bf16, row-major) x B^T
//   where B is stored as [N,K] row-major, i.e. the column-major B of the
//   titan.rs GEMM with transpose_rhs (projects/titan-runtime/src/lib.rs:955-989).
//
// The pipeline (umma_pipeline.cuh) is one persistent CTA per SM: TMA producer
// warp, MMA warp with two 128x256 fp32 TMEM accumulators, four epilogue warps.
// This policy maps tiles and k-blocks to TMA coordinates: A tile [128 x 64] at
// (k, m), B tile [256 x 64] at (k, n), 128-byte swizzle; tiles are visited in
// groups of 16 M-blocks so the tiles in flight share A rows and B columns in L2.
// K tails and M/N tails come back from TMA as zeros; the epilogue masks them.
#include "umma_pipeline.cuh"

namespace {

using namespace tb;

constexpr uint32_t kFailGemm = 0x47000000u;

struct GemmPolicy {
  const CUtensorMap* ta;
  const CUtensorMap* tb;
  __nv_bfloat16* c;
  int M, N, K;
  long long ldc;
  bool vec_ok;
  int num_m, num_n;

  __device__ int num_tiles() const { return num_m * num_n; }
  __device__ int num_k_blocks() const { return (K + umma::BK - 1) / umma::BK; }
  __device__ void prefetch() const {
    tma_prefetch_desc(ta);
    tma_prefetch_desc(tb);
  }
  __device__ void tile(int t, int& m_blk, int& n_blk) const { umma::grouped_tile(t, num_m, num_n, 16, m_blk, n_blk); }
  __device__ void load(uint8_t* a_dst, uint8_t* b_dst, uint64_t* bar, int m_blk, int n_blk, int kb) const {
    tma_load_2d(a_dst, ta, bar, kb * umma::BK, m_blk * umma::BM);
    tma_load_2d(b_dst, tb, bar, kb * umma::BK, n_blk * umma::BN);
  }
  __device__ void store(int row, int m_blk, int n_blk, int col, const uint32_t (&r)[32]) const {
    const int gr = m_blk * umma::BM + row;
    const int gc = n_blk * umma::BN + col;
    if (gr >= M || gc >= N) return;
    umma::store_bf16_chunk(c + (long long)gr * ldc + gc, N - gc, vec_ok, r, nullptr);
  }
};

}  // namespace

extern "C" __global__ void __launch_bounds__(TB_GEMM_THREADS, 1)
    gemm_bf16_tn(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                 __nv_bfloat16* __restrict__ c, int M, int N, int K, long long ldc, uint32_t* status) {
  GemmPolicy p;
  p.ta = &tmap_a;
  p.tb = &tmap_b;
  p.c = c;
  p.M = M;
  p.N = N;
  p.K = K;
  p.ldc = ldc;
  p.vec_ok = (ldc % 8) == 0 && (reinterpret_cast<uintptr_t>(c) & 15) == 0;
  p.num_m = (M + umma::BM - 1) / umma::BM;
  p.num_n = (N + umma::BN - 1) / umma::BN;
  umma::run(p, status, kFailGemm);
}
