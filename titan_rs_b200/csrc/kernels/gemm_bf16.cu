// bf16 GEMM with fp32 accumulation on the 5th-generation tensor cores.
//
//   C[M,N] (bf16, row-major, leading dimension ldc) = A[M,K] (bf16, row-major) x B^T
//   where B is stored as [N,K] row-major, i.e. the column-major B of the
//   titan.rs GEMM with transpose_rhs (projects/titan-runtime/src/lib.rs:955-989).
//
// Design (one persistent CTA per SM, 192 threads, warp-specialised):
//   warp 0      TMA producer: A tile [128 x 64] and B tile [256 x 64] per stage,
//               128-byte swizzle, 4-stage shared-memory ring (48 KB per stage).
//   warp 1      allocates 512 TMEM columns (two 128x256 fp32 accumulators) and
//               one lane issues tcgen05.mma (M=128, N=256, K=16, kind::f16);
//               tcgen05.commit releases smem stages and publishes accumulators.
//   warps 2..5  epilogue: tcgen05.ld 32 columns at a time from the accumulator,
//               convert to bf16, 128-bit stores to C; then release the
//               accumulator so the MMA warp can start tile i+2 in it while
//               tile i+1 is already accumulating in the other one.
// Tiles are visited in groups of 16 M-blocks so the 148 tiles in flight share
// A rows and B columns in L2.
//
// Every wait is bounded (sm100.cuh); on a timeout the kernel records a code in
// `status`, drains its in-flight copies and MMAs, frees TMEM and exits.
#include "kernel_configs.h"
#include "sm100.cuh"

namespace {

using namespace tb;

constexpr int BM = TB_GEMM_BM, BN = TB_GEMM_BN, BK = TB_GEMM_BK, STAGES = TB_GEMM_STAGES;
constexpr int A_BYTES = BM * BK * 2;  // 16 KB
constexpr int B_BYTES = BN * BK * 2;  // 32 KB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int THREADS = TB_GEMM_THREADS;
constexpr int TMEM_COLS = 2 * BN;
constexpr int GROUP_M = 16;
constexpr uint32_t IDESC = idesc_bf16_f32(BM, BN);

struct Barriers {
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint64_t drain;
  uint32_t tmem_base;
};

static_assert(sizeof(Barriers) <= TB_GEMM_BARRIER_BYTES, "barrier block overflows its reservation");
static_assert(STAGES * STAGE_BYTES + 1024 + TB_GEMM_BARRIER_BYTES == TB_GEMM_SMEM_BYTES, "smem layout");
static_assert(TB_GEMM_SMEM_BYTES <= 232448, "exceeds the 227 KB per-CTA shared memory limit");

// Failure codes written to the status word: 0x47xx_yyzz = GEMM, role, site.
constexpr uint32_t kFailProducer = 0x47010000u;
constexpr uint32_t kFailMma = 0x47020000u;
constexpr uint32_t kFailEpilogue = 0x47030000u;

__device__ __forceinline__ void tile_coords(int t, int num_m, int num_n, int& m_blk, int& n_blk) {
  const int group_size = GROUP_M * num_n;
  const int group = t / group_size;
  const int first_m = group * GROUP_M;
  const int gm = min(num_m - first_m, GROUP_M);
  const int r = t - group * group_size;
  m_blk = first_m + r % gm;
  n_blk = r / gm;
}

__device__ __forceinline__ void store_row_chunk(__nv_bfloat16* __restrict__ c, long long ldc, int row, int col0,
                                                int M, int N, bool vec_ok, const uint32_t (&r)[32]) {
  if (row >= M) return;
  __nv_bfloat16* dst = c + (long long)row * ldc + col0;
  if (vec_ok && col0 + 32 <= N) {
    uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint4 v;
      v.x = pack_bf16x2(__uint_as_float(r[8 * q + 0]), __uint_as_float(r[8 * q + 1]));
      v.y = pack_bf16x2(__uint_as_float(r[8 * q + 2]), __uint_as_float(r[8 * q + 3]));
      v.z = pack_bf16x2(__uint_as_float(r[8 * q + 4]), __uint_as_float(r[8 * q + 5]));
      v.w = pack_bf16x2(__uint_as_float(r[8 * q + 6]), __uint_as_float(r[8 * q + 7]));
      d4[q] = v;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (col0 + j < N) dst[j] = __float2bfloat16_rn(__uint_as_float(r[j]));
  }
}

}  // namespace

extern "C" __global__ void __launch_bounds__(THREADS, 1)
    gemm_bf16_tn(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                 __nv_bfloat16* __restrict__ c, int M, int N, int K, long long ldc, uint32_t* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Barriers* bars = reinterpret_cast<Barriers*>(smem + STAGES * STAGE_BYTES);

  const int warp = warp_id(), lane = lane_id();
  const int num_m = (M + BM - 1) / BM, num_n = (N + BN - 1) / BN;
  const int tiles = num_m * num_n;
  const int num_k = (K + BK - 1) / BK;
  const bool vec_ok = (ldc % 8) == 0 && (reinterpret_cast<uintptr_t>(c) & 15) == 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&bars->acc_full[a], 1);
      mbar_init(&bars->acc_empty[a], 4);
    }
    mbar_init(&bars->drain, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(&bars->tmem_base, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem_base = bars->tmem_base;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      tma_prefetch_desc(&tmap_a);
      tma_prefetch_desc(&tmap_b);
      uint32_t issued[STAGES] = {0, 0, 0, 0};
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
        int m_blk, n_blk;
        tile_coords(t, num_m, num_n, m_blk, n_blk);
        for (int kb = 0; kb < num_k; ++kb) {
          if (!mbar_wait(&bars->empty[stage], phase ^ 1)) {
            report_status(status, kFailProducer | 1);
            ok = false;
            break;
          }
          uint8_t* a_dst = smem + stage * STAGE_BYTES;
          uint8_t* b_dst = a_dst + A_BYTES;
          mbar_arrive_expect_tx(&bars->full[stage], STAGE_BYTES);
          tma_load_2d(a_dst, &tmap_a, &bars->full[stage], kb * BK, m_blk * BM);
          tma_load_2d(b_dst, &tmap_b, &bars->full[stage], kb * BK, n_blk * BN);
          ++issued[stage];
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok) {
        // Drain: every issued copy must land before the CTA's shared memory is released.
        for (int s = 0; s < STAGES; ++s)
          if (issued[s] && !mbar_wait(&bars->full[s], (issued[s] - 1) & 1)) report_status(status, kFailProducer | 2);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      int stage = 0, acc = 0;
      uint32_t phase = 0, acc_phase = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
        if (!mbar_wait(&bars->acc_empty[acc], acc_phase ^ 1)) {
          report_status(status, kFailMma | 1);
          break;
        }
        tc_fence_after_sync();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < num_k; ++kb) {
          if (!mbar_wait(&bars->full[stage], phase)) {
            report_status(status, kFailMma | 2);
            ok = false;
            break;
          }
          tc_fence_after_sync();
          const uint32_t a_addr = smem_addr(smem + stage * STAGE_BYTES);
          const uint32_t b_addr = a_addr + A_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t adesc = sdesc_sw128(a_addr + k * 32, 16, 1024);
            const uint64_t bdesc = sdesc_sw128(b_addr + k * 32, 16, 1024);
            umma_bf16_ss(d_tmem, adesc, bdesc, IDESC, (kb | k) != 0);
          }
          umma_commit(&bars->empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit(&bars->acc_full[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
      // Drain: all MMAs this thread issued complete before TMEM is freed.
      umma_commit(&bars->drain);
      if (!mbar_wait(&bars->drain, 0)) report_status(status, kFailMma | 3);
    }
  } else {
    // ---------------- epilogue (warps 2..5) ----------------
    const int quarter = warp & 3;  // TMEM lanes this warp may access: [32*quarter, 32*quarter+32)
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
      int m_blk, n_blk;
      tile_coords(t, num_m, num_n, m_blk, n_blk);
      bool ok = mbar_wait(&bars->acc_full[acc], acc_phase);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) {
        if (lane == 0) report_status(status, kFailEpilogue | 1);
        break;
      }
      tc_fence_after_sync();
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * BN;
      const int row = m_blk * BM + quarter * 32 + lane;
#pragma unroll 1
      for (int col = 0; col < BN; col += 32) {
        uint32_t r[32];
        tmem_ld_x32(taddr + col, r);
        tmem_ld_wait();
        store_row_chunk(c, ldc, row, n_blk * BN + col, M, N, vec_ok, r);
      }
      tc_fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->acc_empty[acc]);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
  }

  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after_sync();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

