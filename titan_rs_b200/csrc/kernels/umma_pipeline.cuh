// Persistent, warp-specialised tcgen05 GEMM pipeline shared by the GEMM and the
// implicit-GEMM convolution. A problem policy supplies the tile space
// (num_tiles, tile, k_blocks = the k-block range of a tile) and two per-tile cursors
// that do their index arithmetic once per tile: loader(t, m_blk, n_blk, kb0) -> L,
// L.load(a_dst, b_dst, bar) issuing the TMA loads of the next k-block, and
// storer(row, t, m_blk, n_blk) -> W, W.store(col, acc) for 32 accumulator columns of
// one row. This file owns the shared-memory ring, the MMA issue and the TMEM
// accumulators.
//
//   D[128 x 256] (+)= A[128 x 64] * B[256 x 64]^T per k-block, bf16 in, fp32 in TMEM.
//   warp 0      TMA producer (Policy::load), 4-stage ring of 48 KB stages.
//   warp 1      TMEM owner (512 columns = two 128x256 fp32 accumulators); one
//               lane issues tcgen05.mma M=128 N=256 K=16, commits release stages
//               and publish accumulators.
//   warps 2..5  epilogue (Policy::store) of accumulator i while the MMA warp
//               already fills accumulator i^1 with the next tile.
// Every wait is bounded; on a timeout the kernel records `fail_base | site` in
// the status word, drains its copies and MMAs, frees TMEM and exits.
#pragma once

#include "epilogue_math.cuh"
#include "kernel_configs.h"
#include "sm100.cuh"

namespace tb {
namespace umma {

constexpr int BM = TB_GEMM_BM, BN = TB_GEMM_BN, BK = TB_GEMM_BK, STAGES = TB_GEMM_STAGES;
constexpr int A_BYTES = BM * BK * 2;  // 16 KB
constexpr int B_BYTES = BN * BK * 2;  // 32 KB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int TMEM_COLS = 2 * BN;
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
// Dynamic shared memory past the ring and the barriers (from the 1 KB-aligned base) is
// free for a policy's epilogue staging; its kernel is launched with the extra bytes.
constexpr int EPILOGUE_SMEM_OFFSET = STAGES * STAGE_BYTES + TB_GEMM_BARRIER_BYTES;
static_assert(TB_GEMM_AG_SMEM_BYTES <= 232448, "fused all-gather staging exceeds the 227 KB limit");

__device__ __forceinline__ uint8_t* epilogue_smem() {
  extern __shared__ uint8_t smem_raw[];
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023)) +
         EPILOGUE_SMEM_OFFSET;
}

// Grouped rasterisation: `group` M-blocks share each sweep over the N-blocks.
__device__ __forceinline__ void grouped_tile(int t, int num_m, int num_n, int group, int& m_blk, int& n_blk) {
  const int group_size = group * num_n;
  const int g = t / group_size;
  const int first_m = g * group;
  const int gm = min(num_m - first_m, group);
  const int r = t - g * group_size;
  m_blk = first_m + r % gm;
  n_blk = r / gm;
}

// Packs 32 fp32 accumulator columns (+ optional per-column bias, then an optional
// activation, epilogue_math.cuh) into bf16 and stores them.
__device__ __forceinline__ void store_bf16_chunk(__nv_bfloat16* dst, int valid_cols, bool vec_ok,
                                                 const uint32_t (&r)[32], const float* bias, int act = kActNone) {
  float f[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) f[j] = __uint_as_float(r[j]);
  if (bias) {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (j < valid_cols) f[j] += bias[j];
  }
  if (act != kActNone) {
#pragma unroll
    for (int j = 0; j < 32; ++j) f[j] = activate(f[j], act);
  }
  if (vec_ok && valid_cols >= 32) {
    uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint4 v;
      v.x = pack_bf16x2(f[8 * q + 0], f[8 * q + 1]);
      v.y = pack_bf16x2(f[8 * q + 2], f[8 * q + 3]);
      v.z = pack_bf16x2(f[8 * q + 4], f[8 * q + 5]);
      v.w = pack_bf16x2(f[8 * q + 6], f[8 * q + 7]);
      d4[q] = v;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (j < valid_cols) dst[j] = __float2bfloat16_rn(f[j]);
  }
}

template <class Policy>
__device__ __forceinline__ void run(const Policy& p, uint32_t* status, uint32_t fail_base) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Barriers* bars = reinterpret_cast<Barriers*>(smem + STAGES * STAGE_BYTES);

  const int warp = warp_id(), lane = lane_id();
  const int tiles = p.num_tiles();

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
      p.prefetch();
      uint32_t issued = 0;  // k-blocks loaded so far; stage s was filled (issued + STAGES - 1 - s) / STAGES times
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
        int m_blk, n_blk;
        p.tile(t, m_blk, n_blk);
        int kb0, kb1;
        p.k_blocks(t, kb0, kb1);
        auto ld = p.loader(t, m_blk, n_blk, kb0);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&bars->empty[stage], phase ^ 1)) {
            report_status(status, fail_base | 0x0101);
            ok = false;
            break;
          }
          uint8_t* a_dst = smem + stage * STAGE_BYTES;
          mbar_arrive_expect_tx(&bars->full[stage], STAGE_BYTES);
          ld.load(a_dst, a_dst + A_BYTES, &bars->full[stage]);
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok) {
        for (int s = 0; s < STAGES; ++s) {
          const uint32_t fills = (issued + STAGES - 1 - s) / STAGES;
          if (fills && !mbar_wait(&bars->full[s], (fills - 1) & 1)) report_status(status, fail_base | 0x0102);
        }
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
          report_status(status, fail_base | 0x0201);
          break;
        }
        tc_fence_after_sync();
        const uint32_t d_tmem = tmem_base + acc * BN;
        int kb0, kb1;
        p.k_blocks(t, kb0, kb1);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&bars->full[stage], phase)) {
            report_status(status, fail_base | 0x0202);
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
            umma_bf16_ss(d_tmem, adesc, bdesc, IDESC, (kb > kb0) || (k > 0));
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
      umma_commit(&bars->drain);
      if (!mbar_wait(&bars->drain, 0)) report_status(status, fail_base | 0x0203);
    }
  } else {
    // ---------------- epilogue (warps 2..5) ----------------
    const int quarter = warp & 3;  // TMEM lanes this warp may access: [32*quarter, 32*quarter+32)
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
      int m_blk, n_blk;
      p.tile(t, m_blk, n_blk);
      const bool ok = __all_sync(0xffffffffu, mbar_wait(&bars->acc_full[acc], acc_phase));
      if (!ok) {
        if (lane == 0) report_status(status, fail_base | 0x0301);
        break;
      }
      tc_fence_after_sync();
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * BN;
      const auto st = p.storer(quarter * 32 + lane, t, m_blk, n_blk);
#pragma unroll 1
      for (int col = 0; col < BN; col += 32) {
        uint32_t r[32];
        tmem_ld_x32(taddr + col, r);
        tmem_ld_wait();
        st.store(col, r);
      }
      tc_fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->acc_empty[acc]);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
    p.finish();
  }

  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after_sync();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

}  // namespace umma
}  // namespace tb
