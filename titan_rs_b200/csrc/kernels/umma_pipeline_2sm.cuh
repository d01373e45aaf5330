// Persistent tcgen05 GEMM pipeline on CTA pairs (2-SM MMA, `cta_group::2`).
//
// A cluster of two CTAs on two SMs computes one 256 x 256 output tile:
//   D[256 x 256] (+)= A[256 x 64] * B[256 x 64]^T per k-block, bf16 in, fp32 in TMEM.
// CTA rank r of the pair holds A rows [128 r, 128 r + 128) and B rows (output
// columns) [128 r, 128 r + 128) of the tile in its shared memory, at the same
// offsets in both CTAs. One lane of the even CTA issues tcgen05.mma.cta_group::2
// with M = 256, N = 256: the tensor cores of both SMs read both CTAs' B halves and
// each SM its own A half, and each CTA's TMEM receives its own 128 rows x 256
// columns. Per SM, one k-block moves 32 KB from L2 instead of 48 KB for the
// single-SM 128 x 256 tile at the same work per SM.
//
//   warp 0      TMA producer in each CTA: its A and B halves into its own stage; the
//               transaction bytes of both CTAs land on the even CTA's `full` barrier
//               (2-SM tensor loads, each CTA reading only its own tiles).
//   warp 1      TMEM owner in each CTA (tcgen05.alloc.cta_group::2, 512 columns = two
//               128 x 256 fp32 accumulators); in the even CTA one lane issues the MMAs
//               and commits with .multicast::cluster to both CTAs' `empty` and
//               `acc_full` barriers.
//   warps 2..5  epilogue of each CTA's 128 rows; after draining an accumulator they
//               arrive on the even CTA's `acc_empty` (4 local + 4 remote arrivals).
//   warps 6..   optional side warps of a policy (the fused all-gather's push warps).
// Problems plug in as policies (run() below): the tile space, per-tile load and store
// cursors (index arithmetic once per tile, never per k-block: the single producer lane
// is on the critical path), M- or N-contiguous operand tiles (A stored [K, M], B
// stored [K, N]), and a pair count for kernels whose other CTAs do another job.
// Every mbarrier wait is bounded; both CTAs always reach the two cluster barriers
// (after barrier initialisation, and before TMEM is freed), so a failure in one role
// ends as a status code, not a hang.
#pragma once

#include "umma_pipeline.cuh"

namespace tb {
namespace umma2 {

constexpr int BM = 128;   // rows per CTA (256 per pair)
constexpr int BN = 256;   // output columns per pair tile
constexpr int BK = 64;
constexpr int STAGES = TB_GEMM2_STAGES;
constexpr int A_BYTES = BM * BK * 2;            // 16 KB
constexpr int B_BYTES = (BN / 2) * BK * 2;      // 16 KB: this CTA's half of B
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;  // 32 KB per CTA
constexpr int TMEM_COLS = 2 * BN;
constexpr uint32_t IDESC = idesc_bf16_f32(2 * BM, BN);

template <int Stages>
struct Barriers {
  uint64_t full[Stages];    // even CTA: both CTAs' bytes of a stage have landed
  uint64_t empty[Stages];   // each CTA: the pair's MMAs are done with this CTA's stage
  uint64_t acc_full[2];     // each CTA: its accumulator rows are ready
  uint64_t acc_empty[2];    // even CTA: both CTAs' epilogues drained the accumulator
  uint64_t drain;
  uint32_t tmem_base;
};
// Dynamic shared memory of a kernel with `stages` ring stages (1 KB of alignment slack included).
__host__ __device__ constexpr int smem_bytes(int stages) { return stages * STAGE_BYTES + 1024 + TB_GEMM2_BARRIER_BYTES; }
static_assert(sizeof(Barriers<8>) <= TB_GEMM2_BARRIER_BYTES, "barrier block overflows its reservation");
static_assert(smem_bytes(STAGES) == TB_GEMM2_SMEM_BYTES, "smem layout");
static_assert(TB_GEMM2_SMEM_BYTES <= 232448, "exceeds the 227 KB per-CTA shared memory limit");
static_assert(TB_GEMM2_AG_SMEM_BYTES <= 232448, "fused all-gather staging exceeds the 227 KB limit");
static_assert(TB_GEMM2_AG_SMEM_BYTES == smem_bytes(TB_GEMM2_AG_STAGES) + 128 + 8 * 32 * 256, "all-gather smem layout");

// Dynamic shared memory past the ring and the barriers (from the 1 KB-aligned base) is
// free for a policy's epilogue staging; its kernel is launched with the extra bytes.
template <int Stages = STAGES>
__device__ __forceinline__ uint8_t* epilogue_smem() {
  extern __shared__ uint8_t smem_raw[];
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023)) +
         Stages * STAGE_BYTES + TB_GEMM2_BARRIER_BYTES;
}

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Shared::cluster address of the same shared-memory location in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t map_to_rank(uint32_t smem, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem), "r"(rank));
  return r;
}

__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

// 2-D tile load into this CTA's shared memory whose completion bytes go to the even
// CTA's barrier (`bar_cluster` is that barrier's shared::cluster address).
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, uint32_t bar_cluster, int32_t x,
                                                 int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
      "[%2];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void tma_load_3d_pair(void* dst, const CUtensorMap* map, uint32_t bar_cluster, int32_t x,
                                                 int32_t y, int32_t z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, "
      "%5}], [%2];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(x), "r"(y), "r"(z)
      : "memory");
}

__device__ __forceinline__ void tma_load_4d_pair(void* dst, const CUtensorMap* map, uint32_t bar_cluster, int32_t x,
                                                 int32_t y, int32_t z, int32_t w) {
  asm volatile(
      "cp.async.bulk.tensor.4d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, "
      "%5, %6}], [%2];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(x), "r"(y), "r"(z), "r"(w)
      : "memory");
}

__device__ __forceinline__ void umma_bf16_ss_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                                  uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrives on `bar` (same offset) in every CTA of `cta_mask` once the pair's MMAs so far are done.
__device__ __forceinline__ void umma_commit_pair(uint64_t* bar, uint16_t cta_mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_addr(bar)),
      "h"(cta_mask)
      : "memory");
}

// Arrives on the issuing CTA's `bar` once the pair's MMAs so far are done.
__device__ __forceinline__ void umma_commit_pair_local(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst, uint32_t cols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(dst)), "r"(cols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t tmem, uint32_t cols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(cols) : "memory");
}

// A problem policy supplies the tile space in 128-row blocks (m_blocks) and 256-column
// blocks (n_blocks), the k-block count (k_blocks), and two per-tile cursors that do
// their index arithmetic once per tile, so the single producer lane spends its time
// issuing copies (a runtime integer division per k-block costs more than the copy):
//   loader(m_blk, n_blk, half) -> L;  L.load(a_dst, b_dst, bar) loads the next k-block:
//        A rows of 128-row block m_blk and B rows [256 n_blk + 128 half, +128), completing
//        on `bar` (the even CTA's `full`, a shared::cluster address) with the *_pair
//        tensor loads;
//   storer(row, m_blk, n_blk, ordinal, status) -> W;  W.store(col, acc) stores 32 fp32
//        accumulator columns [col, col + 32) of one row (ordinal = the CTA's tile count
//        so far, for policies that hand tiles on through their own barriers).
// Pair tile t covers 128-row blocks 2 pm and 2 pm + 1 (CTA rank 0 and 1).
// A policy may add kSideWarps warps after the six pipeline warps (the block has
// 192 + 32 kSideWarps threads): they run side(i, first_tile, tile_stride, tiles, num_pm,
// num_n, status, fail_base) beside the pipeline, after init() has set up any barriers
// they share with the epilogue. kAMajorMN / kBMajorMN select M- / N-contiguous tiles
// (two 64-element boxes of 64 K-rows per operand, CTA and stage). pair_count() is the number of CTA pairs running the
// pipeline (the grid, unless the kernel gives other CTAs another job);
// tile_stored(t, rank, lane) runs in each epilogue warp after it stored its rows of pair
// tile t. PolicyBase supplies the defaults.
struct PolicyBase {
  static constexpr int kSideWarps = 0;
  static constexpr bool kAMajorMN = false;  // A tiles M-contiguous (A stored [K, M]) instead of K-contiguous
  static constexpr bool kBMajorMN = false;  // B tiles N-contiguous (B stored [K, N]) instead of K-contiguous
  __device__ void init() const {}
  __device__ void side(int, int, int, int, int, int, uint32_t*, uint32_t) const {}
  __device__ void finish() const {}
  __device__ int pair_count() const { return gridDim.x >> 1; }
  __device__ void tile_stored(int, int, int) const {}
};

template <class Policy, int Stages = STAGES, int Group = TB_GEMM2_GROUP>
__device__ __forceinline__ void run(const Policy& p, uint32_t* status, uint32_t fail_base) {
  static_assert(smem_bytes(Stages) <= 232448, "exceeds the 227 KB per-CTA shared memory limit");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Barriers<Stages>* bars = reinterpret_cast<Barriers<Stages>*>(smem + Stages * STAGE_BYTES);
  const int warp = warp_id(), lane = lane_id();
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  const int num_pm = (p.m_blocks() + 1) / 2;  // 256-row pair tiles
  const int num_n = p.n_blocks();
  const int tiles = num_pm * num_n;
  const int pair = blockIdx.x >> 1, pairs = p.pair_count();
  const int num_k = p.k_blocks();

  if (threadIdx.x == 0) {
    for (int s = 0; s < Stages; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&bars->acc_full[a], 1);
      mbar_init(&bars->acc_empty[a], 8);  // 4 epilogue warps in each CTA
    }
    mbar_init(&bars->drain, 1);
    p.init();              // the policy's own barriers (side warps), if any
    fence_barrier_init();  // .release.cluster: visible to the peer CTA
  }
  cluster_sync();  // both CTAs' barriers exist before anything arrives remotely
  if (warp == 1) {
    tmem_alloc_pair(&bars->tmem_base, TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem_base = bars->tmem_base;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer (both CTAs) ----------------
      p.prefetch();
      uint32_t issued = 0;  // k-blocks loaded so far; stage s was filled (issued + Stages - 1 - s) / Stages times
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      // The even CTA's `full` barriers as shared::cluster addresses (consecutive, 8 bytes apart).
      const uint32_t full_even0 = map_to_rank(smem_addr(&bars->full[0]), 0);
      for (int t = pair; t < tiles && ok; t += pairs) {
        int m_blk, n_blk;
        umma::grouped_tile(t, num_pm, num_n, Group, m_blk, n_blk);
        m_blk = 2 * m_blk + (int)rank;
        auto ld = p.loader(m_blk, n_blk, (int)rank);
        for (int kb = 0; kb < num_k; ++kb) {
          if (!mbar_wait(&bars->empty[stage], phase ^ 1)) {
            report_status(status, fail_base | 0x0101);
            ok = false;
            break;
          }
          uint8_t* a_dst = smem + stage * STAGE_BYTES;
          if (leader) mbar_arrive_expect_tx(&bars->full[stage], 2 * STAGE_BYTES);
          ld.load(a_dst, a_dst + A_BYTES, full_even0 + 8u * (uint32_t)stage);
          ++issued;
          if (++stage == Stages) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok && leader) {
        // The issued copies land on this CTA's `full` barriers: wait for them before TMEM goes.
        for (int s = 0; s < Stages; ++s) {
          const uint32_t fills = (issued + Stages - 1 - s) / Stages;
          if (fills && !mbar_wait(&bars->full[s], (fills - 1) & 1)) report_status(status, fail_base | 0x0102);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      // ---------------- MMA issuer (even CTA) ----------------
      int stage = 0, acc = 0;
      uint32_t phase = 0, acc_phase = 0;
      bool ok = true;
      const uint32_t stage0 = smem_addr(smem);
      for (int t = pair; t < tiles && ok; t += pairs) {
        if (!mbar_wait(&bars->acc_empty[acc], acc_phase ^ 1)) {
          report_status(status, fail_base | 0x0201);
          break;
        }
        tc_fence_after_sync();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < num_k; ++kb) {
          if (!mbar_wait(&bars->full[stage], phase)) {
            report_status(status, fail_base | 0x0202);
            ok = false;
            break;
          }
          tc_fence_after_sync();
          const uint32_t a_addr = stage0 + stage * STAGE_BYTES;
          // K-major operand: rows of 64 K, 16 K = 32 bytes. MN-major operand: 64-element
          // boxes of 64 K-rows (8 KB apart), 16 K = 16 rows = 2 KB.
          const uint64_t a_desc = Policy::kAMajorMN ? sdesc_sw128(a_addr, 8192, 1024) : sdesc_sw128(a_addr, 16, 1024);
          const uint64_t b_desc = Policy::kBMajorMN ? sdesc_sw128(a_addr + A_BYTES, 8192, 1024)
                                                    : sdesc_sw128(a_addr + A_BYTES, 16, 1024);
          constexpr uint32_t a_step = Policy::kAMajorMN ? (2048 >> 4) : 2;
          constexpr uint32_t b_step = Policy::kBMajorMN ? (2048 >> 4) : 2;
          constexpr uint32_t idesc = idesc_bf16_f32(2 * BM, BN, Policy::kBMajorMN, Policy::kAMajorMN);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            umma_bf16_ss_pair(d_tmem, a_desc + (uint64_t)(k * a_step), b_desc + (uint64_t)(k * b_step), idesc,
                              (kb > 0) || (k > 0));
          umma_commit_pair(&bars->empty[stage], 0x3);
          if (++stage == Stages) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit_pair(&bars->acc_full[acc], 0x3);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
      umma_commit_pair_local(&bars->drain);
      if (!mbar_wait(&bars->drain, 0)) report_status(status, fail_base | 0x0203);
    }
  } else if (warp >= 6) {
    // ---------------- side warps (warps 6.., policies with kSideWarps > 0) ----------------
    p.side(warp - 6, pair, pairs, tiles, num_pm, num_n, status, fail_base);
  } else {
    // ---------------- epilogue (warps 2..5 of both CTAs) ----------------
    const int quarter = warp & 3;
    const uint32_t acc_empty_even[2] = {map_to_rank(smem_addr(&bars->acc_empty[0]), 0),
                                        map_to_rank(smem_addr(&bars->acc_empty[1]), 0)};
    int acc = 0;
    uint32_t acc_phase = 0;
    int ordinal = 0;  // this CTA's tile count so far
    for (int t = pair; t < tiles; t += pairs, ++ordinal) {
      int m_blk, n_blk;
      umma::grouped_tile(t, num_pm, num_n, Group, m_blk, n_blk);
      m_blk = 2 * m_blk + (int)rank;
      const bool ok = __all_sync(0xffffffffu, mbar_wait(&bars->acc_full[acc], acc_phase));
      if (!ok) {
        if (lane == 0) report_status(status, fail_base | 0x0301);
        break;
      }
      tc_fence_after_sync();
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * BN;
      const auto st = p.storer(quarter * 32 + lane, m_blk, n_blk, ordinal, status);
#pragma unroll 1
      for (int col = 0; col < BN; col += 32) {
        uint32_t r[32];
        tmem_ld_x32(taddr + col, r);
        tmem_ld_wait();
        st.store(col, r);
      }
      p.tile_stored(t, (int)rank, lane);
      tc_fence_before_sync();
      __syncwarp();
      if (lane == 0) {
        if (leader) mbar_arrive(&bars->acc_empty[acc]);
        else mbar_arrive_remote(acc_empty_even[acc]);
      }
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
    p.finish();
  }

  tc_fence_before_sync();
  cluster_sync();  // no CTA frees TMEM or exits while its pair's MMAs may still use its memory
  if (warp == 1) {
    tc_fence_after_sync();
    tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
}

}  // namespace umma2
}  // namespace tb
