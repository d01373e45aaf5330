// Problem policies for the tcgen05 GEMM pipeline (umma_pipeline.cuh) and the
// split-K reduction, shared by every translation unit that instantiates them.
//
//   GemmPolicy     C[M,N] bf16 = act(A[M,K] x B^T + bias), B stored [N,K] (column-major B);
//                  bias and act optional (the fused epilogue of gemm.bias_act).
//   SplitKPolicy   fp32 partial tiles of the same product; work unit
//                  t = split * (num_m * num_n) + output tile, each split covering
//                  kb_per_split k-blocks of 64 (the last one possibly fewer, none empty),
//                  written to `partial` laid out [splits][M][N].
//   splitk_reduce  C[m, n] = bf16( sum_{s < splits} partial[s][m][n] ), summed in
//                  split order, so the result is deterministic.
//   AllGatherPolicy  the GEMM of one rank's column block, fused with the all-gather:
//                  every packed output chunk is stored into each rank's copy of the
//                  row-major C (peer copies through CUDA IPC mappings over NVLink).
//   Gemm2Policy    GemmPolicy's product on the 2-SM pipeline (umma_pipeline_2sm.cuh):
//                  tensor maps with 128-row boxes for A and B.
//   AllGather2Policy      the fused all-gather on the 2-SM pipeline, its epilogue staging
//                  tiles in shared memory for four push warps.
//   AllGatherLocalPolicy  the GEMM CTAs of the fused all-gather with dedicated pusher
//                  CTAs: own C only, plus per-tile ready counts.
#pragma once

#include "umma_pipeline.cuh"
#include "umma_pipeline_2sm.cuh"

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
  const float* bias = nullptr;  // optional fp32 [N], added to the accumulator
  int act = kActNone;           // optional activation after the bias

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
  // A rows m_blk*128.., B rows n_blk*256.., K from kb0*64 on, one k-block per load().
  struct Loader {
    const CUtensorMap *ta, *tb;
    int row, col, k;
    __device__ void load(uint8_t* a_dst, uint8_t* b_dst, uint64_t* bar) {
      tma_load_2d(a_dst, ta, bar, k, row);
      tma_load_2d(b_dst, tb, bar, k, col);
      k += umma::BK;
    }
  };
  __device__ Loader loader(int, int m_blk, int n_blk, int kb0) const {
    return Loader{ta, tb, m_blk * umma::BM, n_blk * umma::BN, kb0 * umma::BK};
  }
  struct Storer {
    __nv_bfloat16* dst;  // row start at the tile's first column; null when the row is past M
    const float* bias;   // at the tile's first column, or null
    int cols;            // valid columns from the tile's first column
    int act;
    bool vec_ok;
    __device__ void store(int col, const uint32_t (&r)[32]) const {
      if (!dst || col >= cols) return;
      umma::store_bf16_chunk(dst + col, cols - col, vec_ok, r, bias ? bias + col : nullptr, act);
    }
  };
  __device__ Storer storer(int row, int, int m_blk, int n_blk) const {
    const int gr = m_blk * umma::BM + row;
    const int gc = n_blk * umma::BN;
    return Storer{gr < M ? c + (long long)gr * ldc + gc : nullptr, bias ? bias + gc : nullptr, N - gc, act, vec_ok};
  }
  __device__ void finish() const {}
};

struct Gemm2Policy : umma2::PolicyBase {
  const CUtensorMap* ta;
  const CUtensorMap* tb;
  __nv_bfloat16* c;
  int M, N, K;
  long long ldc;
  bool vec_ok;
  const float* bias = nullptr;
  int act = kActNone;

  __device__ int m_blocks() const { return (M + 127) / 128; }
  __device__ int n_blocks() const { return (N + umma2::BN - 1) / umma2::BN; }
  __device__ int k_blocks() const { return (K + umma2::BK - 1) / umma2::BK; }
  __device__ void prefetch() const {
    tma_prefetch_desc(ta);
    tma_prefetch_desc(tb);
  }
  struct Loader {
    const CUtensorMap *ta, *tb;
    int row, col, k;
    __device__ void load(uint8_t* a_dst, uint8_t* b_dst, uint32_t bar) {
      umma2::tma_load_2d_pair(a_dst, ta, bar, k, row);
      umma2::tma_load_2d_pair(b_dst, tb, bar, k, col);
      k += umma2::BK;
    }
  };
  __device__ Loader loader(int m_blk, int n_blk, int half) const {
    return Loader{ta, tb, m_blk * 128, n_blk * umma2::BN + half * 128, 0};
  }
  struct Storer {
    __nv_bfloat16* dst;  // row start at the tile's first column; null when the row is past M
    const float* bias;   // at the tile's first column, or null
    int cols;            // valid columns from the tile's first column
    int act;
    bool vec_ok;
    __device__ void store(int col, const uint32_t (&r)[32]) const {
      if (!dst || col >= cols) return;
      umma::store_bf16_chunk(dst + col, cols - col, vec_ok, r, bias ? bias + col : nullptr, act);
    }
  };
  __device__ Storer storer(int row, int m_blk, int n_blk, int, uint32_t*) const {
    const int gr = m_blk * 128 + row;
    const int gc = n_blk * umma2::BN;
    return Storer{gr < M ? c + (long long)gr * ldc + gc : nullptr, bias ? bias + gc : nullptr, N - gc, act, vec_ok};
  }
};

// Output bases of every rank's C for the fused GEMM + all-gather (index = rank).
struct RankOutputs {
  __nv_bfloat16* base[TB_MAX_RANKS];
};

// This rank computes C[:, col0 : col0 + N] of the row-major C[M, ldc] that every rank
// holds, and writes each output row segment into all `ranks` copies. Stores to a peer
// cross NVLink, where many small scattered writes waste the link, so each epilogue warp
// first collects its 32 rows x 128 columns (4 accumulator chunks) in shared memory
// (16-byte segments XOR-swizzled by row, so neither the row-wise writes nor the
// segment-wise reads conflict) and then writes them out with 16 lanes per 256-byte
// row segment: this rank's own copy first, then its successors', so at any moment the
// ranks write to different peers.
struct AllGatherPolicy : GemmPolicy {
  const RankOutputs* outs;  // kernel parameter space
  int ranks, self;
  long long col0;

  struct Storer {
    const RankOutputs* outs;
    uint8_t* stage;  // this warp's [32 rows][256 B] staging block
    int lane, row0, gc0, M, N, ranks, self;
    long long ldc, col0;
    __device__ void store(int col, const uint32_t (&r)[32]) const {
      const int first_seg = (col & 127) >> 3;  // 0, 4, 8, 12
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint4 v;
        v.x = pack_bf16x2(__uint_as_float(r[8 * q + 0]), __uint_as_float(r[8 * q + 1]));
        v.y = pack_bf16x2(__uint_as_float(r[8 * q + 2]), __uint_as_float(r[8 * q + 3]));
        v.z = pack_bf16x2(__uint_as_float(r[8 * q + 4]), __uint_as_float(r[8 * q + 5]));
        v.w = pack_bf16x2(__uint_as_float(r[8 * q + 6]), __uint_as_float(r[8 * q + 7]));
        *reinterpret_cast<uint4*>(stage + lane * 256 + (((first_seg + q) ^ (lane & 15)) << 4)) = v;
      }
      if ((col & 127) != 96) return;  // the 128-column half is complete after its fourth chunk
      __syncwarp();
      const int seg = lane & 15;                     // 16-byte segment (8 columns) of a row
      const int gc = gc0 + (col & ~127) + seg * 8;  // this lane's local column
      for (int it = 0; it < 16; ++it) {
        const int rr = 2 * it + (lane >> 4);
        const uint4 v = *reinterpret_cast<const uint4*>(stage + rr * 256 + ((seg ^ (rr & 15)) << 4));
        const int gr = row0 + rr;
        if (gr < M && gc < N) {
          const long long off = (long long)gr * ldc + col0 + gc;
          for (int i = 0, d = self; i < ranks; ++i, d = (d + 1 == ranks) ? 0 : d + 1)
            *reinterpret_cast<uint4*>(outs->base[d] + off) = v;
        }
      }
      __syncwarp();  // the next half overwrites the staging block
    }
  };
  __device__ Storer storer(int row, int, int m_blk, int n_blk) const {
    return Storer{outs, umma::epilogue_smem() + (row >> 5) * (32 * 256), row & 31, m_blk * umma::BM + (row & ~31),
                  n_blk * umma::BN, M, N, ranks, self, ldc, col0};
  }
  // The peer stores of this thread are performed system-wide before the kernel ends,
  // hence before the barrier that follows it on the stream signals any peer.
  __device__ void finish() const { __threadfence_system(); }
};

// AllGatherPolicy's product on the 2-SM pipeline, with the peer stores taken off the
// epilogue. Writing a tile into every rank's C over NVLink takes about as long as
// computing it, and an epilogue that did it would hold its TMEM accumulator (and so
// the tensor cores) until the link had taken everything. Here the four epilogue warps
// only pack their 32 rows into shared memory, one 32 x 128 slot per half tile (eight
// slots = one whole 128 x 256 tile per CTA), and free the accumulator; four side
// ("push") warps, one per epilogue warp, drain the slots to all ranks while the next
// tile computes. Slot handshake: mbarriers slot_full / slot_empty (one arrival each),
// phase = the CTA's tile ordinal.
// `enabled` is false after a failed entry handshake: the CTA still runs the pipeline
// with its pair (both CTAs must reach the pipeline's cluster barriers) but stores nothing.
struct AllGather2Policy : Gemm2Policy {
  static constexpr int kSideWarps = 4;
  static constexpr int kStages = TB_GEMM2_AG_STAGES;  // 5 x 32 KB + 64 KB of slots fit in 227 KB
  static constexpr int kSlotBytes = 32 * 256;
  static constexpr int kStagingBytes = 128 + 8 * kSlotBytes;
  const RankOutputs* outs;  // kernel parameter space
  int ranks, self;
  long long col0;
  bool enabled;

  struct Slots {
    uint64_t full[8];
    uint64_t empty[8];
  };
  __device__ static Slots* slots() { return reinterpret_cast<Slots*>(umma2::epilogue_smem<kStages>()); }
  __device__ static uint8_t* slot(int i) { return umma2::epilogue_smem<kStages>() + 128 + i * kSlotBytes; }

  __device__ void init() const {
    for (int i = 0; i < 8; ++i) {
      mbar_init(&slots()->full[i], 1);
      mbar_init(&slots()->empty[i], 1);
    }
  }

  struct Storer {
    int lane, quarter;
    uint32_t parity;
    uint32_t* status;
    __device__ void store(int col, const uint32_t (&r)[32]) const {
      const int half = col >> 7, s = quarter * 2 + half;
      uint8_t* stage = slot(s);
      if ((col & 127) == 0) {
        // The push warp has drained this slot's previous tile (first use passes at once).
        if (!__all_sync(0xffffffffu, mbar_wait(&slots()->empty[s], parity ^ 1)) && lane == 0)
          report_status(status, 0x47420601);
      }
      const int first_seg = (col & 127) >> 3;  // 0, 4, 8, 12
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint4 v;
        v.x = pack_bf16x2(__uint_as_float(r[8 * q + 0]), __uint_as_float(r[8 * q + 1]));
        v.y = pack_bf16x2(__uint_as_float(r[8 * q + 2]), __uint_as_float(r[8 * q + 3]));
        v.z = pack_bf16x2(__uint_as_float(r[8 * q + 4]), __uint_as_float(r[8 * q + 5]));
        v.w = pack_bf16x2(__uint_as_float(r[8 * q + 6]), __uint_as_float(r[8 * q + 7]));
        *reinterpret_cast<uint4*>(stage + lane * 256 + (((first_seg + q) ^ (lane & 15)) << 4)) = v;
      }
      if ((col & 127) == 96) {  // the half is complete after its fourth chunk
        __syncwarp();
        if (lane == 0) mbar_arrive(&slots()->full[s]);
      }
    }
  };
  __device__ Storer storer(int row, int, int, int it, uint32_t* status) const {
    return Storer{row & 31, row >> 5, (uint32_t)it & 1u, status};
  }

  // Push warp i drains epilogue warp i's slots: 32 rows x 128 columns per slot, 16 lanes
  // per 256-byte row segment, into this rank's own C first, then its successors'.
  __device__ void side(int i, int first, int stride, int tiles, int num_pm, int num_n, uint32_t* status,
                       uint32_t fail_base) const {
    const int lane = lane_id(), seg = lane & 15;
    const int rank = (int)umma2::cluster_rank();
    uint32_t parity = 0;
    bool ok = true;
    for (int t = first; t < tiles && ok; t += stride, parity ^= 1) {
      int m_blk, n_blk;
      umma::grouped_tile(t, num_pm, num_n, TB_GEMM2_GROUP, m_blk, n_blk);
      m_blk = 2 * m_blk + rank;
      const int row0 = m_blk * 128 + i * 32;
      for (int half = 0; half < 2; ++half) {
        const int s = i * 2 + half;
        if (!__all_sync(0xffffffffu, mbar_wait(&slots()->full[s], parity))) {
          if (lane == 0) report_status(status, fail_base | 0x0701);
          ok = false;
          break;
        }
        const uint8_t* stage = slot(s);
        const int gc = n_blk * umma2::BN + half * 128 + seg * 8;
        if (enabled) {
          for (int it = 0; it < 16; ++it) {
            const int rr = 2 * it + (lane >> 4);
            const uint4 v = *reinterpret_cast<const uint4*>(stage + rr * 256 + ((seg ^ (rr & 15)) << 4));
            const int gr = row0 + rr;
            if (gr < M && gc < N) {
              const long long off = (long long)gr * ldc + col0 + gc;
              for (int k = 0, d = self; k < ranks; ++k, d = (d + 1 == ranks) ? 0 : d + 1)
                *reinterpret_cast<uint4*>(outs->base[d] + off) = v;
            }
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&slots()->empty[s]);
      }
    }
    // These threads' peer stores are performed system-wide before the pipeline's final
    // cluster barrier, hence before the kernel's exit handshake.
    __threadfence_system();
  }
};

// Gemm2Policy's product for the other storage orders: A stored [K, M] (transpose_lhs,
// AT) and/or B stored [K, N] (the reference's default, no transpose_rhs, BN). An
// M- or N-contiguous operand comes as two {64, 64 K} boxes per CTA and stage from a
// tensor map over its [K, rows] storage; the MMA reads it MN-major.
template <bool AT, bool BN_>
struct Gemm2LayoutPolicy : Gemm2Policy {
  static constexpr bool kAMajorMN = AT;
  static constexpr bool kBMajorMN = BN_;
  struct Loader {
    const CUtensorMap *ta, *tb;
    int row, col, k;
    __device__ void load(uint8_t* a_dst, uint8_t* b_dst, uint32_t bar) {
      if constexpr (AT) {
        umma2::tma_load_2d_pair(a_dst, ta, bar, row, k);
        umma2::tma_load_2d_pair(a_dst + 8192, ta, bar, row + 64, k);
      } else {
        umma2::tma_load_2d_pair(a_dst, ta, bar, k, row);
      }
      if constexpr (BN_) {
        umma2::tma_load_2d_pair(b_dst, tb, bar, col, k);
        umma2::tma_load_2d_pair(b_dst + 8192, tb, bar, col + 64, k);
      } else {
        umma2::tma_load_2d_pair(b_dst, tb, bar, k, col);
      }
      k += umma2::BK;
    }
  };
  __device__ Loader loader(int m_blk, int n_blk, int half) const {
    return Loader{ta, tb, m_blk * 128, n_blk * umma2::BN + half * 128, 0};
  }
};

// The GEMM half of the fused all-gather with dedicated pusher CTAs
// (gemm_bf16_tn_allgather_2sm_push): the pipeline's CTAs write this rank's column block
// into its own C only (c = own C at column col0) and count each CTA-tile's stored
// quarters in ready[2 t + rank] (four per tile: one per epilogue warp); pusher CTAs on
// other SMs copy finished tiles to the peers. Peer stores from the SMs that run the
// tensor-core pipeline slow that pipeline far more than the stores take (the
// stores wait in the same memory-instruction path as its TMA and MMA issue), so these
// SMs keep to local memory.
struct AllGatherLocalPolicy : Gemm2Policy {
  uint32_t* ready;
  int gemm_pairs;
  bool enabled;  // false after a failed entry handshake: same tiles, nothing stored
  __device__ int pair_count() const { return gemm_pairs; }
  __device__ Storer storer(int row, int m_blk, int n_blk, int ordinal, uint32_t* status) const {
    Storer w = Gemm2Policy::storer(row, m_blk, n_blk, ordinal, status);
    if (!enabled) w.dst = nullptr;
    return w;
  }
  __device__ void tile_stored(int t, int rank, int lane) const {
    __syncwarp();
    if (lane == 0) {
      __threadfence();  // this warp's stores (seen through the warp barrier) before the count
      atomicAdd(&ready[2 * t + rank], 1u);
    }
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
  __device__ GemmPolicy::Loader loader(int, int m_blk, int n_blk, int kb0) const {
    return GemmPolicy::Loader{ta, tb, m_blk * umma::BM, n_blk * umma::BN, kb0 * umma::BK};
  }
  struct Storer {
    float* dst;  // this row of split s's partial plane at the tile's first column; null past M
    int cols;    // valid columns from the tile's first column
    bool vec_ok;
    __device__ void store(int col, const uint32_t (&r)[32]) const {
      if (!dst || col >= cols) return;
      SplitKPolicy::store_chunk(dst + col, cols - col, vec_ok, r);
    }
  };
  __device__ Storer storer(int row, int t, int m_blk, int n_blk) const {
    const int s = t / (num_m * num_n);
    const int gr = m_blk * umma::BM + row;
    const int gc = n_blk * umma::BN;
    return Storer{gr < M ? partial + ((long long)s * M + gr) * N + gc : nullptr, N - gc, vec_ok};
  }
  __device__ static void store_chunk(float* dst, int valid, bool vec_ok, const uint32_t (&r)[32]) {
    if (vec_ok && valid >= 32) {
#pragma unroll
      for (int q = 0; q < 8; ++q)
        reinterpret_cast<float4*>(dst)[q] = make_float4(__uint_as_float(r[4 * q]), __uint_as_float(r[4 * q + 1]),
                                                        __uint_as_float(r[4 * q + 2]), __uint_as_float(r[4 * q + 3]));
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (j < valid) dst[j] = __uint_as_float(r[j]);
    }
  }
  __device__ void finish() const {}
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
