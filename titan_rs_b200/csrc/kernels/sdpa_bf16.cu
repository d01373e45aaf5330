// Causal (or full) scaled-dot-product attention forward, bf16 in/out, fp32
// softmax statistics, on the 5th-generation tensor cores. Head dim D = 128.
//
// Semantics follow the titan.rs CPU reference (projects/titan-runtime/src/lib.rs:1090-1151):
// O = softmax(Q K^T / sqrt(D)) V over BHTD tensors, extended with a causal mask in
// which query i attends to keys j <= i (top-left aligned when Tq != Tk).
//
// Work unit: one CTA per (128-row query tile, batch*head); the grid is flat and
// head-major with the heaviest causal tiles of each head first. 192 threads,
// warp-specialised:
//   warp 0      TMA producer: the Q tile once, then K_j / V_j tiles (128 keys x 128 dims,
//               two 64-column 128-byte-swizzled boxes each) through 2-stage rings.
//   warp 1      owns 512 TMEM columns: S double buffer (2 x 128 fp32 columns) and
//               the O accumulator (128 columns). One lane issues
//                 S_j  = Q K_j^T  (M=128, N=128, K=16 x 8, both operands K-major)
//                 O   += P_j V_j  (M=128, N=128, K=16 x 8, V read MN-major)
//               S_{j+1} is issued before O += P_j V_j so the tensor core works on
//               the next scores while the softmax warps exponentiate.
//   warps 2..5  one query row per thread (its TMEM lane): online softmax in the
//               log2 domain (exp2 on the MUFU), causal/tail masking on boundary
//               tiles, P_j written as bf16 into a 128-byte-swizzled shared-memory
//               tile (the MMA's A operand), and the final O / l written as bf16.
// The running row maximum is only moved (and O rescaled in TMEM) when it grows
// by more than 2^8; the exponentials then stay below 256, so the result is
// exactly the online softmax with fewer rescales. S and P never reach HBM.
//
// Every wait is bounded; on a timeout the kernel records a code in `status`,
// drains its copies and MMAs, frees TMEM and exits.
#include "kernel_configs.h"
#include "sm100.cuh"

namespace {

using namespace tb;

constexpr int BM = 128, BN = 128, HD = 128;
constexpr int TILE_BYTES = 128 * HD * 2;  // 32 KB: 128 rows x 128 bf16 (two 16 KB swizzled boxes)
constexpr int HALF_BYTES = TILE_BYTES / 2;
constexpr int THREADS = TB_SDPA_THREADS;
constexpr uint32_t IDESC_S = idesc_bf16_f32(BM, BN, false);
constexpr uint32_t IDESC_O = idesc_bf16_f32(BM, HD, true);  // B = V, MN-major
constexpr float kLazyRescaleLog2 = 8.0f;

struct Barriers {
  uint64_t q_full;
  uint64_t k_full[2], k_empty[2];
  uint64_t v_full[2], v_empty[2];
  uint64_t s_full[2], s_empty[2];
  uint64_t p_full[2], p_empty[2];
  uint64_t o_done;
  uint64_t drain;
  uint32_t tmem_base;
};
static_assert(sizeof(Barriers) <= TB_SDPA_BARRIER_BYTES, "barrier block overflows its reservation");

// Shared-memory offsets (from a 1024-byte aligned base).
constexpr int OFF_Q = 0;
constexpr int OFF_K = OFF_Q + TILE_BYTES;
constexpr int OFF_V = OFF_K + 2 * TILE_BYTES;
constexpr int OFF_P = OFF_V + 2 * TILE_BYTES;
constexpr int OFF_BAR = OFF_P + 2 * TILE_BYTES;
static_assert(OFF_BAR + TB_SDPA_BARRIER_BYTES + 1024 == TB_SDPA_SMEM_BYTES, "smem layout");
static_assert(TB_SDPA_SMEM_BYTES <= 232448, "exceeds the 227 KB per-CTA shared memory limit");

constexpr uint32_t kFailProducer = 0x53010000u;
constexpr uint32_t kFailMma = 0x53020000u;
constexpr uint32_t kFailSoftmax = 0x53030000u;

__device__ __forceinline__ float exp2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Loads one 128-row x 128-dim bf16 tile (rows `row0..` of head `bh`) as two swizzled boxes.
__device__ __forceinline__ void load_tile(uint8_t* dst, const CUtensorMap* map, uint64_t* bar, int row0, int bh) {
  tma_load_3d(dst, map, bar, 0, row0, bh);
  tma_load_3d(dst + HALF_BYTES, map, bar, 64, row0, bh);
}

// Descriptor of the k-th 16-wide K slice of a K-major 128 x 128 tile (two 64-column boxes).
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t tile_addr, int k) {
  return sdesc_sw128(tile_addr + (k >> 2) * HALF_BYTES + (k & 3) * 32, 16, 1024);
}

// Descriptor of rows [16k, 16k+16) of the V tile read MN-major (N = head dim).
// Atoms: 8 key rows x 64 dims (1 KB); next 8 keys at +1024 (SBO); dims 64..127 at +16 KB (LBO).
__device__ __forceinline__ uint64_t v_desc(uint32_t tile_addr, int k) {
  return sdesc_sw128(tile_addr + k * 2048, HALF_BYTES, 1024);
}

}  // namespace

// q, k, v, o: [BH, T, 128] bf16 via 3-D tensor maps (dims {128, T, BH}, box {64, 128, 1}).
// scale_log2 = log2(e) / sqrt(D).
extern "C" __global__ void __launch_bounds__(THREADS, 1)
    sdpa_fwd_bf16_d128(const __grid_constant__ CUtensorMap tmap_q, const __grid_constant__ CUtensorMap tmap_k,
                       const __grid_constant__ CUtensorMap tmap_v, __nv_bfloat16* __restrict__ out, int Tq, int Tk,
                       int causal, float scale_log2, uint32_t* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Barriers* bars = reinterpret_cast<Barriers*>(smem + OFF_BAR);
  const int warp = warp_id(), lane = lane_id();
  // Flat grid, head-major: the query tiles of one head run together (so that
  // head's K/V stays in L2), heaviest causal tiles first within the head.
  const int num_qt = (Tq + BM - 1) / BM;
  const int bh = blockIdx.x / num_qt;
  const int qt = num_qt - 1 - (int)(blockIdx.x % num_qt);
  const int kv_tiles_all = (Tk + BN - 1) / BN;
  const int n = causal ? min(kv_tiles_all, qt + 1) : kv_tiles_all;

  if (threadIdx.x == 0) {
    mbar_init(&bars->q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars->k_full[i], 1);
      mbar_init(&bars->k_empty[i], 1);
      mbar_init(&bars->v_full[i], 1);
      mbar_init(&bars->v_empty[i], 1);
      mbar_init(&bars->s_full[i], 1);
      mbar_init(&bars->s_empty[i], 4);
      mbar_init(&bars->p_full[i], 4);
      mbar_init(&bars->p_empty[i], 1);
    }
    mbar_init(&bars->o_done, 1);
    mbar_init(&bars->drain, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(&bars->tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem = bars->tmem_base;
  const uint32_t tmem_o = tmem + 2 * BN;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      tma_prefetch_desc(&tmap_q);
      tma_prefetch_desc(&tmap_k);
      tma_prefetch_desc(&tmap_v);
      mbar_arrive_expect_tx(&bars->q_full, TILE_BYTES);
      load_tile(smem + OFF_Q, &tmap_q, &bars->q_full, qt * BM, bh);
      uint32_t k_issued[2] = {0, 0}, v_issued[2] = {0, 0};
      bool ok = true;
      for (int j = 0; j < n && ok; ++j) {
        const int st = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        if (!mbar_wait(&bars->k_empty[st], ph ^ 1)) {
          report_status(status, kFailProducer | 1);
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&bars->k_full[st], TILE_BYTES);
        load_tile(smem + OFF_K + st * TILE_BYTES, &tmap_k, &bars->k_full[st], j * BN, bh);
        ++k_issued[st];
        if (!mbar_wait(&bars->v_empty[st], ph ^ 1)) {
          report_status(status, kFailProducer | 2);
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&bars->v_full[st], TILE_BYTES);
        load_tile(smem + OFF_V + st * TILE_BYTES, &tmap_v, &bars->v_full[st], j * BN, bh);
        ++v_issued[st];
      }
      if (!ok) {
        if (!mbar_wait(&bars->q_full, 0)) report_status(status, kFailProducer | 3);
        for (int s = 0; s < 2; ++s) {
          if (k_issued[s] && !mbar_wait(&bars->k_full[s], (k_issued[s] - 1) & 1)) report_status(status, kFailProducer | 4);
          if (v_issued[s] && !mbar_wait(&bars->v_full[s], (v_issued[s] - 1) & 1)) report_status(status, kFailProducer | 5);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      bool ok = mbar_wait(&bars->q_full, 0);
      if (!ok) report_status(status, kFailMma | 1);
      tc_fence_after_sync();
      const uint32_t q_addr = smem_addr(smem + OFF_Q);
      for (int j = 0; j <= n && ok; ++j) {
        if (j < n) {
          const int st = j & 1;
          const uint32_t ph = (j >> 1) & 1;
          if (!mbar_wait(&bars->k_full[st], ph) || !mbar_wait(&bars->s_empty[st], ph ^ 1)) {
            report_status(status, kFailMma | 2);
            ok = false;
            break;
          }
          tc_fence_after_sync();
          const uint32_t k_addr = smem_addr(smem + OFF_K + st * TILE_BYTES);
#pragma unroll
          for (int k = 0; k < HD / 16; ++k)
            umma_bf16_ss(tmem + st * BN, kmajor_desc(q_addr, k), kmajor_desc(k_addr, k), IDESC_S, k > 0);
          umma_commit(&bars->s_full[st]);
          umma_commit(&bars->k_empty[st]);
        }
        if (j >= 1) {
          const int jj = j - 1, st = jj & 1;
          const uint32_t ph = (jj >> 1) & 1;
          if (!mbar_wait(&bars->p_full[st], ph) || !mbar_wait(&bars->v_full[st], ph)) {
            report_status(status, kFailMma | 3);
            ok = false;
            break;
          }
          tc_fence_after_sync();
          const uint32_t p_addr = smem_addr(smem + OFF_P + st * TILE_BYTES);
          const uint32_t v_addr = smem_addr(smem + OFF_V + st * TILE_BYTES);
#pragma unroll
          for (int k = 0; k < BN / 16; ++k)
            umma_bf16_ss(tmem_o, kmajor_desc(p_addr, k), v_desc(v_addr, k), IDESC_O, (jj > 0) || (k > 0));
          umma_commit(&bars->p_empty[st]);
          umma_commit(&bars->v_empty[st]);
          umma_commit(&bars->o_done);
        }
      }
      umma_commit(&bars->drain);
      if (!mbar_wait(&bars->drain, 0)) report_status(status, kFailMma | 4);
    }
  } else {
    // ---------------- softmax / correction / epilogue (warps 2..5) ----------------
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // row of the tile == TMEM lane
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const int q_row = qt * BM + r;
    float m_used = -INFINITY;  // running max in the scaled log2 domain
    float l = 0.f;
    bool ok = true;
    for (int j = 0; j < n; ++j) {
      const int st = j & 1;
      const uint32_t ph = (j >> 1) & 1;
      ok = __all_sync(0xffffffffu, mbar_wait(&bars->s_full[st], ph));
      if (!ok) {
        if (lane == 0) report_status(status, kFailSoftmax | 1);
        break;
      }
      tc_fence_after_sync();
      float s[BN];
#pragma unroll
      for (int c = 0; c < BN; c += 32) {
        uint32_t raw[32];
        tmem_ld_x32(tmem + lane_off + st * BN + c, raw);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i) s[c + i] = __uint_as_float(raw[i]);
      }
      tc_fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->s_empty[st]);

      const int kv0 = j * BN;
      // Leading keys of this tile the row may see; four max accumulators keep the
      // reduction off one long dependency chain.
      const int valid = (causal ? min(Tk, q_row + 1) : Tk) - kv0;
      float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
      if (valid < BN) {
#pragma unroll
        for (int c = 0; c < BN; ++c)
          if (c >= valid) s[c] = -INFINITY;
      }
#pragma unroll
      for (int c = 0; c < BN; ++c) mx4[c & 3] = fmaxf(mx4[c & 3], s[c]);
      const float mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3])) * scale_log2;
      // Lazy rescale: move the reference maximum only when it grows by > 2^8.
      const bool grow = mx > m_used + kLazyRescaleLog2;
      if (__any_sync(0xffffffffu, grow)) {
        const float m_new = grow ? mx : m_used;
        const float alpha = exp2_approx(m_used - m_new);  // 0 on the first tile
        l *= alpha;
        if (j > 0) {
          // O holds sum_{t<j} P_t V_t: wait until the last of those MMAs finished, rescale in place.
          ok = __all_sync(0xffffffffu, mbar_wait(&bars->o_done, (j - 1) & 1));
          if (!ok) {
            if (lane == 0) report_status(status, kFailSoftmax | 2);
            break;
          }
          tc_fence_after_sync();
#pragma unroll 1
          for (int c = 0; c < HD; c += 16) {
            uint32_t o[16];
            tmem_ld_x16(tmem_o + lane_off + c, o);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 16; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
            tmem_st_x16(tmem_o + lane_off + c, o);
          }
          tmem_st_wait();
        }
        m_used = m_new;
      }
      // P = 2^(s*scale - m_used) (one FFMA each, bf16), l += rowsum(P) in fp32.
      uint32_t packed[BN / 2];
      float rs4[4] = {0.f, 0.f, 0.f, 0.f};
      const float neg_m = -m_used;
#pragma unroll
      for (int c = 0; c < BN; c += 2) {
        const float p0 = exp2_approx(fmaf(s[c], scale_log2, neg_m));
        const float p1 = exp2_approx(fmaf(s[c + 1], scale_log2, neg_m));
        rs4[(c >> 1) & 3] += p0 + p1;
        packed[c / 2] = pack_bf16x2(p0, p1);
      }
      l += (rs4[0] + rs4[1]) + (rs4[2] + rs4[3]);
      ok = __all_sync(0xffffffffu, mbar_wait(&bars->p_empty[st], ph ^ 1));
      if (!ok) {
        if (lane == 0) report_status(status, kFailSoftmax | 3);
        break;
      }
      // Row r of the P tile: 16 chunks of 8 keys, 128-byte swizzle (chunk ^ (row & 7)).
      uint8_t* p_tile = smem + OFF_P + st * TILE_BYTES;
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        const int sub = c >> 3, cc = c & 7;
        uint4 v = make_uint4(packed[4 * c], packed[4 * c + 1], packed[4 * c + 2], packed[4 * c + 3]);
        *reinterpret_cast<uint4*>(p_tile + sub * HALF_BYTES + r * 128 + ((cc ^ (r & 7)) << 4)) = v;
      }
      fence_proxy_async_smem();
      tc_fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->p_full[st]);
    }
    if (ok) {
      // ---------------- epilogue: O / l -> bf16 ----------------
      ok = __all_sync(0xffffffffu, mbar_wait(&bars->o_done, (n - 1) & 1));
      if (!ok) {
        if (lane == 0) report_status(status, kFailSoftmax | 4);
      } else {
        tc_fence_after_sync();
        const float inv_l = 1.0f / l;
        __nv_bfloat16* dst = out + ((long long)bh * Tq + q_row) * HD;
#pragma unroll 1
        for (int c = 0; c < HD; c += 32) {
          uint32_t o[32];
          tmem_ld_x32(tmem_o + lane_off + c, o);
          tmem_ld_wait();
          if (q_row < Tq) {
            uint4* d4 = reinterpret_cast<uint4*>(dst + c);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              uint4 w;
              w.x = pack_bf16x2(__uint_as_float(o[8 * q + 0]) * inv_l, __uint_as_float(o[8 * q + 1]) * inv_l);
              w.y = pack_bf16x2(__uint_as_float(o[8 * q + 2]) * inv_l, __uint_as_float(o[8 * q + 3]) * inv_l);
              w.z = pack_bf16x2(__uint_as_float(o[8 * q + 4]) * inv_l, __uint_as_float(o[8 * q + 5]) * inv_l);
              w.w = pack_bf16x2(__uint_as_float(o[8 * q + 6]) * inv_l, __uint_as_float(o[8 * q + 7]) * inv_l);
              d4[q] = w;
            }
          }
        }
      }
    }
  }

  tc_fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after_sync();
    tmem_dealloc(tmem, 512);
  }
}
