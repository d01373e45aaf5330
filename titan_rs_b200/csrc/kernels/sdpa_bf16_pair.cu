// Causal (or full) attention forward, bf16 in/out, fp32 softmax statistics,
// head dim 128: two query tiles per CTA with ping-pong softmax warpgroups.
//
// Semantics: the titan.rs CPU reference (projects/titan-runtime/src/lib.rs:1090-1151),
// O = softmax(Q K^T / sqrt(D)) V over BHTD, plus a causal mask (query i sees keys j <= i,
// top-left aligned when Tq != Tk).
//
// One CTA per (pair of 128-row query tiles A = 2i, B = 2i+1, batch*head); 320 threads:
//   warp 0       TMA producer: Q_A and Q_B once, then K_j / V_j (128 keys x 128 dims,
//                two 64-column 128-byte-swizzled boxes each) through 2-stage rings.
//   warp 1       owns all 512 TMEM columns: S_A | S_B | O_A | O_B (128 fp32 columns each).
//                One lane issues, per key tile j,
//                  PV_A(j-1) then S_A(j), PV_B(j-1) then S_B(j)
//                so the tensor core works on one tile's products while the other
//                tile's warpgroup exponentiates.
//                  S_X(j)  = Q_X K_j^T   (SS: both operands K-major in shared memory)
//                  O_X    += P_X(j) V_j  (TS: P read from TMEM, V MN-major in shared memory)
//   warps 2..5   softmax group for tile A, warps 6..9 for tile B (each group covers the
//                four TMEM lane quarters, since warp w reaches lanes 32*(w%4)..): one query row per
//                thread (its TMEM lane). The S row is streamed from TMEM once in
//                32-column chunks and exponentiated against the current reference max
//                (one FFMA each; one exponential in four on the FMA pipe, the rest on
//                the MUFU); P is held in registers, then written back as bf16 pairs
//                over the first 64 columns of the same S region, where the TS-MMA
//                reads it. The reference max moves (O is rescaled in TMEM and the row
//                recomputed from the still-intact S) only when the row max grows by
//                more than 2^8, so P stays below 256 and the result is the exact online
//                softmax.
// Ordering: tcgen05.commit arrives once ALL earlier MMAs of the issuing thread are
// done, so "S_X(j) ready" also means PV_X(j-1) finished reading P_X and writing O_X:
// the softmax warps may then overwrite S/P and rescale O without further waits.
//
// Every wait is bounded; on a timeout the kernel records a code in `status`,
// drains its copies and MMAs, frees TMEM and exits.
#include "kernel_configs.h"
#include "sm100.cuh"

namespace {

using namespace tb;

constexpr int BM = 128, BN = 128, HD = 128;
constexpr int TILE_BYTES = 128 * HD * 2;  // 32 KB
constexpr int HALF_BYTES = TILE_BYTES / 2;
constexpr int THREADS = TB_SDPA2_THREADS;
constexpr uint32_t IDESC_S = idesc_bf16_f32(BM, BN, false);
constexpr uint32_t IDESC_O = idesc_bf16_f32(BM, HD, true);  // B = V, MN-major
constexpr float kLazyRescaleLog2 = 8.0f;

struct Barriers {
  uint64_t q_full;
  uint64_t k_full[2], k_empty[2];
  uint64_t v_full[2], v_empty[2];
  uint64_t s_full[2];  // per query tile (A, B)
  uint64_t p_full[2];  // per query tile
  uint64_t o_final;
  uint64_t drain;
  uint32_t tmem_base;
};
static_assert(sizeof(Barriers) <= TB_SDPA2_BARRIER_BYTES, "barrier block overflows its reservation");

constexpr int OFF_Q = 0;  // Q_A, Q_B
constexpr int OFF_K = OFF_Q + 2 * TILE_BYTES;
constexpr int OFF_V = OFF_K + 2 * TILE_BYTES;
constexpr int OFF_BAR = OFF_V + 2 * TILE_BYTES;
static_assert(OFF_BAR + TB_SDPA2_BARRIER_BYTES + 1024 == TB_SDPA2_SMEM_BYTES, "smem layout");
static_assert(TB_SDPA2_SMEM_BYTES <= 232448, "exceeds the 227 KB per-CTA shared memory limit");

constexpr uint32_t kFailProducer = 0x50010000u;
constexpr uint32_t kFailMma = 0x50020000u;
constexpr uint32_t kFailSoftmax = 0x50030000u;

__device__ __forceinline__ float exp2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 2^x on the FMA pipe, for x <= 8 (the lazy-rescale bound): Cody-Waite split
// x = n + f with n = floor(x), f in [0, 1); 2^f from a degree-3 polynomial
// fitted for this kernel (weighted least squares toward minimax relative error
// on [0, 1), p(0) = 1; max relative error 8.6e-5, below the 2^-9 rounding of the
// bf16 P it feeds); 2^n added to the exponent field. Inputs below -127 give 0
// or a denormal, which bf16 P and the row sum treat as zero.
__device__ __forceinline__ float exp2_poly(float x) {
  x = fmaxf(x, -127.0f);
  const float n = floorf(x);
  const float f = x - n;
  float p = fmaf(0.0770670622587204f, f, 0.22764495015144348f);
  p = fmaf(p, f, 0.6951168179512024f);
  p = fmaf(p, f, 1.0f);
  return __int_as_float(__float_as_int(p) + (static_cast<int>(n) << 23));
}

// Makes later uses of registers filled by tcgen05.ld depend on the preceding
// tcgen05.wait::ld (the two asm statements share no operands otherwise).
template <int N>
__device__ __forceinline__ void reg_fence(uint32_t (&r)[N]) {
#pragma unroll
  for (int i = 0; i < N; ++i) asm volatile("" : "+r"(r[i]));
}

// One pass over a 128-column S row in TMEM: applies the causal/tail mask,
// returns the row sum of p = 2^(s*scale_log2 + neg_m) (bf16-packed into
// `packed`, one exponential in four on the FMA pipe) and updates `mraw`, the
// row max of the raw scores. With exps == false only the max is computed.
// `valid` = number of leading columns of this key tile the row may see
// (min(Tk, q+1) - kv0 when causal, Tk - kv0 otherwise; >= BN means all).
__device__ __forceinline__ float softmax_row_pass(uint32_t s_tmem, int valid, float scale_log2, float neg_m, bool exps,
                                                  uint32_t (&packed)[BN / 2], float& mraw) {
  // Four independent max / sum accumulators keep the reductions off one long
  // dependency chain.
  float rs[4] = {0.f, 0.f, 0.f, 0.f};
  float mx[4] = {mraw, -INFINITY, -INFINITY, -INFINITY};
  const bool need_mask = valid < BN;
#pragma unroll
  for (int c = 0; c < BN; c += 32) {
    uint32_t cur[32];
    tmem_ld_x32(s_tmem + c, cur);
    tmem_ld_wait();
    reg_fence(cur);
    const int lim = valid - c;  // columns i >= lim of this chunk are masked
    if (need_mask) {
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (i >= lim) cur[i] = __float_as_uint(-INFINITY);
    }
#pragma unroll
    for (int i = 0; i < 32; ++i) mx[i & 3] = fmaxf(mx[i & 3], __uint_as_float(cur[i]));
    if (exps) {
#pragma unroll
      for (int i = 0; i < 32; i += 2) {
        const float x0 = fmaf(__uint_as_float(cur[i]), scale_log2, neg_m);
        const float x1 = fmaf(__uint_as_float(cur[i + 1]), scale_log2, neg_m);
        float p0 = exp2_approx(x0);
        float p1 = (i & 2) ? exp2_poly(x1) : exp2_approx(x1);
        if (need_mask) {
          if (i >= lim) p0 = 0.f;
          if (i + 1 >= lim) p1 = 0.f;
        }
        rs[(i >> 1) & 3] += p0 + p1;
        packed[(c + i) / 2] = pack_bf16x2(p0, p1);
      }
    }
  }
  mraw = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3]));
  return (rs[0] + rs[1]) + (rs[2] + rs[3]);
}

// P as bf16 pairs into columns [0, 64) of the S region (warp-collective).
__device__ __forceinline__ void store_p(uint32_t s_tmem, const uint32_t (&packed)[BN / 2]) {
#pragma unroll
  for (int c = 0; c < BN / 2; c += 16) tmem_st_x16(s_tmem + c, *reinterpret_cast<const uint32_t(*)[16]>(&packed[c]));
}

// The rare recompute after the reference max moved: exponentials against the
// new max, P written to TMEM here. Kept out of line (with its own P registers)
// so the common path keeps its registers.
__device__ __noinline__ float softmax_row_recompute_store(uint32_t s_tmem, int valid, float scale_log2, float neg_m) {
  uint32_t packed[BN / 2];
  float unused = -INFINITY;
  const float rs = softmax_row_pass(s_tmem, valid, scale_log2, neg_m, true, packed, unused);
  store_p(s_tmem, packed);
  return rs;
}

__device__ __forceinline__ void load_tile(uint8_t* dst, const CUtensorMap* map, uint64_t* bar, int row0, int bh) {
  tma_load_3d(dst, map, bar, 0, row0, bh);
  tma_load_3d(dst + HALF_BYTES, map, bar, 64, row0, bh);
}

__device__ __forceinline__ uint64_t kmajor_desc(uint32_t tile_addr, int k) {
  return sdesc_sw128(tile_addr + (k >> 2) * HALF_BYTES + (k & 3) * 32, 16, 1024);
}

__device__ __forceinline__ uint64_t v_desc(uint32_t tile_addr, int k) {
  return sdesc_sw128(tile_addr + k * 2048, HALF_BYTES, 1024);
}

}  // namespace

// q, k, v, o: [BH, T, 128] bf16 (3-D tensor maps {128, T, BH}, box {64, 128, 1}).
// scale_log2 = log2(e) / sqrt(D).
extern "C" __global__ void __launch_bounds__(THREADS, 1)
    sdpa_fwd_bf16_d128_pair(const __grid_constant__ CUtensorMap tmap_q, const __grid_constant__ CUtensorMap tmap_k,
                            const __grid_constant__ CUtensorMap tmap_v, __nv_bfloat16* __restrict__ out, int Tq,
                            int Tk, int causal, float scale_log2, uint32_t* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Barriers* bars = reinterpret_cast<Barriers*>(smem + OFF_BAR);
  const int warp = warp_id(), lane = lane_id();
  // Flat grid, head-major (a head's K/V stays in L2), heaviest causal pairs first.
  const int num_pairs = (Tq + 2 * BM - 1) / (2 * BM);
  const int bh = blockIdx.x / num_pairs;
  const int pair = num_pairs - 1 - (int)(blockIdx.x % num_pairs);
  const int qt0 = 2 * pair;                     // query tile A; tile B = qt0 + 1
  const int kv_tiles_all = (Tk + BN - 1) / BN;
  // Key tiles each query tile needs.
  const int n_a = causal ? min(kv_tiles_all, qt0 + 1) : kv_tiles_all;
  const int n_b = causal ? min(kv_tiles_all, qt0 + 2) : kv_tiles_all;  // n_b >= n_a

  if (threadIdx.x == 0) {
    mbar_init(&bars->q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars->k_full[i], 1);
      mbar_init(&bars->k_empty[i], 1);
      mbar_init(&bars->v_full[i], 1);
      mbar_init(&bars->v_empty[i], 1);
      mbar_init(&bars->s_full[i], 1);
      mbar_init(&bars->p_full[i], 4);
    }
    mbar_init(&bars->o_final, 1);
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

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      tma_prefetch_desc(&tmap_q);
      tma_prefetch_desc(&tmap_k);
      tma_prefetch_desc(&tmap_v);
      mbar_arrive_expect_tx(&bars->q_full, 2 * TILE_BYTES);
      load_tile(smem + OFF_Q, &tmap_q, &bars->q_full, qt0 * BM, bh);
      load_tile(smem + OFF_Q + TILE_BYTES, &tmap_q, &bars->q_full, (qt0 + 1) * BM, bh);
      uint32_t k_issued[2] = {0, 0}, v_issued[2] = {0, 0};
      bool ok = true;
      for (int j = 0; j < n_b && ok; ++j) {
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
      const uint32_t q_addr[2] = {smem_addr(smem + OFF_Q), smem_addr(smem + OFF_Q + TILE_BYTES)};
      const int n_tiles[2] = {n_a, n_b};
      // j = key tile whose scores are issued this iteration; PV of tile j-1 goes first.
      for (int j = 0; j <= n_b && ok; ++j) {
        const int st = j & 1, pst = (j - 1) & 1;
        const uint32_t ph = (j >> 1) & 1, pph = ((j - 1) >> 1) & 1;
        bool k_ready = false, v_ready = false;
        for (int x = 0; x < 2 && ok; ++x) {
          // O_x += P_x(j-1) V_{j-1}
          if (j >= 1 && j - 1 < n_tiles[x]) {
            if (!v_ready) {
              if (!mbar_wait(&bars->v_full[pst], pph)) {
                report_status(status, kFailMma | 2);
                ok = false;
                break;
              }
              v_ready = true;
            }
            if (!mbar_wait(&bars->p_full[x], (j - 1) & 1)) {
              report_status(status, kFailMma | 3);
              ok = false;
              break;
            }
            tc_fence_after_sync();
            const uint32_t v_addr = smem_addr(smem + OFF_V + pst * TILE_BYTES);
            const uint32_t p_tmem = tmem + x * BN;  // P_x: first 64 columns of S_x (bf16 pairs)
            const uint32_t o_tmem = tmem + (2 + x) * BN;
#pragma unroll
            for (int k = 0; k < BN / 16; ++k)
              umma_bf16_ts(o_tmem, p_tmem + k * 8, v_desc(v_addr, k), IDESC_O, (j - 1 > 0) || (k > 0));
          }
          // S_x(j) = Q_x K_j^T
          if (j < n_tiles[x]) {
            if (!k_ready) {
              if (!mbar_wait(&bars->k_full[st], ph)) {
                report_status(status, kFailMma | 4);
                ok = false;
                break;
              }
              k_ready = true;
              tc_fence_after_sync();
            }
            const uint32_t k_addr = smem_addr(smem + OFF_K + st * TILE_BYTES);
#pragma unroll
            for (int k = 0; k < HD / 16; ++k)
              umma_bf16_ss(tmem + x * BN, kmajor_desc(q_addr[x], k), kmajor_desc(k_addr, k), IDESC_S, k > 0);
            umma_commit(&bars->s_full[x]);
          }
        }
        if (!ok) break;
        if (v_ready) umma_commit(&bars->v_empty[pst]);
        if (k_ready) umma_commit(&bars->k_empty[st]);
      }
      umma_commit(&bars->o_final);
      umma_commit(&bars->drain);
      if (!mbar_wait(&bars->drain, 0)) report_status(status, kFailMma | 5);
    }
  } else {
    // ---------------- softmax warpgroups ----------------
    const int x = (warp >= 6) ? 1 : 0;  // query tile of this softmax group
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t s_tmem = tmem + lane_off + x * BN;
    const uint32_t o_tmem = tmem + lane_off + (2 + x) * BN;
    const int qt = qt0 + x;
    const int q_row = qt * BM + r;
    const int n = x ? n_b : n_a;
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < n; ++j) {
      ok = __all_sync(0xffffffffu, mbar_wait(&bars->s_full[x], j & 1));
      if (!ok) {
        if (lane == 0) report_status(status, kFailSoftmax | 1);
        break;
      }
      tc_fence_after_sync();
      const int kv0 = j * BN;
      const int valid = (causal ? min(Tk, q_row + 1) : Tk) - kv0;  // visible leading keys of this tile
      // Stream the S row in 32-column chunks (the next chunk's TMEM load overlaps
      // this chunk's math), exponentiating against the current reference max.
      // P stays in registers until the row is known not to need a larger max.
      uint32_t packed[BN / 2];
      float mraw = -INFINITY;
      float rs = softmax_row_pass(s_tmem, valid, scale_log2, -m_used, m_used != -INFINITY, packed, mraw);
      const float mx = mraw * scale_log2;  // scale_log2 > 0 commutes with max
      const bool grow = mx > m_used + kLazyRescaleLog2;
      if (__any_sync(0xffffffffu, grow)) {
        const float m_new = grow ? mx : m_used;
        const float alpha = exp2_approx(m_used - m_new);
        l *= alpha;
        if (j > 0) {
          // O_x = sum_{t<j} P_x(t) V_t is complete (S_x(j) was committed after PV_x(j-1)).
#pragma unroll 1
          for (int c = 0; c < HD; c += 16) {
            uint32_t o[16];
            tmem_ld_x16(o_tmem + c, o);
            tmem_ld_wait();
            reg_fence(o);
#pragma unroll
            for (int i = 0; i < 16; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
            tmem_st_x16(o_tmem + c, o);
          }
        }
        m_used = m_new;
        // S is still intact in TMEM (P is written below): recompute against the new max.
        rs = softmax_row_recompute_store(s_tmem, valid, scale_log2, -m_used);
      } else {
        // P_x(j) as bf16 pairs into columns [0, 64) of S_x, where the TS-MMA reads it.
        store_p(s_tmem, packed);
      }
      l += rs;
      tmem_st_wait();
      tc_fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->p_full[x]);
    }
    if (ok) {
      ok = __all_sync(0xffffffffu, mbar_wait(&bars->o_final, 0));
      if (!ok) {
        if (lane == 0) report_status(status, kFailSoftmax | 2);
      } else {
        tc_fence_after_sync();
        const float inv_l = 1.0f / l;
        __nv_bfloat16* dst = out + ((long long)bh * Tq + q_row) * HD;
#pragma unroll 1
        for (int c = 0; c < HD; c += 32) {
          uint32_t o[32];
          tmem_ld_x32(o_tmem + c, o);
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
