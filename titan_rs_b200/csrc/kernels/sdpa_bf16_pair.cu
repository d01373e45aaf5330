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
//                  PV_A(j-1) (two halves) then S_A(j), PV_B(j-1) then S_B(j)
//                so the tensor core works on one tile's products while the other
//                tile's warpgroup exponentiates.
//                  S_X(j)  = Q_X K_j^T   (SS: both operands K-major in shared memory)
//                  O_X    += P_X(j) V_j  (TS: P read from TMEM, V MN-major in shared memory)
//   warps 2..5   softmax group for tile A, warps 6..9 for tile B (each group covers the
//                four TMEM lane quarters, since warp w reaches lanes 32*(w%4)..): one query row per
//                thread (its TMEM lane). Per key tile, pass 1 reads the 128 scores
//                from TMEM in 32-column chunks for the row max; pass 2 exponentiates
//                against the reference max (packed FFMA2 for s*scale - m; a share of
//                the exponentials on the FMA/ALU pipes, the rest on the MUFU) and
//                writes P as bf16 pairs over the first 64 columns of the same S
//                region, where the TS-MMA reads it: keys [0, 64) first, announced on
//                p_half so the MMA lane issues their half of PV while the warps finish
//                keys [64, 128) (p_full). The reference max moves, and O is rescaled
//                in TMEM, only when the row max grows by more than 2^8, so P stays
//                below 256 and the result is the exact online softmax.
// Ordering: tcgen05.commit arrives once ALL earlier MMAs of the issuing thread are
// done, so "S_X(j) ready" also means PV_X(j-1) finished reading P_X and writing O_X:
// the softmax warps may then overwrite S/P and rescale O without further waits.
//
// Every wait is bounded; on a timeout the kernel records a code in `status`,
// drains its copies and MMAs, frees TMEM and exits.
#include "attn_math.cuh"
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
// The reference max of a row moves (and O is rescaled) only when a key tile's row
// max exceeds it by more than 2^8, so P <= 256 and the result is the exact online
// softmax with the rescale skipped on most tiles.
constexpr float kLazyRescaleLog2 = 8.0f;

struct Barriers {
  uint64_t q_full;
  uint64_t k_full[2], k_empty[2];
  uint64_t v_full[2], v_empty[2];
  uint64_t s_full[2];  // per query tile (A, B)
  uint64_t p_half[2];  // per query tile: P of keys [0, 64) is in TMEM
  uint64_t p_full[2];  // per query tile: P of keys [64, 128) is in TMEM
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

// Makes later uses of registers filled by tcgen05.ld depend on the preceding
// tcgen05.wait::ld (the two asm statements share no operands otherwise).
template <int N>
__device__ __forceinline__ void reg_fence(uint32_t (&r)[N]) {
#pragma unroll
  for (int i = 0; i < N; ++i) asm volatile("" : "+r"(r[i]));
}

// Sets columns >= lim of a 32-column S chunk to -inf (its exponential is exactly 0
// on both exponential paths).
__device__ __forceinline__ void mask_chunk(uint32_t (&cur)[32], int lim) {
#pragma unroll
  for (int i = 0; i < 32; ++i)
    if (i >= lim) cur[i] = __float_as_uint(-INFINITY);
}

// Masks the chunk when the tile needs it and folds it into four max accumulators.
__device__ __forceinline__ void mask_max_chunk(uint32_t (&cur)[32], int lim, bool need_mask, float (&mx)[4]) {
  if (need_mask) mask_chunk(cur, lim);
#pragma unroll
  for (int i = 0; i < 32; i += 8) {
#pragma unroll
    for (int q = 0; q < 4; ++q) mx[q] = fmax3f(mx[q], __uint_as_float(cur[i + 2 * q]), __uint_as_float(cur[i + 2 * q + 1]));
  }
}

// p = 2^(s * scale_log2 - m) for one 32-column S chunk (kPolyPairsOf8 pairs in
// every 8 on the FMA/ALU pipes, the rest on the MUFU), added to the four packed
// row-sum accumulators and stored as 16 columns of bf16 pairs at p_tmem.
template <int kPolyPairsOf8>
__device__ __forceinline__ void exp_chunk_store(const uint32_t (&cur)[32], float2 scale2, float2 neg_m2, float2 (&rs)[4],
                                                uint32_t p_tmem) {
  uint32_t packed[16];
#pragma unroll
  for (int i = 0; i < 32; i += 2) {
    const float2 x = __ffma2_rn(make_float2(__uint_as_float(cur[i]), __uint_as_float(cur[i + 1])), scale2, neg_m2);
    const float2 p = ((i >> 1) & 7) < kPolyPairsOf8 ? exp2_poly2(x) : make_float2(exp2_mufu(x.x), exp2_mufu(x.y));
    rs[(i >> 1) & 3] = __fadd2_rn(rs[(i >> 1) & 3], p);
    packed[i / 2] = pack_bf16x2(p.x, p.y);
  }
  tmem_st_x16(p_tmem, packed);
}

// Rescale of O by alpha for one row: 128 fp32 columns in TMEM.
__device__ __forceinline__ void rescale_o(uint32_t o_tmem, float alpha) {
#pragma unroll 1
  for (int c = 0; c < HD; c += 16) {
    uint32_t o[16];
    tmem_ld_x16(o_tmem + c, o);
    tmem_ld_wait();
    reg_fence(o);
#pragma unroll
    for (int i = 0; i < 16; i += 2) {
      const float2 v =
          __fmul2_rn(make_float2(__uint_as_float(o[i]), __uint_as_float(o[i + 1])), make_float2(alpha, alpha));
      o[i] = __float_as_uint(v.x);
      o[i + 1] = __float_as_uint(v.y);
    }
    tmem_st_x16(o_tmem + c, o);
  }
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

// Moves a shared-memory descriptor's start address by `units` 16-byte units. The
// start-address field is the descriptor's low 14 bits and every address here is
// below 256 KB, so a 32-bit add on the low word never carries out of the field.
__device__ __forceinline__ uint64_t desc_add(uint64_t d, uint32_t units) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "r"(static_cast<uint32_t>(d) + units), "r"(static_cast<uint32_t>(d >> 32)));
  return r;
}

// O (+)= P V for keys [64 h, 64 h + 64) of a 128-key tile: P from TMEM (bf16 pairs,
// 8 columns per 16 keys), V MN-major in shared memory (16 keys = 2 KB per slice).
__device__ __forceinline__ void issue_pv_half(uint32_t o_tmem, uint32_t p_tmem, uint64_t vd, int h, bool accumulate) {
#pragma unroll
  for (int k = 4 * h; k < 4 * h + 4; ++k)
    umma_bf16_ts(o_tmem, p_tmem + k * 8, desc_add(vd, k * (2048 >> 4)), IDESC_O, (k > 0 || accumulate) ? 1u : 0u);
}

// S = Q K^T for one 128-key tile: both operands K-major, 16 dims per slice (two
// 64-dim boxes of HALF_BYTES; 32 bytes per slice inside a box).
__device__ __forceinline__ void issue_s(uint32_t s_tmem, uint64_t qd, uint64_t kd) {
#pragma unroll
  for (int k = 0; k < HD / 16; ++k) {
    const uint32_t off = (k >> 2) * (HALF_BYTES >> 4) + (k & 3) * 2;
    umma_bf16_ss(s_tmem, desc_add(qd, off), desc_add(kd, off), IDESC_S, k > 0 ? 1u : 0u);
  }
}

}  // namespace

// q, k, v, o: [BH, T, 128] bf16 (3-D tensor maps {128, T, BH}, box {64, 128, 1}).
// scale_log2 = log2(e) / sqrt(D).
template <int kPolyPairsOf8>
__device__ __forceinline__ void sdpa_pair_body(const CUtensorMap& tmap_q, const CUtensorMap& tmap_k,
                                               const CUtensorMap& tmap_v, __nv_bfloat16* __restrict__ out, int Tq,
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
      mbar_init(&bars->p_half[i], 4);
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
      // One lane issues every MMA, so its instruction stream is kept short: all
      // descriptors are formed here once, and each MMA only adds a compile-time
      // K-slice offset to the low word of one of them.
      bool ok = mbar_wait(&bars->q_full, 0);
      if (!ok) report_status(status, kFailMma | 1);
      const uint64_t qd_a = kmajor_desc(smem_addr(smem + OFF_Q), 0);
      const uint64_t qd_b = kmajor_desc(smem_addr(smem + OFF_Q + TILE_BYTES), 0);
      const uint64_t kd0 = kmajor_desc(smem_addr(smem + OFF_K), 0);
      const uint64_t vd0 = v_desc(smem_addr(smem + OFF_V), 0);
      // j = key tile whose scores are issued this iteration; PV of tile j-1 goes first.
      for (int j = 0; j <= n_b && ok; ++j) {
        const int st = j & 1, pst = (j - 1) & 1;
        const uint32_t ph = (j >> 1) & 1, pph = ((j - 1) >> 1) & 1;
        const uint64_t kd = desc_add(kd0, st * (TILE_BYTES >> 4));
        const uint64_t vd = desc_add(vd0, pst * (TILE_BYTES >> 4));
        const bool pv_a = j >= 1 && j - 1 < n_a, pv_b = j >= 1 && j - 1 < n_b;  // n_a <= n_b
        const bool s_a = j < n_a, s_b = j < n_b;
        if (pv_b && !mbar_wait(&bars->v_full[pst], pph)) {
          report_status(status, kFailMma | 2);
          ok = false;
          break;
        }
        // K_j was loaded long before P_A(j-1) is ready: wait for it first, so that
        // S_A(j) issues right behind PV_A(j-1).
        const bool k_ready = s_b;
        if (k_ready && !mbar_wait(&bars->k_full[st], ph)) {
          report_status(status, kFailMma | 4);
          ok = false;
          break;
        }
        // Tile A: O_A += P_A(j-1) V_{j-1}, then S_A(j) = Q_A K_j^T; then the same for tile B.
        for (int x = 0; x < 2; ++x) {
          if (x ? pv_b : pv_a) {
            // The first half of P_x(j-1) arrives while its warps still exponentiate the second.
            if (!mbar_wait(&bars->p_half[x], (j - 1) & 1)) {
              report_status(status, kFailMma | 3);
              ok = false;
              break;
            }
            tc_fence_after_sync();
            issue_pv_half(tmem + (2 + x) * BN, tmem + x * BN, vd, 0, j - 1 > 0);
            if (!mbar_wait(&bars->p_full[x], (j - 1) & 1)) {
              report_status(status, kFailMma | 6);
              ok = false;
              break;
            }
            tc_fence_after_sync();
            issue_pv_half(tmem + (2 + x) * BN, tmem + x * BN, vd, 1, true);
          }
          if (x ? s_b : s_a) {
            tc_fence_after_sync();
            issue_s(tmem + x * BN, x ? qd_b : qd_a, kd);
            umma_commit(&bars->s_full[x]);
          }
        }
        if (!ok) break;
        if (pv_b) umma_commit(&bars->v_empty[pst]);
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
    const float2 scale2 = make_float2(scale_log2, scale_log2);
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < n; ++j) {
      ok = __all_sync(0xffffffffu, mbar_wait(&bars->s_full[x], j & 1));
      if (!ok) {
        if (lane == 0) report_status(status, kFailSoftmax | 1);
        break;
      }
      tc_fence_after_sync();
      const int valid = (causal ? min(Tk, q_row + 1) : Tk) - j * BN;  // visible leading keys of this tile
      const bool need_mask = valid < BN;
      // Pass 1: the row max over all 128 columns; chunks 0 and 1 stay in registers.
      uint32_t ca[32], cb[32], ct[32];
      tmem_ld_x32(s_tmem, ca);
      tmem_ld_x32(s_tmem + 32, cb);
      tmem_ld_x32(s_tmem + 64, ct);
      tmem_ld_wait();
      reg_fence(ca);
      reg_fence(cb);
      reg_fence(ct);
      float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
      mask_max_chunk(ca, valid, need_mask, mx4);
      mask_max_chunk(cb, valid - 32, need_mask, mx4);
      mask_max_chunk(ct, valid - 64, need_mask, mx4);
      tmem_ld_x32(s_tmem + 96, ct);
      tmem_ld_wait();
      reg_fence(ct);
      mask_max_chunk(ct, valid - 96, need_mask, mx4);
      const float mx = fmaxf(fmax3f(mx4[0], mx4[1], mx4[2]), mx4[3]) * scale_log2;  // scale_log2 > 0 commutes with max
      const bool grow = mx > m_used + kLazyRescaleLog2;
      if (__any_sync(0xffffffffu, grow)) {
        const float m_new = grow ? mx : m_used;
        const float alpha = exp2_mufu(m_used - m_new);  // 0 on the first tile
        l *= alpha;
        // O_x = sum_{t<j} P_x(t) V_t is complete (S_x(j) was committed after PV_x(j-1)),
        // and no PV of this tile starts before p_half below.
        if (j > 0) rescale_o(o_tmem, alpha);
        m_used = m_new;
      }
      // Pass 2: P_x(j) as bf16 pairs over columns [0, 64) of S_x, where the TS-MMA reads
      // it. Keys [0, 64) first (S chunks 0 and 1, in registers; their P covers columns
      // [0, 32), which pass 1 has read), then p_half lets the MMA warp start on them
      // while keys [64, 128) (columns the P never touches) are reloaded and done.
      const float2 neg_m2 = make_float2(-m_used, -m_used);
      float2 rs4[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
      tmem_ld_x32(s_tmem + 64, ct);
      exp_chunk_store<kPolyPairsOf8>(ca, scale2, neg_m2, rs4, s_tmem);
      exp_chunk_store<kPolyPairsOf8>(cb, scale2, neg_m2, rs4, s_tmem + 16);
      tmem_st_wait();
      tc_fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->p_half[x]);
      tmem_ld_x32(s_tmem + 96, ca);
      tmem_ld_wait();
      reg_fence(ct);
      reg_fence(ca);
      if (need_mask) {
        mask_chunk(ct, valid - 64);
        mask_chunk(ca, valid - 96);
      }
      exp_chunk_store<kPolyPairsOf8>(ct, scale2, neg_m2, rs4, s_tmem + 32);
      exp_chunk_store<kPolyPairsOf8>(ca, scale2, neg_m2, rs4, s_tmem + 48);
      const float2 rsum = __fadd2_rn(__fadd2_rn(rs4[0], rs4[1]), __fadd2_rn(rs4[2], rs4[3]));
      l += rsum.x + rsum.y;
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
          reg_fence(o);
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

#define TB_SDPA_PAIR_ENTRY(name, poly)                                                                              \
  extern "C" __global__ void __launch_bounds__(THREADS, 1)                                                       \
      name(const __grid_constant__ CUtensorMap tmap_q, const __grid_constant__ CUtensorMap tmap_k,             \
           const __grid_constant__ CUtensorMap tmap_v, __nv_bfloat16* __restrict__ out, int Tq, int Tk, int causal, \
           float scale_log2, uint32_t* status) {                                                                 \
    sdpa_pair_body<poly>(tmap_q, tmap_k, tmap_v, out, Tq, Tk, causal, scale_log2, status);                       \
  }

// Two score pairs in every eight take the FMA/ALU exponential (measured fastest of
// 1, 2 and 3 on the C4 workload).
TB_SDPA_PAIR_ENTRY(sdpa_fwd_bf16_d128_pair, 2)
