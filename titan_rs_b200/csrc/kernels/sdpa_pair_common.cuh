// Pieces shared by the two-query-tile attention kernels (sdpa_bf16_pair.cu, one CTA
// per query-tile pair; sdpa_bf16_persist.cu, persistent CTAs): tile geometry, the
// shared-memory descriptors, the MMA issue of S = Q K^T and O += P V, and the
// per-key-tile softmax step of one query row.
#pragma once

#include "attn_math.cuh"
#include "sm100.cuh"

namespace tb {
namespace sdpa2 {

constexpr int BM = 128, BN = 128, HD = 128;
constexpr int TILE_BYTES = 128 * HD * 2;  // 32 KB
constexpr int HALF_BYTES = TILE_BYTES / 2;
constexpr uint32_t IDESC_S = idesc_bf16_f32(BM, BN, false);
constexpr uint32_t IDESC_O = idesc_bf16_f32(BM, HD, true);  // B = V, MN-major
// The reference max of a row moves (and O is rescaled) only when a key tile's row
// max exceeds it by more than 2^8, so P <= 256 and the result is the exact online
// softmax with the rescale skipped on most tiles.
constexpr float kLazyRescaleLog2 = 8.0f;

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

// L2 prefetch of the tile load_tile would read (two 64-column boxes).
__device__ __forceinline__ void prefetch_tile(const CUtensorMap* map, int row0, int bh) {
  tma_prefetch_l2_3d(map, 0, row0, bh);
  tma_prefetch_l2_3d(map, 64, row0, bh);
}

// Key tiles the producer asks L2 for ahead of their loads. The ring holds two stages,
// so a tile's load can start only about one key-tile period before its MMAs; the CTA
// that leads its head group would meet DRAM latency there without the prefetch. One
// tile ahead measured best (1064-1066 TFLOP/s at C4 against 1058-1061 for two and
// 1041-1050 for four).
constexpr int kPrefetchAhead = 1;

// Work order of the (batch*head, query-tile pair) items: groups of kHeadGroup heads
// (their K and V, 2 MB a head at T = 4096, stay in L2 while the group runs) and, inside
// a group, pair-major from the heaviest causal pair (the last one) down, so the long
// pairs of every head start first and the short ones fill in at the end.
constexpr int kHeadGroup = 16;
struct PairSchedule {
  int bh_count, num_pairs;
  __device__ __forceinline__ void item(int u, int& bh, int& pair) const {
    const int per_group = kHeadGroup * num_pairs;
    const int g = u / per_group;
    const int r = u - g * per_group;
    const int heads = min(kHeadGroup, bh_count - g * kHeadGroup);
    pair = num_pairs - 1 - r / heads;
    bh = g * kHeadGroup + r % heads;
  }
};

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

// One key tile of one query row's online softmax (the caller waited for S): reads
// the row's 128 scores from TMEM into registers once, takes the row max, moves the
// reference max m_used (rescaling l and, when `rescale_ok`, O) only when the max grew
// by more than 2^kLazyRescaleLog2, and writes P as bf16 pairs over columns [0, 64) of
// the S region, where the TS-MMA reads it (every score is in registers by then, so the
// overwritten columns are free): keys [0, 64) first, announced on `p_half` so the MMA
// lane issues their half of PV while keys [64, 128) are done (`p_full`). `valid` =
// visible leading keys of the tile (causal mask and Tk), < 128 only on the diagonal
// or the last tile.
template <int kPolyPairsOf8>
__device__ __forceinline__ void softmax_tile(uint32_t s_tmem, uint32_t o_tmem, int valid, bool rescale_ok,
                                             float scale_log2, float& m_used, float& l, uint64_t* p_half,
                                             uint64_t* p_full) {
  const int lane = lane_id();
  const bool need_mask = valid < BN;
  uint32_t c0[32], c1[32], c2[32], c3[32];
  tmem_ld_x32(s_tmem, c0);
  tmem_ld_x32(s_tmem + 32, c1);
  tmem_ld_x32(s_tmem + 64, c2);
  tmem_ld_x32(s_tmem + 96, c3);
  tmem_ld_wait();
  reg_fence(c0);
  reg_fence(c1);
  reg_fence(c2);
  reg_fence(c3);
  float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
  mask_max_chunk(c0, valid, need_mask, mx4);
  mask_max_chunk(c1, valid - 32, need_mask, mx4);
  mask_max_chunk(c2, valid - 64, need_mask, mx4);
  mask_max_chunk(c3, valid - 96, need_mask, mx4);
  const float mx = fmaxf(fmax3f(mx4[0], mx4[1], mx4[2]), mx4[3]) * scale_log2;  // scale_log2 > 0 commutes with max
  const bool grow = mx > m_used + kLazyRescaleLog2;
  if (__any_sync(0xffffffffu, grow)) {
    const float m_new = grow ? mx : m_used;
    const float alpha = exp2_mufu(m_used - m_new);  // 0 on a row's first tile
    l *= alpha;
    if (rescale_ok) rescale_o(o_tmem, alpha);
    m_used = m_new;
  }
  const float2 scale2 = make_float2(scale_log2, scale_log2);
  const float2 neg_m2 = make_float2(-m_used, -m_used);
  float2 rs4[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
  exp_chunk_store<kPolyPairsOf8>(c0, scale2, neg_m2, rs4, s_tmem);
  exp_chunk_store<kPolyPairsOf8>(c1, scale2, neg_m2, rs4, s_tmem + 16);
  tmem_st_wait();
  tc_fence_before_sync();
  __syncwarp();
  if (lane == 0) mbar_arrive(p_half);
  exp_chunk_store<kPolyPairsOf8>(c2, scale2, neg_m2, rs4, s_tmem + 32);
  exp_chunk_store<kPolyPairsOf8>(c3, scale2, neg_m2, rs4, s_tmem + 48);
  const float2 rsum = __fadd2_rn(__fadd2_rn(rs4[0], rs4[1]), __fadd2_rn(rs4[2], rs4[3]));
  l += rsum.x + rsum.y;
  tmem_st_wait();
  tc_fence_before_sync();
  __syncwarp();
  if (lane == 0) mbar_arrive(p_full);
}

// The finished row: O / l in bf16, 128 columns from TMEM to global memory (16-byte
// stores), skipped for rows past Tq.
__device__ __forceinline__ void store_row(uint32_t o_tmem, float l, __nv_bfloat16* dst, bool in_range) {
  const float inv_l = 1.0f / l;
#pragma unroll 1
  for (int c = 0; c < HD; c += 32) {
    uint32_t o[32];
    tmem_ld_x32(o_tmem + c, o);
    tmem_ld_wait();
    reg_fence(o);
    if (in_range) {
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

}  // namespace sdpa2
}  // namespace tb
