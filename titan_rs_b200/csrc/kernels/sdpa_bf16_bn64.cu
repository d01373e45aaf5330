// Causal (or full) attention forward, bf16 in/out, fp32 softmax statistics,
// head dim 128, 64-key tiles, two CTAs per SM.
//
// Semantics: the titan.rs CPU reference (projects/titan-runtime/src/lib.rs:1090-1151),
// O = softmax(Q K^T / sqrt(D)) V over BHTD, plus a causal mask (query i sees keys j <= i,
// top-left aligned when Tq != Tk).
//
// One CTA per (128-row query tile, batch*head); 192 threads; ~97 KB of shared
// memory and 256 TMEM columns per CTA, so two CTAs share each SM and each SM
// runs eight softmax warps against one tensor core.
//   warp 0      TMA producer: the Q tile (two 64-column swizzled boxes) once, then
//               K_j / V_j tiles of 64 keys x 128 dims through 2-stage rings.
//   warp 1      owns 256 TMEM columns: S double buffer (2 x 64 fp32 columns) and O
//               (128 columns). One lane issues, per key tile j,
//                 S_j = Q K_j^T          (SS, M=128 N=64, both K-major)
//                 O  += P_{j-1} V_{j-1}   (TS, M=128 N=128: P read from TMEM, V MN-major)
//               so S_j is computed while the softmax warps work on tile j-1.
//   warps 2..5  one query row per thread (its TMEM lane): the 64 scores of a tile
//               are read from TMEM into registers, masked on the diagonal/tail,
//               reduced with four max and four sum accumulators, exponentiated
//               (one FFMA each; one in four on the FMA pipe, the rest on the MUFU)
//               and written back as bf16 pairs over the first 32 columns of the
//               same S buffer, where the TS-MMA reads P. The reference max moves,
//               and O is rescaled in TMEM, only when the row max grows by more than
//               2^8 (P < 256: the result is the exact online softmax).
// Buffer reuse: S_j overwrites the buffer of tile j-2; the MMA issues it after
// O += P_{j-2} V_{j-2} (in order), which was issued after the softmax released P_{j-2}.
//
// Every wait is bounded; on a timeout the kernel records a code in `status`,
// drains its copies and MMAs, frees TMEM and exits.
#include "attn_math.cuh"
#include "kernel_configs.h"
#include "sm100.cuh"

namespace {

using namespace tb;

constexpr int BM = 128, BN = 64, HD = 128;
constexpr int Q_BYTES = BM * HD * 2;       // 32 KB: two 16 KB boxes of [128 rows x 64 dims]
constexpr int Q_HALF = Q_BYTES / 2;
constexpr int KV_BYTES = BN * HD * 2;      // 16 KB: two 8 KB boxes of [64 keys x 64 dims]
constexpr int KV_HALF = KV_BYTES / 2;
constexpr int THREADS = TB_SDPA3_THREADS;
constexpr int TMEM_COLS = 256;
constexpr uint32_t IDESC_S = idesc_bf16_f32(BM, BN, false);
constexpr uint32_t IDESC_O = idesc_bf16_f32(BM, HD, true);  // B = V, MN-major
constexpr float kLazyRescaleLog2 = 8.0f;

struct Barriers {
  uint64_t q_full;
  uint64_t k_full[2], k_empty[2];
  uint64_t v_full[2], v_empty[2];
  uint64_t s_full[2];
  uint64_t p_full[2];
  uint64_t o_done;
  uint64_t drain;
  uint32_t tmem_base;
};
static_assert(sizeof(Barriers) <= TB_SDPA3_BARRIER_BYTES, "barrier block overflows its reservation");

constexpr int OFF_Q = 0;
constexpr int OFF_K = OFF_Q + Q_BYTES;
constexpr int OFF_V = OFF_K + 2 * KV_BYTES;
constexpr int OFF_BAR = OFF_V + 2 * KV_BYTES;
static_assert(OFF_BAR + TB_SDPA3_BARRIER_BYTES + 1024 == TB_SDPA3_SMEM_BYTES, "smem layout");
static_assert(2 * TB_SDPA3_SMEM_BYTES <= 233472, "two CTAs must fit the SM's shared memory");

constexpr uint32_t kFailProducer = 0x51010000u;
constexpr uint32_t kFailMma = 0x51020000u;
constexpr uint32_t kFailSoftmax = 0x51030000u;

template <int N>
__device__ __forceinline__ void reg_fence(uint32_t (&r)[N]) {
#pragma unroll
  for (int i = 0; i < N; ++i) asm volatile("" : "+r"(r[i]));
}

// Q tile: K-slice k (16 dims) of a [128 x 128] tile stored as two 64-dim boxes.
__device__ __forceinline__ uint64_t q_desc(uint32_t addr, int k) {
  return sdesc_sw128(addr + (k >> 2) * Q_HALF + (k & 3) * 32, 16, 1024);
}
// K tile: K-slice k (16 dims) of a [64 keys x 128 dims] tile stored as two 64-dim boxes.
__device__ __forceinline__ uint64_t k_desc(uint32_t addr, int k) {
  return sdesc_sw128(addr + (k >> 2) * KV_HALF + (k & 3) * 32, 16, 1024);
}
// V tile read MN-major: keys [16k, 16k+16); 8-key atoms 1 KB apart (SBO), dims 64..127 at +8 KB (LBO).
__device__ __forceinline__ uint64_t v_desc(uint32_t addr, int k) { return sdesc_sw128(addr + k * 2048, KV_HALF, 1024); }

}  // namespace

// q, k, v, o: [BH, T, 128] bf16. Q map box {64, 128, 1}; K/V maps box {64, 64, 1}.
// kPolyPairsOf8: score pairs, out of every 8, whose exponentials run on the FMA/ALU
// pipes instead of the MUFU.
template <int kPolyPairsOf8>
__device__ __forceinline__ void sdpa_bn64_body(const CUtensorMap& tmap_q, const CUtensorMap& tmap_k,
                                               const CUtensorMap& tmap_v, __nv_bfloat16* __restrict__ out, int Tq,
                                               int Tk, int causal, float scale_log2, uint32_t* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Barriers* bars = reinterpret_cast<Barriers*>(smem + OFF_BAR);
  const int warp = warp_id(), lane = lane_id();
  // Flat grid, head-major (a head's K/V stays in L2), heaviest causal tiles first.
  const int num_qt = (Tq + BM - 1) / BM;
  const int bh = blockIdx.x / num_qt;
  const int qt = num_qt - 1 - (int)(blockIdx.x % num_qt);
  const int kv_tiles_all = (Tk + BN - 1) / BN;
  const int n = causal ? min(kv_tiles_all, (qt * BM + BM - 1) / BN + 1) : kv_tiles_all;

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
    mbar_init(&bars->o_done, 1);
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
  const uint32_t tmem = bars->tmem_base;
  const uint32_t tmem_o = tmem + 2 * BN;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      tma_prefetch_desc(&tmap_q);
      tma_prefetch_desc(&tmap_k);
      tma_prefetch_desc(&tmap_v);
      mbar_arrive_expect_tx(&bars->q_full, Q_BYTES);
      tma_load_3d(smem + OFF_Q, &tmap_q, &bars->q_full, 0, qt * BM, bh);
      tma_load_3d(smem + OFF_Q + Q_HALF, &tmap_q, &bars->q_full, 64, qt * BM, bh);
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
        uint8_t* kd = smem + OFF_K + st * KV_BYTES;
        mbar_arrive_expect_tx(&bars->k_full[st], KV_BYTES);
        tma_load_3d(kd, &tmap_k, &bars->k_full[st], 0, j * BN, bh);
        tma_load_3d(kd + KV_HALF, &tmap_k, &bars->k_full[st], 64, j * BN, bh);
        ++k_issued[st];
        if (!mbar_wait(&bars->v_empty[st], ph ^ 1)) {
          report_status(status, kFailProducer | 2);
          ok = false;
          break;
        }
        uint8_t* vd = smem + OFF_V + st * KV_BYTES;
        mbar_arrive_expect_tx(&bars->v_full[st], KV_BYTES);
        tma_load_3d(vd, &tmap_v, &bars->v_full[st], 0, j * BN, bh);
        tma_load_3d(vd + KV_HALF, &tmap_v, &bars->v_full[st], 64, j * BN, bh);
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
          if (!mbar_wait(&bars->k_full[st], ph)) {
            report_status(status, kFailMma | 2);
            ok = false;
            break;
          }
          tc_fence_after_sync();
          const uint32_t k_addr = smem_addr(smem + OFF_K + st * KV_BYTES);
#pragma unroll
          for (int k = 0; k < HD / 16; ++k)
            umma_bf16_ss(tmem + st * BN, q_desc(q_addr, k), k_desc(k_addr, k), IDESC_S, k > 0);
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
          const uint32_t v_addr = smem_addr(smem + OFF_V + st * KV_BYTES);
#pragma unroll
          for (int k = 0; k < BN / 16; ++k)
            umma_bf16_ts(tmem_o, tmem + st * BN + k * 8, v_desc(v_addr, k), IDESC_O, (jj > 0) || (k > 0));
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
    const int r = quarter * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const int q_row = qt * BM + r;
    const int row_limit = causal ? min(Tk, q_row + 1) : Tk;  // keys [0, row_limit) are visible
    float m_used = -INFINITY, l = 0.f;
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
      const uint32_t s_tmem = tmem + lane_off + st * BN;
      uint32_t s[BN];
      tmem_ld_x32(s_tmem, *reinterpret_cast<uint32_t(*)[32]>(&s[0]));
      tmem_ld_x32(s_tmem + 32, *reinterpret_cast<uint32_t(*)[32]>(&s[32]));
      tmem_ld_wait();
      reg_fence(s);
      const int valid = row_limit - j * BN;
      if (valid < BN) {
#pragma unroll
        for (int c = 0; c < BN; ++c)
          if (c >= valid) s[c] = __float_as_uint(-INFINITY);
      }
      float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int c = 0; c < BN; c += 8) {
#pragma unroll
        for (int q = 0; q < 4; ++q)
          mx4[q] = fmax3f(mx4[q], __uint_as_float(s[c + 2 * q]), __uint_as_float(s[c + 2 * q + 1]));
      }
      const float mx = fmaxf(fmax3f(mx4[0], mx4[1], mx4[2]), mx4[3]) * scale_log2;
      const bool grow = mx > m_used + kLazyRescaleLog2;
      if (__any_sync(0xffffffffu, grow)) {
        const float m_new = grow ? mx : m_used;
        const float alpha = exp2_mufu(m_used - m_new);  // 0 on the first tile
        l *= alpha;
        if (j > 0) {
          // O holds sum_{t<j} P_t V_t: wait for the last of those MMAs, then rescale in place.
          ok = __all_sync(0xffffffffu, mbar_wait(&bars->o_done, (j - 1) & 1));
          if (!ok) {
            if (lane == 0) report_status(status, kFailSoftmax | 2);
            break;
          }
          tc_fence_after_sync();
          const float2 alpha2 = make_float2(alpha, alpha);
#pragma unroll 1
          for (int c = 0; c < HD; c += 16) {
            uint32_t o[16];
            tmem_ld_x16(tmem_o + lane_off + c, o);
            tmem_ld_wait();
            reg_fence(o);
#pragma unroll
            for (int i = 0; i < 16; i += 2) {
              const float2 v = __fmul2_rn(make_float2(__uint_as_float(o[i]), __uint_as_float(o[i + 1])), alpha2);
              o[i] = __float_as_uint(v.x);
              o[i + 1] = __float_as_uint(v.y);
            }
            tmem_st_x16(tmem_o + lane_off + c, o);
          }
        }
        m_used = m_new;
      }
      // x = s * scale - m per pair (FFMA2); masked scores are -inf and give exactly 0 on both paths.
      const float2 scale2 = make_float2(scale_log2, scale_log2);
      const float2 neg_m2 = make_float2(-m_used, -m_used);
      float2 rs[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
      uint32_t packed[BN / 2];
#pragma unroll
      for (int c = 0; c < BN; c += 2) {
        const float2 x = __ffma2_rn(make_float2(__uint_as_float(s[c]), __uint_as_float(s[c + 1])), scale2, neg_m2);
        const float2 p = ((c >> 1) & 7) < kPolyPairsOf8 ? exp2_poly2(x) : make_float2(exp2_mufu(x.x), exp2_mufu(x.y));
        rs[(c >> 1) & 3] = __fadd2_rn(rs[(c >> 1) & 3], p);
        packed[c / 2] = pack_bf16x2(p.x, p.y);
      }
      const float2 rsum = __fadd2_rn(__fadd2_rn(rs[0], rs[1]), __fadd2_rn(rs[2], rs[3]));
      l += rsum.x + rsum.y;
      // P_j as bf16 pairs into the first 32 columns of its S buffer, where the TS-MMA reads it.
      tmem_st_x16(s_tmem, *reinterpret_cast<const uint32_t(*)[16]>(&packed[0]));
      tmem_st_x16(s_tmem + 16, *reinterpret_cast<const uint32_t(*)[16]>(&packed[16]));
      tmem_st_wait();
      tc_fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->p_full[st]);
    }
    if (ok) {
      // ---------------- epilogue: O / l -> bf16 ----------------
      ok = __all_sync(0xffffffffu, mbar_wait(&bars->o_done, (n - 1) & 1));
      if (!ok) {
        if (lane == 0) report_status(status, kFailSoftmax | 3);
      } else {
        tc_fence_after_sync();
        const float inv_l = 1.0f / l;
        __nv_bfloat16* dst = out + ((long long)bh * Tq + q_row) * HD;
#pragma unroll 1
        for (int c = 0; c < HD; c += 32) {
          uint32_t o[32];
          tmem_ld_x32(tmem_o + lane_off + c, o);
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
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

#define TB_SDPA_BN64_ENTRY(name, poly)                                                                              \
  extern "C" __global__ void __launch_bounds__(THREADS, 2)                                                       \
      name(const __grid_constant__ CUtensorMap tmap_q, const __grid_constant__ CUtensorMap tmap_k,             \
           const __grid_constant__ CUtensorMap tmap_v, __nv_bfloat16* __restrict__ out, int Tq, int Tk, int causal, \
           float scale_log2, uint32_t* status) {                                                                 \
    sdpa_bn64_body<poly>(tmap_q, tmap_k, tmap_v, out, Tq, Tk, causal, scale_log2, status);                       \
  }

// Two score pairs in every eight take the FMA/ALU exponential (measured fastest of
// 2, 3 and 4 on the C4 workload).
TB_SDPA_BN64_ENTRY(sdpa_fwd_bf16_d128_bn64, 2)
