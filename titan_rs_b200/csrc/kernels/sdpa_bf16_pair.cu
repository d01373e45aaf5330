// Causal (or full) attention forward, bf16 in/out, fp32 softmax statistics,
// head dim 128: two query tiles per CTA with ping-pong softmax warpgroups.
//
// Semantics: the titan.rs CPU reference (projects/titan-runtime/src/lib.rs:1090-1151),
// O = softmax(Q K^T / sqrt(D)) V over BHTD, plus a causal mask (query i sees keys j <= i,
// top-left aligned when Tq != Tk).
//
// One CTA per (pair of 128-row query tiles A = 2i, B = 2i+1, batch*head); 384 threads in
// three warpgroups (control: warps 0-3, softmax A: 4-7, softmax B: 8-11):
//   warp 0       TMA producer: Q_A and Q_B once, then K_j and V_{j-1} (128 keys x 128
//                dims, two 64-column 128-byte-swizzled boxes each) into stage j & 1 of a
//                2-stage ring (one full and one empty barrier per stage).
//   warp 1       owns all 512 TMEM columns: S_A | S_B | O_A | O_B (128 fp32 columns each).
//                One lane issues, per key tile j,
//                  PV_A(j-1) (two halves) then S_A(j), PV_B(j-1) then S_B(j)
//                so the tensor core works on one tile's products while the other
//                tile's warpgroup exponentiates.
//                  S_X(j)  = Q_X K_j^T   (SS: both operands K-major in shared memory)
//                  O_X    += P_X(j) V_j  (TS: P read from TMEM, V MN-major in shared memory)
//   warps 2, 3   idle (they complete the control warpgroup, which gives its registers
//                to the softmax warpgroups: 56 each against 216).
//   warps 4..7   softmax group for tile A, warps 8..11 for tile B (each group covers the
//                four TMEM lane quarters, since warp w reaches lanes 32*(w%4)..): one query row per
//                thread (its TMEM lane). Per key tile the thread reads its row's 128
//                scores from TMEM into registers once; pass 1 takes the row max;
//                pass 2 exponentiates
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
#include "kernel_configs.h"
#include "sdpa_pair_common.cuh"

namespace {

using namespace tb;
using namespace tb::sdpa2;

struct Barriers {
  uint64_t q_full;
  uint64_t kv_full[2], kv_empty[2];  // stage j & 1 holds K_j and V_{j-1}
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
  // Flat grid in the shared work order (groups of heads, heaviest causal pairs first;
  // the block scheduler hands the next block to the first free SM).
  const int num_pairs = (Tq + 2 * BM - 1) / (2 * BM);
  int bh, pair;
  PairSchedule{(int)(gridDim.x / num_pairs), num_pairs}.item((int)blockIdx.x, bh, pair);
  const int qt0 = 2 * pair;                     // query tile A; tile B = qt0 + 1
  const int kv_tiles_all = (Tk + BN - 1) / BN;
  // Key tiles each query tile needs.
  const int n_a = causal ? min(kv_tiles_all, qt0 + 1) : kv_tiles_all;
  const int n_b = causal ? min(kv_tiles_all, qt0 + 2) : kv_tiles_all;  // n_b >= n_a

  if (threadIdx.x == 0) {
    mbar_init(&bars->q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars->kv_full[i], 1);
      mbar_init(&bars->kv_empty[i], 1);
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
  static_assert(TB_SDPA2_PAIR_THREADS == 384, "three warpgroups");
  static_assert(128 * TB_SDPA2_PAIR_CONTROL_REGS + 256 * TB_SDPA2_PAIR_SOFTMAX_REGS <=
                    TB_SDPA2_PAIR_THREADS * TB_SDPA2_PAIR_LAUNCH_REGS,
                "the warpgroups' registers exceed the launch allocation");
  // Each role runs inside the branch of its register count, so the compiler gives the
  // softmax code 216 registers and the control code 56.
  if (warp < 4) {
    setmaxnreg_dec<TB_SDPA2_PAIR_CONTROL_REGS>();
    if (warp == 0) {
      if (lane == 0) {
        // ---------------- TMA producer ----------------
        tma_prefetch_desc(&tmap_q);
        tma_prefetch_desc(&tmap_k);
        tma_prefetch_desc(&tmap_v);
        mbar_arrive_expect_tx(&bars->q_full, 2 * TILE_BYTES);
        load_tile(smem + OFF_Q, &tmap_q, &bars->q_full, qt0 * BM, bh);
        load_tile(smem + OFF_Q + TILE_BYTES, &tmap_q, &bars->q_full, (qt0 + 1) * BM, bh);
        // Stage j & 1 of the ring holds K_j and V_{j-1}: the two tiles the MMA lane's
        // iteration j reads, so it waits once and releases once per iteration.
        uint32_t issued[2] = {0, 0};
        bool ok = true;
        for (int j = 0; j < kPrefetchAhead && j < n_b; ++j) {
          prefetch_tile(&tmap_k, j * BN, bh);
          prefetch_tile(&tmap_v, j * BN, bh);
        }
        for (int j = 0; j <= n_b && ok; ++j) {
          if (j + kPrefetchAhead < n_b) {
            prefetch_tile(&tmap_k, (j + kPrefetchAhead) * BN, bh);
            prefetch_tile(&tmap_v, (j + kPrefetchAhead) * BN, bh);
          }
          const int st = j & 1;
          const uint32_t ph = (j >> 1) & 1;
          if (!mbar_wait(&bars->kv_empty[st], ph ^ 1)) {
            report_status(status, kFailProducer | 1);
            ok = false;
            break;
          }
          const bool has_k = j < n_b, has_v = j >= 1;
          mbar_arrive_expect_tx(&bars->kv_full[st], (has_k ? TILE_BYTES : 0) + (has_v ? TILE_BYTES : 0));
          if (has_k) load_tile(smem + OFF_K + st * TILE_BYTES, &tmap_k, &bars->kv_full[st], j * BN, bh);
          if (has_v) load_tile(smem + OFF_V + st * TILE_BYTES, &tmap_v, &bars->kv_full[st], (j - 1) * BN, bh);
          ++issued[st];
        }
        if (!ok) {
          if (!mbar_wait(&bars->q_full, 0)) report_status(status, kFailProducer | 3);
          for (int s = 0; s < 2; ++s)
            if (issued[s] && !mbar_wait(&bars->kv_full[s], (issued[s] - 1) & 1))
              report_status(status, kFailProducer | 4);
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
          const int st = j & 1;
          const uint64_t kd = desc_add(kd0, st * (TILE_BYTES >> 4));
          const uint64_t vd = desc_add(vd0, st * (TILE_BYTES >> 4));
          const bool pv_a = j >= 1 && j - 1 < n_a, pv_b = j >= 1;  // n_a <= n_b; j <= n_b
          const bool s_a = j < n_a, s_b = j < n_b;
          if (!mbar_wait(&bars->kv_full[st], (j >> 1) & 1)) {
            report_status(status, kFailMma | 2);
            ok = false;
            break;
          }
          // Tile A: O_A += P_A(j-1) V_{j-1}, then S_A(j) = Q_A K_j^T; then the same for tile B.
          // S_x(j) overwrites P_x(j-1) after the PV that reads it (the tensor core runs
          // them in order), and its softmax warps read S_x(j-1) before announcing p_full.
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
              issue_s(tmem + x * BN, x ? qd_b : qd_a, kd);
              umma_commit(&bars->s_full[x]);
            }
          }
          if (!ok) break;
          umma_commit(&bars->kv_empty[st]);  // after this iteration's MMAs have read K_j and V_{j-1}
        }
        umma_commit(&bars->o_final);
        umma_commit(&bars->drain);
        if (!mbar_wait(&bars->drain, 0)) report_status(status, kFailMma | 5);
      }
    }
  } else {
    setmaxnreg_inc<TB_SDPA2_PAIR_SOFTMAX_REGS>();
    // ---------------- softmax warpgroups ----------------
    const int x = (warp >= 8) ? 1 : 0;  // query tile of this softmax group
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
      // O_x = sum_{t<j} P_x(t) V_t is complete (S_x(j) was committed after PV_x(j-1)), and
      // no PV of this tile starts before p_half: the rescale may touch O from j = 1 on.
      const int valid = (causal ? min(Tk, q_row + 1) : Tk) - j * BN;  // visible leading keys of this tile
      softmax_tile<kPolyPairsOf8>(s_tmem, o_tmem, valid, j > 0, scale_log2, m_used, l, &bars->p_half[x],
                                  &bars->p_full[x]);
    }
    if (ok) {
      ok = __all_sync(0xffffffffu, mbar_wait(&bars->o_final, 0));
      if (!ok) {
        if (lane == 0) report_status(status, kFailSoftmax | 2);
      } else {
        tc_fence_after_sync();
        store_row(o_tmem, l, out + ((long long)bh * Tq + q_row) * HD, q_row < Tq);
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

// One CTA per SM: 12 warps launched at 168 registers a thread (three on each SM
// sub-partition); the softmax warps then hold 216, enough for a row's 128 scores in
// registers beside the exponential's temporaries.
#define TB_SDPA_PAIR_ENTRY(name, poly)                                                                              \
  extern "C" __global__ void __launch_bounds__(TB_SDPA2_PAIR_THREADS, 1)                                         \
      name(const __grid_constant__ CUtensorMap tmap_q, const __grid_constant__ CUtensorMap tmap_k,             \
           const __grid_constant__ CUtensorMap tmap_v, __nv_bfloat16* __restrict__ out, int Tq, int Tk, int causal, \
           float scale_log2, uint32_t* status) {                                                                 \
    sdpa_pair_body<poly>(tmap_q, tmap_k, tmap_v, out, Tq, Tk, causal, scale_log2, status);                       \
  }

// Every exponential on the MUFU: measured fastest of 0 to 3 FMA/ALU pairs in 8 on the C4
// workload once the scores stay in registers (1014 against 1002, 985 and 970 TFLOP/s
// for an isolated launch); the polynomial's extra instructions take issue slots from the
// MMA lane, which shares its sub-partition with two softmax warps.
TB_SDPA_PAIR_ENTRY(sdpa_fwd_bf16_d128_pair, 0)
