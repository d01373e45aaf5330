// Causal (or full) attention forward, bf16 in/out, fp32 softmax statistics, head dim
// 128: the two-query-tile pipeline of sdpa_bf16_pair.cu run by persistent CTAs.
//
// Semantics: the titan.rs CPU reference (projects/titan-runtime/src/lib.rs:1090-1151),
// O = softmax(Q K^T / sqrt(D)) V over BHTD, plus a causal mask (query i sees keys j <= i,
// top-left aligned when Tq != Tk).
//
// One CTA per SM takes work items (batch*head, pair of 128-row query tiles A = 2i,
// B = 2i+1) from one list: CTA c starts with item c, and each later item comes from a
// global counter (atomicAdd, zeroed before the launch), so a CTA that finishes early
// takes the next item and the SMs end together. The list holds groups of 16 heads
// (their K and V, 2 MB a head at T = 4096, stay in L2 while the group runs) and, inside
// a group, every head's heaviest causal pair first. The producer thread draws the item
// numbers and passes them to the other roles through a two-slot ring in shared memory
// (item_full / item_empty). The roles are those of the pair kernel (three warpgroups:
// control = TMA producer warp, MMA warp and two idle warps at 56 registers; softmax A and
// softmax B at 216; TMEM = S_A | S_B | O_A | O_B), and the item boundary is pipelined
// instead of paid by a new CTA:
//   - the producer loads the next item's Q as soon as the last S MMA of the current item
//     has read Q (q_empty), and its K/V stream on through the same rings;
//   - the MMA lane issues the next item's S_A(0) and S_B(0) right behind the current
//     item's last PVs (the tensor core runs them in order, so P is read before S
//     overwrites it), and holds the next item's first PV_x, which overwrites O_x, until
//     softmax group x has read the finished O_x (o_empty);
//   - each softmax group stores its finished rows (o_full) while the tensor core already
//     computes the next item's scores.
// All barrier phases run on counters over the CTA's whole item sequence.
//
// Every wait is bounded; on a timeout the kernel records a code in `status`, drains its
// copies and MMAs, frees TMEM and exits.
#include "kernel_configs.h"
#include "sdpa_pair_common.cuh"

namespace {

using namespace tb;
using namespace tb::sdpa2;

struct Barriers {
  uint64_t q_full, q_empty;
  uint64_t k_full[2], k_empty[2];
  uint64_t v_full[2], v_empty[2];
  uint64_t s_full[2];   // per query tile (A, B)
  uint64_t p_half[2];   // per query tile: P of keys [0, 64) is in TMEM
  uint64_t p_full[2];   // per query tile: P of keys [64, 128) is in TMEM
  uint64_t o_full[2];   // per query tile: every PV of the item is done
  uint64_t o_empty[2];  // per query tile: its softmax group has read O (4 warps)
  uint64_t item_full[2];   // ring of item numbers: written by the producer
  uint64_t item_empty[2];  // read by the MMA lane and the eight softmax warps
  uint64_t drain;
  int32_t item[2];
  uint32_t tmem_base;
};
static_assert(sizeof(Barriers) <= TB_SDPA2_BARRIER_BYTES, "barrier block overflows its reservation");

constexpr int OFF_Q = 0;  // Q_A, Q_B
constexpr int OFF_K = OFF_Q + 2 * TILE_BYTES;
constexpr int OFF_V = OFF_K + 2 * TILE_BYTES;
constexpr int OFF_BAR = OFF_V + 2 * TILE_BYTES;
static_assert(OFF_BAR + TB_SDPA2_BARRIER_BYTES + 1024 == TB_SDPA2_SMEM_BYTES, "smem layout");

constexpr uint32_t kFailProducer = 0x50110000u;
constexpr uint32_t kFailMma = 0x50120000u;
constexpr uint32_t kFailSoftmax = 0x50130000u;
constexpr int kItemReaders = 1 + 8;  // MMA lane, softmax warps

}  // namespace

// q, k, v, o: [BH, T, 128] bf16 (3-D tensor maps {128, T, BH}, box {64, 128, 1}).
// scale_log2 = log2(e) / sqrt(D).
template <int kPolyPairsOf8>
__device__ __forceinline__ void sdpa_persist_body(const CUtensorMap& tmap_q, const CUtensorMap& tmap_k,
                                                  const CUtensorMap& tmap_v, __nv_bfloat16* __restrict__ out, int BH,
                                                  int Tq, int Tk, int causal, float scale_log2, uint32_t* next_item,
                                                  uint32_t* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Barriers* bars = reinterpret_cast<Barriers*>(smem + OFF_BAR);
  const int warp = warp_id(), lane = lane_id();
  const PairSchedule sched{BH, (Tq + 2 * BM - 1) / (2 * BM)};
  const int items = BH * sched.num_pairs;
  const int kv_tiles_all = (Tk + BN - 1) / BN;
  // Key tiles query tile qt needs.
  auto key_tiles = [&](int qt) { return causal ? min(kv_tiles_all, qt + 1) : kv_tiles_all; };

  if (threadIdx.x == 0) {
    mbar_init(&bars->q_full, 1);
    mbar_init(&bars->q_empty, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars->k_full[i], 1);
      mbar_init(&bars->k_empty[i], 1);
      mbar_init(&bars->v_full[i], 1);
      mbar_init(&bars->v_empty[i], 1);
      mbar_init(&bars->s_full[i], 1);
      mbar_init(&bars->p_half[i], 4);
      mbar_init(&bars->p_full[i], 4);
      mbar_init(&bars->o_full[i], 1);
      mbar_init(&bars->o_empty[i], 4);
      mbar_init(&bars->item_full[i], 1);
      mbar_init(&bars->item_empty[i], kItemReaders);
    }
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

  // Each role runs inside the branch of its register count.
  if (warp < 4) {
    setmaxnreg_dec<TB_SDPA2_PAIR_CONTROL_REGS>();
    if (warp == 0) {
      if (lane == 0) {
        // ---------------- TMA producer ----------------
        tma_prefetch_desc(&tmap_q);
        tma_prefetch_desc(&tmap_k);
        tma_prefetch_desc(&tmap_v);
        uint32_t kv = 0, q_issued = 0, k_issued[2] = {0, 0}, v_issued[2] = {0, 0};
        bool ok = true;
        // Item numbers: the first is the CTA's index, each later one comes from the
        // counter (drawn one item ahead, so its latency hides behind the loads).
        int u = blockIdx.x;
        int u_next = blockIdx.x < items ? (int)gridDim.x + (int)atomicAdd(next_item, 1u) : items;
        for (uint32_t it = 0; ok; ++it) {
          const int slot = it & 1;
          if (!mbar_wait(&bars->item_empty[slot], ((it >> 1) & 1) ^ 1)) {
            report_status(status, kFailProducer | 7);
            ok = false;
            break;
          }
          bars->item[slot] = u < items ? u : -1;
          mbar_arrive(&bars->item_full[slot]);  // release: the readers see the number
          if (u >= items) break;
          int bh, pair;
          sched.item(u, bh, pair);
          const int qt0 = 2 * pair, n_b = key_tiles(qt0 + 1);
          // The previous item's last S MMA has read Q.
          if (q_issued && !mbar_wait(&bars->q_empty, (q_issued - 1) & 1)) {
            report_status(status, kFailProducer | 1);
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&bars->q_full, 2 * TILE_BYTES);
          load_tile(smem + OFF_Q, &tmap_q, &bars->q_full, qt0 * BM, bh);
          load_tile(smem + OFF_Q + TILE_BYTES, &tmap_q, &bars->q_full, (qt0 + 1) * BM, bh);
          ++q_issued;
          for (int j = 0; j < kPrefetchAhead && j < n_b; ++j) {
            prefetch_tile(&tmap_k, j * BN, bh);
            prefetch_tile(&tmap_v, j * BN, bh);
          }
          for (int j = 0; j < n_b; ++j, ++kv) {
            if (j + kPrefetchAhead < n_b) {
              prefetch_tile(&tmap_k, (j + kPrefetchAhead) * BN, bh);
              prefetch_tile(&tmap_v, (j + kPrefetchAhead) * BN, bh);
            }
            const int st = kv & 1;
            const uint32_t ph = (kv >> 1) & 1;
            if (!mbar_wait(&bars->k_empty[st], ph ^ 1)) {
              report_status(status, kFailProducer | 2);
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&bars->k_full[st], TILE_BYTES);
            load_tile(smem + OFF_K + st * TILE_BYTES, &tmap_k, &bars->k_full[st], j * BN, bh);
            ++k_issued[st];
            if (!mbar_wait(&bars->v_empty[st], ph ^ 1)) {
              report_status(status, kFailProducer | 3);
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&bars->v_full[st], TILE_BYTES);
            load_tile(smem + OFF_V + st * TILE_BYTES, &tmap_v, &bars->v_full[st], j * BN, bh);
            ++v_issued[st];
          }
          u = u_next;
          if (u < items) u_next = (int)gridDim.x + (int)atomicAdd(next_item, 1u);
        }
        if (!ok) {
          // Every issued copy lands before the CTA may exit.
          if (q_issued && !mbar_wait(&bars->q_full, (q_issued - 1) & 1)) report_status(status, kFailProducer | 4);
          for (int s = 0; s < 2; ++s) {
            if (k_issued[s] && !mbar_wait(&bars->k_full[s], (k_issued[s] - 1) & 1))
              report_status(status, kFailProducer | 5);
            if (v_issued[s] && !mbar_wait(&bars->v_full[s], (v_issued[s] - 1) & 1))
              report_status(status, kFailProducer | 6);
          }
        }
      }
    } else if (warp == 1) {
      if (lane == 0) {
        // ---------------- MMA issuer ----------------
        const uint64_t qd_a = kmajor_desc(smem_addr(smem + OFF_Q), 0);
        const uint64_t qd_b = kmajor_desc(smem_addr(smem + OFF_Q + TILE_BYTES), 0);
        const uint64_t kd0 = kmajor_desc(smem_addr(smem + OFF_K), 0);
        const uint64_t vd0 = v_desc(smem_addr(smem + OFF_V), 0);
        uint32_t kv = 0, tiles_x[2] = {0, 0};  // over the CTA's items so far
        bool ok = true;
        for (uint32_t it = 0; ok; ++it) {
          const int slot = it & 1;
          if (!mbar_wait(&bars->item_full[slot], (it >> 1) & 1)) {
            report_status(status, kFailMma | 8);
            ok = false;
            break;
          }
          const int u = bars->item[slot];
          mbar_arrive(&bars->item_empty[slot]);
          if (u < 0) break;
          int bh, pair;
          sched.item(u, bh, pair);
          (void)bh;
          const int qt0 = 2 * pair;
          const int n_x[2] = {key_tiles(qt0), key_tiles(qt0 + 1)};  // n_x[0] <= n_x[1]
          if (!mbar_wait(&bars->q_full, it & 1)) {
            report_status(status, kFailMma | 1);
            ok = false;
            break;
          }
          // j = key tile whose scores are issued this iteration; PV of tile j-1 goes first.
          for (int j = 0; j <= n_x[1] && ok; ++j) {
            const uint32_t kj = kv + j, vj = kv + j - 1;
            const int st = kj & 1, pst = vj & 1;
            const uint32_t ph = (kj >> 1) & 1, pph = (vj >> 1) & 1;
            const uint64_t kd = desc_add(kd0, st * (TILE_BYTES >> 4));
            const uint64_t vd = desc_add(vd0, pst * (TILE_BYTES >> 4));
            const bool pv_b = j >= 1;
            const bool s_b = j < n_x[1];
            if (pv_b && !mbar_wait(&bars->v_full[pst], pph)) {
              report_status(status, kFailMma | 2);
              ok = false;
              break;
            }
            if (s_b && !mbar_wait(&bars->k_full[st], ph)) {
              report_status(status, kFailMma | 3);
              ok = false;
              break;
            }
            for (int x = 0; x < 2 && ok; ++x) {
              if (j >= 1 && j - 1 < n_x[x]) {
                // The item's first PV_x overwrites O_x: the previous item's O_x must be read.
                if (j == 1 && it > 0 && !mbar_wait(&bars->o_empty[x], (it - 1) & 1)) {
                  report_status(status, kFailMma | 4);
                  ok = false;
                  break;
                }
                const uint32_t pphase = (tiles_x[x] + j - 1) & 1;
                if (!mbar_wait(&bars->p_half[x], pphase)) {
                  report_status(status, kFailMma | 5);
                  ok = false;
                  break;
                }
                tc_fence_after_sync();
                issue_pv_half(tmem + (2 + x) * BN, tmem + x * BN, vd, 0, j - 1 > 0);
                if (!mbar_wait(&bars->p_full[x], pphase)) {
                  report_status(status, kFailMma | 6);
                  ok = false;
                  break;
                }
                tc_fence_after_sync();
                issue_pv_half(tmem + (2 + x) * BN, tmem + x * BN, vd, 1, true);
                if (j == n_x[x]) umma_commit(&bars->o_full[x]);  // the item's last PV_x
              }
              if (j < n_x[x]) {
                tc_fence_after_sync();
                issue_s(tmem + x * BN, x ? qd_b : qd_a, kd);
                umma_commit(&bars->s_full[x]);
              }
            }
            if (!ok) break;
            if (j == n_x[1] - 1) umma_commit(&bars->q_empty);  // the item's last S MMA was just issued
            if (pv_b) umma_commit(&bars->v_empty[pst]);
            if (s_b) umma_commit(&bars->k_empty[st]);
          }
          kv += n_x[1];
          tiles_x[0] += n_x[0];
          tiles_x[1] += n_x[1];
        }
        umma_commit(&bars->drain);
        if (!mbar_wait(&bars->drain, 0)) report_status(status, kFailMma | 7);
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
    uint32_t sc = 0;  // S tiles this group has finished
    bool ok = true;
    for (uint32_t it = 0; ok; ++it) {
      const int slot = it & 1;
      ok = __all_sync(0xffffffffu, mbar_wait(&bars->item_full[slot], (it >> 1) & 1));
      if (!ok) {
        if (lane == 0) report_status(status, kFailSoftmax | 3);
        break;
      }
      const int u = bars->item[slot];
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->item_empty[slot]);
      if (u < 0) break;
      int bh, pair;
      sched.item(u, bh, pair);
      const int qt = 2 * pair + x;
      const int q_row = qt * BM + r;
      const int n = key_tiles(qt);
      float m_used = -INFINITY, l = 0.f;
      for (int j = 0; j < n; ++j, ++sc) {
        ok = __all_sync(0xffffffffu, mbar_wait(&bars->s_full[x], sc & 1));
        if (!ok) {
          if (lane == 0) report_status(status, kFailSoftmax | 1);
          break;
        }
        tc_fence_after_sync();
        // S_x(j) was committed after PV_x(j-1): O_x holds the tiles before j and no PV of
        // tile j starts before p_half, so the rescale may touch O from j = 1 on.
        const int valid = (causal ? min(Tk, q_row + 1) : Tk) - j * BN;
        softmax_tile<kPolyPairsOf8>(s_tmem, o_tmem, valid, j > 0, scale_log2, m_used, l, &bars->p_half[x],
                                    &bars->p_full[x]);
      }
      if (!ok) break;
      ok = __all_sync(0xffffffffu, mbar_wait(&bars->o_full[x], it & 1));
      if (!ok) {
        if (lane == 0) report_status(status, kFailSoftmax | 2);
        break;
      }
      tc_fence_after_sync();
      store_row(o_tmem, l, out + ((long long)bh * Tq + q_row) * HD, q_row < Tq);
      // O_x is read: the next item's first PV_x may overwrite it.
      tc_fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->o_empty[x]);
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

// One CTA per SM, 12 warps launched at 168 registers a thread; the softmax warps then
// hold 216 (the pair kernel's split). `next_item` is a zeroed 32-bit counter.
extern "C" __global__ void __launch_bounds__(TB_SDPA2_PAIR_THREADS, 1)
    sdpa_fwd_bf16_d128_persist(const __grid_constant__ CUtensorMap tmap_q, const __grid_constant__ CUtensorMap tmap_k,
                               const __grid_constant__ CUtensorMap tmap_v, __nv_bfloat16* __restrict__ out, int BH,
                               int Tq, int Tk, int causal, float scale_log2, uint32_t* next_item, uint32_t* status) {
  // Every exponential on the MUFU, as in the pair kernel.
  sdpa_persist_body<0>(tmap_q, tmap_k, tmap_v, out, BH, Tq, Tk, causal, scale_log2, next_item, status);
}
