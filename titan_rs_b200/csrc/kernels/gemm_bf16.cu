// bf16 GEMM with fp32 accumulation on the 5th-generation tensor cores.
//
//   C[M,N] (bf16, row-major, leading dimension ldc) = A[M,K] (bf16, row-major) x B^T
//   where B is stored as [N,K] row-major, i.e. the column-major B of the
//   titan.rs GEMM with transpose_rhs (projects/titan-runtime/src/lib.rs:955-989).
//
// Two pipelines: umma_pipeline.cuh, one persistent CTA per SM on 128x256 tiles (TMA
// producer warp, MMA warp with two 128x256 fp32 TMEM accumulators, four epilogue
// warps), and umma_pipeline_2sm.cuh, CTA pairs on 256x256 tiles with
// tcgen05.mma.cta_group::2 (the default once the output fills the SMs). The policies
// (gemm_policies.cuh) map tiles and k-blocks to TMA coordinates, 128-byte swizzle;
// tiles are visited in groups of 2048 rows of A so the tiles in flight share A rows
// and B columns in L2. K tails and M/N tails come back from TMA as zeros; the
// epilogue masks them.
//
// Fused all-gather (gemm_bf16_tn_allgather, _2sm, _2sm_push): the N-sharded GEMM of one
// rank whose output tiles reach all ranks' row-major C through NVLink peer stores (CUDA
// IPC mappings) while the remaining tiles compute; the ranks synchronise through flags
// in each other's memory (peer_signal.cuh). The stores come from the epilogue (1-SM),
// from push warps fed through shared memory (_2sm), or from dedicated pusher CTAs that
// copy finished tiles out of this rank's C (_2sm_push, from four ranks).
//
// Split-K (gemm_bf16_tn_splitk + splitk_reduce_bf16): when the output has too
// few 128x256 tiles to occupy the SMs, each tile's K range is cut into slices
// that run as separate work units writing fp32 partials to scratch memory; the
// reduction sums them in a fixed order.
#include "gemm_policies.cuh"
#include "peer_signal.cuh"

namespace {
constexpr uint32_t kFailGemm = 0x47000000u;
constexpr uint32_t kFailGemm2 = 0x47320000u;
constexpr uint32_t kFailSplitK = 0x4B000000u;
constexpr uint32_t kFailAllGather = 0x47410000u;
constexpr uint32_t kFailAllGather2 = 0x47420000u;
}  // namespace

extern "C" __global__ void __launch_bounds__(TB_GEMM_THREADS, 1)
    gemm_bf16_tn(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                 __nv_bfloat16* __restrict__ c, int M, int N, int K, long long ldc, uint32_t* status) {
  tb::gemm::GemmPolicy p;
  p.ta = &tmap_a;
  p.tb = &tmap_b;
  p.c = c;
  p.M = M;
  p.N = N;
  p.K = K;
  p.ldc = ldc;
  p.vec_ok = (ldc % 8) == 0 && (reinterpret_cast<uintptr_t>(c) & 15) == 0;
  p.num_m = (M + tb::umma::BM - 1) / tb::umma::BM;
  p.num_n = (N + tb::umma::BN - 1) / tb::umma::BN;
  tb::umma::run(p, status, kFailGemm);
}

// The same product on CTA pairs (umma_pipeline_2sm.cuh): 256x256 tiles, each CTA
// loading a 128-row A block and half of the 256-row B block per k-block. Launched
// with clusters of 2 along x; tensor maps with 128-row boxes for A and B.
extern "C" __global__ void __launch_bounds__(TB_GEMM_THREADS, 1)
    gemm_bf16_tn_2sm(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                     __nv_bfloat16* __restrict__ c, int M, int N, int K, long long ldc, uint32_t* status) {
  tb::gemm::Gemm2Policy p;
  p.ta = &tmap_a;
  p.tb = &tmap_b;
  p.c = c;
  p.M = M;
  p.N = N;
  p.K = K;
  p.ldc = ldc;
  p.vec_ok = (ldc % 8) == 0 && (reinterpret_cast<uintptr_t>(c) & 15) == 0;
  tb::umma2::run(p, status, kFailGemm2);
}

// The other storage orders on CTA pairs (Gemm2LayoutPolicy): an operand stored [K, rows]
// comes through a tensor map over that storage with {64, 64} boxes. C = act(A B + bias)
// as in gemm_bf16_tn_bias_act (bias null and act none for the plain product).
//   gemm_bf16_nn_2sm     A [M, K], B [K, N]
//   gemm_bf16_ta_2sm     A [K, M] (transpose_lhs), B [N, K] (transpose_rhs)
//   gemm_bf16_ta_nn_2sm  A [K, M] (transpose_lhs), B [K, N]
#define TB_GEMM2_LAYOUT_ENTRY(name, at, bn)                                                                       \
  extern "C" __global__ void __launch_bounds__(TB_GEMM_THREADS, 1)                                                \
      name(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,                \
           __nv_bfloat16* __restrict__ c, const float* __restrict__ bias, int act, int M, int N, int K,           \
           long long ldc, uint32_t* status) {                                                                     \
    tb::gemm::Gemm2LayoutPolicy<at, bn> p;                                                                       \
    p.bias = bias;                                                                                                \
    p.act = act;                                                                                                  \
    p.ta = &tmap_a;                                                                                               \
    p.tb = &tmap_b;                                                                                               \
    p.c = c;                                                                                                      \
    p.M = M;                                                                                                      \
    p.N = N;                                                                                                      \
    p.K = K;                                                                                                      \
    p.ldc = ldc;                                                                                                  \
    p.vec_ok = (ldc % 8) == 0 && (reinterpret_cast<uintptr_t>(c) & 15) == 0;                                      \
    tb::umma2::run(p, status, kFailGemm2);                                                                        \
  }
TB_GEMM2_LAYOUT_ENTRY(gemm_bf16_nn_2sm, false, true)
TB_GEMM2_LAYOUT_ENTRY(gemm_bf16_ta_2sm, true, false)
TB_GEMM2_LAYOUT_ENTRY(gemm_bf16_ta_nn_2sm, true, true)

// gemm_bf16_tn_bias_act on the 2-SM pipeline.
extern "C" __global__ void __launch_bounds__(TB_GEMM_THREADS, 1)
    gemm_bf16_tn_bias_act_2sm(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                              __nv_bfloat16* __restrict__ c, const float* __restrict__ bias, int act, int M, int N,
                              int K, long long ldc, uint32_t* status) {
  tb::gemm::Gemm2Policy p;
  p.ta = &tmap_a;
  p.tb = &tmap_b;
  p.c = c;
  p.M = M;
  p.N = N;
  p.K = K;
  p.ldc = ldc;
  p.vec_ok = (ldc % 8) == 0 && (reinterpret_cast<uintptr_t>(c) & 15) == 0;
  p.bias = bias;
  p.act = act;
  tb::umma2::run(p, status, kFailGemm2);
}

// GEMM with a fused epilogue: C = act(A B^T + bias) (bias fp32 [N] or null; act an
// epilogue_math.cuh Activation), rounded to bf16 once.
extern "C" __global__ void __launch_bounds__(TB_GEMM_THREADS, 1)
    gemm_bf16_tn_bias_act(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                          __nv_bfloat16* __restrict__ c, const float* __restrict__ bias, int act, int M, int N, int K,
                          long long ldc, uint32_t* status) {
  tb::gemm::GemmPolicy p;
  p.ta = &tmap_a;
  p.tb = &tmap_b;
  p.c = c;
  p.M = M;
  p.N = N;
  p.K = K;
  p.ldc = ldc;
  p.vec_ok = (ldc % 8) == 0 && (reinterpret_cast<uintptr_t>(c) & 15) == 0;
  p.num_m = (M + tb::umma::BM - 1) / tb::umma::BM;
  p.num_n = (N + tb::umma::BN - 1) / tb::umma::BN;
  p.bias = bias;
  p.act = act;
  tb::umma::run(p, status, kFailGemm);
}

// Fused GEMM + all-gather: this rank's N-shard (B rows [N, K]) of C[M, ldc], written
// at column col0 into every rank's C through `outs` (its own entry included).
// Call `epoch` of the registered output, synchronised with the other ranks in-kernel:
//   entry  CTA 0 announces the epoch in every peer's signal block; each CTA waits until
//          every peer has announced it (so every peer is done with its C) before it
//          computes and stores anything;
//   exit   the last CTA to finish (all stores fenced system-wide) tells every peer its
//          stores have landed and waits until every peer has said the same, so the
//          kernel completes only when this rank's C is whole.
extern "C" __global__ void __launch_bounds__(TB_GEMM_THREADS, 1)
    gemm_bf16_tn_allgather(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                           const __grid_constant__ tb::gemm::RankOutputs outs,
                           const __grid_constant__ tb::RankSignals sig, int ranks, int self, uint32_t epoch, int M,
                           int N, int K, long long ldc, long long col0, uint32_t* status) {
  const bool entry_ok = tb::call_entry(sig, ranks, self, epoch, status, kFailAllGather | 0x0501);
  if (entry_ok) {
    tb::gemm::AllGatherPolicy p;
    p.ta = &tmap_a;
    p.tb = &tmap_b;
    p.c = nullptr;
    p.M = M;
    p.N = N;
    p.K = K;
    p.ldc = ldc;
    p.vec_ok = true;  // the host requires 16-byte aligned bases, ldc % 8 == 0, col0 % 8 == 0 and N % 8 == 0
    p.num_m = (M + tb::umma::BM - 1) / tb::umma::BM;
    p.num_n = (N + tb::umma::BN - 1) / tb::umma::BN;
    p.outs = &outs;
    p.ranks = ranks;
    p.self = self;
    p.col0 = col0;
    tb::umma::run(p, status, kFailAllGather);
  }
  // Every epilogue thread fenced its stores (AllGatherPolicy::finish) before run()'s
  // final __syncthreads (a CTA whose entry failed stored nothing).
  tb::call_exit(sig, ranks, self, epoch, entry_ok, status, kFailAllGather | 0x0502);
}

// The fused GEMM + all-gather on CTA pairs (clusters of 2 along x, 128-row boxes for A
// and B, TB_GEMM2_AG_THREADS threads: the pipeline's six warps and four push warps).
// Same handshake as gemm_bf16_tn_allgather; a CTA whose entry wait fails still runs the
// pair pipeline (its partner waits for it at cluster barriers) with stores off.
extern "C" __global__ void __launch_bounds__(TB_GEMM2_AG_THREADS, 1)
    gemm_bf16_tn_allgather_2sm(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                               const __grid_constant__ tb::gemm::RankOutputs outs,
                               const __grid_constant__ tb::RankSignals sig, int ranks, int self, uint32_t epoch, int M,
                               int N, int K, long long ldc, long long col0, uint32_t* status) {
  const bool entry_ok = tb::call_entry(sig, ranks, self, epoch, status, kFailAllGather | 0x0501);
  tb::gemm::AllGather2Policy p;
  p.ta = &tmap_a;
  p.tb = &tmap_b;
  p.c = nullptr;
  p.M = M;
  p.N = N;
  p.K = K;
  p.ldc = ldc;
  p.vec_ok = true;  // the host requires 16-byte aligned bases, ldc % 8 == 0, col0 % 8 == 0 and N % 8 == 0
  p.outs = &outs;
  p.ranks = ranks;
  p.self = self;
  p.col0 = col0;
  p.enabled = entry_ok != 0;
  tb::umma2::run<tb::gemm::AllGather2Policy, TB_GEMM2_AG_STAGES>(p, status, kFailAllGather2);
  // Every push-warp thread fenced its stores (AllGather2Policy::side) before run()'s
  // final cluster barrier.
  tb::call_exit(sig, ranks, self, epoch, entry_ok, status, kFailAllGather | 0x0502);
}

// Pusher role of gemm_bf16_tn_allgather_2sm_push: the grid's pusher CTAs split the
// CTA-tiles of this rank's column block into 32-row quarters (in tile order, which is
// the order the pipeline finishes them), wait until the tile's four quarters are stored
// in this rank's C (ready count 4), and copy each row (one 16-byte segment per lane,
// read from L2) into every other rank's C.
__device__ __forceinline__ void push_finished_tiles(const tb::gemm::RankOutputs* outs, int ranks, int self, int M,
                                                    int N, long long ldc, long long col0, const uint32_t* ready,
                                                    int tiles, int num_pm, int num_n, int first_pusher,
                                                    uint32_t* status) {
  const int warps_per_cta = blockDim.x >> 5, lane = tb::lane_id();
  const int w = ((int)blockIdx.x - first_pusher) * warps_per_cta + (int)tb::warp_id();
  const int stride = ((int)gridDim.x - first_pusher) * warps_per_cta;
  const __nv_bfloat16* own = outs->base[self];
  for (int c = w; c < tiles * 8; c += stride) {
    const int t = c >> 3, r = (c >> 2) & 1, q = c & 3;
    int m_blk, n_blk;
    tb::umma::grouped_tile(t, num_pm, num_n, TB_GEMM2_GROUP, m_blk, n_blk);
    const int row0 = (2 * m_blk + r) * 128 + q * 32;
    if (row0 >= M) continue;
    const uint64_t start = tb::global_timer_ns();  // each tile is waited for at most ~1 s
    while (tb::ld_acquire_gpu(&ready[2 * t + r]) < 4u) {
      if (tb::global_timer_ns() - start > tb::kWaitLimitNs) {
        if (lane == 0) tb::report_status(status, kFailAllGather | 0x0801);
        return;
      }
    }
    const int gc = n_blk * 256 + lane * 8;
    if (gc >= N) continue;
    const int rows = min(32, M - row0);
    for (int rr = 0; rr < rows; ++rr) {
      const long long off = (long long)(row0 + rr) * ldc + col0 + gc;
      const uint4 v = __ldcg(reinterpret_cast<const uint4*>(own + off));
      for (int k = 1, d = self + 1 == ranks ? 0 : self + 1; k < ranks; ++k, d = (d + 1 == ranks) ? 0 : d + 1)
        *reinterpret_cast<uint4*>(outs->base[d] + off) = v;
    }
  }
}

// The fused GEMM + all-gather for many ranks: CTAs [0, 2 gemm_pairs) run the pair
// pipeline into this rank's own C (AllGatherLocalPolicy); the rest push finished tiles
// to the peers. Launched with clusters of 2, TB_GEMM2_PUSH_THREADS threads and
// TB_GEMM2_SMEM_BYTES of shared memory for every CTA (one CTA per SM, so pushers have
// SMs of their own); `ready` holds 2 x pair-tiles counters zeroed before the launch.
// Same entry and exit handshake as the other fused kernels; a CTA whose entry wait
// fails stores nothing (GEMM CTAs still run the pair pipeline with their partner).
extern "C" __global__ void __launch_bounds__(TB_GEMM2_PUSH_THREADS, 1)
    gemm_bf16_tn_allgather_2sm_push(const __grid_constant__ CUtensorMap tmap_a,
                                    const __grid_constant__ CUtensorMap tmap_b,
                                    const __grid_constant__ tb::gemm::RankOutputs outs,
                                    const __grid_constant__ tb::RankSignals sig, int ranks, int self, uint32_t epoch,
                                    int M, int N, int K, long long ldc, long long col0, uint32_t* ready,
                                    int gemm_pairs, uint32_t* status) {
  const bool entry_ok = tb::call_entry(sig, ranks, self, epoch, status, kFailAllGather | 0x0501);
  const int num_pm = (M + 255) / 256, num_n = (N + 255) / 256;
  if ((int)blockIdx.x < 2 * gemm_pairs) {
    tb::gemm::AllGatherLocalPolicy p;
    p.ta = &tmap_a;
    p.tb = &tmap_b;
    p.c = outs.base[self] + col0;
    p.M = M;
    p.enabled = entry_ok != 0;
    p.N = N;
    p.K = K;
    p.ldc = ldc;
    p.vec_ok = true;  // the host requires 16-byte aligned bases, ldc % 8 == 0, col0 % 8 == 0 and N % 8 == 0
    p.ready = ready;
    p.gemm_pairs = gemm_pairs;
    tb::umma2::run(p, status, kFailAllGather2);
  } else if (entry_ok && ranks > 1) {
    push_finished_tiles(&outs, ranks, self, M, N, ldc, col0, ready, num_pm * num_n, num_pm, num_n, 2 * gemm_pairs,
                        status);
  }
  __threadfence_system();  // this thread's peer stores, before the exit handshake
  __syncthreads();
  tb::call_exit(sig, ranks, self, epoch, entry_ok, status, kFailAllGather | 0x0502);
}

extern "C" __global__ void __launch_bounds__(TB_GEMM_THREADS, 1)
    gemm_bf16_tn_splitk(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                        float* __restrict__ partial, int M, int N, int K, int splits, int kb_per_split,
                        uint32_t* status) {
  tb::gemm::run_splitk(&tmap_a, &tmap_b, partial, M, N, K, splits, kb_per_split, status, kFailSplitK);
}

extern "C" __global__ void __launch_bounds__(256) splitk_reduce_bf16(const float* __restrict__ partial,
                                                                    __nv_bfloat16* __restrict__ c, int M, int N,
                                                                    int splits, long long ldc) {
  tb::gemm::splitk_reduce(partial, c, M, N, splits, ldc);
}
