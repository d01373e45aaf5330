// "gemm" operator entry: the contract of execute_cuda_gemm and the CPU gemm
// (titan-runtime/src/lib.rs:2289-2404, 955-989), then the kernel choice:
//   BF16, A row-major, B column-major (transpose_rhs), K % 8 == 0, 16-byte
//        aligned buffers        -> gemm_bf16_tn_2sm (tcgen05 on CTA pairs, TMA, TMEM) when the
//                                  output fills the SMs, gemm_bf16_tn (one SM per tile) when it
//                                  does not, gemm_bf16_tn_splitk when too few tiles exist
//   BF16, other storage orders (B stored [K, N] and/or A stored [K, M] by transpose_lhs),
//        contiguous extents % 8 == 0, aligned
//                               -> gemm_bf16_nn_2sm / gemm_bf16_ta_2sm / gemm_bf16_ta_nn_2sm (the
//                                  same pairs reading those operands M- or N-contiguous)
//   BF16, any other layout      -> gemm_bf16_staged (the operands the TMA cannot read copied
//                                  K-major with K rounded up to 8, then the kernels above) from
//                                  2^24 multiply-adds, gemm_bf16_generic (CUDA cores) below
//   F32                         -> gemm_f32_tiled (CUDA cores, bit-exact with the CPU reference)
#include "../kernels/kernel_configs.h"
#include <algorithm>

#include "ops_common.hpp"

namespace tb {

tb_status launch_gemm_bf16_tn(Session* s, Stream* st, CUdeviceptr a, CUdeviceptr b, CUdeviceptr c, int M, int N,
                              int K, long long ldc) {
  CUtensorMap ta, tbm;
  tb_status rc = tmap_bf16_2d(&ta, a, (uint64_t)M, (uint64_t)K, (uint64_t)K, TB_GEMM_BM, TB_GEMM_BK,
                              CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = tmap_bf16_2d(&tbm, b, (uint64_t)N, (uint64_t)K, (uint64_t)K, TB_GEMM_BN, TB_GEMM_BK,
                    CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  CUfunction fn = nullptr;
  rc = builtin_function(s, "gemm_bf16", "gemm_bf16_tn", &fn);
  if (rc) return rc;
  const long long tiles = (long long)((M + TB_GEMM_BM - 1) / TB_GEMM_BM) * ((N + TB_GEMM_BN - 1) / TB_GEMM_BN);
  const unsigned grid = (unsigned)(tiles < s->sm_count ? tiles : s->sm_count);
  CUdeviceptr status = s->status.device;
  void* params[] = {&ta, &tbm, &c, &M, &N, &K, &ldc, &status};
  return launch_builtin(s, st, fn, grid, 1, 1, TB_GEMM_THREADS, TB_GEMM_SMEM_BYTES, params, "gemm_bf16_tn");
}

// 2-SM form: clusters of two CTAs on 256x256 tiles (gemm_bf16_tn_2sm). The persistent
// grid is as many pairs as can be resident at once (the driver's cluster occupancy), at
// most one per tile.
tb_status launch_gemm_bf16_tn_2sm(Session* s, Stream* st, CUdeviceptr a, CUdeviceptr b, CUdeviceptr c, int M, int N,
                                  int K, long long ldc) {
  CUtensorMap ta, tbm;
  tb_status rc = tmap_bf16_2d(&ta, a, (uint64_t)M, (uint64_t)K, (uint64_t)K, 128, TB_GEMM_BK,
                              CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = tmap_bf16_2d(&tbm, b, (uint64_t)N, (uint64_t)K, (uint64_t)K, 128, TB_GEMM_BK, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  CUfunction fn = nullptr;
  rc = builtin_function(s, "gemm_bf16", "gemm_bf16_tn_2sm", &fn);
  if (rc) return rc;
  const long long pair_tiles = (long long)((M + 255) / 256) * ((N + 255) / 256);
  CUdeviceptr status = s->status.device;
  void* params[] = {&ta, &tbm, &c, &M, &N, &K, &ldc, &status};
  return launch_builtin_pairs(s, st, fn, pair_tiles, TB_GEMM_THREADS, TB_GEMM2_SMEM_BYTES, params, "gemm_bf16_tn_2sm");
}

// The storage orders other than A [M, K] x B [N, K] on CTA pairs, at any size: an
// operand stored [K, rows] (A with transpose_lhs, B without transpose_rhs) is read
// through a tensor map over that storage with {64, 64} boxes and fed to the MMA
// M- or N-contiguous. `name` is gemm_bf16_nn_2sm, gemm_bf16_ta_2sm or gemm_bf16_ta_nn_2sm.
// lda / ldb: row pitches (elements) of A and B as stored; 0 = the contiguous extent.
tb_status launch_gemm_bf16_layout_2sm(Session* s, Stream* st, const char* name, bool a_km, bool b_kn, CUdeviceptr a,
                                      CUdeviceptr b, CUdeviceptr c, int M, int N, int K, long long ldc,
                                      CUdeviceptr bias = 0, int act = TB_ACT_NONE, uint64_t lda = 0,
                                      uint64_t ldb = 0) {
  CUtensorMap ta, tbm;
  if (!lda) lda = a_km ? (uint64_t)M : (uint64_t)K;
  if (!ldb) ldb = b_kn ? (uint64_t)N : (uint64_t)K;
  tb_status rc = a_km ? tmap_bf16_2d(&ta, a, (uint64_t)K, (uint64_t)M, lda, 64, 64, CU_TENSOR_MAP_SWIZZLE_128B)
                      : tmap_bf16_2d(&ta, a, (uint64_t)M, (uint64_t)K, lda, 128, TB_GEMM_BK,
                                     CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = b_kn ? tmap_bf16_2d(&tbm, b, (uint64_t)K, (uint64_t)N, ldb, 64, 64, CU_TENSOR_MAP_SWIZZLE_128B)
            : tmap_bf16_2d(&tbm, b, (uint64_t)N, (uint64_t)K, ldb, 128, TB_GEMM_BK, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  CUfunction fn = nullptr;
  rc = builtin_function(s, "gemm_bf16", name, &fn);
  if (rc) return rc;
  const long long pair_tiles = (long long)((M + 255) / 256) * ((N + 255) / 256);
  CUdeviceptr status = s->status.device;
  void* params[] = {&ta, &tbm, &c, &bias, &act, &M, &N, &K, &ldc, &status};
  return launch_builtin_pairs(s, st, fn, pair_tiles, TB_GEMM_THREADS, TB_GEMM2_SMEM_BYTES, params, name);
}

// The layout kernel for an A/B storage order other than A [M, K] x B [N, K], or null
// when the order is that one or a TMA row would not start 16-byte aligned.
static const char* layout_kernel_for(bool tl, bool tr, uint64_t M, uint64_t N, uint64_t K, CUdeviceptr any_ptrs) {
  const char* name = !tl && !tr ? "gemm_bf16_nn_2sm" : tl && tr ? "gemm_bf16_ta_2sm" : tl ? "gemm_bf16_ta_nn_2sm"
                                                                                        : nullptr;
  const bool ok = name && ((tl ? M : K) % 8) == 0 && ((tr ? K : N) % 8) == 0 && (any_ptrs & 15) == 0;
  return ok ? name : nullptr;
}

// The unsplit tensor-core GEMM the operator runs by default: the 2-SM kernel once the
// output holds at least a full wave of 128x256 tiles (it moves a third less operand data
// per FLOP from L2 into shared memory), else the 1-SM kernel, whose 128-row tiles waste
// less of a short M.
tb_status launch_gemm_bf16_default(Session* s, Stream* st, CUdeviceptr a, CUdeviceptr b, CUdeviceptr c, int M, int N,
                                   int K, long long ldc) {
  const long long tiles = (long long)((M + TB_GEMM_BM - 1) / TB_GEMM_BM) * ((N + TB_GEMM_BN - 1) / TB_GEMM_BN);
  if (M >= 256 && tiles >= s->sm_count) return launch_gemm_bf16_tn_2sm(s, st, a, b, c, M, N, K, ldc);
  return launch_gemm_bf16_tn(s, st, a, b, c, M, N, K, ldc);
}

// Row-padded copy of a bf16 operand stored as `rows` rows of `cols` contiguous elements
// (pitch ld_src): dst holds the same rows with pitch round_up(cols, 8) and zeros after
// column `cols` (stage_bf16_pad_rows, one thread per 16-byte chunk of dst).
static tb_status launch_stage_bf16(Session* s, Stream* st, CUdeviceptr src, CUdeviceptr dst, int rows, int cols,
                                   long long ld_src) {
  CUfunction fn = nullptr;
  tb_status rc = builtin_function(s, "layout", "stage_bf16_pad_rows", &fn);
  if (rc) return rc;
  int ld_dst = (cols + 7) / 8 * 8;
  const long long chunks = (long long)rows * (ld_dst / 8);
  const unsigned grid = (unsigned)std::min<long long>((chunks + 255) / 256, s->sm_count * 8LL);
  void* params[] = {&src, &dst, &rows, &cols, &ld_src, &ld_dst};
  return launch_builtin(s, st, fn, grid, 1, 1, 256, 0, params, "stage_bf16_pad_rows");
}

// op(A) (M x K, strides as0/as1) times op(B) (K x N, strides bs0/bs1) for storage the TMA
// cannot describe. Each operand keeps its storage order; one whose contiguous extent is
// not a multiple of 8 (or whose base is not 16-byte aligned) is copied with its rows
// padded to a multiple of 8 elements into the stream's scratch (no transpose), and the
// tensor-core kernel for that storage order reads the copy with its padded pitch:
//   A [M, K] x B [N, K]  gemm_bf16_tn(_2sm) over K rounded up to 8 (both pads are zero)
//   any other order      gemm_bf16_nn_2sm / _ta_2sm / _ta_nn_2sm, logical extents
// C = act(A B^T + bias) on the K-major operands A [M, K] and B [N, K] (gemm_bf16_tn_bias_act
// and its CTA-pair form, chosen as for the plain GEMM unless `candidate` names one).
static tb_status launch_gemm_bf16_tn_bias_act(Session* s, Stream* st, CUdeviceptr pa, CUdeviceptr pb, CUdeviceptr pc,
                                              int M, int N, int K, CUdeviceptr pbias, int act, const char* candidate,
                                              long long ldc = 0) {
  const long long tiles = (long long)((M + TB_GEMM_BM - 1) / TB_GEMM_BM) * ((N + TB_GEMM_BN - 1) / TB_GEMM_BN);
  const bool pairs = candidate ? strcmp(candidate, "gemm_bf16_tn_bias_act_2sm") == 0
                               : (M >= 256 && tiles >= s->sm_count);
  const uint32_t box_rows_b = pairs ? 128 : TB_GEMM_BN;
  CUtensorMap ta, tbm;
  tb_status rc;
  if ((rc = tmap_bf16_2d(&ta, pa, (uint64_t)M, (uint64_t)K, (uint64_t)K, TB_GEMM_BM, TB_GEMM_BK,
                         CU_TENSOR_MAP_SWIZZLE_128B)) ||
      (rc = tmap_bf16_2d(&tbm, pb, (uint64_t)N, (uint64_t)K, (uint64_t)K, box_rows_b, TB_GEMM_BK,
                         CU_TENSOR_MAP_SWIZZLE_128B)))
    return rc;
  CUfunction fn = nullptr;
  const char* name = pairs ? "gemm_bf16_tn_bias_act_2sm" : "gemm_bf16_tn_bias_act";
  rc = builtin_function(s, "gemm_bf16", name, &fn);
  if (rc) return rc;
  CUdeviceptr c = pc, status = s->status.device;
  if (!ldc) ldc = N;
  void* params[] = {&ta, &tbm, &c, &pbias, &act, &M, &N, &K, &ldc, &status};
  if (pairs) {
    const long long pair_tiles = (long long)((M + 255) / 256) * ((N + 255) / 256);
    return launch_builtin_pairs(s, st, fn, pair_tiles, TB_GEMM_THREADS, TB_GEMM2_SMEM_BYTES, params, name);
  }
  const unsigned grid = (unsigned)(tiles < s->sm_count ? tiles : s->sm_count);
  return launch_builtin(s, st, fn, grid, 1, 1, TB_GEMM_THREADS, TB_GEMM_SMEM_BYTES, params, name);
}

static tb_status launch_gemm_bf16_staged(Session* s, Stream* st, CUdeviceptr a, long long as0, long long as1,
                                         CUdeviceptr b, long long bs0, long long bs1, CUdeviceptr c, int M, int N,
                                         int K, bool epilogue = false, CUdeviceptr bias = 0,
                                         int act = TB_ACT_NONE) {
  // Storage of each operand: A is [K, M] when its M stride is 1 (transpose_lhs), else
  // [M, K]; B is [K, N] when its N stride is 1, else [N, K] (transpose_rhs).
  const bool a_km = as0 == 1 && as1 != 1, b_kn = bs1 == 1 && bs0 != 1;
  const int a_rows = a_km ? K : M, a_cols = a_km ? M : K;
  const int b_rows = b_kn ? K : N, b_cols = b_kn ? N : K;
  const long long a_ld = a_km ? as1 : as0, b_ld = b_kn ? bs0 : bs1;
  const bool stage_a = (a_cols % 8) != 0 || (a & 15) != 0 || a_ld != a_cols;
  const bool stage_b = (b_cols % 8) != 0 || (b & 15) != 0 || b_ld != b_cols;
  // An output whose rows do not start 16-byte aligned is computed into an aligned copy
  // with vector stores, then moved into place (unstage_bf16_rows).
  const bool stage_c = (N % 8) != 0 || (c & 15) != 0;
  const uint64_t a_pitch = (uint64_t)(a_cols + 7) / 8 * 8, b_pitch = (uint64_t)(b_cols + 7) / 8 * 8;
  const int c_pitch = (N + 7) / 8 * 8;
  const size_t a_span = stage_a ? ((size_t)a_rows * a_pitch * 2 + 255) & ~(size_t)255 : 0;
  const size_t b_span = stage_b ? ((size_t)b_rows * b_pitch * 2 + 255) & ~(size_t)255 : 0;
  const size_t c_span = stage_c ? (size_t)M * c_pitch * 2 : 0;
  CUdeviceptr ws = 0;
  tb_status rc = TB_OK;
  if (a_span + b_span + c_span) rc = stream_scratch(s, st, a_span + b_span + c_span, &ws);
  if (rc) return rc;
  const CUdeviceptr ka = stage_a ? ws : a, kb = stage_b ? ws + a_span : b, kc = stage_c ? ws + a_span + b_span : c;
  const long long ldc = stage_c ? c_pitch : N;
  if ((stage_a && (rc = launch_stage_bf16(s, st, a, ka, a_rows, a_cols, a_ld))) ||
      (stage_b && (rc = launch_stage_bf16(s, st, b, kb, b_rows, b_cols, b_ld))))
    return rc;
  if (!a_km && !b_kn) {
    // Both K-major: the copies (or the operands, when K % 8 == 0) have pitch round_up(K, 8).
    const int kp = (int)a_pitch;
    rc = epilogue ? launch_gemm_bf16_tn_bias_act(s, st, ka, kb, kc, M, N, kp, bias, act, nullptr, ldc)
                  : launch_gemm_bf16_default(s, st, ka, kb, kc, M, N, kp, ldc);
  } else {
    const char* name = a_km ? (b_kn ? "gemm_bf16_ta_nn_2sm" : "gemm_bf16_ta_2sm") : "gemm_bf16_nn_2sm";
    rc = launch_gemm_bf16_layout_2sm(s, st, name, a_km, b_kn, ka, kb, kc, M, N, K, ldc, bias, act,
                                     stage_a ? a_pitch : (uint64_t)a_ld, stage_b ? b_pitch : (uint64_t)b_ld);
  }
  if (rc) return rc;
  if (stage_c) {
    CUfunction fn = nullptr;
    if ((rc = builtin_function(s, "layout", "unstage_bf16_rows", &fn))) return rc;
    CUdeviceptr src = kc, dst = c;
    int rows = M, cols = N, ld_src = c_pitch;
    long long ld_dst = N;
    const long long units = (long long)rows * (cols / 8 + 2);
    const unsigned grid = (unsigned)std::min<long long>((units + 255) / 256, s->sm_count * 8LL);
    void* params[] = {&src, &dst, &rows, &cols, &ld_src, &ld_dst};
    if ((rc = launch_builtin(s, st, fn, grid, 1, 1, 256, 0, params, "unstage_bf16_rows"))) return rc;
  }
  note_candidate("gemm_bf16_staged");
  return TB_OK;
}

// Fused N-sharded GEMM + all-gather: this rank's [M, N] column block of the row-major
// C[M, ldc] at column col0, stored into every rank's C (outs[i] = rank i's base); the
// ranks synchronise through their signal blocks (signals[i] = rank i's) for call `epoch`.
// Pusher CTAs for the fused all-gather: TITAN_B200_ALLGATHER_PUSHERS (an even count, 0 =
// none) if set; else none below four ranks (the tensor work of the SMs they would take
// outweighs the stores: 2428 against 2281 TFLOP/s with 16 at 2 ranks for C3), 16 from
// four ranks (best of 0, 16, 32 at 4 ranks: 3354, 3931, 3819) and 32 from eight (3917
// against 3860 with 16), where each rank receives 112 MB against 0.1 ms of compute.
static int allgather_pushers(int ranks) {
  if (const char* e = getenv("TITAN_B200_ALLGATHER_PUSHERS")) {
    const int v = atoi(e);
    return v > 0 ? (v + 1) & ~1 : 0;
  }
  return ranks >= 8 ? 32 : ranks >= 4 ? 16 : 0;
}

tb_status launch_gemm_bf16_tn_allgather(Session* s, Stream* st, CUdeviceptr a, CUdeviceptr b, const CUdeviceptr* outs,
                                        const CUdeviceptr* signals, int ranks, int self, uint32_t epoch, int M, int N,
                                        int K, long long ldc, long long col0, CUdeviceptr ready, size_t ready_count) {
  if (ranks < 1 || ranks > TB_MAX_RANKS) return unsupported("fused all-gather supports 1 to 8 ranks");
  // The kernel stores whole 16-byte segments (8 columns) into every rank's C.
  if (ldc % 8 != 0 || col0 % 8 != 0 || N % 8 != 0) return unsupported("fused all-gather needs 8-column alignment");
  for (int i = 0; i < ranks; ++i)
    if (outs[i] & 15) return unsupported("fused all-gather needs 16-byte aligned outputs");
  // CTA pairs under the same rule as the plain GEMM (gemm_bf16_tn_allgather_2sm).
  const long long tiles = (long long)((M + TB_GEMM_BM - 1) / TB_GEMM_BM) * ((N + TB_GEMM_BN - 1) / TB_GEMM_BN);
  const bool pairs = M >= 256 && tiles >= s->sm_count;
  CUtensorMap ta, tbm;
  tb_status rc = tmap_bf16_2d(&ta, a, (uint64_t)M, (uint64_t)K, (uint64_t)K, TB_GEMM_BM, TB_GEMM_BK,
                              CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = tmap_bf16_2d(&tbm, b, (uint64_t)N, (uint64_t)K, (uint64_t)K, pairs ? 128u : (uint32_t)TB_GEMM_BN, TB_GEMM_BK,
                    CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  CUfunction fn = nullptr;
  const char* name = pairs ? "gemm_bf16_tn_allgather_2sm" : "gemm_bf16_tn_allgather";
  rc = builtin_function(s, "gemm_bf16", name, &fn);
  if (rc) return rc;
  struct {
    CUdeviceptr base[TB_MAX_RANKS];
  } rank_outputs = {}, rank_signals = {};
  for (int i = 0; i < ranks; ++i) {
    rank_outputs.base[i] = outs[i];
    rank_signals.base[i] = signals[i];
  }
  CUdeviceptr status = s->status.device;
  const long long pair_tiles = (long long)((M + 255) / 256) * ((N + 255) / 256);
  const int pushers = pairs && ranks > 1 ? allgather_pushers(ranks) : 0;
  if (pushers > 0 && ready && (size_t)(2 * pair_tiles) <= ready_count) {
    // Dedicated pusher CTAs (gemm_bf16_tn_allgather_2sm_push); tile counters zeroed first.
    CUfunction pfn = nullptr;
    rc = builtin_function(s, "gemm_bf16", "gemm_bf16_tn_allgather_2sm_push", &pfn);
    if (rc) return rc;
    int clusters = 0;
    rc = pair_occupancy(s, st, pfn, TB_GEMM2_PUSH_THREADS, TB_GEMM2_SMEM_BYTES, "gemm_bf16_tn_allgather_2sm_push",
                        &clusters);
    if (rc) return rc;
    if (clusters > pushers / 2) {
      int gemm_pairs = clusters - pushers / 2;
      if (gemm_pairs > pair_tiles) gemm_pairs = (int)pair_tiles;
      TB_CU("cuMemsetD32Async", driver()->cuMemsetD32Async(ready, 0, (size_t)(2 * pair_tiles), st->raw));
      void* pp[] = {&ta, &tbm, &rank_outputs, &rank_signals, &ranks, &self, &epoch, &M, &N, &K, &ldc, &col0,
                    &ready, &gemm_pairs, &status};
      return launch_builtin(s, st, pfn, (unsigned)(2 * gemm_pairs + pushers), 1, 1, TB_GEMM2_PUSH_THREADS,
                            TB_GEMM2_SMEM_BYTES, pp, "gemm_bf16_tn_allgather_2sm_push", 2);
    }
  }
  void* params[] = {&ta, &tbm, &rank_outputs, &rank_signals, &ranks, &self, &epoch, &M, &N, &K, &ldc, &col0, &status};
  if (pairs) {
    return launch_builtin_pairs(s, st, fn, pair_tiles, TB_GEMM2_AG_THREADS, TB_GEMM2_AG_SMEM_BYTES, params, name);
  }
  const unsigned grid = (unsigned)(tiles < s->sm_count ? tiles : s->sm_count);
  return launch_builtin(s, st, fn, grid, 1, 1, TB_GEMM_THREADS, TB_GEMM_AG_SMEM_BYTES, params, name);
}

// Split-K plan for an output with too few 128x256 tiles to fill the SMs.
struct SplitPlan {
  int splits = 1, kb_per_split = 0;
};

SplitPlan plan_split_k(int sm_count, int M, int N, int K, bool force) {
  SplitPlan p;
  const int tiles = ((M + TB_GEMM_BM - 1) / TB_GEMM_BM) * ((N + TB_GEMM_BN - 1) / TB_GEMM_BN);
  const int num_k = (K + TB_GEMM_BK - 1) / TB_GEMM_BK;
  if (!force && (tiles * 2 > sm_count || num_k < 8)) return p;
  int splits = sm_count / tiles;
  if (splits < 2) splits = 2;
  if (splits > 32) splits = 32;
  if (splits > num_k) splits = num_k;
  if (splits < 2) return p;
  p.kb_per_split = (num_k + splits - 1) / splits;
  p.splits = (num_k + p.kb_per_split - 1) / p.kb_per_split;  // every split gets >= 1 k-block
  return p;
}

tb_status launch_gemm_bf16_splitk(Session* s, Stream* st, CUdeviceptr a, CUdeviceptr b, CUdeviceptr c, int M, int N,
                                  int K, long long ldc, int splits, int kb_per_split, CUdeviceptr partial) {
  CUtensorMap ta, tbm;
  tb_status rc = tmap_bf16_2d(&ta, a, (uint64_t)M, (uint64_t)K, (uint64_t)K, TB_GEMM_BM, TB_GEMM_BK,
                              CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = tmap_bf16_2d(&tbm, b, (uint64_t)N, (uint64_t)K, (uint64_t)K, TB_GEMM_BN, TB_GEMM_BK,
                    CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  CUfunction fn = nullptr, red = nullptr;
  if ((rc = builtin_function(s, "gemm_bf16", "gemm_bf16_tn_splitk", &fn)) ||
      (rc = builtin_function(s, "gemm_bf16", "splitk_reduce_bf16", &red)))
    return rc;
  const long long units =
      (long long)((M + TB_GEMM_BM - 1) / TB_GEMM_BM) * ((N + TB_GEMM_BN - 1) / TB_GEMM_BN) * splits;
  const unsigned grid = (unsigned)(units < s->sm_count ? units : s->sm_count);
  CUdeviceptr status = s->status.device;
  void* params[] = {&ta, &tbm, &partial, &M, &N, &K, &splits, &kb_per_split, &status};
  rc = launch_builtin(s, st, fn, grid, 1, 1, TB_GEMM_THREADS, TB_GEMM_SMEM_BYTES, params, "gemm_bf16_tn_splitk");
  if (rc) return rc;
  void* rparams[] = {&partial, &c, &M, &N, &splits, &ldc};
  const unsigned long long vecs = ((unsigned long long)M * N + 3) / 4;
  unsigned long long rgrid = (vecs + 255) / 256;
  if (rgrid > (unsigned long long)s->sm_count * 16) rgrid = (unsigned long long)s->sm_count * 16;
  rc = launch_builtin(s, st, red, (unsigned)rgrid, 1, 1, 256, 0, rparams, "splitk_reduce_bf16");
  if (rc) return rc;
  note_launch("gemm_bf16_tn_splitk");
  return TB_OK;
}

}  // namespace tb

using namespace tb;

extern "C" tb_status tb_op_gemm(tb_session* session, tb_stream* stream, const tb_tensor* lhs, const tb_tensor* rhs,
                                const tb_tensor* output, const tb_attr* attrs, uint32_t num_attrs, tb_event** out) {
  Session* s = reinterpret_cast<Session*>(session);
  if (!s) return set_error(TB_ERR_INVALID, "contract", "null session");
  if (!lhs || !rhs || !output) return contract("gemm requires exactly two rank-2 inputs and one output");
  const char* candidate = nullptr;  // optional: name of a registered kernel to run (autotuning / tests)
  for (uint32_t i = 0; i < num_attrs; ++i) {
    if (attrs[i].key && strcmp(attrs[i].key, "candidate") == 0 && attrs[i].str) {
      candidate = attrs[i].str;
      continue;
    }
    if (!attrs[i].key || (strcmp(attrs[i].key, "transpose_lhs") != 0 && strcmp(attrs[i].key, "transpose_rhs") != 0))
      return contract("CUDA GEMM received unsupported attributes");
  }
  static const char* kCandidates[] = {"gemm_bf16_tn",      "gemm_bf16_tn_2sm", "gemm_bf16_nn_2sm",
                                      "gemm_bf16_ta_2sm",  "gemm_bf16_ta_nn_2sm", "gemm_bf16_tn_splitk",
                                      "gemm_bf16_staged",  "gemm_bf16_generic", "gemm_f32_tiled"};
  bool known = !candidate;
  for (const char* k : kCandidates) known = known || strcmp(candidate, k) == 0;
  if (!known)
    return contract(std::string("unknown GEMM candidate ") + candidate);
  bool tl = false, tr = false;
  for (uint32_t i = 0; i < num_attrs; ++i) {
    if (strcmp(attrs[i].key, "candidate") == 0) continue;
    if (attrs[i].str || attrs[i].value < 0 || attrs[i].value > 1)
      return contract(std::string(attrs[i].key) + " must be a bool");
    if (strcmp(attrs[i].key, "transpose_lhs") == 0) tl = attrs[i].value != 0;
    if (strcmp(attrs[i].key, "transpose_rhs") == 0) tr = attrs[i].value != 0;
  }
  const uint32_t dt = lhs->dtype;
  if (!(dt == TB_F32 || dt == TB_BF16) || rhs->dtype != dt || output->dtype != dt)
    return contract("CUDA GEMM requires F32 (or BF16) input and output tensors of one dtype");
  if (lhs->rank != 2 || rhs->rank != 2) return contract("gemm requires exactly two rank-2 inputs");
  if (!is_contiguous(lhs) || !is_contiguous(rhs)) return contract("CUDA GEMM requires contiguous rank-2 inputs");
  if (output->rank != 2 || !is_contiguous(output)) return contract("CUDA GEMM requires a contiguous rank-2 output");
  const uint64_t m = tl ? lhs->shape[1] : lhs->shape[0];
  const uint64_t k = tl ? lhs->shape[0] : lhs->shape[1];
  const uint64_t rk = tr ? rhs->shape[1] : rhs->shape[0];
  const uint64_t n = tr ? rhs->shape[0] : rhs->shape[1];
  if (k != rk) return contract("gemm inner dimensions must match");
  if (output->shape[0] != m || output->shape[1] != n) return contract("gemm output shape mismatch");
  if (m == 0 || n == 0 || k == 0) return contract("CUDA GEMM M, N, and K must be non-zero");
  if (m > 0x7fffffffull || n > 0x7fffffffull || k > 0x7fffffffull) return contract("CUDA GEMM M exceeds u32 ABI");
  Stream* st = nullptr;
  tb_status rc = check_stream(s, stream, &st);
  if (rc) return rc;
  Buffer *ba = nullptr, *bb = nullptr, *bc = nullptr;
  if ((rc = tensor_buffer(s, lhs, "gemm lhs", &ba)) || (rc = tensor_buffer(s, rhs, "gemm rhs", &bb)) ||
      (rc = tensor_buffer(s, output, "gemm output", &bc)))
    return rc;
  rc = activate(s);
  if (rc) return rc;
  int M = (int)m, N = (int)n, K = (int)k;
  // Strides of op(A) (m, k) and op(B) (k, n) in elements.
  long long as0 = tl ? 1 : (long long)lhs->shape[1], as1 = tl ? (long long)lhs->shape[1] : 1;
  long long bs0 = tr ? 1 : (long long)rhs->shape[1], bs1 = tr ? (long long)rhs->shape[1] : 1;
  CUdeviceptr pa = ba->ptr, pb = bb->ptr, pc = bc->ptr;
  CUfunction fn = nullptr;
  if (dt == TB_BF16) {
    // Storage orders other than A [M, K] x B [N, K]: the layout kernels, when every row
    // the TMA reads starts 16-byte aligned (the contiguous extent of each operand is a
    // multiple of 8 elements).
    const char* layout_kernel = layout_kernel_for(tl, tr, (uint64_t)M, (uint64_t)N, (uint64_t)K, pa | pb | pc);
    const bool layout_ok = layout_kernel != nullptr;
    const bool want_layout = candidate && (strcmp(candidate, "gemm_bf16_nn_2sm") == 0 ||
                                           strcmp(candidate, "gemm_bf16_ta_2sm") == 0 ||
                                           strcmp(candidate, "gemm_bf16_ta_nn_2sm") == 0);
    if (want_layout && (!layout_ok || strcmp(candidate, layout_kernel) != 0))
      return unsupported(std::string("candidate ") + candidate + " does not take this layout or alignment");
    // Output rows that start 16-byte aligned take the epilogue's vector stores; others are
    // written through an aligned copy by the staged path (the split-K reduction writes
    // consecutive elements from consecutive threads, so it takes any output).
    const bool c_vec = (N % 8) == 0 && (pc & 15) == 0;
    const bool big = (uint64_t)M * N * K >= (1ull << 24);
    if (layout_ok && (want_layout || (!candidate && (c_vec || !big)))) {
      rc = launch_gemm_bf16_layout_2sm(s, st, layout_kernel, tl, !tr, pa, pb, pc, M, N, K, (long long)N);
      if (rc) return rc;
      return record_event(s, st, nullptr, out);
    }
    const bool tma_ok = !tl && tr && (K % 8) == 0 && ((pa | pb | pc) & 15) == 0;
    const bool split_default = !candidate && tma_ok && plan_split_k(s->sm_count, M, N, K, false).splits >= 2;
    // Any other storage goes through the staged copies once the product is large enough
    // for the tensor cores to repay them (2^24 multiply-adds).
    const bool want_staged = candidate && strcmp(candidate, "gemm_bf16_staged") == 0;
    if (want_staged || (!candidate && big && (!tma_ok || (!c_vec && !split_default)))) {
      rc = launch_gemm_bf16_staged(s, st, pa, as0, as1, pb, bs0, bs1, pc, M, N, K);
      if (rc) return rc;
      return record_event(s, st, nullptr, out);
    }
    const bool want_generic = candidate && strcmp(candidate, "gemm_bf16_generic") == 0;
    if (candidate && !tma_ok && !want_generic)
      return unsupported(std::string("candidate ") + candidate + " does not take this layout or alignment");
    if (candidate && strcmp(candidate, "gemm_f32_tiled") == 0)
      return unsupported("candidate gemm_f32_tiled does not take BF16");
    const bool force_split = candidate && strcmp(candidate, "gemm_bf16_tn_splitk") == 0;
    const bool want_2sm = candidate && strcmp(candidate, "gemm_bf16_tn_2sm") == 0;
    const SplitPlan plan = tma_ok && !want_generic && !want_2sm && !(candidate && strcmp(candidate, "gemm_bf16_tn") == 0)
                               ? plan_split_k(s->sm_count, M, N, K, force_split)
                               : SplitPlan{};
    if (force_split && plan.splits < 2) return unsupported("candidate gemm_bf16_tn_splitk needs at least 2 k-blocks");
    if (tma_ok && !want_generic && plan.splits >= 2) {
      CUdeviceptr partial = 0;
      rc = stream_scratch(s, st, (size_t)plan.splits * M * N * sizeof(float), &partial);
      if (rc) return rc;
      rc = launch_gemm_bf16_splitk(s, st, pa, pb, pc, M, N, K, (long long)N, plan.splits, plan.kb_per_split,
                                   partial);
    } else if (want_2sm) {
      rc = launch_gemm_bf16_tn_2sm(s, st, pa, pb, pc, M, N, K, (long long)N);
    } else if (tma_ok && !want_generic && candidate) {
      rc = launch_gemm_bf16_tn(s, st, pa, pb, pc, M, N, K, (long long)N);
    } else if (tma_ok && !want_generic) {
      rc = launch_gemm_bf16_default(s, st, pa, pb, pc, M, N, K, (long long)N);
    } else {
      rc = builtin_function(s, "compat", "gemm_bf16_generic", &fn);
      if (rc) return rc;
      void* params[] = {&pa, &pb, &pc, &M, &N, &K, &as0, &as1, &bs0, &bs1};
      uint64_t total = (uint64_t)M * N;
      uint64_t grid = (total + 255) / 256;
      if (grid > (uint64_t)s->sm_count * 32) grid = (uint64_t)s->sm_count * 32;
      rc = launch_builtin(s, st, fn, (unsigned)grid, 1, 1, 256, 0, params, "gemm_bf16_generic");
    }
  } else {
    if (candidate && strcmp(candidate, "gemm_f32_tiled") != 0)
      return unsupported(std::string("candidate ") + candidate + " does not take F32");
    // 64 x 64 tiles unless that leaves most SMs idle, then 16 x 16 (same per-output
    // summation order, so the same bits).
    const long long blocks64 = (long long)((N + 63) / 64) * ((M + 63) / 64);
    const int tile = blocks64 < 2LL * s->sm_count ? 16 : 64;
    rc = builtin_function(s, "compat", tile == 16 ? "gemm_f32_tiled16" : "gemm_f32_tiled", &fn);
    if (rc) return rc;
    void* params[] = {&pa, &pb, &pc, &M, &N, &K, &as0, &as1, &bs0, &bs1};
    rc = launch_builtin(s, st, fn, (unsigned)((N + tile - 1) / tile), (unsigned)((M + tile - 1) / tile), 1, 256, 0,
                        params, "gemm_f32_tiled");
  }
  if (rc) return rc;
  return record_event(s, st, nullptr, out);
}

// "gemm.bias_act": C = act(A B^T + bias) in one tcgen05 GEMM whose epilogue adds the
// fp32 bias and applies the activation on the fp32 accumulator before the single bf16
// rounding (the GEMM-epilogue fusion of the reference's gemm, broadcast.add, gelu and
// silu operators: titan-runtime/src/lib.rs:955-989, 625-640, 3064).
extern "C" tb_status tb_op_gemm_bias_act(tb_session* session, tb_stream* stream, const tb_tensor* lhs,
                                         const tb_tensor* rhs, const tb_tensor* bias, const tb_tensor* output,
                                         const tb_attr* attrs, uint32_t num_attrs, tb_event** out) {
  Session* s = reinterpret_cast<Session*>(session);
  if (!s) return set_error(TB_ERR_INVALID, "contract", "null session");
  if (!lhs || !rhs || !output) return contract("gemm.bias_act requires two rank-2 inputs, an optional bias and one output");
  bool tl = false, tr = false;
  int act = TB_ACT_NONE;
  const char* candidate = nullptr;
  for (uint32_t i = 0; i < num_attrs; ++i) {
    const char* key = attrs[i].key;
    if (!key) return contract("gemm.bias_act received an unnamed attribute");
    if (strcmp(key, "candidate") == 0) {
      if (!attrs[i].str || (strcmp(attrs[i].str, "gemm_bf16_tn_bias_act") != 0 &&
                            strcmp(attrs[i].str, "gemm_bf16_tn_bias_act_2sm") != 0 &&
                            strcmp(attrs[i].str, "gemm_bf16_nn_2sm") != 0 && strcmp(attrs[i].str, "gemm_bf16_ta_2sm") != 0 &&
                            strcmp(attrs[i].str, "gemm_bf16_ta_nn_2sm") != 0 &&
                            strcmp(attrs[i].str, "gemm_bf16_staged") != 0))
        return contract(std::string("unknown gemm.bias_act candidate ") + (attrs[i].str ? attrs[i].str : "(null)"));
      candidate = attrs[i].str;
    } else if (strcmp(key, "activation") == 0) {
      if (!attrs[i].str) return contract("gemm.bias_act activation must be a string");
      if (strcmp(attrs[i].str, "none") == 0) act = TB_ACT_NONE;
      else if (strcmp(attrs[i].str, "gelu") == 0) act = TB_ACT_GELU;
      else if (strcmp(attrs[i].str, "silu") == 0) act = TB_ACT_SILU;
      else return contract(std::string("gemm.bias_act activation must be none, gelu or silu, not ") + attrs[i].str);
    } else if (strcmp(key, "transpose_lhs") == 0 || strcmp(key, "transpose_rhs") == 0) {
      if (attrs[i].str || attrs[i].value < 0 || attrs[i].value > 1) return contract(std::string(key) + " must be a bool");
      (strcmp(key, "transpose_lhs") == 0 ? tl : tr) = attrs[i].value != 0;
    } else {
      return contract("gemm.bias_act received unsupported attributes");
    }
  }
  if (lhs->dtype != TB_BF16 || rhs->dtype != TB_BF16 || output->dtype != TB_BF16)
    return contract("gemm.bias_act requires BF16 A, B and C");
  if (lhs->rank != 2 || rhs->rank != 2) return contract("gemm requires exactly two rank-2 inputs");
  if (!is_contiguous(lhs) || !is_contiguous(rhs) || output->rank != 2 || !is_contiguous(output))
    return contract("gemm.bias_act requires contiguous rank-2 tensors");
  const uint64_t m = tl ? lhs->shape[1] : lhs->shape[0];
  const uint64_t k = tl ? lhs->shape[0] : lhs->shape[1];
  const uint64_t rk = tr ? rhs->shape[1] : rhs->shape[0];
  const uint64_t n = tr ? rhs->shape[0] : rhs->shape[1];
  if (k != rk) return contract("gemm inner dimensions must match");
  if (output->shape[0] != m || output->shape[1] != n) return contract("gemm output shape mismatch");
  if (m == 0 || n == 0 || k == 0) return contract("CUDA GEMM M, N, and K must be non-zero");
  if (m > 0x7fffffffull || n > 0x7fffffffull || k > 0x7fffffffull) return contract("CUDA GEMM M exceeds u32 ABI");
  if (bias && (bias->dtype != TB_F32 || bias->rank != 1 || bias->shape[0] != n || !is_contiguous(bias)))
    return contract("gemm.bias_act bias must be a contiguous F32 [N] tensor");
  Stream* st = nullptr;
  tb_status rc = check_stream(s, stream, &st);
  if (rc) return rc;
  Buffer *ba = nullptr, *bb = nullptr, *bc = nullptr, *bbias = nullptr;
  if ((rc = tensor_buffer(s, lhs, "gemm lhs", &ba)) || (rc = tensor_buffer(s, rhs, "gemm rhs", &bb)) ||
      (rc = tensor_buffer(s, output, "gemm output", &bc)) || (bias && (rc = tensor_buffer(s, bias, "gemm bias", &bbias))))
    return rc;
  const CUdeviceptr pa = ba->ptr, pb = bb->ptr, pc = bc->ptr, pbias = bbias ? bbias->ptr : 0;
  int M = (int)m, N = (int)n, K = (int)k;
  // Strides of op(A) (m, k) and op(B) (k, n) in elements, for the staged path.
  const long long as0 = tl ? 1 : (long long)lhs->shape[1], as1 = tl ? (long long)lhs->shape[1] : 1;
  const long long bs0 = tr ? 1 : (long long)rhs->shape[1], bs1 = tr ? (long long)rhs->shape[1] : 1;
  const bool want_staged = candidate && strcmp(candidate, "gemm_bf16_staged") == 0;
  // Output rows that do not start 16-byte aligned are written through the staged path's
  // aligned copy of C.
  const bool c_vec = (N % 8) == 0 && (pc & 15) == 0;
  rc = activate(s);
  if (rc) return rc;
  if (tl || !tr) {
    // Other storage orders: the layout kernels, whose epilogue takes the bias and activation;
    // storage they cannot read goes through the staged copies.
    const char* lk = layout_kernel_for(tl, tr, m, n, k, pa | pb | pc);
    if (!lk || want_staged || (!candidate && !c_vec)) {
      rc = launch_gemm_bf16_staged(s, st, pa, as0, as1, pb, bs0, bs1, pc, M, N, K, true, pbias, act);
      if (rc) return rc;
      return record_event(s, st, nullptr, out);
    }
    if (candidate && strcmp(candidate, lk) != 0)
      return unsupported(std::string("candidate ") + candidate + " does not take this layout");
    rc = launch_gemm_bf16_layout_2sm(s, st, lk, tl, !tr, pa, pb, pc, M, N, K, (long long)N, pbias, act);
    if (rc) return rc;
    return record_event(s, st, nullptr, out);
  }
  if (want_staged || k % 8 != 0 || ((pa | pb | pc) & 15) != 0 || (!candidate && !c_vec)) {
    rc = launch_gemm_bf16_staged(s, st, pa, as0, as1, pb, bs0, bs1, pc, M, N, K, true, pbias, act);
    if (rc) return rc;
    return record_event(s, st, nullptr, out);
  }
  if (candidate && strcmp(candidate, "gemm_bf16_tn_bias_act") != 0 && strcmp(candidate, "gemm_bf16_tn_bias_act_2sm") != 0)
    return unsupported(std::string("candidate ") + candidate + " does not take this layout");
  rc = launch_gemm_bf16_tn_bias_act(s, st, pa, pb, pc, M, N, K, pbias, act, candidate);
  if (rc) return rc;
  return record_event(s, st, nullptr, out);
}
