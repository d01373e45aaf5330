// Launch constants shared by the sm_100a kernels and the host code that launches them.
#pragma once

// bf16 GEMM (gemm_bf16.cu): 128x256x64 tiles, 4 smem stages, 192 threads.
#define TB_GEMM_BM 128
#define TB_GEMM_BN 256
#define TB_GEMM_BK 64
#define TB_GEMM_STAGES 4
#define TB_GEMM_THREADS 192
#define TB_GEMM_BARRIER_BYTES 128
#define TB_GEMM_SMEM_BYTES (TB_GEMM_STAGES * (TB_GEMM_BM + TB_GEMM_BN) * TB_GEMM_BK * 2 + 1024 + TB_GEMM_BARRIER_BYTES)

// 2-SM bf16 GEMM (gemm_bf16_tn_2sm): CTA pairs computing 256x256 tiles with
// tcgen05.mma.cta_group::2; 32 KB per-CTA stages, pair tiles visited in groups of
// TB_GEMM2_GROUP 256-row blocks.
#define TB_GEMM2_STAGES 6
#define TB_GEMM2_GROUP 8
#define TB_GEMM2_BARRIER_BYTES 256
#define TB_GEMM2_SMEM_BYTES (TB_GEMM2_STAGES * 2 * 128 * TB_GEMM_BK * 2 + 1024 + TB_GEMM2_BARRIER_BYTES)

// Ranks the fused GEMM + all-gather writes to (one node), and its epilogue staging:
// 4 warps x 32 rows x 128 bf16 columns beyond the pipeline's shared memory.
#define TB_MAX_RANKS 8
#define TB_SIGNAL_BLOCK_BYTES 128
#define TB_GEMM_AG_STAGE_BYTES (4 * 32 * 256)
#define TB_GEMM_AG_SMEM_BYTES (TB_GEMM_SMEM_BYTES + TB_GEMM_AG_STAGE_BYTES)
// Fused all-gather on CTA pairs: 5 ring stages + 128 B of slot barriers + eight
// 8 KB staging slots, and four push warps beside the six pipeline warps.
#define TB_GEMM2_AG_STAGES 5
#define TB_GEMM2_AG_SMEM_BYTES (TB_GEMM2_AG_STAGES * 2 * 128 * TB_GEMM_BK * 2 + 1024 + TB_GEMM2_BARRIER_BYTES + 128 + 8 * 32 * 256)
#define TB_GEMM2_AG_THREADS (TB_GEMM_THREADS + 4 * 32)
// Fused all-gather with dedicated pusher CTAs: 16 warps per CTA (the pipeline uses
// six of them in GEMM CTAs; pusher CTAs use all sixteen for peer stores).
#define TB_GEMM2_PUSH_THREADS 512

// Causal SDPA forward (sdpa_bf16.cu): 128-row query tiles, 128-key tiles, head dim 128.
// Shared memory: Q 32 KB + K ring 2x32 KB + V ring 2x32 KB + P 2x32 KB + barriers.
#define TB_SDPA_BM 128
#define TB_SDPA_BN 128
#define TB_SDPA_HD 128
#define TB_SDPA_THREADS 192
#define TB_SDPA_BARRIER_BYTES 256
#define TB_SDPA_SMEM_BYTES (7 * 32768 + TB_SDPA_BARRIER_BYTES + 1024)

// Two-query-tile SDPA (sdpa_bf16_pair.cu, sdpa_bf16_persist.cu): Q 2x32 KB + a 2-stage
// ring of K and V tiles (2 x 64 KB) + barriers; P lives in tensor memory. Three
// warpgroups (control: producer, MMA and two idle warps; softmax A; softmax B), with
// registers moved from the control warpgroup to the softmax ones: 384 threads launched
// at TB_SDPA2_PAIR_LAUNCH_REGS registers = 128 x TB_SDPA2_PAIR_CONTROL_REGS + 256 x
// TB_SDPA2_PAIR_SOFTMAX_REGS.
#define TB_SDPA2_BARRIER_BYTES 256
#define TB_SDPA2_SMEM_BYTES (6 * 32768 + TB_SDPA2_BARRIER_BYTES + 1024)
#define TB_SDPA2_PAIR_THREADS 384
#define TB_SDPA2_PAIR_LAUNCH_REGS 168
#define TB_SDPA2_PAIR_CONTROL_REGS 56
#define TB_SDPA2_PAIR_SOFTMAX_REGS 216

// 64-key-tile SDPA (sdpa_bf16_bn64.cu), two CTAs per SM: Q 32 KB + K ring 2x16 KB +
// V ring 2x16 KB + barriers; 256 TMEM columns per CTA.
#define TB_SDPA3_BN 64
#define TB_SDPA3_THREADS 192
#define TB_SDPA3_BARRIER_BYTES 256
#define TB_SDPA3_SMEM_BYTES (32768 + 4 * 16384 + TB_SDPA3_BARRIER_BYTES + 1024)

// Epilogue activations (epilogue_math.cuh), shared with the host operators.
#define TB_ACT_NONE 0
#define TB_ACT_GELU 1
#define TB_ACT_SILU 2
