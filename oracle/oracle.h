/*
 * TEST INFRASTRUCTURE ONLY: the CPU parity oracle.
 *
 * A plain-C restatement of the titan.rs CPU scalar operators that the CUDA
 * kernels in this repository must agree with. Only tests/, the smoke check
 * in __graft_entry__.py and bench.py's cpu_baseline / reference leg may
 * load it, and only as the checker or the timed CPU baseline. The product
 * path never calls it.
 *
 * Reference functions restated (paths inside the titan.rs project):
 *   softmax                       projects/titan-runtime/src/lib.rs:933-953
 *   gemm (transpose_lhs/rhs)      projects/titan-runtime/src/lib.rs:955-989
 *   conv2d (NCHW/OIHW, groups)    projects/titan-runtime/src/lib.rs:991-1088
 *   scaled_dot_product_attention  projects/titan-runtime/src/lib.rs:1090-1151
 *
 * Loop order and f32 accumulation follow those functions exactly; the file is
 * compiled with -ffp-contract=off so no multiply-add is fused (Rust does not
 * contract either), which keeps the f32 results bit-identical to the
 * reference's.
 *
 * Extensions the reference does not have (parity for these is pinned only by
 * this restatement, not by a reference test): bf16 inputs (exactly widened to
 * f32, then the same f32 loops), causal masking (query i sees keys j <= i),
 * column-major B for GEMM (== the reference's transpose_rhs), and NHWC/KRSC
 * convolution indexing. The *_points / *_rows variants evaluate the same
 * loops for a chosen subset of output elements so full-size configurations
 * can be checked in seconds.
 */
#ifndef TITAN_ORACLE_H
#define TITAN_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes: 0 ok, otherwise a contract error (message via oracle_last_error). */
const char* oracle_last_error(void);
int oracle_num_threads(void);

/* bf16 <-> f32 (round to nearest even; NaN kept quiet). */
float oracle_bf16_to_f32(uint16_t v);
uint16_t oracle_f32_to_bf16(float f);

/* rt:933-953. Softmax over `axis_len` with `outer` x `inner` independent lanes. */
int oracle_softmax_f32(const float* x, float* y, size_t outer, size_t axis_len, size_t inner);
/* Same arithmetic for a contiguous [rows, cols] tensor, rows split over threads. */
int oracle_softmax_rows_f32_mt(const float* x, float* y, size_t rows, size_t cols, int threads);

/* rt:955-989. lhs is [lhs_rows, lhs_cols], rhs is [rhs_rows, rhs_cols]. */
int oracle_gemm_f32(const float* lhs, const float* rhs, float* out, size_t lhs_rows, size_t lhs_cols,
                    size_t rhs_rows, size_t rhs_cols, int transpose_lhs, int transpose_rhs,
                    size_t out_rows, size_t out_cols);
/* Row-parallel variant of the same loops (threads <= 0: all cores). */
int oracle_gemm_f32_mt(const float* lhs, const float* rhs, float* out, size_t m, size_t n, size_t k,
                       int threads);

/* rt:991-1088. bias may be NULL. out shape must be [N, Cout, Ho, Wo]. */
int oracle_conv2d_nchw_f32(const float* x, const float* w, const float* bias, float* out,
                           size_t batch, size_t cin, size_t h, size_t wd,
                           size_t cout, size_t wcin, size_t kh, size_t kw,
                           size_t stride_h, size_t stride_w, size_t pad_h, size_t pad_w,
                           size_t dil_h, size_t dil_w, size_t groups,
                           size_t out_n, size_t out_c, size_t out_h, size_t out_w);

/* rt:1090-1151 (+ causal extension). q [B,H,Tq,D], k/v [B,H,Tk,D], out [B,H,Tq,D]. */
int oracle_sdpa_f32(const float* q, const float* k, const float* v, float* out,
                    size_t b, size_t h, size_t tq, size_t tk, size_t d, int causal);

/* ---- bf16 extensions, evaluated at selected output points ---- */

/* C[row, col] = sum_k A[row,k] * B(k,col) in f32, k ascending.
 * A is [M,K] row-major; B is column-major [K,N] (b_col_major=1, element (k,n) at n*K+k)
 * or row-major [K,N] (b_col_major=0). */
int oracle_gemm_bf16_points(const uint16_t* a, const uint16_t* bm, int b_col_major,
                            size_t m, size_t n, size_t k,
                            const int64_t* rows, const int64_t* cols, size_t npoints,
                            float* out, int threads);

/* Full rows of SDPA for selected (batch, head, query) triples, flattened as
 * ((b*H + h)*Tq + i). out is [nrows, D]. */
int oracle_sdpa_bf16_rows(const uint16_t* q, const uint16_t* k, const uint16_t* v,
                          size_t b, size_t h, size_t tq, size_t tk, size_t d, int causal,
                          float scale, const int64_t* row_ids, size_t nrows, float* out, int threads);

/* NHWC conv outputs at selected flattened indices ((n*Ho + y)*Wo + x)*Cout + co.
 * x is [N,H,W,Cin]; w is KRSC [Cout,R,S,Cin]; bias (f32, may be NULL). */
int oracle_conv2d_nhwc_bf16_points(const uint16_t* x, const uint16_t* w, const float* bias,
                                   size_t batch, size_t h, size_t wd, size_t cin,
                                   size_t cout, size_t r, size_t s,
                                   size_t stride_h, size_t stride_w, size_t pad_h, size_t pad_w,
                                   size_t dil_h, size_t dil_w, size_t out_h, size_t out_w,
                                   const int64_t* idx, size_t npoints, float* out, int threads);

/* Seeded synthetic inputs: elements [first, first + count) of the fill with `seed`
 * (SplitMix64 bits, 53-bit uniforms, Box-Muller normals), as f32 (bf16 = 0) or as
 * bf16 bit patterns rounded to nearest even (bf16 = 1). Any slice can be made alone. */
int oracle_fill_uniform(void* dst, int bf16, uint64_t first, size_t count, uint64_t seed, double low, double high,
                        int threads);
int oracle_fill_normal(void* dst, int bf16, uint64_t first, size_t count, uint64_t seed, double mean,
                       double stddev, int threads);

#ifdef __cplusplus
}
#endif
#endif
