/*
 * TEST INFRASTRUCTURE ONLY: CPU parity oracle (see oracle.h for the contract
 * and the list of titan.rs functions restated here). Build with
 * -O2 -ffp-contract=off -fno-fast-math so that every f32 multiply and add is
 * rounded separately, exactly as the Rust reference computes them.
 */
#include "oracle.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static __thread char g_error[256];

static int fail(const char* msg) {
  snprintf(g_error, sizeof g_error, "%s", msg);
  return 1;
}

const char* oracle_last_error(void) { return g_error; }

int oracle_num_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

static int resolve_threads(int threads) {
  if (threads > 0) return threads;
  return oracle_num_threads();
}

float oracle_bf16_to_f32(uint16_t v) {
  uint32_t bits = (uint32_t)v << 16;
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

uint16_t oracle_f32_to_bf16(float f) {
  uint32_t bits;
  memcpy(&bits, &f, 4);
  if ((bits & 0x7f800000u) == 0x7f800000u && (bits & 0x007fffffu) != 0) {
    return (uint16_t)((bits >> 16) | 0x0040u); /* quiet NaN */
  }
  uint32_t lsb = (bits >> 16) & 1u;
  bits += 0x7fffu + lsb; /* round to nearest, ties to even */
  return (uint16_t)(bits >> 16);
}

/* f32::max as used by `fold(f32::NEG_INFINITY, f32::max)`: NaN operands are ignored. */
static float rust_max(float a, float b) { return fmaxf(a, b); }

/* projects/titan-runtime/src/lib.rs:933-953 */
int oracle_softmax_f32(const float* x, float* y, size_t outer, size_t axis_len, size_t inner) {
  for (size_t o = 0; o < outer; ++o) {
    for (size_t in = 0; in < inner; ++in) {
      size_t base = (o * axis_len) * inner + in;
      float maximum = -INFINITY;
      for (size_t a = 0; a < axis_len; ++a) maximum = rust_max(maximum, x[base + a * inner]);
      float denominator = 0.0f;
      for (size_t a = 0; a < axis_len; ++a) denominator += expf(x[base + a * inner] - maximum);
      for (size_t a = 0; a < axis_len; ++a) y[base + a * inner] = expf(x[base + a * inner] - maximum) / denominator;
    }
  }
  return 0;
}

int oracle_softmax_rows_f32_mt(const float* x, float* y, size_t rows, size_t cols, int threads) {
  long long nrows = (long long)rows;
#pragma omp parallel for schedule(static) num_threads(resolve_threads(threads))
  for (long long r = 0; r < nrows; ++r) {
    oracle_softmax_f32(x + (size_t)r * cols, y + (size_t)r * cols, 1, cols, 1);
  }
  return 0;
}

/* projects/titan-runtime/src/lib.rs:955-989 */
int oracle_gemm_f32(const float* lhs, const float* rhs, float* out, size_t lhs_rows, size_t lhs_cols,
                    size_t rhs_rows, size_t rhs_cols, int transpose_lhs, int transpose_rhs,
                    size_t out_rows, size_t out_cols) {
  size_t m = transpose_lhs ? lhs_cols : lhs_rows;
  size_t k = transpose_lhs ? lhs_rows : lhs_cols;
  size_t rhs_k = transpose_rhs ? rhs_cols : rhs_rows;
  size_t n = transpose_rhs ? rhs_rows : rhs_cols;
  if (k != rhs_k) return fail("gemm inner dimensions must match");
  if (out_rows != m || out_cols != n) return fail("gemm output shape mismatch");
  for (size_t row = 0; row < m; ++row) {
    for (size_t column = 0; column < n; ++column) {
      float sum = 0.0f;
      for (size_t inner = 0; inner < k; ++inner) {
        size_t li = transpose_lhs ? inner * lhs_cols + row : row * lhs_cols + inner;
        size_t ri = transpose_rhs ? column * rhs_cols + inner : inner * rhs_cols + column;
        sum += lhs[li] * rhs[ri];
      }
      out[row * n + column] = sum;
    }
  }
  return 0;
}

int oracle_gemm_f32_mt(const float* lhs, const float* rhs, float* out, size_t m, size_t n, size_t k,
                       int threads) {
  long long mm = (long long)m;
#pragma omp parallel for schedule(static) num_threads(resolve_threads(threads))
  for (long long row = 0; row < mm; ++row) {
    for (size_t column = 0; column < n; ++column) {
      float sum = 0.0f;
      for (size_t inner = 0; inner < k; ++inner) sum += lhs[(size_t)row * k + inner] * rhs[inner * n + column];
      out[(size_t)row * n + column] = sum;
    }
  }
  return 0;
}

/* projects/titan-runtime/src/lib.rs:991-1088 */
int oracle_conv2d_nchw_f32(const float* x, const float* w, const float* bias, float* out,
                           size_t batch, size_t cin, size_t h, size_t wd,
                           size_t cout, size_t wcin, size_t kh, size_t kw,
                           size_t stride_h, size_t stride_w, size_t pad_h, size_t pad_w,
                           size_t dil_h, size_t dil_w, size_t groups,
                           size_t out_n, size_t out_c, size_t out_h, size_t out_w) {
  if (stride_h == 0 || stride_w == 0 || dil_h == 0 || dil_w == 0 || groups == 0)
    return fail("conv2d stride, dilation, and groups must be non-zero");
  if (cin == 0 || h == 0 || wd == 0 || cout == 0 || kh == 0 || kw == 0 || cin % groups != 0 ||
      cout % groups != 0 || wcin != cin / groups)
    return fail("conv2d channels, groups, and kernel dimensions are invalid");
  size_t eff_h = dil_h * (kh - 1) + 1, eff_w = dil_w * (kw - 1) + 1;
  size_t padded_h = h + 2 * pad_h, padded_w = wd + 2 * pad_w;
  if (eff_h > padded_h || eff_w > padded_w) return fail("conv2d kernel geometry exceeds padded input");
  size_t ho = (padded_h - eff_h) / stride_h + 1, wo = (padded_w - eff_w) / stride_w + 1;
  if (out_n != batch || out_c != cout || out_h != ho || out_w != wo) return fail("conv2d output shape mismatch");
  size_t cpg = cin / groups, opg = cout / groups;
  for (size_t n = 0; n < batch; ++n) {
    for (size_t oc = 0; oc < cout; ++oc) {
      size_t group = oc / opg;
      for (size_t oh = 0; oh < ho; ++oh) {
        for (size_t ow = 0; ow < wo; ++ow) {
          float sum = bias ? bias[oc] : 0.0f;
          for (size_t c = 0; c < cpg; ++c) {
            for (size_t r = 0; r < kh; ++r) {
              size_t ih = oh * stride_h + r * dil_h;
              if (ih < pad_h || ih - pad_h >= h) continue;
              for (size_t s = 0; s < kw; ++s) {
                size_t iw = ow * stride_w + s * dil_w;
                if (iw < pad_w || iw - pad_w >= wd) continue;
                size_t ic = group * cpg + c;
                size_t xi = ((n * cin + ic) * h + (ih - pad_h)) * wd + (iw - pad_w);
                size_t wi = ((oc * cpg + c) * kh + r) * kw + s;
                sum += x[xi] * w[wi];
              }
            }
          }
          out[((n * cout + oc) * ho + oh) * wo + ow] = sum;
        }
      }
    }
  }
  return 0;
}

/* One query row of projects/titan-runtime/src/lib.rs:1090-1151 on f32 data.
 * scores is caller-provided scratch of length tk. Causal: keys j > i are excluded. */
static void sdpa_row(const float* qrow, const float* kbase, const float* vbase, float* orow, size_t tk,
                     size_t d, float scale, size_t visible, float* scores) {
  for (size_t j = 0; j < visible; ++j) {
    float s = 0.0f;
    for (size_t e = 0; e < d; ++e) s += qrow[e] * kbase[j * d + e];
    s *= scale;
    scores[j] = s;
  }
  (void)tk;
  float maximum = -INFINITY;
  for (size_t j = 0; j < visible; ++j) maximum = rust_max(maximum, scores[j]);
  float denominator = 0.0f;
  for (size_t j = 0; j < visible; ++j) denominator += expf(scores[j] - maximum);
  for (size_t e = 0; e < d; ++e) {
    float result = 0.0f;
    for (size_t j = 0; j < visible; ++j) {
      float weight = expf(scores[j] - maximum) / denominator;
      result += weight * vbase[j * d + e];
    }
    orow[e] = result;
  }
}

int oracle_sdpa_f32(const float* q, const float* k, const float* v, float* out,
                    size_t b, size_t h, size_t tq, size_t tk, size_t d, int causal) {
  if (tq == 0 || tk == 0 || d == 0)
    return fail("scaled dot-product attention requires non-zero Tq, Tk, and D dimensions");
  float scale = 1.0f / sqrtf((float)d);
  float* scores = (float*)malloc(sizeof(float) * tk);
  if (!scores) return fail("out of memory");
  for (size_t bi = 0; bi < b; ++bi) {
    for (size_t hi = 0; hi < h; ++hi) {
      const float* kb = k + (bi * h + hi) * tk * d;
      const float* vb = v + (bi * h + hi) * tk * d;
      for (size_t i = 0; i < tq; ++i) {
        size_t visible = causal ? (i + 1 < tk ? i + 1 : tk) : tk;
        sdpa_row(q + ((bi * h + hi) * tq + i) * d, kb, vb, out + ((bi * h + hi) * tq + i) * d, tk, d, scale,
                 visible, scores);
      }
    }
  }
  free(scores);
  return 0;
}

int oracle_gemm_bf16_points(const uint16_t* a, const uint16_t* bm, int b_col_major,
                            size_t m, size_t n, size_t k,
                            const int64_t* rows, const int64_t* cols, size_t npoints,
                            float* out, int threads) {
  long long np = (long long)npoints;
  int bad = 0;
#pragma omp parallel for schedule(dynamic, 16) num_threads(resolve_threads(threads)) reduction(| : bad)
  for (long long p = 0; p < np; ++p) {
    int64_t row = rows[p], col = cols[p];
    if (row < 0 || col < 0 || (size_t)row >= m || (size_t)col >= n) {
      bad = 1;
      continue;
    }
    float sum = 0.0f;
    const uint16_t* arow = a + (size_t)row * k;
    if (b_col_major) {
      const uint16_t* bcol = bm + (size_t)col * k;
      for (size_t kk = 0; kk < k; ++kk) sum += oracle_bf16_to_f32(arow[kk]) * oracle_bf16_to_f32(bcol[kk]);
    } else {
      for (size_t kk = 0; kk < k; ++kk) sum += oracle_bf16_to_f32(arow[kk]) * oracle_bf16_to_f32(bm[kk * n + col]);
    }
    out[p] = sum;
  }
  return bad ? fail("gemm point out of range") : 0;
}

int oracle_sdpa_bf16_rows(const uint16_t* q, const uint16_t* k, const uint16_t* v,
                          size_t b, size_t h, size_t tq, size_t tk, size_t d, int causal,
                          float scale, const int64_t* row_ids, size_t nrows, float* out, int threads) {
  if (tq == 0 || tk == 0 || d == 0)
    return fail("scaled dot-product attention requires non-zero Tq, Tk, and D dimensions");
  if (!(scale > 0.0f)) scale = 1.0f / sqrtf((float)d);
  long long nr = (long long)nrows;
  int bad = 0;
#pragma omp parallel num_threads(resolve_threads(threads)) reduction(| : bad)
  {
    float* scores = (float*)malloc(sizeof(float) * tk);
    float* kf = (float*)malloc(sizeof(float) * tk * d);
    float* vf = (float*)malloc(sizeof(float) * tk * d);
    float* qf = (float*)malloc(sizeof(float) * d);
    if (!scores || !kf || !vf || !qf) bad = 1;
    int64_t cached_bh = -1;
#pragma omp for schedule(dynamic, 1)
    for (long long p = 0; p < nr; ++p) {
      if (bad) continue;
      int64_t id = row_ids[p];
      if (id < 0 || (size_t)id >= b * h * tq) {
        bad = 1;
        continue;
      }
      size_t i = (size_t)id % tq;
      int64_t bh = id / (int64_t)tq;
      size_t visible = causal ? (i + 1 < tk ? i + 1 : tk) : tk;
      if (bh != cached_bh) {
        /* Widen this (b,h)'s K and V once; row ids sorted by (b,h) reuse it. */
        const uint16_t* kb = k + (size_t)bh * tk * d;
        const uint16_t* vb = v + (size_t)bh * tk * d;
        for (size_t t = 0; t < tk * d; ++t) {
          kf[t] = oracle_bf16_to_f32(kb[t]);
          vf[t] = oracle_bf16_to_f32(vb[t]);
        }
        cached_bh = bh;
      }
      for (size_t e = 0; e < d; ++e) qf[e] = oracle_bf16_to_f32(q[(size_t)id * d + e]);
      sdpa_row(qf, kf, vf, out + (size_t)p * d, tk, d, scale, visible, scores);
    }
    free(scores);
    free(kf);
    free(vf);
    free(qf);
  }
  return bad ? fail("sdpa row id out of range or allocation failed") : 0;
}

int oracle_conv2d_nhwc_bf16_points(const uint16_t* x, const uint16_t* w, const float* bias,
                                   size_t batch, size_t h, size_t wd, size_t cin,
                                   size_t cout, size_t r, size_t s,
                                   size_t stride_h, size_t stride_w, size_t pad_h, size_t pad_w,
                                   size_t dil_h, size_t dil_w, size_t out_h, size_t out_w,
                                   const int64_t* idx, size_t npoints, float* out, int threads) {
  long long np = (long long)npoints;
  int bad = 0;
#pragma omp parallel for schedule(dynamic, 16) num_threads(resolve_threads(threads)) reduction(| : bad)
  for (long long p = 0; p < np; ++p) {
    int64_t id = idx[p];
    if (id < 0 || (size_t)id >= batch * out_h * out_w * cout) {
      bad = 1;
      continue;
    }
    size_t co = (size_t)id % cout;
    size_t rest = (size_t)id / cout;
    size_t ox = rest % out_w;
    rest /= out_w;
    size_t oy = rest % out_h;
    size_t n = rest / out_h;
    /* Same accumulation order as the NCHW reference: channel, then kernel row, then column. */
    float sum = bias ? bias[co] : 0.0f;
    for (size_t c = 0; c < cin; ++c) {
      for (size_t kr = 0; kr < r; ++kr) {
        size_t ih = oy * stride_h + kr * dil_h;
        if (ih < pad_h || ih - pad_h >= h) continue;
        for (size_t ks = 0; ks < s; ++ks) {
          size_t iw = ox * stride_w + ks * dil_w;
          if (iw < pad_w || iw - pad_w >= wd) continue;
          float xv = oracle_bf16_to_f32(x[((n * h + (ih - pad_h)) * wd + (iw - pad_w)) * cin + c]);
          float wv = oracle_bf16_to_f32(w[((co * r + kr) * s + ks) * cin + c]);
          sum += xv * wv;
        }
      }
    }
    out[p] = sum;
  }
  return bad ? fail("conv2d point out of range") : 0;
}

/* ---- seeded synthetic inputs ----
 * The counter-based generator of the benchmark inputs, restated so the CPU-side
 * legs (the reference arm, the checker) can make the same tensors without the
 * product library. Element i depends only on (seed, i): SplitMix64's finaliser
 * (Steele, Lea and Flood, "Fast splittable pseudorandom number generators",
 * OOPSLA 2014) of key + (i + 1) * golden-ratio increment gives 64 bits; a uniform
 * takes the top 53 bits; normals are the Box-Muller pair (Box and Muller 1958) of
 * elements (2j, 2j + 1), cos for the even element and sin for the odd one. */
static uint64_t sm64_mix(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

static double sm64_unit(uint64_t key, uint64_t i) {
  const uint64_t bits = sm64_mix(key + (i + 1) * 0x9E3779B97F4A7C15ull);
  return (double)(bits >> 11) * (1.0 / 9007199254740992.0);
}

static void fill_store(void* dst, int bf16, size_t j, double v) {
  const float f = (float)v;
  if (bf16)
    ((uint16_t*)dst)[j] = oracle_f32_to_bf16(f);
  else
    ((float*)dst)[j] = f;
}

int oracle_fill_uniform(void* dst, int bf16, uint64_t first, size_t count, uint64_t seed, double low, double high,
                        int threads) {
  if (!dst && count) return fail("null destination");
  const uint64_t key = sm64_mix(seed ^ 0x5851F42D4C957F2Dull);
  const int t = resolve_threads(threads);
#pragma omp parallel for num_threads(t) schedule(static)
  for (size_t j = 0; j < count; ++j) fill_store(dst, bf16, j, low + (high - low) * sm64_unit(key, first + j));
  return 0;
}

int oracle_fill_normal(void* dst, int bf16, uint64_t first, size_t count, uint64_t seed, double mean,
                       double stddev, int threads) {
  if (!dst && count) return fail("null destination");
  const uint64_t key = sm64_mix(seed ^ 0x2545F4914F6CDD1Dull);
  const double two_pi = 6.283185307179586476925286766559;
  const int t = resolve_threads(threads);
#pragma omp parallel for num_threads(t) schedule(static)
  for (size_t j = 0; j < count; ++j) {
    const uint64_t i = first + j, pair = i & ~(uint64_t)1;
    const double u1 = 1.0 - sm64_unit(key, pair); /* (0, 1] */
    const double u2 = sm64_unit(key, pair + 1);
    const double r = sqrt(-2.0 * log(u1));
    const double z = (i & 1) ? r * sin(two_pi * u2) : r * cos(two_pi * u2);
    fill_store(dst, bf16, j, mean + stddev * z);
  }
  return 0;
}

