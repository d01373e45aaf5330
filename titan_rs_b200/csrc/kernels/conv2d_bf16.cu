// Conv2d forward, bf16 NHWC input, KRSC weights, fp32 accumulation, bf16 NHWC
// output (+ optional fp32 bias), as an implicit GEMM on the tensor cores.
//
// Semantics follow the titan.rs CPU reference (projects/titan-runtime/src/lib.rs:991-1088):
// zero padding, stride, dilation, optional bias; groups == 1 on this path.
//
//   GEMM view: M = N*Ho*Wo output pixels, N = Cout, K = R*S*Cin.
//   An M tile is 128 output pixels laid out as 2 images x 8 output rows x 8
//   output columns. For k-block (r, s, c0) its A tile is ONE 4-D TMA box of the
//   NHWC input: {64 channels from c0, 8 columns from wo0*sw - pw + s*dw,
//   8 rows from ho0*sh - ph + r*dh, 2 images from n0}, traversal strides
//   {1, sw, sh, 1}. TMA writes it as 128 rows of 128 bytes in (n, h, w) order with
//   the 128-byte swizzle, which is exactly the K-major operand layout; padding
//   comes for free because out-of-range (also negative) coordinates read zeros.
//   The B tile is a 3-D box {64 channels, 1 filter tap, 256 output channels} of
//   the weights viewed as [Cout][R*S][Cin]; its channel tail also reads zeros.
// The shared pipeline (umma_pipeline.cuh) does the rest; the epilogue writes
// each accumulator row to its NHWC output pixel, 32 channels per 128-bit burst.
#include "umma_pipeline.cuh"
#include "umma_pipeline_2sm.cuh"

namespace {

using namespace tb;

constexpr uint32_t kFailConv = 0x43000000u;
constexpr uint32_t kFailConv2 = 0x43320000u;

// Output-pixel cursor shared by both forms: the pixel of row `row` of M block m_blk at
// the tile's first channel, or null outside the output.
struct ConvStorer {
  __nv_bfloat16* dst;
  const float* bias;
  int cols;  // valid channels from the tile's first channel
  bool vec_ok;
  __device__ void store(int col, const uint32_t (&acc)[32]) const {
    if (!dst || col >= cols) return;
    umma::store_bf16_chunk(dst + col, cols - col, vec_ok, acc, bias ? bias + col : nullptr);
  }
};

// Problem geometry shared by the 1-SM and 2-SM policies. A 128-row M block m_blk is
// 2 images x 8 output rows x 8 output columns.
struct ConvGeometry {
  const CUtensorMap* tx;
  const CUtensorMap* tw;
  __nv_bfloat16* y;
  const float* bias;
  int batch, C, Cout, R, S, Ho, Wo, sh, sw, ph, pw, dh, dw;
  int tiles_img, tiles_h, tiles_w, c_blocks, num_n;
  bool vec_ok;

  __device__ int num_m() const { return tiles_img * tiles_h * tiles_w; }
  __device__ void prefetch() const {
    tma_prefetch_desc(tx);
    tma_prefetch_desc(tw);
  }
  __device__ void pixel_tile(int m_blk, int& n0, int& ho0, int& wo0) const {
    const int wi = m_blk % tiles_w;
    const int hi = (m_blk / tiles_w) % tiles_h;
    const int ni = m_blk / (tiles_w * tiles_h);
    n0 = ni * 2;
    ho0 = hi * 8;
    wo0 = wi * 8;
  }
  // Row `row` of M block m_blk is output pixel (n, ho, wo); channels from co.
  __device__ ConvStorer conv_storer(int row, int m_blk, int co) const {
    int n0, ho0, wo0;
    pixel_tile(m_blk, n0, ho0, wo0);
    const int n = n0 + (row >> 6), ho = ho0 + ((row >> 3) & 7), wo = wo0 + (row & 7);
    const bool in = n < batch && ho < Ho && wo < Wo;
    return ConvStorer{in ? y + (((long long)n * Ho + ho) * Wo + wo) * Cout + co : nullptr, bias ? bias + co : nullptr,
                      Cout - co, vec_ok};
  }
};

// Walks k-blocks in the order kb = (r * S + s) * c_blocks + cb with counters; Pair
// selects the 2-SM tensor loads (completion on the even CTA's barrier).
template <bool Pair>
struct ConvLoader {
  const CUtensorMap *tx, *tw;
  int w0, h0, n0, co;  // input box origin for tap (0, 0); first output channel
  int r, s, cb, rs;    // current tap and channel block
  int S, c_blocks, dh, dw;
  template <class Bar>
  __device__ void load(uint8_t* a_dst, uint8_t* b_dst, Bar bar) {
    if constexpr (Pair) {
      umma2::tma_load_4d_pair(a_dst, tx, bar, cb * 64, w0 + s * dw, h0 + r * dh, n0);
      umma2::tma_load_3d_pair(b_dst, tw, bar, cb * 64, rs, co);
    } else {
      tma_load_4d(a_dst, tx, bar, cb * 64, w0 + s * dw, h0 + r * dh, n0);
      tma_load_3d(b_dst, tw, bar, cb * 64, rs, co);
    }
    if (++cb == c_blocks) {
      cb = 0;
      ++rs;
      if (++s == S) {
        s = 0;
        ++r;
      }
    }
  }
};

struct ConvPolicy : ConvGeometry {
  __device__ int num_tiles() const { return num_m() * num_n; }
  __device__ void k_blocks(int, int& kb0, int& kb1) const {
    kb0 = 0;
    kb1 = R * S * c_blocks;
  }
  __device__ void tile(int t, int& m_blk, int& n_blk) const {
    umma::grouped_tile(t, num_m(), num_n, 16, m_blk, n_blk);
  }
  __device__ ConvLoader<false> loader(int, int m_blk, int n_blk, int) const {
    int n0, ho0, wo0;
    pixel_tile(m_blk, n0, ho0, wo0);
    return ConvLoader<false>{tx, tw, wo0 * sw - pw, ho0 * sh - ph, n0, n_blk * umma::BN, 0, 0, 0, 0,
                             S, c_blocks, dh, dw};
  }
  __device__ ConvStorer storer(int row, int, int m_blk, int n_blk) const {
    return conv_storer(row, m_blk, n_blk * umma::BN);
  }
  __device__ void finish() const {}
};

// The 2-SM form: each CTA of a pair loads its own 128-pixel input box and its half
// (128 output channels) of the 256-channel weight box; the weight map's box is
// {64, 1, 128}. The odd CTA of a final pair past the last M block reads zeros and
// stores nothing.
struct Conv2Policy : ConvGeometry, umma2::PolicyBase {
  __device__ int m_blocks() const { return num_m(); }
  __device__ int n_blocks() const { return num_n; }
  __device__ int k_blocks() const { return R * S * c_blocks; }
  __device__ ConvLoader<true> loader(int m_blk, int n_blk, int half) const {
    int n0, ho0, wo0;
    pixel_tile(m_blk, n0, ho0, wo0);
    return ConvLoader<true>{tx, tw, wo0 * sw - pw, ho0 * sh - ph, n0, n_blk * umma2::BN + half * 128, 0, 0, 0, 0,
                            S, c_blocks, dh, dw};
  }
  __device__ ConvStorer storer(int row, int m_blk, int n_blk, int, uint32_t*) const {
    return conv_storer(row, m_blk, n_blk * umma2::BN);
  }
};

}  // namespace

// Fills the geometry from the kernel arguments (identical for both forms).
__device__ __forceinline__ void conv_geometry(ConvGeometry& p, const CUtensorMap* tx, const CUtensorMap* tw,
                                              __nv_bfloat16* y, const float* bias, int batch, int C, int Cout, int R,
                                              int S, int Ho, int Wo, int sh, int sw, int ph, int pw, int dh, int dw) {
  p.tx = tx;
  p.tw = tw;
  p.y = y;
  p.bias = bias;
  p.batch = batch;
  p.C = C;
  p.Cout = Cout;
  p.R = R;
  p.S = S;
  p.Ho = Ho;
  p.Wo = Wo;
  p.sh = sh;
  p.sw = sw;
  p.ph = ph;
  p.pw = pw;
  p.dh = dh;
  p.dw = dw;
  p.tiles_img = (batch + 1) / 2;
  p.tiles_h = (Ho + 7) / 8;
  p.tiles_w = (Wo + 7) / 8;
  p.c_blocks = (C + 63) / 64;
  p.num_n = (Cout + 255) / 256;
  p.vec_ok = (Cout % 8) == 0 && (reinterpret_cast<uintptr_t>(y) & 15) == 0;
}

// x: 4-D map {C, W, H, N}, box {64, 8*sw, 8*sh, 2}, element strides {1, sw, sh, 1};
// w: 3-D map {C, R*S, Cout}, box {64, 1, 256}; both 128-byte swizzled.
extern "C" __global__ void __launch_bounds__(TB_GEMM_THREADS, 1)
    conv2d_fprop_bf16_nhwc(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_w,
                           __nv_bfloat16* __restrict__ y, const float* __restrict__ bias, int batch, int C, int Cout,
                           int R, int S, int Ho, int Wo, int sh, int sw, int ph, int pw, int dh, int dw,
                           uint32_t* status) {
  ConvPolicy p;
  conv_geometry(p, &tmap_x, &tmap_w, y, bias, batch, C, Cout, R, S, Ho, Wo, sh, sw, ph, pw, dh, dw);
  umma::run(p, status, kFailConv);
}

// The same convolution on CTA pairs (launched with clusters of 2 along x); the weight
// map's box is {64, 1, 128}.
extern "C" __global__ void __launch_bounds__(TB_GEMM_THREADS, 1)
    conv2d_fprop_bf16_nhwc_2sm(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_w,
                               __nv_bfloat16* __restrict__ y, const float* __restrict__ bias, int batch, int C,
                               int Cout, int R, int S, int Ho, int Wo, int sh, int sw, int ph, int pw, int dh, int dw,
                               uint32_t* status) {
  Conv2Policy p;
  conv_geometry(p, &tmap_x, &tmap_w, y, bias, batch, C, Cout, R, S, Ho, Wo, sh, sw, ph, pw, dh, dw);
  umma2::run(p, status, kFailConv2);
}
