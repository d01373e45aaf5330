// CUDA-core kernels for the titan.rs f32 operator ABIs and for shapes the
// tensor-core paths do not take. They are here so that every request the
// reference accepts still runs on the GPU; the B200 hot path is the bf16
// tcgen05 kernels and the fp32 softmax.
//
//   gemm_f32        reference ABI (A, B, C, M, N, K), row-major,
//                   titan-backend-cuda/src/lib.rs:663-677; any launch geometry.
//   gemm_f32_tiled  64x64 tiles, 4x4 outputs per thread, transposes via strides.
//   gemm_bf16_generic  bf16 in/out, f32 accumulate, any strides.
//   conv2d_f32      reference ABI (x, w, bias, y + 17 i32), NCHW/OIHW, groups,
//                   dilation, stride, padding, optional bias (lib.rs:680-709).
//   scaled_dot_product_attention_f32  reference ABI (Q, K, V, O, B, H, Tq, Tk, D),
//                   one warp per query row with an online softmax.
//
// The GEMM and conv2d kernels accumulate in the reference's loop order with
// separately rounded multiplies and adds (__fmul_rn / __fadd_rn), the same
// arithmetic as the Rust CPU loops (projects/titan-runtime/src/lib.rs:955-1088),
// so their results equal the CPU reference bit for bit.
#include <cuda_bf16.h>
#include <math.h>
#include <stdint.h>

namespace {

__device__ __forceinline__ float mul_add_unfused(float acc, float a, float b) { return __fadd_rn(acc, __fmul_rn(a, b)); }

// Element (r, c) of a rank-2 matrix with strides (rs, cs).
template <typename T>
__device__ __forceinline__ float ld(const T* p, long long r, long long c, long long rs, long long cs);
template <>
__device__ __forceinline__ float ld<float>(const float* p, long long r, long long c, long long rs, long long cs) {
  return p[r * rs + c * cs];
}
template <>
__device__ __forceinline__ float ld<__nv_bfloat16>(const __nv_bfloat16* p, long long r, long long c, long long rs,
                                                   long long cs) {
  return __bfloat162float(p[r * rs + c * cs]);
}

}  // namespace

extern "C" __global__ void gemm_f32(const float* __restrict__ a, const float* __restrict__ b, float* __restrict__ c,
                                    int M, int N, int K) {
  const long long total = (long long)M * N;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long row = i / N, col = i % N;
    float sum = 0.f;
    for (int k = 0; k < K; ++k) sum = mul_add_unfused(sum, a[row * K + k], b[(long long)k * N + col]);
    c[i] = sum;
  }
}

// C[M,N] = op(A) op(B); A element (m,k) at a[m*as0 + k*as1], B element (k,n) at b[k*bs0 + n*bs1].
// A block computes a TM x TM tile with 256 threads, each an RM x RM patch, stepping K by
// KS through shared memory; every output still adds its products in ascending k, each
// rounded before the add (the reference's loop), whatever the tile size.
template <int TM, int RM, int KS>
__device__ __forceinline__ void gemm_f32_tile(const float* __restrict__ a, const float* __restrict__ b,
                                              float* __restrict__ c, int M, int N, int K, long long as0,
                                              long long as1, long long bs0, long long bs1) {
  static_assert((TM / RM) * (TM / RM) == 256, "256 threads per block");
  __shared__ float As[KS][TM + 1];
  __shared__ float Bs[KS][TM + 1];
  constexpr int TPR = TM / RM;  // threads per tile row
  const int tx = threadIdx.x % TPR, ty = threadIdx.x / TPR;
  const int m0 = blockIdx.y * TM, n0 = blockIdx.x * TM;
  float acc[RM][RM] = {};
  for (int k0 = 0; k0 < K; k0 += KS) {
    for (int i = threadIdx.x; i < KS * TM; i += 256) {
      const int kk = i / TM, mm = i % TM;
      const int m = m0 + mm, k = k0 + kk;
      As[kk][mm] = (m < M && k < K) ? a[(long long)m * as0 + (long long)k * as1] : 0.f;
      const int n = n0 + mm;
      Bs[kk][mm] = (n < N && k < K) ? b[(long long)k * bs0 + (long long)n * bs1] : 0.f;
    }
    __syncthreads();
    const int kmax = min(KS, K - k0);
    for (int kk = 0; kk < kmax; ++kk) {
#pragma unroll
      for (int i = 0; i < RM; ++i)
#pragma unroll
        for (int j = 0; j < RM; ++j)
          acc[i][j] = mul_add_unfused(acc[i][j], As[kk][ty * RM + i], Bs[kk][tx * RM + j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < RM; ++i)
#pragma unroll
    for (int j = 0; j < RM; ++j) {
      const int m = m0 + ty * RM + i, n = n0 + tx * RM + j;
      if (m < M && n < N) c[(long long)m * N + n] = acc[i][j];
    }
}

// 64 x 64 tiles: outputs large enough to give every SM blocks.
extern "C" __global__ void __launch_bounds__(256) gemm_f32_tiled(const float* __restrict__ a,
                                                                 const float* __restrict__ b, float* __restrict__ c,
                                                                 int M, int N, int K, long long as0, long long as1,
                                                                 long long bs0, long long bs1) {
  gemm_f32_tile<64, 4, 16>(a, b, c, M, N, K, as0, as1, bs0, bs1);
}

// 16 x 16 tiles, one output per thread, K in steps of 64 (fewer load-and-barrier
// rounds for a thread's single chain of products): small outputs (C1's 256 x 256 is 256
// blocks instead of 16).
extern "C" __global__ void __launch_bounds__(256) gemm_f32_tiled16(const float* __restrict__ a,
                                                                   const float* __restrict__ b, float* __restrict__ c,
                                                                   int M, int N, int K, long long as0, long long as1,
                                                                   long long bs0, long long bs1) {
  gemm_f32_tile<16, 1, 64>(a, b, c, M, N, K, as0, as1, bs0, bs1);
}

extern "C" __global__ void gemm_bf16_generic(const __nv_bfloat16* __restrict__ a, const __nv_bfloat16* __restrict__ b,
                                             __nv_bfloat16* __restrict__ c, int M, int N, int K, long long as0,
                                             long long as1, long long bs0, long long bs1) {
  const long long total = (long long)M * N;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long row = i / N, col = i % N;
    float sum = 0.f;
    for (int k = 0; k < K; ++k) sum = fmaf(ld(a, row, k, as0, as1), ld(b, (long long)k, col, bs0, bs1), sum);
    c[i] = __float2bfloat16_rn(sum);
  }
}

extern "C" __global__ void conv2d_f32(const float* __restrict__ x, const float* __restrict__ w,
                                      const float* __restrict__ bias, float* __restrict__ y, int batch, int cin, int h,
                                      int wd, int cout, int kh, int kw, int ho, int wo, int sh, int sw, int ph, int pw,
                                      int dh, int dw, int groups, int has_bias) {
  const long long total = (long long)batch * cout * ho * wo;
  const int cpg = cin / groups, opg = cout / groups;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int ow = (int)(i % wo);
    const int oh = (int)((i / wo) % ho);
    const int oc = (int)((i / ((long long)wo * ho)) % cout);
    const int n = (int)(i / ((long long)wo * ho * cout));
    const int group = oc / opg;
    float sum = has_bias ? bias[oc] : 0.f;
    for (int ci = 0; ci < cpg; ++ci) {
      for (int r = 0; r < kh; ++r) {
        const int ih = oh * sh + r * dh - ph;
        if (ih < 0 || ih >= h) continue;
        for (int s = 0; s < kw; ++s) {
          const int iw = ow * sw + s * dw - pw;
          if (iw < 0 || iw >= wd) continue;
          const int ic = group * cpg + ci;
          sum = mul_add_unfused(sum, x[(((long long)n * cin + ic) * h + ih) * wd + iw],
                                w[(((long long)oc * cpg + ci) * kh + r) * kw + s]);
        }
      }
    }
    y[i] = sum;
  }
}

// One warp per query row, online softmax over the keys; D <= 256 (8 values per lane).
extern "C" __global__ void scaled_dot_product_attention_f32(const float* __restrict__ q, const float* __restrict__ k,
                                                            const float* __restrict__ v, float* __restrict__ o, int B,
                                                            int H, int Tq, int Tk, int D) {
  const int lane = threadIdx.x & 31;
  const long long rows = (long long)B * H * Tq;
  const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
  const float scale = 1.0f / sqrtf((float)D);
  for (long long row = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); row < rows; row += warps) {
    const long long bh = row / Tq;
    const float* qr = q + row * D;
    const float* kb = k + bh * (long long)Tk * D;
    const float* vb = v + bh * (long long)Tk * D;
    float qv[8], acc[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int d = lane + 32 * j;
      qv[j] = d < D ? qr[d] : 0.f;
      acc[j] = 0.f;
    }
    float m = -INFINITY, l = 0.f;
    for (int t = 0; t < Tk; ++t) {
      float part = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int d = lane + 32 * j;
        if (d < D) part = fmaf(qv[j], kb[(long long)t * D + d], part);
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) part += __shfl_xor_sync(0xffffffffu, part, off);
      const float s = part * scale;
      const float mn = fmaxf(m, s);
      const float corr = expf(m - mn);
      const float p = expf(s - mn);
      l = l * corr + p;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int d = lane + 32 * j;
        if (d < D) acc[j] = fmaf(p, vb[(long long)t * D + d], acc[j] * corr);
      }
      m = mn;
    }
    const float inv = 1.0f / l;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int d = lane + 32 * j;
      if (d < D) o[row * D + d] = acc[j] * inv;
    }
  }
}

// bf16 NHWC conv for shapes the implicit-GEMM kernel does not take (groups,
// channel counts that are not multiples of 8, strides above 1): one thread per
// output element, fp32 accumulation, optional fp32 bias. x [N,H,W,C],
// w [Cout,R,S,C/groups], y [N,Ho,Wo,Cout].
extern "C" __global__ void conv2d_bf16_nhwc_generic(const __nv_bfloat16* __restrict__ x,
                                                    const __nv_bfloat16* __restrict__ w,
                                                    const float* __restrict__ bias, __nv_bfloat16* __restrict__ y,
                                                    int batch, int h, int wd, int cin, int cout, int kh, int kw,
                                                    int ho, int wo, int sh, int sw, int ph, int pw, int dh, int dw,
                                                    int groups) {
  const long long total = (long long)batch * ho * wo * cout;
  const int cpg = cin / groups, opg = cout / groups;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int oc = (int)(i % cout);
    const long long pix = i / cout;
    const int ow = (int)(pix % wo);
    const int oh = (int)((pix / wo) % ho);
    const int n = (int)(pix / ((long long)wo * ho));
    const int g = oc / opg;
    float sum = bias ? bias[oc] : 0.f;
    for (int r = 0; r < kh; ++r) {
      const int ih = oh * sh + r * dh - ph;
      if (ih < 0 || ih >= h) continue;
      for (int s = 0; s < kw; ++s) {
        const int iw = ow * sw + s * dw - pw;
        if (iw < 0 || iw >= wd) continue;
        const __nv_bfloat16* xp = x + (((long long)n * h + ih) * wd + iw) * cin + g * cpg;
        const __nv_bfloat16* wp = w + (((long long)oc * kh + r) * kw + s) * cpg;
        for (int c = 0; c < cpg; ++c) sum = fmaf(__bfloat162float(xp[c]), __bfloat162float(wp[c]), sum);
      }
    }
    y[i] = __float2bfloat16_rn(sum);
  }
}

// bf16 attention for shapes the tensor-core kernel does not take (D != 128,
// unaligned buffers): one warp per query row, online softmax in fp32, D <= 256.
// causal != 0 masks keys j > i (top-left aligned). Scores are multiplied by `scale`
// (1/sqrt(D) unless the operator's scale attribute says otherwise).
extern "C" __global__ void sdpa_bf16_generic(const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k,
                                             const __nv_bfloat16* __restrict__ v, __nv_bfloat16* __restrict__ o,
                                             int B, int H, int Tq, int Tk, int D, int causal, float scale) {
  const int lane = threadIdx.x & 31;
  const long long rows = (long long)B * H * Tq;
  const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
  for (long long row = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); row < rows; row += warps) {
    const long long bh = row / Tq;
    const int i = (int)(row % Tq);
    const int visible = causal ? min(Tk, i + 1) : Tk;
    const __nv_bfloat16* qr = q + row * D;
    const __nv_bfloat16* kb = k + bh * (long long)Tk * D;
    const __nv_bfloat16* vb = v + bh * (long long)Tk * D;
    float qv[8], acc[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int d = lane + 32 * j;
      qv[j] = d < D ? __bfloat162float(qr[d]) : 0.f;
      acc[j] = 0.f;
    }
    float m = -INFINITY, l = 0.f;
    for (int t = 0; t < visible; ++t) {
      float part = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int d = lane + 32 * j;
        if (d < D) part = fmaf(qv[j], __bfloat162float(kb[(long long)t * D + d]), part);
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) part += __shfl_xor_sync(0xffffffffu, part, off);
      const float s = part * scale;
      const float mn = fmaxf(m, s);
      const float corr = expf(m - mn);
      const float p = expf(s - mn);
      l = l * corr + p;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int d = lane + 32 * j;
        if (d < D) acc[j] = fmaf(p, __bfloat162float(vb[(long long)t * D + d]), acc[j] * corr);
      }
      m = mn;
    }
    const float inv = 1.0f / l;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int d = lane + 32 * j;
      if (d < D) o[row * D + d] = __float2bfloat16_rn(acc[j] * inv);
    }
  }
}
