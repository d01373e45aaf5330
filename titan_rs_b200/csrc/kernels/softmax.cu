// Row softmax, fp32, over the last axis of a contiguous [rows, cols] tensor.
//
// Same math as titan.rs (projects/titan-runtime/src/lib.rs:933-953 and the
// PTX entry projects/titan-backend-cuda/src/ptx/entries/softmax.rs): subtract
// the row maximum, exponentiate, divide by the row sum. The reference kernel
// runs one thread per row with uncoalesced scalar loads and five passes over
// global memory; here the op is purely HBM-bound and is laid out for it:
//
//   * register path (cols % 4 == 0, cols <= 4096): one warp per row. The row is
//     read once with 128-bit streaming loads (lane i reads float4 i, i+32, ...,
//     so each warp instruction covers 512 contiguous bytes), kept in
//     registers, reduced with warp shuffles (max, then sum of exp), and written
//     once with 128-bit streaming stores: exactly 4 B read + 4 B written per
//     element, the algorithmic minimum.
//   * streaming path (any other shape): one CTA per row, online max/sum in a
//     first read, normalised write in a second read.
//   * bf16 rows (softmax_bf16_rows, an extension for bf16 graphs): one warp per
//     row, fp32 arithmetic with expf, one bf16 rounding per output.
//
// exp(x - m) is evaluated as 2^((x - m) * log2 e) with the hardware ex2
// instruction; (x - m) is formed first, as the reference does, so the argument
// error stays relative to |x - m| and the result is within a few ulp of expf.
#include <cuda_bf16.h>
#include <math.h>
#include <stdint.h>

namespace {

constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ float exp2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// One row held in registers by one warp: NV float4 per lane (cols <= 128*NV, cols % 4 == 0).
template <int NV>
__device__ __forceinline__ void row_in_registers(const float* __restrict__ x, float* __restrict__ y, int cols,
                                                 int lane) {
  const float4* xv = reinterpret_cast<const float4*>(x);
  float4* yv = reinterpret_cast<float4*>(y);
  const int nvec = cols >> 2;
  float4 v[NV];
  float m = -INFINITY;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int idx = lane + 32 * i;
    if (idx < nvec) {
      v[i] = __ldcs(xv + idx);
    } else {
      v[i] = make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
    }
    m = fmaxf(m, fmaxf(fmaxf(v[i].x, v[i].y), fmaxf(v[i].z, v[i].w)));
  }
  m = warp_max(m);
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    v[i].x = exp2_approx((v[i].x - m) * kLog2e);
    v[i].y = exp2_approx((v[i].y - m) * kLog2e);
    v[i].z = exp2_approx((v[i].z - m) * kLog2e);
    v[i].w = exp2_approx((v[i].w - m) * kLog2e);
    s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
  }
  s = warp_sum(s);
  const float inv = 1.0f / s;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int idx = lane + 32 * i;
    if (idx < nvec) {
      float4 o = make_float4(v[i].x * inv, v[i].y * inv, v[i].z * inv, v[i].w * inv);
      __stcs(yv + idx, o);
    }
  }
}

template <int NV>
__device__ __forceinline__ void warp_rows(const float* __restrict__ in, float* __restrict__ out, int rows, int cols) {
  const int lane = threadIdx.x & 31;
  const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
  for (long long row = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); row < rows; row += warps) {
    row_in_registers<NV>(in + row * (long long)cols, out + row * (long long)cols, cols, lane);
  }
}

// Combines two (max, sum-of-exp relative to max) pairs.
__device__ __forceinline__ void combine(float& m, float& s, float m2, float s2) {
  const float mn = fmaxf(m, m2);
  if (mn == -INFINITY) return;
  s = s * exp2_approx((m - mn) * kLog2e) + s2 * exp2_approx((m2 - mn) * kLog2e);
  m = mn;
}

// One CTA per row, any cols: pass 1 online max/sum, pass 2 normalised write.
// Only whole warps take part (a caller-chosen block that is not a multiple of
// 32 leaves its last partial warp idle; a block under 32 threads runs serially
// on thread 0), so every shuffle sees 32 active lanes.
__device__ __forceinline__ void cta_rows(const float* __restrict__ in, float* __restrict__ out, int rows, int cols) {
  __shared__ float sm[32], ss[32];
  __shared__ float row_m, row_s;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nthreads = blockDim.x & ~31;
  const int nwarps = nthreads >> 5;
  const bool serial = nthreads == 0;
  const bool active = serial ? threadIdx.x == 0 : (int)threadIdx.x < nthreads;
  const int stride = serial ? 1 : nthreads;
  for (long long row = blockIdx.x; row < rows; row += gridDim.x) {
    const float* x = in + row * (long long)cols;
    float* y = out + row * (long long)cols;
    float m = -INFINITY, s = 0.f;
    if (active) {
      for (int c = threadIdx.x; c < cols; c += stride) {
        const float v = x[c];
        if (v > m) {
          s = s * exp2_approx((m - v) * kLog2e) + 1.0f;
          m = v;
        } else {
          s += exp2_approx((v - m) * kLog2e);
        }
      }
      if (!serial) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
          const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
          combine(m, s, m2, s2);
        }
        if (lane == 0) {
          sm[warp] = m;
          ss[warp] = s;
        }
      } else {
        sm[0] = m;
        ss[0] = s;
      }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      float mm = sm[0], sx = ss[0];
      for (int w = 1; w < nwarps; ++w) combine(mm, sx, sm[w], ss[w]);
      row_m = mm;
      row_s = sx;
    }
    __syncthreads();
    const float mm = row_m;
    const float inv = 1.0f / row_s;
    if (active)
      for (int c = threadIdx.x; c < cols; c += stride) y[c] = exp2_approx((x[c] - mm) * kLog2e) * inv;
    __syncthreads();
  }
}

}  // namespace

// Specialised entries used by tb_op_softmax: one warp per row, any grid.
#define TB_SOFTMAX_WARP_ENTRY(NV)                                                                       \
  extern "C" __global__ void __launch_bounds__(128) softmax_f32_warp##NV(const float* __restrict__ in, \
                                                                         float* __restrict__ out, int rows, int cols) { \
    warp_rows<NV>(in, out, rows, cols);                                                                 \
  }
TB_SOFTMAX_WARP_ENTRY(1)
TB_SOFTMAX_WARP_ENTRY(2)
TB_SOFTMAX_WARP_ENTRY(4)
TB_SOFTMAX_WARP_ENTRY(8)
TB_SOFTMAX_WARP_ENTRY(16)
TB_SOFTMAX_WARP_ENTRY(32)

extern "C" __global__ void __launch_bounds__(1024) softmax_f32_stream(const float* __restrict__ in,
                                                                      float* __restrict__ out, int rows, int cols) {
  cta_rows(in, out, rows, cols);
}

// The reference ABI, unchanged: softmax_f32_abi() = (in: F32 buffer, out: F32
// buffer, rows: I32, cols: I32), titan-backend-cuda/src/lib.rs:343-355. It is
// correct for any launch geometry (grid-stride loops), including the
// reference's own grid = ceil(rows/128), block = 128.
extern "C" __global__ void softmax_f32(const float* __restrict__ in, float* __restrict__ out, int rows, int cols) {
  const bool aligned = ((reinterpret_cast<uintptr_t>(in) | reinterpret_cast<uintptr_t>(out)) & 15u) == 0;
  if (aligned && (cols & 3) == 0 && cols <= 4096 && (blockDim.x & 31) == 0) {
    if (cols <= 128) warp_rows<1>(in, out, rows, cols);
    else if (cols <= 256) warp_rows<2>(in, out, rows, cols);
    else if (cols <= 512) warp_rows<4>(in, out, rows, cols);
    else if (cols <= 1024) warp_rows<8>(in, out, rows, cols);
    else if (cols <= 2048) warp_rows<16>(in, out, rows, cols);
    else warp_rows<32>(in, out, rows, cols);
  } else {
    cta_rows(in, out, rows, cols);
  }
}

// ---------------------------------------------------------------------------
// bf16 rows (an extension: the reference's softmax is f32 only). One warp per row,
// fp32 arithmetic, the row read twice: pass 1 keeps a running (max, sum of
// exp(x - max)) per lane and merges the lanes; pass 2 writes exp(x - max) / sum,
// rounded to bf16 once. -inf inputs contribute zero; a row of only -inf gives NaN,
// as exp(x - max) / sum does in the reference. VEC = 8 reads 16-byte vectors (row
// starts 16-byte aligned, cols % 8 == 0), VEC = 1 single elements.
namespace {

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}

__device__ __forceinline__ void softmax_merge(float& m, float& s, float m2, float s2) {
  const float mn = fmaxf(m, m2);
  const float a = m == -INFINITY ? 0.0f : s * expf(m - mn);
  const float b = m2 == -INFINITY ? 0.0f : s2 * expf(m2 - mn);
  m = mn;
  s = a + b;
}

template <int VEC>
__device__ __forceinline__ void load_bf16(const __nv_bfloat16* p, float (&v)[VEC]) {
  if constexpr (VEC == 8) {
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      v[2 * j] = __uint_as_float(w[j] << 16);
      v[2 * j + 1] = __uint_as_float(w[j] & 0xffff0000u);
    }
  } else {
    v[0] = __bfloat162float(*p);
  }
}

template <int VEC>
__device__ void softmax_bf16_row(const __nv_bfloat16* __restrict__ x, __nv_bfloat16* __restrict__ y, int cols,
                                 int lane) {
  float m = -INFINITY, s = 0.0f;
  for (int c = lane * VEC; c < cols; c += 32 * VEC) {
    float v[VEC];
    load_bf16<VEC>(x + c, v);
#pragma unroll
    for (int j = 0; j < VEC; ++j) {
      const float t = v[j];
      if (t == -INFINITY) continue;
      if (t > m) {
        s = s * expf(m - t) + 1.0f;
        m = t;
      } else {
        s += expf(t - m);
      }
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1)
    softmax_merge(m, s, __shfl_xor_sync(0xffffffffu, m, off), __shfl_xor_sync(0xffffffffu, s, off));
  for (int c = lane * VEC; c < cols; c += 32 * VEC) {
    float v[VEC];
    load_bf16<VEC>(x + c, v);
    if constexpr (VEC == 8) {
      uint4 u;
      u.x = pack_bf16(expf(v[0] - m) / s, expf(v[1] - m) / s);
      u.y = pack_bf16(expf(v[2] - m) / s, expf(v[3] - m) / s);
      u.z = pack_bf16(expf(v[4] - m) / s, expf(v[5] - m) / s);
      u.w = pack_bf16(expf(v[6] - m) / s, expf(v[7] - m) / s);
      *reinterpret_cast<uint4*>(y + c) = u;
    } else {
      y[c] = __float2bfloat16_rn(expf(v[0] - m) / s);
    }
  }
}

}  // namespace

// rows x cols bf16, contiguous; grid-stride over rows, one warp per row.
extern "C" __global__ void __launch_bounds__(256) softmax_bf16_rows(const __nv_bfloat16* __restrict__ in,
                                                                   __nv_bfloat16* __restrict__ out, int rows,
                                                                   int cols) {
  const int lane = threadIdx.x & 31;
  const int warps = gridDim.x * (blockDim.x >> 5);
  const bool vec = cols % 8 == 0 && ((reinterpret_cast<uintptr_t>(in) | reinterpret_cast<uintptr_t>(out)) & 15) == 0;
  for (int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += warps) {
    const long long base = (long long)r * cols;
    if (vec) softmax_bf16_row<8>(in + base, out + base, cols, lane);
    else softmax_bf16_row<1>(in + base, out + base, cols, lane);
  }
}
