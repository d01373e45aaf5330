// Seeded synthetic inputs. Element i of a fill depends only on (seed, i):
// a SplitMix64 finaliser turns the counter into 64 random bits, uniforms take
// the top 53 bits, and normals come from the Box-Muller transform of the pair
// (2j, 2j+1). Any slice can therefore be regenerated on its own, and the fill
// splits across threads without changing a single bit.
#include <cmath>
#include <thread>
#include <vector>

#include "internal.hpp"

namespace {

inline uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

inline uint64_t bits_at(uint64_t key, uint64_t i) { return mix64(key + (i + 1) * 0x9E3779B97F4A7C15ull); }

// Uniform in [0, 1) with 53 random bits.
inline double unit(uint64_t bits) { return (double)(bits >> 11) * (1.0 / 9007199254740992.0); }

inline uint16_t to_bf16(float f) {
  uint32_t b;
  memcpy(&b, &f, 4);
  if ((b & 0x7f800000u) == 0x7f800000u && (b & 0x007fffffu)) return (uint16_t)((b >> 16) | 0x40u);
  b += 0x7fffu + ((b >> 16) & 1u);
  return (uint16_t)(b >> 16);
}

inline void store(void* dst, uint32_t dtype, size_t i, double v) {
  float f = (float)v;
  if (dtype == TB_F32)
    static_cast<float*>(dst)[i] = f;
  else
    static_cast<uint16_t*>(dst)[i] = to_bf16(f);
}

template <typename Fn>
void parallel_range(size_t count, int threads, Fn fn) {
  unsigned hw = std::thread::hardware_concurrency();
  size_t t = threads > 0 ? (size_t)threads : (hw ? hw : 1);
  if (count < (1u << 16)) t = 1;
  if (t > count) t = count ? count : 1;
  if (t == 1) {
    fn(0, count);
    return;
  }
  std::vector<std::thread> pool;
  size_t chunk = (count + t - 1) / t;
  chunk = (chunk + 1) & ~(size_t)1;  // keep Box-Muller pairs inside one chunk
  for (size_t b = 0; b < count; b += chunk) pool.emplace_back(fn, b, b + chunk < count ? b + chunk : count);
  for (auto& th : pool) th.join();
}

}  // namespace

extern "C" {

tb_status tb_fill_uniform(void* dst, uint32_t dtype, size_t count, uint64_t seed, double low, double high,
                          int threads) {
  if (!dst && count) return tb::set_error(TB_ERR_INVALID, "fill", "null destination");
  if (dtype != TB_F32 && dtype != TB_BF16) return tb::set_error(TB_ERR_INVALID, "fill", "dtype must be F32 or BF16");
  const uint64_t key = mix64(seed ^ 0x5851F42D4C957F2Dull);
  parallel_range(count, threads, [&](size_t b, size_t e) {
    for (size_t i = b; i < e; ++i) store(dst, dtype, i, low + (high - low) * unit(bits_at(key, i)));
  });
  return TB_OK;
}

tb_status tb_fill_normal(void* dst, uint32_t dtype, size_t count, uint64_t seed, double mean, double stddev,
                         int threads) {
  if (!dst && count) return tb::set_error(TB_ERR_INVALID, "fill", "null destination");
  if (dtype != TB_F32 && dtype != TB_BF16) return tb::set_error(TB_ERR_INVALID, "fill", "dtype must be F32 or BF16");
  const uint64_t key = mix64(seed ^ 0x2545F4914F6CDD1Dull);
  const double two_pi = 6.283185307179586476925286766559;
  parallel_range(count, threads, [&](size_t b, size_t e) {
    for (size_t i = b & ~(size_t)1; i < e; i += 2) {
      const double u1 = 1.0 - unit(bits_at(key, i));  // (0, 1]
      const double u2 = unit(bits_at(key, i + 1));
      const double r = std::sqrt(-2.0 * std::log(u1));
      const double z0 = r * std::cos(two_pi * u2), z1 = r * std::sin(two_pi * u2);
      if (i >= b && i < e) store(dst, dtype, i, mean + stddev * z0);
      if (i + 1 >= b && i + 1 < e) store(dst, dtype, i + 1, mean + stddev * z1);
    }
  });
  return TB_OK;
}

}  // extern "C"
