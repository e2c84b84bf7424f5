// Counter-based synthetic weight generator shared by stb_fill_normal and the Llama initialiser.
// splitmix64 keyed by (seed, stream, index), Marsaglia polar normal with a hand-written log, every
// double operation explicitly rounded so the CPU restatement (compiled without contraction)
// produces the same bits.
#pragma once

#include "common.cuh"

namespace stb {

__device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ULL;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebULL;
  return z ^ (z >> 31);
}

__device__ __forceinline__ uint64_t rng_u64(uint64_t seed, uint64_t stream, uint64_t index) {
  uint64_t key = mix64(seed ^ (0x9e3779b97f4a7c15ULL * (stream + 1)));
  return mix64(key + 0x9e3779b97f4a7c15ULL * (index + 1));
}

// ln x for positive normal doubles by 2*atanh((m-1)/(m+1)); every operation is an explicitly
// rounded IEEE double operation so the host restatement compiled without contraction yields the
// same bits.
__device__ __forceinline__ double rng_log(double x) {
  unsigned long long b = (unsigned long long)__double_as_longlong(x);
  int e = (int)((b >> 52) & 0x7ff) - 1023;
  b = (b & 0x000fffffffffffffULL) | 0x3ff0000000000000ULL;
  double m = __longlong_as_double((long long)b);
  if (m > 1.4142135623730951) {
    m = __dmul_rn(m, 0.5);
    e = e + 1;
  }
  double t = __ddiv_rn(__dsub_rn(m, 1.0), __dadd_rn(m, 1.0));
  double t2 = __dmul_rn(t, t);
  double p = 1.0 / 25.0;
  p = __dadd_rn(__dmul_rn(p, t2), 1.0 / 23.0);
  p = __dadd_rn(__dmul_rn(p, t2), 1.0 / 21.0);
  p = __dadd_rn(__dmul_rn(p, t2), 1.0 / 19.0);
  p = __dadd_rn(__dmul_rn(p, t2), 1.0 / 17.0);
  p = __dadd_rn(__dmul_rn(p, t2), 1.0 / 15.0);
  p = __dadd_rn(__dmul_rn(p, t2), 1.0 / 13.0);
  p = __dadd_rn(__dmul_rn(p, t2), 1.0 / 11.0);
  p = __dadd_rn(__dmul_rn(p, t2), 1.0 / 9.0);
  p = __dadd_rn(__dmul_rn(p, t2), 1.0 / 7.0);
  p = __dadd_rn(__dmul_rn(p, t2), 1.0 / 5.0);
  p = __dadd_rn(__dmul_rn(p, t2), 1.0 / 3.0);
  p = __dadd_rn(__dmul_rn(p, t2), 1.0);
  double lp = __dmul_rn(__dmul_rn(2.0, t), p);
  double le = __dmul_rn((double)e, 0x1.62e42fefa39efp-1);
  return __dadd_rn(le, lp);
}

// Marsaglia polar normal; attempt j uses counter 64*index + j.
__device__ __forceinline__ double rng_normal_dev(uint64_t seed, uint64_t stream, uint64_t index) {
  for (uint64_t j = 0; j < 64; j++) {
    uint64_t r = rng_u64(seed, stream, index * 64 + j);
    double u = __dsub_rn(__dmul_rn(__dadd_rn((double)(r >> 32), 0.5), 0x1p-31), 1.0);
    double v = __dsub_rn(__dmul_rn(__dadd_rn((double)(r & 0xffffffffULL), 0.5), 0x1p-31), 1.0);
    double s = __dadd_rn(__dmul_rn(u, u), __dmul_rn(v, v));
    if (s >= 1.0 || s == 0.0) continue;
    double l = rng_log(s);
    double q = __ddiv_rn(__dmul_rn(-2.0, l), s);
    return __dmul_rn(u, __dsqrt_rn(q));
  }
  return 0.0;
}

}  // namespace stb
