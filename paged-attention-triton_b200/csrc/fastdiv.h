// Division of a 32-bit unsigned integer by a divisor that is fixed for a
// launch, as one multiply-high, a subtract, an add and two shifts:
// T. Granlund and P. L. Montgomery, "Division by Invariant Integers using
// Multiplication", PLDI 1994, Figure 4.1 (unsigned division, N = 32):
//
//   l  = ceil(log2 d)
//   m' = floor(2^32 * (2^l - d) / d) + 1
//   q  = (t1 + ((n - t1) >> min(l, 1))) >> max(l - 1, 0),  t1 = mulhi(m', n)
//
// exact for every 0 <= n < 2^32 and 1 <= d < 2^32. The host computes
// (m', shifts) once per launch; the kernel's schedule decode uses them in place
// of a general integer division. Plain C++ as well, so the CPU tests compile it.
#pragma once

#include <stdint.h>

#if defined(__CUDACC__)
#define PA_FD_HD __host__ __device__ __forceinline__
#else
#define PA_FD_HD inline
#endif

namespace pa {

struct FastDiv {
  uint32_t m;    // m'
  uint32_t s1;   // min(l, 1)
  uint32_t s2;   // max(l - 1, 0)
  uint32_t d;    // the divisor itself (multiplies back a quotient)
};

// 1 <= d < 2^31 (callers clamp a zero divisor to 1; nothing is divided by it then).
inline FastDiv make_fastdiv(uint32_t d) {
  if (d == 0) d = 1;
  uint32_t l = 0;
  while (l < 32 && (uint64_t(1) << l) < d) ++l;
  FastDiv f;
  // (2^l - d) < d <= 2^31, so the product stays below 2^63 and m' below 2^32.
  f.m = static_cast<uint32_t>(((uint64_t(1) << 32) * ((uint64_t(1) << l) - d)) / d + 1);
  f.s1 = l < 1 ? l : 1;
  f.s2 = l > 1 ? l - 1 : 0;
  f.d = d;
  return f;
}

PA_FD_HD uint32_t fd_mulhi(uint32_t a, uint32_t b) {
#if defined(__CUDA_ARCH__)
  return __umulhi(a, b);
#else
  return static_cast<uint32_t>((static_cast<uint64_t>(a) * b) >> 32);
#endif
}

PA_FD_HD uint32_t fast_div(uint32_t n, const FastDiv& f) {
  const uint32_t t = fd_mulhi(n, f.m);
  return (t + ((n - t) >> f.s1)) >> f.s2;
}

}  // namespace pa
