// The feature-segment layout shared by the tensor-core moment kernels, and the
// small TMEM / shared-memory accessors they use.
//
// The monomials of degree <= t are enumerated in aligned runs of 8
// ("segments") that share a prefix: value = x~[p1] * x~[p2] * x~[c0 + u],
// u = 0..7, over the extended row x~ of DX = dp + 8 entries (dp = d rounded up
// to 8): x~[0,d) = x, x~[d,dp) = 0, x~[dp] = 1, the rest 0.  Rows:
//   constant + linear   p1 = p2 = dp, c over [0, DX)
//   degree 2            p1 = a, p2 = dp, c over [8 floor(a/8), dp), a < d
//   degree 3            p1 = a, p2 = b, c over [8 floor(b/8), dp), a <= b < d
// A segment position that is not a canonical monomial (c below the prefix, or
// past d) gets key coefficient 0, so its state row stays exactly zero and its
// query-side value never matters.  This spends ~10% extra MMA work (degree 2,
// d = 64) to let every feature run be produced with vector loads.  The key
// coefficient (1/prod alpha!, or 0; streaming_taylor_coreset_attention.py:78-93)
// is applied to a state row when its change is folded into the fp32 state, not
// to every key feature: for the coefficients 1/2 and 1 that scaling is exact.
#pragma once

#include <stdint.h>

#include "tc_util.cuh"

namespace sa {
namespace mseg {

__host__ __device__ inline int dpad8(int d) { return (d + 7) / 8 * 8; }

// Number of 8-feature segments of dimension d and degree t.
__host__ __device__ inline int64_t seg_count(int d, int t) {
  const int dp = dpad8(d), w = dp / 8;
  int64_t n = w + 1;
  if (t >= 2)
    for (int a = 0; a < d; ++a) n += w - a / 8;
  if (t >= 3)
    for (int b = 0; b < d; ++b) n += (int64_t)(b + 1) * (w - b / 8);
  return n;
}

// segment s -> prefix indices and first c; past the end: a zero segment
__device__ inline void seg_of(int64_t s, int d, int t, int& p1, int& p2, int& c0) {
  const int dp = dpad8(d), w = dp / 8;
  if (s < w + 1) {
    p1 = p2 = dp;
    c0 = 8 * (int)s;
    return;
  }
  s -= w + 1;
  if (t >= 2) {
    for (int a = 0; a < d; ++a) {
      const int cnt = w - a / 8;
      if (s < cnt) {
        p1 = a;
        p2 = dp;
        c0 = 8 * (a / 8 + (int)s);
        return;
      }
      s -= cnt;
    }
  }
  if (t >= 3) {
    for (int b = 0; b < d; ++b) {
      const int cnt = w - b / 8;
      for (int a = 0; a <= b; ++a) {
        if (s < cnt) {
          p1 = a;
          p2 = b;
          c0 = 8 * (b / 8 + (int)s);
          return;
        }
        s -= cnt;
      }
    }
  }
  p1 = p2 = dp + 1;  // x~[dp+1] == 0
  c0 = dp;
}

// Key-side factor of x~[p1] x~[p2] x~[c]: 1/prod(alpha_j!) for a canonical
// monomial of degree <= t, else 0.
__device__ inline float seg_key_coef(int p1, int p2, int c, int d, int t) {
  const int dp = dpad8(d);
  if (p1 > dp || p2 > dp) return 0.0f;
  if (c >= d && c != dp) return 0.0f;
  int idx[3];
  int k = 0;
  if (p1 < d) idx[k++] = p1;
  if (p2 < d) idx[k++] = p2;
  if (c < d) idx[k++] = c;
  if (k > t) return 0.0f;
  if (p2 < d) {
    if (c < p2) return 0.0f;
  } else if (p1 < d) {
    if (c < p1) return 0.0f;
  }
  if (k == 2 && idx[0] == idx[1]) return 0.5f;
  if (k == 3) {
    if (idx[0] == idx[1] && idx[1] == idx[2]) return 1.0f / 6.0f;
    if (idx[0] == idx[1] || idx[1] == idx[2]) return 0.5f;
  }
  return 1.0f;
}

// segment table entry: p1 | p2 << 10 | c0 << 20
__device__ inline uint32_t seg_pack(int64_t s, int d, int t) {
  int p1, p2, c0;
  seg_of(s, d, t, p1, p2, c0);
  return (uint32_t)p1 | ((uint32_t)p2 << 10) | ((uint32_t)c0 << 20);
}

// N consecutive 32-bit columns (4, 8 or 16) of this thread's TMEM lane, then wait.
template <int N>
__device__ __forceinline__ void tmem_ld_wait(uint32_t taddr, float (&v)[N]) {
  uint32_t r[N];
  if constexpr (N == 16) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
  } else if constexpr (N == 8) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
  } else {
    static_assert(N == 4, "4, 8 or 16 columns");
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(taddr));
  }
  tc::tmem_wait_ld();
#pragma unroll
  for (int j = 0; j < N; ++j) v[j] = __uint_as_float(r[j]);
}

// 8 consecutive 32-bit columns of this thread's TMEM lane (no wait).
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&r)[8]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};"
               ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
               : "memory");
}

__device__ __forceinline__ float4 ld4(const float* p) { return *reinterpret_cast<const float4*>(p); }

// tf32 hi part of x by truncation (one logic op).  lo = x - hi is still exact,
// |lo| < 2^-10 |x| instead of 2^-11 with round-to-nearest, which leaves the
// 3xTF32 products within ~2^-20 relative.  NaNs from arithmetic (high mantissa
// bits set) stay NaN.
__device__ __forceinline__ uint32_t tf32_trunc(float x) { return __float_as_uint(x) & 0xffffe000u; }

}  // namespace mseg
}  // namespace sa
