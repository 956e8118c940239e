// Shared helpers for the sm_100a kernels and the C ABI of libsa_b200.so.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/streaming_attention.h"

namespace sa {

// Records a message for sa_last_error() on this host thread and returns code.
int set_error(int code, const char* fmt, ...);

// Maps the last CUDA launch error (if any) to SA_ERR_CUDA.
int check_launch(const char* what);

// How long one bounded device-side wait of the tensor-core kernels may take
// before its CTA gives up and records an error in the status word
// (sa_set_wait_limit_ns; 2 s unless set).
uint64_t wait_limit_ns();

// sa_fast_attention; `allow_fork` lets the moment scan run on a second stream
// of its own (made at the first such call per host thread and caller stream).
int fast_attention_run(const float* q, const float* k, const float* v, int64_t bh, int64_t n, int d, int dv,
                       int degree, int block_size, float scale, int compressor, const float* dirs, const float* coins,
                       const int32_t* perms, float eps, float* out, int32_t* rep_idx, void* workspace,
                       size_t workspace_bytes, void* stream, bool allow_fork);

__host__ __device__ inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Device-side index checks, compiled in only with -DSA_DEVICE_CHECKS (the
// libsa_b200_checks.so build).  SA_DEVICE_CHECK(cond, status, code, index) is
// then false when `cond` fails, after recording `code` in the launch status
// word (the first failure of a launch wins) and `index` in the 8 bytes at
// status + 2; the caller skips the access it guards.  In the ordinary build it
// is `true` and `cond` is not evaluated.  Codes 900..999 are checks; the
// status word's other codes (101..309) are bounded waits that gave up.
#ifdef SA_DEVICE_CHECKS
__device__ __forceinline__ bool device_check_failed(int* status, int code, long long index) {
  if (status && atomicCAS(status, 0, code) == 0) *reinterpret_cast<volatile long long*>(status + 2) = index;
  return false;
}
#define SA_DEVICE_CHECK(cond, status, code, index) \
  ((cond) ? true : ::sa::device_check_failed((status), (code), (long long)(index)))
#else
#define SA_DEVICE_CHECK(cond, status, code, index) true
#endif
constexpr int kCheckFirst = 900, kCheckLast = 999;

// Feature count sum_{l<=t} C(d+l-1, l) for t <= 3.
__host__ __device__ inline int64_t feature_count(int d, int t) {
  int64_t f = 1;
  if (t >= 1) f += d;
  if (t >= 2) f += (int64_t)d * (d + 1) / 2;
  if (t >= 3) f += (int64_t)d * (d + 1) * (d + 2) / 6;
  return f;
}

// Monomial of feature f in combinations_with_replacement order
// (streaming_taylor_coreset_attention.py:170; for degree 2 identical to the
// triu order of fast_article_attention.py:173).  Index d stands for the
// constant 1, so every feature is x[a]*x[b]*x[c] over a row with x[d] = 1.
// coef is the key-side Taylor factor 1/prod(alpha_j!) (streaming...py:78-93).
struct Monomial {
  int a, b, c;
  float coef;
};

__host__ __device__ inline Monomial monomial_of(int64_t f, int d) {
  Monomial m{d, d, d, 1.0f};
  if (f == 0) return m;
  f -= 1;
  if (f < d) {
    m.a = (int)f;
    return m;
  }
  f -= d;
  const int64_t n2 = (int64_t)d * (d + 1) / 2;
  if (f < n2) {
    int a = 0;
    while (f >= d - a) {
      f -= d - a;
      ++a;
    }
    m.a = a;
    m.b = a + (int)f;
    m.coef = (m.a == m.b) ? 0.5f : 1.0f;
    return m;
  }
  f -= n2;
  int a = 0;
  while (true) {
    const int64_t rem = d - a;
    const int64_t cnt = rem * (rem + 1) / 2;
    if (f < cnt) break;
    f -= cnt;
    ++a;
  }
  int b = a;
  while (f >= d - b) {
    f -= d - b;
    ++b;
  }
  m.a = a;
  m.b = b;
  m.c = b + (int)f;
  if (m.a == m.b && m.b == m.c)
    m.coef = 1.0f / 6.0f;
  else if (m.a == m.b || m.b == m.c)
    m.coef = 0.5f;
  return m;
}

// Optional tf32 hi / fp32 remainder copies of the gathered reps, the operand
// format of the tensor-core residual (zero padded to dp / dvp columns).
struct SplitOut {
  float* khi = nullptr;   // rep keys, tf32 hi / fp32 remainder, [bh, R, dp]
  float* klo = nullptr;
  int dp = 0;
  int64_t w_stride = 0;  // per-sequence stride of rep_w
};

// tf32 (round to nearest, ties away from zero) of x, in a 32-bit container.
__device__ __forceinline__ uint32_t tc_split_hi(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return r;
}

// exp_{<=t}(x) accumulated as the reference does: term *= x / r; out += term
// (fast_article_attention.py:95-104).
// Division by 1 and 2 is written as the (exactly equal) multiplications.
__device__ __forceinline__ float taylor_poly(float x, int degree) {
  float out = 1.0f;
  if (degree >= 1) {
    float term = x;
    out = out + term;
    if (degree >= 2) {
      term = term * x * 0.5f;
      out = out + term;
      for (int r = 3; r <= degree; ++r) {
        term = __fdiv_rn(term * x, (float)r);
        out = out + term;
      }
    }
  }
  return out;
}

}  // namespace sa
