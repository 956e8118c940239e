// C ABI of libsa_b200.so (declared in include/streaming_attention.h).
//
// Argument checks mirror the reference's ValueError conditions
// (fast_article_attention.py:552-561, :361, :392-393) and report them as
// SA_ERR_INVALID_ARG with a message; every CUDA error is caught here and
// returned as SA_ERR_CUDA.  No entry point allocates device memory: outputs
// and scratch belong to the caller.
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include "sa_common.cuh"

namespace sa {

int launch_compress(const float* k, const float* v, int64_t bh, int64_t n, int d, int dv, int bs, int compressor,
                    const float* dirs, const float* coins, const int32_t* perms, int32_t* rep_idx, float* rep_k,
                    float* rep_v, float* rep_w, cudaStream_t stream);
int launch_low_moments(const float* q, const float* k, const float* v, int64_t bh, int64_t n, int d, int dv,
                       int degree, int bs, float scale, float* low, cudaStream_t stream);
int launch_residual(const float* q, const float* k, const float* v, const float* rk, const float* rv,
                    const float* rw, const float* low, int64_t bh, int64_t n, int d, int dv, int degree, int bs,
                    int compressor, float scale, float eps, float* out, cudaStream_t s);

namespace {
thread_local char g_err[512] = {0};
}

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int check_launch(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(SA_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return SA_OK;
}

namespace {

int check_common(const void* q, const void* k, const void* v, int64_t bh, int64_t n, int d, int dv, int degree,
                 int bs) {
  if (bh < 0 || n < 0) return set_error(SA_ERR_INVALID_ARG, "bh and n must be non-negative");
  if (d <= 0 || dv <= 0) return set_error(SA_ERR_INVALID_ARG, "dim and value_dim must be positive");
  if (bs <= 0) return set_error(SA_ERR_INVALID_ARG, "block_size must be positive");
  if (degree < 0) return set_error(SA_ERR_INVALID_ARG, "degree must be non-negative");
  if (degree > SA_MAX_DEGREE)
    return set_error(SA_ERR_UNSUPPORTED, "degree %d is not supported (maximum %d)", degree, SA_MAX_DEGREE);
  if (bh > 0 && n > 0 && (!q || !k || !v)) return set_error(SA_ERR_INVALID_ARG, "null input pointer");
  if (n > ((int64_t)1 << 31)) return set_error(SA_ERR_UNSUPPORTED, "sequence length above 2^31");
  return SA_OK;
}

int check_compressor(int c) {
  if (c != SA_COMPRESSOR_NONE && c != SA_COMPRESSOR_SORTED_PAIR && c != SA_COMPRESSOR_RANDOM)
    return set_error(SA_ERR_INVALID_ARG, "compressor must be one of {'sorted_pair', 'random', 'none'}");
  return SA_OK;
}

constexpr size_t kAlign = 256;
inline size_t align_up(size_t x) { return (x + kAlign - 1) & ~(kAlign - 1); }

struct Workspace {
  size_t low, rep_k, rep_v, rep_w, rep_idx, total;
};

Workspace plan(int64_t bh, int64_t n, int d, int dv, int bs, int compressor) {
  Workspace w{};
  size_t off = 0;
  w.low = off;
  off = align_up(off + (size_t)bh * n * (dv + 1) * sizeof(float));
  const int64_t nc = n > 0 ? (n - 1) / bs : 0;
  const int64_t R = (compressor == SA_COMPRESSOR_NONE) ? 0 : nc * ((bs + 1) / 2);
  w.rep_k = off;
  off = align_up(off + (size_t)bh * R * d * sizeof(float));
  w.rep_v = off;
  off = align_up(off + (size_t)bh * R * dv * sizeof(float));
  w.rep_w = off;
  off = align_up(off + (size_t)bh * R * sizeof(float));
  w.rep_idx = off;
  off = align_up(off + (size_t)bh * R * sizeof(int32_t));
  w.total = off;
  return w;
}

}  // namespace
}  // namespace sa

using namespace sa;

extern "C" {

int sa_version(void) { return 100; }

const char* sa_last_error(void) { return g_err; }

int sa_feature_count(int dim, int degree, int64_t* count) {
  if (!count) return set_error(SA_ERR_INVALID_ARG, "null output pointer");
  if (dim <= 0) return set_error(SA_ERR_INVALID_ARG, "dim must be positive");
  if (degree < 0) return set_error(SA_ERR_INVALID_ARG, "degree must be non-negative");
  if (degree > SA_MAX_DEGREE)
    return set_error(SA_ERR_UNSUPPORTED, "degree %d is not supported (maximum %d)", degree, SA_MAX_DEGREE);
  *count = feature_count(dim, degree);
  return SA_OK;
}

int sa_block_counts(int64_t n, int block_size, int compressor, int64_t* completed_blocks, int64_t* reps_per_block) {
  if (block_size <= 0) return set_error(SA_ERR_INVALID_ARG, "block_size must be positive");
  if (n < 0) return set_error(SA_ERR_INVALID_ARG, "n must be non-negative");
  int rc = check_compressor(compressor);
  if (rc) return rc;
  if (completed_blocks) *completed_blocks = n > 0 ? (n - 1) / block_size : 0;
  if (reps_per_block) *reps_per_block = (compressor == SA_COMPRESSOR_NONE) ? block_size : (block_size + 1) / 2;
  return SA_OK;
}

int sa_compress_blocks(const float* k, const float* v, int64_t bh, int64_t n, int d, int dv, int block_size,
                       int compressor, const float* dirs, const float* coins, const int32_t* perms, int32_t* rep_idx,
                       float* rep_k, float* rep_v, float* rep_w, void* stream) {
  int rc = check_common(k, k, v, bh, n, d, dv, 0, block_size);
  if (rc) return rc;
  rc = check_compressor(compressor);
  if (rc) return rc;
  if (compressor == SA_COMPRESSOR_NONE)
    return set_error(SA_ERR_INVALID_ARG, "compressor none keeps every key; nothing to compress");
  return launch_compress(k, v, bh, n, d, dv, block_size, compressor, dirs, coins, perms, rep_idx, rep_k, rep_v,
                         rep_w, (cudaStream_t)stream);
}

int sa_low_moments(const float* q, const float* k, const float* v, int64_t bh, int64_t n, int d, int dv, int degree,
                   int block_size, float scale, float* low, void* stream) {
  int rc = check_common(q, k, v, bh, n, d, dv, degree, block_size);
  if (rc) return rc;
  if (bh > 0 && n > 0 && !low) return set_error(SA_ERR_INVALID_ARG, "null output pointer");
  return launch_low_moments(q, k, v, bh, n, d, dv, degree, block_size, scale, low, (cudaStream_t)stream);
}

int sa_residual_combine(const float* q, const float* k, const float* v, const float* rep_k, const float* rep_v,
                        const float* rep_w, const float* low, int64_t bh, int64_t n, int d, int dv, int degree,
                        int block_size, int compressor, float scale, float eps, float* out, void* stream) {
  int rc = check_common(q, k, v, bh, n, d, dv, degree, block_size);
  if (rc) return rc;
  rc = check_compressor(compressor);
  if (rc) return rc;
  if (bh > 0 && n > 0 && (!low || !out)) return set_error(SA_ERR_INVALID_ARG, "null low or out pointer");
  const int64_t nc = n > 0 ? (n - 1) / block_size : 0;
  if (bh > 0 && nc > 0 && (!rep_k || !rep_v)) return set_error(SA_ERR_INVALID_ARG, "null rep pointer");
  return launch_residual(q, k, v, rep_k, rep_v, rep_w, low, bh, n, d, dv, degree, block_size, compressor, scale, eps,
                         out, (cudaStream_t)stream);
}

int sa_fast_attention_workspace_size(int64_t bh, int64_t n, int d, int dv, int degree, int block_size, int compressor,
                                     size_t* bytes) {
  if (!bytes) return set_error(SA_ERR_INVALID_ARG, "null output pointer");
  int rc = check_common(nullptr, nullptr, nullptr, 0, n, d, dv, degree, block_size);
  if (rc) return rc;
  if (bh < 0) return set_error(SA_ERR_INVALID_ARG, "bh must be non-negative");
  rc = check_compressor(compressor);
  if (rc) return rc;
  *bytes = plan(bh, n, d, dv, block_size, compressor).total;
  return SA_OK;
}

int sa_fast_attention(const float* q, const float* k, const float* v, int64_t bh, int64_t n, int d, int dv, int degree,
                      int block_size, float scale, int compressor, const float* dirs, const float* coins,
                      const int32_t* perms, float eps, float* out, int32_t* rep_idx, void* workspace,
                      size_t workspace_bytes, void* stream) {
  int rc = check_common(q, k, v, bh, n, d, dv, degree, block_size);
  if (rc) return rc;
  rc = check_compressor(compressor);
  if (rc) return rc;
  if (bh == 0 || n == 0) return SA_OK;
  if (!out) return set_error(SA_ERR_INVALID_ARG, "null output pointer");
  const Workspace w = plan(bh, n, d, dv, block_size, compressor);
  if (!workspace || workspace_bytes < w.total)
    return set_error(SA_ERR_WORKSPACE, "workspace of %zu bytes is smaller than the %zu required", workspace_bytes,
                     w.total);
  if (((uintptr_t)workspace) % kAlign)
    return set_error(SA_ERR_INVALID_ARG, "workspace must be %zu-byte aligned", kAlign);
  char* ws = static_cast<char*>(workspace);
  float* low = reinterpret_cast<float*>(ws + w.low);
  cudaStream_t s = (cudaStream_t)stream;
  const int64_t nc = (n - 1) / block_size;
  const float* rk = k;
  const float* rv = v;
  const float* rw = nullptr;
  if (compressor != SA_COMPRESSOR_NONE && nc > 0) {
    float* rep_k = reinterpret_cast<float*>(ws + w.rep_k);
    float* rep_v = reinterpret_cast<float*>(ws + w.rep_v);
    float* rep_w = reinterpret_cast<float*>(ws + w.rep_w);
    int32_t* ridx = rep_idx ? rep_idx : reinterpret_cast<int32_t*>(ws + w.rep_idx);
    rc = launch_compress(k, v, bh, n, d, dv, block_size, compressor, dirs, coins, perms, ridx, rep_k, rep_v, rep_w, s);
    if (rc) return rc;
    rk = rep_k;
    rv = rep_v;
    rw = rep_w;
  }
  rc = launch_low_moments(q, k, v, bh, n, d, dv, degree, block_size, scale, low, s);
  if (rc) return rc;
  return launch_residual(q, k, v, rk, rv, rw, low, bh, n, d, dv, degree, block_size, compressor, scale, eps, out, s);
}

}  // extern "C"
