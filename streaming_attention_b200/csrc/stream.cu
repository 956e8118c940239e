// The streaming (decode) form of the method: the per-token pieces behind the
// reference's ArticleStreamingAttention (streaming_taylor_coreset_attention.py:
// TaylorMomentSketch :229-296, MergeReduceCoreset :332-506, query :572-606).
//
// State lives in caller-owned device buffers: the moment sketch num [F, dv] and
// den [F] (fp32), a pending block of raw keys / values, and the
// merge-and-reduce levels (keys, values, float32 weights).  The host drives
// the level structure and draws the compressor's random numbers from the CPU
// generator in the reference's order; these kernels do the arithmetic:
//
//   stream_update_kernel    num[f, :] += (w phi_k(key)[f]) v,  den[f] += w phi_k(key)[f]
//                           (product then add, both rounded: the reference's
//                           `add_(wf[:, None] * value)` order)
//   stream_compress_kernel  one block of n weighted items -> ceil(n/2): sorted_pair
//                           (float64 projection scores, bitonic sort by
//                           (score, index), pair (2i, 2i+1), keep a with
//                           probability w_a / (w_a + w_b), weight w_a + w_b, odd
//                           tail kept) or random (given permutation, weights
//                           times n/m)
//   stream_query_*          phi_q(s q) . [num, den] over feature tiles (one CTA
//                           per tile, partials in the workspace), then one CTA
//                           adds the tiles in order, the coreset tail
//                           w (exp(x) - P_t(x)) [v, 1] over the pending block
//                           (weight 1) and the levels, and divides.
#include <float.h>
#include <math.h>

#include "sa_common.cuh"

namespace sa {

namespace {

#define SA_MAX_DIM_STREAM 1024       // largest key dimension of the streaming state

constexpr int kUpdFeat = 32;        // features per CTA of the update kernel
constexpr int kQryFeat = 256;       // features per CTA of the query kernel
constexpr int kQryThreads = 256;
constexpr int kFinThreads = 256;

// x~[i]: the vector entry, or 1 for the "absent" index d of a lower-degree monomial
__device__ __forceinline__ float xt(const float* x, int i, int d) { return i < d ? x[i] : 1.0f; }

// Monomial f of x (no coefficient): x[a] * x[b] * x[c], in that order.
__device__ __forceinline__ float monomial_value(const float* x, const Monomial& m, int d) {
  return __fmul_rn(__fmul_rn(xt(x, m.a, d), xt(x, m.b, d)), xt(x, m.c, d));
}

__global__ void stream_update_kernel(const float* __restrict__ key, const float* __restrict__ value, int d, int dv,
                                     int64_t F, float w, float* __restrict__ num, float* __restrict__ den) {
  __shared__ float ks[SA_MAX_DIM_STREAM];
  __shared__ float wf[kUpdFeat];
  for (int i = threadIdx.x; i < d; i += blockDim.x) ks[i] = key[i];
  __syncthreads();
  const int64_t f0 = (int64_t)blockIdx.x * kUpdFeat;
  const int nf = (int)min((int64_t)kUpdFeat, F - f0);
  if (threadIdx.x < nf) {
    const Monomial m = monomial_of(f0 + threadIdx.x, d);
    // key[idx].prod() * coeff, then weight (streaming_taylor_coreset_attention.py:196-199, :274-277)
    const float feat = __fmul_rn(monomial_value(ks, m, d), m.coef);
    const float v = __fmul_rn(w, feat);
    wf[threadIdx.x] = v;
    den[f0 + threadIdx.x] = __fadd_rn(den[f0 + threadIdx.x], v);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < nf * dv; e += blockDim.x) {
    const int fl = e / dv, c = e - fl * dv;
    float* p = num + (f0 + fl) * dv + c;
    *p = __fadd_rn(*p, __fmul_rn(wf[fl], __ldg(value + c)));
  }
}

__device__ __forceinline__ bool key_less(double sa, int ia, double sb, int ib) {
  return sa < sb || (sa == sb && ia < ib);
}

__global__ void stream_compress_kernel(const float* __restrict__ keys, const float* __restrict__ values,
                                       const float* __restrict__ weights, int n, int d, int dv, int m, int pow2,
                                       int use_perm, const float* __restrict__ dir, const float* __restrict__ coins,
                                       const int32_t* __restrict__ perm, float* __restrict__ out_keys,
                                       float* __restrict__ out_values, float* __restrict__ out_weights) {
  extern __shared__ __align__(16) unsigned char smem[];
  double* score = reinterpret_cast<double*>(smem);          // [pow2]
  int* idx = reinterpret_cast<int*>(score + pow2);          // [pow2]
  int* sel = idx + pow2;                                    // [m]
  float* selw = reinterpret_cast<float*>(sel + m);          // [m]
  const int tid = threadIdx.x;
  if (use_perm) {
    // uniform half-sample with inverse-probability weight (:426-433)
    const float factor = (float)((double)n / (double)m);
    for (int p = tid; p < m; p += blockDim.x) {
      const int s = perm[p];
      sel[p] = s;
      selw[p] = __fmul_rn(weights[s], factor);
    }
  } else {
    for (int i = tid; i < pow2; i += blockDim.x) {
      if (i < n) {
        double acc = 0.0;
        for (int a = 0; a < d; ++a) acc += (double)keys[(int64_t)i * d + a] * (double)dir[a];
        score[i] = acc;
        idx[i] = i;
      } else {
        score[i] = DBL_MAX;
        idx[i] = 0x7fffffff;
      }
    }
    __syncthreads();
    // bitonic sort of (score, index) ascending
    for (int k = 2; k <= pow2; k <<= 1) {
      for (int j = k >> 1; j > 0; j >>= 1) {
        for (int i = tid; i < pow2; i += blockDim.x) {
          const int l = i ^ j;
          if (l > i) {
            const bool up = (i & k) == 0;
            const bool gt = key_less(score[l], idx[l], score[i], idx[i]);
            if (gt == up) {
              const double ts = score[i];
              score[i] = score[l];
              score[l] = ts;
              const int ti = idx[i];
              idx[i] = idx[l];
              idx[l] = ti;
            }
          }
        }
        __syncthreads();
      }
    }
    // pair neighbours, keep a with probability w_a / (w_a + w_b) (:446-457)
    const int pairs = n / 2;
    for (int p = tid; p < pairs; p += blockDim.x) {
      const int ia = idx[2 * p], ib = idx[2 * p + 1];
      const float wa = weights[ia], wb = weights[ib];
      const float wsum = __fadd_rn(wa, wb);
      const float prob_a = __fdiv_rn(wa, fmaxf(wsum, 1e-30f));
      sel[p] = coins[p] < prob_a ? ia : ib;
      selw[p] = wsum;
    }
    if ((n & 1) && tid == 0) {   // odd tail kept with its weight (:459-462)
      sel[pairs] = idx[n - 1];
      selw[pairs] = weights[idx[n - 1]];
    }
  }
  __syncthreads();
  for (int e = tid; e < m * d; e += blockDim.x) {
    const int p = e / d, a = e - p * d;
    out_keys[e] = keys[(int64_t)sel[p] * d + a];
  }
  for (int e = tid; e < m * dv; e += blockDim.x) {
    const int p = e / dv, a = e - p * dv;
    out_values[e] = values[(int64_t)sel[p] * dv + a];
  }
  for (int p = tid; p < m; p += blockDim.x) out_weights[p] = selw[p];
}

// Partial low sums of one tile of kQryFeat features: part[tile, :dv] = sum_f
// phi_q[f] num[f, :], part[tile, dv] = sum_f phi_q[f] den[f].
__global__ void stream_query_tiles_kernel(const float* __restrict__ query, int d, int dv, int64_t F, float scale,
                                          const float* __restrict__ num, const float* __restrict__ den,
                                          float* __restrict__ part) {
  __shared__ float qs[SA_MAX_DIM_STREAM];
  __shared__ float fq[kQryFeat];
  for (int i = threadIdx.x; i < d; i += blockDim.x) qs[i] = __fmul_rn(query[i], scale);   // q * scale (:585)
  __syncthreads();
  const int64_t f0 = (int64_t)blockIdx.x * kQryFeat;
  const int nf = (int)min((int64_t)kQryFeat, F - f0);
  if (threadIdx.x < nf) fq[threadIdx.x] = monomial_value(qs, monomial_of(f0 + threadIdx.x, d), d);
  __syncthreads();
  for (int c = threadIdx.x; c <= dv; c += blockDim.x) {
    float acc = 0.0f;
    if (c < dv) {
      for (int i = 0; i < nf; ++i) acc = fmaf(fq[i], num[(f0 + i) * dv + c], acc);
    } else {
      for (int i = 0; i < nf; ++i) acc = fmaf(fq[i], den[f0 + i], acc);
    }
    part[(int64_t)blockIdx.x * (dv + 1) + c] = acc;
  }
}

// One CTA: low sums from the tiles (in tile order), the coreset tail over the
// pending block (weight 1) and the levels, the divide.
__global__ void stream_query_finish_kernel(const float* __restrict__ query, int d, int dv, int degree, float scale,
                                           const float* __restrict__ part, int ntiles,
                                           const float* __restrict__ bk, const float* __restrict__ bv, int64_t nb,
                                           const float* __restrict__ lk, const float* __restrict__ lv,
                                           const float* __restrict__ lw, int64_t nl, float eps,
                                           float* __restrict__ out, float* __restrict__ dens) {
  extern __shared__ float fsm[];
  float* e_s = fsm;                      // [nb + nl] tail weights w (exp(x) - P_t(x))
  float* lowv = e_s + (nb + nl);         // [dv + 1]
  float* red = lowv + (dv + 1);          // [blockDim.x]
  const int tid = threadIdx.x;
  for (int c = tid; c <= dv; c += blockDim.x) {
    float acc = 0.0f;
    for (int t = 0; t < ntiles; ++t) acc = __fadd_rn(acc, part[(int64_t)t * (dv + 1) + c]);
    lowv[c] = acc;
  }
  const int64_t ni = nb + nl;
  for (int64_t r = tid; r < ni; r += blockDim.x) {
    const float* kr = r < nb ? bk + r * d : lk + (r - nb) * d;
    float dot = 0.0f;
    for (int a = 0; a < d; ++a) dot = fmaf(kr[a], query[a], dot);
    const float x = __fmul_rn(scale, dot);            // scale * (keys @ query) (:590)
    const float w = r < nb ? 1.0f : lw[r - nb];
    e_s[r] = __fmul_rn(w, expf(x) - taylor_poly(x, degree));
  }
  __syncthreads();
  // tail denominator: per-thread partials in a fixed order, then a tree
  float tden = 0.0f;
  for (int64_t r = tid; r < ni; r += blockDim.x) tden += e_s[r];
  red[tid] = tden;
  __syncthreads();
  for (int s = blockDim.x >> 1; s > 0; s >>= 1) {
    if (tid < s) red[tid] += red[tid + s];
    __syncthreads();
  }
  const float tail_den = red[0];
  const float low_den = lowv[dv];
  const float den = low_den + tail_den;
  const float safe = fmaxf(den, eps);
  for (int c = tid; c < dv; c += blockDim.x) {
    float acc = 0.0f;
    for (int64_t r = 0; r < ni; ++r) {
      const float vr = r < nb ? bv[r * dv + c] : lv[(r - nb) * dv + c];
      acc = fmaf(e_s[r], vr, acc);
    }
    out[c] = __fdiv_rn(lowv[c] + acc, safe);
  }
  if (dens && tid == 0) {
    dens[0] = den;
    dens[1] = low_den;
    dens[2] = tail_den;
  }
}

int stream_checks(int d, int dv, int degree, int64_t* F) {
  if (d <= 0 || dv <= 0) return set_error(SA_ERR_INVALID_ARG, "dim and value_dim must be positive");
  if (d > SA_MAX_DIM_STREAM)
    return set_error(SA_ERR_UNSUPPORTED, "streaming state supports dim <= %d", SA_MAX_DIM_STREAM);
  if (degree < 0) return set_error(SA_ERR_INVALID_ARG, "degree must be non-negative");
  if (degree > SA_MAX_DEGREE) return set_error(SA_ERR_UNSUPPORTED, "degree > %d is not supported", SA_MAX_DEGREE);
  *F = feature_count(d, degree);
  return SA_OK;
}

}  // namespace

}  // namespace sa

using namespace sa;

extern "C" {

int sa_stream_update(const float* key, const float* value, int d, int dv, int degree, float weight, float* num_state,
                     float* den_state, void* stream) {
  int64_t F = 0;
  int rc = stream_checks(d, dv, degree, &F);
  if (rc) return rc;
  if (!key || !value || !num_state || !den_state) return set_error(SA_ERR_INVALID_ARG, "null pointer");
  const int64_t blocks = ceil_div(F, kUpdFeat);
  stream_update_kernel<<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(key, value, d, dv, F, weight, num_state,
                                                                          den_state);
  return check_launch("stream_update_kernel");
}

int sa_stream_compress(const float* keys, const float* values, const float* weights, int64_t n, int d, int dv,
                       int compressor, const float* direction, const float* coins, const int32_t* perm,
                       float* out_keys, float* out_values, float* out_weights, void* stream) {
  if (d <= 0 || dv <= 0) return set_error(SA_ERR_INVALID_ARG, "dim and value_dim must be positive");
  if (compressor != SA_COMPRESSOR_SORTED_PAIR && compressor != SA_COMPRESSOR_RANDOM)
    return set_error(SA_ERR_INVALID_ARG, "compressor must be sorted_pair or random (none keeps the block)");
  if (n < 2) return set_error(SA_ERR_INVALID_ARG, "a block of %lld items needs no compression", (long long)n);
  if (n > 8192) return set_error(SA_ERR_UNSUPPORTED, "blocks of more than 8192 items are not supported");
  if (!keys || !values || !weights || !out_keys || !out_values || !out_weights)
    return set_error(SA_ERR_INVALID_ARG, "null pointer");
  const int m = (int)((n + 1) / 2);
  const bool use_perm = compressor == SA_COMPRESSOR_RANDOM || n <= 2;
  if (use_perm && !perm) return set_error(SA_ERR_INVALID_ARG, "perm is required");
  if (!use_perm && (!direction || !coins)) return set_error(SA_ERR_INVALID_ARG, "direction and coins are required");
  int pow2 = 1;
  while (pow2 < n) pow2 <<= 1;
  const size_t smem = (size_t)pow2 * (sizeof(double) + sizeof(int)) + (size_t)m * (sizeof(int) + sizeof(float));
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(stream_compress_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess) return set_error(SA_ERR_CUDA, "stream_compress smem attribute: %s", cudaGetErrorString(e));
  }
  stream_compress_kernel<<<1, 512, smem, (cudaStream_t)stream>>>(keys, values, weights, (int)n, d, dv, m, pow2,
                                                                 use_perm ? 1 : 0, direction, coins, perm, out_keys,
                                                                 out_values, out_weights);
  return check_launch("stream_compress_kernel");
}

int sa_stream_query_workspace_size(int d, int dv, int degree, size_t* bytes) {
  if (!bytes) return set_error(SA_ERR_INVALID_ARG, "null output pointer");
  int64_t F = 0;
  int rc = stream_checks(d, dv, degree, &F);
  if (rc) return rc;
  *bytes = (size_t)ceil_div(F, kQryFeat) * (size_t)(dv + 1) * sizeof(float);
  return SA_OK;
}

int sa_stream_query(const float* query, int d, int dv, int degree, float scale, const float* num_state,
                    const float* den_state, const float* buf_keys, const float* buf_values, int64_t n_buf,
                    const float* lvl_keys, const float* lvl_values, const float* lvl_weights, int64_t n_lvl, float eps,
                    float* out, float* dens, void* workspace, size_t workspace_bytes, void* stream) {
  int64_t F = 0;
  int rc = stream_checks(d, dv, degree, &F);
  if (rc) return rc;
  if (!query || !num_state || !den_state || !out) return set_error(SA_ERR_INVALID_ARG, "null pointer");
  if (n_buf < 0 || n_lvl < 0) return set_error(SA_ERR_INVALID_ARG, "item counts must be non-negative");
  if ((n_buf > 0 && (!buf_keys || !buf_values)) || (n_lvl > 0 && (!lvl_keys || !lvl_values || !lvl_weights)))
    return set_error(SA_ERR_INVALID_ARG, "null item pointer");
  const int64_t tiles = ceil_div(F, kQryFeat);
  const size_t need = (size_t)tiles * (size_t)(dv + 1) * sizeof(float);
  if (!workspace || workspace_bytes < need)
    return set_error(SA_ERR_WORKSPACE, "workspace of %zu bytes is smaller than the %zu required", workspace_bytes,
                     need);
  const size_t fin_smem = ((size_t)(n_buf + n_lvl) + (size_t)(dv + 1) + kFinThreads) * sizeof(float);
  if (fin_smem > 200 * 1024) return set_error(SA_ERR_UNSUPPORTED, "too many coreset items for one query");
  if (fin_smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(stream_query_finish_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)fin_smem);
    if (e != cudaSuccess) return set_error(SA_ERR_CUDA, "stream_query smem attribute: %s", cudaGetErrorString(e));
  }
  cudaStream_t s = (cudaStream_t)stream;
  float* part = static_cast<float*>(workspace);
  stream_query_tiles_kernel<<<(unsigned)tiles, kQryThreads, 0, s>>>(query, d, dv, F, scale, num_state, den_state,
                                                                    part);
  rc = check_launch("stream_query_tiles_kernel");
  if (rc) return rc;
  stream_query_finish_kernel<<<1, kFinThreads, fin_smem, s>>>(query, d, dv, degree, scale, part, (int)tiles,
                                                              buf_keys, buf_values, n_buf, lvl_keys, lvl_values,
                                                              lvl_weights, n_lvl, eps, out, dens);
  return check_launch("stream_query_finish_kernel");
}

}  // extern "C"
