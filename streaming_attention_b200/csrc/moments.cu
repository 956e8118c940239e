// Low-degree Taylor moments as a block-granular scan (SIMT fp32 kernel).
//
// The reference keeps a moment state S = sum_j phi_k(k_j) [v_j, 1] over the
// symmetric monomial feature map phi (fast_article_attention.py:151-181 and
// :217-259; general degree at streaming_taylor_coreset_attention.py:118-296)
// and answers query i with phi_q(scale*q_i) . S.  Here the state is advanced
// one block at a time: every query of block c reads S_{<c}, the moments of the
// blocks before it; the keys of the query's own block are handled in the
// residual kernel with the full exp (low + exact residual of the current block
// sum to exp there, fast_article_attention.py:501-512).
//
// One CTA per (column slice, head).  The CTA holds the F x NS slice of the
// state (NS of the dv+1 columns [v, 1]) in shared memory for the whole scan,
// so no state ever goes to HBM: per block it first answers the block's
// queries from S_{<c}, then adds the block's keys.
#include "sa_common.cuh"

namespace sa {

namespace {

constexpr int kMomThreads = 128;

// Key-side coefficient 1/prod(alpha_j!) of the monomial x[a]x[b]x[c]
// (a <= b <= c, index d = the constant 1).
__device__ __forceinline__ float key_coef(int a, int b, int c, int d) {
  const bool ab = (a == b) && (a < d);
  const bool bc = (b == c) && (b < d);
  return (ab && bc) ? (1.0f / 6.0f) : ((ab || bc) ? 0.5f : 1.0f);
}

template <int NS>
__global__ void __launch_bounds__(kMomThreads)
low_moments_kernel(const float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ v,
                   int64_t n, int d, int dv, int bs, float scale, int F, int nslices, int tt_max,
                   float* __restrict__ low) {
  extern __shared__ float4 smem4[];
  float* S = reinterpret_cast<float*>(smem4);                  // [F][NS]
  float* Vs = S + (size_t)F * NS;                              // [tt_max][NS]
  const int xs = d + 2;                                        // row stride (x[d] = 1)
  float* X = Vs + (size_t)tt_max * NS;                         // [tt_max][xs]
  uint32_t* ftab = reinterpret_cast<uint32_t*>(X + (size_t)tt_max * xs);  // a | b<<10 | c<<20

  const int tid = threadIdx.x;
  const int slice = blockIdx.x;
  const int64_t h = blockIdx.y;
  const int cols = dv + 1;
  const int per = (cols + nslices - 1) / nslices;
  const int col0 = slice * per;
  const int ncols = min(per, cols - col0);

  for (int f = tid; f < F; f += blockDim.x) {
    const Monomial mo = monomial_of(f, d);
    ftab[f] = (uint32_t)mo.a | ((uint32_t)mo.b << 10) | ((uint32_t)mo.c << 20);
#pragma unroll
    for (int j = 0; j < NS; ++j) S[(size_t)f * NS + j] = 0.0f;
  }
  __syncthreads();

  const float* qh = q + h * n * d;
  const float* kh = k + h * n * d;
  const float* vh = v + h * n * dv;
  float* lowh = low + h * n * cols;

  for (int64_t b0 = 0; b0 < n; b0 += bs) {
    const int64_t b1 = min(b0 + (int64_t)bs, n);
    // ---- queries of this block read S_{<c}
    for (int64_t t0 = b0; t0 < b1; t0 += tt_max) {
      const int tt = (int)min((int64_t)tt_max, b1 - t0);
      for (int e = tid; e < tt * d; e += blockDim.x) {
        const int r = e / d, a = e - r * d;
        X[r * xs + a] = __ldg(qh + (t0 + r) * d + a) * scale;
      }
      for (int r = tid; r < tt; r += blockDim.x) X[r * xs + d] = 1.0f;
      __syncthreads();
      if (tid < tt) {
        float acc[NS];
#pragma unroll
        for (int j = 0; j < NS; ++j) acc[j] = 0.0f;
        const float* x = X + tid * xs;
        for (int f = 0; f < F; ++f) {
          const uint32_t p = ftab[f];
          const float phi = x[p & 1023] * x[(p >> 10) & 1023] * x[p >> 20];
          const float4* srow = reinterpret_cast<const float4*>(S + (size_t)f * NS);
#pragma unroll
          for (int j4 = 0; j4 < NS / 4; ++j4) {
            const float4 s4 = srow[j4];
            acc[4 * j4 + 0] = fmaf(phi, s4.x, acc[4 * j4 + 0]);
            acc[4 * j4 + 1] = fmaf(phi, s4.y, acc[4 * j4 + 1]);
            acc[4 * j4 + 2] = fmaf(phi, s4.z, acc[4 * j4 + 2]);
            acc[4 * j4 + 3] = fmaf(phi, s4.w, acc[4 * j4 + 3]);
          }
        }
        float* o = lowh + (t0 + tid) * cols + col0;
#pragma unroll
        for (int j = 0; j < NS; ++j)
          if (j < ncols) o[j] = acc[j];
      }
      __syncthreads();
    }
    if (b1 >= n) break;  // no later query reads the last block
    // ---- add the block's keys to the state
    for (int64_t t0 = b0; t0 < b1; t0 += tt_max) {
      const int tt = (int)min((int64_t)tt_max, b1 - t0);
      for (int e = tid; e < tt * d; e += blockDim.x) {
        const int r = e / d, a = e - r * d;
        X[r * xs + a] = __ldg(kh + (t0 + r) * d + a);
      }
      for (int e = tid; e < tt * NS; e += blockDim.x) {
        const int r = e / NS, j = e - r * NS;
        const int col = col0 + j;
        float val = 0.0f;
        if (j < ncols) val = (col < dv) ? __ldg(vh + (t0 + r) * dv + col) : 1.0f;
        Vs[r * NS + j] = val;
      }
      for (int r = tid; r < tt; r += blockDim.x) X[r * xs + d] = 1.0f;
      __syncthreads();
      for (int f = tid; f < F; f += blockDim.x) {
        const uint32_t p = ftab[f];
        const int ia = p & 1023, ib = (p >> 10) & 1023, ic = p >> 20;
        const float cf = key_coef(ia, ib, ic, d);
        float acc[NS];
#pragma unroll
        for (int j = 0; j < NS; ++j) acc[j] = 0.0f;
        for (int r = 0; r < tt; ++r) {
          const float* x = X + r * xs;
          const float phi = x[ia] * x[ib] * x[ic] * cf;
          const float4* vrow = reinterpret_cast<const float4*>(Vs + r * NS);
#pragma unroll
          for (int j4 = 0; j4 < NS / 4; ++j4) {
            const float4 v4 = vrow[j4];
            acc[4 * j4 + 0] = fmaf(phi, v4.x, acc[4 * j4 + 0]);
            acc[4 * j4 + 1] = fmaf(phi, v4.y, acc[4 * j4 + 1]);
            acc[4 * j4 + 2] = fmaf(phi, v4.z, acc[4 * j4 + 2]);
            acc[4 * j4 + 3] = fmaf(phi, v4.w, acc[4 * j4 + 3]);
          }
        }
        float4* srow = reinterpret_cast<float4*>(S + (size_t)f * NS);
#pragma unroll
        for (int j4 = 0; j4 < NS / 4; ++j4) {
          float4 s4 = srow[j4];
          s4.x += acc[4 * j4 + 0];
          s4.y += acc[4 * j4 + 1];
          s4.z += acc[4 * j4 + 2];
          s4.w += acc[4 * j4 + 3];
          srow[j4] = s4;
        }
      }
      __syncthreads();
    }
  }
}

size_t moments_smem(int ns, int F, int d, int tt) {
  return (size_t)F * ns * 4 + (size_t)tt * ns * 4 + (size_t)tt * (d + 2) * 4 + (size_t)F * 4;
}

template <int NS>
int launch_ns(const float* q, const float* k, const float* v, int64_t bh, int64_t n, int d, int dv, int bs,
              float scale, int F, int tt, float* low, cudaStream_t stream) {
  const int cols = dv + 1;
  const int nslices = (cols + NS - 1) / NS;
  const size_t smem = moments_smem(NS, F, d, tt);
  cudaFuncSetAttribute(low_moments_kernel<NS>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  dim3 grid((unsigned)nslices, (unsigned)bh);
  low_moments_kernel<NS><<<grid, kMomThreads, smem, stream>>>(q, k, v, n, d, dv, bs, scale, F, nslices, tt, low);
  return check_launch("low_moments_kernel");
}

}  // namespace

int launch_low_moments(const float* q, const float* k, const float* v, int64_t bh, int64_t n, int d, int dv,
                       int degree, int bs, float scale, float* low, cudaStream_t stream) {
  if (bh == 0 || n == 0) return SA_OK;
  if (bh > 65535) return set_error(SA_ERR_UNSUPPORTED, "more than 65535 heads in one launch");
  if (d > 1000) return set_error(SA_ERR_UNSUPPORTED, "dim > 1000 is not supported by the moment kernel");
  const int64_t F64 = feature_count(d, degree);
  if (F64 >= (1 << 20)) return set_error(SA_ERR_UNSUPPORTED, "feature count %lld too large", (long long)F64);
  const int F = (int)F64;
  const size_t budget = 225 * 1024;
  for (int tt = kMomThreads; tt >= 32; tt >>= 1) {
    if (moments_smem(16, F, d, tt) <= budget) return launch_ns<16>(q, k, v, bh, n, d, dv, bs, scale, F, tt, low, stream);
    if (moments_smem(8, F, d, tt) <= budget) return launch_ns<8>(q, k, v, bh, n, d, dv, bs, scale, F, tt, low, stream);
    if (moments_smem(4, F, d, tt) <= budget) return launch_ns<4>(q, k, v, bh, n, d, dv, bs, scale, F, tt, low, stream);
  }
  return set_error(SA_ERR_UNSUPPORTED, "feature count %lld too large for the moment kernel's shared memory",
                   (long long)F64);
}

}  // namespace sa
