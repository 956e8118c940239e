// Exact causal softmax attention on the CUDA cores (fp32 FMA): the shapes the
// tensor-core flash kernel does not take (d > 64 or dv > 128, up to 128 / 256)
// and the SA_FORCE_SIMT comparison path.  Same result as flash_tc.cu
// (triton_article_attention.py:372-435): online softmax, out = acc / max(l, 1e-20).
//
// One CTA per (64-query tile, sequence), 256 threads: four threads per query
// row, each scoring 8 of a 32-key tile and accumulating a quarter of the value
// columns.  The row maximum is shared among the four threads with shuffles;
// the accumulator is rescaled by exp(m_old - m_new) every tile.
#include <math.h>

#include "sa_common.cuh"

namespace sa {

namespace {

constexpr int kFQ = 64;
constexpr int kFK = 32;
constexpr int kFThreads = 256;

template <int DP, int DVP>
__global__ void __launch_bounds__(kFThreads)
flash_simt_kernel(const float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ v, int64_t n,
                  int d, int dv, float scale, float* __restrict__ out) {
  constexpr int CPT = DVP / 4;
  extern __shared__ float4 flash_smem4[];
  // layout: Kt [DP][kFK+4] | Vs [kFK][DVP] | Qs [kFQ][DP+1] | E [kFQ][kFK+1]
  auto Kt = reinterpret_cast<float(*)[kFK + 4]>(flash_smem4);
  auto Vs = reinterpret_cast<float(*)[DVP]>(&Kt[DP][0]);
  auto Qs = reinterpret_cast<float(*)[DP + 1]>(&Vs[kFK][0]);
  auto E = reinterpret_cast<float(*)[kFK + 1]>(&Qs[kFQ][0]);

  const int tid = threadIdx.x;
  const int qi = tid >> 2, cg = tid & 3;
  const int64_t h = blockIdx.y;
  const int64_t n_qt = (n + kFQ - 1) / kFQ;
  const int64_t q0 = (n_qt - 1 - blockIdx.x) * kFQ;   // heavy tiles first
  const int nq = (int)min((int64_t)kFQ, n - q0);
  const int64_t i = q0 + qi;
  const bool valid = qi < nq;
  const int64_t q_last = q0 + nq - 1;

  const float* qh = q + h * n * d;
  for (int e = tid; e < kFQ * DP; e += kFThreads) {
    const int r = e / DP, a = e - r * DP;
    Qs[r][a] = (r < nq && a < d) ? __ldg(qh + (q0 + r) * d + a) * scale : 0.0f;
  }
  float acc[CPT];
#pragma unroll
  for (int c = 0; c < CPT; ++c) acc[c] = 0.0f;
  float m = -INFINITY, l = 0.0f;

  const float* kh = k + h * n * d;
  const float* vh = v + h * n * dv;
  for (int64_t j0 = 0; j0 <= q_last; j0 += kFK) {
    const int tk = (int)min((int64_t)kFK, q_last + 1 - j0);
    __syncthreads();
    for (int e = tid; e < kFK * DP; e += kFThreads) {
      const int r = e / DP, a = e - r * DP;
      Kt[a][r] = (r < tk && a < d) ? __ldg(kh + (j0 + r) * d + a) : 0.0f;
    }
    for (int e = tid; e < kFK * DVP; e += kFThreads) {
      const int r = e / DVP, c = e - r * DVP;
      Vs[r][c] = (r < tk && c < dv) ? __ldg(vh + (j0 + r) * dv + c) : 0.0f;
    }
    __syncthreads();
    float x[8];
#pragma unroll
    for (int rr = 0; rr < 8; ++rr) x[rr] = 0.0f;
    for (int a = 0; a < d; ++a) {
      const float qa = Qs[qi][a];
      const float4 k0 = *reinterpret_cast<const float4*>(&Kt[a][cg * 8]);
      const float4 k1 = *reinterpret_cast<const float4*>(&Kt[a][cg * 8 + 4]);
      x[0] = fmaf(qa, k0.x, x[0]);
      x[1] = fmaf(qa, k0.y, x[1]);
      x[2] = fmaf(qa, k0.z, x[2]);
      x[3] = fmaf(qa, k0.w, x[3]);
      x[4] = fmaf(qa, k1.x, x[4]);
      x[5] = fmaf(qa, k1.y, x[5]);
      x[6] = fmaf(qa, k1.z, x[6]);
      x[7] = fmaf(qa, k1.w, x[7]);
    }
    // visible keys: j <= i (j < n follows)
    float pm = -INFINITY;
#pragma unroll
    for (int rr = 0; rr < 8; ++rr) {
      const int rl = cg * 8 + rr;
      if (valid && rl < tk && j0 + rl <= i) pm = fmaxf(pm, x[rr]);
    }
    pm = fmaxf(pm, __shfl_xor_sync(0xffffffffu, pm, 1));
    pm = fmaxf(pm, __shfl_xor_sync(0xffffffffu, pm, 2));
    const float m_new = fmaxf(m, pm);
    // m_new = -inf only for a row with nothing visible yet: keep everything at 0
    const float alpha = (m_new == -INFINITY) ? 1.0f : __expf(m - m_new);
#pragma unroll
    for (int rr = 0; rr < 8; ++rr) {
      const int rl = cg * 8 + rr;
      const bool on = valid && rl < tk && j0 + rl <= i;
      E[qi][rl] = on ? __expf(x[rr] - m_new) : 0.0f;
    }
    m = m_new;
    l *= alpha;
#pragma unroll
    for (int c = 0; c < CPT; ++c) acc[c] *= alpha;
    __syncthreads();
    for (int r = 0; r < tk; ++r) {
      const float e = E[qi][r];
      l += e;
      const float4* vrow = reinterpret_cast<const float4*>(&Vs[r][cg * CPT]);
#pragma unroll
      for (int c4 = 0; c4 < CPT / 4; ++c4) {
        const float4 vv = vrow[c4];
        acc[4 * c4 + 0] = fmaf(e, vv.x, acc[4 * c4 + 0]);
        acc[4 * c4 + 1] = fmaf(e, vv.y, acc[4 * c4 + 1]);
        acc[4 * c4 + 2] = fmaf(e, vv.z, acc[4 * c4 + 2]);
        acc[4 * c4 + 3] = fmaf(e, vv.w, acc[4 * c4 + 3]);
      }
    }
  }
  if (valid) {
    const float dmax = fmaxf(l, 1.0e-20f);
    float* orow = out + (h * n + i) * (int64_t)dv;
#pragma unroll
    for (int c = 0; c < CPT; ++c) {
      const int col = cg * CPT + c;
      if (col < dv) orow[col] = __fdiv_rn(acc[c], dmax);
    }
  }
}

template <int DP, int DVP>
int launch_fdp(const float* q, const float* k, const float* v, int64_t bh, int64_t n, int d, int dv, float scale,
               float* out, cudaStream_t s) {
  dim3 grid((unsigned)ceil_div(n, kFQ), (unsigned)bh);
  const size_t smem = sizeof(float) * ((size_t)DP * (kFK + 4) + (size_t)kFK * DVP + (size_t)kFQ * (DP + 1) +
                                       (size_t)kFQ * (kFK + 1));
  cudaError_t e = cudaFuncSetAttribute(flash_simt_kernel<DP, DVP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem);
  if (e != cudaSuccess) return set_error(SA_ERR_CUDA, "flash_simt smem attribute: %s", cudaGetErrorString(e));
  flash_simt_kernel<DP, DVP><<<grid, kFThreads, smem, s>>>(q, k, v, n, d, dv, scale, out);
  return check_launch("flash_simt_kernel");
}

template <int DP>
int launch_fdv(const float* q, const float* k, const float* v, int64_t bh, int64_t n, int d, int dv, float scale,
               float* out, cudaStream_t s) {
  if (dv <= 16) return launch_fdp<DP, 16>(q, k, v, bh, n, d, dv, scale, out, s);
  if (dv <= 32) return launch_fdp<DP, 32>(q, k, v, bh, n, d, dv, scale, out, s);
  if (dv <= 64) return launch_fdp<DP, 64>(q, k, v, bh, n, d, dv, scale, out, s);
  if (dv <= 128) return launch_fdp<DP, 128>(q, k, v, bh, n, d, dv, scale, out, s);
  return launch_fdp<DP, 256>(q, k, v, bh, n, d, dv, scale, out, s);
}

}  // namespace

int launch_flash_simt(const float* q, const float* k, const float* v, int64_t bh, int64_t n, int d, int dv,
                      float scale, float* out, cudaStream_t s) {
  if (bh == 0 || n == 0) return SA_OK;
  if (d > 128 || dv > 256) return set_error(SA_ERR_UNSUPPORTED, "flash: d <= 128 and dv <= 256");
  if (bh > 65535) return set_error(SA_ERR_UNSUPPORTED, "more than 65535 heads in one launch");
  if (d <= 16) return launch_fdv<16>(q, k, v, bh, n, d, dv, scale, out, s);
  if (d <= 32) return launch_fdv<32>(q, k, v, bh, n, d, dv, scale, out, s);
  if (d <= 64) return launch_fdv<64>(q, k, v, bh, n, d, dv, scale, out, s);
  return launch_fdv<128>(q, k, v, bh, n, d, dv, scale, out, s);
}

}  // namespace sa
