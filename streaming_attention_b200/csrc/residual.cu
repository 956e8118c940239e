// Residual (tail) kernel with the final combine (SIMT fp32 kernel).
//
// For query i in block c = i / bs it adds
//   sum over reps r of the blocks before c:  w_r (exp(x) - P_t(x)) [v_r, 1]
//     (_block_coreset_residual_tail, fast_article_attention.py:488-499; for
//      compressor none every earlier key is a rep of weight 1, :437-464)
//   sum over keys j of block c with j <= i:  exp(x) [v_j, 1]
//     (the exact current-block residual of :501-512 plus the low-degree part
//      of the same keys, which the block-granular moment scan leaves out)
// with x = scale * q_i.k, to the low term, then writes
// out = num / max(den, eps) (:596-598).
//
// One CTA per (64-query tile, head); reps and keys stream through shared
// memory in tiles of 32, flash style, with numerator and denominator in
// registers.
#include <math.h>

#include "sa_common.cuh"

namespace sa {

namespace {

constexpr int kTQ = 64;
constexpr int kTK = 32;
constexpr int kResThreads = 256;

template <int DP, int DVP>
__global__ void __launch_bounds__(kResThreads)
residual_kernel(const float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ v,
                const float* __restrict__ rk, const float* __restrict__ rv, const float* __restrict__ rw,
                const float* __restrict__ low, int64_t n, int d, int dv, int degree, int bs, int64_t m_blk,
                int64_t reps_per_head, float scale, float eps, bool clamp, float* __restrict__ out) {
  constexpr int CPT = DVP / 4;
  extern __shared__ float4 res_smem4[];
  // layout: Kt [DP][kTK+4] | Vs [kTK][DVP] | Qs [kTQ][DP+1] | E [kTQ][kTK+1] | Ws [kTK]
  auto Kt = reinterpret_cast<float(*)[kTK + 4]>(res_smem4);
  auto Vs = reinterpret_cast<float(*)[DVP]>(&Kt[DP][0]);
  auto Qs = reinterpret_cast<float(*)[DP + 1]>(&Vs[kTK][0]);
  auto E = reinterpret_cast<float(*)[kTK + 1]>(&Qs[kTQ][0]);
  float* Ws = &E[kTQ][0];

  const int tid = threadIdx.x;
  const int qi = tid >> 2, cg = tid & 3;
  const int64_t h = blockIdx.y;
  const int64_t q0 = (int64_t)blockIdx.x * kTQ;
  const int nq = (int)min((int64_t)kTQ, n - q0);
  const int64_t i = q0 + qi;
  const bool valid = qi < nq;
  const int64_t ci = valid ? i / bs : 0;
  const int64_t q_last = q0 + nq - 1;

  const float* qh = q + h * n * d;
  for (int e = tid; e < kTQ * DP; e += kResThreads) {
    const int r = e / DP, a = e - r * DP;
    Qs[r][a] = (r < nq && a < d) ? __ldg(qh + (q0 + r) * d + a) : 0.0f;
  }

  float acc[CPT];
#pragma unroll
  for (int c = 0; c < CPT; ++c) acc[c] = 0.0f;
  float den = 0.0f;

  // ---- phase 1: reps of completed blocks before the query's block
  const int64_t r_end = (q_last / bs) * m_blk;
  const int64_t lim = ci * m_blk;
  const float* rkh = rk + h * reps_per_head * d;
  const float* rvh = rv + h * reps_per_head * dv;
  const float* rwh = rw ? rw + h * reps_per_head : nullptr;
  for (int64_t r0 = 0; r0 < r_end; r0 += kTK) {
    const int tk = (int)min((int64_t)kTK, r_end - r0);
    __syncthreads();
    for (int e = tid; e < kTK * DP; e += kResThreads) {
      const int r = e / DP, a = e - r * DP;
      Kt[a][r] = (r < tk && a < d) ? __ldg(rkh + (r0 + r) * d + a) : 0.0f;
    }
    for (int e = tid; e < kTK * DVP; e += kResThreads) {
      const int r = e / DVP, c = e - r * DVP;
      Vs[r][c] = (r < tk && c < dv) ? __ldg(rvh + (r0 + r) * dv + c) : 0.0f;
    }
    if (tid < kTK) Ws[tid] = (tid < tk) ? (rwh ? __ldg(rwh + r0 + tid) : 1.0f) : 0.0f;
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
#pragma unroll
    for (int rr = 0; rr < 8; ++rr) {
      const int rl = cg * 8 + rr;
      const int64_t r = r0 + rl;
      float e = 0.0f;
      if (valid && rl < tk && r < lim) {
        const float xs = x[rr] * scale;
        e = Ws[rl] * (expf(clamp ? fminf(xs, 80.0f) : xs) - taylor_poly(xs, degree));
      }
      E[qi][rl] = e;
    }
    __syncthreads();
    for (int r = 0; r < tk; ++r) {
      const float e = E[qi][r];
      den += e;
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

  // ---- phase 2: exact current block, exp over keys j in [block start, i]
  const float* kh = k + h * n * d;
  const float* vh = v + h * n * dv;
  const int64_t kb0 = (q0 / bs) * bs;
  const int64_t my_b0 = ci * bs;
  for (int64_t j0 = kb0; j0 <= q_last; j0 += kTK) {
    const int tk = (int)min((int64_t)kTK, q_last + 1 - j0);
    __syncthreads();
    for (int e = tid; e < kTK * DP; e += kResThreads) {
      const int r = e / DP, a = e - r * DP;
      Kt[a][r] = (r < tk && a < d) ? __ldg(kh + (j0 + r) * d + a) : 0.0f;
    }
    for (int e = tid; e < kTK * DVP; e += kResThreads) {
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
#pragma unroll
    for (int rr = 0; rr < 8; ++rr) {
      const int rl = cg * 8 + rr;
      const int64_t j = j0 + rl;
      float e = 0.0f;
      if (valid && rl < tk && j <= i && j >= my_b0) {
        const float xs = x[rr] * scale;
        e = expf(clamp ? fminf(xs, 80.0f) : xs);
      }
      E[qi][rl] = e;
    }
    __syncthreads();
    for (int r = 0; r < tk; ++r) {
      const float e = E[qi][r];
      den += e;
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

  // ---- combine with the low term and divide
  if (valid) {
    const float* lrow = low + (h * n + i) * (int64_t)(dv + 1);
    const float dtot = __ldg(lrow + dv) + den;
    const float inv_den = fmaxf(dtot, eps);
    float* orow = out + (h * n + i) * (int64_t)dv;
#pragma unroll
    for (int c = 0; c < CPT; ++c) {
      const int col = cg * CPT + c;
      if (col < dv) orow[col] = (__ldg(lrow + col) + acc[c]) / inv_den;
    }
  }
}

template <int DP, int DVP>
int launch_dp(const float* q, const float* k, const float* v, const float* rk, const float* rv, const float* rw,
              const float* low, int64_t bh, int64_t n, int d, int dv, int degree, int bs, int64_t m_blk,
              int64_t reps_per_head, float scale, float eps, bool clamp, float* out, cudaStream_t stream) {
  dim3 grid((unsigned)ceil_div(n, kTQ), (unsigned)bh);
  const size_t smem = sizeof(float) * ((size_t)DP * (kTK + 4) + (size_t)kTK * DVP + (size_t)kTQ * (DP + 1) +
                                       (size_t)kTQ * (kTK + 1) + kTK);
  cudaFuncSetAttribute(residual_kernel<DP, DVP>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  residual_kernel<DP, DVP><<<grid, kResThreads, smem, stream>>>(q, k, v, rk, rv, rw, low, n, d, dv, degree, bs, m_blk,
                                                             reps_per_head, scale, eps, clamp, out);
  return check_launch("residual_kernel");
}

template <int DP>
int launch_dv(const float* q, const float* k, const float* v, const float* rk, const float* rv, const float* rw,
              const float* low, int64_t bh, int64_t n, int d, int dv, int degree, int bs, int64_t m_blk,
              int64_t rph, float scale, float eps, bool clamp, float* out, cudaStream_t s) {
  if (dv <= 16) return launch_dp<DP, 16>(q, k, v, rk, rv, rw, low, bh, n, d, dv, degree, bs, m_blk, rph, scale, eps, clamp, out, s);
  if (dv <= 32) return launch_dp<DP, 32>(q, k, v, rk, rv, rw, low, bh, n, d, dv, degree, bs, m_blk, rph, scale, eps, clamp, out, s);
  if (dv <= 64) return launch_dp<DP, 64>(q, k, v, rk, rv, rw, low, bh, n, d, dv, degree, bs, m_blk, rph, scale, eps, clamp, out, s);
  return launch_dp<DP, 128>(q, k, v, rk, rv, rw, low, bh, n, d, dv, degree, bs, m_blk, rph, scale, eps, clamp, out, s);
}

}  // namespace

// Reps of m_blk per completed block (rows r of head h at rk + (h * rph + r) * d;
// rph = rows per head); clamp caps the exp argument at 80 (the segment-mean
// variant, triton_article_attention.py:331-333).
int launch_residual_reps(const float* q, const float* k, const float* v, const float* rk, const float* rv,
                         const float* rw, const float* low, int64_t bh, int64_t n, int d, int dv, int degree, int bs,
                         int64_t m_blk, int64_t rph, float scale, float eps, bool clamp, float* out, cudaStream_t s) {
  if (bh == 0 || n == 0) return SA_OK;
  if (d > 128 || dv > 128) return set_error(SA_ERR_UNSUPPORTED, "dim and value_dim above 128 are not supported");
  if (bh > 65535) return set_error(SA_ERR_UNSUPPORTED, "more than 65535 heads in one launch");
  if (d <= 16) return launch_dv<16>(q, k, v, rk, rv, rw, low, bh, n, d, dv, degree, bs, m_blk, rph, scale, eps, clamp, out, s);
  if (d <= 32) return launch_dv<32>(q, k, v, rk, rv, rw, low, bh, n, d, dv, degree, bs, m_blk, rph, scale, eps, clamp, out, s);
  if (d <= 64) return launch_dv<64>(q, k, v, rk, rv, rw, low, bh, n, d, dv, degree, bs, m_blk, rph, scale, eps, clamp, out, s);
  return launch_dv<128>(q, k, v, rk, rv, rw, low, bh, n, d, dv, degree, bs, m_blk, rph, scale, eps, clamp, out, s);
}

int launch_residual(const float* q, const float* k, const float* v, const float* rk, const float* rv,
                    const float* rw, const float* low, int64_t bh, int64_t n, int d, int dv, int degree, int bs,
                    int compressor, float scale, float eps, float* out, cudaStream_t s) {
  const int64_t nc = n > 0 ? (n - 1) / bs : 0;
  const int64_t m_blk = (compressor == SA_COMPRESSOR_NONE) ? bs : (bs + 1) / 2;
  // compressor none reads the keys themselves: n rows per head
  const int64_t rph = (compressor == SA_COMPRESSOR_NONE) ? n : nc * m_blk;
  return launch_residual_reps(q, k, v, rk, rv, rw, low, bh, n, d, dv, degree, bs, m_blk, rph, scale, eps, false, out,
                              s);
}

}  // namespace sa
