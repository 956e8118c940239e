// C1: per-block coreset compressor (sorted_pair and random).
//
// Follows _compress_one_completed_block (fast_article_attention.py:312-361)
// and _build_completed_block_reps (:364-434): every completed block (one that
// has a later query) is halved.  sorted_pair projects the block's keys on a
// unit direction, sorts, pairs neighbours (0,1),(2,3),... and keeps one key of
// each pair with probability proportional to its weight (u < wa/(wa+wb),
// streaming_taylor_coreset_attention.py:452-457; with the unit weights of a
// fresh block this is the u < 0.5 of fast_article_attention.py:348), giving it
// the pair's summed weight; an odd last key is carried with its own weight.
// random keeps perm[:m] with weight n/m (:326-330), also used for blocks of
// <= 2 keys (:333-337).
//
// One CTA per (completed block, head).  Scores are float64 sums of exact
// float32*float32 products taken sequentially over the feature axis, so the
// order equals the one the CPU oracle computes; the sort is a shared-memory
// bitonic sort over (score, index) keys, so equal scores keep index order.
#include <float.h>
#include <math.h>

#include "sa_common.cuh"

namespace sa {

namespace {

constexpr int kCompressThreads = 256;

// Order-preserving map of a double to uint64 (NaN above +inf, -0 == +0).
__device__ __forceinline__ unsigned long long orderable(double x) {
  if (x != x) return 0xFFFFFFFFFFFFFFFEull;  // NaN: after every number
  x = x + 0.0;                               // -0.0 -> +0.0
  unsigned long long u = (unsigned long long)__double_as_longlong(x);
  return (u & 0x8000000000000000ull) ? ~u : (u | 0x8000000000000000ull);
}

__global__ void __launch_bounds__(kCompressThreads)
compress_blocks_kernel(const float* __restrict__ k, const float* __restrict__ v, int64_t n, int d, int dv,
                       int bs, int nc, int m, int pow2, int use_perm, const float* __restrict__ dirs,
                       const float* __restrict__ coins, const int32_t* __restrict__ perms,
                       int32_t* __restrict__ rep_idx, float* __restrict__ rep_k, float* __restrict__ rep_v,
                       float* __restrict__ rep_w, const SplitOut sp, int64_t idx_offset, int* status,
                       int stage) {
  extern __shared__ unsigned char smem_raw[];
  unsigned long long* skey = reinterpret_cast<unsigned long long*>(smem_raw);
  int* sidx = reinterpret_cast<int*>(skey + pow2);
  int* sel = sidx + pow2;
  float* selw = reinterpret_cast<float*>(sel + m);
  double* sdir = reinterpret_cast<double*>(
      reinterpret_cast<unsigned char*>(smem_raw) + (((size_t)pow2 * 12 + (size_t)m * 8 + 15) & ~(size_t)15));
  float* skb = reinterpret_cast<float*>(sdir + d);   // (stage) the block's keys, row stride d + 1

  const int c = blockIdx.x;
  const int64_t h = blockIdx.y;
  const int64_t start = (int64_t)c * bs;
  const int tid = threadIdx.x;
  const int64_t blk = h * nc + c;

  if (use_perm) {
    const float w = (float)((double)bs / (double)m);
    for (int p = tid; p < m; p += blockDim.x) {
      sel[p] = perms[blk * m + p];
      selw[p] = w;
    }
  } else {
    for (int a = tid; a < d; a += blockDim.x) sdir[a] = (double)dirs[blk * d + a];
    const float* kb = k + (h * n + start) * d;
    if (stage) {
      // the block's keys into shared memory with 16-byte loads (d % 4 == 0, 16-byte
      // aligned rows), rows d + 1 floats apart so that the per-thread row reads
      // below fall on distinct banks; the sum order is unchanged
      const int d4 = d >> 2;
      const float4* src = reinterpret_cast<const float4*>(kb);
      for (int e = tid; e < bs * d4; e += blockDim.x) {
        const float4 x = __ldg(src + e);
        const int r = e / d4, c = (e - r * d4) * 4;
        float* dst = skb + r * (d + 1) + c;
        dst[0] = x.x;
        dst[1] = x.y;
        dst[2] = x.z;
        dst[3] = x.w;
      }
    }
    __syncthreads();
    for (int t = tid; t < pow2; t += blockDim.x) {
      unsigned long long key = 0xFFFFFFFFFFFFFFFFull;  // padding sorts last
      if (t < bs) {
        double acc = 0.0;
        if (stage) {
          const float* row = skb + t * (d + 1);
          for (int a = 0; a < d; ++a) acc = fma((double)row[a], sdir[a], acc);
        } else {
          const float* row = kb + (int64_t)t * d;
          for (int a = 0; a < d; ++a) acc = fma((double)__ldg(row + a), sdir[a], acc);
        }
        key = orderable(acc);
      }
      skey[t] = key;
      sidx[t] = t;
    }
    __syncthreads();
    // bitonic sort, ascending by (key, index)
    for (int size = 2; size <= pow2; size <<= 1) {
      for (int stride = size >> 1; stride > 0; stride >>= 1) {
        for (int t = tid; t < (pow2 >> 1); t += blockDim.x) {
          const int lo = 2 * t - (t & (stride - 1));
          const int hi = lo + stride;
          const bool up = ((lo & size) == 0);
          const unsigned long long klo = skey[lo], khi = skey[hi];
          const int ilo = sidx[lo], ihi = sidx[hi];
          const bool gt = (klo > khi) || (klo == khi && ilo > ihi);
          if (gt == up) {
            skey[lo] = khi;
            skey[hi] = klo;
            sidx[lo] = ihi;
            sidx[hi] = ilo;
          }
        }
        __syncthreads();
      }
    }
    const int pairs = bs / 2;
    const float* cb = coins + (int64_t)blk * pairs;
    for (int p = tid; p < pairs; p += blockDim.x) {
      const float wa = 1.0f, wb = 1.0f;  // a fresh block has unit weights
      const float wsum = wa + wb;
      const float prob_a = wa / fmaxf(wsum, 1e-30f);
      const bool choose_a = cb[p] < prob_a;
      sel[p] = choose_a ? sidx[2 * p] : sidx[2 * p + 1];
      selw[p] = wsum;
    }
    if ((bs & 1) && tid == 0) {
      sel[pairs] = sidx[bs - 1];
      selw[pairs] = 1.0f;
    }
  }
  __syncthreads();

  // write the selection and gather the rep rows (one warp per rep); a
  // selected key lies in the block (perms come from a host table)
  const int64_t rbase = h * (int64_t)nc * m + (int64_t)c * m;
  const int64_t wbase = h * sp.w_stride + (int64_t)c * m;
  for (int p = tid; p < m; p += blockDim.x) {
    if (!SA_DEVICE_CHECK(sel[p] >= 0 && sel[p] < bs, status, 901, blk * m + p)) continue;
    if (rep_idx) rep_idx[rbase + p] = (int32_t)(idx_offset + start + sel[p]);
    if (rep_w) rep_w[wbase + p] = selw[p];
  }
  const int lane = tid & 31, warp = tid >> 5, nwarps = blockDim.x >> 5;
  for (int p = warp; p < m; p += nwarps) {
    if (!SA_DEVICE_CHECK(sel[p] >= 0 && sel[p] < bs, status, 901, blk * m + p)) continue;
    const int64_t src = h * n + start + sel[p];
    if (rep_k)
      for (int a = lane; a < d; a += 32) rep_k[(rbase + p) * d + a] = __ldg(k + src * d + a);
    if (rep_v)
      for (int a = lane; a < dv; a += 32) rep_v[(rbase + p) * dv + a] = __ldg(v + src * dv + a);
    if (sp.khi) {
      for (int a = lane; a < sp.dp; a += 32) {
        const float x = a < d ? __ldg(k + src * d + a) : 0.0f;
        const float hi = __uint_as_float(tc_split_hi(x));
        sp.khi[(rbase + p) * sp.dp + a] = hi;
        sp.klo[(rbase + p) * sp.dp + a] = x - hi;
      }
    }
  }
}

// Split rows of a [rows, cols] fp32 matrix into tf32 hi and fp32 remainder
// arrays of width cols_pad (zero padded), the operand format of the
// tensor-core residual.
__global__ void split_rows_kernel(const float* __restrict__ src, int64_t rows, int cols, int cols_pad,
                                  float* __restrict__ hi, float* __restrict__ lo) {
  const int64_t total = rows * cols_pad;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = e / cols_pad;
    const int c = (int)(e - r * cols_pad);
    const float x = c < cols ? __ldg(src + r * cols + c) : 0.0f;
    const float h = __uint_as_float(tc_split_hi(x));
    hi[e] = h;
    lo[e] = x - h;
  }
}

// The same split of n4 float4 elements (rows without padding).
__global__ void split_flat4_kernel(const float4* __restrict__ src, int64_t n4, float4* __restrict__ hi,
                                   float4* __restrict__ lo) {
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n4; e += (int64_t)gridDim.x * blockDim.x) {
    const float4 x = __ldg(src + e);
    const float4 h = make_float4(__uint_as_float(tc_split_hi(x.x)), __uint_as_float(tc_split_hi(x.y)),
                                 __uint_as_float(tc_split_hi(x.z)), __uint_as_float(tc_split_hi(x.w)));
    hi[e] = h;
    lo[e] = make_float4(x.x - h.x, x.y - h.y, x.z - h.z, x.w - h.w);
  }
}

// Transposing split: src [bh, rows, cols] -> hi / lo [bh, cols_pad, rows_pad]
// (tf32 hi and fp32 remainder, zero padded), through a 32 x 32 shared tile so
// that both the reads and the writes are coalesced.  This is the K-major
// layout of V for the tensor cores (keys contiguous per value column).
__global__ void split_transpose_kernel(const float* __restrict__ src, int64_t rows, int cols, int cols_pad,
                                       int64_t rows_pad, float* __restrict__ hi, float* __restrict__ lo) {
  __shared__ float tile[32][33];
  const int64_t h = blockIdx.z;
  const int64_t r0 = (int64_t)blockIdx.x * 32;
  const int c0 = blockIdx.y * 32;
  const int tx = threadIdx.x, ty = threadIdx.y;   // 32 x 8
  const float* sh = src + h * rows * cols;
  for (int yy = ty; yy < 32; yy += 8) {
    const int64_t r = r0 + yy;
    const int c = c0 + tx;
    tile[yy][tx] = (r < rows && c < cols) ? __ldg(sh + r * cols + c) : 0.0f;
  }
  __syncthreads();
  float* hh = hi + h * cols_pad * rows_pad;
  float* lh = lo + h * cols_pad * rows_pad;
  for (int yy = ty; yy < 32; yy += 8) {
    const int c = c0 + yy;
    const int64_t r = r0 + tx;
    if (c < cols_pad && r < rows_pad) {
      const float x = tile[tx][yy];
      const float xh = __uint_as_float(tc_split_hi(x));
      hh[(int64_t)c * rows_pad + r] = xh;
      lh[(int64_t)c * rows_pad + r] = x - xh;
    }
  }
}

// The same transposing split in 64-row x 64-column tiles with 16-byte loads and
// stores (cols % 4 == 0, rows_pad % 4 == 0, 16-byte aligned buffers): a warp
// moves 512 contiguous bytes per access instead of 128, and a CTA four times
// the data of the 32 x 32 form.
__global__ void __launch_bounds__(256)
split_transpose4_kernel(const float* __restrict__ src, int64_t rows, int cols, int cols_pad, int64_t rows_pad,
                        float* __restrict__ hi, float* __restrict__ lo) {
  __shared__ float tile[64][65];
  const int64_t h = blockIdx.z;
  const int64_t r0 = (int64_t)blockIdx.x * 64;
  const int c0 = blockIdx.y * 64;
  const int tid = threadIdx.x;
  const float* sh = src + h * rows * cols;
  // 64 rows x 16 float4 columns in; a column group c of 4 lies wholly inside
  // or outside the row (cols % 4 == 0)
  for (int e = tid; e < 64 * 16; e += 256) {
    const int r = e >> 4, q = e & 15;
    const int64_t row = r0 + r;
    const int col = c0 + 4 * q;
    float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
    if (row < rows && col < cols) x = __ldg(reinterpret_cast<const float4*>(sh + row * cols + col));
    tile[r][4 * q + 0] = x.x;
    tile[r][4 * q + 1] = x.y;
    tile[r][4 * q + 2] = x.z;
    tile[r][4 * q + 3] = x.w;
  }
  __syncthreads();
  float* hh = hi + h * cols_pad * rows_pad;
  float* lh = lo + h * cols_pad * rows_pad;
  // 64 output rows (value columns) x 16 float4 of keys out
  for (int e = tid; e < 64 * 16; e += 256) {
    const int cc = e >> 4, q = e & 15;
    const int c = c0 + cc;
    const int64_t rr = r0 + 4 * q;
    if (c < cols_pad && rr < rows_pad) {
      float x[4], xh[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        x[j] = tile[4 * q + j][cc];
        xh[j] = __uint_as_float(tc_split_hi(x[j]));
      }
      *reinterpret_cast<float4*>(hh + (int64_t)c * rows_pad + rr) = make_float4(xh[0], xh[1], xh[2], xh[3]);
      *reinterpret_cast<float4*>(lh + (int64_t)c * rows_pad + rr) =
          make_float4(x[0] - xh[0], x[1] - xh[1], x[2] - xh[2], x[3] - xh[3]);
    }
  }
}

}  // namespace

int launch_compress(const float* k, const float* v, int64_t bh, int64_t n, int d, int dv, int bs, int compressor,
                    const float* dirs, const float* coins, const int32_t* perms, int32_t* rep_idx, float* rep_k,
                    float* rep_v, float* rep_w, SplitOut sp, cudaStream_t stream, int64_t nc_force,
                    int64_t idx_offset, int* status) {
  // blocks to compress: the completed ones ((n - 1) / bs), or nc_force >= 0 blocks
  // (a shard of a longer sequence whose last block is completed by later tokens)
  const int64_t nc = nc_force >= 0 ? nc_force : (n > 0 ? (n - 1) / bs : 0);
  if (nc * (int64_t)bs > n) return set_error(SA_ERR_INVALID_ARG, "more blocks to compress than the sequence holds");
  const int m = (bs + 1) / 2;
  if (nc == 0 || bh == 0) return SA_OK;
  if (sp.w_stride == 0) sp.w_stride = nc * m;
  if (nc > 2147483647LL || bh > 65535) return set_error(SA_ERR_UNSUPPORTED, "too many blocks or heads for one launch");
  const bool use_perm = (compressor == SA_COMPRESSOR_RANDOM) || bs <= 2;
  if (use_perm && !perms) return set_error(SA_ERR_INVALID_ARG, "perms table is required");
  if (!use_perm && (!dirs || !coins)) return set_error(SA_ERR_INVALID_ARG, "dirs and coins tables are required");
  int pow2 = 1;
  while (pow2 < bs) pow2 <<= 1;
  if (pow2 > 4096) return set_error(SA_ERR_UNSUPPORTED, "block_size > 4096 is not supported by the compressor");
  // sorted_pair stages the block's keys in shared memory when they fit in 96 KB
  // and rows allow 16-byte loads
  const size_t key_tile = (size_t)bs * (size_t)(d + 1) * 4;
  const int stage = (!use_perm && (d & 3) == 0 && (reinterpret_cast<uintptr_t>(k) & 15) == 0 &&
                     key_tile <= 96 * 1024) ? 1 : 0;
  const size_t smem = (((size_t)pow2 * 12 + (size_t)m * 8 + 15) & ~(size_t)15) + (size_t)d * 8 +
                      (stage ? key_tile : 0);
  if (smem > 48 * 1024) {
    cudaFuncSetAttribute(compress_blocks_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  }
  dim3 grid((unsigned)nc, (unsigned)bh);
  compress_blocks_kernel<<<grid, kCompressThreads, smem, stream>>>(k, v, n, d, dv, bs, (int)nc, m, pow2,
                                                                   use_perm ? 1 : 0, dirs, coins, perms, rep_idx,
                                                                   rep_k, rep_v, rep_w, sp, idx_offset, status,
                                                                   stage);
  return check_launch("compress_blocks_kernel");
}

int launch_split_t(const float* src, int64_t bh, int64_t rows, int cols, int cols_pad, int64_t rows_pad, float* hi,
                   float* lo, cudaStream_t stream) {
  if (bh == 0 || rows_pad == 0) return SA_OK;
  if (bh > 65535 || (rows_pad + 31) / 32 > 2147483647LL)
    return set_error(SA_ERR_UNSUPPORTED, "too many sequences for one launch");
  if (cols % 4 == 0 && rows_pad % 4 == 0 &&
      ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(hi) | reinterpret_cast<uintptr_t>(lo)) & 15) ==
          0) {
    dim3 grid4((unsigned)((rows_pad + 63) / 64), (unsigned)((cols_pad + 63) / 64), (unsigned)bh);
    split_transpose4_kernel<<<grid4, 256, 0, stream>>>(src, rows, cols, cols_pad, rows_pad, hi, lo);
    return check_launch("split_transpose4_kernel");
  }
  dim3 grid((unsigned)((rows_pad + 31) / 32), (unsigned)((cols_pad + 31) / 32), (unsigned)bh);
  split_transpose_kernel<<<grid, dim3(32, 8), 0, stream>>>(src, rows, cols, cols_pad, rows_pad, hi, lo);
  return check_launch("split_transpose_kernel");
}

int launch_split(const float* src, int64_t rows, int cols, int cols_pad, float* hi, float* lo, cudaStream_t stream) {
  if (rows == 0) return SA_OK;
  const int64_t total = rows * cols_pad;
  const int threads = 256;
  if (cols == cols_pad && cols % 4 == 0 &&
      ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(hi) | reinterpret_cast<uintptr_t>(lo)) & 15) == 0) {
    // unpadded rows: the split is elementwise over the whole array, 16 bytes a thread
    const int64_t n4 = total / 4;
    const int64_t blocks = min((n4 + threads - 1) / threads, (int64_t)148 * 16);
    split_flat4_kernel<<<(unsigned)blocks, threads, 0, stream>>>(reinterpret_cast<const float4*>(src), n4,
                                                                 reinterpret_cast<float4*>(hi),
                                                                 reinterpret_cast<float4*>(lo));
    return check_launch("split_flat4_kernel");
  }
  const int64_t blocks = min((total + threads - 1) / threads, (int64_t)148 * 16);
  split_rows_kernel<<<(unsigned)blocks, threads, 0, stream>>>(src, rows, cols, cols_pad, hi, lo);
  return check_launch("split_rows_kernel");
}

}  // namespace sa
