// Segment-mean reps of the completed blocks (the deterministic coreset of the
// fused variant, triton_article_attention.py:190-245).
//
// Block c of a sequence (tokens c*bs .. c*bs+bs-1) is represented by the means
// of its bs/stride runs of `stride` adjacent tokens, each standing for stride
// keys (weight = stride).  Since bs is a multiple of stride, rep r of a head
// is the mean of tokens r*stride .. r*stride+stride-1: the reps of every
// completed block with a later query ((n-1)/bs blocks) form one [R, cols]
// array per head, R = (n-1)/bs * bs/stride.
//
// HBM-bound (reads R*stride rows, writes R rows): one thread per 4-column
// group of one rep row, consecutive threads on consecutive columns, so each
// of the stride loads of a warp is a coalesced row segment.
#include <algorithm>

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "sa_common.cuh"

namespace sa {

namespace {

// Round to the inputs' storage type: the reference's reps are tensors of the
// key dtype (a float16/bfloat16 mean is rounded to that type before the
// kernel reads it back as float32).
__device__ __forceinline__ float round_rep(float x, int rep_dtype) {
  if (rep_dtype == SA_REP_FLOAT16) return __half2float(__float2half_rn(x));
  if (rep_dtype == SA_REP_BFLOAT16) return __bfloat162float(__float2bfloat16_rn(x));
  return x;
}

__device__ __forceinline__ float4 add4(float4 a, float4 b) {
  return make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w);
}

// VEC = 4: float4 column groups (cols % 4 == 0, 16-byte aligned rows); 1: scalars.
template <int VEC>
__global__ void __launch_bounds__(256)
segment_mean_kernel(const float* __restrict__ src, int64_t n, int cols, int64_t R, int stride, float inv_stride,
                    int rep_dtype, int64_t groups, float* __restrict__ dst) {
  const int cg = cols / VEC;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < groups;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = e / cg;  // h * R + r
    const int c = (int)(e - row * cg) * VEC;
    const int64_t h = row / R;
    const int64_t r = row - h * R;
    const float* p = src + (h * n + r * stride) * cols + c;
    float* o = dst + row * cols + c;
    if constexpr (VEC == 4) {
      float4 acc = __ldg(reinterpret_cast<const float4*>(p));
      for (int t = 1; t < stride; ++t) acc = add4(acc, __ldg(reinterpret_cast<const float4*>(p + (int64_t)t * cols)));
      *reinterpret_cast<float4*>(o) =
          make_float4(round_rep(acc.x * inv_stride, rep_dtype), round_rep(acc.y * inv_stride, rep_dtype),
                      round_rep(acc.z * inv_stride, rep_dtype), round_rep(acc.w * inv_stride, rep_dtype));
    } else {
      float acc = __ldg(p);
      for (int t = 1; t < stride; ++t) acc += __ldg(p + (int64_t)t * cols);
      *o = round_rep(acc * inv_stride, rep_dtype);
    }
  }
}

int launch_one(const float* src, int64_t bh, int64_t n, int cols, int64_t R, int stride, int rep_dtype, float* dst,
               cudaStream_t s) {
  const bool vec = cols % 4 == 0 && ((uintptr_t)src % 16) == 0 && ((uintptr_t)dst % 16) == 0;
  const int64_t groups = bh * R * (vec ? cols / 4 : cols);
  if (groups == 0) return SA_OK;
  // the mean multiplies by 1/stride, as torch's mean reduction does
  const float inv = 1.0f / (float)stride;
  const int64_t blocks = std::min<int64_t>((groups + 255) / 256, (int64_t)148 * 16);
  if (vec)
    segment_mean_kernel<4><<<(unsigned)blocks, 256, 0, s>>>(src, n, cols, R, stride, inv, rep_dtype, groups, dst);
  else
    segment_mean_kernel<1><<<(unsigned)blocks, 256, 0, s>>>(src, n, cols, R, stride, inv, rep_dtype, groups, dst);
  return check_launch("segment_mean_kernel");
}

__global__ void fill_kernel(float* __restrict__ dst, int64_t count, float value) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < count; i += (int64_t)gridDim.x * blockDim.x)
    dst[i] = value;
}

}  // namespace

// rep_k [bh, R, d] and rep_v [bh, R, dv] from k [bh, n, d], v [bh, n, dv].
int launch_segment_mean(const float* k, const float* v, int64_t bh, int64_t n, int d, int dv, int bs, int stride,
                        int key_dtype, int value_dtype, float* rep_k, float* rep_v, cudaStream_t s) {
  const int64_t nc = n > 0 ? (n - 1) / bs : 0;
  const int64_t R = nc * (bs / stride);
  if (bh == 0 || R == 0) return SA_OK;
  int rc = launch_one(k, bh, n, d, R, stride, key_dtype, rep_k, s);
  if (rc) return rc;
  return launch_one(v, bh, n, dv, R, stride, value_dtype, rep_v, s);
}

int launch_fill(float* dst, int64_t count, float value, cudaStream_t s) {
  if (count == 0) return SA_OK;
  const int64_t blocks = std::min<int64_t>((count + 255) / 256, (int64_t)148 * 8);
  fill_kernel<<<(unsigned)blocks, 256, 0, s>>>(dst, count, value);
  return check_launch("fill_kernel");
}

}  // namespace sa
