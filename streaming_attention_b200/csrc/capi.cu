// C ABI of libsa_b200.so (declared in include/streaming_attention.h).
//
// Argument checks mirror the reference's ValueError conditions
// (fast_article_attention.py:552-561, :361, :392-393) and report them as
// SA_ERR_INVALID_ARG with a message; every CUDA error is caught here and
// returned as SA_ERR_CUDA.  No entry point allocates device memory: outputs
// and scratch belong to the caller.
//
// Two kernel families:
//  * tensor cores (tcgen05 / TMEM / TMA, 3xTF32) for d <= 64, dv <= 128
//    (residual) and dv <= 64 (moments): the operands are first split into a
//    tf32 "hi" and an fp32 remainder by split_rows_kernel / the compressor;
//  * CUDA cores (fp32 FMA) for every other shape, and on request
//    (SA_FORCE_SIMT=1, for A/B comparisons).
#include <cuda.h>
#include <stdarg.h>

#include <atomic>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "sa_common.cuh"

namespace sa {

int launch_compress(const float* k, const float* v, int64_t bh, int64_t n, int d, int dv, int bs, int compressor,
                    const float* dirs, const float* coins, const int32_t* perms, int32_t* rep_idx, float* rep_k,
                    float* rep_v, float* rep_w, SplitOut sp, cudaStream_t stream,
                    int64_t nc_force = -1, int64_t idx_offset = 0, int* status = nullptr);
int launch_split(const float* src, int64_t rows, int cols, int cols_pad, float* hi, float* lo, cudaStream_t stream);
int launch_split_t(const float* src, int64_t bh, int64_t rows, int cols, int cols_pad, int64_t rows_pad, float* hi,
                   float* lo, cudaStream_t stream);
int residual_tc_dp(int d);
int residual_tc_dvp(int dv);
int launch_residual_tc(const CUtensorMap* maps, const float* q, const float* rep_w, int64_t r_pad, const float* low,
                       int groups, float* out, int* status, int64_t bh, int64_t n, int d, int dv, int degree, int bs,
                       int64_t m_blk, float scale, float eps, cudaStream_t stream, int64_t c_off = 0,
                       bool clamp_exp = false);
int moments_tc_groups(int d, int dv, int degree);
int64_t moments_tc_master_floats(int64_t bh, int d, int dv, int degree);
int launch_moments_tc(const CUtensorMap* maps, const float* q, const float* k, float* part, float* master,
                      int* status, int64_t bh, int64_t n, int d, int dv, int degree, int bs, float scale,
                      cudaStream_t stream, int mode = 0, float* den_io = nullptr);
int launch_sum_groups(const float* part, int groups, int64_t stride, float* out, cudaStream_t stream);
int64_t moments_tc_den_floats(int64_t bh, int d, int dv, int degree);
int launch_state_prefix(const float* states, int nprev, int64_t n_master, int64_t n_den, float* master, float* den,
                        cudaStream_t stream);
int launch_low_moments(const float* q, const float* k, const float* v, int64_t bh, int64_t n, int d, int dv,
                       int degree, int bs, float scale, float* low, cudaStream_t stream);
int launch_residual(const float* q, const float* k, const float* v, const float* rk, const float* rv,
                    const float* rw, const float* low, int64_t bh, int64_t n, int d, int dv, int degree, int bs,
                    int compressor, float scale, float eps, float* out, cudaStream_t s);
int launch_residual_reps(const float* q, const float* k, const float* v, const float* rk, const float* rv,
                         const float* rw, const float* low, int64_t bh, int64_t n, int d, int dv, int degree, int bs,
                         int64_t m_blk, int64_t rph, float scale, float eps, bool clamp, float* out, cudaStream_t s);
int launch_segment_mean(const float* k, const float* v, int64_t bh, int64_t n, int d, int dv, int bs, int stride,
                        int key_dtype, int value_dtype, float* rep_k, float* rep_v, cudaStream_t s);
int launch_fill(float* dst, int64_t count, float value, cudaStream_t s);
int launch_flash_tc(const CUtensorMap* maps, const float* q, float* out, int* status, int64_t bh, int64_t n, int d,
                    int dv, float scale, cudaStream_t stream);
int launch_flash_simt(const float* q, const float* k, const float* v, int64_t bh, int64_t n, int d, int dv,
                      float scale, float* out, cudaStream_t s);

namespace {
thread_local char g_err[512] = {0};
// sa_set_wait_limit_ns (0: the default)
std::atomic<uint64_t> g_wait_limit_ns{0};
// sa_set_stage_events, per host thread
constexpr int kMaxStageEvents = 8;
thread_local cudaEvent_t g_stage_events[kMaxStageEvents] = {};
thread_local int g_stage_count = 0;

// Records stage event i of sa_fast_attention on stream s, if the calling
// thread asked for it.
void stage_mark(int i, cudaStream_t s) {
  if (i < g_stage_count && g_stage_events[i]) cudaEventRecord(g_stage_events[i], s);
}
}  // namespace

uint64_t wait_limit_ns() {
  const uint64_t v = g_wait_limit_ns.load(std::memory_order_relaxed);
  return v ? v : 2000000000ull;
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

// Reps per completed block of the merge-reduce compressors; compressor none
// reads every key of a block as its own rep.
inline int64_t reps_per_block(int compressor, int bs) {
  return compressor == SA_COMPRESSOR_NONE ? bs : (bs + 1) / 2;
}

constexpr size_t kAlign = 256;
inline size_t align_up(size_t x) { return (x + kAlign - 1) & ~(kAlign - 1); }

bool force_simt() {
  const char* force = getenv("SA_FORCE_SIMT");
  return force && force[0] == '1';
}

// Workspace layout.  Offset 0 always holds the launch status word (int, 0 = ok).
// tc:     tensor-core residual: tf32 hi / fp32 remainder copies of k, v
//         (padded to dp / dvp columns) and of the gathered reps; rep weights
//         padded per sequence to a multiple of 64.
// groups: >0 when the tensor-core moment kernel runs: `low` then holds that
//         many partial slices [groups, bh, n, dv+1] (summed by the residual).
struct Workspace {
  bool tc = false;
  int groups = 0;
  int dp = 0, dvp = 0;
  int64_t R = 0, r_pad = 0, n_pad = 0;
  // k splits are row-major [bh, rows, dp]; v splits are transposed, [bh, dvp, pitch]
  // (keys contiguous: the K-major layout of V for the tensor cores)
  size_t status = 0, low = 0, master = 0, khi = 0, klo = 0, vthi = 0, vtlo = 0;
  size_t rkhi = 0, rklo = 0, rvthi = 0, rvtlo = 0, rep_k = 0, rep_v = 0, rep_w = 0, rep_idx = 0, total = 0;
  size_t den_io = 0;  // sharded forward: the feature sums of the moment state
};

// kSegment: the segment-mean variant (reps made by the segment-mean kernel as
// plain rows, then split; `stride` adjacent tokens per rep, 1 = the keys).
enum class Plan { kFull, kResidualOnly, kMomentsOnly, kSegment };

Workspace plan(int64_t bh, int64_t n, int d, int dv, int degree, int bs, int compressor, Plan what, int stride = 0) {
  Workspace w{};
  const bool simt = force_simt();
  w.dp = residual_tc_dp(d);
  w.dvp = residual_tc_dvp(dv);
  // TMA reads V^T tiles starting at block boundaries: the key coordinate must be
  // a multiple of 4 floats (16 bytes)
  const bool aligned_blocks = bs % 4 == 0;
  w.tc = w.dp > 0 && w.dvp > 0 && !simt && aligned_blocks;
  w.groups = (!simt && aligned_blocks && what != Plan::kResidualOnly) ? moments_tc_groups(d, dv, degree) : 0;
  if (w.groups > 0 && w.dvp == 0) w.dvp = dv <= 32 ? 32 : 64;
  const int64_t nc = n > 0 ? (n - 1) / bs : 0;
  if (what == Plan::kSegment)
    w.R = stride > 1 ? nc * (bs / stride) : 0;
  else
    w.R = (compressor == SA_COMPRESSOR_NONE) ? 0 : nc * ((bs + 1) / 2);
  w.r_pad = (w.R + 63) / 64 * 64;
  w.n_pad = (n + 3) / 4 * 4;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t at = off;
    off = align_up(off + bytes);
    return at;
  };
  const size_t f = sizeof(float);
  w.status = take(16);   // status word, then the index of a failed device check
  if (what != Plan::kResidualOnly) w.low = take((size_t)(w.groups > 0 ? w.groups : 1) * bh * n * (dv + 1) * f);
  if (w.groups > 0) w.master = take((size_t)moments_tc_master_floats(bh, d, dv, degree) * f);
  const bool need_v_split = w.groups > 0 || (w.tc && what != Plan::kMomentsOnly);
  if (w.tc && what != Plan::kMomentsOnly) {
    w.khi = take((size_t)bh * n * w.dp * f);
    w.klo = take((size_t)bh * n * w.dp * f);
  }
  if (need_v_split) {
    w.vthi = take((size_t)bh * w.dvp * w.n_pad * f);
    w.vtlo = take((size_t)bh * w.dvp * w.n_pad * f);
  }
  if (what != Plan::kMomentsOnly) {
    const bool seg = what == Plan::kSegment;
    if (w.tc) {
      w.rkhi = take((size_t)bh * w.R * w.dp * f);
      w.rklo = take((size_t)bh * w.R * w.dp * f);
      w.rvthi = take((size_t)bh * w.dvp * w.r_pad * f);
      w.rvtlo = take((size_t)bh * w.dvp * w.r_pad * f);
      w.rep_w = take((size_t)bh * w.r_pad * f);
      if (seg) w.rep_k = take((size_t)bh * w.R * d * f);   // segment means, then split
      if (what == Plan::kFull || seg) w.rep_v = take((size_t)bh * w.R * dv * f);   // rep rows, then transposed
    } else if (what == Plan::kFull || seg) {
      w.rep_k = take((size_t)bh * w.R * d * f);
      w.rep_v = take((size_t)bh * w.R * dv * f);
      w.rep_w = take((size_t)bh * w.R * f);
    }
    if (what == Plan::kFull) w.rep_idx = take((size_t)bh * w.R * sizeof(int32_t));
  }
  w.total = off;
  return w;
}

// The driver's tensor-map encoder, looked up at run time so that the library
// loads on machines without a driver (the CPU-side tests only load it).
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_tiled_fn() {
  static EncodeTiledFn fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// 3-D tensor map over a [outer, rows, pitch] fp32 array of which the first
// `inner` entries of each row are valid; box {32, box_rows, 1}, zero fill out of
// bounds.
int encode_map(CUtensorMap* map, const void* base, int64_t inner, int64_t pitch, int64_t rows, int64_t outer,
               int box_rows, CUtensorMapSwizzle swizzle) {
  if (inner < 1) inner = 1;
  if (pitch < inner) pitch = inner;
  cuuint64_t dims[3] = {(cuuint64_t)inner, (cuuint64_t)(rows > 0 ? rows : 1), (cuuint64_t)(outer > 0 ? outer : 1)};
  cuuint64_t strides[2] = {(cuuint64_t)pitch * 4, (cuuint64_t)pitch * 4 * (cuuint64_t)(rows > 0 ? rows : 1)};
  cuuint32_t box[3] = {32, (cuuint32_t)box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  const EncodeTiledFn enc = encode_tiled_fn();
  if (!enc) return set_error(SA_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<void*>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(SA_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return SA_OK;
}

int encode_map_3d(CUtensorMap* map, const void* base, int inner, int64_t rows, int64_t outer, int box_rows,
                  CUtensorMapSwizzle swizzle) {
  return encode_map(map, base, inner, inner, rows, outer, box_rows, swizzle);
}

// Split operands of one key set (the reps, or every key of the sequences).
struct TCOperands {
  const float* khi;
  const float* klo;
  int64_t krows;          // k splits: [bh, krows, dp]
  const float* vthi;
  const float* vtlo;
  int64_t vrows, vpitch;  // v splits: [bh, dvp, vpitch], vrows valid keys
};

// Tensor maps over the split operands, then the tensor-core residual.  Both
// operands are K-major with the 128-byte swizzle: K tiles are 64 key rows of a
// 32-column chunk; V^T tiles are dvp value rows of a 32-key chunk.
int residual_tc_from_split(const Workspace& w, const TCOperands& rep, const TCOperands& cur, const float* rep_w,
                           const float* q, const float* low, int groups, float* out, int* status, int64_t bh,
                           int64_t n, int d, int dv, int degree, int block_size, int64_t m_blk, float scale,
                           float eps, cudaStream_t s, int64_t c_off = 0, bool clamp_exp = false) {
  CUtensorMap maps[8];
  const TCOperands* ops[2] = {&rep, &cur};
  for (int j = 0; j < 2; ++j) {
    const TCOperands& o = *ops[j];
    int rc = encode_map_3d(&maps[4 * j + 0], o.khi, w.dp, o.krows, bh, 64, CU_TENSOR_MAP_SWIZZLE_128B);
    if (!rc) rc = encode_map_3d(&maps[4 * j + 1], o.klo, w.dp, o.krows, bh, 64, CU_TENSOR_MAP_SWIZZLE_128B);
    if (!rc) rc = encode_map(&maps[4 * j + 2], o.vthi, o.vrows, o.vpitch, w.dvp, bh, w.dvp, CU_TENSOR_MAP_SWIZZLE_128B);
    if (!rc) rc = encode_map(&maps[4 * j + 3], o.vtlo, o.vrows, o.vpitch, w.dvp, bh, w.dvp, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  return launch_residual_tc(maps, q, rep_w, w.r_pad, low, groups, out, status, bh, n, d, dv, degree, block_size,
                            m_blk, scale, eps, s, c_off, clamp_exp);
}

// Tensor-core moments into `part` ([groups, bh, n, dv+1]) from the transposed
// split v ([bh, dvp, n_pad]; K-major tiles of dvp value rows x 32 keys).
int moments_tc_from_split(const Workspace& w, char* ws, const float* vthi, const float* vtlo, const float* q,
                          const float* k, float* part, int* status, int64_t bh, int64_t n, int d, int dv, int degree,
                          int block_size, float scale, cudaStream_t s, int mode = 0, float* den_io = nullptr) {
  CUtensorMap maps[2];
  int rc = encode_map(&maps[0], vthi, n, w.n_pad, w.dvp, bh, w.dvp, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = encode_map(&maps[1], vtlo, n, w.n_pad, w.dvp, bh, w.dvp, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  float* master = reinterpret_cast<float*>(ws + w.master);
  return launch_moments_tc(maps, q, k, part, master, status, bh, n, d, dv, degree, block_size, scale, s, mode,
                           den_io);
}

// Workspace of the sharded forward (one shard of a sequence split along N).
// Buffers that do not depend on rep_rows come first, so begin (which does not
// know rep_rows yet) and end see the same offsets.
Workspace plan_shard(int64_t bh, int64_t n, int d, int dv, int degree, int bs, int64_t rep_rows) {
  Workspace w{};
  w.dp = residual_tc_dp(d);
  w.dvp = residual_tc_dvp(dv);
  w.tc = w.dp > 0 && w.dvp > 0 && bs % 4 == 0 && !force_simt();
  w.groups = w.tc ? moments_tc_groups(d, dv, degree) : 0;
  if (w.groups == 0) w.tc = false;
  w.R = rep_rows;
  w.r_pad = (rep_rows + 63) / 64 * 64;
  w.n_pad = (n + 3) / 4 * 4;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t at = off;
    off = align_up(off + bytes);
    return at;
  };
  const size_t f = sizeof(float);
  w.status = take(16);   // status word, then the index of a failed device check
  w.low = take((size_t)2 * (w.groups > 0 ? w.groups : 1) * bh * n * (dv + 1) * f);   // local + prefix slices
  w.master = take((size_t)moments_tc_master_floats(bh, d, dv, degree) * f);
  w.den_io = take((size_t)moments_tc_den_floats(bh, d, dv, degree) * f);
  w.khi = take((size_t)bh * n * w.dp * f);
  w.klo = take((size_t)bh * n * w.dp * f);
  w.vthi = take((size_t)bh * w.dvp * w.n_pad * f);
  w.vtlo = take((size_t)bh * w.dvp * w.n_pad * f);
  w.rkhi = take((size_t)bh * w.R * w.dp * f);
  w.rklo = take((size_t)bh * w.R * w.dp * f);
  w.rvthi = take((size_t)bh * w.dvp * w.r_pad * f);
  w.rvtlo = take((size_t)bh * w.dvp * w.r_pad * f);
  w.rep_w = take((size_t)bh * w.r_pad * f);
  w.total = off;
  return w;
}

// Argument checks of the segment-mean variant, in the reference's order
// (triton_article_attention.py:487-501); the width limits belong to the
// forward only (the rep builder, :216-223, takes any width).
int check_segment(const void* q, const void* k, const void* v, int64_t bh, int64_t n, int d, int dv, int degree,
                  int bs, int stride, int key_dtype, int value_dtype, bool forward = true) {
  if (degree < 0 || degree > 2)
    return set_error(SA_ERR_UNSUPPORTED, "the segment-mean variant supports degree 0, 1, or 2");
  if (bs <= 0 || stride <= 0) return set_error(SA_ERR_INVALID_ARG, "block_size and compress_stride must be positive");
  if (bs % stride != 0) return set_error(SA_ERR_INVALID_ARG, "block_size must be divisible by compress_stride");
  int rc = check_common(q, k, v, bh, n, d, dv, degree, bs);
  if (rc) return rc;
  if (forward && d > 128) return set_error(SA_ERR_INVALID_ARG, "this compact kernel supports D <= 128");
  if (forward && dv > 256) return set_error(SA_ERR_INVALID_ARG, "this compact kernel supports Dv <= 256");
  if (forward && dv > 128) return set_error(SA_ERR_UNSUPPORTED, "value_dim above 128: split the value columns");
  for (const int t : {key_dtype, value_dtype})
    if (t < SA_REP_FLOAT32 || t > SA_REP_BFLOAT16)
      return set_error(SA_ERR_INVALID_ARG, "rep dtypes must be SA_REP_FLOAT32, SA_REP_FLOAT16 or SA_REP_BFLOAT16");
  return SA_OK;
}

// Workspace of the exact flash kernel: the status word and the tf32 splits of
// k ([bh, n, dp]) and of v transposed ([bh, dvp, n_pad]); empty on the
// CUDA-core path (d > 64, dv > 128, or SA_FORCE_SIMT=1).
Workspace plan_flash(int64_t bh, int64_t n, int d, int dv) {
  Workspace w{};
  w.dp = residual_tc_dp(d);
  w.dvp = residual_tc_dvp(dv);
  w.tc = w.dp > 0 && w.dvp > 0 && !force_simt();
  if (!w.tc) return w;
  w.n_pad = (n + 3) / 4 * 4;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t at = off;
    off = align_up(off + bytes);
    return at;
  };
  const size_t f = sizeof(float);
  w.status = take(16);   // status word, then the index of a failed device check
  w.khi = take((size_t)bh * n * w.dp * f);
  w.klo = take((size_t)bh * n * w.dp * f);
  w.vthi = take((size_t)bh * w.dvp * w.n_pad * f);
  w.vtlo = take((size_t)bh * w.dvp * w.n_pad * f);
  w.total = off;
  return w;
}

int check_flash(const void* q, const void* k, const void* v, int64_t bh, int64_t n, int d, int dv) {
  if (bh < 0 || n < 0) return set_error(SA_ERR_INVALID_ARG, "bh and n must be non-negative");
  if (d <= 0 || dv <= 0) return set_error(SA_ERR_INVALID_ARG, "dim and value_dim must be positive");
  if (d > 128) return set_error(SA_ERR_INVALID_ARG, "this compact kernel supports D <= 128");
  if (dv > 256) return set_error(SA_ERR_INVALID_ARG, "this compact kernel supports Dv <= 256");
  if (bh > 0 && n > 0 && (!q || !k || !v)) return set_error(SA_ERR_INVALID_ARG, "null input pointer");
  if (n > ((int64_t)1 << 31)) return set_error(SA_ERR_UNSUPPORTED, "sequence length above 2^31");
  return SA_OK;
}

int check_workspace(const Workspace& w, const void* workspace, size_t workspace_bytes) {
  if (!workspace || workspace_bytes < w.total)
    return set_error(SA_ERR_WORKSPACE, "workspace of %zu bytes is smaller than the %zu required", workspace_bytes,
                     w.total);
  if (((uintptr_t)workspace) % kAlign)
    return set_error(SA_ERR_INVALID_ARG, "workspace must be %zu-byte aligned", kAlign);
  return SA_OK;
}

// The status word and, 8 bytes further, the index a failed device check
// recorded (checks builds): both cleared at the start of every call.
int reset_status(int* status, cudaStream_t s) {
  const cudaError_t ce = cudaMemsetAsync(status, 0, 16, s);
  if (ce != cudaSuccess) return set_error(SA_ERR_CUDA, "status reset: %s", cudaGetErrorString(ce));
  return SA_OK;
}

}  // namespace
}  // namespace sa

using namespace sa;

namespace sa {
namespace {

// The moment scan's own stream for one caller stream (per host thread and
// device), and the two events that fork the forward onto it and join it back.
struct ForkStreams {
  cudaStream_t caller;
  int device;
  cudaStream_t moments;
  cudaEvent_t fork, join;
};
constexpr int kMaxForks = 16;
thread_local ForkStreams g_forks[kMaxForks];
thread_local int g_nforks = 0;
// sa_set_moment_fork, per host thread
thread_local bool g_fork_enabled = true;

// The fork record of caller stream s on the current device, made at its first
// use (a stream of the device's highest priority and two events); nullptr when
// the stream is being captured into a graph, when this thread already has
// kMaxForks records, or when making one fails -- the forward then runs in
// order on s.
ForkStreams* fork_for(cudaStream_t s) {
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(s, &cap) != cudaSuccess || cap != cudaStreamCaptureStatusNone) {
    cudaGetLastError();
    return nullptr;
  }
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  for (int i = 0; i < g_nforks; ++i)
    if (g_forks[i].caller == s && g_forks[i].device == dev) return &g_forks[i];
  if (g_nforks == kMaxForks) return nullptr;
  int least = 0, greatest = 0;
  ForkStreams f{s, dev, nullptr, nullptr, nullptr};
  bool ok = cudaDeviceGetStreamPriorityRange(&least, &greatest) == cudaSuccess &&
            cudaStreamCreateWithPriority(&f.moments, cudaStreamNonBlocking, greatest) == cudaSuccess &&
            cudaEventCreateWithFlags(&f.fork, cudaEventDisableTiming) == cudaSuccess &&
            cudaEventCreateWithFlags(&f.join, cudaEventDisableTiming) == cudaSuccess;
  if (!ok) {
    cudaGetLastError();
    if (f.join) cudaEventDestroy(f.join);
    if (f.fork) cudaEventDestroy(f.fork);
    if (f.moments) cudaStreamDestroy(f.moments);
    return nullptr;
  }
  g_forks[g_nforks] = f;
  return &g_forks[g_nforks++];
}

}  // namespace

// One forward of the fast path (sa_fast_attention).  In order on the caller's
// stream: the k and v splits, the compressor and the split of its rep values,
// the moment scan, the residual.  With `allow_fork` (and the tensor-core
// kernels, a compressor, no stage events and no graph capture) the v split and
// the moment scan run on a stream of the device's highest priority while the
// caller's stream runs the k split, the compressor and the rep split, and the
// residual waits for both: the moment scan holds one CTA per SM, so when it
// leaves SMs idle (fewer than 148 CTAs in its last round) the compressor's
// small CTAs run there, and the priority keeps them from delaying it.
int fast_attention_run(const float* q, const float* k, const float* v, int64_t bh, int64_t n, int d, int dv,
                       int degree, int block_size, float scale, int compressor, const float* dirs, const float* coins,
                       const int32_t* perms, float eps, float* out, int32_t* rep_idx, void* workspace,
                       size_t workspace_bytes, void* stream, bool allow_fork) {
  int rc = check_common(q, k, v, bh, n, d, dv, degree, block_size);
  if (rc) return rc;
  rc = check_compressor(compressor);
  if (rc) return rc;
  if (bh == 0 || n == 0) return SA_OK;
  if (!out) return set_error(SA_ERR_INVALID_ARG, "null output pointer");
  const Workspace w = plan(bh, n, d, dv, degree, block_size, compressor, Plan::kFull);
  rc = check_workspace(w, workspace, workspace_bytes);
  if (rc) return rc;
  char* ws = static_cast<char*>(workspace);
  float* low = reinterpret_cast<float*>(ws + w.low);
  int* status = reinterpret_cast<int*>(ws + w.status);
  cudaStream_t s = (cudaStream_t)stream;
  const int64_t nc = (n - 1) / block_size;
  const bool compress = compressor != SA_COMPRESSOR_NONE && nc > 0;
  int32_t* ridx = rep_idx ? rep_idx : reinterpret_cast<int32_t*>(ws + w.rep_idx);
  rc = reset_status(status, s);
  if (rc) return rc;
  stage_mark(0, s);

  // operand splits shared by the tensor-core kernels
  float* khi = reinterpret_cast<float*>(ws + w.khi);
  float* klo = reinterpret_cast<float*>(ws + w.klo);
  float* vthi = reinterpret_cast<float*>(ws + w.vthi);
  float* vtlo = reinterpret_cast<float*>(ws + w.vtlo);
  const int groups = w.groups > 0 ? w.groups : 1;

  auto split_v = [&](cudaStream_t st) -> int {
    if (w.tc || w.groups > 0) return launch_split_t(v, bh, n, dv, w.dvp, w.n_pad, vthi, vtlo, st);
    return SA_OK;
  };
  auto moments = [&](cudaStream_t st) -> int {
    if (w.groups > 0)
      return moments_tc_from_split(w, ws, vthi, vtlo, q, k, low, status, bh, n, d, dv, degree, block_size, scale, st);
    return launch_low_moments(q, k, v, bh, n, d, dv, degree, block_size, scale, low, st);
  };

  // C1: compressor (and the split of its rep values)
  const float* rk = k;
  const float* rv = v;
  float* rw = nullptr;
  const TCOperands cur_ops{khi, klo, n, vthi, vtlo, n, w.n_pad};
  TCOperands rep_ops = cur_ops;
  auto compress_reps = [&](cudaStream_t st) -> int {
    if (!compress) return SA_OK;
    if (w.tc) {
      SplitOut sp;
      sp.khi = reinterpret_cast<float*>(ws + w.rkhi);
      sp.klo = reinterpret_cast<float*>(ws + w.rklo);
      sp.dp = w.dp;
      sp.w_stride = w.r_pad;
      rw = reinterpret_cast<float*>(ws + w.rep_w);
      float* rep_v = reinterpret_cast<float*>(ws + w.rep_v);
      const cudaError_t ce = cudaMemsetAsync(rw, 0, (size_t)bh * w.r_pad * sizeof(float), st);
      if (ce != cudaSuccess) return set_error(SA_ERR_CUDA, "rep weight reset: %s", cudaGetErrorString(ce));
      int r = launch_compress(k, v, bh, n, d, dv, block_size, compressor, dirs, coins, perms, ridx, nullptr, rep_v,
                              rw, sp, st, -1, 0, status);
      if (r) return r;
      float* rvthi = reinterpret_cast<float*>(ws + w.rvthi);
      float* rvtlo = reinterpret_cast<float*>(ws + w.rvtlo);
      r = launch_split_t(rep_v, bh, w.R, dv, w.dvp, w.r_pad, rvthi, rvtlo, st);
      if (r) return r;
      rep_ops = TCOperands{sp.khi, sp.klo, w.R, rvthi, rvtlo, w.R, w.r_pad};
      return SA_OK;
    }
    float* rep_k = reinterpret_cast<float*>(ws + w.rep_k);
    float* rep_v = reinterpret_cast<float*>(ws + w.rep_v);
    rw = reinterpret_cast<float*>(ws + w.rep_w);
    const int r = launch_compress(k, v, bh, n, d, dv, block_size, compressor, dirs, coins, perms, ridx, rep_k, rep_v,
                                  rw, SplitOut{}, st, -1, 0, status);
    if (r) return r;
    rk = rep_k;
    rv = rep_v;
    return SA_OK;
  };

  ForkStreams* f = nullptr;
  if (allow_fork && g_fork_enabled && w.tc && w.groups > 0 && compress && g_stage_count == 0) f = fork_for(s);
  if (f) {
    cudaError_t ce = cudaEventRecord(f->fork, s);
    if (ce == cudaSuccess) ce = cudaStreamWaitEvent(f->moments, f->fork, 0);
    if (ce != cudaSuccess) return set_error(SA_ERR_CUDA, "fork of the moment scan: %s", cudaGetErrorString(ce));
    // the moment scan's stream first, so that its CTAs are queued before the compressor's
    rc = split_v(f->moments);
    if (!rc) rc = moments(f->moments);
    int rc2 = launch_split(k, bh * n, d, w.dp, khi, klo, s);
    if (!rc2) rc2 = compress_reps(s);
    // join even after a failed launch: nothing of this call may outlive it on the side stream
    ce = cudaEventRecord(f->join, f->moments);
    if (ce == cudaSuccess) ce = cudaStreamWaitEvent(s, f->join, 0);
    if (rc) return rc;
    if (rc2) return rc2;
    if (ce != cudaSuccess) return set_error(SA_ERR_CUDA, "join of the moment scan: %s", cudaGetErrorString(ce));
  } else {
    if (w.tc) {
      rc = launch_split(k, bh * n, d, w.dp, khi, klo, s);
      if (rc) return rc;
    }
    rc = split_v(s);
    if (rc) return rc;
    stage_mark(1, s);
    rc = compress_reps(s);
    if (rc) return rc;
    stage_mark(2, s);
    rc = moments(s);
    if (rc) return rc;
    stage_mark(3, s);
  }

  // R: residual + combine
  if (w.tc) {
    rc = residual_tc_from_split(w, rep_ops, cur_ops, rw, q, low, groups, out, status, bh, n, d, dv, degree,
                                block_size, reps_per_block(compressor, block_size), scale, eps, s);
  } else {
    if (groups > 1)  // the CUDA-core residual reads one summed slice
      rc = launch_sum_groups(low, groups, bh * n * (dv + 1), low, s);
    if (!rc)
      rc = launch_residual(q, k, v, rk, rv, rw, low, bh, n, d, dv, degree, block_size, compressor, scale, eps, out,
                           s);
  }
  if (!rc) stage_mark(4, s);
  return rc;
}

}  // namespace sa

extern "C" {

int sa_version(void) { return 110; }

int sa_workspace_status(const void* workspace, void* stream) {
  if (!workspace) return set_error(SA_ERR_INVALID_ARG, "null workspace");
  int64_t word[2] = {0, 0};   // status word (low 4 bytes of word[0]), then a failed check's index
  cudaError_t e = cudaMemcpyAsync(word, workspace, sizeof(word), cudaMemcpyDeviceToHost, (cudaStream_t)stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize((cudaStream_t)stream);
  if (e != cudaSuccess) return set_error(SA_ERR_CUDA, "status read: %s", cudaGetErrorString(e));
  int code = 0;
  memcpy(&code, word, sizeof(int));
  if (code >= kCheckFirst && code <= kCheckLast)
    return set_error(SA_ERR_DEVICE_CHECK, "device check %d failed at index %lld", code, (long long)word[1]);
  if (code != 0) return set_error(SA_ERR_TIMEOUT, "a bounded device-side wait gave up (wait code %d)", code);
  return SA_OK;
}

int sa_set_moment_fork(int enable) {
  g_fork_enabled = enable != 0;
  return SA_OK;
}

int sa_moment_fork_enabled(void) { return g_fork_enabled ? 1 : 0; }

int sa_device_checks_enabled(void) {
#ifdef SA_DEVICE_CHECKS
  return 1;
#else
  return 0;
#endif
}

int sa_set_wait_limit_ns(uint64_t limit_ns) {
  g_wait_limit_ns.store(limit_ns, std::memory_order_relaxed);
  return SA_OK;
}

int sa_set_stage_events(void* const* events, int count) {
  if (count < 0 || count > kMaxStageEvents)
    return set_error(SA_ERR_INVALID_ARG, "count must lie in [0, %d]", kMaxStageEvents);
  if (count > 0 && !events) return set_error(SA_ERR_INVALID_ARG, "null event array");
  for (int i = 0; i < kMaxStageEvents; ++i)
    g_stage_events[i] = i < count ? static_cast<cudaEvent_t>(events[i]) : nullptr;
  g_stage_count = count;
  return SA_OK;
}

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
                         rep_w, SplitOut{}, (cudaStream_t)stream);
}

int sa_low_moments_workspace_size(int64_t bh, int64_t n, int d, int dv, int degree, int block_size, size_t* bytes) {
  if (!bytes) return set_error(SA_ERR_INVALID_ARG, "null output pointer");
  int rc = check_common(nullptr, nullptr, nullptr, 0, n, d, dv, degree, block_size);
  if (rc) return rc;
  if (bh < 0) return set_error(SA_ERR_INVALID_ARG, "bh must be non-negative");
  const Workspace w = plan(bh, n, d, dv, degree, block_size, SA_COMPRESSOR_NONE, Plan::kMomentsOnly);
  *bytes = w.groups > 0 ? w.total : 0;
  return SA_OK;
}

int sa_low_moments(const float* q, const float* k, const float* v, int64_t bh, int64_t n, int d, int dv, int degree,
                   int block_size, float scale, float* low, void* workspace, size_t workspace_bytes, void* stream) {
  int rc = check_common(q, k, v, bh, n, d, dv, degree, block_size);
  if (rc) return rc;
  if (bh == 0 || n == 0) return SA_OK;
  if (!low) return set_error(SA_ERR_INVALID_ARG, "null output pointer");
  cudaStream_t s = (cudaStream_t)stream;
  const Workspace w = plan(bh, n, d, dv, degree, block_size, SA_COMPRESSOR_NONE, Plan::kMomentsOnly);
  if (w.groups == 0) return launch_low_moments(q, k, v, bh, n, d, dv, degree, block_size, scale, low, s);
  rc = check_workspace(w, workspace, workspace_bytes);
  if (rc) return rc;
  char* ws = static_cast<char*>(workspace);
  int* status = reinterpret_cast<int*>(ws + w.status);
  rc = reset_status(status, s);
  if (rc) return rc;
  float* vthi = reinterpret_cast<float*>(ws + w.vthi);
  float* vtlo = reinterpret_cast<float*>(ws + w.vtlo);
  float* part = reinterpret_cast<float*>(ws + w.low);
  rc = launch_split_t(v, bh, n, dv, w.dvp, w.n_pad, vthi, vtlo, s);
  if (rc) return rc;
  rc = moments_tc_from_split(w, ws, vthi, vtlo, q, k, part, status, bh, n, d, dv, degree, block_size, scale, s);
  if (rc) return rc;
  return launch_sum_groups(part, w.groups, bh * n * (dv + 1), low, s);
}

int sa_residual_combine_workspace_size(int64_t bh, int64_t n, int d, int dv, int block_size, int compressor,
                                       size_t* bytes) {
  if (!bytes) return set_error(SA_ERR_INVALID_ARG, "null output pointer");
  int rc = check_common(nullptr, nullptr, nullptr, 0, n, d, dv, 0, block_size);
  if (rc) return rc;
  if (bh < 0) return set_error(SA_ERR_INVALID_ARG, "bh must be non-negative");
  rc = check_compressor(compressor);
  if (rc) return rc;
  const Workspace w = plan(bh, n, d, dv, 0, block_size, compressor, Plan::kResidualOnly);
  *bytes = w.tc ? w.total : 0;
  return SA_OK;
}

int sa_residual_combine(const float* q, const float* k, const float* v, const float* rep_k, const float* rep_v,
                        const float* rep_w, const float* low, int64_t bh, int64_t n, int d, int dv, int degree,
                        int block_size, int compressor, float scale, float eps, float* out, void* workspace,
                        size_t workspace_bytes, void* stream) {
  int rc = check_common(q, k, v, bh, n, d, dv, degree, block_size);
  if (rc) return rc;
  rc = check_compressor(compressor);
  if (rc) return rc;
  if (bh == 0 || n == 0) return SA_OK;
  if (!low || !out) return set_error(SA_ERR_INVALID_ARG, "null low or out pointer");
  const int64_t nc = (n - 1) / block_size;
  const bool have_reps = compressor != SA_COMPRESSOR_NONE && nc > 0;
  if (have_reps && (!rep_k || !rep_v || !rep_w)) return set_error(SA_ERR_INVALID_ARG, "null rep pointer");
  cudaStream_t s = (cudaStream_t)stream;
  const Workspace w = plan(bh, n, d, dv, degree, block_size, compressor, Plan::kResidualOnly);
  if (!w.tc)
    return launch_residual(q, k, v, rep_k, rep_v, rep_w, low, bh, n, d, dv, degree, block_size, compressor, scale,
                           eps, out, s);
  rc = check_workspace(w, workspace, workspace_bytes);
  if (rc) return rc;
  char* ws = static_cast<char*>(workspace);
  int* status = reinterpret_cast<int*>(ws + w.status);
  rc = reset_status(status, s);
  if (rc) return rc;
  float* cur[4] = {reinterpret_cast<float*>(ws + w.khi), reinterpret_cast<float*>(ws + w.klo),
                   reinterpret_cast<float*>(ws + w.vthi), reinterpret_cast<float*>(ws + w.vtlo)};
  rc = launch_split(k, bh * n, d, w.dp, cur[0], cur[1], s);
  if (rc) return rc;
  rc = launch_split_t(v, bh, n, dv, w.dvp, w.n_pad, cur[2], cur[3], s);
  if (rc) return rc;
  const TCOperands cur_ops{cur[0], cur[1], n, cur[2], cur[3], n, w.n_pad};
  TCOperands rep_ops = cur_ops;
  float* wpad = nullptr;
  if (have_reps) {
    float* r[4] = {reinterpret_cast<float*>(ws + w.rkhi), reinterpret_cast<float*>(ws + w.rklo),
                   reinterpret_cast<float*>(ws + w.rvthi), reinterpret_cast<float*>(ws + w.rvtlo)};
    rc = launch_split(rep_k, bh * w.R, d, w.dp, r[0], r[1], s);
    if (rc) return rc;
    rc = launch_split_t(rep_v, bh, w.R, dv, w.dvp, w.r_pad, r[2], r[3], s);
    if (rc) return rc;
    wpad = reinterpret_cast<float*>(ws + w.rep_w);
    cudaError_t ce = cudaMemsetAsync(wpad, 0, (size_t)bh * w.r_pad * sizeof(float), s);
    if (ce == cudaSuccess)
      ce = cudaMemcpy2DAsync(wpad, (size_t)w.r_pad * sizeof(float), rep_w, (size_t)w.R * sizeof(float),
                             (size_t)w.R * sizeof(float), (size_t)bh, cudaMemcpyDeviceToDevice, s);
    if (ce != cudaSuccess) return set_error(SA_ERR_CUDA, "rep weight copy: %s", cudaGetErrorString(ce));
    rep_ops = TCOperands{r[0], r[1], w.R, r[2], r[3], w.R, w.r_pad};
  }
  return residual_tc_from_split(w, rep_ops, cur_ops, wpad, q, low, 1, out, status, bh, n, d, dv, degree, block_size,
                                reps_per_block(compressor, block_size), scale, eps, s);
}

int sa_fast_attention_workspace_size(int64_t bh, int64_t n, int d, int dv, int degree, int block_size, int compressor,
                                     size_t* bytes) {
  if (!bytes) return set_error(SA_ERR_INVALID_ARG, "null output pointer");
  int rc = check_common(nullptr, nullptr, nullptr, 0, n, d, dv, degree, block_size);
  if (rc) return rc;
  if (bh < 0) return set_error(SA_ERR_INVALID_ARG, "bh must be non-negative");
  rc = check_compressor(compressor);
  if (rc) return rc;
  *bytes = plan(bh, n, d, dv, degree, block_size, compressor, Plan::kFull).total;
  return SA_OK;
}

int sa_fast_attention(const float* q, const float* k, const float* v, int64_t bh, int64_t n, int d, int dv, int degree,
                      int block_size, float scale, int compressor, const float* dirs, const float* coins,
                      const int32_t* perms, float eps, float* out, int32_t* rep_idx, void* workspace,
                      size_t workspace_bytes, void* stream) {
  return sa::fast_attention_run(q, k, v, bh, n, d, dv, degree, block_size, scale, compressor, dirs, coins, perms, eps,
                                out, rep_idx, workspace, workspace_bytes, stream, true);
}


/* ---- one shard of a sequence split along N (config 5 across GPUs) ---- */

int sa_shard_state_floats(int64_t bh, int d, int dv, int degree, int64_t* floats) {
  if (!floats) return set_error(SA_ERR_INVALID_ARG, "null output pointer");
  int rc = check_common(nullptr, nullptr, nullptr, 0, 1, d, dv, degree, 4);
  if (rc) return rc;
  if (moments_tc_groups(d, dv, degree) <= 0)
    return set_error(SA_ERR_UNSUPPORTED, "the sharded forward needs the tensor-core moment scan (dv <= 64)");
  *floats = moments_tc_master_floats(bh, d, dv, degree) + moments_tc_den_floats(bh, d, dv, degree);
  return SA_OK;
}

int sa_shard_workspace_size(int64_t bh, int64_t n, int d, int dv, int degree, int block_size, int64_t rep_rows,
                            size_t* bytes) {
  if (!bytes) return set_error(SA_ERR_INVALID_ARG, "null output pointer");
  int rc = check_common(nullptr, nullptr, nullptr, 0, n, d, dv, degree, block_size);
  if (rc) return rc;
  if (bh < 0 || rep_rows < 0) return set_error(SA_ERR_INVALID_ARG, "bh and rep_rows must be non-negative");
  const Workspace w = plan_shard(bh, n, d, dv, degree, block_size, rep_rows);
  if (!w.tc)
    return set_error(SA_ERR_UNSUPPORTED,
                     "the sharded forward needs the tensor-core kernels (d <= 64, dv <= 64, block_size % 4 == 0)");
  *bytes = w.total;
  return SA_OK;
}

int sa_shard_begin(const float* q, const float* k, const float* v, int64_t bh, int64_t n, int d, int dv, int degree,
                   int block_size, float scale, int compressor, const float* dirs, const float* coins,
                   const int32_t* perms, int64_t n_compress, int64_t c_off, float* state_out, float* rep_k,
                   float* rep_v, float* rep_w, int32_t* rep_idx, void* workspace, size_t workspace_bytes,
                   void* stream) {
  int rc = check_common(q, k, v, bh, n, d, dv, degree, block_size);
  if (!rc) rc = check_compressor(compressor);
  if (rc) return rc;
  if (bh == 0 || n == 0) return SA_OK;
  if (!state_out) return set_error(SA_ERR_INVALID_ARG, "null state pointer");
  if (n_compress < 0 || n_compress * (int64_t)block_size > n || c_off < 0)
    return set_error(SA_ERR_INVALID_ARG, "n_compress blocks must lie in the shard and c_off be non-negative");
  const bool compress = compressor != SA_COMPRESSOR_NONE && n_compress > 0;
  if (compress && (!rep_k || !rep_v || !rep_w)) return set_error(SA_ERR_INVALID_ARG, "null rep pointer");
  const Workspace w = plan_shard(bh, n, d, dv, degree, block_size, 0);
  if (!w.tc)
    return set_error(SA_ERR_UNSUPPORTED,
                     "the sharded forward needs the tensor-core kernels (d <= 64, dv <= 64, block_size % 4 == 0)");
  rc = check_workspace(w, workspace, workspace_bytes);
  if (rc) return rc;
  char* ws = static_cast<char*>(workspace);
  cudaStream_t s = (cudaStream_t)stream;
  int* status = reinterpret_cast<int*>(ws + w.status);
  rc = reset_status(status, s);
  float* khi = reinterpret_cast<float*>(ws + w.khi);
  float* klo = reinterpret_cast<float*>(ws + w.klo);
  float* vthi = reinterpret_cast<float*>(ws + w.vthi);
  float* vtlo = reinterpret_cast<float*>(ws + w.vtlo);
  if (!rc) rc = launch_split(k, bh * n, d, w.dp, khi, klo, s);
  if (!rc) rc = launch_split_t(v, bh, n, dv, w.dvp, w.n_pad, vthi, vtlo, s);
  if (!rc && compress)
    rc = launch_compress(k, v, bh, n, d, dv, block_size, compressor, dirs, coins, perms, rep_idx, rep_k, rep_v, rep_w,
                         SplitOut{}, s, n_compress, c_off * (int64_t)block_size, status);
  float* master = reinterpret_cast<float*>(ws + w.master);
  float* den_io = reinterpret_cast<float*>(ws + w.den_io);
  if (!rc)
    rc = moments_tc_from_split(w, ws, vthi, vtlo, q, k, reinterpret_cast<float*>(ws + w.low), status, bh, n, d, dv,
                               degree, block_size, scale, s, 1, den_io);
  if (rc) return rc;
  const int64_t nm = moments_tc_master_floats(bh, d, dv, degree), nd = moments_tc_den_floats(bh, d, dv, degree);
  cudaError_t ce = cudaMemcpyAsync(state_out, master, (size_t)nm * sizeof(float), cudaMemcpyDeviceToDevice, s);
  if (ce == cudaSuccess)
    ce = cudaMemcpyAsync(state_out + nm, den_io, (size_t)nd * sizeof(float), cudaMemcpyDeviceToDevice, s);
  if (ce != cudaSuccess) return set_error(SA_ERR_CUDA, "state copy: %s", cudaGetErrorString(ce));
  return SA_OK;
}

int sa_shard_end(const float* q, const float* k, const float* v, int64_t bh, int64_t n, int d, int dv, int degree,
                 int block_size, float scale, int compressor, float eps, const float* states_before, int n_before,
                 int64_t c_off, const float* rep_k, const float* rep_v, const float* rep_w, int64_t rep_rows,
                 float* out, void* workspace, size_t workspace_bytes, void* stream) {
  int rc = check_common(q, k, v, bh, n, d, dv, degree, block_size);
  if (!rc) rc = check_compressor(compressor);
  if (rc) return rc;
  if (bh == 0 || n == 0) return SA_OK;
  if (!out) return set_error(SA_ERR_INVALID_ARG, "null output pointer");
  if (n_before < 0 || (n_before > 0 && !states_before)) return set_error(SA_ERR_INVALID_ARG, "bad earlier states");
  if (rep_rows > 0 && (!rep_k || !rep_v || !rep_w)) return set_error(SA_ERR_INVALID_ARG, "null rep pointer");
  const Workspace w = plan_shard(bh, n, d, dv, degree, block_size, rep_rows);
  if (!w.tc)
    return set_error(SA_ERR_UNSUPPORTED,
                     "the sharded forward needs the tensor-core kernels (d <= 64, dv <= 64, block_size % 4 == 0)");
  rc = check_workspace(w, workspace, workspace_bytes);
  if (rc) return rc;
  char* ws = static_cast<char*>(workspace);
  cudaStream_t s = (cudaStream_t)stream;
  int* status = reinterpret_cast<int*>(ws + w.status);
  float* master = reinterpret_cast<float*>(ws + w.master);
  float* den_io = reinterpret_cast<float*>(ws + w.den_io);
  const int64_t nm = moments_tc_master_floats(bh, d, dv, degree), nd = moments_tc_den_floats(bh, d, dv, degree);
  // the state of every earlier shard, then its contribution to this shard's
  // queries (a second set of partial slices; none for the first shard)
  float* low = reinterpret_cast<float*>(ws + w.low);
  float* vthi = reinterpret_cast<float*>(ws + w.vthi);
  float* vtlo = reinterpret_cast<float*>(ws + w.vtlo);
  const int64_t slice = bh * n * (dv + 1);
  if (n_before > 0) {
    rc = launch_state_prefix(states_before, n_before, nm, nd, master, den_io, s);
    if (!rc)
      rc = moments_tc_from_split(w, ws, vthi, vtlo, q, k, low + (int64_t)w.groups * slice, status, bh, n, d, dv,
                                 degree, block_size, scale, s, 2, den_io);
    if (rc) return rc;
  }
  const int groups = n_before > 0 ? 2 * w.groups : w.groups;
  float* r[4] = {reinterpret_cast<float*>(ws + w.rkhi), reinterpret_cast<float*>(ws + w.rklo),
                 reinterpret_cast<float*>(ws + w.rvthi), reinterpret_cast<float*>(ws + w.rvtlo)};
  float* wpad = reinterpret_cast<float*>(ws + w.rep_w);
  if (rep_rows > 0) {
    rc = launch_split(rep_k, bh * rep_rows, d, w.dp, r[0], r[1], s);
    if (!rc) rc = launch_split_t(rep_v, bh, rep_rows, dv, w.dvp, w.r_pad, r[2], r[3], s);
    if (rc) return rc;
    cudaError_t ce = cudaMemsetAsync(wpad, 0, (size_t)bh * w.r_pad * sizeof(float), s);
    if (ce == cudaSuccess)
      ce = cudaMemcpy2DAsync(wpad, (size_t)w.r_pad * sizeof(float), rep_w, (size_t)rep_rows * sizeof(float),
                             (size_t)rep_rows * sizeof(float), (size_t)bh, cudaMemcpyDeviceToDevice, s);
    if (ce != cudaSuccess) return set_error(SA_ERR_CUDA, "rep weight copy: %s", cudaGetErrorString(ce));
  }
  const TCOperands cur_ops{reinterpret_cast<float*>(ws + w.khi), reinterpret_cast<float*>(ws + w.klo), n, vthi, vtlo,
                           n, w.n_pad};
  const TCOperands rep_ops{r[0], r[1], rep_rows, r[2], r[3], rep_rows, w.r_pad};
  return residual_tc_from_split(w, rep_ops, cur_ops, rep_rows > 0 ? wpad : nullptr, q, low, groups, out,
                                status, bh, n, d, dv, degree, block_size, reps_per_block(compressor, block_size),
                                scale, eps, s, c_off);
}


/* ---- the segment-mean variant (triton_article_attention.py:190-578) ---- */

int sa_segment_mean_reps(const float* k, const float* v, int64_t bh, int64_t n, int d, int dv, int block_size,
                         int compress_stride, int key_dtype, int value_dtype, float* rep_k, float* rep_v,
                         void* stream) {
  int rc = check_segment(k, k, v, bh, n, d, dv, 0, block_size, compress_stride, key_dtype, value_dtype, false);
  if (rc) return rc;
  const int64_t R = n > 0 ? (n - 1) / block_size * (block_size / compress_stride) : 0;
  if (bh == 0 || R == 0) return SA_OK;
  if (!rep_k || !rep_v) return set_error(SA_ERR_INVALID_ARG, "null rep pointer");
  return launch_segment_mean(k, v, bh, n, d, dv, block_size, compress_stride, key_dtype, value_dtype, rep_k, rep_v,
                             (cudaStream_t)stream);
}

int sa_article_segment_mean_workspace_size(int64_t bh, int64_t n, int d, int dv, int degree, int block_size,
                                           int compress_stride, size_t* bytes) {
  if (!bytes) return set_error(SA_ERR_INVALID_ARG, "null output pointer");
  int rc = check_segment(nullptr, nullptr, nullptr, 0, n, d, dv, degree, block_size, compress_stride, 0, 0);
  if (rc) return rc;
  if (bh < 0) return set_error(SA_ERR_INVALID_ARG, "bh must be non-negative");
  *bytes = plan(bh, n, d, dv, degree, block_size, SA_COMPRESSOR_NONE, Plan::kSegment, compress_stride).total;
  return SA_OK;
}

// Same pipeline as sa_fast_attention with the segment-mean kernel in place of
// the compressor: reps of weight compress_stride, bs/compress_stride per block
// (compress_stride 1: every earlier key, weight 1, read in place), and the
// exp argument capped at 80 in the residual.
int sa_article_segment_mean(const float* q, const float* k, const float* v, int64_t bh, int64_t n, int d, int dv,
                            int degree, int block_size, int compress_stride, float scale, int key_dtype,
                            int value_dtype, float eps, float* out, void* workspace, size_t workspace_bytes,
                            void* stream) {
  int rc = check_segment(q, k, v, bh, n, d, dv, degree, block_size, compress_stride, key_dtype, value_dtype);
  if (rc) return rc;
  if (bh == 0 || n == 0) return SA_OK;
  if (!out) return set_error(SA_ERR_INVALID_ARG, "null output pointer");
  const Workspace w = plan(bh, n, d, dv, degree, block_size, SA_COMPRESSOR_NONE, Plan::kSegment, compress_stride);
  rc = check_workspace(w, workspace, workspace_bytes);
  if (rc) return rc;
  char* ws = static_cast<char*>(workspace);
  float* low = reinterpret_cast<float*>(ws + w.low);
  int* status = reinterpret_cast<int*>(ws + w.status);
  cudaStream_t s = (cudaStream_t)stream;
  rc = reset_status(status, s);
  if (rc) return rc;
  const bool reps = w.R > 0;
  const int64_t m_blk = compress_stride > 1 ? block_size / compress_stride : block_size;

  float* khi = reinterpret_cast<float*>(ws + w.khi);
  float* klo = reinterpret_cast<float*>(ws + w.klo);
  float* vthi = reinterpret_cast<float*>(ws + w.vthi);
  float* vtlo = reinterpret_cast<float*>(ws + w.vtlo);
  if (w.tc) {
    rc = launch_split(k, bh * n, d, w.dp, khi, klo, s);
    if (rc) return rc;
  }
  if (w.tc || w.groups > 0) {
    rc = launch_split_t(v, bh, n, dv, w.dvp, w.n_pad, vthi, vtlo, s);
    if (rc) return rc;
  }

  // reps: the segment means of the completed blocks, weight compress_stride
  float* rep_k = reinterpret_cast<float*>(ws + w.rep_k);
  float* rep_v = reinterpret_cast<float*>(ws + w.rep_v);
  float* rw = reinterpret_cast<float*>(ws + w.rep_w);
  const TCOperands cur_ops{khi, klo, n, vthi, vtlo, n, w.n_pad};
  TCOperands rep_ops = cur_ops;
  if (reps) {
    rc = launch_segment_mean(k, v, bh, n, d, dv, block_size, compress_stride, key_dtype, value_dtype, rep_k, rep_v,
                             s);
    if (!rc) rc = launch_fill(rw, bh * (w.tc ? w.r_pad : w.R), (float)compress_stride, s);
    if (rc) return rc;
    if (w.tc) {
      float* r[4] = {reinterpret_cast<float*>(ws + w.rkhi), reinterpret_cast<float*>(ws + w.rklo),
                     reinterpret_cast<float*>(ws + w.rvthi), reinterpret_cast<float*>(ws + w.rvtlo)};
      rc = launch_split(rep_k, bh * w.R, d, w.dp, r[0], r[1], s);
      if (!rc) rc = launch_split_t(rep_v, bh, w.R, dv, w.dvp, w.r_pad, r[2], r[3], s);
      if (rc) return rc;
      rep_ops = TCOperands{r[0], r[1], w.R, r[2], r[3], w.R, w.r_pad};
    }
  }

  // low-degree moments
  if (w.groups > 0)
    rc = moments_tc_from_split(w, ws, vthi, vtlo, q, k, low, status, bh, n, d, dv, degree, block_size, scale, s);
  else
    rc = launch_low_moments(q, k, v, bh, n, d, dv, degree, block_size, scale, low, s);
  if (rc) return rc;
  const int groups = w.groups > 0 ? w.groups : 1;

  // residual + combine
  if (w.tc)
    return residual_tc_from_split(w, rep_ops, cur_ops, reps ? rw : nullptr, q, low, groups, out, status, bh, n, d,
                                  dv, degree, block_size, m_blk, scale, eps, s, 0, true);
  if (groups > 1) {
    rc = launch_sum_groups(low, groups, bh * n * (dv + 1), low, s);
    if (rc) return rc;
  }
  return launch_residual_reps(q, k, v, reps ? rep_k : k, reps ? rep_v : v, reps ? rw : nullptr, low, bh, n, d, dv,
                              degree, block_size, m_blk, reps ? w.R : n, scale, eps, true, out, s);
}

/* ---- exact causal attention (triton_article_attention.py:372-435, :580-637) ---- */

int sa_flash_causal_attention_workspace_size(int64_t bh, int64_t n, int d, int dv, size_t* bytes) {
  if (!bytes) return set_error(SA_ERR_INVALID_ARG, "null output pointer");
  const int rc = check_flash(nullptr, nullptr, nullptr, 0, n, d, dv);
  if (rc) return rc;
  if (bh < 0) return set_error(SA_ERR_INVALID_ARG, "bh must be non-negative");
  *bytes = plan_flash(bh, n, d, dv).total;
  return SA_OK;
}

int sa_flash_causal_attention(const float* q, const float* k, const float* v, int64_t bh, int64_t n, int d, int dv,
                              float scale, float* out, void* workspace, size_t workspace_bytes, void* stream) {
  int rc = check_flash(q, k, v, bh, n, d, dv);
  if (rc) return rc;
  if (bh == 0 || n == 0) return SA_OK;
  if (!out) return set_error(SA_ERR_INVALID_ARG, "null output pointer");
  cudaStream_t s = (cudaStream_t)stream;
  const Workspace w = plan_flash(bh, n, d, dv);
  if (!w.tc) return launch_flash_simt(q, k, v, bh, n, d, dv, scale, out, s);
  rc = check_workspace(w, workspace, workspace_bytes);
  if (rc) return rc;
  char* ws = static_cast<char*>(workspace);
  int* status = reinterpret_cast<int*>(ws + w.status);
  rc = reset_status(status, s);
  if (rc) return rc;
  float* khi = reinterpret_cast<float*>(ws + w.khi);
  float* klo = reinterpret_cast<float*>(ws + w.klo);
  float* vthi = reinterpret_cast<float*>(ws + w.vthi);
  float* vtlo = reinterpret_cast<float*>(ws + w.vtlo);
  rc = launch_split(k, bh * n, d, w.dp, khi, klo, s);
  if (!rc) rc = launch_split_t(v, bh, n, dv, w.dvp, w.n_pad, vthi, vtlo, s);
  if (rc) return rc;
  CUtensorMap maps[4];
  rc = encode_map_3d(&maps[0], khi, w.dp, n, bh, 64, CU_TENSOR_MAP_SWIZZLE_128B);
  if (!rc) rc = encode_map_3d(&maps[1], klo, w.dp, n, bh, 64, CU_TENSOR_MAP_SWIZZLE_128B);
  if (!rc) rc = encode_map(&maps[2], vthi, n, w.n_pad, w.dvp, bh, w.dvp, CU_TENSOR_MAP_SWIZZLE_128B);
  if (!rc) rc = encode_map(&maps[3], vtlo, n, w.n_pad, w.dvp, bh, w.dvp, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  return launch_flash_tc(maps, q, out, status, bh, n, d, dv, scale, s);
}

}  // extern "C"
