// sa_fast_attention_static_scratch: the whole forward without any allocation.
//
// sa_fast_attention needs a caller-provided device workspace (the per-query
// low-degree sums and the packed coreset reps).  Some callers cannot hand one
// over: a host program whose device memory is owned end to end by another
// allocator (a framework that reserves almost all of HBM up front and accounts
// for every byte), a latency-critical serving loop that forbids cudaMalloc
// after start-up because it synchronises the device, or a plain-C / ctypes
// caller that has no device allocator of its own.  For them this entry point
// takes its scratch from one fixed array compiled into the library.
//
// The array is SA_STATIC_SCRATCH_BYTES (64 MiB) of device memory that every
// GPU which loads the library holds until the process exits.  Every call on a
// device shares it and it keeps whatever the previous call left there; no
// part of it needs to start at zero, because each kernel writes every element
// it later reads.  Two calls whose kernels overlap on the GPU (different
// streams, or different host threads, without ordering between them) race on
// the array and corrupt each other's results; callers must order them.
//
// Set-up: host code cannot use the array's name as a device pointer (it names
// a host-side stand-in), so the device address goes to the kernels instead,
// taken with cudaGetSymbolAddress with the caller's device current.  The first
// call on a device also loads the library's device code there; make it before
// any stream capture begins.  The address is taken again on every call (a
// host-side table lookup once the code is loaded) rather than cached: after a
// cudaDeviceReset, or when the device's context is destroyed and made again,
// the code is reloaded and the array can sit at a new address, and a cached
// one would then point at memory the library no longer owns.
#include "sa_common.cuh"

namespace {

static_assert(SA_STATIC_SCRATCH_BYTES % 256 == 0, "static scratch must be a multiple of 256 bytes");

static __device__ __align__(256) unsigned char g_static_scratch[SA_STATIC_SCRATCH_BYTES];

// The array's address in the current device's context.
int static_scratch_address(void** out) {
  void* p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_static_scratch);
  if (e != cudaSuccess || p == nullptr)
    return sa::set_error(SA_ERR_CUDA, "cudaGetSymbolAddress(static scratch): %s", cudaGetErrorString(e));
  *out = p;
  return SA_OK;
}

}  // namespace

extern "C" int sa_fast_attention_static_scratch(const float* q, const float* k, const float* v, int64_t bh,
                                                int64_t n, int d, int dv, int degree, int block_size, float scale,
                                                int compressor, const float* dirs, const float* coins,
                                                const int32_t* perms, float eps, float* out, int32_t* rep_idx,
                                                void* stream) {
  size_t need = 0;
  int rc = sa_fast_attention_workspace_size(bh, n, d, dv, degree, block_size, compressor, &need);
  if (rc) return rc;
  if (need > (size_t)SA_STATIC_SCRATCH_BYTES)
    return sa::set_error(SA_ERR_INVALID_ARG,
                         "this problem needs %zu bytes of scratch but the static scratch holds %zu; "
                         "use sa_fast_attention with a caller workspace",
                         need, (size_t)SA_STATIC_SCRATCH_BYTES);
  if (bh == 0 || n == 0)
    return sa::fast_attention_run(q, k, v, bh, n, d, dv, degree, block_size, scale, compressor, dirs, coins, perms,
                                  eps, out, rep_idx, nullptr, 0, stream, false);
  void* ws = nullptr;
  rc = static_scratch_address(&ws);
  if (rc) return rc;
  // in order on the caller's stream: no second stream is made on this path
  return sa::fast_attention_run(q, k, v, bh, n, d, dv, degree, block_size, scale, compressor, dirs, coins, perms, eps,
                                out, rep_idx, ws, (size_t)SA_STATIC_SCRATCH_BYTES, stream, false);
}
