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
// Set-up: the first call on each device (with that device current) looks up
// the array's device address with cudaGetSymbolAddress and caches it.  Host
// code cannot use the array's name as a device pointer (it names a host-side
// stand-in), which is why the looked-up address is what goes to the kernels.
// Make that first call before any stream capture begins.
#include <mutex>

#include "sa_common.cuh"

namespace {

static_assert(SA_STATIC_SCRATCH_BYTES % 256 == 0, "static scratch must be a multiple of 256 bytes");

static __device__ __align__(256) unsigned char g_static_scratch[SA_STATIC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
void* g_scratch_addr[kMaxDevices] = {};

int static_scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return sa::set_error(SA_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return sa::set_error(SA_ERR_UNSUPPORTED, "device index %d too large", dev);
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_addr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_static_scratch);
    if (e != cudaSuccess || p == nullptr)
      return sa::set_error(SA_ERR_CUDA, "cudaGetSymbolAddress(static scratch): %s", cudaGetErrorString(e));
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
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
    return sa_fast_attention(q, k, v, bh, n, d, dv, degree, block_size, scale, compressor, dirs, coins, perms, eps,
                             out, rep_idx, nullptr, 0, stream);
  void* ws = nullptr;
  rc = static_scratch_address(&ws);
  if (rc) return rc;
  return sa_fast_attention(q, k, v, bh, n, d, dv, degree, block_size, scale, compressor, dirs, coins, perms, eps, out,
                           rep_idx, ws, (size_t)SA_STATIC_SCRATCH_BYTES, stream);
}
