// Split-K f32 GEMM for callers that cannot allocate device memory.
//
// Who needs it: code that runs where cudaMalloc is unavailable or forbidden --
// host code inside another framework's memory manager that owns every device
// byte, or real-time paths that must not hit the allocator.  Such a
// caller still owns A, B and C; the only extra memory the split-K GEMM needs,
// the partial products of the K slices, lives in a fixed static device array of
// this library instead of a workspace the caller would have to allocate.
//
// The array (SB_GEMM_SPLITK_NOALLOC_MAX_FLOATS floats, 16 MiB) exists on every
// GPU that loads the library, for the life of the process.  All calls on a
// device share it: two calls whose kernels overlap on that GPU (different
// streams, or different host threads) race on it and corrupt each other's
// results; serialize them.  Each call overwrites every partial it reads, so
// nothing in the array has to start at zero.
#include <cuda_runtime.h>

#include <mutex>

#include "../../../include/sheaf_b200.h"
#include "kernels.h"

namespace sb {
namespace {

static __device__ __align__(256) float g_splitk_partials[SB_GEMM_SPLITK_NOALLOC_MAX_FLOATS];

constexpr int kMaxDevices = 64;
float* g_partials_ptr[kMaxDevices] = {};
std::mutex g_setup_mu;

// Device address of the static array on `dev` (current device).  In host code
// the symbol name is only a handle; the address comes from the runtime, once
// per device, and stays valid while the device's primary context lives (a
// host framework that resets the device must not call this entry point
// afterwards in the same process).
sb_status_code partials_on(int dev, float** out) {
  std::lock_guard<std::mutex> g(g_setup_mu);
  if (!g_partials_ptr[dev]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_splitk_partials);
    if (e != cudaSuccess || !p) {
      cudaGetLastError();
      return SB_STATUS_UNAVAILABLE;
    }
    g_partials_ptr[dev] = (float*)p;
  }
  *out = g_partials_ptr[dev];
  return SB_STATUS_OK;
}

}  // namespace
}  // namespace sb

extern "C" SB_API sb_status_code sb_gemm_f32_splitk_noalloc(const float* a, const float* b, float* c, int64_t m,
                                                            int64_t n, int64_t k, void* cuda_stream) {
  using namespace sb;
  if (m < 0 || n < 0 || k < 0) return SB_STATUS_INVALID_ARGUMENT;
  if (m == 0 || n == 0) return SB_STATUS_OK;
  if (!c || (k > 0 && (!a || !b))) return SB_STATUS_INVALID_ARGUMENT;
  // one CUDA-core launch covers at most kSimtMaxM rows (65535 row tiles)
  if (m > kSimtMaxM || n > (1ll << 31) || k > (1ll << 40)) return SB_STATUS_INVALID_ARGUMENT;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return SB_STATUS_UNAVAILABLE;
  }
  if (dev < 0 || dev >= kMaxDevices) return SB_STATUS_UNAVAILABLE;
  cudaStream_t stream = (cudaStream_t)cuda_stream;

  GemmArgs g{};
  g.a = a;
  g.b = b;
  g.c = c;
  g.batch = 1;
  g.M = m;
  g.N = n;
  g.K = k;
  g.sab = 0; g.sam = k; g.sak = 1;   // A row-major m x k
  g.sbb = 0; g.sbk = n; g.sbn = 1;   // B row-major k x n
  g.scb = m * n; g.scm = n; g.scn = 1;

  // the session's CUDA-core split-K rule, so both paths sum in the same order
  const SimtSplit sp = simt_split(m, n, k, 1);
  const int64_t splits = sp.splits, chunk = sp.k_chunk;
  cudaError_t e;
  if (splits > 1) {
    if (splits * m * n > (int64_t)SB_GEMM_SPLITK_NOALLOC_MAX_FLOATS) return SB_STATUS_RESOURCE_EXHAUSTED;
    float* partials = nullptr;
    sb_status_code st = partials_on(dev, &partials);
    if (st != SB_STATUS_OK) return st;
    GemmArgs p = g;
    p.c = partials;
    p.batch = splits;
    p.k_chunk = chunk;
    p.scb = m * n;
    e = gemm_simt(p, stream);
    if (e == cudaSuccess) e = splitk_reduce(partials, c, splits, m, n, n, 0, stream);
  } else {
    e = gemm_simt(g, stream);
  }
  // shapes are validated above, so a launch error here is the device's (it
  // stays visible to the caller's own error checks)
  return e == cudaSuccess ? SB_STATUS_OK : SB_STATUS_INTERNAL;
}
