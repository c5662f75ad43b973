// Stable sort of (f32 key, i32 payload) rows along the last dimension, the
// `stablehlo.sort` Sheaf emits for top_k (lowering/stablehlo/indexing_ops.rs:
// 476-540: keys with an iota payload, comparator GT, is_stable = true).
//
// Rank sort: every element counts the elements that precede it (key order,
// then original position), which is its output position; one thread per
// element, keys staged through shared memory in tiles.  Deterministic and
// stable by construction; O(n^2) per row, which at vocabulary sizes (65 ..
// 50304) is a few hundred microseconds at most.  Keys are compared through a
// monotone integer image of their bits (-0 folded onto +0, NaN above +inf), a
// total order, so the ranks are a permutation.  Output row: [sorted keys |
// payload bits], the packed layout of OpKind::SortPairs.
#include "kernels.h"
#include "pdl.h"

namespace sb {
namespace {

constexpr int kThreads = 256;
constexpr int kTile = 4096;

__device__ __forceinline__ int order_key(float x) {
  int u = x == 0.f ? 0 : __float_as_int(x);
  return u ^ ((u >> 31) & 0x7fffffff);
}

__global__ void __launch_bounds__(kThreads) sort_rank_kernel(const float* __restrict__ keys,
                                                             const int* __restrict__ payload,
                                                             float* __restrict__ out, int n, int desc) {
  pdl_prologue();
  __shared__ int tile[kTile];
  const size_t row = blockIdx.y;
  const float* k = keys + row * n;
  const int i = blockIdx.x * kThreads + threadIdx.x;
  const int ki = i < n ? order_key(k[i]) : 0;
  int rank = 0;
  for (int t0 = 0; t0 < n; t0 += kTile) {
    const int cnt = min(kTile, n - t0);
    __syncthreads();
    for (int j = threadIdx.x; j < cnt; j += kThreads) tile[j] = order_key(k[t0 + j]);
    __syncthreads();
    if (i < n) {
      if (desc) {
        for (int j = 0; j < cnt; ++j) {
          const int kj = tile[j];
          rank += (kj > ki) | ((kj == ki) & (t0 + j < i));
        }
      } else {
        for (int j = 0; j < cnt; ++j) {
          const int kj = tile[j];
          rank += (kj < ki) | ((kj == ki) & (t0 + j < i));
        }
      }
    }
  }
  if (i < n) {
    float* o = out + row * 2 * (size_t)n;
    o[rank] = k[i];
    o[n + rank] = __int_as_float(payload[row * n + i]);
  }
}

}  // namespace

cudaError_t sort_pairs(const float* keys, const int* payload, float* out, int64_t rows, int64_t n, bool descending,
                       cudaStream_t stream) {
  if (rows <= 0 || n <= 0) return cudaSuccess;
  if (n > (1ll << 30) || rows > 65535) return cudaErrorNotSupported;
  const dim3 grid((unsigned)((n + kThreads - 1) / kThreads), (unsigned)rows);
  return launch_pdl(sort_rank_kernel, grid, dim3(kThreads), 0, stream, keys, payload, out, (int)n,
                    descending ? 1 : 0);
}

}  // namespace sb
