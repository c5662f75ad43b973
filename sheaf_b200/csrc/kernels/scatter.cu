// Row scatter-add: out[v, :] = sum of adj[r, :] over the rows r whose index
// key(r) equals v, r in increasing order; rows of out that no key hits are 0.
//
// This is the gradient of an embedding lookup (table[idx]).  Sheaf's reverse-
// mode rule writes it as transpose(one_hot(idx, V)) @ adj
// (sheaf/src/autodiff/reverse.rs:1015-1041); the planner replaces that product
// by this op (csrc/embed_grad.cpp).  Keys are the index values: f32 (Sheaf
// passes token ids as f32) or i32; a key that is not an integer in [0, V) hits
// no row, as its one-hot row is all zeros.
//
// Deterministic, no floating-point atomics: the rows are put in (key, row)
// order by a stable counting sort, and each output row is summed by one warp
// in that order.
//   1. per chunk of kChunk rows, a key histogram (integer atomics: the counts
//      do not depend on the order of the increments);
//   2. per key, the exclusive prefix of the chunk counts (where the chunk's
//      rows of that key start among all rows of that key) and the total;
//   3. the exclusive prefix of the totals over the keys (segment starts);
//   4. per row, its position in the sorted order: segment start + chunk
//      prefix + the number of earlier rows of the same key inside the chunk;
//   5. per key, one warp sums its segment's adj rows (float4 columns).
#include <algorithm>

#include "kernels.h"
#include "pdl.h"
#include "tc_common.h"

namespace sb {
namespace {

// rows per chunk = threads per block: one row per thread, whose rank among the
// chunk's earlier rows of the same key is counted over at most 255 keys in
// shared memory (1024-row chunks took ~25 us in that count)
constexpr int kChunk = 256;
constexpr int kThreads = 256;

// Index of row r, or v when it hits no row.
__device__ __forceinline__ int key_of(const void* idx, int idx_f32, int64_t r, int v) {
  if (idx_f32) {
    const float x = ((const float*)idx)[r];
    // integers in [0, v) only (NaN fails both comparisons)
    if (!(x >= 0.f && x < (float)v) || x != floorf(x)) return v;
    return (int)x;
  }
  const int k = ((const int*)idx)[r];
  return (k >= 0 && k < v) ? k : v;
}

__global__ void __launch_bounds__(kThreads) hist_kernel(const void* idx, int idx_f32, int64_t n, int v,
                                                        int* __restrict__ hist) {
  pdl_prologue();
  const int64_t c = blockIdx.x;
  const int64_t r0 = c * kChunk, r1 = min(n, r0 + kChunk);
  for (int64_t r = r0 + threadIdx.x; r < r1; r += kThreads) {
    const int k = key_of(idx, idx_f32, r, v);
    if (k < v) atomicAdd(&hist[c * v + k], 1);
  }
}

// hist[c][k] := rows of key k in chunks before c; total[k] := all rows of key k.
// One warp per key: 32 chunks at a time, an exclusive scan across the lanes
// (integer sums: the same result as a serial scan), a carry between groups.
__global__ void __launch_bounds__(kThreads) colscan_kernel(int* __restrict__ hist, int* __restrict__ total,
                                                           int chunks, int v) {
  pdl_prologue();
  const int lane = threadIdx.x & 31;
  constexpr int kWarps = kThreads / 32;
  for (int64_t k = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5); k < v; k += (int64_t)gridDim.x * kWarps) {
    int run = 0;
    for (int c0 = 0; c0 < chunks; c0 += 32) {
      const int c = c0 + lane;
      const int t = c < chunks ? hist[(int64_t)c * v + k] : 0;
      int incl = t;
#pragma unroll
      for (int s = 1; s < 32; s <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, s);
        if (lane >= s) incl += y;
      }
      if (c < chunks) hist[(int64_t)c * v + k] = run + incl - t;
      run += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) total[k] = run;
  }
}

// offs[k] := exclusive prefix over keys of total (rounded up to a multiple of
// `round`: segments padded to whole chunks), offs[v] = the sum
__device__ __forceinline__ int rounded(int x, int round) { return (x + round - 1) / round * round; }

__global__ void __launch_bounds__(1024) offsets_kernel(const int* __restrict__ total, int* __restrict__ offs, int v,
                                                       int round) {
  pdl_prologue();
  __shared__ int part[1024];
  const int per = (v + 1023) / 1024;
  const int k0 = threadIdx.x * per, k1 = min(v, k0 + per);
  int s = 0;
  for (int k = k0; k < k1; ++k) s += rounded(total[k], round);
  part[threadIdx.x] = s;
  __syncthreads();
  // inclusive scan of the 1024 partial sums (Hillis-Steele)
  for (int d = 1; d < 1024; d <<= 1) {
    const int x = threadIdx.x >= d ? part[threadIdx.x - d] : 0;
    __syncthreads();
    part[threadIdx.x] += x;
    __syncthreads();
  }
  int run = threadIdx.x ? part[threadIdx.x - 1] : 0;
  for (int k = k0; k < k1; ++k) {
    offs[k] = run;
    run += rounded(total[k], round);
  }
  if (threadIdx.x == 1023) offs[v] = part[1023];
}

__global__ void __launch_bounds__(kThreads) place_kernel(const void* idx, int idx_f32, int64_t n, int v,
                                                         const int* __restrict__ hist, const int* __restrict__ offs,
                                                         int* __restrict__ perm) {
  pdl_prologue();
  __shared__ int keys[kChunk];
  const int64_t c = blockIdx.x;
  const int64_t r0 = c * kChunk;
  const int m = (int)(n - r0 < kChunk ? n - r0 : kChunk);
  for (int i = threadIdx.x; i < m; i += kThreads) keys[i] = key_of(idx, idx_f32, r0 + i, v);
  __syncthreads();
  for (int i = threadIdx.x; i < m; i += kThreads) {
    const int k = keys[i];
    if (k >= v) continue;
    int lr = 0;
    for (int j = 0; j < i; ++j) lr += keys[j] == k;
    perm[offs[k] + hist[c * v + k] + lr] = (int)(r0 + i);
  }
}

// one warp per output row k: out[k, :] = sum over its segment, in order
__global__ void __launch_bounds__(kThreads) segsum_kernel(const float* __restrict__ adj, const int* __restrict__ offs,
                                                          const int* __restrict__ perm, float* __restrict__ out,
                                                          int v, int64_t d, int vec, int64_t n, int* err) {
  pdl_prologue();
  const int lane = threadIdx.x & 31;
  const int warps = kThreads / 32;
  for (int64_t k = (int64_t)blockIdx.x * warps + (threadIdx.x >> 5); k < v; k += (int64_t)gridDim.x * warps) {
    int s0 = offs[k], s1 = offs[k + 1];
    if (s0 < 0 || s1 < s0 || s1 > n) {  // inconsistent segment: recorded, and skipped
      if (lane == 0) atomicExch(err, 41);
      s0 = s1 = 0;
    }
    float* o = out + k * d;
    if (vec) {
      for (int64_t col = lane * 4; col < d; col += 128) {
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int s = s0; s < s1; ++s) {
          const float4 x = *(const float4*)(adj + (int64_t)perm[s] * d + col);
          acc.x += x.x; acc.y += x.y; acc.z += x.z; acc.w += x.w;
        }
        *(float4*)(o + col) = acc;
      }
    } else {
      for (int64_t col = lane; col < d; col += 32) {
        float acc = 0.f;
        for (int s = s0; s < s1; ++s) acc += adj[(int64_t)perm[s] * d + col];
        o[col] = acc;
      }
    }
  }
}

// Few keys, many rows each (a small vocabulary): one warp per key would sum
// hundreds of rows in sequence.  Instead every key's segment is padded to
// whole chunks of kRun positions (padding rows are -1), pass 1 sums each chunk
// (one warp per 128 columns of a chunk), pass 2 sums each key's chunk
// partials in chunk order.
constexpr int kRun = 32;

__global__ void __launch_bounds__(kThreads) chunk_sum_kernel(const float* __restrict__ adj, const int* __restrict__ offs,
                                                             const int* __restrict__ perm, float* __restrict__ part,
                                                             int v, int64_t d, int64_t max_chunks, int64_t n, int* err) {
  pdl_prologue();
  const int lane = threadIdx.x & 31;
  int64_t chunks = offs[v] / kRun;
  if (chunks < 0 || chunks > max_chunks) {  // inconsistent offsets: recorded, nothing summed
    if (threadIdx.x == 0) atomicExch(err, 42);
    chunks = 0;
  }
  const int64_t cols = (d + 127) / 128;
  for (int64_t w = (int64_t)blockIdx.x * (kThreads / 32) + (threadIdx.x >> 5); w < chunks * cols;
       w += (int64_t)gridDim.x * (kThreads / 32)) {
    const int64_t c = w / cols, col = (w % cols) * 128 + lane * 4;
    if (col >= d) continue;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 8
    for (int i = 0; i < kRun; ++i) {
      const int r = perm[c * kRun + i];
      if (r < 0 || r >= n) continue;
      const float4 x = *(const float4*)(adj + (int64_t)r * d + col);
      acc.x += x.x; acc.y += x.y; acc.z += x.z; acc.w += x.w;
    }
    *(float4*)(part + c * d + col) = acc;
  }
}

__global__ void __launch_bounds__(kThreads) key_sum_kernel(const float* __restrict__ part, const int* __restrict__ offs,
                                                           float* __restrict__ out, int v, int64_t d, int64_t max_chunks,
                                                           int* err) {
  pdl_prologue();
  const int lane = threadIdx.x & 31;
  const int64_t cols = (d + 127) / 128;
  for (int64_t w = (int64_t)blockIdx.x * (kThreads / 32) + (threadIdx.x >> 5); w < (int64_t)v * cols;
       w += (int64_t)gridDim.x * (kThreads / 32)) {
    const int64_t k = w / cols, col = (w % cols) * 128 + lane * 4;
    if (col >= d) continue;
    int c0 = offs[k] / kRun, c1 = offs[k + 1] / kRun;
    if (c0 < 0 || c1 < c0 || c1 > max_chunks) {
      if (lane == 0) atomicExch(err, 43);
      c0 = c1 = 0;
    }
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int c = c0; c < c1; ++c) {
      const float4 x = *(const float4*)(part + (int64_t)c * d + col);
      acc.x += x.x; acc.y += x.y; acc.z += x.z; acc.w += x.w;
    }
    *(float4*)(out + k * d + col) = acc;
  }
}

int64_t chunks_of(int64_t n) { return (n + kChunk - 1) / kChunk; }

// the chunked two-pass sum: few keys for the rows, float4 columns
bool chunked(int64_t n, int64_t v, int64_t d) { return v * 8 <= n && d % 4 == 0; }

}  // namespace

size_t scatter_add_rows_workspace(int64_t n, int64_t v, int64_t d) {
  // hist [chunks][v], total [v], offs [v + 1], perm [n] (ints); chunked:
  // perm padded to n + v * kRun, then the chunk partials (floats, 16-byte
  // aligned)
  if (!chunked(n, v, d)) return (size_t)(chunks_of(n) * v + v + (v + 1) + n) * sizeof(int);
  const int64_t ints = chunks_of(n) * v + v + (v + 1) + n + v * kRun;
  const int64_t max_chunks = n / kRun + v;
  return (size_t)((ints + 3) / 4 * 4) * sizeof(int) + (size_t)(max_chunks * d) * sizeof(float);
}

cudaError_t scatter_add_rows(const void* idx, bool idx_f32, const float* adj, float* out, int64_t n, int64_t d,
                             int64_t v, void* ws, cudaStream_t stream) {
  if (v <= 0 || d <= 0) return cudaSuccess;
  if (n < 0 || v >= (1ll << 31) - 1 || n >= (1ll << 31)) return cudaErrorInvalidValue;
  int* err = tc_error_word();  // the device error word of the tensor-core kernels
  if (!err) return cudaErrorNotSupported;
  const int64_t chunks = chunks_of(n);
  const bool two_pass = chunked(n, v, d) && (((uintptr_t)adj | (uintptr_t)out) & 15) == 0;
  int* hist = (int*)ws;
  int* total = hist + chunks * v;
  int* offs = total + v;
  int* perm = offs + v + 1;
  const int64_t perm_len = two_pass ? n + v * kRun : n;
  const int64_t ints = chunks * v + v + (v + 1) + perm_len;
  float* part = (float*)((int*)ws + (ints + 3) / 4 * 4);
  cudaError_t e;
  if (n > 0) {
    e = cudaMemsetAsync(hist, 0, (size_t)(chunks * v) * sizeof(int), stream);
    if (e != cudaSuccess) return e;
    e = launch_pdl(hist_kernel, dim3((unsigned)chunks), dim3(kThreads), 0, stream, idx, (int)idx_f32, n, (int)v, hist);
    if (e != cudaSuccess) return e;
  }
  const unsigned vb = (unsigned)std::min<int64_t>((v + kThreads / 32 - 1) / (kThreads / 32), 148 * 8);
  e = launch_pdl(colscan_kernel, dim3(vb), dim3(kThreads), 0, stream, hist, total, (int)chunks, (int)v);
  if (e != cudaSuccess) return e;
  e = launch_pdl(offsets_kernel, dim3(1), dim3(1024), 0, stream, (const int*)total, offs, (int)v,
                 two_pass ? kRun : 1);
  if (e != cudaSuccess) return e;
  if (two_pass) {  // padding positions of the segments hold -1
    e = cudaMemsetAsync(perm, 0xff, (size_t)perm_len * sizeof(int), stream);
    if (e != cudaSuccess) return e;
  }
  if (n > 0) {
    e = launch_pdl(place_kernel, dim3((unsigned)chunks), dim3(kThreads), 0, stream, idx, (int)idx_f32, n, (int)v,
                   (const int*)hist, (const int*)offs, perm);
    if (e != cudaSuccess) return e;
  }
  if (two_pass) {
    const int64_t max_chunks = n / kRun + v, cols = (d + 127) / 128;
    const unsigned b1 = (unsigned)std::min<int64_t>((max_chunks * cols + 7) / 8, 148 * 16);
    e = launch_pdl(chunk_sum_kernel, dim3(b1), dim3(kThreads), 0, stream, adj, (const int*)offs, (const int*)perm,
                   part, (int)v, d, max_chunks, n, err);
    if (e != cudaSuccess) return e;
    const unsigned b2 = (unsigned)std::min<int64_t>((v * cols + 7) / 8, 148 * 16);
    return launch_pdl(key_sum_kernel, dim3(b2), dim3(kThreads), 0, stream, (const float*)part, (const int*)offs, out,
                      (int)v, d, max_chunks, err);
  }
  const int vec = (d % 4 == 0) && ((((uintptr_t)adj) | ((uintptr_t)out)) & 15) == 0;
  const unsigned sb = (unsigned)std::min<int64_t>((v + kThreads / 32 - 1) / (kThreads / 32), 148 * 16);
  return launch_pdl(segsum_kernel, dim3(sb), dim3(kThreads), 0, stream, adj, (const int*)offs, (const int*)perm, out,
                    (int)v, d, vec, n, err);
}

}  // namespace sb
