// Fused optimizer step over all parameter leaves (multi-tensor apply):
// clip-by-global-norm followed by AdamW, in place on device buffers.  Replaces
// the per-leaf interpreter/JIT work of Sheaf's training loop
// (examples/nanoGPT/train.shf:26-33 calling lib/optim.shf:36-58 adamw-step and
// :72-83 global-norm / clip-by-global-norm).
//
// The element space of all leaves is cut into fixed chunks (OptChunk, built on
// the host).  Pass 1: one block per chunk sums g^2 with a fixed tree.  Pass 2:
// every block reduces the chunk partials in the same fixed order (so every
// block sees the identical norm and the result is deterministic), derives the
// clip factor, and updates its chunk: g' = g * clip; m = b1 m + (1 - b1) g';
// v = b2 v + (1 - b2) g'^2; p = p - lr (wd p + (m bc_m) / (sqrt(v bc_v) + eps)),
// in f32 in the reference's operation order.
#include "kernels.h"
#include "pdl.h"

namespace sb {
namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ float block_sum(float x, float* red) {
  for (int s = 16; s > 0; s >>= 1) x += __shfl_xor_sync(0xffffffffu, x, s);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) red[warp] = x;
  __syncthreads();
  if (warp == 0) {
    x = lane < kThreads / 32 ? red[lane] : 0.f;
    for (int s = 16; s > 0; s >>= 1) x += __shfl_xor_sync(0xffffffffu, x, s);
    if (lane == 0) red[0] = x;
  }
  __syncthreads();
  const float r = red[0];
  __syncthreads();
  return r;
}

__global__ void __launch_bounds__(kThreads) sumsq_kernel(const OptLeaf* __restrict__ leaves,
                                                         const OptChunk* __restrict__ chunks,
                                                         float* __restrict__ partials) {
  pdl_prologue();
  __shared__ float red[kThreads / 32];
  const OptChunk c = chunks[blockIdx.x];
  const float* g = leaves[c.leaf].g + c.off;
  float acc = 0.f;
  for (int64_t i = threadIdx.x; i < c.len; i += kThreads) acc += g[i] * g[i];
  const float s = block_sum(acc, red);
  if (threadIdx.x == 0) partials[blockIdx.x] = s;
}

__global__ void __launch_bounds__(kThreads) adamw_kernel(const OptLeaf* __restrict__ leaves,
                                                         const OptChunk* __restrict__ chunks, int n_chunks,
                                                         const float* __restrict__ partials,
                                                         float* __restrict__ norm_out, AdamwScalars a) {
  pdl_prologue();
  __shared__ float red[kThreads / 32];
  float clip = 1.f;
  if (a.clip || norm_out) {
    float acc = 0.f;
    for (int i = threadIdx.x; i < n_chunks; i += kThreads) acc += partials[i];
    const float norm = sqrtf(block_sum(acc, red));
    if (norm_out && blockIdx.x == 0 && threadIdx.x == 0) *norm_out = norm;
    if (a.clip) clip = fminf(1.f, a.max_norm / (norm + 1e-8f));
  }
  const OptChunk c = chunks[blockIdx.x];
  const OptLeaf L = leaves[c.leaf];
  for (int64_t i = c.off + threadIdx.x; i < c.off + c.len; i += kThreads) {
    const float g = a.clip ? L.g[i] * clip : L.g[i];
    const float m = a.b1 * L.m[i] + a.one_minus_b1 * g;
    const float v = a.b2 * L.v[i] + a.one_minus_b2 * (g * g);
    const float p = L.p[i];
    L.m[i] = m;
    L.v[i] = v;
    L.p[i] = p - a.lr * (a.wd * p + (m * a.bc_m) / (sqrtf(v * a.bc_v) + a.eps));
  }
}

}  // namespace

cudaError_t adamw_step(const OptLeaf* leaves, const OptChunk* chunks, int n_chunks, float* partials,
                       float* norm_out, const AdamwScalars& a, cudaStream_t stream) {
  if (n_chunks <= 0) return cudaSuccess;
  if (a.clip || norm_out) {
    cudaError_t e = launch_pdl(sumsq_kernel, dim3(n_chunks), dim3(kThreads), 0, stream, leaves, chunks, partials);
    if (e != cudaSuccess) return e;
  }
  return launch_pdl(adamw_kernel, dim3(n_chunks), dim3(kThreads), 0, stream, leaves, chunks, n_chunks, partials,
                    norm_out, a);
}

}  // namespace sb
