// Small hand-written helper kernels.
#include <cuda_bf16.h>

#include "kernels.h"
#include "pdl.h"
#include "tc_common.h"

namespace sb {
namespace {

__device__ __forceinline__ float rna_tf32(float x) {
  uint32_t u;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(u) : "f"(x));
  return __uint_as_float(u);
}

// Streaming copy with rounding: n4 float4 groups (when both pointers are
// 16-byte aligned), then a scalar tail.
__global__ void __launch_bounds__(256) round_tf32_kernel(const float* __restrict__ src, float* __restrict__ dst,
                                                         int64_t n, int64_t n4) {
  pdl_prologue();
  const float4* s4 = reinterpret_cast<const float4*>(src);
  float4* d4 = reinterpret_cast<float4*>(dst);
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
    float4 v = s4[i];
    d4[i] = make_float4(rna_tf32(v.x), rna_tf32(v.y), rna_tf32(v.z), rna_tf32(v.w));
  }
  for (int64_t i = n4 * 4 + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    dst[i] = rna_tf32(src[i]);
}

// f32 -> bf16, round to nearest even: 8 elements per thread step (two float4
// loads, one 16-byte store) when both pointers are 16-byte aligned, then a
// scalar tail.
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

__global__ void __launch_bounds__(256) bf16_kernel(const float* __restrict__ src, uint16_t* __restrict__ dst,
                                                   int64_t n, int64_t n8) {
  pdl_prologue();
  const float4* s4 = reinterpret_cast<const float4*>(src);
  uint4* d8 = reinterpret_cast<uint4*>(dst);
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n8; i += (int64_t)gridDim.x * blockDim.x) {
    const float4 a = s4[2 * i], b = s4[2 * i + 1];
    d8[i] = make_uint4(pack_bf16(a.x, a.y), pack_bf16(a.z, a.w), pack_bf16(b.x, b.y), pack_bf16(b.z, b.w));
  }
  for (int64_t i = n8 * 8 + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    __nv_bfloat16 h = __float2bfloat16_rn(src[i]);
    dst[i] = *reinterpret_cast<uint16_t*>(&h);
  }
}

}  // namespace

cudaError_t bf16_copy(const float* src, uint16_t* dst, int64_t n, cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  const bool aligned = ((((uintptr_t)src) | ((uintptr_t)dst)) & 15) == 0;
  const int64_t n8 = aligned ? n / 8 : 0;
  int64_t blocks = ((aligned ? n8 : n) + 255) / 256;
  if (blocks < 1) blocks = 1;
  if (blocks > 148 * 8) blocks = 148 * 8;
  return launch_pdl(bf16_kernel, dim3((unsigned)blocks), dim3(256), 0, stream, src, dst, n, n8);
}

// Every block walks the segments in order with a grid-stride loop over each:
// 4-wide where both pointers of a segment are 16-byte aligned, then the tail.
__global__ void __launch_bounds__(256) round_tf32_segments_kernel(const RoundSegments s) {
  pdl_prologue();
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  for (int k = 0; k < s.count; ++k) {
    const float* src = s.src[k];
    float* dst = s.dst[k];
    const int64_t n = s.n[k];
    const int64_t n4 = ((((uintptr_t)src) | ((uintptr_t)dst)) & 15) == 0 ? n / 4 : 0;
    for (int64_t i = t; i < n4; i += stride) {
      const float4 v = reinterpret_cast<const float4*>(src)[i];
      reinterpret_cast<float4*>(dst)[i] = make_float4(rna_tf32(v.x), rna_tf32(v.y), rna_tf32(v.z), rna_tf32(v.w));
    }
    for (int64_t i = n4 * 4 + t; i < n; i += stride) dst[i] = rna_tf32(src[i]);
  }
}

// bf16 copies: 8 elements per step where both pointers of a segment are
// 16-byte aligned, then the tail, round to nearest even as bf16_kernel.
__global__ void __launch_bounds__(256) bf16_segments_kernel(const Bf16Segments s) {
  pdl_prologue();
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  for (int k = 0; k < s.count; ++k) {
    const float* src = s.src[k];
    uint16_t* dst = s.dst[k];
    const int64_t n = s.n[k];
    const int64_t n8 = ((((uintptr_t)src) | ((uintptr_t)dst)) & 15) == 0 ? n / 8 : 0;
    for (int64_t i = t; i < n8; i += stride) {
      const float4 a = reinterpret_cast<const float4*>(src)[2 * i];
      const float4 b = reinterpret_cast<const float4*>(src)[2 * i + 1];
      reinterpret_cast<uint4*>(dst)[i] =
          make_uint4(pack_bf16(a.x, a.y), pack_bf16(a.z, a.w), pack_bf16(b.x, b.y), pack_bf16(b.z, b.w));
    }
    for (int64_t i = n8 * 8 + t; i < n; i += stride) {
      const __nv_bfloat16 h = __float2bfloat16_rn(src[i]);
      dst[i] = *reinterpret_cast<const uint16_t*>(&h);
    }
  }
}

cudaError_t bf16_segments(const Bf16Segments& segs, cudaStream_t stream) {
  if (segs.count <= 0) return cudaSuccess;
  if (segs.count > kRoundSegments) return cudaErrorInvalidValue;
  int64_t total = 0;
  for (int k = 0; k < segs.count; ++k) total += segs.n[k];
  int64_t blocks = (total / 8 + 255) / 256;
  if (blocks < 1) blocks = 1;
  if (blocks > 148 * 8) blocks = 148 * 8;
  return launch_pdl(bf16_segments_kernel, dim3((unsigned)blocks), dim3(256), 0, stream, segs);
}

cudaError_t round_tf32_segments(const RoundSegments& segs, cudaStream_t stream) {
  if (segs.count <= 0) return cudaSuccess;
  if (segs.count > kRoundSegments) return cudaErrorInvalidValue;
  int64_t total = 0;
  for (int k = 0; k < segs.count; ++k) total += segs.n[k];
  int64_t blocks = (total / 4 + 255) / 256;
  if (blocks < 1) blocks = 1;
  if (blocks > 148 * 8) blocks = 148 * 8;
  return launch_pdl(round_tf32_segments_kernel, dim3((unsigned)blocks), dim3(256), 0, stream, segs);
}

cudaError_t round_tf32_copy(const float* src, float* dst, int64_t n, cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  const bool aligned = ((((uintptr_t)src) | ((uintptr_t)dst)) & 15) == 0;
  const int64_t n4 = aligned ? n / 4 : 0;
  int64_t blocks = ((aligned ? n4 : n) + 255) / 256;
  if (blocks < 1) blocks = 1;
  if (blocks > 148 * 8) blocks = 148 * 8;
  return launch_pdl(round_tf32_kernel, dim3((unsigned)blocks), dim3(256), 0, stream, src, dst, n, n4);
}

namespace {

__global__ void __launch_bounds__(256) gelu_kernel(const float* __restrict__ x, float* __restrict__ y, int64_t n,
                                                   int round) {
  pdl_prologue();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float g = tc::gelu_tanh_f(x[i]);
    y[i] = round ? rna_tf32(g) : g;
  }
}

}  // namespace

cudaError_t gelu_tanh(const float* x, float* y, int64_t n, int round_tf32, cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  int64_t blocks = (n + 255) / 256;
  if (blocks > 148 * 8) blocks = 148 * 8;
  return launch_pdl(gelu_kernel, dim3((unsigned)blocks), dim3(256), 0, stream, x, y, n, round_tf32);
}

}  // namespace sb

namespace sb {
namespace {

__global__ void __launch_bounds__(256) splitk_reduce_kernel(const float* __restrict__ p, float* __restrict__ c,
                                                            int64_t splits, int64_t M, int64_t N, int64_t ldc,
                                                            int round) {
  pdl_prologue();
  const int64_t mn = M * N;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < mn; i += (int64_t)gridDim.x * blockDim.x) {
    float acc = 0.f;
    for (int64_t s = 0; s < splits; ++s) acc += p[s * mn + i];
    if (round) acc = rna_tf32(acc);
    c[(i / N) * ldc + (i % N)] = acc;
  }
}

// 4 adjacent outputs per thread (N and ldc multiples of 4, 16-byte aligned
// buffers), the split loop unrolled so that several partial loads are in
// flight; same summation order (splits ascending) as the scalar kernel.
__global__ void __launch_bounds__(256) splitk_reduce4_kernel(const float4* __restrict__ p, float* __restrict__ c,
                                                             int splits, int mn4, int n4, int ldc, int round) {
  pdl_prologue();
  const int i4 = blockIdx.x * blockDim.x + threadIdx.x;
  if (i4 >= mn4) return;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 8
  for (int s = 0; s < splits; ++s) {
    const float4 v = p[(size_t)s * mn4 + i4];
    acc.x += v.x;
    acc.y += v.y;
    acc.z += v.z;
    acc.w += v.w;
  }
  if (round) acc = make_float4(rna_tf32(acc.x), rna_tf32(acc.y), rna_tf32(acc.z), rna_tf32(acc.w));
  const int row = i4 / n4, col = (i4 - row * n4) * 4;
  *(float4*)(c + (size_t)row * ldc + col) = acc;
}

// Every block walks the reductions in order with a grid-stride loop over each
// (4 outputs per thread where N, ldc and both buffers allow it); per output
// the partials are added in ascending split order, as in the kernels above.
__global__ void __launch_bounds__(256) splitk_reduce_segments_kernel(const ReduceSegments r) {
  pdl_prologue();
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  for (int k = 0; k < r.count; ++k) {
    const SplitReduce& g = r.seg[k];
    const int64_t mn = g.M * g.N;
    const bool vec = g.N % 4 == 0 && g.ldc % 4 == 0 && (((uintptr_t)g.partials | (uintptr_t)g.c) & 15) == 0;
    if (vec) {
      const float4* p = reinterpret_cast<const float4*>(g.partials);
      const int64_t mn4 = mn / 4, n4 = g.N / 4;
      for (int64_t i4 = t; i4 < mn4; i4 += stride) {
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int64_t s = 0; s < g.splits; ++s) {
          const float4 v = p[s * mn4 + i4];
          acc.x += v.x;
          acc.y += v.y;
          acc.z += v.z;
          acc.w += v.w;
        }
        if (g.round) acc = make_float4(rna_tf32(acc.x), rna_tf32(acc.y), rna_tf32(acc.z), rna_tf32(acc.w));
        const int64_t row = i4 / n4, col = (i4 - row * n4) * 4;
        *(float4*)(g.c + row * g.ldc + col) = acc;
      }
    } else {
      for (int64_t i = t; i < mn; i += stride) {
        float acc = 0.f;
        for (int64_t s = 0; s < g.splits; ++s) acc += g.partials[s * mn + i];
        if (g.round) acc = rna_tf32(acc);
        g.c[(i / g.N) * g.ldc + (i % g.N)] = acc;
      }
    }
  }
}

// Block b finishes 8 columns of one sum: blocks [blk0[k], blk0[k+1]) belong
// to sum k (C/8 blocks each).
struct ColSumLaunch {
  ColSums r;
  int blk0[kColSegments + 1];
};

__global__ void __launch_bounds__(256) col_sum_segments_kernel(const ColSumLaunch l) {
  pdl_prologue();
  __shared__ float part_[32][8];
  int k = 0;
  while (k + 1 < l.r.count && (int)blockIdx.x >= l.blk0[k + 1]) ++k;
  const ColSum& g = l.r.seg[k];
  const int cx = threadIdx.x & 7, ry = threadIdx.x >> 3;
  const int col = ((int)blockIdx.x - l.blk0[k]) * 8 + cx;
  float v = 0.f;
  if (col < g.C)
    for (int b = ry; b < g.parts; b += 32) v = v + g.s[(int64_t)b * g.C + col];
  part_[ry][cx] = v;
  __syncthreads();
  for (int w = 16; w > 0; w >>= 1) {
    if (ry < w) part_[ry][cx] = part_[ry][cx] + part_[ry + w][cx];
    __syncthreads();
  }
  if (ry == 0 && col < g.C) g.out[col] = part_[0][cx] + 0.0f;
}

}  // namespace

cudaError_t col_sum_segments(const ColSums& r, cudaStream_t stream) {
  if (r.count <= 0) return cudaSuccess;
  if (r.count > kColSegments) return cudaErrorInvalidValue;
  ColSumLaunch l;
  l.r = r;
  l.blk0[0] = 0;
  for (int k = 0; k < r.count; ++k) l.blk0[k + 1] = l.blk0[k] + (r.seg[k].C + 7) / 8;
  if (l.blk0[r.count] <= 0) return cudaSuccess;
  return launch_pdl(col_sum_segments_kernel, dim3((unsigned)l.blk0[r.count]), dim3(256), 0, stream, l);
}

cudaError_t splitk_reduce_segments(const ReduceSegments& r, cudaStream_t stream) {
  if (r.count <= 0) return cudaSuccess;
  if (r.count > kReduceSegments) return cudaErrorInvalidValue;
  int64_t total = 0;
  for (int k = 0; k < r.count; ++k) total += r.seg[k].M * r.seg[k].N;
  int64_t blocks = (total / 4 + 255) / 256;
  if (blocks < 1) blocks = 1;
  if (blocks > 148 * 8) blocks = 148 * 8;
  return launch_pdl(splitk_reduce_segments_kernel, dim3((unsigned)blocks), dim3(256), 0, stream, r);
}

cudaError_t splitk_reduce(const float* partials, float* c, int64_t splits, int64_t M, int64_t N, int64_t ldc,
                          int round_tf32, cudaStream_t stream) {
  int64_t mn = M * N;
  if (mn <= 0) return cudaSuccess;
  if (N % 4 == 0 && ldc % 4 == 0 && ((uintptr_t)partials & 15) == 0 && ((uintptr_t)c & 15) == 0 &&
      mn / 4 < (1ll << 31) && splits < (1ll << 31)) {
    const int64_t mn4 = mn / 4;
    return launch_pdl(splitk_reduce4_kernel, dim3((unsigned)((mn4 + 255) / 256)), dim3(256), 0, stream,
        (const float4*)partials, c, (int)splits, (int)mn4, (int)(N / 4), (int)ldc, round_tf32);
  }
  int64_t blocks = (mn + 255) / 256;
  if (blocks > 148 * 8) blocks = 148 * 8;
  return launch_pdl(splitk_reduce_kernel, dim3((unsigned)blocks), dim3(256), 0, stream, partials, c, splits, M, N, ldc,
                    round_tf32);
}

}  // namespace sb
