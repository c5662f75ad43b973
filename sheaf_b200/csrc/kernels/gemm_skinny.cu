// Skinny GEMMs on CUDA cores: C = A @ B where A has at most 8 rows (the
// one-position decoding step, x[1, D] @ W^T) or, transposed, B has at most 8
// columns.  A 128-row tensor-core or CUDA-core tile would compute 16x more
// rows than exist; these kernels read every element of B once, with all of a
// warp's loads independent, and are bound by the bandwidth (L2 or HBM) of
// streaming B.  Arithmetic is f32 FMA in every precision mode (bf16 elements
// widened exactly); the summation order depends only on the shape and the
// layout, not on the launch.
#include "kernels.h"
#include "pdl.h"

namespace sb {
namespace {

constexpr int kFull = -1;  // all lanes of the warp

__device__ __forceinline__ float ld1(const float* p) { return __ldg(p); }
__device__ __forceinline__ float ld1(const uint16_t* p) { return __uint_as_float((uint32_t)__ldg(p) << 16); }
// four consecutive elements, 16-byte (f32) or 8-byte (bf16) aligned
__device__ __forceinline__ float4 ld4(const float* p) { return __ldg((const float4*)p); }
__device__ __forceinline__ float4 ld4(const uint16_t* p) {
  const uint2 u = __ldg((const uint2*)p);
  return make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xffff0000u), __uint_as_float(u.y << 16),
                     __uint_as_float(u.y & 0xffff0000u));
}

__device__ __forceinline__ float out_value(float x, int round_out) {
  if (!round_out) return x;
  uint32_t u;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(u) : "f"(x));
  return __uint_as_float(u);
}

// One warp per output column n (8 per CTA); the lanes stride along K and the
// column's MR row sums are reduced by a fixed butterfly.  VEC: B's column and
// A's rows are K-contiguous and 4-element aligned, K % 4 == 0 (4 elements per
// lane per load); otherwise element loads at any strides.
template <typename T, int MR, bool VEC>
__global__ void __launch_bounds__(256) skinny_k(GemmArgs p) {
  pdl_prologue();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t n = (int64_t)blockIdx.x * 8 + warp;
  if (n >= p.N) return;  // warp-uniform; the kernel has no block barrier
  const int rows = (int)p.M;
  for (int64_t z = blockIdx.y; z < p.batch; z += gridDim.y) {
    const T* A = (const T*)p.a + z * p.sab;
    const T* B = (const T*)p.b + z * p.sbb + n * p.sbn;
    float acc[MR];
#pragma unroll
    for (int m = 0; m < MR; ++m) acc[m] = 0.f;
    if (VEC) {
#pragma unroll 4
      for (int64_t k = 4 * lane; k < p.K; k += 128) {
        const float4 b = ld4(B + k);
#pragma unroll
        for (int m = 0; m < MR; ++m) {
          if (m < rows) {
            const float4 a = ld4(A + m * p.sam + k);
            acc[m] = fmaf(a.x, b.x, acc[m]);
            acc[m] = fmaf(a.y, b.y, acc[m]);
            acc[m] = fmaf(a.z, b.z, acc[m]);
            acc[m] = fmaf(a.w, b.w, acc[m]);
          }
        }
      }
    } else {
#pragma unroll 4
      for (int64_t k = lane; k < p.K; k += 32) {
        const float b = ld1(B + k * p.sbk);
#pragma unroll
        for (int m = 0; m < MR; ++m)
          if (m < rows) acc[m] = fmaf(ld1(A + m * p.sam + k * p.sak), b, acc[m]);
      }
    }
#pragma unroll
    for (int m = 0; m < MR; ++m)
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) acc[m] += __shfl_xor_sync((unsigned)kFull, acc[m], off);
    if (lane == 0) {
      float* C = p.c + z * p.scb + n * p.scn;
#pragma unroll
      for (int m = 0; m < MR; ++m)
        if (m < rows) C[m * p.scm] = out_value(acc[m], p.round_out);
    }
  }
}

// B with unit stride along N: lane = output column (32 per CTA, one 128-byte
// row segment per warp load), the 8 warps take interleaved K rows, and their
// partial sums are added in warp order through shared memory.
template <typename T, int MR>
__global__ void __launch_bounds__(256) skinny_n(GemmArgs p) {
  __shared__ float part[8][MR][32];
  pdl_prologue();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t n = (int64_t)blockIdx.x * 32 + lane;
  const int rows = (int)p.M;
  for (int64_t z = blockIdx.y; z < p.batch; z += gridDim.y) {
    const T* A = (const T*)p.a + z * p.sab;
    const T* B = (const T*)p.b + z * p.sbb + n;
    float acc[MR];
#pragma unroll
    for (int m = 0; m < MR; ++m) acc[m] = 0.f;
    if (n < p.N) {
#pragma unroll 4
      for (int64_t k = warp; k < p.K; k += 8) {
        const float b = ld1(B + k * p.sbk);
#pragma unroll
        for (int m = 0; m < MR; ++m)
          if (m < rows) acc[m] = fmaf(ld1(A + m * p.sam + k * p.sak), b, acc[m]);
      }
    }
#pragma unroll
    for (int m = 0; m < MR; ++m) part[warp][m][lane] = acc[m];
    __syncthreads();
    if (warp == 0 && n < p.N) {
      float* C = p.c + z * p.scb + n * p.scn;
#pragma unroll
      for (int m = 0; m < MR; ++m) {
        if (m < rows) {
          float s = part[0][m][lane];
#pragma unroll
          for (int w = 1; w < 8; ++w) s += part[w][m][lane];
          C[m * p.scm] = out_value(s, p.round_out);
        }
      }
    }
    __syncthreads();
  }
}

// C^T = B^T A^T: the same product with the roles of rows and columns swapped.
GemmArgs transposed(const GemmArgs& g) {
  GemmArgs t = g;
  t.a = g.b;
  t.b = g.a;
  t.M = g.N;
  t.N = g.M;
  t.sab = g.sbb;
  t.sam = g.sbn;
  t.sak = g.sbk;
  t.sbb = g.sab;
  t.sbk = g.sak;
  t.sbn = g.sam;
  t.scm = g.scn;
  t.scn = g.scm;
  return t;
}

template <typename T, int MR>
cudaError_t launch_rows(const GemmArgs& g, cudaStream_t stream) {
  const unsigned gz = (unsigned)(g.batch < 65535 ? g.batch : 65535);
  const size_t es = sizeof(T);
  if (g.sbk == 1) {
    const bool vec = g.sak == 1 && g.K % 4 == 0 && g.sbn % 4 == 0 && (g.M <= 1 || g.sam % 4 == 0) &&
                     g.sab % 4 == 0 && g.sbb % 4 == 0 && ((uintptr_t)g.a % (4 * es)) == 0 &&
                     ((uintptr_t)g.b % (4 * es)) == 0;
    const dim3 grid((unsigned)((g.N + 7) / 8), gz);
    if (vec) return launch_pdl(skinny_k<T, MR, true>, grid, dim3(256), 0, stream, g);
    return launch_pdl(skinny_k<T, MR, false>, grid, dim3(256), 0, stream, g);
  }
  if (g.sbn == 1) return launch_pdl(skinny_n<T, MR>, dim3((unsigned)((g.N + 31) / 32), gz), dim3(256), 0, stream, g);
  return launch_pdl(skinny_k<T, MR, false>, dim3((unsigned)((g.N + 7) / 8), gz), dim3(256), 0, stream, g);
}

template <typename T>
cudaError_t launch_skinny(const GemmArgs& g, cudaStream_t stream) {
  if (g.M <= 1) return launch_rows<T, 1>(g, stream);
  if (g.M <= 2) return launch_rows<T, 2>(g, stream);
  if (g.M <= 4) return launch_rows<T, 4>(g, stream);
  return launch_rows<T, 8>(g, stream);
}

}  // namespace

bool gemm_is_skinny(const GemmArgs& g) {
  return g.k_chunk == 0 && g.M > 0 && g.N > 0 && g.batch > 0 && (g.M <= kSkinnyMax || g.N <= kSkinnyMax);
}

cudaError_t gemm_skinny(const GemmArgs& g, cudaStream_t stream) {
  if (!gemm_is_skinny(g)) return cudaErrorNotSupported;
  const GemmArgs r = g.M <= kSkinnyMax ? g : transposed(g);
  if (r.bf16) return launch_skinny<uint16_t>(r, stream);
  return launch_skinny<float>(r, stream);
}

}  // namespace sb
