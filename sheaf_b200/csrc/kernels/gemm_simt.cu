// f32 GEMM on CUDA cores for arbitrary operand strides (the fp32 precision mode
// and the fallback for layouts the tensor-core kernel does not take).
// 128x128x8 block tile, 256 threads, 8x8 outputs per thread, register-staged
// double buffering of the shared-memory tiles.
#include "kernels.h"
#include "pdl.h"

namespace sb {
namespace {

constexpr int BM = 128, BN = 128, BK = 8;

// operand element as f32: f32 as is, bf16 widened (bf16 is the top half of
// an f32)
__device__ __forceinline__ float ld_elem(const float* p) { return *p; }
__device__ __forceinline__ float ld_elem(const uint16_t* p) { return __uint_as_float((uint32_t)*p << 16); }

template <typename T>
__global__ void __launch_bounds__(256) sgemm_strided(GemmArgs p) {
  pdl_prologue();
  __shared__ float As[2][BK][BM + 4];
  __shared__ float Bs[2][BK][BN + 4];
  const int tid = threadIdx.x;
  const int ty = tid / 16, tx = tid % 16;
  const int64_t m0 = (int64_t)blockIdx.y * BM, n0 = (int64_t)blockIdx.x * BN;
  const bool a_kc = p.sak == 1 && p.sam != 1;  // K contiguous: load along k
  const bool b_kc = p.sbk == 1 && p.sbn != 1;

  for (int64_t bz = blockIdx.z; bz < p.batch; bz += gridDim.z) {
    const T* A = (const T*)p.a + bz * p.sab;
    const T* B = (const T*)p.b + bz * p.sbb;
    int64_t kbeg = 0, kend = p.K;
    if (p.k_chunk > 0) {  // split-K: z indexes the K range, operands are shared
      A = (const T*)p.a;
      B = (const T*)p.b;
      kbeg = bz * p.k_chunk;
      kend = kbeg + p.k_chunk < p.K ? kbeg + p.k_chunk : p.K;
    }
    float acc[8][8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;

    float ra[4], rb[4];
    // element coordinates this thread loads for A and B tiles
    int am[4], ak[4], bk[4], bn[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      if (a_kc) { am[e] = tid / 2; ak[e] = (tid % 2) * 4 + e; }
      else { ak[e] = tid / 32; am[e] = (tid % 32) * 4 + e; }
      if (b_kc) { bn[e] = tid / 2; bk[e] = (tid % 2) * 4 + e; }
      else { bk[e] = tid / 32; bn[e] = (tid % 32) * 4 + e; }
    }
    auto load = [&](int64_t k0) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        int64_t m = m0 + am[e], k = k0 + ak[e];
        ra[e] = (m < p.M && k < kend) ? ld_elem(A + m * p.sam + k * p.sak) : 0.f;
        int64_t kb = k0 + bk[e], n = n0 + bn[e];
        rb[e] = (kb < kend && n < p.N) ? ld_elem(B + kb * p.sbk + n * p.sbn) : 0.f;
      }
    };
    auto store = [&](int buf) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        As[buf][ak[e]][am[e]] = ra[e];
        Bs[buf][bk[e]][bn[e]] = rb[e];
      }
    };
    const int64_t ktiles = (kend - kbeg + BK - 1) / BK;
    load(kbeg);
    store(0);
    __syncthreads();
    for (int64_t t = 0; t < ktiles; ++t) {
      const int cur = t & 1;
      if (t + 1 < ktiles) load(kbeg + (t + 1) * BK);
#pragma unroll
      for (int kk = 0; kk < BK; ++kk) {
        float a[8], b[8];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          a[i] = As[cur][kk][ty * 4 + i];
          a[i + 4] = As[cur][kk][ty * 4 + 64 + i];
          b[i] = Bs[cur][kk][tx * 4 + i];
          b[i + 4] = Bs[cur][kk][tx * 4 + 64 + i];
        }
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
          for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
      }
      if (t + 1 < ktiles) {
        store(cur ^ 1);
        __syncthreads();
      }
    }
    float* C = p.c + bz * p.scb;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      int64_t m = m0 + ty * 4 + (i & 3) + (i >= 4 ? 64 : 0);
      if (m >= p.M) continue;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        int64_t n = n0 + tx * 4 + (j & 3) + (j >= 4 ? 64 : 0);
        if (n < p.N) C[m * p.scm + n * p.scn] = acc[i][j];
      }
    }
    __syncthreads();
  }
}

}  // namespace

cudaError_t gemm_simt(const GemmArgs& g, cudaStream_t stream) {
  if (g.M <= 0 || g.N <= 0 || g.batch <= 0) return cudaSuccess;
  dim3 grid((unsigned)((g.N + BN - 1) / BN), (unsigned)((g.M + BM - 1) / BM),
            (unsigned)(g.batch < 65535 ? g.batch : 65535));
  if (grid.y > 65535) return cudaErrorInvalidConfiguration;
  if (g.bf16) return launch_pdl(sgemm_strided<uint16_t>, grid, dim3(256), 0, stream, g);
  return launch_pdl(sgemm_strided<float>, grid, dim3(256), 0, stream, g);
}

}  // namespace sb
