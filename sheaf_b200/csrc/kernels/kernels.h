// Hand-written CUDA kernels of the backend (compiled by nvcc for sm_100a).
#pragma once
#include <cuda_runtime.h>

#include <cstdint>

namespace sb {

// Strided batched GEMM: C[b,m,n] = sum_k A[b,m,k] * B[b,k,n] (all f32 in memory).
// Strides are in elements; C is written, never accumulated.
struct GemmArgs {
  const float* a;
  const float* b;
  float* c;
  int64_t batch, M, N, K;
  int64_t sab, sam, sak;
  int64_t sbb, sbk, sbn;
  int64_t scb, scm, scn;
  int round_out = 0;  // tcgen05 path: store C rounded to nearest TF32
  // split-K (batch == 1 only): when > 0, "batch" index s computes the K range
  // [s*k_chunk, min(K, (s+1)*k_chunk)) into c + s*scb
  int64_t k_chunk = 0;
};

// C[i] = sum_s P[s*M*N + i] over `splits` partial products (row-major M x N
// partials, C with leading dimension ldc), optionally rounded to TF32.
cudaError_t splitk_reduce(const float* partials, float* c, int64_t splits, int64_t M, int64_t N, int64_t ldc,
                          int round_tf32, cudaStream_t stream);

// Dispatch: precision 1 (TF32) tries the tcgen05 kernel, anything else or an
// unsupported layout runs on CUDA cores; split-K through `ws` when the output
// has few tiles.  *used_tc reports whether the tensor-core kernel ran.
size_t gemm_workspace(const GemmArgs& g, int precision);
cudaError_t gemm(const GemmArgs& g, int precision, void* ws, size_t ws_bytes, cudaStream_t stream, bool* used_tc);

// dst[i] = src[i] rounded to nearest TF32 (cvt.rna), n elements.
cudaError_t round_tf32_copy(const float* src, float* dst, int64_t n, cudaStream_t stream);

// f32 FMA on CUDA cores; any strides.
cudaError_t gemm_simt(const GemmArgs& g, cudaStream_t stream);

// tcgen05 tensor-core GEMM (kind::tf32 on f32 operands, or kind::f16 on bf16
// copies when bf16 == true).  Returns cudaErrorNotSupported when the operand
// layout is outside what the kernel handles; the caller then uses gemm_simt.
cudaError_t gemm_tcgen05(const GemmArgs& g, bool bf16, void* workspace, size_t workspace_bytes,
                         cudaStream_t stream);
// Workspace the tcgen05 path needs for this problem (bf16 operand copies).
size_t gemm_tcgen05_workspace(const GemmArgs& g, bool bf16);
// Non-zero when a tcgen05 GEMM gave up on a bounded wait (1: ring slot,
// 2: operand tiles, 3: accumulator).  Reads a device word (synchronizing).
int gemm_tcgen05_error();

}  // namespace sb
