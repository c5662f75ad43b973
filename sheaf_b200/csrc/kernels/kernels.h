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
  // A and B hold bf16 elements (a, b address bf16 data; strides in elements):
  // tcgen05 kind::f16, or the CUDA-core kernel widening each element to f32
  int bf16 = 0;
  // split-K (batch == 1 only): when > 0, "batch" index s computes the K range
  // [s*k_chunk, min(K, (s+1)*k_chunk)) into c + s*scb
  int64_t k_chunk = 0;
  // fused epilogue: epi == kEpiGelu also writes c2 = gelu(C) elementwise
  // (Sheaf's tanh form), c2 laid out as c, rounded to TF32 when round_out2
  int epi = 0;
  float* c2 = nullptr;
  int round_out2 = 0;
};

constexpr int kEpiGelu = 1;

// C[i] = sum_s P[s*M*N + i] over `splits` partial products (row-major M x N
// partials, C with leading dimension ldc), optionally rounded to TF32.
cudaError_t splitk_reduce(const float* partials, float* c, int64_t splits, int64_t M, int64_t N, int64_t ldc,
                          int round_tf32, cudaStream_t stream);

// One split-K reduction left for later (see gemm): C[i] = sum over s of
// partials[s*M*N + i], splits ascending, C with row stride ldc, rounded to
// TF32 when round.  splits == 0: nothing pending.
struct SplitReduce {
  const float* partials = nullptr;
  float* c = nullptr;
  int64_t splits = 0, M = 0, N = 0, ldc = 0;
  int round = 0;
};
// Up to kReduceSegments pending reductions in one launch, each with the
// summation order of splitk_reduce (bit-identical results).
constexpr int kReduceSegments = 32;
struct ReduceSegments {
  SplitReduce seg[kReduceSegments];
  int count = 0;
};
cudaError_t splitk_reduce_segments(const ReduceSegments& r, cudaStream_t stream);

// Column sums finished later: out[c] = sum over parts p of s[p*C + c] for
// c < C, added as a row group's finish kernel adds them (parts split over 32
// lanes with stride 32, in order, then a fixed 32-lane tree, then + 0.0f).
struct ColSum {
  const float* s = nullptr;
  float* out = nullptr;
  int C = 0, parts = 0;
};
constexpr int kColSegments = 32;
struct ColSums {
  ColSum seg[kColSegments];
  int count = 0;
};
cudaError_t col_sum_segments(const ColSums& r, cudaStream_t stream);

// Split-K rule of the CUDA-core GEMM (shared by the session path and the
// allocation-free entry point, so both compute identical partial sums).
struct SimtSplit {
  int64_t splits = 1, k_chunk = 0;
};
SimtSplit simt_split(int64_t M, int64_t N, int64_t K, int64_t batch);
// Largest M the CUDA-core GEMM launches in one grid (65535 row tiles of 128).
constexpr int64_t kSimtMaxM = 65535ll * 128;

// Dispatch: precision 1 (TF32) tries the tcgen05 kernel, anything else or an
// unsupported layout runs on CUDA cores; split-K through `ws` when the output
// has few tiles.  *used_tc reports whether the tensor-core kernel ran.  With
// `deferred` set, a split product (without a fused epilogue) leaves its
// partial sums in ws and describes their reduction in *deferred instead of
// launching it: the caller runs it (splitk_reduce_segments) before C is read
// and before ws is reused.
size_t gemm_workspace(const GemmArgs& g, int precision);
cudaError_t gemm(const GemmArgs& g, int precision, void* ws, size_t ws_bytes, cudaStream_t stream, bool* used_tc,
                 SplitReduce* deferred = nullptr);

// Two independent GEMMs (neither reads the other's output) in one tensor-core
// launch: the tiles of g[0], then those of g[1], one persistent tile sequence,
// with the configuration measured for the pair.  For the products of a
// backward pass whose tiles alone would leave SMs idle (a layer's dX and dW).
// Each split product leaves its partial sums in its part of ws (the first
// gemm_workspace(g[0]) bytes, rounded up to 256, then g[1]'s) and describes
// their reduction in deferred[q]; both products' results are as gemm() gives
// them.  cudaErrorNotSupported (nothing launched) when either product needs
// another path (CUDA cores, padded operands, a fused epilogue, operands of
// different types) or when either writes memory that the other reads or
// writes (the two run at the same time); the caller then runs them one by one.
constexpr int kGemmGroupMax = 2;
cudaError_t gemm_pair(const GemmArgs g[2], int precision, void* ws, size_t ws_bytes, cudaStream_t stream,
                      SplitReduce deferred[2]);

// dst[i] = bf16(src[i]), round to nearest even, n elements.
cudaError_t bf16_copy(const float* src, uint16_t* dst, int64_t n, cudaStream_t stream);

// dst[i] = src[i] rounded to nearest TF32 (cvt.rna), n elements.
cudaError_t round_tf32_copy(const float* src, float* dst, int64_t n, cudaStream_t stream);

// Up to kRoundSegments such copies in one launch (the per-call TF32 copies of
// a function's weights): segment i copies n[i] elements from src[i] to dst[i].
constexpr int kRoundSegments = 48;
struct RoundSegments {
  const float* src[kRoundSegments];
  float* dst[kRoundSegments];
  int64_t n[kRoundSegments];
  int count;
};
cudaError_t round_tf32_segments(const RoundSegments& segs, cudaStream_t stream);

// The same for bf16 copies (round to nearest even): consecutive conversion
// steps of a call (the bf16 copies of its weights) in one launch.
struct Bf16Segments {
  const float* src[kRoundSegments];
  uint16_t* dst[kRoundSegments];
  int64_t n[kRoundSegments];
  int count;
};
cudaError_t bf16_segments(const Bf16Segments& segs, cudaStream_t stream);

// y = gelu(x) = 0.5 * (x * (1 + tanh(0.7978846 * (x + 0.044715 * (x * (x *
// x)))))) in f32, Sheaf's gelu (sheaf/lib/nn.shf) in its operation order;
// optionally rounded to TF32.  The unfused form of the GEMM epilogue.
cudaError_t gelu_tanh(const float* x, float* y, int64_t n, int round_tf32, cudaStream_t stream);

// f32 FMA on CUDA cores; any strides.
cudaError_t gemm_simt(const GemmArgs& g, cudaStream_t stream);

// GEMMs with at most kSkinnyMax rows (or, transposed, columns) run on the
// CUDA cores, B streamed once: no workspace, f32 FMA in every precision mode.
constexpr int64_t kSkinnyMax = 8;
bool gemm_is_skinny(const GemmArgs& g);
cudaError_t gemm_skinny(const GemmArgs& g, cudaStream_t stream);

// tcgen05 tensor-core GEMM (kind::tf32 on f32 operands).  tc_plan fixes the
// split-K factor of a problem by a rule on its shape and proposes a kernel
// configuration (single-CTA or CTA-pair tiles, tile width, TMEM accumulators)
// by a cost model; false when the operand layout is outside what the
// tensor-core kernels handle (the caller then uses gemm_simt).  gemm_tcgen05
// runs configuration `cfg` (0 .. tc_num_configs() - 1) on g, where g is
// already split (batch = splits, k_chunk) when the plan split K.  Every
// configuration gives bit-identical results for the same split.
// tc_forced_config() is the configuration forced by the environment, or -1.
struct TcPlan {
  int cfg = -1;
  int64_t splits = 1, k_chunk = 0;
};
bool tc_plan(const GemmArgs& g, TcPlan* plan);
int tc_num_configs();
int tc_forced_config();
cudaError_t gemm_tcgen05(const GemmArgs& g, int cfg, cudaStream_t stream);
// The same for n <= kGemmGroupMax products of one operand type in one launch
// (g[q] already split where its plan split K).
cudaError_t gemm_tcgen05_group(const GemmArgs* g, int n, int cfg, cudaStream_t stream);
// Non-zero when a tcgen05 kernel gave up on a bounded wait (GEMM 1: ring slot,
// 2: operand tiles, 3: accumulator; attention 11..35) or found its shared
// memory window misaligned (9), or the row scatter-add found inconsistent
// segment offsets (41..43).  Reads a device word (synchronizing).
int gemm_tcgen05_error();

// Fused attention, head dim 64 (kernels/attention.cu).  Views are [B,H,T,64]
// with unit stride on the last dim; strides in elements.
enum class AttnKind : int { Fwd = 0, BwdQ = 1, BwdKV = 2 };
struct AttnView {
  const float* p = nullptr;
  int64_t sb = 0, sh = 0, st = 0;
};
struct AttnArgs {
  AttnKind kind = AttnKind::Fwd;
  int64_t B = 0, H = 0, T = 0, hd = 0;
  float scale = 1.f;      // multiplier of q.k before the softmax
  bool causal = false;    // key index > query index is masked out
  bool round_out = false; // store Y / dQ / dK / dV rounded to TF32
  AttnView q, k, v, dy, y;
  const float* lse = nullptr;  // [B,H,T] row log2-sum-exp (backward)
  int64_t l_sb = 0, l_sh = 0, l_st = 0;
  const float* dsum = nullptr; // [B,H,T] rowsum(dY * Y) (BwdKV)
  int64_t d_sb = 0, d_sh = 0, d_st = 0;
  // Default packing (out_ld, stats, out_v unset):
  // Fwd:   [Y (B,T,H,64) | L (B,H,T)]
  // BwdQ:  [dQ (B,T,H,64) | D (B,H,T)]
  // BwdKV: [dK (B,T,H,64) | dV (B,T,H,64)]
  // out_ld (elements between consecutive tokens of the (B,T,H,64) outputs,
  // a multiple of 4, at least H*64), stats (L / D) and out_v (dV) override
  // it, e.g. to interleave dQ, dK, dV as one (B,T,3,H,64) buffer.
  float* out = nullptr;
  int64_t out_ld = 0;
  float* stats = nullptr;
  float* out_v = nullptr;
};
cudaError_t attention(const AttnArgs& a, cudaStream_t stream);

// Row scatter-add (kernels/scatter.cu): out[k, :] = sum over rows r of adj
// (n x d, row-major) with key(r) == k, in row order; out is v x d.  Keys from
// idx (n values, f32 holding integers, or i32); keys outside [0, v) or not
// integral hit nothing.  ws holds scatter_add_rows_workspace(n, v, d) bytes.
size_t scatter_add_rows_workspace(int64_t n, int64_t v, int64_t d);
cudaError_t scatter_add_rows(const void* idx, bool idx_f32, const float* adj, float* out, int64_t n, int64_t d,
                             int64_t v, void* ws, cudaStream_t stream);

// Stable sort of rows of (f32 key, i32 payload) (kernels/sort.cu): out row =
// [sorted keys | payload bits as f32], descending or ascending by key.
cudaError_t sort_pairs(const float* keys, const int* payload, float* out, int64_t rows, int64_t n, bool descending,
                       cudaStream_t stream);

// Fused clip-by-global-norm + AdamW (kernels/optim.cu).  Leaves and chunks
// live in device memory; partials holds one float per chunk.  norm_out (device,
// may be null) receives the global L2 norm of the gradients before clipping.
struct OptLeaf {
  float* p;
  const float* g;
  float* m;
  float* v;
  int64_t n;
};
struct OptChunk {
  int leaf;
  int64_t off, len;
};
struct AdamwScalars {
  float lr, b1, b2, one_minus_b1, one_minus_b2, eps, wd, bc_m, bc_v, max_norm;
  int clip;
};
cudaError_t adamw_step(const OptLeaf* leaves, const OptChunk* chunks, int n_chunks, float* partials,
                       float* norm_out, const AdamwScalars& a, cudaStream_t stream);

}  // namespace sb
