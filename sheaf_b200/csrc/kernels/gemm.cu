// GEMM dispatch: tensor-core (tcgen05) path when the precision and operand
// layouts allow it, CUDA-core path otherwise; split-K for problems whose output
// has too few tiles to fill 148 SMs (e.g. weight gradients of shape D x D with
// the whole token count as the contraction).
#include <algorithm>
#include <array>
#include <map>
#include <mutex>

#include "kernels.h"
#include "pdl.h"

namespace sb {

// The CUDA-core GEMM's split-K rule: when the 128 x 128 output tiles of a
// single GEMM cannot fill the GPU and K is long, K is cut into ranges of at
// least 512 (multiples of `granule`) for about two waves of CTAs.
static SimtSplit choose_split(const GemmArgs& g, int64_t tile_m, int64_t tile_n, int64_t granule) {
  SimtSplit s;
  if (g.batch != 1 || g.K < 2048) return s;
  int64_t tiles = ((g.M + tile_m - 1) / tile_m) * ((g.N + tile_n - 1) / tile_n);
  if (tiles >= 120) return s;
  int64_t want = (2 * 148 + tiles - 1) / tiles;            // ~2 waves of CTAs
  int64_t max_by_k = g.K / 512;                           // at least 512 of K per split
  int64_t n = want < max_by_k ? want : max_by_k;
  if (n < 2) return s;
  int64_t chunk = (g.K + n - 1) / n;
  chunk = (chunk + granule - 1) / granule * granule;
  s.k_chunk = chunk;
  s.splits = (g.K + chunk - 1) / chunk;
  return s;
}

SimtSplit simt_split(int64_t M, int64_t N, int64_t K, int64_t batch) {
  GemmArgs g{};
  g.M = M;
  g.N = N;
  g.K = K;
  g.batch = batch;
  return choose_split(g, 128, 128, 8);
}

namespace {

// An operand whose unit-stride (inner) dimension is fine but whose row stride
// or base address is not 16-byte aligned (e.g. a vocabulary of 65 as the
// inner extent) is copied to a dense buffer with the row stride rounded up to
// 4 floats, keeping its major-ness; the tensor maps use the logical extents,
// so the padding columns are never read.
struct PadOp {
  bool on = false;
  int64_t rows = 0, inner = 0, s_row = 0, s_batch = 0, ld = 0;
  size_t elems = 0;
};

struct Padding {
  PadOp a, b;
  TcPlan plan;
  size_t a_off = 0, b_off = 0, split_bytes = 0, total = 0;
};

constexpr size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// Describes operand (rows x inner per batch) with strides (s_row, 1) and
// batch stride s_batch as a padded dense copy; the padded view has row stride
// ld and batch stride rows * ld.
PadOp pad_op(int64_t batch, int64_t rows, int64_t inner, int64_t s_row, int64_t s_batch, int64_t q) {
  PadOp o;
  o.on = true;
  o.rows = rows;
  o.inner = inner;
  o.s_row = s_row;
  o.s_batch = s_batch;
  o.ld = (inner + q - 1) / q * q;
  o.elems = (size_t)(batch * rows * o.ld);
  return o;
}

// The tensor-core plan of g, padding A and/or B when only their row strides or
// base addresses keep g off the tensor cores.  *view is g with the padded
// operands at (fake, aligned) workspace offsets; false when no padding helps.
bool pad_plan(const GemmArgs& g, Padding* pd, GemmArgs* view) {
  if (g.batch > 1 && (g.sab < 0 || g.sbb < 0)) return false;
  GemmArgs v = g;
  const int64_t q = g.bf16 ? 8 : 4;  // elements per 16 bytes
  const size_t es = g.bf16 ? 2 : 4;
  // A: K-major (sak == 1, rows M) or M-major (sam == 1, rows K)
  const bool a_ok = ((uintptr_t)g.a & 15) == 0 &&
                    ((g.sak == 1 && g.sam % q == 0 && g.sam >= g.K) || (g.sam == 1 && g.sak % q == 0 && g.sak >= g.M)) &&
                    (g.batch == 1 || g.sab % q == 0);
  if (!a_ok) {
    if (g.sak == 1 && g.sam >= g.K) pd->a = pad_op(g.batch, g.M, g.K, g.sam, g.sab, q);
    else if (g.sam == 1 && g.sak >= g.M) pd->a = pad_op(g.batch, g.K, g.M, g.sak, g.sab, q);
    else return false;
    if (g.sak == 1) { v.sam = pd->a.ld; v.sak = 1; }
    else { v.sak = pd->a.ld; v.sam = 1; }
    v.sab = pd->a.rows * pd->a.ld;
  }
  const bool b_ok = ((uintptr_t)g.b & 15) == 0 &&
                    ((g.sbk == 1 && g.sbn % q == 0 && g.sbn >= g.K) || (g.sbn == 1 && g.sbk % q == 0 && g.sbk >= g.N)) &&
                    (g.batch == 1 || g.sbb % q == 0);
  if (!b_ok) {
    if (g.sbk == 1 && g.sbn >= g.K) pd->b = pad_op(g.batch, g.N, g.K, g.sbn, g.sbb, q);
    else if (g.sbn == 1 && g.sbk >= g.N) pd->b = pad_op(g.batch, g.K, g.N, g.sbk, g.sbb, q);
    else return false;
    if (g.sbk == 1) { v.sbn = pd->b.ld; v.sbk = 1; }
    else { v.sbk = pd->b.ld; v.sbn = 1; }
    v.sbb = pd->b.rows * pd->b.ld;
  }
  if (!pd->a.on && !pd->b.on) return false;
  // plan with aligned stand-in addresses; the real ones are set at run time
  if (pd->a.on) v.a = reinterpret_cast<const float*>(uintptr_t(1) << 12);
  if (pd->b.on) v.b = reinterpret_cast<const float*>(uintptr_t(1) << 12);
  if (!tc_plan(v, &pd->plan)) return false;
  pd->split_bytes = pd->plan.splits > 1 ? align256((size_t)(pd->plan.splits * g.M * g.N) * sizeof(float)) : 0;
  pd->a_off = pd->split_bytes;
  pd->b_off = pd->a_off + (pd->a.on ? align256(pd->a.elems * es) : 0);
  pd->total = pd->b_off + (pd->b.on ? align256(pd->b.elems * es) : 0);
  *view = v;
  return true;
}

// One thread per element of the padded copy's logical extent.  Index math in
// the narrowest type that holds it (64-bit division is slow).
template <typename T, typename I>
__global__ void __launch_bounds__(256) pad_copy_kernel(const T* __restrict__ src, T* __restrict__ dst, I batch,
                                                       I rows, I inner, int64_t s_row, int64_t s_batch, I ld) {
  pdl_prologue();
  const I n = batch * rows * inner;
  for (I i = (I)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (I)gridDim.x * blockDim.x) {
    const I rr = i / inner;
    const I c = i - rr * inner;
    const I b = rr / rows;
    const I r = rr - b * rows;
    dst[((int64_t)b * rows + r) * ld + c] = src[(int64_t)b * s_batch + (int64_t)r * s_row + c];
  }
}

template <typename T>
cudaError_t pad_copy_t(const T* src, T* dst, int64_t batch, const PadOp& o, cudaStream_t stream) {
  const int64_t n = batch * o.rows * o.inner;
  if (n <= 0) return cudaSuccess;
  const int64_t blocks = std::min<int64_t>((n + 255) / 256, 148 * 16);
  if (n < (int64_t(1) << 31) - 148 * 16 * 256)
    return launch_pdl(pad_copy_kernel<T, uint32_t>, dim3((unsigned)blocks), dim3(256), 0, stream, src, dst,
                      (uint32_t)batch, (uint32_t)o.rows, (uint32_t)o.inner, o.s_row, o.s_batch, (uint32_t)o.ld);
  return launch_pdl(pad_copy_kernel<T, int64_t>, dim3((unsigned)blocks), dim3(256), 0, stream, src, dst, batch,
                    o.rows, o.inner, o.s_row, o.s_batch, o.ld);
}

// Padded copy of an operand of f32 or (bf16) 16-bit elements.
cudaError_t pad_copy(const float* src, float* dst, int64_t batch, const PadOp& o, bool bf16, cudaStream_t stream) {
  if (bf16) return pad_copy_t((const uint16_t*)src, (uint16_t*)dst, batch, o, stream);
  return pad_copy_t(src, dst, batch, o, stream);
}

}  // namespace

size_t gemm_workspace(const GemmArgs& g, int precision) {
  if (gemm_is_skinny(g)) return 0;
  if (precision == 1 || g.bf16) {
    TcPlan p;
    if (tc_plan(g, &p)) return p.splits > 1 ? (size_t)(p.splits * g.M * g.N) * sizeof(float) : 0;
    Padding pd;
    GemmArgs v;
    if (pad_plan(g, &pd, &v)) return pd.total;
  }
  SimtSplit s = choose_split(g, 128, 128, 8);
  return s.splits > 1 ? (size_t)(s.splits * g.M * g.N) * sizeof(float) : 0;
}

namespace {

// g split along K into `splits` partial products written to ws.
GemmArgs split_args(const GemmArgs& g, int64_t splits, int64_t k_chunk, void* ws) {
  GemmArgs run = g;
  run.c = (float*)ws;
  run.batch = splits;
  run.k_chunk = k_chunk;
  run.scb = g.M * g.N;
  run.scm = g.N;
  run.scn = 1;
  run.round_out = 0;
  run.epi = 0;  // partial sums: the epilogue applies to the total
  return run;
}

// Measured choice of the tensor-core configuration, once per problem
// signature (shapes, strides, split, 16-byte alignment of the pointers): each
// configuration runs once to warm up and twice timed on the real operands
// (the output is rewritten by the call that follows, with the same values:
// configurations differ only in tiling, not in summation order), and the
// fastest is kept.  The cost model's proposal stands while the stream is being
// captured into a graph, or when the environment forces a configuration.
using TuneKey = std::array<int64_t, 20>;
std::mutex tune_mu;
std::map<TuneKey, int> tune_cache;
std::map<std::array<int64_t, 40>, int> tune_pair_cache;

TuneKey tune_key(const GemmArgs& run) {
  return {run.batch, run.M, run.N, run.K, run.sab, run.sam, run.sak, run.sbb, run.sbk, run.sbn,
          run.scb, run.scm, run.scn, run.k_chunk, run.round_out, (int64_t)((uintptr_t)run.a & 15),
          (int64_t)((uintptr_t)run.b & 15), (int64_t)((uintptr_t)run.c & 15), (int64_t)run.bf16,
          (int64_t)run.epi};
}

// The fastest configuration for which run_cfg(c) succeeds, each timed twice
// after one warm-up run; -1 while the stream is being captured or when no
// configuration ran.
template <typename F>
int measure_configs(F run_cfg, cudaStream_t stream) {
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(stream, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone) return -1;
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  if (cudaEventCreate(&e0) != cudaSuccess || cudaEventCreate(&e1) != cudaSuccess) {
    if (e0) cudaEventDestroy(e0);
    return -1;
  }
  int best = -1;
  float best_ms = 1e30f;
  for (int c = 0; c < tc_num_configs(); ++c) {
    if (run_cfg(c) != cudaSuccess) continue;
    cudaEventRecord(e0, stream);
    bool ok = run_cfg(c) == cudaSuccess && run_cfg(c) == cudaSuccess;
    cudaEventRecord(e1, stream);
    float ms = 0.f;
    if (!ok || cudaEventSynchronize(e1) != cudaSuccess || cudaEventElapsedTime(&ms, e0, e1) != cudaSuccess) continue;
    if (ms < best_ms) {
      best_ms = ms;
      best = c;
    }
  }
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  return best;
}

int tuned_config(const GemmArgs& run, int proposed, cudaStream_t stream) {
  if (tc_forced_config() >= 0) return proposed;
  const TuneKey key = tune_key(run);
  std::lock_guard<std::mutex> lock(tune_mu);
  auto it = tune_cache.find(key);
  if (it != tune_cache.end()) return it->second;
  const int best = measure_configs([&](int c) { return gemm_tcgen05(run, c, stream); }, stream);
  if (best < 0) return proposed;
  tune_cache[key] = best;
  return best;
}

// The same for the launch of two products: keyed by both signatures, timed as
// one launch.
int tuned_pair_config(const GemmArgs run[2], int proposed, cudaStream_t stream) {
  if (tc_forced_config() >= 0) return proposed;
  std::array<int64_t, 40> key;
  const TuneKey k0 = tune_key(run[0]), k1 = tune_key(run[1]);
  std::copy(k0.begin(), k0.end(), key.begin());
  std::copy(k1.begin(), k1.end(), key.begin() + k0.size());
  std::lock_guard<std::mutex> lock(tune_mu);
  auto it = tune_pair_cache.find(key);
  if (it != tune_pair_cache.end()) return it->second;
  const int best = measure_configs([&](int c) { return gemm_tcgen05_group(run, 2, c, stream); }, stream);
  if (best < 0) return proposed;
  tune_pair_cache[key] = best;
  return best;
}

}  // namespace

namespace {

// The product itself; *fused reports whether the tensor-core kernel also
// wrote the fused epilogue's output (unsplit launches only: split-K partials
// must not pass through it).
cudaError_t gemm_main(const GemmArgs& g, int precision, void* ws, size_t ws_bytes, cudaStream_t stream,
                      bool* used_tc, bool* fused, SplitReduce* deferred) {
  // the reduction of a split product: launched now, or described for the caller
  auto reduce = [&](int64_t splits, int round) -> cudaError_t {
    if (deferred) {
      deferred->partials = (const float*)ws;
      deferred->c = g.c;
      deferred->splits = splits;
      deferred->M = g.M;
      deferred->N = g.N;
      deferred->ldc = g.scm;
      deferred->round = round;
      return cudaSuccess;
    }
    return splitk_reduce((const float*)ws, g.c, splits, g.M, g.N, g.scm, round, stream);
  };
  if (gemm_is_skinny(g)) return gemm_skinny(g, stream);
  // bf16 operands run on the tensor cores in every precision mode (their
  // products are exact in f32, so kind::f16 is the graph's arithmetic)
  if (precision == 1 || g.bf16) {
    TcPlan p;
    if (tc_plan(g, &p)) {
      const bool split = p.splits > 1 && ws && ws_bytes >= (size_t)(p.splits * g.M * g.N) * sizeof(float);
      const GemmArgs run = split ? split_args(g, p.splits, p.k_chunk, ws) : g;
      cudaError_t e = gemm_tcgen05(run, tuned_config(run, p.cfg, stream), stream);
      if (e == cudaSuccess) {
        *used_tc = true;
        *fused = !split;
        if (!split) return cudaSuccess;
        return reduce(p.splits, g.round_out);
      }
      if (e != cudaErrorNotSupported) return e;
    } else {
      Padding pd;
      GemmArgs v;
      if (pad_plan(g, &pd, &v) && ws && ws_bytes >= pd.total) {
        char* base = (char*)ws;
        if (pd.a.on) {
          v.a = (const float*)(base + pd.a_off);
          cudaError_t e = pad_copy(g.a, (float*)v.a, g.batch, pd.a, g.bf16 != 0, stream);
          if (e != cudaSuccess) return e;
        }
        if (pd.b.on) {
          v.b = (const float*)(base + pd.b_off);
          cudaError_t e = pad_copy(g.b, (float*)v.b, g.batch, pd.b, g.bf16 != 0, stream);
          if (e != cudaSuccess) return e;
        }
        const bool split = pd.plan.splits > 1;
        const GemmArgs run = split ? split_args(v, pd.plan.splits, pd.plan.k_chunk, ws) : v;
        cudaError_t e = gemm_tcgen05(run, tuned_config(run, pd.plan.cfg, stream), stream);
        if (e != cudaSuccess) return e;
        *used_tc = true;
        *fused = !split;
        if (!split) return cudaSuccess;
        return reduce(pd.plan.splits, g.round_out);
      }
    }
  }
  SimtSplit s = choose_split(g, 128, 128, 8);
  const bool split = s.splits > 1 && ws && ws_bytes >= (size_t)(s.splits * g.M * g.N) * sizeof(float);
  cudaError_t e = gemm_simt(split ? split_args(g, s.splits, s.k_chunk, ws) : g, stream);
  if (e != cudaSuccess || !split) return e;
  return reduce(s.splits, 0);
}

}  // namespace

cudaError_t gemm(const GemmArgs& g, int precision, void* ws, size_t ws_bytes, cudaStream_t stream, bool* used_tc,
                 SplitReduce* deferred) {
  *used_tc = false;
  if (deferred) *deferred = SplitReduce{};
  if (g.M <= 0 || g.N <= 0 || g.batch <= 0) return cudaSuccess;
  // the fused epilogue's output is laid out densely like C (the unfused form
  // below reads C as one contiguous array)
  if (g.epi && (g.epi != kEpiGelu || !g.c2 || g.scn != 1 || g.scm != g.N || (g.batch > 1 && g.scb != g.M * g.N)))
    return cudaErrorInvalidValue;
  bool fused = false;
  // a fused epilogue applies to the reduced product: its split-K sum is not deferred
  cudaError_t e = gemm_main(g, precision, ws, ws_bytes, stream, used_tc, &fused, g.epi ? nullptr : deferred);
  if (e != cudaSuccess || !g.epi || fused) return e;
  return gelu_tanh(g.c, g.c2, g.batch * g.M * g.N, g.round_out2, stream);
}

namespace {

// Bytes [lo, hi) that a strided rows x cols (x batch) array of es-byte
// elements spans; ok = false for a negative stride (no span is claimed).
struct Span {
  uintptr_t lo = 0, hi = 0;
  bool ok = true;
};

Span span_of(const void* p, int64_t batch, int64_t sb, int64_t rows, int64_t sr, int64_t cols, int64_t sc,
             int64_t es) {
  Span r;
  if ((batch > 1 && sb < 0) || (rows > 1 && sr < 0) || (cols > 1 && sc < 0)) {
    r.ok = false;
    return r;
  }
  const int64_t last = (batch - 1) * sb + (rows - 1) * sr + (cols - 1) * sc;
  r.lo = (uintptr_t)p;
  r.hi = r.lo + (uintptr_t)((last + 1) * es);
  return r;
}

bool apart(const Span& x, const Span& y) { return x.ok && y.ok && (x.hi <= y.lo || y.hi <= x.lo); }

// The products of a pair run at the same time, so neither may write memory
// that the other reads or writes.  A plan frees a value's memory after its
// last reader, so the second product's output may have been placed where the
// first product's operand was, which is safe only one step after the other.
bool independent(const GemmArgs& w, const GemmArgs& r) {
  const int64_t es = r.bf16 ? 2 : 4;
  const Span out = span_of(w.c, w.batch, w.scb, w.M, w.scm, w.N, w.scn, 4);
  const Span ra = span_of(r.a, r.batch, r.sab, r.M, r.sam, r.K, r.sak, es);
  const Span rb = span_of(r.b, r.batch, r.sbb, r.K, r.sbk, r.N, r.sbn, es);
  const Span rc = span_of(r.c, r.batch, r.scb, r.M, r.scm, r.N, r.scn, 4);
  return apart(out, ra) && apart(out, rb) && apart(out, rc);
}

}  // namespace

cudaError_t gemm_pair(const GemmArgs g[2], int precision, void* ws, size_t ws_bytes, cudaStream_t stream,
                      SplitReduce deferred[2]) {
  deferred[0] = SplitReduce{};
  deferred[1] = SplitReduce{};
  if (!independent(g[0], g[1]) || !independent(g[1], g[0])) return cudaErrorNotSupported;
  GemmArgs run[2];
  TcPlan plan[2];
  size_t off = 0;
  for (int q = 0; q < 2; ++q) {
    const GemmArgs& a = g[q];
    if (a.M <= 0 || a.N <= 0 || a.batch <= 0 || a.epi || a.bf16 != g[0].bf16 || gemm_is_skinny(a))
      return cudaErrorNotSupported;
    if (precision != 1 && !a.bf16) return cudaErrorNotSupported;
    if (!tc_plan(a, &plan[q])) return cudaErrorNotSupported;
    run[q] = a;
    if (plan[q].splits > 1) {
      const size_t need = (size_t)(plan[q].splits * a.M * a.N) * sizeof(float);
      if (!ws || off + need > ws_bytes) return cudaErrorNotSupported;
      run[q] = split_args(a, plan[q].splits, plan[q].k_chunk, (char*)ws + off);
      off += (need + 255) & ~(size_t)255;
    }
  }
  // the cost model's proposal for the larger product stands where nothing is measured
  const double f0 = (double)g[0].M * g[0].N * g[0].K * g[0].batch, f1 = (double)g[1].M * g[1].N * g[1].K * g[1].batch;
  const int cfg = tuned_pair_config(run, f0 >= f1 ? plan[0].cfg : plan[1].cfg, stream);
  cudaError_t e = gemm_tcgen05_group(run, 2, cfg, stream);
  if (e != cudaSuccess) return e;
  for (int q = 0; q < 2; ++q) {
    if (plan[q].splits <= 1) continue;
    deferred[q].partials = run[q].c;
    deferred[q].c = g[q].c;
    deferred[q].splits = plan[q].splits;
    deferred[q].M = g[q].M;
    deferred[q].N = g[q].N;
    deferred[q].ldc = g[q].scm;
    deferred[q].round = g[q].round_out;
  }
  return cudaSuccess;
}

}  // namespace sb
