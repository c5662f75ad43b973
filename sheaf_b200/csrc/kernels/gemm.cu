// GEMM dispatch: tensor-core (tcgen05) path when the precision and operand
// layouts allow it, CUDA-core path otherwise; split-K for problems whose output
// has too few tiles to fill 148 SMs (e.g. weight gradients of shape D x D with
// the whole token count as the contraction).
#include "kernels.h"

namespace sb {
namespace {

struct Split {
  int64_t splits = 1, k_chunk = 0;
};

Split choose_split(const GemmArgs& g, int64_t tile_m, int64_t tile_n, int64_t granule) {
  Split s;
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

}  // namespace

size_t gemm_workspace(const GemmArgs& g, int precision) {
  if (precision == 1) {
    TcPlan p;
    if (tc_plan(g, &p)) return p.splits > 1 ? (size_t)(p.splits * g.M * g.N) * sizeof(float) : 0;
  }
  Split s = choose_split(g, 128, 128, 8);
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
  return run;
}

}  // namespace

cudaError_t gemm(const GemmArgs& g, int precision, void* ws, size_t ws_bytes, cudaStream_t stream, bool* used_tc) {
  *used_tc = false;
  if (g.M <= 0 || g.N <= 0 || g.batch <= 0) return cudaSuccess;
  if (precision == 1) {
    TcPlan p;
    if (tc_plan(g, &p)) {
      const bool split = p.splits > 1 && ws && ws_bytes >= (size_t)(p.splits * g.M * g.N) * sizeof(float);
      cudaError_t e = gemm_tcgen05(split ? split_args(g, p.splits, p.k_chunk, ws) : g, p.cfg, stream);
      if (e == cudaSuccess) {
        *used_tc = true;
        if (!split) return cudaSuccess;
        return splitk_reduce((const float*)ws, g.c, p.splits, g.M, g.N, g.scm, g.round_out, stream);
      }
      if (e != cudaErrorNotSupported) return e;
    }
  }
  Split s = choose_split(g, 128, 128, 8);
  const bool split = s.splits > 1 && ws && ws_bytes >= (size_t)(s.splits * g.M * g.N) * sizeof(float);
  cudaError_t e = gemm_simt(split ? split_args(g, s.splits, s.k_chunk, ws) : g, stream);
  if (e != cudaSuccess || !split) return e;
  return splitk_reduce((const float*)ws, g.c, s.splits, g.M, g.N, g.scm, 0, stream);
}

}  // namespace sb
