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

bool tc_candidate(const GemmArgs& g, int precision) {
  return precision == 1 && g.M >= 64 && g.N >= 32 && g.K >= 32 &&
         ((g.sak == 1 && g.sam % 4 == 0) || (g.sam == 1 && g.sak % 4 == 0)) &&
         ((g.sbk == 1 && g.sbn % 4 == 0) || (g.sbn == 1 && g.sbk % 4 == 0));
}

}  // namespace

size_t gemm_workspace(const GemmArgs& g, int precision) {
  bool tc = tc_candidate(g, precision);
  Split s = choose_split(g, 128, tc ? (g.N <= 64 ? 64 : 128) : 128, tc ? 32 : 8);
  return s.splits > 1 ? (size_t)(s.splits * g.M * g.N) * sizeof(float) : 0;
}

cudaError_t gemm(const GemmArgs& g, int precision, void* ws, size_t ws_bytes, cudaStream_t stream, bool* used_tc) {
  *used_tc = false;
  if (g.M <= 0 || g.N <= 0 || g.batch <= 0) return cudaSuccess;
  bool tc = tc_candidate(g, precision);
  Split s = choose_split(g, 128, tc ? (g.N <= 64 ? 64 : 128) : 128, tc ? 32 : 8);
  GemmArgs run = g;
  bool split = s.splits > 1 && ws && ws_bytes >= (size_t)(s.splits * g.M * g.N) * sizeof(float);
  if (split) {
    run.c = (float*)ws;
    run.batch = s.splits;
    run.k_chunk = s.k_chunk;
    run.scb = g.M * g.N;
    run.scm = g.N;
    run.scn = 1;
    run.round_out = 0;
  }
  cudaError_t e = cudaErrorNotSupported;
  if (tc) {
    e = gemm_tcgen05(run, false, nullptr, 0, stream);
    if (e == cudaSuccess) *used_tc = true;
  }
  if (e == cudaErrorNotSupported) e = gemm_simt(run, stream);
  if (e != cudaSuccess || !split) return e;
  return splitk_reduce((const float*)ws, g.c, s.splits, g.M, g.N, g.scm, g.round_out && *used_tc, stream);
}

}  // namespace sb
