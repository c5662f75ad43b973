// Fused scaled-dot-product attention on tcgen05 tensor cores (kind::tf32),
// head dim 64, optional causal mask.  These kernels replace the region Sheaf's
// `causal_self_attention` (sheaf/lib/nn.shf) lowers to — dot(Q, K^T) / c,
// select(tril, ., -1e10), the max/exp/sum/divide softmax and dot(P, V) — and
// the reverse-mode graph its AD emits for it, so the [B,H,T,T] score, weight
// and gradient tensors never reach HBM.
//
//   attn_fwd    per (128-query block, head, batch): S = Q K_j^T in TMEM, online
//               softmax in registers (one thread per query row), P to shared
//               memory, O_j = P V_j in TMEM, O = O * alpha + O_j in registers.
//               Writes Y in [B,T,H,64] layout and the row log-sum-exp (log2
//               domain) L in [B,H,T].
//   attn_bwd_q  per query block: recomputes S and dP = dY V_j^T, dS = P (dP - D)
//               * scale, dQ += dS K_j in TMEM.  D = rowsum(dY * Y) is computed
//               first and written out for attn_bwd_kv.
//   attn_bwd_kv per 128-key block: S^T = K Q_i^T and dP^T = V dY_i^T, then
//               dV += P^T dY_i and dK += dS^T Q_i in TMEM.
// No atomics: every output element is written by exactly one thread, so the
// results are deterministic.
//
// Thread t of the 128-thread CTA owns TMEM lane t (one row of every tile);
// thread 0 issues TMA loads and tcgen05.mma.  Every mbarrier wait is bounded;
// on expiry the CTA records an error code in the shared tcgen05 error word,
// stops, frees its TMEM and exits.
#include <cuda.h>

#include <cmath>

#include "kernels.h"
#include "tc_common.h"

namespace sb {
namespace {

using namespace tc;

constexpr int HD = 64;
constexpr int kThreads = 128;
constexpr float kLog2e = 1.4426950408889634f;

// K-major operand row r of a [rows x 64] tile: two 32-column chunks of rows x
// 128 B, 16-byte units XOR-swizzled by (r & 7) exactly as TMA SWIZZLE_128B
// lays them out (tile base 1024-byte aligned).
__device__ __forceinline__ void st_row_kmajor(uint8_t* tile, int rows, int r, const float* v) {
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    uint8_t* rp = tile + c * rows * 128 + r * 128;
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const float* s = v + c * 32 + u * 4;
      *(float4*)(rp + ((u ^ (r & 7)) << 4)) = make_float4(s[0], s[1], s[2], s[3]);
    }
  }
}

// 64 consecutive TMEM columns of this thread's lane.
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, float* v) {
  uint32_t r[64];
  tmem_ld16_async(taddr, r);
  tmem_ld16_async(taddr + 16, r + 16);
  tmem_ld16_async(taddr + 32, r + 32);
  tmem_ld16_async(taddr + 48, r + 48);
  tmem_wait_ld();
#pragma unroll
  for (int i = 0; i < 64; ++i) v[i] = __uint_as_float(r[i]);
}

// Two 32-column TMA boxes of a [B,H,T,64] view (map dims {64, T, H, B}).
__device__ __forceinline__ void load_tile(uint8_t* dst, const CUtensorMap* m, uint64_t* bar, int rows, int t0, int h,
                                          int b) {
  tma_load_4d(dst, m, bar, 0, t0, h, b);
  tma_load_4d(dst + rows * 128, m, bar, 32, t0, h, b);
}

__device__ __forceinline__ void issue_mma_k64(uint32_t tmem_d, uint32_t a, int a_rows, uint32_t b, int b_rows,
                                              bool b_mn, uint32_t idesc, bool accumulate) {
#pragma unroll
  for (int kk = 0; kk < 8; ++kk) {
    const uint64_t ad = desc_kmajor(a, a_rows, kk);
    const uint64_t bd = b_mn ? desc_mnmajor(b, b_rows, kk) : desc_kmajor(b, b_rows, kk);
    mma_tf32(tmem_d, ad, bd, idesc, (accumulate || kk > 0) ? 1u : 0u);
  }
}

struct Params {
  int B, H, T;
  float scale;  // multiplier of q.k
  int causal;
  int round_out;
  // plain-load views (element strides): Y and dY rows for D, L and D rows
  const float* y; long long y_sb, y_sh, y_st;
  const float* dy; long long dy_sb, dy_sh, dy_st;
  const float* lse; long long l_sb, l_sh, l_st;
  const float* dsum; long long d_sb, d_sh, d_st;
  float* out;
};

__device__ __forceinline__ size_t bthd(const Params& p, int b, int t, int h) {
  return (((size_t)b * p.T + t) * p.H + h) * HD;
}

__device__ __forceinline__ void store_row(float* dst, const float* v, bool round) {
#pragma unroll
  for (int c = 0; c < HD; c += 4) {
    float4 q = make_float4(v[c], v[c + 1], v[c + 2], v[c + 3]);
    if (round) q = make_float4(rna_tf32(q.x), rna_tf32(q.y), rna_tf32(q.z), rna_tf32(q.w));
    *(float4*)(dst + c) = q;
  }
}

// ---------------------------------------------------------------- forward
namespace fwd {
constexpr int BM = 128, BN = 64;
constexpr int Q_OFF = 0, K_OFF = 32768, V_OFF = 49152, P_OFF = 65536, BAR_OFF = 98304;
constexpr int SMEM = 1024 + BAR_OFF + 128;
constexpr uint32_t TMEM_COLS = 128;  // S: 0..63, O_j: 64..127
}  // namespace fwd

__global__ void __launch_bounds__(kThreads, 2)
    attn_fwd(const __grid_constant__ CUtensorMap mQ, const __grid_constant__ CUtensorMap mK,
             const __grid_constant__ CUtensorMap mV, const Params p, int* err) {
  using namespace fwd;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t *sQ = sm + Q_OFF, *sK = sm + K_OFF, *sV = sm + V_OFF, *sP = sm + P_OFF;
  uint64_t* bars = (uint64_t*)(sm + BAR_OFF);
  uint64_t *bar_q = bars, *bar_k = bars + 1, *bar_v = bars + 2, *bar_s = bars + 3, *bar_o = bars + 4;
  uint32_t* tslot = (uint32_t*)(bars + 5);
  volatile int* abort_flag = (volatile int*)(tslot + 1);

  const int tid = threadIdx.x, warp = tid >> 5;
  const int q0 = blockIdx.x * BM, h = blockIdx.y, b = blockIdx.z;
  const int row = q0 + tid;
  int nkv = p.T / BN;
  if (p.causal) nkv = min(nkv, (q0 + BM) / BN);

  if (tid == 0) {
    for (int i = 0; i < 5; ++i) mbar_init(bars + i, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    fence_proxy_async();
  }
  if (warp == 0) tmem_alloc(tslot, TMEM_COLS);
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tslot;
  const uint32_t lane = (uint32_t)(warp * 32) << 16;

  if (tid == 0) {
    mbar_expect_tx(bar_q, BM * HD * 4);
    load_tile(sQ, &mQ, bar_q, BM, q0, h, b);
    mbar_expect_tx(bar_k, BN * HD * 4);
    load_tile(sK, &mK, bar_k, BN, 0, h, b);
    mbar_expect_tx(bar_v, BN * HD * 4);
    load_tile(sV, &mV, bar_v, BN, 0, h, b);
  }
  const float scale2 = p.scale * kLog2e;
  const uint32_t id_s = idesc_tf32(BM, BN, 0, 0), id_o = idesc_tf32(BM, HD, 0, 1);
  float o[HD];
#pragma unroll
  for (int c = 0; c < HD; ++c) o[c] = 0.f;
  float m = -INFINITY, l = 0.f;
  bool done = true;
  for (int j = 0; j < nkv; ++j) {
    const uint32_t ph = (uint32_t)j & 1u;
    if (tid == 0) {
      if ((j > 0 || mbar_wait(bar_q, 0, abort_flag, err, 11)) && mbar_wait(bar_k, ph, abort_flag, err, 12)) {
        fence_after();
        issue_mma_k64(tmem, smem_u32(sQ), BM, smem_u32(sK), BN, false, id_s, false);
        mma_commit(bar_s);
      }
    }
    mbar_wait(bar_s, ph, abort_flag, err, 13);
    __syncthreads();
    if (*abort_flag) { done = false; break; }
    fence_after();
    // K_j is consumed: prefetch K_{j+1}
    if (tid == 0 && j + 1 < nkv) {
      mbar_expect_tx(bar_k, BN * HD * 4);
      load_tile(sK, &mK, bar_k, BN, (j + 1) * BN, h, b);
    }
    float x[BN];
    tmem_ld64(tmem + lane, x);
    float mx = m;
#pragma unroll
    for (int c = 0; c < BN; ++c) {
      x[c] *= scale2;
      if (p.causal && j * BN + c > row) x[c] = -INFINITY;
      mx = fmaxf(mx, x[c]);
    }
    const float alpha = exp2f(m - mx);
    float rs = 0.f;
#pragma unroll
    for (int c = 0; c < BN; ++c) {
      x[c] = rna_tf32(exp2f(x[c] - mx));
      rs += x[c];
    }
    l = l * alpha + rs;
    m = mx;
    st_row_kmajor(sP, BM, tid, x);
    fence_proxy_async();
    fence_before();
    __syncthreads();
    if (tid == 0) {
      fence_after();
      if (mbar_wait(bar_v, ph, abort_flag, err, 14)) {
        issue_mma_k64(tmem + 64, smem_u32(sP), BM, smem_u32(sV), BN, true, id_o, false);
        mma_commit(bar_o);
      }
    }
    mbar_wait(bar_o, ph, abort_flag, err, 15);
    __syncthreads();
    if (*abort_flag) { done = false; break; }
    fence_after();
    // V_j is consumed: prefetch V_{j+1}
    if (tid == 0 && j + 1 < nkv) {
      mbar_expect_tx(bar_v, BN * HD * 4);
      load_tile(sV, &mV, bar_v, BN, (j + 1) * BN, h, b);
    }
    float ob[HD];
    tmem_ld64(tmem + lane + 64, ob);
#pragma unroll
    for (int c = 0; c < HD; ++c) o[c] = o[c] * alpha + ob[c];
    fence_before();
  }
  if (done) {
    const float inv = 1.f / l;
#pragma unroll
    for (int c = 0; c < HD; ++c) o[c] *= inv;
    store_row(p.out + bthd(p, b, row, h), o, p.round_out != 0);
    const size_t n = (size_t)p.B * p.T * p.H * HD;
    p.out[n + ((size_t)b * p.H + h) * p.T + row] = m + log2f(l);
  }
  fence_before();
  __syncthreads();
  if (warp == 0) {
    fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

// ---------------------------------------------------------------- backward, dQ
namespace bq {
constexpr int BM = 128, BN = 64;
constexpr int Q_OFF = 0, DO_OFF = 32768, KK_OFF = 65536, VK_OFF = 81920, KM_OFF = 98304, DS_OFF = 114688,
              BAR_OFF = 147456;
constexpr int SMEM = 1024 + BAR_OFF + 128;
constexpr uint32_t TMEM_COLS = 256;  // S: 0..63, dP: 64..127, dQ: 128..191
}  // namespace bq

__global__ void __launch_bounds__(kThreads, 1)
    attn_bwd_q(const __grid_constant__ CUtensorMap mQ, const __grid_constant__ CUtensorMap mDO,
               const __grid_constant__ CUtensorMap mK, const __grid_constant__ CUtensorMap mKm,
               const __grid_constant__ CUtensorMap mV, const Params p, int* err) {
  using namespace bq;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t *sQ = sm + Q_OFF, *sDO = sm + DO_OFF, *sK = sm + KK_OFF, *sV = sm + VK_OFF, *sKm = sm + KM_OFF,
          *sDS = sm + DS_OFF;
  uint64_t* bars = (uint64_t*)(sm + BAR_OFF);
  uint64_t *bar_q = bars, *bar_kv = bars + 1, *bar_km = bars + 2, *bar_s = bars + 3, *bar_dq = bars + 4;
  uint32_t* tslot = (uint32_t*)(bars + 5);
  volatile int* abort_flag = (volatile int*)(tslot + 1);

  const int tid = threadIdx.x, warp = tid >> 5;
  const int q0 = blockIdx.x * BM, h = blockIdx.y, b = blockIdx.z;
  const int row = q0 + tid;
  int nkv = p.T / BN;
  if (p.causal) nkv = min(nkv, (q0 + BM) / BN);

  if (tid == 0) {
    for (int i = 0; i < 5; ++i) mbar_init(bars + i, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    fence_proxy_async();
  }
  if (warp == 0) tmem_alloc(tslot, TMEM_COLS);
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tslot;
  const uint32_t lane = (uint32_t)(warp * 32) << 16;

  if (tid == 0) {
    mbar_expect_tx(bar_q, 2 * BM * HD * 4);
    load_tile(sQ, &mQ, bar_q, BM, q0, h, b);
    load_tile(sDO, &mDO, bar_q, BM, q0, h, b);
    mbar_expect_tx(bar_kv, 2 * BN * HD * 4);
    load_tile(sK, &mK, bar_kv, BN, 0, h, b);
    load_tile(sV, &mV, bar_kv, BN, 0, h, b);
  }
  // D = rowsum(dY * Y), L: this thread's row
  float D = 0.f;
  {
    const float* yr = p.y + b * p.y_sb + h * p.y_sh + row * p.y_st;
    const float* dr = p.dy + b * p.dy_sb + h * p.dy_sh + row * p.dy_st;
#pragma unroll 4
    for (int c = 0; c < HD; c += 4) {
      const float4 a = *(const float4*)(yr + c), g = *(const float4*)(dr + c);
      D += a.x * g.x + a.y * g.y + a.z * g.z + a.w * g.w;
    }
  }
  const float L2 = p.lse[b * p.l_sb + h * p.l_sh + row * p.l_st];
  const float scale2 = p.scale * kLog2e;
  const uint32_t id_s = idesc_tf32(BM, BN, 0, 0), id_q = idesc_tf32(BM, HD, 0, 1);
  bool done = true;
  for (int j = 0; j < nkv; ++j) {
    const uint32_t ph = (uint32_t)j & 1u;
    if (tid == 0) {
      if ((j > 0 || mbar_wait(bar_q, 0, abort_flag, err, 21)) && mbar_wait(bar_kv, ph, abort_flag, err, 22)) {
        fence_after();
        issue_mma_k64(tmem, smem_u32(sQ), BM, smem_u32(sK), BN, false, id_s, false);
        issue_mma_k64(tmem + 64, smem_u32(sDO), BM, smem_u32(sV), BN, false, id_s, false);
        mma_commit(bar_s);
      }
    }
    mbar_wait(bar_s, ph, abort_flag, err, 23);
    __syncthreads();
    if (*abort_flag) { done = false; break; }
    fence_after();
    // S/dP of block j (and the dQ MMA of block j-1) are done: K_j, V_j (K-major)
    // and the MN-major K buffer are free.
    if (tid == 0) {
      mbar_expect_tx(bar_km, BN * HD * 4);
      load_tile(sKm, &mKm, bar_km, BN, j * BN, h, b);
    }
    float s[BN], dp[BN];
    tmem_ld64(tmem + lane, s);
    tmem_ld64(tmem + lane + 64, dp);
    if (tid == 0 && j + 1 < nkv) {
      mbar_expect_tx(bar_kv, 2 * BN * HD * 4);
      load_tile(sK, &mK, bar_kv, BN, (j + 1) * BN, h, b);
      load_tile(sV, &mV, bar_kv, BN, (j + 1) * BN, h, b);
    }
#pragma unroll
    for (int c = 0; c < BN; ++c) {
      const bool masked = p.causal && j * BN + c > row;
      const float pr = masked ? 0.f : exp2f(s[c] * scale2 - L2);
      s[c] = rna_tf32(pr * (dp[c] - D) * p.scale);
    }
    st_row_kmajor(sDS, BM, tid, s);
    fence_proxy_async();
    fence_before();
    __syncthreads();
    if (tid == 0) {
      fence_after();
      if (mbar_wait(bar_km, ph, abort_flag, err, 24)) {
        issue_mma_k64(tmem + 128, smem_u32(sDS), BM, smem_u32(sKm), BN, true, id_q, j > 0);
        if (j + 1 == nkv) mma_commit(bar_dq);
      }
    }
  }
  if (done) {
    mbar_wait(bar_dq, 0, abort_flag, err, 25);
    __syncthreads();
    done = !*abort_flag;
  }
  if (done) {
    fence_after();
    float dq[HD];
    tmem_ld64(tmem + lane + 128, dq);
    store_row(p.out + bthd(p, b, row, h), dq, p.round_out != 0);
    const size_t n = (size_t)p.B * p.T * p.H * HD;
    p.out[n + ((size_t)b * p.H + h) * p.T + row] = D;
  }
  fence_before();
  __syncthreads();
  if (warp == 0) {
    fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

// ---------------------------------------------------------------- backward, dK dV
namespace bkv {
constexpr int BN = 128, BQ = 64;
constexpr int K_OFF = 0, V_OFF = 32768, QK_OFF = 65536, DOK_OFF = 81920, QM_OFF = 98304, DOM_OFF = 114688,
              PT_OFF = 131072, DST_OFF = 163840, LD_OFF = 196608, BAR_OFF = 197120;
constexpr int SMEM = 1024 + BAR_OFF + 128;
constexpr uint32_t TMEM_COLS = 256;  // S^T: 0..63, dP^T: 64..127, dV: 128..191, dK: 192..255
}  // namespace bkv

__global__ void __launch_bounds__(kThreads, 1)
    attn_bwd_kv(const __grid_constant__ CUtensorMap mK, const __grid_constant__ CUtensorMap mV,
                const __grid_constant__ CUtensorMap mQ, const __grid_constant__ CUtensorMap mDO,
                const __grid_constant__ CUtensorMap mQm, const __grid_constant__ CUtensorMap mDOm, const Params p,
                int* err) {
  using namespace bkv;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t *sK = sm + K_OFF, *sV = sm + V_OFF, *sQ = sm + QK_OFF, *sDO = sm + DOK_OFF, *sQm = sm + QM_OFF,
          *sDOm = sm + DOM_OFF, *sPT = sm + PT_OFF, *sDST = sm + DST_OFF;
  float* sL = (float*)(sm + LD_OFF);
  float* sD = sL + BQ;
  uint64_t* bars = (uint64_t*)(sm + BAR_OFF);
  uint64_t *bar_kv = bars, *bar_a = bars + 1, *bar_b = bars + 2, *bar_s = bars + 3, *bar_o = bars + 4;
  uint32_t* tslot = (uint32_t*)(bars + 5);
  volatile int* abort_flag = (volatile int*)(tslot + 1);

  const int tid = threadIdx.x, warp = tid >> 5;
  const int k0 = blockIdx.x * BN, h = blockIdx.y, b = blockIdx.z;
  const int row = k0 + tid;  // key index of this thread's row
  const int i0 = p.causal ? k0 / BQ : 0;
  const int nq = p.T / BQ - i0;

  if (tid == 0) {
    for (int i = 0; i < 5; ++i) mbar_init(bars + i, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    fence_proxy_async();
  }
  if (warp == 0) tmem_alloc(tslot, TMEM_COLS);
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tslot;
  const uint32_t lane = (uint32_t)(warp * 32) << 16;

  if (tid == 0) {
    mbar_expect_tx(bar_kv, 2 * BN * HD * 4);
    load_tile(sK, &mK, bar_kv, BN, k0, h, b);
    load_tile(sV, &mV, bar_kv, BN, k0, h, b);
    mbar_expect_tx(bar_a, 2 * BQ * HD * 4);
    load_tile(sQ, &mQ, bar_a, BQ, i0 * BQ, h, b);
    load_tile(sDO, &mDO, bar_a, BQ, i0 * BQ, h, b);
  }
  const float scale2 = p.scale * kLog2e;
  const uint32_t id_s = idesc_tf32(BN, BQ, 0, 0), id_g = idesc_tf32(BN, HD, 0, 1);
  bool done = nq > 0;
  for (int it = 0; it < nq; ++it) {
    const int q0 = (i0 + it) * BQ;
    const uint32_t ph = (uint32_t)it & 1u;
    if (tid == 0) {
      if ((it > 0 || mbar_wait(bar_kv, 0, abort_flag, err, 31)) && mbar_wait(bar_a, ph, abort_flag, err, 32)) {
        fence_after();
        issue_mma_k64(tmem, smem_u32(sK), BN, smem_u32(sQ), BQ, false, id_s, false);
        issue_mma_k64(tmem + 64, smem_u32(sV), BN, smem_u32(sDO), BQ, false, id_s, false);
        mma_commit(bar_s);
      }
    }
    if (tid < BQ) sL[tid] = p.lse[b * p.l_sb + h * p.l_sh + (q0 + tid) * p.l_st];
    else sD[tid - BQ] = p.dsum[b * p.d_sb + h * p.d_sh + (q0 + tid - BQ) * p.d_st];
    mbar_wait(bar_s, ph, abort_flag, err, 33);
    __syncthreads();
    if (*abort_flag) { done = false; break; }
    fence_after();
    // S^T/dP^T of this block and the dV/dK MMAs of the previous one are done.
    if (tid == 0) {
      mbar_expect_tx(bar_b, 2 * BQ * HD * 4);
      load_tile(sQm, &mQm, bar_b, BQ, q0, h, b);
      load_tile(sDOm, &mDOm, bar_b, BQ, q0, h, b);
    }
    float s[BQ], dp[BQ];
    tmem_ld64(tmem + lane, s);
    tmem_ld64(tmem + lane + 64, dp);
    if (tid == 0 && it + 1 < nq) {
      mbar_expect_tx(bar_a, 2 * BQ * HD * 4);
      load_tile(sQ, &mQ, bar_a, BQ, q0 + BQ, h, b);
      load_tile(sDO, &mDO, bar_a, BQ, q0 + BQ, h, b);
    }
#pragma unroll
    for (int c = 0; c < BQ; ++c) {
      const bool masked = p.causal && row > q0 + c;
      const float pr = masked ? 0.f : exp2f(s[c] * scale2 - sL[c]);
      s[c] = rna_tf32(pr);
      dp[c] = rna_tf32(pr * (dp[c] - sD[c]) * p.scale);
    }
    st_row_kmajor(sPT, BN, tid, s);
    st_row_kmajor(sDST, BN, tid, dp);
    fence_proxy_async();
    fence_before();
    __syncthreads();
    if (tid == 0) {
      fence_after();
      if (mbar_wait(bar_b, ph, abort_flag, err, 34)) {
        issue_mma_k64(tmem + 128, smem_u32(sPT), BN, smem_u32(sDOm), BQ, true, id_g, it > 0);
        issue_mma_k64(tmem + 192, smem_u32(sDST), BN, smem_u32(sQm), BQ, true, id_g, it > 0);
        if (it + 1 == nq) mma_commit(bar_o);
      }
    }
  }
  if (done) {
    mbar_wait(bar_o, 0, abort_flag, err, 35);
    __syncthreads();
    done = !*abort_flag;
  }
  if (done) {
    fence_after();
    float g[HD];
    const size_t n = (size_t)p.B * p.T * p.H * HD;
    tmem_ld64(tmem + lane + 192, g);
    store_row(p.out + bthd(p, b, row, h), g, p.round_out != 0);
    tmem_ld64(tmem + lane + 128, g);
    store_row(p.out + n + bthd(p, b, row, h), g, p.round_out != 0);
  }
  fence_before();
  __syncthreads();
  if (warp == 0) {
    fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

bool aligned16(const void* ptr) { return ((uintptr_t)ptr & 15) == 0; }

bool view_ok(const AttnView& v, const AttnArgs& a) {
  if (!v.p || !aligned16(v.p)) return false;
  for (int64_t s : {v.sb, v.sh, v.st})
    if (s <= 0 || s % 4) return false;
  (void)a;
  return true;
}

bool map_of(CUtensorMap* m, const AttnView& v, const AttnArgs& a, int rows, bool mn) {
  const uint64_t dims[4] = {(uint64_t)HD, (uint64_t)a.T, (uint64_t)a.H, (uint64_t)a.B};
  const uint64_t str[3] = {(uint64_t)v.st * 4, (uint64_t)v.sh * 4, (uint64_t)v.sb * 4};
  return tc_make_map(m, v.p, 4, dims, str, (uint32_t)rows, mn);
}

template <typename K>
cudaError_t set_smem(K kern, int bytes) {
  return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
}

}  // namespace

cudaError_t attention(const AttnArgs& a, cudaStream_t stream) {
  if (a.hd != HD || a.T < 128 || a.T % 128 || a.B < 1 || a.H < 1 || a.B > 65535 || a.H > 65535 || !a.out ||
      !aligned16(a.out))
    return cudaErrorNotSupported;
  if ((int64_t)a.B * a.H * a.T * HD > (1ll << 40)) return cudaErrorNotSupported;
  if (!view_ok(a.q, a) || !view_ok(a.k, a) || !view_ok(a.v, a)) return cudaErrorNotSupported;
  int* err = tc_error_word();
  if (!err) return cudaErrorNotSupported;
  Params p{};
  p.B = (int)a.B;
  p.H = (int)a.H;
  p.T = (int)a.T;
  p.scale = a.scale;
  p.causal = a.causal ? 1 : 0;
  p.round_out = a.round_out ? 1 : 0;
  p.out = a.out;
  const dim3 grid((unsigned)(a.T / 128), (unsigned)a.H, (unsigned)a.B);
  if (a.kind == AttnKind::Fwd) {
    CUtensorMap mq, mk, mv;
    if (!map_of(&mq, a.q, a, fwd::BM, false) || !map_of(&mk, a.k, a, fwd::BN, false) ||
        !map_of(&mv, a.v, a, fwd::BN, true))
      return cudaErrorNotSupported;
    static cudaError_t attr = set_smem(attn_fwd, fwd::SMEM);
    if (attr != cudaSuccess) return attr;
    attn_fwd<<<grid, kThreads, fwd::SMEM, stream>>>(mq, mk, mv, p, err);
    return cudaGetLastError();
  }
  if (!view_ok(a.dy, a) || !a.lse) return cudaErrorNotSupported;
  p.dy = a.dy.p; p.dy_sb = a.dy.sb; p.dy_sh = a.dy.sh; p.dy_st = a.dy.st;
  p.lse = a.lse; p.l_sb = a.l_sb; p.l_sh = a.l_sh; p.l_st = a.l_st;
  if (a.kind == AttnKind::BwdQ) {
    if (!view_ok(a.y, a)) return cudaErrorNotSupported;
    p.y = a.y.p; p.y_sb = a.y.sb; p.y_sh = a.y.sh; p.y_st = a.y.st;
    CUtensorMap mq, mdo, mk, mkm, mv;
    if (!map_of(&mq, a.q, a, bq::BM, false) || !map_of(&mdo, a.dy, a, bq::BM, false) ||
        !map_of(&mk, a.k, a, bq::BN, false) || !map_of(&mkm, a.k, a, bq::BN, true) ||
        !map_of(&mv, a.v, a, bq::BN, false))
      return cudaErrorNotSupported;
    static cudaError_t attr = set_smem(attn_bwd_q, bq::SMEM);
    if (attr != cudaSuccess) return attr;
    attn_bwd_q<<<grid, kThreads, bq::SMEM, stream>>>(mq, mdo, mk, mkm, mv, p, err);
    return cudaGetLastError();
  }
  if (a.kind != AttnKind::BwdKV || !a.dsum) return cudaErrorNotSupported;
  p.dsum = a.dsum; p.d_sb = a.d_sb; p.d_sh = a.d_sh; p.d_st = a.d_st;
  CUtensorMap mk, mv, mq, mdo, mqm, mdom;
  if (!map_of(&mk, a.k, a, bkv::BN, false) || !map_of(&mv, a.v, a, bkv::BN, false) ||
      !map_of(&mq, a.q, a, bkv::BQ, false) || !map_of(&mdo, a.dy, a, bkv::BQ, false) ||
      !map_of(&mqm, a.q, a, bkv::BQ, true) || !map_of(&mdom, a.dy, a, bkv::BQ, true))
    return cudaErrorNotSupported;
  static cudaError_t attr = set_smem(attn_bwd_kv, bkv::SMEM);
  if (attr != cudaSuccess) return attr;
  attn_bwd_kv<<<grid, kThreads, bkv::SMEM, stream>>>(mk, mv, mq, mdo, mqm, mdom, p, err);
  return cudaGetLastError();
}

}  // namespace sb
