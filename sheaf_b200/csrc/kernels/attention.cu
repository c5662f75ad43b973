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
#include "pdl.h"
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
  float* stats;  // [B,H,T] row statistics written by the pass (L forward, D in the dQ pass)
};

// ---------------------------------------------------------------- forward
namespace fwd {
constexpr int BM = 128, BN = 64;
// shared memory: Q (BM x 64; reused to stage Y), K_j and V_j double-buffered
constexpr int Q_OFF = 0, K_OFF = 32768, V_OFF = 65536, TILE = BN * HD * 4, BAR_OFF = 98304;
constexpr int SMEM = BAR_OFF + 256;
// TMEM: S_j, then P_j in place, in columns (j & 1) * 64; O_j = P_j V_j in
// columns 128 + (j & 1) * 64
constexpr uint32_t TMEM_COLS = 256;
}  // namespace fwd

// Software-pipelined: while the threads turn S_j into P_j, the tensor cores
// compute S_{j+1} (issued as soon as S_j is in registers) and O_{j-1}; the
// threads fold O_{j-1} into the running output after issuing O_j.  P_j is
// written back over S_j in TMEM and read from there by the O_j MMA, so it
// never touches shared memory.  K and V tiles are double-buffered.
__global__ void __launch_bounds__(kThreads, 2)
    attn_fwd(const __grid_constant__ CUtensorMap mQ, const __grid_constant__ CUtensorMap mK,
             const __grid_constant__ CUtensorMap mV, const __grid_constant__ CUtensorMap mY, const Params p,
             int* err) {
  pdl_prologue();
  using namespace fwd;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  if (smem_u32(smem_raw) & 1023u) {  // uniform: every thread leaves before any barrier
    if (threadIdx.x == 0) atomicExch(err, 10);
    return;
  }
  uint8_t* sm = smem_raw;
  uint8_t* sQ = sm + Q_OFF;
  auto sK = [&](int i) { return sm + K_OFF + i * TILE; };
  auto sV = [&](int i) { return sm + V_OFF + i * TILE; };
  uint64_t* bars = (uint64_t*)(sm + BAR_OFF);
  uint64_t *bar_q = bars, *bar_k = bars + 1, *bar_v = bars + 3, *bar_s = bars + 5, *bar_o = bars + 7;
  uint32_t* tslot = (uint32_t*)(bars + 9);
  volatile int* abort_flag = (volatile int*)(tslot + 1);

  const int tid = threadIdx.x, warp = tid >> 5;
  const int q0 = blockIdx.x * BM, h = blockIdx.y, b = blockIdx.z;
  const int row = q0 + tid;
  int nkv = p.T / BN;
  if (p.causal) nkv = min(nkv, (q0 + BM) / BN);

  if (tid == 0) {
    for (int i = 0; i < 9; ++i) mbar_init(bars + i, 1);
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
  const uint32_t id_s = idesc_tf32(BM, BN, 0, 0), id_o = idesc_tf32(BM, HD, 0, 1);

  if (tid == 0) {
    mbar_expect_tx(bar_q, BM * HD * 4);
    load_tile(sQ, &mQ, bar_q, BM, q0, h, b);
    for (int i = 0; i < 2 && i < nkv; ++i) {
      mbar_expect_tx(&bar_k[i], TILE);
      load_tile(sK(i), &mK, &bar_k[i], BN, i * BN, h, b);
      mbar_expect_tx(&bar_v[i], TILE);
      load_tile(sV(i), &mV, &bar_v[i], BN, i * BN, h, b);
    }
    if (mbar_wait(bar_q, 0, abort_flag, err, 11) && mbar_wait(&bar_k[0], 0, abort_flag, err, 12)) {
      fence_after();
      issue_mma_k64(tmem, smem_u32(sQ), BM, smem_u32(sK(0)), BN, false, id_s, false);
      mma_commit(&bar_s[0]);
    }
  }
  const float scale2 = p.scale * kLog2e;
  float o[HD];
#pragma unroll
  for (int c = 0; c < HD; ++c) o[c] = 0.f;
  float m = -INFINITY, l = 0.f, alpha_prev = 0.f;
  bool done = true;
  for (int j = 0; j < nkv; ++j) {
    const int sb = j & 1;
    const uint32_t ph = (uint32_t)(j >> 1) & 1u;
    mbar_wait(&bar_s[sb], ph, abort_flag, err, 13);
    __syncthreads();
    if (*abort_flag) { done = false; break; }
    fence_after();
    float x[BN];
    tmem_ld64(tmem + lane + (uint32_t)(sb * 64), x);
    if (tid == 0) {
      // S_{j+1} into the other buffer: P_{j-1} there was consumed by O_{j-1},
      // issued earlier by this thread (tcgen05 MMAs run in issue order)
      if (j + 1 < nkv) {
        const int nb = sb ^ 1;
        if (mbar_wait(&bar_k[nb], (uint32_t)((j + 1) >> 1) & 1u, abort_flag, err, 12)) {
          issue_mma_k64(tmem + (uint32_t)(nb * 64), smem_u32(sQ), BM, smem_u32(sK(nb)), BN, false, id_s, false);
          mma_commit(&bar_s[nb]);
        }
      }
      // S_j has read K_j: its buffer takes K_{j+2}
      if (j + 2 < nkv) {
        mbar_expect_tx(&bar_k[sb], TILE);
        load_tile(sK(sb), &mK, &bar_k[sb], BN, (j + 2) * BN, h, b);
      }
    }
    float mx = m;
#pragma unroll
    for (int c = 0; c < BN; ++c) {
      x[c] *= scale2;
      if (p.causal && j * BN + c > row) x[c] = -INFINITY;
      mx = fmaxf(mx, x[c]);
    }
    const float alpha = ex2(m - mx);
    float rs = 0.f;
#pragma unroll
    for (int c = 0; c < BN; ++c) {
      x[c] = rna_tf32(ex2(x[c] - mx));
      rs += x[c];
    }
    l = l * alpha + rs;
    m = mx;
#pragma unroll
    for (int c = 0; c < BN; c += 16) tmem_st16(tmem + lane + (uint32_t)(sb * 64 + c), x + c);
    tmem_wait_st();
    fence_before();
    __syncthreads();
    if (tid == 0) {
      fence_after();
      if (mbar_wait(&bar_v[sb], ph, abort_flag, err, 14)) {
#pragma unroll
        for (int kk = 0; kk < BN / 8; ++kk)
          mma_tf32_ts(tmem + 128 + (uint32_t)(sb * 64), tmem + (uint32_t)(sb * 64 + kk * 8),
                      desc_mnmajor(smem_u32(sV(sb)), BN, kk), id_o, kk > 0 ? 1u : 0u);
        mma_commit(&bar_o[sb]);
      }
    }
    if (j > 0) {
      // fold O_{j-1} (relative to the max after tile j-1) into the output
      const int pb = sb ^ 1;
      if (!mbar_wait(&bar_o[pb], (uint32_t)((j - 1) >> 1) & 1u, abort_flag, err, 15)) { done = false; }
      fence_after();
      float ob[HD];
      tmem_ld64(tmem + lane + 128 + (uint32_t)(pb * 64), ob);
#pragma unroll
      for (int c = 0; c < HD; ++c) o[c] = o[c] * alpha_prev + ob[c];
      // O_{j-1} has read V_{j-1}: its buffer takes V_{j+1}
      if (tid == 0 && j + 1 < nkv) {
        mbar_expect_tx(&bar_v[pb], TILE);
        load_tile(sV(pb), &mV, &bar_v[pb], BN, (j + 1) * BN, h, b);
      }
    }
    alpha_prev = alpha;
  }
  if (done && nkv > 0) {
    const int pb = (nkv - 1) & 1;
    mbar_wait(&bar_o[pb], (uint32_t)((nkv - 1) >> 1) & 1u, abort_flag, err, 15);
  }
  __syncthreads();
  done = done && !*abort_flag;
  if (done) {
    fence_after();
    float ob[HD];
    tmem_ld64(tmem + lane + 128 + (uint32_t)(((nkv - 1) & 1) * 64), ob);
    const float inv = 1.f / l;
#pragma unroll
    for (int c = 0; c < HD; ++c) {
      o[c] = (o[c] * alpha_prev + ob[c]) * inv;
      if (p.round_out) o[c] = rna_tf32(o[c]);
    }
    // every S MMA has completed: Q's buffer stages the Y block for two TMA stores
    st_row_kmajor(sQ, BM, tid, o);
    fence_proxy_async();
    p.stats[((size_t)b * p.H + h) * p.T + row] = m + log2f(l);
  }
  fence_before();
  __syncthreads();
  if (done && tid == 0) {
    tma_store_4d(&mY, sQ, 0, q0, h, b);
    tma_store_4d(&mY, sQ + BM * 128, 32, q0, h, b);
    bulk_commit();
    bulk_wait_all();
  }
  if (warp == 0) {
    fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

// ---------------------------------------------------------------- backward, dQ
namespace bq {
constexpr int BM = 128, BN = 64;
// Q (reused to stage dQ) and dY blocks, K_j and V_j K-major, K_j MN-major
constexpr int Q_OFF = 0, DO_OFF = 32768, KK_OFF = 65536, VK_OFF = 81920, KM_OFF = 98304, BAR_OFF = 114688;
constexpr int SMEM = BAR_OFF + 256;
// TMEM: S, then dS in place, 0..63; dP 64..127; dQ 128..191
constexpr uint32_t TMEM_COLS = 256;
}  // namespace bq

// Two CTAs per SM: dS is written back over S in TMEM and read from there by
// the dQ MMA, so the CTA needs no shared-memory tile for it.
__global__ void __launch_bounds__(kThreads, 2)
    attn_bwd_q(const __grid_constant__ CUtensorMap mQ, const __grid_constant__ CUtensorMap mDO,
               const __grid_constant__ CUtensorMap mK, const __grid_constant__ CUtensorMap mKm,
               const __grid_constant__ CUtensorMap mV, const __grid_constant__ CUtensorMap mDQ, const Params p,
               int* err) {
  pdl_prologue();
  using namespace bq;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  if (smem_u32(smem_raw) & 1023u) {
    if (threadIdx.x == 0) atomicExch(err, 20);
    return;
  }
  uint8_t* sm = smem_raw;
  uint8_t *sQ = sm + Q_OFF, *sDO = sm + DO_OFF, *sK = sm + KK_OFF, *sV = sm + VK_OFF, *sKm = sm + KM_OFF;
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
  // D = rowsum(dY * Y) of this thread's row: computed in the first iteration,
  // while the first S / dP MMAs run
  float D = 0.f;
  const float L2 = p.lse[b * p.l_sb + h * p.l_sh + row * p.l_st];
  const float scale2 = p.scale * kLog2e;
  const uint32_t id_s = idesc_tf32(BM, BN, 0, 0), id_q = idesc_tf32(BM, HD, 0, 1);
  bool done = true;
  for (int j = 0; j < nkv; ++j) {
    const uint32_t ph = (uint32_t)j & 1u;
    if (tid == 0) {
      if ((j > 0 || mbar_wait(bar_q, 0, abort_flag, err, 21)) && mbar_wait(bar_kv, ph, abort_flag, err, 22)) {
        fence_after();
        // S_j overwrites dS_{j-1}, read by the dQ MMA of block j-1 issued before it
        issue_mma_k64(tmem, smem_u32(sQ), BM, smem_u32(sK), BN, false, id_s, false);
        issue_mma_k64(tmem + 64, smem_u32(sDO), BM, smem_u32(sV), BN, false, id_s, false);
        mma_commit(bar_s);
      }
    }
    if (j == 0) {
      const float* yr = p.y + b * p.y_sb + h * p.y_sh + row * p.y_st;
      const float* dr = p.dy + b * p.dy_sb + h * p.dy_sh + row * p.dy_st;
#pragma unroll 4
      for (int c = 0; c < HD; c += 4) {
        const float4 a = *(const float4*)(yr + c), g = *(const float4*)(dr + c);
        D += a.x * g.x + a.y * g.y + a.z * g.z + a.w * g.w;
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
      const float pr = masked ? 0.f : ex2(s[c] * scale2 - L2);
      s[c] = rna_tf32(pr * (dp[c] - D) * p.scale);
    }
#pragma unroll
    for (int c = 0; c < BN; c += 16) tmem_st16(tmem + lane + (uint32_t)c, s + c);
    tmem_wait_st();
    fence_before();
    __syncthreads();
    if (tid == 0) {
      fence_after();
      if (mbar_wait(bar_km, ph, abort_flag, err, 24)) {
#pragma unroll
        for (int kk = 0; kk < BN / 8; ++kk)
          mma_tf32_ts(tmem + 128, tmem + (uint32_t)(kk * 8), desc_mnmajor(smem_u32(sKm), BN, kk), id_q,
                      (j > 0 || kk > 0) ? 1u : 0u);
        if (j + 1 == nkv) mma_commit(bar_dq);
      }
    }
  }
  if (done) mbar_wait(bar_dq, 0, abort_flag, err, 25);
  __syncthreads();
  done = done && !*abort_flag;
  if (done) {
    fence_after();
    float dq[HD];
    tmem_ld64(tmem + lane + 128, dq);
    if (p.round_out) {
#pragma unroll
      for (int c = 0; c < HD; ++c) dq[c] = rna_tf32(dq[c]);
    }
    // every S MMA has completed: Q's buffer stages the dQ block
    st_row_kmajor(sQ, BM, tid, dq);
    fence_proxy_async();
    p.stats[((size_t)b * p.H + h) * p.T + row] = D;
  }
  fence_before();
  __syncthreads();
  if (done && tid == 0) {
    tma_store_4d(&mDQ, sQ, 0, q0, h, b);
    tma_store_4d(&mDQ, sQ + BM * 128, 32, q0, h, b);
    bulk_commit();
    bulk_wait_all();
  }
  if (warp == 0) {
    fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

// ---------------------------------------------------------------- backward, dK dV
namespace bkv {
constexpr int BN = 128, BQ = 32;
// K and V blocks (BN x 64, K-major; reused to stage dK and dV), Q_i and dY_i
// K-major and MN-major (BQ x 64 each), L_i and D_i
constexpr int K_OFF = 0, V_OFF = 32768, QK_OFF = 65536, DOK_OFF = 73728, QM_OFF = 81920, DOM_OFF = 90112,
              LD_OFF = 98304, BAR_OFF = 98560;
constexpr int SMEM = BAR_OFF + 256;
constexpr int QTILE = BQ * HD * 4;
// TMEM: S^T then P^T 0..31, dP^T then dS^T 32..63, dV 64..127, dK 128..191
constexpr uint32_t TMEM_COLS = 256;
}  // namespace bkv

// Two CTAs per SM: 32-query steps keep the Q_i / dY_i tiles small, and P^T
// and dS^T are written back over S^T and dP^T in TMEM, where the dV and dK
// MMAs read them.
__global__ void __launch_bounds__(kThreads, 2)
    attn_bwd_kv(const __grid_constant__ CUtensorMap mK, const __grid_constant__ CUtensorMap mV,
                const __grid_constant__ CUtensorMap mQ, const __grid_constant__ CUtensorMap mDO,
                const __grid_constant__ CUtensorMap mQm, const __grid_constant__ CUtensorMap mDOm,
                const __grid_constant__ CUtensorMap mDK, const __grid_constant__ CUtensorMap mDV, const Params p,
                int* err) {
  pdl_prologue();
  using namespace bkv;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  if (smem_u32(smem_raw) & 1023u) {
    if (threadIdx.x == 0) atomicExch(err, 30);
    return;
  }
  uint8_t* sm = smem_raw;
  uint8_t *sK = sm + K_OFF, *sV = sm + V_OFF, *sQ = sm + QK_OFF, *sDO = sm + DOK_OFF, *sQm = sm + QM_OFF,
          *sDOm = sm + DOM_OFF;
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
    mbar_expect_tx(bar_a, 2 * QTILE);
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
        // S^T / dP^T overwrite P^T / dS^T of the previous step, read by the dV /
        // dK MMAs issued before them
        issue_mma_k64(tmem, smem_u32(sK), BN, smem_u32(sQ), BQ, false, id_s, false);
        issue_mma_k64(tmem + BQ, smem_u32(sV), BN, smem_u32(sDO), BQ, false, id_s, false);
        mma_commit(bar_s);
      }
    }
    if (tid < BQ) sL[tid] = p.lse[b * p.l_sb + h * p.l_sh + (q0 + tid) * p.l_st];
    else if (tid < 2 * BQ) sD[tid - BQ] = p.dsum[b * p.d_sb + h * p.d_sh + (q0 + tid - BQ) * p.d_st];
    mbar_wait(bar_s, ph, abort_flag, err, 33);
    __syncthreads();
    if (*abort_flag) { done = false; break; }
    fence_after();
    // S^T/dP^T of this step and the dV/dK MMAs of the previous one are done.
    if (tid == 0) {
      mbar_expect_tx(bar_b, 2 * QTILE);
      load_tile(sQm, &mQm, bar_b, BQ, q0, h, b);
      load_tile(sDOm, &mDOm, bar_b, BQ, q0, h, b);
    }
    float s[BQ], dp[BQ];
    {
      uint32_t r[2 * BQ];
      tmem_ld16_async(tmem + lane, r);
      tmem_ld16_async(tmem + lane + 16, r + 16);
      tmem_ld16_async(tmem + lane + 32, r + 32);
      tmem_ld16_async(tmem + lane + 48, r + 48);
      tmem_wait_ld();
#pragma unroll
      for (int c = 0; c < BQ; ++c) {
        s[c] = __uint_as_float(r[c]);
        dp[c] = __uint_as_float(r[BQ + c]);
      }
    }
    if (tid == 0 && it + 1 < nq) {
      mbar_expect_tx(bar_a, 2 * QTILE);
      load_tile(sQ, &mQ, bar_a, BQ, q0 + BQ, h, b);
      load_tile(sDO, &mDO, bar_a, BQ, q0 + BQ, h, b);
    }
#pragma unroll
    for (int c = 0; c < BQ; ++c) {
      const bool masked = p.causal && row > q0 + c;
      const float pr = masked ? 0.f : ex2(s[c] * scale2 - sL[c]);
      s[c] = rna_tf32(pr);
      dp[c] = rna_tf32(pr * (dp[c] - sD[c]) * p.scale);
    }
    tmem_st16(tmem + lane, s);
    tmem_st16(tmem + lane + 16, s + 16);
    tmem_st16(tmem + lane + BQ, dp);
    tmem_st16(tmem + lane + BQ + 16, dp + 16);
    tmem_wait_st();
    fence_before();
    __syncthreads();
    if (tid == 0) {
      fence_after();
      if (mbar_wait(bar_b, ph, abort_flag, err, 34)) {
#pragma unroll
        for (int kk = 0; kk < BQ / 8; ++kk) {
          mma_tf32_ts(tmem + 64, tmem + (uint32_t)(kk * 8), desc_mnmajor(smem_u32(sDOm), BQ, kk), id_g,
                      (it > 0 || kk > 0) ? 1u : 0u);
          mma_tf32_ts(tmem + 128, tmem + (uint32_t)(BQ + kk * 8), desc_mnmajor(smem_u32(sQm), BQ, kk), id_g,
                      (it > 0 || kk > 0) ? 1u : 0u);
        }
        if (it + 1 == nq) mma_commit(bar_o);
      }
    }
  }
  if (done) mbar_wait(bar_o, 0, abort_flag, err, 35);
  __syncthreads();
  done = done && !*abort_flag;
  if (done) {
    // every MMA has completed: the K and V buffers stage dK and dV
    fence_after();
    float g[HD];
    tmem_ld64(tmem + lane + 128, g);
    if (p.round_out) {
#pragma unroll
      for (int c = 0; c < HD; ++c) g[c] = rna_tf32(g[c]);
    }
    st_row_kmajor(sK, BN, tid, g);
    tmem_ld64(tmem + lane + 64, g);
    if (p.round_out) {
#pragma unroll
      for (int c = 0; c < HD; ++c) g[c] = rna_tf32(g[c]);
    }
    st_row_kmajor(sV, BN, tid, g);
    fence_proxy_async();
  }
  fence_before();
  __syncthreads();
  if (done && tid == 0) {
    tma_store_4d(&mDK, sK, 0, k0, h, b);
    tma_store_4d(&mDK, sK + BN * 128, 32, k0, h, b);
    tma_store_4d(&mDV, sV, 0, k0, h, b);
    tma_store_4d(&mDV, sV + BN * 128, 32, k0, h, b);
    bulk_commit();
    bulk_wait_all();
  }
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

// Store map of a [B,T,H,64] output block (dims {64, T, H, B}) whose tokens
// are `ld` elements apart: boxes of 32 columns x `rows` rows of one head,
// 128-byte swizzle (the layout st_row_kmajor writes).
bool out_map(CUtensorMap* m, float* out, int64_t ld, const AttnArgs& a, int rows) {
  const uint64_t dims[4] = {(uint64_t)HD, (uint64_t)a.T, (uint64_t)a.H, (uint64_t)a.B};
  const uint64_t str[3] = {(uint64_t)ld * 4, (uint64_t)HD * 4, (uint64_t)a.T * ld * 4};
  return tc_make_map(m, out, 4, dims, str, (uint32_t)rows, false);
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
  const int64_t n = a.B * a.T * a.H * HD;
  const int64_t ld = a.out_ld ? a.out_ld : a.H * HD;
  if (ld < a.H * HD || ld % 4) return cudaErrorNotSupported;
  float* stats = a.stats ? a.stats : a.out + n;
  float* out_v = a.out_v ? a.out_v : a.out + n;
  if (!aligned16(out_v)) return cudaErrorNotSupported;
  int* err = tc_error_word();
  if (!err) return cudaErrorNotSupported;
  Params p{};
  p.B = (int)a.B;
  p.H = (int)a.H;
  p.T = (int)a.T;
  p.scale = a.scale;
  p.causal = a.causal ? 1 : 0;
  p.round_out = a.round_out ? 1 : 0;
  p.stats = stats;
  const dim3 grid((unsigned)(a.T / 128), (unsigned)a.H, (unsigned)a.B);
  if (a.kind == AttnKind::Fwd) {
    CUtensorMap mq, mk, mv, my;
    if (!map_of(&mq, a.q, a, fwd::BM, false) || !map_of(&mk, a.k, a, fwd::BN, false) ||
        !map_of(&mv, a.v, a, fwd::BN, true) || !out_map(&my, a.out, ld, a, fwd::BM))
      return cudaErrorNotSupported;
    static cudaError_t attr = set_smem(attn_fwd, fwd::SMEM);
    if (attr != cudaSuccess) return attr;
    return launch_pdl(attn_fwd, grid, dim3(kThreads), fwd::SMEM, stream, mq, mk, mv, my, p, err);
  }
  if (!view_ok(a.dy, a) || !a.lse) return cudaErrorNotSupported;
  p.dy = a.dy.p; p.dy_sb = a.dy.sb; p.dy_sh = a.dy.sh; p.dy_st = a.dy.st;
  p.lse = a.lse; p.l_sb = a.l_sb; p.l_sh = a.l_sh; p.l_st = a.l_st;
  if (a.kind == AttnKind::BwdQ) {
    if (!view_ok(a.y, a)) return cudaErrorNotSupported;
    p.y = a.y.p; p.y_sb = a.y.sb; p.y_sh = a.y.sh; p.y_st = a.y.st;
    CUtensorMap mq, mdo, mk, mkm, mv, mdq;
    if (!map_of(&mq, a.q, a, bq::BM, false) || !map_of(&mdo, a.dy, a, bq::BM, false) ||
        !map_of(&mk, a.k, a, bq::BN, false) || !map_of(&mkm, a.k, a, bq::BN, true) ||
        !map_of(&mv, a.v, a, bq::BN, false) || !out_map(&mdq, a.out, ld, a, bq::BM))
      return cudaErrorNotSupported;
    static cudaError_t attr = set_smem(attn_bwd_q, bq::SMEM);
    if (attr != cudaSuccess) return attr;
    return launch_pdl(attn_bwd_q, grid, dim3(kThreads), bq::SMEM, stream, mq, mdo, mk, mkm, mv, mdq, p, err);
  }
  if (a.kind != AttnKind::BwdKV || !a.dsum) return cudaErrorNotSupported;
  p.dsum = a.dsum; p.d_sb = a.d_sb; p.d_sh = a.d_sh; p.d_st = a.d_st;
  CUtensorMap mk, mv, mq, mdo, mqm, mdom, mdk, mdv;
  if (!map_of(&mk, a.k, a, bkv::BN, false) || !map_of(&mv, a.v, a, bkv::BN, false) ||
      !map_of(&mq, a.q, a, bkv::BQ, false) || !map_of(&mdo, a.dy, a, bkv::BQ, false) ||
      !map_of(&mqm, a.q, a, bkv::BQ, true) || !map_of(&mdom, a.dy, a, bkv::BQ, true) ||
      !out_map(&mdk, a.out, ld, a, bkv::BN) || !out_map(&mdv, out_v, ld, a, bkv::BN))
    return cudaErrorNotSupported;
  static cudaError_t attr = set_smem(attn_bwd_kv, bkv::SMEM);
  if (attr != cudaSuccess) return attr;
  return launch_pdl(attn_bwd_kv, grid, dim3(kThreads), bkv::SMEM, stream, mk, mv, mq, mdo, mqm, mdom, mdk, mdv, p,
                    err);
}

}  // namespace sb
