// tcgen05 tensor-core GEMM for sm_100a: C[z] = A[z] @ B[z] with f32 operands in
// global memory read by the tensor cores as TF32 (kind::tf32), or bf16 operands
// (kind::f16 with bf16 A and B), f32 accumulation in TMEM and f32 C.  z is a
// batch index or, for split-K, a K range.  A pipeline stage holds 128 bytes of
// K per operand row either way (32 tf32 or 64 bf16 values), so the shared-
// memory layout, the ring and the epilogue are the same for both.
//
// Persistent: PER_SM CTAs per SM walk the 128 x BN output tiles t = blockIdx.x,
// blockIdx.x + gridDim.x, ... (grouped order, see Tiles, so CTAs that run
// together share A and B tiles in L2).  A launch computes one product or two
// independent ones (GemmGroup: the tiles of the first, then those of the
// second, in the same sequence).  192 threads, warp-specialized:
//   warp 0      TMA producer (one lane): 128B-swizzled K slices of A and B into
//               a STAGES-deep shared-memory ring that runs across tiles,
//               completion via mbarrier transaction bytes;
//   warp 1      MMA issuer (one lane): 4 x tcgen05.mma (K = 8 each) per 32-wide
//               K slice into one of two 128 x BN TMEM accumulators;
//               tcgen05.commit frees ring slots and hands a finished
//               accumulator to the epilogue;
//   warps 2..5  epilogue: tcgen05.ld 32x32b from the four TMEM lane quadrants,
//               optional TF32 rounding, predicated stores to C, then release
//               the accumulator.  With two accumulators the epilogue of tile i
//               overlaps the main loop of tile i + 1.
// Operands may be K-major or MN-major (the transpose bits of the instruction
// descriptor), so x @ W^T, G @ W and X^T @ G all run without transposing copies.
// Every mbarrier wait is bounded (globaltimer); on expiry the CTA records an
// error code, stops issuing work, frees its TMEM and exits.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <mutex>

#include "kernels.h"
#include "pdl.h"
#include "tc_common.h"

namespace sb {

PFN_cuTensorMapEncodeTiled_v12000 encode_fn();

namespace {

constexpr int BM = 128;
constexpr int BK = 32;                       // f32 elements = 128 bytes: one swizzle row
constexpr int kThreads = 192;

using namespace tc;

__device__ __forceinline__ void tma_ld(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y, int z, bool is3d) {
  if (is3d) tma_load_3d(dst, map, bar, x, y, z);
  else tma_load_2d(dst, map, bar, x, y);
}

// MN-major operand through a chunked map (dims {32, K, MN/32[, batch]}): one
// load brings all 32-wide chunks of a stage, laid out BK * 128 B apart.
__device__ __forceinline__ void tma_ld_chunks(void* dst, const CUtensorMap* map, uint64_t* bar, int k, int chunk0,
                                              int z, bool batched) {
  if (batched) tma_load_4d(dst, map, bar, 0, k, chunk0, z);
  else tma_load_3d(dst, map, bar, 0, k, chunk0);
}

template <int BN, int STAGES>
struct Smem {
  static constexpr int A_BYTES = BM * BK * 4;
  static constexpr int B_BYTES = BN * BK * 4;
  static constexpr int STAGE = A_BYTES + B_BYTES;
  // two 32 x 16 f32 staging buffers per epilogue warp
  static constexpr int EPI_BYTES = 4 * 2 * 32 * 16 * 4;
  // the dynamic shared memory window is 1024-byte aligned (checked at entry),
  // so PER_SM CTAs of every configuration fit in an SM's 228 KB
  static constexpr int BYTES = STAGES * STAGE + EPI_BYTES + 256;
};

// Tile t -> (z, m, n).  Within a slice z, tiles run in groups of kGroupM
// M-tiles, column by column, so the ~148 tiles in flight cover a kGroupM x ~18
// block of C and re-read A and B from L2 rather than HBM.
constexpr int kGroupM = 8;
struct Tiles {
  int m_tiles, n_tiles, per_z, total;
  int bm;  // tile height: 128 (one CTA) or 256 (CTA pair)
  __device__ void at(int t, int* z, int* m0, int* n0, int bn) const {
    *z = t / per_z;
    const int r = t - *z * per_z;
    const int gsz = kGroupM * n_tiles;
    const int g = r / gsz, rr = r - g * gsz;
    const int mf = g * kGroupM;
    const int gm = min(kGroupM, m_tiles - mf);
    *m0 = (mf + rr % gm) * bm;
    *n0 = (rr / gm) * bn;
  }
};

// One product of a launch: its operand and store maps and the scalars the
// three roles read (C = C2's layout; kchunk in K steps, 0 when not split).
struct GemmProblem {
  CUtensorMap tmA, tmB, tmC, tmC2;
  float* C;
  float* C2;
  long long scb, ldc;
  int M, N, K;
  int a_mn, b_mn, a3d, b3d, a_chunks, b_chunks, c_tma, c3d, round_out, kchunk, epi, round_out2;
  Tiles tl;
};

// The products of one launch: the tiles of problem 0, then those of problem
// 1, as one persistent tile sequence, so that independent GEMMs (a layer's
// dX and dW in a backward pass) fill the SMs together and cost one launch.
// Every problem has the same store path (all TMA stores or none), so a warp's
// staging buffers are never written by plain stores while a TMA store of the
// other problem still reads them.
// NP = 1 for a single product: the kernel then indexes a constant problem
// (parameters read as directly as scalar kernel arguments) and takes a
// parameter block of one problem.
template <int NP>
struct GemmGroup {
  GemmProblem p[NP];
  int count;
  int start[NP + 1];  // first tile of problem q; start[count] = all tiles
};

// Tile t of a group: problem q, output slice z, tile origin (m0, n0), K steps
// [kt0, kt1) and the operand slice zab that the loads address (0 for a split
// product, whose slices are K ranges of one operand pair).
struct TileAt {
  int q, z, m0, n0, kt0, kt1, zab;
};
template <int BKE, int NP>
__device__ __forceinline__ TileAt locate(const GemmGroup<NP>& g, int t, int bn) {
  TileAt a;
  a.q = (NP > 1 && t >= g.start[NP > 1 ? 1 : 0]) ? 1 : 0;
  const GemmProblem& P = g.p[a.q];
  P.tl.at(t - g.start[a.q], &a.z, &a.m0, &a.n0, bn);
  const int ktiles = (P.K + BKE - 1) / BKE;
  a.kt0 = 0;
  a.kt1 = ktiles;
  a.zab = a.z;
  if (P.kchunk > 0) {
    a.kt0 = a.z * P.kchunk;
    a.kt1 = min(a.kt0 + P.kchunk, ktiles);
    a.zab = 0;
  }
  return a;
}

// Epilogue store of a 32-row x 16-column chunk held one row per lane (v =
// columns col0..col0+15 of row row0 + lane).  The warp passes it through its
// 2 KB shared-memory slot so that each store instruction writes 8 rows x 64
// contiguous bytes instead of 32 rows x 16 bytes (the row-per-lane stores ran
// at ~1.5 TB/s).  16-byte units are XOR-swizzled by (row >> 1) & 3: both the
// row-wise writes and the column-wise reads are bank-conflict free.
__device__ __forceinline__ void store_chunk(float* slot, const float* v, int lane, float* C, int row0, int col0, int M,
                                            int N, long long ldc, bool vec) {
#pragma unroll
  for (int u = 0; u < 4; ++u)
    ((float4*)(slot + lane * 16))[u ^ ((lane >> 1) & 3)] = make_float4(v[4 * u], v[4 * u + 1], v[4 * u + 2], v[4 * u + 3]);
  __syncwarp();
  const int sub = lane >> 2, u = lane & 3, col = col0 + 4 * u;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int r = 8 * k + sub, row = row0 + r;
    const float4 x = ((const float4*)(slot + r * 16))[u ^ ((r >> 1) & 3)];
    if (row < M) {
      float* dst = C + (long long)row * ldc + col;
      if (vec && col + 4 <= N) {
        *(float4*)dst = x;
      } else {
        if (col < N) dst[0] = x.x;
        if (col + 1 < N) dst[1] = x.y;
        if (col + 2 < N) dst[2] = x.z;
        if (col + 3 < N) dst[3] = x.w;
      }
    }
  }
  __syncwarp();
}

// Orders uses of registers written by an asynchronous tcgen05.ld after the
// tcgen05.wait::ld that completes it.
__device__ __forceinline__ void reg_fence16(uint32_t* r) {
#pragma unroll
  for (int i = 0; i < 16; ++i) asm volatile("" : "+r"(r[i]));
}

// Second output of the fused epilogue (Epi::epi == kEpiGelu): C2 = gelu(C).
struct Epi {
  const CUtensorMap* tm = nullptr;  // store map of C2 (when c_tma)
  float* c = nullptr;               // C2 of this output slice
  int epi = 0;
  int round_out = 0;
};

// One 32 x 16 chunk of values (one row per lane) to C: through the warp's
// double-buffered staging tile and a TMA store, or by plain stores.
__device__ __forceinline__ void store_chunk16(const float* v, float* bufs, int lane, int* sb, const CUtensorMap* tmC,
                                              bool c_tma, bool c3d, int z, float* cz, int row0, int n, int M, int N,
                                              long long ldc, bool vec) {
  if (c_tma) {
    float* buf = bufs + *sb * 512;
    if (lane == 0) bulk_wait_read1();
    __syncwarp();
#pragma unroll
    for (int u = 0; u < 4; ++u)
      ((float4*)(buf + lane * 16))[u ^ ((lane >> 1) & 3)] = make_float4(v[4 * u], v[4 * u + 1], v[4 * u + 2], v[4 * u + 3]);
    fence_proxy_async();
    __syncwarp();
    if (lane == 0) {
      if (c3d) tma_store_3d(tmC, buf, n, row0, z);
      else tma_store_2d(tmC, buf, n, row0);
      bulk_commit();
    }
    *sb ^= 1;
  } else {
    store_chunk(bufs, v, lane, cz, row0, n, M, N, ldc, vec);
  }
}

// One 16-column chunk of this warp's 32 accumulator rows to C (optionally
// rounded to TF32) and, with the fused epilogue, gelu of the same values to
// C2 (gelu of the accumulator, before any rounding of C).
__device__ __forceinline__ void epilogue_chunk(const uint32_t* r, float* bufs, int lane, int* sb,
                                               const CUtensorMap* tmC, bool c_tma, bool c3d, int z, float* cz,
                                               int row0, int n, int M, int N, long long ldc, bool vec, bool zero,
                                               int round_out, const Epi& e2) {
  float v[16];
#pragma unroll
  for (int q = 0; q < 16; ++q) {
    v[q] = zero ? 0.f : __uint_as_float(r[q]);
    if (round_out) v[q] = rna_tf32(v[q]);
  }
  store_chunk16(v, bufs, lane, sb, tmC, c_tma, c3d, z, cz, row0, n, M, N, ldc, vec);
  if (e2.epi == kEpiGelu) {
#pragma unroll
    for (int q = 0; q < 16; ++q) {
      v[q] = gelu_tanh_f(zero ? 0.f : __uint_as_float(r[q]));
      if (e2.round_out) v[q] = rna_tf32(v[q]);
    }
    store_chunk16(v, bufs, lane, sb, e2.tm, c_tma, c3d, z, e2.c, row0, n, M, N, ldc, vec);
  }
}

// Epilogue of one warp's 32 accumulator rows (TMEM lane quadrant at `acc`) to
// rows row0..row0+31, columns n0..n0+BN-1 of output slice z.  With a C tensor
// map (c_tma) each 32 x 16 chunk is staged in one of the warp's two 2 KB
// buffers (64-byte swizzle) and lane 0 issues a TMA store for it, so the
// stores drain asynchronously; a buffer is rewritten only after the store
// issued from it two chunks earlier has read it.  Without a map (row stride
// or base not 16-byte aligned) store_chunk writes through the first buffer.
// Software pipelined: the TMEM load of the next 16 columns is in flight while
// the current ones are staged and stored.
template <int BN>
__device__ __forceinline__ void epilogue_warp(uint32_t acc, float* bufs, int lane, int* sb, const CUtensorMap* tmC,
                                              bool c_tma, bool c3d, int z, float* cz, int row0, int n0, int M, int N,
                                              long long ldc, bool vec, bool zero, int round_out, const Epi& e2) {
  if (row0 >= M || n0 >= N) return;
  uint32_t r0[16], r1[16];
  tmem_ld16_async(acc, r0);
  tmem_wait_ld();
  reg_fence16(r0);
#pragma unroll 1
  for (int c = 0; c < BN && n0 + c < N; c += 32) {
    const bool has1 = c + 16 < BN && n0 + c + 16 < N;
    const bool has2 = c + 32 < BN && n0 + c + 32 < N;
    if (has1) tmem_ld16_async(acc + (uint32_t)(c + 16), r1);
    epilogue_chunk(r0, bufs, lane, sb, tmC, c_tma, c3d, z, cz, row0, n0 + c, M, N, ldc, vec, zero, round_out, e2);
    if (!has1) break;
    tmem_wait_ld();
    reg_fence16(r1);
    if (has2) tmem_ld16_async(acc + (uint32_t)(c + 32), r0);
    epilogue_chunk(r1, bufs, lane, sb, tmC, c_tma, c3d, z, cz, row0, n0 + c + 16, M, N, ldc, vec, zero, round_out,
                   e2);
    if (!has2) break;
    tmem_wait_ld();
    reg_fence16(r0);
  }
}

// Descriptor of an MN-major operand tile at `addr`: chunks of 128-byte rows
// (one row per K value), 32 f32 or 64 bf16 M/N values wide, BK rows deep per
// chunk (4096 / 8192 bytes apart: the leading byte offset).  tf32: the 128-byte
// swizzle with 32-byte atoms, 4-row groups 512 B apart; bf16: the plain
// 128-byte swizzle, 8-row groups 1024 B apart (stride byte offset).
template <bool BF>
__device__ __forceinline__ uint64_t mn_desc(uint32_t addr) {
  return BF ? smem_desc(addr, 64 * 128, 1024, 2) : smem_desc(addr, BK * 128, 512, 1);
}
// start-address step (16-byte units) between the 4 MMAs of a stage on an
// MN-major tile: 8 rows (tf32, K = 8) or 16 rows (bf16, K = 16) of 128 B
template <bool BF>
constexpr uint64_t kMnStep = BF ? (2048 >> 4) : (1024 >> 4);

// TMEM allocations are powers of two of at least 32 columns.
__host__ __device__ constexpr uint32_t tmem_cols(int n) { return n <= 32 ? 32u : n <= 64 ? 64u : n <= 128 ? 128u : n <= 256 ? 256u : 512u; }

template <bool BF, int BN, int STAGES, int PER_SM, int ACC, int NP>
__global__ void __launch_bounds__(kThreads, PER_SM)
    gemm_tcgen05_kernel(const __grid_constant__ GemmGroup<NP> grp, int* err) {
  using S = Smem<BN, STAGES>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  pdl_prologue();
  if (smem_u32(smem_raw) & 1023u) {  // uniform: every thread leaves before any barrier
    if (threadIdx.x == 0) atomicExch(err, 9);
    return;
  }
  uint8_t* smem = smem_raw;
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * S::A_BYTES;
  float* epi_buf = (float*)(smem + STAGES * S::STAGE);
  uint64_t* full = (uint64_t*)(smem + STAGES * S::STAGE + S::EPI_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;   // [2]: MMA -> epilogue
  uint64_t* acc_empty = acc_full + 2;    // [2]: epilogue -> MMA (128 arrivals)
  uint32_t* tmem_slot = (uint32_t*)(acc_empty + 2);
  volatile int* abort_flag = (volatile int*)(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // K values per 128-byte stage row (also M/N values per 128-byte row of an
  // MN-major tile): 32 f32 or 64 bf16
  constexpr int BKE = BF ? 64 : 32;
  constexpr uint32_t TMEM_COLS = tmem_cols(ACC * BN);
  const int total = grp.start[NP];

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 128);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    fence_proxy_async();
  }
  if (warp == 1) tmem_alloc(tmem_slot, TMEM_COLS);
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ring position: slot s, phase ph (advanced after each K step)
      int it = 0, s = 0;
      uint32_t ph = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
        const TileAt at = locate<BKE, NP>(grp, t, BN);
        // this problem's operand description, read once per tile (not per K step)
        const GemmProblem& P = grp.p[at.q];
        const CUtensorMap* tA = &P.tmA;
        const CUtensorMap* tB = &P.tmB;
        const int a_mn = P.a_mn, b_mn = P.b_mn, a_chunks = P.a_chunks, b_chunks = P.b_chunks;
        const bool a3d = P.a3d, b3d = P.b3d;
        for (int kt = at.kt0; kt < at.kt1; ++kt, ++it) {
          if (it >= STAGES && !mbar_wait(&empty[s], ph ^ 1u, abort_flag, err, 1)) { ok = false; break; }
          mbar_expect_tx(&full[s], (uint32_t)S::STAGE);
          uint8_t* a = sA + s * S::A_BYTES;
          uint8_t* b = sB + s * S::B_BYTES;
          if (!a_mn) {
            tma_ld(a, tA, &full[s], kt * BKE, at.m0, at.zab, a3d);
          } else if (a_chunks) {
            tma_ld_chunks(a, tA, &full[s], kt * BKE, at.m0 / BKE, at.zab, a3d);
          } else {
#pragma unroll
            for (int j = 0; j < BM / BKE; ++j)
              tma_ld(a + j * BKE * 128, tA, &full[s], at.m0 + BKE * j, kt * BKE, at.zab, a3d);
          }
          if (!b_mn) {
            tma_ld(b, tB, &full[s], kt * BKE, at.n0, at.zab, b3d);
          } else if (b_chunks) {
            tma_ld_chunks(b, tB, &full[s], kt * BKE, at.n0 / BKE, at.zab, b3d);
          } else {
#pragma unroll
            for (int j = 0; j < BN / BKE; ++j)
              tma_ld(b + j * BKE * 128, tB, &full[s], at.n0 + BKE * j, kt * BKE, at.zab, b3d);
          }
          if (++s == STAGES) { s = 0; ph ^= 1u; }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int it = 0, j = 0, s = 0;
      uint32_t ph = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x, ++j) {
        const TileAt at = locate<BKE, NP>(grp, t, BN);
        const GemmProblem& P = grp.p[at.q];
        const uint32_t idesc = BF ? idesc_bf16(BM, BN, P.a_mn, P.b_mn) : idesc_tf32(BM, BN, P.a_mn, P.b_mn);
        // descriptors of slot 0, K slice 0 (see the CTA-pair kernel)
        const uint64_t a_d0 = P.a_mn ? mn_desc<BF>(smem_u32(sA)) : smem_desc(smem_u32(sA), 16, 1024, 2);
        const uint64_t b_d0 = P.b_mn ? mn_desc<BF>(smem_u32(sB)) : smem_desc(smem_u32(sB), 16, 1024, 2);
        const uint64_t a_kk = P.a_mn ? kMnStep<BF> : 32 >> 4, b_kk = P.b_mn ? kMnStep<BF> : 32 >> 4;
        const int b = ACC == 2 ? (j & 1) : 0, use = ACC == 2 ? (j >> 1) : j;
        if (use > 0 && !mbar_wait(&acc_empty[b], (uint32_t)(use - 1) & 1u, abort_flag, err, 4)) break;
        fence_after();
        const uint32_t acc = tmem + (uint32_t)(b * BN);
        for (int kt = at.kt0; kt < at.kt1; ++kt, ++it) {
          if (!mbar_wait(&full[s], ph, abort_flag, err, 2)) { ok = false; break; }
          fence_after();
          // K-major: rows of 128 B (32 K values), 8-row swizzle atoms 1024 B apart; the
          // k-th MMA starts 32 B further along the row.  MN-major: 128 B (32 M/N
          // values) by BK rows per chunk, chunks BK*128 B apart (LBO), 4-row
          // atoms 512 B apart (SBO); the k-th MMA starts 8 rows (1024 B) down.
          const uint64_t ad = a_d0 + (uint64_t)((s * S::A_BYTES) >> 4);
          const uint64_t bd = b_d0 + (uint64_t)((s * S::B_BYTES) >> 4);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            if (BF) mma_bf16(acc, ad + kk * a_kk, bd + kk * b_kk, idesc, (kt > at.kt0 || kk > 0) ? 1u : 0u);
            else mma_tf32(acc, ad + kk * a_kk, bd + kk * b_kk, idesc, (kt > at.kt0 || kk > 0) ? 1u : 0u);
          }
          mma_commit(&empty[s]);
          if (++s == STAGES) { s = 0; ph ^= 1u; }
        }
        if (!ok) break;
        mma_commit(&acc_full[b]);
      }
    }
  } else {
    // epilogue warps 2..5: TMEM lane quadrant = warp % 4
    const int quad = warp & 3;
    int j = 0, sb = 0;
    for (int t = blockIdx.x; t < total; t += gridDim.x, ++j) {
      const TileAt at = locate<BKE, NP>(grp, t, BN);
      const GemmProblem& P = grp.p[at.q];
      const int b = ACC == 2 ? (j & 1) : 0, use = ACC == 2 ? (j >> 1) : j;
      if (!mbar_wait(&acc_full[b], (uint32_t)use & 1u, abort_flag, err, 3)) break;
      fence_after();
      const int row0 = at.m0 + quad * 32;
      float* cz = P.C + (long long)at.z * P.scb;
      const bool vec = (P.ldc & 3) == 0 && (((uintptr_t)cz) & 15) == 0;
      const uint32_t acc = tmem + (uint32_t)(b * BN) + ((uint32_t)(quad * 32) << 16);
      Epi e2;
      e2.tm = &P.tmC2;
      e2.c = P.C2 + (long long)at.z * P.scb;
      e2.epi = P.epi;
      e2.round_out = P.round_out2;
      epilogue_warp<BN>(acc, epi_buf + (warp - 2) * 1024, lane, &sb, &P.tmC, P.c_tma, P.c3d, at.z, cz, row0, at.n0,
                        P.M, P.N, P.ldc, vec, at.kt1 <= at.kt0, P.round_out, e2);
      fence_before();
      mbar_arrive(&acc_empty[b]);
    }
    if (lane == 0) bulk_wait_all();
  }
  fence_before();
  __syncthreads();
  if (warp == 1) {
    fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

// CTA-pair variant: a cluster of two CTAs computes a 256 x BN tile with
// tcgen05.mma.cta_group::2.  Each CTA loads its 128 rows of A and BN/2 columns
// of B into its own shared memory (pair TMA loads count their bytes on the
// leader's full barrier); the leader's MMA thread issues the pair MMA, which
// reads both CTAs' tiles and accumulates rows 0..127 into the leader's TMEM and
// rows 128..255 into the peer's.  Per SM this moves 25% (BN = 128) or 50%
// (BN = 256) fewer operand bytes per FLOP than the 128 x 128 single-CTA tile.
// Completion is signalled to both CTAs with one non-multicast commit each; the
// peer's epilogue releases an accumulator with a remote mbarrier arrive.
template <bool BF, int BN, int STAGES, int PER_SM, int ACC, int NP>
__global__ void __launch_bounds__(kThreads, PER_SM)
    gemm_tcgen05_pair(const __grid_constant__ GemmGroup<NP> grp, int* err) {
  constexpr int BNH = BN / 2;
  using S = Smem<BNH, STAGES>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  pdl_prologue();
  // both CTAs of a pair have the same layout, so both leave here or neither
  if (smem_u32(smem_raw) & 1023u) {
    if (threadIdx.x == 0) atomicExch(err, 9);
    return;
  }
  uint8_t* smem = smem_raw;
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * S::A_BYTES;
  float* epi_buf = (float*)(smem + STAGES * S::STAGE);
  uint64_t* full = (uint64_t*)(smem + STAGES * S::STAGE + S::EPI_BYTES);  // leader: both CTAs' bytes
  uint64_t* empty = full + STAGES;                            // each CTA: slot free
  uint64_t* acc_full = empty + STAGES;                        // each CTA: accumulator ready
  uint64_t* acc_empty = acc_full + 2;                         // leader: 256 arrivals
  uint32_t* tmem_slot = (uint32_t*)(acc_empty + 2);
  volatile int* abort_flag = (volatile int*)(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  const int pair = (int)(blockIdx.x >> 1), npairs = (int)(gridDim.x >> 1);
  // K values per 128-byte stage row (also M/N values per 128-byte row of an
  // MN-major tile): 32 f32 or 64 bf16
  constexpr int BKE = BF ? 64 : 32;
  constexpr uint32_t TMEM_COLS = tmem_cols(ACC * BN);
  const int total = grp.start[NP];

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 256);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    fence_proxy_async();
  }
  if (warp == 1) tmem_alloc_pair(tmem_slot, TMEM_COLS);
  fence_before();
  __syncthreads();
  cluster_sync();
  fence_after();
  const uint32_t tmem = *tmem_slot;

  auto ld = [&](void* dst, const CUtensorMap* map, uint32_t bar, int x, int y, int z, bool is3d) {
    if (is3d) tma_load_3d_pair(dst, map, bar, x, y, z);
    else tma_load_2d_pair(dst, map, bar, x, y);
  };
  auto ld_chunks = [&](void* dst, const CUtensorMap* map, uint32_t bar, int k, int chunk0, int z, bool batched) {
    if (batched) tma_load_4d_pair(dst, map, bar, 0, k, chunk0, z);
    else tma_load_3d_pair(dst, map, bar, 0, k, chunk0);
  };

  if (warp == 0) {
    if (lane == 0) {
      // ring position: slot s, phase ph (advanced after each K step)
      int it = 0, s = 0;
      uint32_t ph = 0;
      const uint32_t full_leader = cluster_addr(&full[0], 0);
      bool ok = true;
      for (int t = pair; t < total && ok; t += npairs) {
        const TileAt at = locate<BKE, NP>(grp, t, BN);
        // this problem's operand description, read once per tile (not per K step)
        const GemmProblem& P = grp.p[at.q];
        const CUtensorMap* tA = &P.tmA;
        const CUtensorMap* tB = &P.tmB;
        const int a_mn = P.a_mn, b_mn = P.b_mn, a_chunks = P.a_chunks, b_chunks = P.b_chunks;
        const bool a3d = P.a3d, b3d = P.b3d;
        const int ma = at.m0 + (int)rank * BM, nb = at.n0 + (int)rank * BNH;
        for (int kt = at.kt0; kt < at.kt1; ++kt, ++it) {
          if (it >= STAGES && !mbar_wait(&empty[s], ph ^ 1u, abort_flag, err, 1)) { ok = false; break; }
          if (leader) mbar_expect_tx(&full[s], 2u * (uint32_t)S::STAGE);
          const uint32_t bar = full_leader + (uint32_t)(s * 8);
          uint8_t* a = sA + s * S::A_BYTES;
          uint8_t* b = sB + s * S::B_BYTES;
          if (!a_mn) {
            ld(a, tA, bar, kt * BKE, ma, at.zab, a3d);
          } else if (a_chunks) {
            ld_chunks(a, tA, bar, kt * BKE, ma / BKE, at.zab, a3d);
          } else {
#pragma unroll
            for (int j = 0; j < BM / BKE; ++j) ld(a + j * BKE * 128, tA, bar, ma + BKE * j, kt * BKE, at.zab, a3d);
          }
          if (!b_mn) {
            ld(b, tB, bar, kt * BKE, nb, at.zab, b3d);
          } else if (b_chunks) {
            ld_chunks(b, tB, bar, kt * BKE, nb / BKE, at.zab, b3d);
          } else {
#pragma unroll
            for (int j = 0; j < BNH / BKE; ++j)
              ld(b + j * BKE * 128, tB, bar, nb + BKE * j, kt * BKE, at.zab, b3d);
          }
          if (++s == STAGES) { s = 0; ph ^= 1u; }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      const uint32_t empty0 = cluster_addr(&empty[0], 0), empty1 = cluster_addr(&empty[0], 1);
      int it = 0, j = 0, s = 0;
      uint32_t ph = 0;
      bool ok = true;
      for (int t = pair; t < total && ok; t += npairs, ++j) {
        const TileAt at = locate<BKE, NP>(grp, t, BN);
        const GemmProblem& P = grp.p[at.q];
        const uint32_t idesc = BF ? idesc_bf16(2 * BM, BN, P.a_mn, P.b_mn) : idesc_tf32(2 * BM, BN, P.a_mn, P.b_mn);
        // descriptors of slot 0, K slice 0; a slot adds its byte offset and a
        // K slice 32 B (K-major) or 1024 / 2048 B (MN-major tf32 / bf16), in
        // 16-byte units, to the start-address field (shared addresses stay below
        // 2^18, no carry)
        const uint64_t a_d0 = P.a_mn ? mn_desc<BF>(smem_u32(sA)) : smem_desc(smem_u32(sA), 16, 1024, 2);
        const uint64_t b_d0 = P.b_mn ? mn_desc<BF>(smem_u32(sB)) : smem_desc(smem_u32(sB), 16, 1024, 2);
        const uint64_t a_kk = P.a_mn ? kMnStep<BF> : 32 >> 4, b_kk = P.b_mn ? kMnStep<BF> : 32 >> 4;
        const int b = ACC == 2 ? (j & 1) : 0, use = ACC == 2 ? (j >> 1) : j;
        if (use > 0 && !mbar_wait(&acc_empty[b], (uint32_t)(use - 1) & 1u, abort_flag, err, 4)) break;
        fence_after();
        const uint32_t acc = tmem + (uint32_t)(b * BN);
        for (int kt = at.kt0; kt < at.kt1; ++kt, ++it) {
          if (!mbar_wait(&full[s], ph, abort_flag, err, 2)) { ok = false; break; }
          fence_after();
          const uint64_t ad = a_d0 + (uint64_t)((s * S::A_BYTES) >> 4);
          const uint64_t bd = b_d0 + (uint64_t)((s * S::B_BYTES) >> 4);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            if (BF) mma_bf16_pair(acc, ad + kk * a_kk, bd + kk * b_kk, idesc, (kt > at.kt0 || kk > 0) ? 1u : 0u);
            else mma_tf32_pair(acc, ad + kk * a_kk, bd + kk * b_kk, idesc, (kt > at.kt0 || kk > 0) ? 1u : 0u);
          }
          mma_commit_pair(empty0 + (uint32_t)(s * 8));
          mma_commit_pair(empty1 + (uint32_t)(s * 8));
          if (++s == STAGES) { s = 0; ph ^= 1u; }
        }
        if (!ok) break;
        mma_commit_pair(cluster_addr(&acc_full[b], 0));
        mma_commit_pair(cluster_addr(&acc_full[b], 1));
      }
    }
  } else {
    const int quad = warp & 3;
    int j = 0, sb = 0;
    for (int t = pair; t < total; t += npairs, ++j) {
      const TileAt at = locate<BKE, NP>(grp, t, BN);
      const GemmProblem& P = grp.p[at.q];
      const int b = ACC == 2 ? (j & 1) : 0, use = ACC == 2 ? (j >> 1) : j;
      if (!mbar_wait(&acc_full[b], (uint32_t)use & 1u, abort_flag, err, 3)) break;
      fence_after();
      const int row0 = at.m0 + (int)rank * BM + quad * 32;
      float* cz = P.C + (long long)at.z * P.scb;
      const bool vec = (P.ldc & 3) == 0 && (((uintptr_t)cz) & 15) == 0;
      const uint32_t accp = tmem + (uint32_t)(b * BN) + ((uint32_t)(quad * 32) << 16);
      Epi e2;
      e2.tm = &P.tmC2;
      e2.c = P.C2 + (long long)at.z * P.scb;
      e2.epi = P.epi;
      e2.round_out = P.round_out2;
      epilogue_warp<BN>(accp, epi_buf + (warp - 2) * 1024, lane, &sb, &P.tmC, P.c_tma, P.c3d, at.z, cz, row0, at.n0,
                        P.M, P.N, P.ldc, vec, at.kt1 <= at.kt0, P.round_out, e2);
      fence_before();
      mbar_arrive_cluster(cluster_addr(&acc_empty[b], 0));
    }
    if (lane == 0) bulk_wait_all();
  }
  fence_before();
  __syncthreads();
  cluster_sync();
  if (warp == 1) {
    fence_after();
    tmem_dealloc_pair(tmem, TMEM_COLS);
  }
}

// 2-D or 3-D operand map: inner (contiguous) extent d0, outer d1, batch d2;
// the box is one 128-byte swizzle row wide and box1 rows tall.
bool make_map(CUtensorMap* m, bool bf, const float* base, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t s1_bytes,
              uint64_t s2_bytes, uint32_t box1, bool is3d, bool mn_major) {
  const uint64_t dims[3] = {d0, d1, d2};
  const uint64_t strides[2] = {s1_bytes, s2_bytes};
  if (bf) return tc_make_map_bf16(m, base, is3d ? 3 : 2, dims, strides, box1);
  return tc_make_map(m, base, is3d ? 3 : 2, dims, strides, box1, mn_major);
}

// Chunked map of an MN-major operand (MN values contiguous, rows of K):
// dims {W, K, MN / W[, batch]} with the W-value chunks 128 B apart (W = 32 f32
// or 64 bf16), box {W, BKE, chunks}, so one load fills a stage's chunks
// BKE * 128 B apart.  Only when MN is a multiple of W (the last chunk ends
// inside the row).
bool make_chunk_map(CUtensorMap* m, bool bf, const float* base, uint64_t mn, uint64_t k, uint64_t batch,
                    uint64_t ld_bytes, uint64_t batch_bytes, uint32_t chunks, bool batched) {
  const uint64_t w = bf ? 64 : 32;
  if (mn % w) return false;
  auto enc = encode_fn();
  if (!enc) return false;
  cuuint64_t d[4] = {w, (cuuint64_t)k, (cuuint64_t)(mn / w), (cuuint64_t)batch};
  cuuint64_t st[3] = {(cuuint64_t)ld_bytes, 128, (cuuint64_t)batch_bytes};
  cuuint32_t box[4] = {(cuuint32_t)w, (cuuint32_t)w, chunks, 1}, es[4] = {1, 1, 1, 1};
  return enc(m, bf ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, batched ? 4u : 3u,
             (void*)base, d, st, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
             bf ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Store map of C (f32, inner extent N, rows M, slices `batch`): 32-row x
// 16-column boxes, 64-byte swizzle.  False when the row stride, the slice
// stride or the base is not 16-byte aligned (the epilogue then stores through
// store_chunk).
bool make_store_map(CUtensorMap* m, const GemmArgs& g) {
  if ((g.scm & 3) || (((uintptr_t)g.c) & 15) || (g.batch > 1 && (g.scb & 3))) return false;
  auto enc = encode_fn();
  if (!enc) return false;
  const bool is3d = g.batch > 1;
  cuuint64_t d[3] = {(cuuint64_t)g.N, (cuuint64_t)g.M, (cuuint64_t)g.batch};
  cuuint64_t st[2] = {(cuuint64_t)g.scm * 4, (cuuint64_t)g.scb * 4};
  cuuint32_t box[3] = {16, 32, 1}, es[3] = {1, 1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, is3d ? 3u : 2u, (void*)g.c, d, st, box, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Store maps of C and, with the fused epilogue, of C2 (laid out as C): both
// or neither, so the epilogue uses one store path for the two outputs.
bool store_maps(const GemmArgs& g, CUtensorMap* mc, CUtensorMap* mc2) {
  if (!make_store_map(mc, g)) return false;
  if (!g.epi) return true;
  GemmArgs g2 = g;
  g2.c = g.c2;
  return make_store_map(mc2, g2);
}

int sm_count() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
  }
  return n;
}

// Operand maps of g for a tile of BM_CTA rows of A and BN_CTA columns of B
// per CTA.  false when a map cannot be encoded (the caller reports
// cudaErrorNotSupported).
template <bool BF>
bool operand_maps(const GemmArgs& g, bool a_mn, bool b_mn, int bn_cta, CUtensorMap* ta, CUtensorMap* tb,
                  int* a_chunks, int* b_chunks, bool* a3d, bool* b3d) {
  constexpr int BKE = BF ? 64 : 32;
  constexpr int64_t es = BF ? 2 : 4;
  const int64_t lda = a_mn ? g.sak : g.sam;
  const int64_t ldb = b_mn ? g.sbk : g.sbn;
  const bool split = g.k_chunk > 0;
  *a3d = !split && g.batch > 1 && g.sab != 0;
  *b3d = !split && g.batch > 1 && g.sbb != 0;
  // A: K-major dims {K, M}, box {row, 128}; M-major dims {M, K}, box {row, BKE}
  *a_chunks = a_mn && make_chunk_map(ta, BF, g.a, g.M, g.K, g.batch, lda * es, g.sab * es, BM / BKE, *a3d);
  *b_chunks = b_mn && (bn_cta % BKE == 0) &&
              make_chunk_map(tb, BF, g.b, g.N, g.K, g.batch, ldb * es, g.sbb * es, bn_cta / BKE, *b3d);
  bool ok = *a_chunks || (a_mn ? make_map(ta, BF, g.a, g.M, g.K, g.batch, lda * es, g.sab * es, BKE, *a3d, true)
                                : make_map(ta, BF, g.a, g.K, g.M, g.batch, lda * es, g.sab * es, BM, *a3d, false));
  ok = ok && (*b_chunks || (b_mn ? make_map(tb, BF, g.b, g.N, g.K, g.batch, ldb * es, g.sbb * es, BKE, *b3d, true)
                                  : make_map(tb, BF, g.b, g.K, g.N, g.batch, ldb * es, g.sbb * es, bn_cta, *b3d,
                                             false)));
  return ok;
}

// Problem g of a launch whose tiles are bm_tile x bn_tile with bn_cta columns
// of B loaded per CTA: operand and store maps and scalars.  false when a map
// cannot be encoded or the problem has too many tiles.
template <bool BF>
bool fill_problem(const GemmArgs& g, bool a_mn, bool b_mn, int bn_cta, int bm_tile, int bn_tile, GemmProblem* P) {
  constexpr int BKE = BF ? 64 : 32;
  int a_chunks = 0, b_chunks = 0;
  bool a3d = false, b3d = false;
  if (!operand_maps<BF>(g, a_mn, b_mn, bn_cta, &P->tmA, &P->tmB, &a_chunks, &b_chunks, &a3d, &b3d)) return false;
  P->tmC = P->tmB;  // placeholder contents when C (C2) has no store map
  P->tmC2 = P->tmB;
  P->c_tma = store_maps(g, &P->tmC, &P->tmC2) ? 1 : 0;
  P->C = g.c;
  P->C2 = g.epi ? g.c2 : g.c;
  P->scb = g.scb;
  P->ldc = g.scm;
  P->M = (int)g.M;
  P->N = (int)g.N;
  P->K = (int)g.K;
  P->a_mn = a_mn;
  P->b_mn = b_mn;
  P->a3d = a3d;
  P->b3d = b3d;
  P->a_chunks = a_chunks;
  P->b_chunks = b_chunks;
  P->c3d = g.batch > 1 ? 1 : 0;
  P->round_out = g.round_out;
  P->kchunk = g.k_chunk > 0 ? (int)(g.k_chunk / BKE) : 0;
  P->epi = g.epi;
  P->round_out2 = g.round_out2;
  P->tl.bm = bm_tile;
  P->tl.m_tiles = (int)((g.M + bm_tile - 1) / bm_tile);
  P->tl.n_tiles = (int)((g.N + bn_tile - 1) / bn_tile);
  P->tl.per_z = P->tl.m_tiles * P->tl.n_tiles;
  const int64_t total = (int64_t)P->tl.per_z * g.batch;
  if (total > (1ll << 30)) return false;
  P->tl.total = (int)total;
  return true;
}

// The launch description of problems gs[0..n): their tile ranges one after
// the other, one store path for all (TMA stores only when every problem has
// its store maps).
template <bool BF, int NP>
bool make_group(const GemmArgs* gs, const bool* a_mn, const bool* b_mn, int n, int bn_cta, int bm_tile, int bn_tile,
                GemmGroup<NP>* G) {
  if (n != NP) return false;
  G->count = n;
  G->start[0] = 0;
  bool all_tma = true;
  for (int q = 0; q < n; ++q) {
    if (!fill_problem<BF>(gs[q], a_mn[q], b_mn[q], bn_cta, bm_tile, bn_tile, &G->p[q])) return false;
    all_tma = all_tma && G->p[q].c_tma;
    const int64_t end = (int64_t)G->start[q] + G->p[q].tl.total;
    if (end > (1ll << 30)) return false;
    G->start[q + 1] = (int)end;
  }
  if (!all_tma)
    for (int q = 0; q < n; ++q) G->p[q].c_tma = 0;
  return true;
}

template <bool BF, int BN, int STAGES, int PER_SM, int ACC, int NP>
cudaError_t launch(const GemmArgs* gs, const bool* a_mn, const bool* b_mn, int n, int* err, cudaStream_t stream) {
  constexpr int BKE = BF ? 64 : 32;
  // an MN-major tile is loaded in whole 128-byte-wide chunks
  for (int q = 0; q < n; ++q)
    if (BF && b_mn[q] && BN % BKE) return cudaErrorNotSupported;
  GemmGroup<NP> G{};
  if (!make_group<BF, NP>(gs, a_mn, b_mn, n, BN, BM, BN, &G)) return cudaErrorNotSupported;
  using S = Smem<BN, STAGES>;
  auto kern = gemm_tcgen05_kernel<BF, BN, STAGES, PER_SM, ACC, NP>;
  static bool attr_set = false;
  if (!attr_set) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, S::BYTES);
    if (e != cudaSuccess) return e;
    attr_set = true;
  }
  const int grid = (int)std::min<int64_t>(G.start[n], (int64_t)PER_SM * sm_count());
  if (grid <= 0) return cudaSuccess;
  return launch_pdl(kern, dim3((unsigned)grid), dim3(kThreads), S::BYTES, stream, G, err);
}

template <bool BF, int BN, int STAGES, int PER_SM, int ACC, int NP>
cudaError_t launch_pair(const GemmArgs* gs, const bool* a_mn, const bool* b_mn, int n, int* err,
                        cudaStream_t stream) {
  constexpr int BNH = BN / 2;
  constexpr int BKE = BF ? 64 : 32;
  // each CTA loads BN / 2 columns of B: whole 128-byte chunks when MN-major
  for (int q = 0; q < n; ++q)
    if (b_mn[q] && BNH % BKE) return cudaErrorNotSupported;
  GemmGroup<NP> G{};
  if (!make_group<BF, NP>(gs, a_mn, b_mn, n, BNH, 2 * BM, BN, &G)) return cudaErrorNotSupported;
  using S = Smem<BNH, STAGES>;
  auto kern = gemm_tcgen05_pair<BF, BN, STAGES, PER_SM, ACC, NP>;
  static bool attr_set = false;
  if (!attr_set) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, S::BYTES);
    if (e != cudaSuccess) return e;
    attr_set = true;
  }
  const int pairs = (int)std::min<int64_t>(G.start[n], (int64_t)PER_SM * sm_count() / 2);
  if (pairs <= 0) return cudaSuccess;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(2 * pairs));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = S::BYTES;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  pdl_attribute(&attr[1]);
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  launch_counter().fetch_add(1, std::memory_order_relaxed);
  return cudaLaunchKernelEx(&cfg, kern, G, err);
}

int* error_word() { return tc_error_word(); }

}  // namespace

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, []() {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (PFN_cuTensorMapEncodeTiled_v12000)p;
  });
  return fn;
}

bool tc_make_map(CUtensorMap* m, const float* base, int rank, const uint64_t* dims, const uint64_t* strides_bytes,
                 uint32_t box_rows, bool mn_major) {
  auto enc = encode_fn();
  if (!enc || rank < 2 || rank > 5) return false;
  cuuint64_t d[5], st[4];
  cuuint32_t box[5], es[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    box[i] = i == 0 ? 32u : (i == 1 ? box_rows : 1u);
    es[i] = 1;
  }
  for (int i = 0; i + 1 < rank; ++i) st[i] = strides_bytes[i];
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, (cuuint32_t)rank, (void*)base, d, st, box, es,
                   CU_TENSOR_MAP_INTERLEAVE_NONE,
                   mn_major ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

bool tc_make_map_bf16(CUtensorMap* m, const void* base, int rank, const uint64_t* dims,
                      const uint64_t* strides_bytes, uint32_t box_rows) {
  auto enc = encode_fn();
  if (!enc || rank < 2 || rank > 5) return false;
  cuuint64_t d[5], st[4];
  cuuint32_t box[5], es[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    box[i] = i == 0 ? 64u : (i == 1 ? box_rows : 1u);
    es[i] = 1;
  }
  for (int i = 0; i + 1 < rank; ++i) st[i] = strides_bytes[i];
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, (cuuint32_t)rank, (void*)base, d, st, box, es,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

int* tc_error_word() {
  static int* p = nullptr;
  static std::once_flag once;
  std::call_once(once, []() {
    if (cudaMalloc(&p, sizeof(int)) == cudaSuccess) cudaMemset(p, 0, sizeof(int));
    else p = nullptr;
  });
  return p;
}


namespace {

// Kernel configurations: single-CTA 128 x BN tiles or CTA-pair 256 x BN
// tiles; ACC TMEM accumulators per CTA; PER_SM resident CTAs per SM (shared
// memory and TMEM are sized so that PER_SM CTAs fit: <= 512 TMEM columns).
struct TcCfg {
  bool pair;
  int bn, acc, per_sm, stages;
};
constexpr TcCfg kCfgs[] = {
    {false, 64, 2, 2, 4},   // 0
    {false, 128, 2, 2, 3},  // 1
    {true, 128, 2, 2, 4},   // 2
    {true, 192, 1, 2, 3},   // 3
    {true, 256, 1, 2, 3},   // 4
    {true, 256, 2, 1, 6},   // 5
};
constexpr int kNumCfgs = (int)(sizeof(kCfgs) / sizeof(kCfgs[0]));

// Cost model (microseconds) of one launch: waves of tile-units times the time
// of one unit, whose K steps are bound by the operand bytes an SM receives
// from L2 (~110 GB/s per SM, shared by the CTAs on it) or by the TF32 tensor
// rate (~5.5 TFLOP/s per SM), plus pipeline fill and, with one accumulator, the
// epilogue.  The constants are from measurements on B200 (matmul 2048..8192,
// the nanoGPT and GPT-2 shapes).
constexpr double kSmBytesPerUs = 110e3, kSmFlopsPerUs = 5.5e6, kFillUs = 2.0, kEpiBytesPerUs = 50e3;

double est_us(const TcCfg& c, int64_t M, int64_t N, int64_t K, int64_t units_z, int sms, bool bf) {
  const int tm = c.pair ? 256 : 128;
  const double tiles = (double)((M + tm - 1) / tm) * (double)((N + c.bn - 1) / c.bn) * (double)units_z;
  const double slots = c.pair ? c.per_sm * sms / 2.0 : (double)c.per_sm * sms;
  const double waves = std::ceil(tiles / slots);
  // a stage is 128 bytes of K per row either way: 32 tf32 or 64 bf16 values,
  // and the bf16 rate is twice the tf32 rate, so a stage costs the same
  const double ksteps = std::ceil((double)K / (bf ? 2 * BK : BK));
  const int bcols = c.pair ? c.bn / 2 : c.bn;
  const double t_mem = (128.0 + bcols) * 128.0 / (kSmBytesPerUs / c.per_sm);
  const double t_mma = 2.0 * 128 * c.bn * BK / (kSmFlopsPerUs / c.per_sm);
  const double t_epi = 128.0 * c.bn * 4 / kEpiBytesPerUs;
  const double unit = kFillUs + ksteps * std::max(t_mem, t_mma) + (c.acc == 1 ? t_epi : 0.0);
  return waves * unit + (c.acc == 2 ? t_epi : 0.0);
}

// Operand strides must be multiples of 16 bytes (tensor maps): 4 f32 or 8
// bf16 elements.
bool tc_layout(const GemmArgs& g, bool* a_mn, bool* b_mn) {
  if (g.M < 64 || g.N < 32 || g.K < 32 || g.batch < 1 || g.batch > 65535) return false;
  if (g.M > (1ll << 30) || g.N > (1ll << 30) || g.K > (1ll << 30)) return false;
  if (g.scn != 1 || g.scm < g.N) return false;
  const int64_t q = g.bf16 ? 8 : 4;
  if (g.sak == 1 && g.sam % q == 0 && g.sam >= g.K) *a_mn = false;
  else if (g.sam == 1 && g.sak % q == 0 && g.sak >= g.M) *a_mn = true;
  else return false;
  if (g.sbk == 1 && g.sbn % q == 0 && g.sbn >= g.K) *b_mn = false;
  else if (g.sbn == 1 && g.sbk % q == 0 && g.sbk >= g.N) *b_mn = true;
  else return false;
  if ((((uintptr_t)g.a) & 15) || (((uintptr_t)g.b) & 15)) return false;
  if (g.batch > 1 && ((g.sab % q) || (g.sbb % q) || g.sab < 0 || g.sbb < 0)) return false;
  return true;
}

}  // namespace

int tc_forced_config() {
  // SHEAF_B200_GEMM_CONFIG=n forces configuration n (0..kNumCfgs-1) for every
  // tensor-core GEMM: used by the tests to run every kernel variant on the
  // same shapes.
  if (const char* e = std::getenv("SHEAF_B200_GEMM_CONFIG")) {
    const int f = std::atoi(e);
    if (f >= 0 && f < kNumCfgs) return f;
  }
  return -1;
}

int tc_num_configs() { return kNumCfgs; }

bool tc_plan(const GemmArgs& g, TcPlan* p) {
  bool a_mn, b_mn;
  if (!tc_layout(g, &a_mn, &b_mn)) return false;
  const int sms = sm_count();
  // Split-K, by a fixed rule so that the summation order (the only part of
  // the result that depends on the plan) does not depend on the kernel
  // configuration: a single GEMM whose 128 x 128 tiles do not cover the SMs
  // is split into as many K ranges as fit one wave of 2 CTAs per SM (a partial
  // second wave costs more than it saves), at least 512 of K each (measured on the nanoGPT step: 1024 or no split
  // at all is slower at batch 8 and 64).
  p->splits = 1;
  p->k_chunk = 0;
  const int64_t tiles = ((g.M + 127) / 128) * ((g.N + 127) / 128);
  if (g.batch == 1 && tiles < sms) {
    const int64_t s = std::min<int64_t>(2 * sms / tiles, g.K / 512);
    if (s >= 2) {
      // K ranges in whole stages (32 tf32 or 64 bf16 values)
      const int64_t gran = g.bf16 ? 2 * BK : BK;
      int64_t chunk = (g.K + s - 1) / s;
      chunk = (chunk + gran - 1) / gran * gran;
      p->splits = (g.K + chunk - 1) / chunk;
      p->k_chunk = p->splits > 1 ? chunk : 0;
    }
  }
  const int forced = tc_forced_config();
  if (forced >= 0) {
    p->cfg = forced;
    return true;
  }
  // configuration by the cost model (the measured choice replaces it where
  // the caller can time the candidates)
  const int64_t kc = p->splits > 1 ? p->k_chunk : g.K;
  double best = 1e300;
  for (int ci = 0; ci < kNumCfgs; ++ci) {
    const TcCfg& c = kCfgs[ci];
    if (c.pair && g.M <= 128) continue;
    if (c.bn > 64 && g.N <= 32) continue;
    // bf16 MN-major B is loaded in 64-wide chunks: a CTA-pair half of 96 does not fit
    if (g.bf16 && b_mn && c.pair && (c.bn / 2) % 64) continue;
    const double t = est_us(c, g.M, g.N, kc, p->splits * g.batch, sms, g.bf16 != 0);
    if (t < best) {
      best = t;
      p->cfg = ci;
    }
  }
  return p->cfg >= 0;
}

namespace {

// Configuration cfg (the kCfgs table) with NP products per launch.
template <bool BF, int NP>
cudaError_t launch_cfg(const GemmArgs* gs, const bool* a_mn, const bool* b_mn, int cfg, int* err,
                       cudaStream_t stream) {
  switch (cfg) {
    case 0: return launch<BF, 64, 4, 2, 2, NP>(gs, a_mn, b_mn, NP, err, stream);
    case 1: return launch<BF, 128, 3, 2, 2, NP>(gs, a_mn, b_mn, NP, err, stream);
    case 2: return launch_pair<BF, 128, 4, 2, 2, NP>(gs, a_mn, b_mn, NP, err, stream);
    case 3: return launch_pair<BF, 192, 3, 2, 1, NP>(gs, a_mn, b_mn, NP, err, stream);
    case 4: return launch_pair<BF, 256, 3, 2, 1, NP>(gs, a_mn, b_mn, NP, err, stream);
    case 5: return launch_pair<BF, 256, 6, 1, 2, NP>(gs, a_mn, b_mn, NP, err, stream);
  }
  return cudaErrorNotSupported;
}

}  // namespace

cudaError_t gemm_tcgen05_group(const GemmArgs* gs, int n, int cfg, cudaStream_t stream) {
  if (n < 1 || n > kGemmGroupMax) return cudaErrorInvalidValue;
  bool a_mn[kGemmGroupMax], b_mn[kGemmGroupMax];
  for (int q = 0; q < n; ++q)
    if (!tc_layout(gs[q], &a_mn[q], &b_mn[q]) || gs[q].bf16 != gs[0].bf16) return cudaErrorNotSupported;
  int* err = error_word();
  if (!err) return cudaErrorNotSupported;
  if (gs[0].bf16)
    return n == 1 ? launch_cfg<true, 1>(gs, a_mn, b_mn, cfg, err, stream)
                  : launch_cfg<true, 2>(gs, a_mn, b_mn, cfg, err, stream);
  return n == 1 ? launch_cfg<false, 1>(gs, a_mn, b_mn, cfg, err, stream)
                : launch_cfg<false, 2>(gs, a_mn, b_mn, cfg, err, stream);
}

cudaError_t gemm_tcgen05(const GemmArgs& g, int cfg, cudaStream_t stream) { return gemm_tcgen05_group(&g, 1, cfg, stream); }

int gemm_tcgen05_error() {
  int* p = error_word();
  int v = 0;
  if (p) cudaMemcpy(&v, p, sizeof v, cudaMemcpyDeviceToHost);
  return v;
}

}  // namespace sb
