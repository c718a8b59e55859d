// gemm.cu -- persistent, warp-specialised tcgen05 GEMM for sm_100a.
//
// C = A . B^T, A [M, K] and B [N, K] bf16 with K contiguous ("K-major"), fp32
// accumulation in tensor memory.  Persistent CTAs loop over output tiles:
//   warp 0      TMA producer: 64-wide K slices of A and B into a ring of
//               128B-swizzled shared-memory stages;
//   warp 1      allocates 512 TMEM columns (two 128x256 fp32 accumulators)
//               and issues tcgen05.mma from one thread; tcgen05.commit frees
//               a ring slot / publishes an accumulator;
//   warps 2..9  epilogue, two warpgroups of 128 columns each: tcgen05.ld 32
//               columns at a time from their TMEM lane quarter, fused
//               epilogue math, per-warp 32x32 staging tiles and TMA stores.
// Two variants: single CTA (128x256 tiles, 4 stages, M=128 MMAs) and, for
// M >= 1024, a CTA pair (cta_group::2, 256x256 tiles over two SMs, each CTA
// holding its 128 A rows and half of B, 6 stages, M=256 MMAs).
// The two accumulators let tile i's epilogue overlap tile i+1's main loop.
// No multicast: every CTA loads its own tiles (the CTA-pair variant runs as
// clusters of two that share the MMA, not the loads).
//
// Grouped mode runs several independent problems that share A/C rows
// segments and use different B row blocks (MoE experts, antithetic
// candidates) in one launch.
//
// The reference has no GEMM (its only contraction is the fp32 GEMV of
// cuda/kernels/src/lib.rs:2359-2423); this kernel is the B200 replacement of
// the "linear" operator for M > 1 (rust/crates/ennx/src/dense/linear.rs:484).
#include <stdlib.h>
#include <string.h>

#include "common.cuh"
#include "kernels.cuh"

namespace ennx {
namespace {

constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4;
constexpr int A_BYTES = BM * BK * 2;  // 16 KB
constexpr int B_BYTES = BN * BK * 2;  // 32 KB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int MAX_STAGES = 6;
// Per-variant geometry.  Single-CTA: 128x256 tiles, 4 stages of A 128x64 +
// B 256x64.  CTA pair (cta_group::2): 256x256 tiles over two SMs, each CTA
// holding A 128x64 and half of B (128x64) per stage, 6 stages.
template <bool PAIR> struct Geo {
  static constexpr int TM = PAIR ? 256 : 128;       // rows per tile unit
  static constexpr int BROWS = PAIR ? 128 : 256;    // B rows loaded per CTA
  static constexpr int NST = PAIR ? 6 : 4;          // pipeline stages
  static constexpr int BBYTES = BROWS * BK * 2;
  static constexpr int STAGE = A_BYTES + BBYTES;
  static constexpr uint32_t IDESC = idesc_bf16_f32(PAIR ? 256 : 128, BN);
};
static_assert(Geo<true>::NST * Geo<true>::STAGE == STAGES * STAGE_BYTES, "both variants use the same ring size");
constexpr int EPI_WARPS = 8;                 // two warpgroups, each owns half of the tile's columns
constexpr int THREADS = 64 + 32 * EPI_WARPS;  // producer warp, MMA warp, epilogue warps
constexpr int EPI_BUF = 32 * 32 * 2;          // per-warp 32x32 bf16 staging tile for TMA stores
constexpr int TMEM_COLS = 512;
constexpr int MAX_GROUPS = 256;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + EPI_WARPS * EPI_BUF + 1024 /*align*/ + 4096 /*barriers, tables*/;

struct Args {
  int M, N, K;
  int groups, rows_per_group, b_group_rows;
  const int* group_offsets;
  int epi;
  float alpha;
  void* C;
  long long ldc;
  const uint16_t* R;
  long long ldr;
  const float* row_scale;
  const int* targets;
  float2* lse;
  float* tlogit;
  int n_tiles;
  int n_parts;  // LSE partials per row: 2 * ceil(N / 256) (one per 128-column half tile)
  int has_tmc;  // C tensor map valid (bf16 outputs): full tiles leave through TMA stores
  int n_fast;   // tile order within a group: N tiles fastest (1) or M tiles fastest (0)
  int* err;
};

struct Smem {  // lives after the stage ring
  uint64_t full[MAX_STAGES], empty[MAX_STAGES], tfull[2], tempty[2];
  uint32_t tmem_base;
  int abort_flag;
  int total_tiles;
  int row0[MAX_GROUPS + 1];       // first A/C row of each group
  int tile0[MAX_GROUPS + 1];      // first tile index of each group
};

struct TileInfo {
  int g, mt, nt, row0, rows;
};

template <int TM>
__device__ __forceinline__ TileInfo decode_tile(const Smem& s, const Args& a, int tile) {
  int lo = 0, hi = a.groups - 1;
  while (lo < hi) {
    int mid = (lo + hi + 1) >> 1;
    if (s.tile0[mid] <= tile) lo = mid; else hi = mid - 1;
  }
  TileInfo t;
  t.g = lo;
  t.row0 = s.row0[lo];
  t.rows = s.row0[lo + 1] - s.row0[lo];
  int mtiles = (t.rows + TM - 1) / TM;
  int local = tile - s.tile0[lo];
  if (a.n_fast) {
    t.nt = local % a.n_tiles;
    t.mt = local / a.n_tiles;
  } else {
    t.mt = local % mtiles;
    t.nt = local / mtiles;
  }
  return t;
}

__device__ __forceinline__ float silu(float x) { return x / (1.0f + __expf(-x)); }

// Epilogue of one 128-row x 256-column accumulator tile (this CTA's rows of
// tile t): warp quarter q reads TMEM lanes 32q..32q+31, warpgroup `half` owns
// columns [128*half, 128*half + 128).  Full tiles leave through the per-warp
// 32x32 staging tile `stg` and TMA stores; group-tail tiles use masked direct
// stores.  tbase = TMEM address of the accumulator at this warp's lane quarter.
template <int TM>
__device__ __forceinline__ void epi_tile(const Args& a, const CUtensorMap* tmC, const TileInfo& t, int rank,
                                         uint32_t tbase, uint8_t* stg, int lane, int q, int half) {
  const uint32_t stg_addr = smem_u32(stg);
  const int cta_row = t.mt * TM + rank * BM;  // first row of this CTA's 128 rows, within the group
  const int mrow = cta_row + q * 32 + lane;
  const bool row_ok = mrow < t.rows;
  const long long grow = (long long)t.row0 + mrow;
  const int warp_row0 = t.row0 + cta_row + q * 32;
  const bool use_tma = a.has_tmc && (cta_row + BM <= t.rows || t.row0 + t.rows == a.M);
  uint32_t v[32];

  // 32 packed bf16 pairs (16 words) of this lane's row -> C[row, col0 .. col0+31]
  auto store_bf16 = [&](const uint32_t (&pk)[16], int col0, int ncols) {
    if (use_tma) {
      if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
      __syncwarp();
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int jj = (j + (lane >> 1)) & 3;  // rotate the 16-byte chunks: fewer bank conflicts
        uint32_t c0, c1, c2, c3;  // constant-index selects keep pk in registers
        c0 = jj == 0 ? pk[0] : jj == 1 ? pk[4] : jj == 2 ? pk[8] : pk[12];
        c1 = jj == 0 ? pk[1] : jj == 1 ? pk[5] : jj == 2 ? pk[9] : pk[13];
        c2 = jj == 0 ? pk[2] : jj == 1 ? pk[6] : jj == 2 ? pk[10] : pk[14];
        c3 = jj == 0 ? pk[3] : jj == 1 ? pk[7] : jj == 2 ? pk[11] : pk[15];
        asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(stg_addr + lane * 64 + jj * 16),
                     "r"(c0), "r"(c1), "r"(c2), "r"(c3)
                     : "memory");
      }
      fence_proxy_async();
      __syncwarp();
      if (lane == 0) {
        asm volatile(
            "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"((uint64_t)tmC),
            "r"(stg_addr), "r"(col0), "r"(warp_row0)
            : "memory");
        asm volatile("cp.async.bulk.commit_group;" ::: "memory");
      }
    } else if (row_ok && col0 < ncols) {
      uint16_t* dst = (uint16_t*)a.C + grow * a.ldc + col0;
      if (col0 + 32 <= ncols) {
#pragma unroll
        for (int j = 0; j < 4; ++j) st_global_v4(dst + 8 * j, pk[4 * j], pk[4 * j + 1], pk[4 * j + 2], pk[4 * j + 3]);
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (col0 + j < ncols) dst[j] = (uint16_t)(pk[j >> 1] >> (16 * (j & 1)));
      }
    }
  };

  if (a.epi == ENNX_B200_EPI_SWIGLU) {
    for (int c = half * 64; c < half * 64 + 64; c += 32) {
      uint32_t u[32];
      tmem_ld32(tbase + c, v);
      tmem_ld32(tbase + c + BN / 2, u);
      tmem_ld_wait();
      uint32_t pk[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        float g0 = __uint_as_float(v[2 * j]) * a.alpha, g1 = __uint_as_float(v[2 * j + 1]) * a.alpha;
        float u0 = __uint_as_float(u[2 * j]) * a.alpha, u1 = __uint_as_float(u[2 * j + 1]) * a.alpha;
        pk[j] = pack_bf16x2(silu(g0) * u0, silu(g1) * u1);
      }
      store_bf16(pk, t.nt * (BN / 2) + c, a.N / 2);
    }
  } else if (a.epi == ENNX_B200_EPI_LSE) {
    float m = -INFINITY, ssum = 0.0f, tl = 0.0f;
    int tgt = row_ok ? a.targets[grow] : -1;
    bool have_t = false;
    for (int c = half * 128; c < half * 128 + 128; c += 32) {
      tmem_ld32(tbase + c, v);
      tmem_ld_wait();
      int col0 = t.nt * BN + c;
      float cm = -INFINITY;
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        float x = __uint_as_float(v[j]) * a.alpha;
        if (col0 + j < a.N) cm = fmaxf(cm, x);
        if (col0 + j == tgt) { tl = x; have_t = true; }
      }
      if (cm > -INFINITY) {
        float nm = fmaxf(m, cm);
        float acc_s = ssum * __expf(m - nm);
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (col0 + j < a.N) acc_s += __expf(__uint_as_float(v[j]) * a.alpha - nm);
        ssum = acc_s;
        m = nm;
      }
    }
    if (row_ok) {
      a.lse[grow * a.n_parts + t.nt * 2 + half] = make_float2(m, ssum);
      if (have_t) a.tlogit[grow] = tl;
    }
  } else {
    const float rs = (a.epi == ENNX_B200_EPI_ROWSCALE && row_ok) ? a.row_scale[grow] : a.alpha;
    for (int c = half * 128; c < half * 128 + 128; c += 32) {
      tmem_ld32(tbase + c, v);
      tmem_ld_wait();
      int col0 = t.nt * BN + c;
      bool full = col0 + 32 <= a.N;
      if (a.epi == ENNX_B200_EPI_F32) {
        if (!row_ok || col0 >= a.N) continue;
        float* dst = (float*)a.C + grow * a.ldc + col0;
        if (full) {
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            float x0 = __uint_as_float(v[4 * j]) * rs, x1 = __uint_as_float(v[4 * j + 1]) * rs;
            float x2 = __uint_as_float(v[4 * j + 2]) * rs, x3 = __uint_as_float(v[4 * j + 3]) * rs;
            st_global_v4(dst + 4 * j, __float_as_uint(x0), __float_as_uint(x1), __float_as_uint(x2),
                         __float_as_uint(x3));
          }
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (col0 + j < a.N) dst[j] = __uint_as_float(v[j]) * rs;
        }
        continue;
      }
      if (use_tma && col0 >= a.N) continue;  // warp-uniform: whole chunk outside C
      float x[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) x[j] = __uint_as_float(v[j]) * rs;
      if (a.R && row_ok && col0 < a.N) {
        const uint16_t* rp = a.R + grow * a.ldr + col0;
        if (full) {
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            uint4 rv = *reinterpret_cast<const uint4*>(rp + 8 * j);
            uint32_t w4[4] = {rv.x, rv.y, rv.z, rv.w};
#pragma unroll
            for (int h = 0; h < 4; ++h) {
              x[8 * j + 2 * h] += bf16_to_f32((uint16_t)(w4[h] & 0xffffu));
              x[8 * j + 2 * h + 1] += bf16_to_f32((uint16_t)(w4[h] >> 16));
            }
          }
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (col0 + j < a.N) x[j] += bf16_to_f32(rp[j]);
        }
      }
      uint32_t pk[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) pk[j] = pack_bf16x2(x[2 * j], x[2 * j + 1]);
      store_bf16(pk, col0, a.N);
    }
  }
}
template <bool PAIR>
__global__ void __launch_bounds__(THREADS, 2)
    gemm_bf16_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmC, Args a) {
  extern __shared__ uint8_t smem_raw[];
  uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* ring = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  uint8_t* epi_smem = ring + STAGES * STAGE_BYTES;
  Smem& s = *reinterpret_cast<Smem*>(epi_smem + EPI_WARPS * EPI_BUF);
  using G = Geo<PAIR>;
  uint8_t* sA = ring;
  uint8_t* sB = ring + G::NST * A_BYTES;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rank = PAIR ? (int)cluster_ctarank() : 0;          // CTA within the pair
  const int unit0 = PAIR ? blockIdx.x >> 1 : blockIdx.x;        // first tile unit
  const int units = PAIR ? gridDim.x >> 1 : gridDim.x;          // tile-unit stride

  if (threadIdx.x == 0) {
    for (int i = 0; i < G::NST; ++i) { mbar_init(&s.full[i], 1); mbar_init(&s.empty[i], 1); }
    for (int i = 0; i < 2; ++i) { mbar_init(&s.tfull[i], 1); mbar_init(&s.tempty[i], (PAIR ? 2 : 1) * EPI_WARPS); }
    s.abort_flag = 0;
    // group table: row offsets (device table or uniform split) and tile prefix
    int tiles = 0;
    for (int g = 0; g < a.groups; ++g) {
      int r0 = a.group_offsets ? a.group_offsets[g] : g * a.rows_per_group;
      int r1 = a.group_offsets ? a.group_offsets[g + 1] : (g + 1) * a.rows_per_group;
      s.row0[g] = r0;
      s.row0[g + 1] = r1;
      s.tile0[g] = tiles;
      int rows = r1 - r0;
      tiles += (rows > 0 ? (rows + G::TM - 1) / G::TM : 0) * a.n_tiles;
    }
    s.tile0[a.groups] = tiles;
    s.total_tiles = tiles;
    fence_barrier_init();
    fence_proxy_async();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if (a.has_tmc) tma_prefetch_desc(&tmC);
  }
  if (warp == 1) {
    if (PAIR) { tmem_alloc_pair(&s.tmem_base, TMEM_COLS); tmem_relinquish_pair(); }
    else { tmem_alloc(&s.tmem_base, TMEM_COLS); tmem_relinquish(); }
  }
  __syncthreads();
  if (PAIR) cluster_sync();  // the peer's barriers exist before any cross-CTA arrive
  tc_fence_after();
  const uint32_t tmem_base = s.tmem_base;
  const int total = s.total_tiles;
  const int KB = a.K / BK;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int tile = unit0; tile < total && !*(volatile int*)&s.abort_flag; tile += units) {
        TileInfo t = decode_tile<G::TM>(s, a, tile);
        int arow = t.row0 + t.mt * G::TM + rank * BM;
        int brow = t.g * a.b_group_rows + t.nt * BN + rank * G::BROWS;
        for (int kb = 0; kb < KB; ++kb) {
          if (!mbar_wait(&s.empty[stage], phase ^ 1u, a.err)) { s.abort_flag = 1; break; }
          if (PAIR) {
            // both CTAs' bytes complete on the leader's barrier; only the leader arrives
            if (rank == 0) mbar_arrive_expect_tx(&s.full[stage], 2 * G::STAGE);
            const uint32_t bar = mapa_shared(&s.full[stage], 0);
            tma_load_2d_pair(sA + stage * A_BYTES, &tmA, bar, kb * BK, arow);
            tma_load_2d_pair(sB + stage * G::BBYTES, &tmB, bar, kb * BK, brow);
          } else {
            mbar_arrive_expect_tx(&s.full[stage], G::STAGE);
            tma_load_2d(sA + stage * A_BYTES, &tmA, &s.full[stage], kb * BK, arow);
            tma_load_2d(sB + stage * G::BBYTES, &tmB, &s.full[stage], kb * BK, brow);
          }
          if (++stage == G::NST) { stage = 0; phase ^= 1u; }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {  // the leader CTA issues the MMAs of the pair
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      for (int tile = unit0; tile < total && !*(volatile int*)&s.abort_flag; tile += units, ++it) {
        int acc = it & 1;
        uint32_t acc_phase = (it >> 1) & 1;
        if (!mbar_wait(&s.tempty[acc], acc_phase ^ 1u, a.err)) { s.abort_flag = 1; break; }
        tc_fence_after();
        uint32_t d = tmem_base + acc * BN;
        bool ok = true;
        for (int kb = 0; kb < KB; ++kb) {
          if (!mbar_wait(&s.full[stage], phase, a.err)) { s.abort_flag = 1; ok = false; break; }
          tc_fence_after();
          uint32_t abase = smem_u32(sA + stage * A_BYTES);
          uint32_t bbase = smem_u32(sB + stage * G::BBYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            if (PAIR)
              umma_f16_pair(d, smem_desc_sw128(abase + k * 32), smem_desc_sw128(bbase + k * 32), G::IDESC,
                            (kb | k) != 0);
            else
              umma_f16(d, smem_desc_sw128(abase + k * 32), smem_desc_sw128(bbase + k * 32), G::IDESC, (kb | k) != 0);
          }
          if (PAIR) umma_commit_pair(&s.empty[stage], 0x3);
          else umma_commit(&s.empty[stage]);
          if (++stage == G::NST) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
        if (PAIR) umma_commit_pair(&s.tfull[acc], 0x3);
        else umma_commit(&s.tfull[acc]);
      }
    }
  } else {
    // Epilogue: warps 2..9.  Warp w reads TMEM lane quarter w % 4 (rows
    // 32*(w%4) .. +31 of the tile); warpgroup h = (w-2)/4 owns columns
    // [h*128, h*128 + 128).  Full tiles leave through per-warp 32x32 staging
    // tiles and TMA stores; group-tail tiles use masked direct stores.
    const int ew = warp - 2;
    const int q = warp & 3;
    const int half = ew >> 2;
    uint8_t* stg = epi_smem + ew * EPI_BUF;
    int it = 0;
    for (int tile = unit0; tile < total; tile += units, ++it) {
      int acc = it & 1;
      uint32_t acc_phase = (it >> 1) & 1;
      if (!mbar_wait(&s.tfull[acc], acc_phase, a.err)) { s.abort_flag = 1; break; }
      tc_fence_after();
      TileInfo t = decode_tile<G::TM>(s, a, tile);
      const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + acc * BN;
      epi_tile<G::TM>(a, &tmC, t, rank, tbase, stg, lane, q, half);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (PAIR) mbar_arrive_cluster(mapa_shared(&s.tempty[acc], 0));  // the leader's MMA waits on both CTAs
        else mbar_arrive(&s.tempty[acc]);
      }
    }
    if (lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
    __syncwarp();
  }

  __syncthreads();
  if (PAIR) cluster_sync();  // both CTAs are done with TMEM and with each other's barriers
  if (warp == 1) {
    tc_fence_after();
    if (PAIR) tmem_dealloc_pair(tmem_base, TMEM_COLS);
    else tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// ===========================================================================
// Perturbed-B variant: the antithetic pair's operands W + E and W - E are
// formed inside the GEMM's operand path, never stored.
//
// Groups come in sign pairs: group e (< P = groups / 2) holds the rows of the
// `+` candidate and group P + e the rows of the `-` candidate; both use B row
// block e of W and of E (the bf16 noise step sigma*eps).  A work unit is
// (e, m, n): 256 rows of each sign against one 256-row N tile, on a CTA pair
// (cta_group::2); accumulators in TMEM columns [0, 256) (`+`) and
// [256, 512) (`-`).  K advances in 32-wide stages through two rings:
//   A ring (4 stages): A+ | A- of this CTA's 128 rows (2 x 8 KB), loaded by
//     the A producer with the pair form of TMA onto the leader's barrier;
//   B ring (8 stages): W | E of this CTA's 128 B rows (2 x 8 KB), loaded by
//     the B producer onto this CTA's own barrier, then rewritten in place by
//     the transform warps, W -> W + E and E -> W - E, in bf16x2 arithmetic
//     (one RNE rounding of the exact sum, the definition of the perturbed
//     weight).  All tiles share one 64-byte-swizzled K-major layout, so the
//     rewrite is a flat element-wise pass over 16-byte chunks.  Two groups of
//     four transform warps take alternate stages; each arrives on the
//     leader's `ready` barrier after a proxy fence.
// The B ring is twice as deep as the A ring because its chain (load,
// rewrite, cross-CTA arrival) is longer.  One B stage feeds both signs' MMAs,
// so W and E cross L2 once per unit, as a plain B operand would.  A sign
// whose 256-row tile is empty (ragged MoE groups) has its loads and MMAs
// skipped.
// ===========================================================================
#ifndef PB_TWARPS_DEF
#define PB_TWARPS_DEF 8
#endif
constexpr int PB_TWARPS = PB_TWARPS_DEF;                      // transform warps (PB_TGROUPS groups)
#ifndef PB_TGROUPS_DEF
#define PB_TGROUPS_DEF 2
#endif
constexpr int PB_TGROUPS = PB_TGROUPS_DEF;                    // transform groups, taking B stages in turn
constexpr int PB_GROUP_THREADS = 32 * PB_TWARPS / PB_TGROUPS;
constexpr int PB_THREADS = 64 + 32 * EPI_WARPS + 32 * PB_TWARPS + 32;  // + the B producer warp: 608
constexpr int PB_BPROD_WARP = 2 + EPI_WARPS + PB_TWARPS;
// K per stage 64 (128-byte swizzled rows: one L2 request moves a whole
// line, where 64-byte rows took twice the requests).  A B stage lives
// longer than an A stage (load, rewrite by the transform warps, then MMA),
// and an A stage is freed only when the MMA two stages back completes, so
// both rings want depth: the kernel has no epilogue staging (direct 16-byte
// stores) and a 2 KB table area, which makes room for 3 A + 4 B stages of
// 32 KB in the 227 KB of shared memory.  (Measured: 2 + 4 stages 20 %
// faster than 6 + 6 stages of K 32, and than 3 + 3 of K 64.)
#ifndef PB_BK_DEF
#define PB_BK_DEF 64
#define PB_NA_DEF 3
#define PB_NB_DEF 4
#endif
constexpr int PB_BK = PB_BK_DEF;                              // K per stage
constexpr int PB_TILE = BM * PB_BK * 2;                       // 128 rows x 2 PB_BK bytes
constexpr int PB_NA = PB_NA_DEF, PB_NB = PB_NB_DEF;
constexpr int PB_SW = PB_BK * 2;                              // swizzle span = row bytes (64 or 128)
constexpr int PB_CH = PB_TILE / 16 / PB_GROUP_THREADS;        // 16-byte chunks of W (and of E) per transform thread
__device__ __forceinline__ uint64_t pb_desc(uint32_t a) { return PB_SW == 128 ? smem_desc_sw128(a) : smem_desc_sw64(a); }
constexpr uint32_t PB_IDESC = idesc_bf16_f32(256, BN);
constexpr int PB_TABLES = 2048;
constexpr int PB_SMEM_BYTES = 1024 /*align*/ + (PB_NA + PB_NB) * 2 * PB_TILE + PB_TABLES;
static_assert(PB_SMEM_BYTES <= 232448, "perturbed-B rings and tables fit 227 KB of shared memory");
static_assert(PB_TGROUPS <= PB_NB, "each transform group starts on its own stage");
static_assert(PB_TILE / 16 == PB_CH * PB_GROUP_THREADS, "whole 16-byte chunks of W and E per transform thread");
static_assert(PB_THREADS * 96 <= 65536, "register budget");

struct PbArgs {
  int pairs;  // P
};

struct PbSmem {  // lives after the epilogue staging tiles
  uint64_t full_a[PB_NA], empty_a[PB_NA];
  uint64_t full_b[PB_NB], ready_b[PB_NB], empty_b[PB_NB];
  uint64_t tfull, tempty[2];
  uint32_t tmem_base;
  int abort_flag;
  int total_units;
  int row0[MAX_GROUPS + 1];
  int unit0[MAX_GROUPS / 2 + 1];
};

struct PbUnit {
  int e, mt, nt;
};

static_assert(sizeof(PbSmem) <= PB_TABLES, "perturbed-B barriers and tables fit their area");

__device__ __forceinline__ PbUnit decode_pb(const PbSmem& s, int pairs, int n_tiles, int unit) {
  int lo = 0, hi = pairs - 1;
  while (lo < hi) {
    int mid = (lo + hi + 1) >> 1;
    if (s.unit0[mid] <= unit) lo = mid; else hi = mid - 1;
  }
  PbUnit u;
  u.e = lo;
  const int mtiles = (s.unit0[lo + 1] - s.unit0[lo]) / n_tiles;
  const int local = unit - s.unit0[lo];
  u.mt = local % mtiles;
  u.nt = local / mtiles;
  return u;
}

__device__ __forceinline__ TileInfo pb_tile(const PbSmem& s, const PbUnit& u, int sign, int pairs) {
  TileInfo t;
  t.g = u.e + sign * pairs;
  t.row0 = s.row0[t.g];
  t.rows = s.row0[t.g + 1] - t.row0;
  t.mt = u.mt;
  t.nt = u.nt;
  return t;
}

__global__ void __maxnreg__(96)
    gemm_pb_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW,
                   const __grid_constant__ CUtensorMap tmE, const __grid_constant__ CUtensorMap tmC, Args a,
                   PbArgs pb) {
  extern __shared__ uint8_t smem_raw[];
  uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* ring = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  uint8_t* ring_a = ring;                                // PB_NA x [A+ | A-]
  uint8_t* ring_b = ring + PB_NA * 2 * PB_TILE;          // PB_NB x [W | E]
  PbSmem& s = *reinterpret_cast<PbSmem*>(ring + (PB_NA + PB_NB) * 2 * PB_TILE);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rank = (int)cluster_ctarank();
  const int first = blockIdx.x >> 1, stride = gridDim.x >> 1;
  const int P = pb.pairs;

  if (threadIdx.x == 0) {
    for (int i = 0; i < PB_NA; ++i) { mbar_init(&s.full_a[i], 1); mbar_init(&s.empty_a[i], 1); }
    for (int i = 0; i < PB_NB; ++i) {
      mbar_init(&s.full_b[i], 1);
      mbar_init(&s.ready_b[i], 2 * PB_TWARPS / PB_TGROUPS);  // one group of four warps in each of the two CTAs
      mbar_init(&s.empty_b[i], 1);
    }
    mbar_init(&s.tfull, 1);
    for (int i = 0; i < 2; ++i) mbar_init(&s.tempty[i], 2 * EPI_WARPS);
    s.abort_flag = 0;
    for (int g = 0; g < a.groups; ++g) {
      s.row0[g] = a.group_offsets ? a.group_offsets[g] : g * a.rows_per_group;
      s.row0[g + 1] = a.group_offsets ? a.group_offsets[g + 1] : (g + 1) * a.rows_per_group;
    }
    int n = 0;
    for (int e = 0; e < P; ++e) {
      const int rp = s.row0[e + 1] - s.row0[e], rm = s.row0[P + e + 1] - s.row0[P + e];
      s.unit0[e] = n;
      n += (max(rp, rm) + 255) / 256 * a.n_tiles;
    }
    s.unit0[P] = n;
    s.total_units = n;
    fence_barrier_init();
    fence_proxy_async();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmW);
    tma_prefetch_desc(&tmE);
    if (a.has_tmc) tma_prefetch_desc(&tmC);
  }
  if (warp == 1) { tmem_alloc_pair(&s.tmem_base, TMEM_COLS); tmem_relinquish_pair(); }
  __syncthreads();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = s.tmem_base;
  const int total = s.total_units;
  const int KB = a.K / PB_BK;
  auto a_ptr = [&](int stage, int sign) { return ring_a + (stage * 2 + sign) * PB_TILE; };
  auto b_ptr = [&](int stage, int part) { return ring_b + (stage * 2 + part) * PB_TILE; };
  auto aborted = [&]() { return *(volatile int*)&s.abort_flag != 0; };

  if (warp == 0) {
    // A producer: this CTA's 128 rows of each active sign; the pair form puts
    // both CTAs' bytes on the leader's barrier
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int unit = first; unit < total && !aborted(); unit += stride) {
        const PbUnit u = decode_pb(s, P, a.n_tiles, unit);
        const TileInfo tp = pb_tile(s, u, 0, P), tm = pb_tile(s, u, 1, P);
        const bool act_p = u.mt * 256 < tp.rows, act_m = u.mt * 256 < tm.rows;
        const uint32_t bytes = 2u * PB_TILE * ((act_p ? 1u : 0u) + (act_m ? 1u : 0u));
        for (int kb = 0; kb < KB; ++kb) {
          if (!mbar_wait(&s.empty_a[stage], phase ^ 1u, a.err)) { s.abort_flag = 1; break; }
          if (rank == 0) mbar_arrive_expect_tx(&s.full_a[stage], bytes);
          const uint32_t bar = mapa_shared(&s.full_a[stage], 0);
          const int kx = kb * PB_BK;
          if (act_p) tma_load_2d_pair(a_ptr(stage, 0), &tmA, bar, kx, tp.row0 + u.mt * 256 + rank * BM);
          if (act_m) tma_load_2d_pair(a_ptr(stage, 1), &tmA, bar, kx, tm.row0 + u.mt * 256 + rank * BM);
          if (++stage == PB_NA) { stage = 0; phase ^= 1u; }
        }
      }
    }
  } else if (warp == PB_BPROD_WARP) {
    // B producer: this CTA's 128 rows of W and E onto this CTA's own barrier
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int unit = first; unit < total && !aborted(); unit += stride) {
        const PbUnit u = decode_pb(s, P, a.n_tiles, unit);
        const int brow = u.e * a.b_group_rows + u.nt * BN + rank * BM;
        for (int kb = 0; kb < KB; ++kb) {
          if (!mbar_wait(&s.empty_b[stage], phase ^ 1u, a.err)) { s.abort_flag = 1; break; }
          mbar_arrive_expect_tx(&s.full_b[stage], 2u * PB_TILE);
          tma_load_2d(b_ptr(stage, 0), &tmW, &s.full_b[stage], kb * PB_BK, brow);
          tma_load_2d(b_ptr(stage, 1), &tmE, &s.full_b[stage], kb * PB_BK, brow);
          if (++stage == PB_NB) { stage = 0; phase ^= 1u; }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      int sa = 0, sb = 0;
      uint32_t pa = 0, pbh = 0;
      int it = 0;
      for (int unit = first; unit < total && !aborted(); unit += stride, ++it) {
        const PbUnit u = decode_pb(s, P, a.n_tiles, unit);
        const bool act_p = u.mt * 256 < pb_tile(s, u, 0, P).rows,
                   act_m = u.mt * 256 < pb_tile(s, u, 1, P).rows;
        const uint32_t acc_phase = it & 1;
        bool ok = true;
        for (int kb = 0; kb < KB; ++kb) {
          if (!mbar_wait(&s.ready_b[sb], pbh, a.err) || !mbar_wait(&s.full_a[sa], pa, a.err)) { ok = false; break; }
          tc_fence_after();
          const uint32_t ab = smem_u32(a_ptr(sa, 0)), bb = smem_u32(b_ptr(sb, 0));
          // `+` accumulator first; at the first stage wait until the epilogue
          // has drained it (the `-` one is drained after it)
          if (kb == 0 && !mbar_wait(&s.tempty[0], acc_phase ^ 1u, a.err)) { ok = false; break; }
          tc_fence_after();
          if (act_p) {
#pragma unroll
            for (int k = 0; k < PB_BK / 16; ++k)
              umma_f16_pair(tmem_base, pb_desc(ab + k * 32), pb_desc(bb + k * 32), PB_IDESC,
                            (kb | k) != 0);
          }
          if (kb == 0 && !mbar_wait(&s.tempty[1], acc_phase ^ 1u, a.err)) { ok = false; break; }
          tc_fence_after();
          if (act_m) {
#pragma unroll
            for (int k = 0; k < PB_BK / 16; ++k)
              umma_f16_pair(tmem_base + BN, pb_desc(ab + PB_TILE + k * 32),
                            pb_desc(bb + PB_TILE + k * 32), PB_IDESC, (kb | k) != 0);
          }
          umma_commit_pair(&s.empty_a[sa], 0x3);
          umma_commit_pair(&s.empty_b[sb], 0x3);
          if (++sa == PB_NA) { sa = 0; pa ^= 1u; }
          if (++sb == PB_NB) { sb = 0; pbh ^= 1u; }
        }
        if (!ok) { s.abort_flag = 1; break; }
        umma_commit_pair(&s.tfull, 0x3);
      }
    }
  } else if (warp < 2 + EPI_WARPS) {
    const int ew = warp - 2;
    const int q = warp & 3;
    const int half = ew >> 2;
    uint8_t* stg = ring;  // unused: no TMA stores in this kernel (Args::has_tmc = 0)
    int it = 0;
    for (int unit = first; unit < total; unit += stride, ++it) {
      if (!mbar_wait(&s.tfull, it & 1, a.err)) { s.abort_flag = 1; break; }
      tc_fence_after();
      const PbUnit u = decode_pb(s, P, a.n_tiles, unit);
      for (int sign = 0; sign < 2; ++sign) {
        const TileInfo t = pb_tile(s, u, sign, P);
        if (u.mt * 256 < t.rows)
          epi_tile<256>(a, &tmC, t, rank, tmem_base + ((uint32_t)(q * 32) << 16) + sign * BN, stg, lane, q, half);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(mapa_shared(&s.tempty[sign], 0));
      }
    }
    if (lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
    __syncwarp();
  } else {
    // transform warps: group tg (warps 10-13 / 14-17) takes the B stages
    // i = tg mod PB_TGROUPS; thread tt rewrites 16-byte chunks tt + 128 j
    // (j < PB_CH) of the W and E slots, W -> W + E and E -> W - E (identical
    // swizzled layouts)
    const int tg = (warp - (2 + EPI_WARPS)) / (PB_TWARPS / PB_TGROUPS);
    const int tt = threadIdx.x - 32 * (2 + EPI_WARPS) - tg * PB_GROUP_THREADS;
    const uint32_t ready_remote = mapa_shared(&s.ready_b[0], 0);  // ready_b[i] = ready_remote + 8 i
    const int my_units = total > first ? (total - first + stride - 1) / stride : 0;
    const int items = my_units * KB;
    int stage = tg;
    uint32_t phase = 0;
    for (int i = tg; i < items; i += PB_TGROUPS) {
      if (aborted()) break;
      if (!mbar_wait(&s.full_b[stage], phase, a.err)) { s.abort_flag = 1; break; }
      const uint32_t bw = smem_u32(b_ptr(stage, 0)) + tt * 16, be = bw + PB_TILE;
      constexpr int CB = PB_CH < 4 ? PB_CH : 4;  // chunks in flight per thread
      constexpr uint32_t CS = 16 * PB_GROUP_THREADS;
#pragma unroll
      for (int j0 = 0; j0 < PB_CH; j0 += CB) {
        uint4 w[CB], e[CB];
#pragma unroll
        for (int j = 0; j < CB; ++j) {
          const uint32_t o = (j0 + j) * CS;
          asm volatile("ld.shared.v4.b32 {%0,%1,%2,%3}, [%4];"
                       : "=r"(w[j].x), "=r"(w[j].y), "=r"(w[j].z), "=r"(w[j].w) : "r"(bw + o));
          asm volatile("ld.shared.v4.b32 {%0,%1,%2,%3}, [%4];"
                       : "=r"(e[j].x), "=r"(e[j].y), "=r"(e[j].z), "=r"(e[j].w) : "r"(be + o));
        }
#pragma unroll
        for (int j = 0; j < CB; ++j) {
          const uint32_t o = (j0 + j) * CS;
          asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(bw + o), "r"(bf16x2_add(w[j].x, e[j].x)),
                       "r"(bf16x2_add(w[j].y, e[j].y)), "r"(bf16x2_add(w[j].z, e[j].z)),
                       "r"(bf16x2_add(w[j].w, e[j].w))
                       : "memory");
          asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(be + o), "r"(bf16x2_sub(w[j].x, e[j].x)),
                       "r"(bf16x2_sub(w[j].y, e[j].y)), "r"(bf16x2_sub(w[j].z, e[j].z)),
                       "r"(bf16x2_sub(w[j].w, e[j].w))
                       : "memory");
        }
      }
      fence_proxy_async();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(ready_remote + 8u * (uint32_t)stage);
      stage += PB_TGROUPS;  // this group's next stage
      if (stage >= PB_NB) { stage -= PB_NB; phase ^= 1u; }
    }
  }

  __syncthreads();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
}

bool g_attr_set[64];
bool g_pb_attr_set[64];

}  // namespace
}  // namespace ennx

namespace ennx {

// Argument checks shared by the plain and the perturbed-B GEMM.
static int32_t check_gemm(const ennx_b200_gemm_params* p, void* C) {
  const int M = p->m, N = p->n, K = p->k;
  const int G = p->groups < 1 ? 1 : p->groups;
  if (M <= 0 || N <= 0 || K <= 0) return set_error(ENNX_B200_INVALID_ARGUMENT, "gemm: empty problem %dx%dx%d", M, N, K);
  if (K % BK != 0) return set_error(ENNX_B200_UNSUPPORTED, "gemm: K=%d must be a multiple of %d", K, BK);
  if (G > MAX_GROUPS) return set_error(ENNX_B200_UNSUPPORTED, "gemm: at most %d groups", MAX_GROUPS);
  if (!p->group_offsets && M % G != 0)
    return set_error(ENNX_B200_INVALID_ARGUMENT, "gemm: M=%d not divisible into %d uniform groups", M, G);
  if (p->lda < K || p->ldb < K || p->lda % 8 || p->ldb % 8)
    return set_error(ENNX_B200_INVALID_ARGUMENT, "gemm: lda/ldb must be >= K and multiples of 8");
  const int epi = p->epilogue;
  if (epi < 0 || epi > ENNX_B200_EPI_LSE) return set_error(ENNX_B200_INVALID_ARGUMENT, "gemm: unknown epilogue %d", epi);
  if (epi == ENNX_B200_EPI_SWIGLU && N % BN != 0)
    return set_error(ENNX_B200_INVALID_ARGUMENT, "gemm: SwiGLU needs N a multiple of %d", BN);
  if (epi == ENNX_B200_EPI_LSE && (!p->targets || !p->lse_partial || !p->target_logit))
    return set_error(ENNX_B200_INVALID_ARGUMENT, "gemm: LSE epilogue needs targets, lse_partial, target_logit");
  if (epi == ENNX_B200_EPI_ROWSCALE && !p->row_scale)
    return set_error(ENNX_B200_INVALID_ARGUMENT, "gemm: ROWSCALE epilogue needs row_scale");
  if (epi != ENNX_B200_EPI_LSE) {
    if (!C) return set_error(ENNX_B200_INVALID_ARGUMENT, "gemm: null C");
    long long out_cols = epi == ENNX_B200_EPI_SWIGLU ? N / 2 : N;
    if (p->ldc < out_cols || (((uintptr_t)C) & 15u) || (p->ldc * (epi == ENNX_B200_EPI_F32 ? 4 : 2)) % 16)
      return set_error(ENNX_B200_INVALID_ARGUMENT, "gemm: C must be 16-byte aligned with ldc >= %lld and 16-byte rows",
                       out_cols);
  }
  if (p->residual && (p->ldr % 8 || ((uintptr_t)p->residual & 15u)))
    return set_error(ENNX_B200_INVALID_ARGUMENT, "gemm: residual must be 16-byte aligned with ldr %% 8 == 0");

  return ENNX_B200_OK;
}

// Kernel arguments common to both variants.
static Args make_args(const ennx_b200_gemm_params* p, void* C, bool bf16_out) {
  const int M = p->m, N = p->n, K = p->k;
  const int G = p->groups < 1 ? 1 : p->groups;
  const int epi = p->epilogue;
  Args a;
  a.M = M; a.N = N; a.K = K;
  a.groups = G;
  a.rows_per_group = p->group_offsets ? 0 : M / G;
  a.b_group_rows = p->b_group_rows;
  a.group_offsets = p->group_offsets;
  a.epi = epi;
  a.alpha = p->alpha == 0.0f ? 1.0f : p->alpha;
  a.C = C; a.ldc = p->ldc;
  a.R = p->residual; a.ldr = p->ldr;
  a.row_scale = p->row_scale;
  a.targets = p->targets;
  a.lse = (float2*)p->lse_partial;
  a.tlogit = p->target_logit;
  a.n_tiles = (N + BN - 1) / BN;
  a.n_parts = 2 * a.n_tiles;
  a.has_tmc = bf16_out ? 1 : 0;
  a.err = nullptr;
  // Tile order within a group.  M tiles fastest (the default): the tiles
  // that run together share one B tile, and every A tile is read once per
  // N tile -- cheap while A stays in L2.  N tiles fastest when a group's A
  // rows cannot stay in L2 but its B block can (e.g. 2 x 16384 rows against
  // a 2048 x 2048 B): then B is the operand re-read, from L2.  (The LM head,
  // 8192 rows against a 151936-row B, must stay M-fastest: N-fastest would
  // stream its 0.6 GB B once per M tile.)
  {
    const double rows_per_group = (double)M / G, l2_share = 48e6;
    const double a_bytes = rows_per_group * K * 2.0, b_bytes = (double)N * K * 2.0;
    a.n_fast = (a_bytes > l2_share && b_bytes <= l2_share) ? 1 : 0;
  }
  if (const char* e = getenv("ENNX_B200_GEMM_ORDER")) a.n_fast = atoi(e);
  return a;
}

int32_t gemm_bf16(const ennx_b200_gemm_params* p, const uint16_t* A, const uint16_t* B, void* C, cudaStream_t st) {
  if (!p || !A || !B) return set_error(ENNX_B200_INVALID_ARGUMENT, "gemm: null argument");
  ENNX_TRY(check_gemm(p, C));
  const int M = p->m, N = p->n, K = p->k;
  const int G = p->groups < 1 ? 1 : p->groups;
  const int epi = p->epilogue;
  // CTA-pair variant for problems with enough rows to fill 256-row tiles;
  // ENNX_B200_GEMM_PAIR=0/1 forces a variant (tests exercise both).
  // Grouped problems with device-side offsets (the expert GEMMs) take the
  // CTA pair only at >= 1024 rows per group on average: at ~512 rows a
  // group's last 256-row tile is often mostly padding, and 128-row tiles
  // waste less (measured: the population step 739 -> 729 ms).
  bool pair = M >= 1024 && (!p->group_offsets || (long long)M / G >= 1024);
  if (const char* e = getenv("ENNX_B200_GEMM_PAIR")) pair = e[0] == '1';
  const int brows = pair ? Geo<true>::BROWS : Geo<false>::BROWS;

  const long long b_rows = (long long)(G - 1) * p->b_group_rows + N;
  CUtensorMap ta, tb, tc;
  ENNX_TRY(make_tmap_2d_bf16(&ta, A, (uint64_t)K, (uint64_t)M, (uint64_t)p->lda, BK, BM, true));
  ENNX_TRY(make_tmap_2d_bf16(&tb, B, (uint64_t)K, (uint64_t)b_rows, (uint64_t)p->ldb, BK, brows, true));
  memset(&tc, 0, sizeof(tc));
  const bool bf16_out = epi == ENNX_B200_EPI_BF16 || epi == ENNX_B200_EPI_SWIGLU || epi == ENNX_B200_EPI_ROWSCALE;
  if (bf16_out) {
    const long long out_cols = epi == ENNX_B200_EPI_SWIGLU ? N / 2 : N;
    ENNX_TRY(make_tmap_2d_bf16(&tc, C, (uint64_t)out_cols, (uint64_t)M, (uint64_t)p->ldc, 32, 32, false));
  }

  Args a = make_args(p, C, bf16_out);
  a.err = device_error_word();
  if (!a.err) return set_error(ENNX_B200_CUDA_ERROR, "gemm: no device error word");

  int dev = 0;
  cudaGetDevice(&dev);
  if (!g_attr_set[dev]) {
    ENNX_CUDA(cudaFuncSetAttribute(gemm_bf16_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES),
              "gemm: set smem");
    ENNX_CUDA(cudaFuncSetAttribute(gemm_bf16_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES),
              "gemm: set smem (pair)");
    g_attr_set[dev] = true;
  }
  if (!pair) {
    long long tiles_bound = ((long long)M / BM + G) * a.n_tiles;
    int grid = sm_count();
    if (tiles_bound < grid) grid = (int)tiles_bound;
    gemm_bf16_kernel<false><<<grid, THREADS, SMEM_BYTES, st>>>(ta, tb, tc, a);
  } else {
    long long units_bound = ((long long)M / Geo<true>::TM + G) * a.n_tiles;
    long long clusters = sm_count() / 2;
    if (units_bound < clusters) clusters = units_bound;
    cudaLaunchConfig_t cfg;
    memset(&cfg, 0, sizeof(cfg));
    cfg.gridDim = dim3((unsigned)(2 * clusters));
    cfg.blockDim = dim3(THREADS);
    cfg.dynamicSmemBytes = SMEM_BYTES;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    ENNX_CUDA(cudaLaunchKernelEx(&cfg, gemm_bf16_kernel<true>, ta, tb, tc, a), "gemm pair launch");
  }
  ENNX_LAUNCH_CHECK("gemm launch");
  return ENNX_B200_OK;
}


int32_t gemm_bf16_perturbed(const ennx_b200_gemm_params* p, const uint16_t* A, const uint16_t* W, const uint16_t* E,
                            void* C, cudaStream_t st) {
  if (!p || !A || !W || !E) return set_error(ENNX_B200_INVALID_ARGUMENT, "gemm_perturbed: null argument");
  if (p->groups < 2 || p->groups % 2)
    return set_error(ENNX_B200_INVALID_ARGUMENT, "gemm_perturbed: groups must be 2 * pairs");
  ENNX_TRY(check_gemm(p, C));
  const int M = p->m, N = p->n, K = p->k;
  const int G = p->groups;
  const int epi = p->epilogue;
  if ((((uintptr_t)W | (uintptr_t)E) & 15u))
    return set_error(ENNX_B200_INVALID_ARGUMENT, "gemm_perturbed: W and E must be 16-byte aligned");
  if (G > 2 && p->b_group_rows < N)
    return set_error(ENNX_B200_INVALID_ARGUMENT, "gemm_perturbed: b_group_rows must be >= N");
  CUtensorMap ta, tw, te, tc;
  const long long b_rows = (long long)(G / 2 - 1) * p->b_group_rows + N;
  ENNX_TRY(make_tmap_2d_bf16_sw(&ta, A, (uint64_t)K, (uint64_t)M, (uint64_t)p->lda, PB_BK, BM, PB_SW));
  ENNX_TRY(make_tmap_2d_bf16_sw(&tw, W, (uint64_t)K, (uint64_t)b_rows, (uint64_t)p->ldb, PB_BK, BM, PB_SW));
  ENNX_TRY(make_tmap_2d_bf16_sw(&te, E, (uint64_t)K, (uint64_t)b_rows, (uint64_t)p->ldb, PB_BK, BM, PB_SW));
  memset(&tc, 0, sizeof(tc));  // no TMA stores in this kernel
  const bool bf16_out = epi == ENNX_B200_EPI_BF16 || epi == ENNX_B200_EPI_SWIGLU || epi == ENNX_B200_EPI_ROWSCALE;
  Args a = make_args(p, C, bf16_out);
  a.has_tmc = 0;  // epilogue: direct 16-byte stores (its shared memory went to the rings)
  a.err = device_error_word();
  if (!a.err) return set_error(ENNX_B200_CUDA_ERROR, "gemm_perturbed: no device error word");
  PbArgs pb;
  pb.pairs = G / 2;
  int dev = 0;
  cudaGetDevice(&dev);
  if (!g_pb_attr_set[dev]) {
    ENNX_CUDA(cudaFuncSetAttribute(gemm_pb_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, PB_SMEM_BYTES),
              "gemm_perturbed: set smem");
    g_pb_attr_set[dev] = true;
  }
  long long units_bound = ((long long)M / 256 + G) * a.n_tiles;
  long long clusters = sm_count() / 2;
  if (units_bound < clusters) clusters = units_bound;
  cudaLaunchConfig_t cfg;
  memset(&cfg, 0, sizeof(cfg));
  cfg.gridDim = dim3((unsigned)(2 * clusters));
  cfg.blockDim = dim3(PB_THREADS);
  cfg.dynamicSmemBytes = PB_SMEM_BYTES;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  ENNX_CUDA(cudaLaunchKernelEx(&cfg, gemm_pb_kernel, ta, tw, te, tc, a, pb), "gemm_perturbed launch");
  ENNX_LAUNCH_CHECK("gemm_perturbed launch");
  return ENNX_B200_OK;
}

}  // namespace ennx

extern "C" int32_t ennx_b200_gemm_bf16(const ennx_b200_gemm_params* p, const uint16_t* A, const uint16_t* B,
                                       void* C, void* stream) {
  return ennx::gemm_bf16(p, A, B, C, (cudaStream_t)stream);
}

extern "C" int32_t ennx_b200_gemm_bf16_perturbed(const ennx_b200_gemm_params* p, const uint16_t* A,
                                                 const uint16_t* W, const uint16_t* E, void* C, void* stream) {
  return ennx::gemm_bf16_perturbed(p, A, W, E, C, (cudaStream_t)stream);
}
