// attention.cu -- causal grouped-query attention on tcgen05 tensor cores.
//
// One CTA = two 128-row query tiles (A: rows q0..q0+127, B: q0+128..q0+255)
// of one (batch, query head), head dim 128; key/value tiles of 128 keys
// shared by both query tiles.  Tensor memory: S_A | O_A | S_B | O_B, 128 fp32
// columns each.  Warp roles:
//   warp 0       TMA producer: both Q tiles once, K and V tiles into a
//                two-slot ring (128-byte swizzle, no multicast);
//   warp 1       one thread issues tcgen05.mma: S_X = Q_X K^T into S_X, and
//                O_X += P_X V with P_X read from TENSOR memory (the A operand
//                of the MMA; P_X is written over the first 64 columns of S_X
//                as packed bf16 pairs) and V read MN-major from shared memory;
//                the two tiles alternate so the MMAs of one tile run while
//                the other tile's softmax runs;
//   warps 2..17  softmax, eight warps per query tile: TMEM lane quarter =
//                warp % 4, and each query row is split between two warps
//                owning 64 key columns each.  A warp reads its 64 scores from
//                TMEM once, applies scale and the causal mask, exchanges the
//                partial row maximum with its partner (64-thread named
//                barrier), keeps the running max in the exp2 domain, writes P
//                into tensor memory, and rescales its half of the O row only
//                when the max grew by more than 2^8 (lazy rescale); at the end
//                it combines the row sums and normalises and stores O.
// Ordering: the MMAs of one thread execute in issue order, so S_X(j+1),
// issued after O_X += P_X(j) V(j), overwrites P_X(j) only after that MMA has
// read it; the commit that publishes S_X(j+1) also proves PV_X(j) complete.
// Every wait is bounded.  No reference counterpart (the reference has no
// attention).
#include "common.cuh"
#include "kernels.cuh"

#include <string.h>

namespace ennx {
namespace {

constexpr int D = 128, BQ = 128, BKV = 128;
constexpr int SUB = 128 * 128;             // bytes of one 128-row x 64-column bf16 sub-tile
constexpr int TILE = 2 * SUB;              // 128 rows x 128 columns
constexpr int SOFTMAX_WARPS = 16;
constexpr int THREADS = 64 + 32 * SOFTMAX_WARPS;  // producer, MMA, 2 x 8 softmax warps
constexpr int SMEM = 2 * TILE /*Q_A, Q_B*/ + 2 * TILE /*K*/ + 2 * TILE /*V*/ + 1024 + 5120;
constexpr uint32_t IDESC_QK = idesc_bf16_f32(128, 128);
constexpr uint32_t IDESC_PV = idesc_bf16_f32(128, 128) | (1u << 16);  // B (V) MN-major
constexpr float kRescaleThreshold = 8.0f;  // log2 units: rescale O only when the max grows by > 2^8

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// D[tmem] (+)= A[tmem] * B[smem desc]^T, kind::f16 (A: M lanes x K, 16-bit
// elements packed in pairs per 32-bit column).
__device__ __forceinline__ void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ uint64_t pack_f32x2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ uint64_t fma_f32x2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t add_f32x2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

__device__ __forceinline__ void named_bar_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

struct Bars {
  uint64_t q_full, kv_full[2], kv_free[2], s_full[2], p_full[2], o_done[2];
  uint32_t tmem_base;
  int abort_flag;
  // [tile][parity of the key tile][half][row]: partial row max / sum exchanged
  // by the two warps of a row; double-buffered so one barrier per tile suffices
  float red[2][2][2][128];
};
static_assert(sizeof(Bars) <= 5120, "barrier block must fit the reserved 5 KB");

__global__ void __launch_bounds__(THREADS, 1)
    gqa_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                  const __grid_constant__ CUtensorMap tmV, uint16_t* __restrict__ o, long long ldo, int seq, int hq,
                  int hkv, float scale_log2, int* err) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* base = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  uint8_t* sQ = base;               // [2] tiles
  uint8_t* sK = sQ + 2 * TILE;      // [2] ring slots
  uint8_t* sV = sK + 2 * TILE;      // [2] ring slots
  Bars& bar = *reinterpret_cast<Bars*>(sV + 2 * TILE);

  const int nblk = (seq + 2 * BQ - 1) / (2 * BQ);
  const int qb = nblk - 1 - (int)blockIdx.x;  // heaviest (longest causal) blocks first
  const int h = blockIdx.y, b = blockIdx.z;
  const int kvh = h / (hq / hkv);
  const int q0 = qb * 2 * BQ;
  const int row_base = b * seq;  // token row of position 0 of this sequence
  // causal: tile A needs key tiles 0 .. q0/128, tile B one more; B may be empty
  const int nt[2] = {q0 / BKV + 1, q0 + BQ < seq ? q0 / BKV + 2 : 0};
  const int nt_max = nt[1] > 0 ? nt[1] : nt[0];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mbar_init(&bar.q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bar.kv_full[i], 1);
      mbar_init(&bar.kv_free[i], 1);
      mbar_init(&bar.s_full[i], 1);
      mbar_init(&bar.p_full[i], 8);
      mbar_init(&bar.o_done[i], 1);
    }
    bar.abort_flag = 0;
    fence_barrier_init();
    fence_proxy_async();
  }
  if (warp == 1) { tmem_alloc(&bar.tmem_base, 512); tmem_relinquish(); }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bar.tmem_base;  // S_A: 0, O_A: 128, S_B: 256, O_B: 384
  volatile int* abort_flag = &bar.abort_flag;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      const int nq = nt[1] > 0 ? 2 : 1;
      mbar_arrive_expect_tx(&bar.q_full, nq * TILE);
      for (int x = 0; x < nq; ++x) {
        tma_load_2d(sQ + x * TILE, &tmQ, &bar.q_full, h * D, row_base + q0 + x * BQ);
        tma_load_2d(sQ + x * TILE + SUB, &tmQ, &bar.q_full, h * D + 64, row_base + q0 + x * BQ);
      }
      for (int j = 0; j < nt_max && !*abort_flag; ++j) {
        const int s = j & 1;
        if (!mbar_wait(&bar.kv_free[s], ((j >> 1) & 1) ^ 1u, err)) { *abort_flag = 1; break; }
        mbar_arrive_expect_tx(&bar.kv_full[s], 2 * TILE);
        const int krow = row_base + j * BKV;
        uint8_t* k = sK + s * TILE;
        uint8_t* v = sV + s * TILE;
        tma_load_2d(k, &tmK, &bar.kv_full[s], kvh * D, krow);
        tma_load_2d(k + SUB, &tmK, &bar.kv_full[s], kvh * D + 64, krow);
        tma_load_2d(v, &tmV, &bar.kv_full[s], kvh * D, krow);
        tma_load_2d(v + SUB, &tmV, &bar.kv_full[s], kvh * D + 64, krow);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      auto s_mma = [&](int x, int j) -> bool {  // S_X = Q_X K(j)^T
        if (!mbar_wait(&bar.kv_full[j & 1], (j >> 1) & 1, err)) return false;
        tc_fence_after();
        const uint32_t qa = smem_u32(sQ + x * TILE), ka = smem_u32(sK + (j & 1) * TILE);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          umma_f16(tmem + x * 256, smem_desc_sw128(qa + (kk >> 2) * SUB + (kk & 3) * 32),
                   smem_desc_sw128(ka + (kk >> 2) * SUB + (kk & 3) * 32), IDESC_QK, kk != 0);
        umma_commit(&bar.s_full[x]);
        return true;
      };
      bool ok = mbar_wait(&bar.q_full, 0, err);
      for (int x = 0; ok && x < 2; ++x)
        if (nt[x] > 0) ok = s_mma(x, 0);
      for (int j = 0; ok && j < nt_max && !*abort_flag; ++j) {
        for (int x = 0; x < 2; ++x) {
          if (j >= nt[x]) continue;
          // O_X += P_X(j) V(j), P_X in tensor memory over the first 64 columns of S_X
          if (!mbar_wait(&bar.p_full[x], j & 1, err)) { ok = false; break; }
          tc_fence_after();
          const uint32_t va = smem_u32(sV + (j & 1) * TILE);
#pragma unroll
          for (int kk = 0; kk < BKV / 16; ++kk)
            umma_f16_ts(tmem + x * 256 + 128, tmem + x * 256 + kk * 8, smem_desc_sw128_mn(va + kk * 2048, SUB),
                        IDESC_PV, (j | kk) != 0);
          umma_commit(&bar.o_done[x]);
          const bool last_user = x == 1 || j >= nt[1];
          if (last_user) umma_commit(&bar.kv_free[j & 1]);
          if (j + 1 < nt[x] && !s_mma(x, j + 1)) { ok = false; break; }
        }
      }
      if (!ok) *abort_flag = 1;
    }
  } else {
    // softmax: tile x, TMEM lane quarter q = warp % 4, key-column half `half`
    const int x = (warp - 2) >> 3;
    const int q = warp & 3;
    const int half = ((warp - 2) >> 2) & 1;
    const int r = q * 32 + lane;
    const int qx0 = q0 + x * BQ;
    const int qpos = qx0 + r;
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    const uint32_t s_col = tmem + lane_off + x * 256;  // S_X (P_X over its first 64 columns)
    const uint32_t o_col = s_col + 128;                 // O_X
    const int pair_bar = 1 + 4 * x + q;                 // shared with the warp owning the other half of these rows
    float m = -INFINITY, l = 0.0f;
    bool ok = true;
    for (int j = 0; j < nt[x]; ++j) {
      // A failed (timed-out) wait does not leave the loop: the warp keeps
      // meeting its partner at the named barrier, which has no timeout, and
      // skips the work; the abort flag stops every other wait early.
      if (ok) ok = !*abort_flag && mbar_wait(&bar.s_full[x], j & 1, err);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) *abort_flag = 1;
      tc_fence_after();
      const int k0 = j * BKV + half * 64;
      const bool diag = k0 + 63 > qx0 || k0 + 64 > seq;  // warp-uniform: this half needs the causal / length mask
      uint32_t v0[32], v1[32];
      if (ok) {
        tmem_ld32(s_col + half * 64, v0);
        tmem_ld32(s_col + half * 64 + 32, v1);
        tmem_ld_wait();
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) v0[i] = v1[i] = 0xff800000u;
      }
      if (diag) {
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          if (k0 + i > qpos || k0 + i >= seq) v0[i] = 0xff800000u;  // -inf
          if (k0 + 32 + i > qpos || k0 + 32 + i >= seq) v1[i] = 0xff800000u;
        }
      }
      // row max of the raw scores (the positive scale commutes with max)
      float mt = -INFINITY;
#pragma unroll
      for (int i = 0; i < 32; ++i) mt = fmaxf(mt, fmaxf(__uint_as_float(v0[i]), __uint_as_float(v1[i])));
      mt *= scale_log2;
      // buffer j & 1: the partner's read of this slot two tiles ago preceded
      // its arrival at the barrier of the tile in between
      bar.red[x][j & 1][half][r] = mt;
      named_bar_sync(pair_bar, 64);  // also: both halves have read S before P overwrites it
      mt = fmaxf(mt, bar.red[x][j & 1][half ^ 1][r]);
      if (!ok) continue;  // after the barrier: nothing below waits on the partner
      const float m_new = fmaxf(m, mt);
      const bool rescale = m == -INFINITY ? true : (m_new > m + kRescaleThreshold);
      const float m_use = rescale ? m_new : m;
      const float alpha = (rescale && m != -INFINITY) ? ex2(m - m_use) : 1.0f;
      // P = exp2(s * scale - m) as one packed fma per pair of scores; a row
      // with no unmasked score so far uses m = 0 (every exp2 argument is -inf)
      const float nm = m_use == -INFINITY ? 0.0f : -m_use;
      const uint64_t c2 = pack_f32x2(scale_log2, scale_log2), nm2 = pack_f32x2(nm, nm);
      uint64_t ls2 = 0ull;
      uint32_t pk[32];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const uint64_t t01 = fma_f32x2(((uint64_t)v0[2 * i + 1] << 32) | v0[2 * i], c2, nm2);
        const uint64_t t23 = fma_f32x2(((uint64_t)v1[2 * i + 1] << 32) | v1[2 * i], c2, nm2);
        const float p0 = ex2(__uint_as_float((uint32_t)t01)), p1 = ex2(__uint_as_float((uint32_t)(t01 >> 32)));
        const float p2 = ex2(__uint_as_float((uint32_t)t23)), p3 = ex2(__uint_as_float((uint32_t)(t23 >> 32)));
        ls2 = add_f32x2(ls2, add_f32x2(pack_f32x2(p0, p1), pack_f32x2(p2, p3)));
        pk[i] = pack_bf16x2(p0, p1);
        pk[16 + i] = pack_bf16x2(p2, p3);
      }
      const float ls = __uint_as_float((uint32_t)ls2) + __uint_as_float((uint32_t)(ls2 >> 32));
      tmem_st32(s_col + half * 32, pk);
      l = l * alpha + ls;
      m = m_use;
      if (j > 0 && __any_sync(0xffffffffu, alpha != 1.0f)) {
        // the s_full wait above proves O_X += P_X(j-1) V(j-1) complete
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
          uint32_t ov[32];
          tmem_ld32(o_col + half * 64 + cc * 32, ov);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) ov[i] = __float_as_uint(__uint_as_float(ov[i]) * alpha);
          tmem_st32(o_col + half * 64 + cc * 32, ov);
        }
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar.p_full[x]);
    }
    if (nt[x] > 0) {
      // row sum over both halves
      bar.red[x][nt[x] & 1][half][r] = l;
      named_bar_sync(pair_bar, 64);
      const float l_tot = l + bar.red[x][nt[x] & 1][half ^ 1][r];
      if (ok && mbar_wait(&bar.o_done[x], (nt[x] - 1) & 1, err)) {
        tc_fence_after();
        const float inv = l_tot > 0.0f ? 1.0f / l_tot : 0.0f;
        uint16_t* orow = o + (long long)(row_base + qpos) * ldo + h * D + half * 64;
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
          uint32_t ov[32];
          tmem_ld32(o_col + half * 64 + cc * 32, ov);
          tmem_ld_wait();
          if (qpos < seq) {
#pragma unroll
            for (int g = 0; g < 4; ++g)
              st_global_v4(orow + cc * 32 + g * 8,
                           pack_bf16x2(__uint_as_float(ov[8 * g]) * inv, __uint_as_float(ov[8 * g + 1]) * inv),
                           pack_bf16x2(__uint_as_float(ov[8 * g + 2]) * inv, __uint_as_float(ov[8 * g + 3]) * inv),
                           pack_bf16x2(__uint_as_float(ov[8 * g + 4]) * inv, __uint_as_float(ov[8 * g + 5]) * inv),
                           pack_bf16x2(__uint_as_float(ov[8 * g + 6]) * inv, __uint_as_float(ov[8 * g + 7]) * inv));
          }
        }
      } else {
        *abort_flag = 1;
      }
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

bool g_attr[64];

}  // namespace

int32_t launch_gqa_attention(const uint16_t* q, long long ldq, const uint16_t* k, long long ldk, const uint16_t* v,
                             long long ldv, uint16_t* o, long long ldo, int batch, int seq, int hq, int hkv,
                             cudaStream_t s) {
  if (hkv <= 0 || hq % hkv) return set_error(ENNX_B200_INVALID_ARGUMENT, "attention: Hq must be a multiple of Hkv");
  if (seq <= 0 || batch <= 0) return set_error(ENNX_B200_INVALID_ARGUMENT, "attention: empty input");
  if ((ldq | ldk | ldv | ldo) % 8 || (((uintptr_t)q | (uintptr_t)k | (uintptr_t)v | (uintptr_t)o) & 15u))
    return set_error(ENNX_B200_INVALID_ARGUMENT, "attention: operands must be 16-byte aligned");
  const long long rows = (long long)batch * seq;
  if (rows > 0x7fffffffLL) return set_error(ENNX_B200_UNSUPPORTED, "attention: too many tokens");
  // tensor maps over the whole [rows, ld] buffers; heads are column offsets
  CUtensorMap tq, tk, tv;
  ENNX_TRY(make_tmap_2d_bf16(&tq, q, (uint64_t)hq * D, (uint64_t)rows, (uint64_t)ldq, 64, 128, true));
  ENNX_TRY(make_tmap_2d_bf16(&tk, k, (uint64_t)hkv * D, (uint64_t)rows, (uint64_t)ldk, 64, 128, true));
  ENNX_TRY(make_tmap_2d_bf16(&tv, v, (uint64_t)hkv * D, (uint64_t)rows, (uint64_t)ldv, 64, 128, true));
  int* err = device_error_word();
  if (!err) return set_error(ENNX_B200_CUDA_ERROR, "attention: no device error word");
  int dev = 0;
  cudaGetDevice(&dev);
  if (!g_attr[dev]) {
    ENNX_CUDA(cudaFuncSetAttribute(gqa_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM), "attn smem");
    g_attr[dev] = true;
  }
  dim3 grid((seq + 2 * BQ - 1) / (2 * BQ), hq, batch);
  const float scale_log2 = 1.4426950408889634f / sqrtf((float)D);
  gqa_tc_kernel<<<grid, THREADS, SMEM, s>>>(tq, tk, tv, o, ldo, seq, hq, hkv, scale_log2, err);
  ENNX_LAUNCH_CHECK("gqa attention");
  return ENNX_B200_OK;
}

}  // namespace ennx
