// attention.cu -- causal grouped-query attention on tcgen05 tensor cores.
//
// One CTA = 128 query rows of one (batch, query head), head dim 128; key/value
// tiles of 128 keys.  Warp roles:
//   warp 0      TMA producer: the Q tile once, K and V tiles into a two-slot
//               ring (128-byte swizzle, no multicast);
//   warp 1      one thread issues tcgen05.mma: S = Q K^T into one of two
//               128x128 fp32 TMEM buffers, then O += P V (P from shared
//               memory, V read MN-major) into a 128x128 fp32 TMEM accumulator;
//   warps 2..9  softmax: query row r (TMEM lane r) is shared by warps 2+r/32
//               and 6+r/32, each owning 64 of the 128 key columns.  They read
//               their half of the S row from TMEM, apply scale and the causal
//               mask, exchange the partial row maximum through shared memory
//               (64-thread named barrier), write P (bf16) into the swizzled
//               shared tile the next MMA consumes, and rescale their half of
//               the O row in TMEM only when the max grew by more than 2^8
//               (lazy rescale); at the end they combine the row sums and
//               normalise and store O.
// S(j+1) is computed while the softmax of tile j runs.  Every wait is bounded.
// No reference counterpart (the reference has no attention).
#include "common.cuh"
#include "kernels.cuh"

#include <string.h>

namespace ennx {
namespace {

constexpr int D = 128, BQ = 128, BKV = 128;
constexpr int SUB = 128 * 128;             // bytes of one 128-row x 64-column bf16 sub-tile
constexpr int TILE = 2 * SUB;              // 128 rows x 128 columns
constexpr int THREADS = 320;  // producer, MMA, 8 softmax warps
constexpr int SMEM = TILE /*Q*/ + 2 * TILE /*K*/ + 2 * TILE /*V*/ + 2 * TILE /*P*/ + 1024 + 2048;
constexpr uint32_t IDESC_QK = idesc_bf16_f32(128, 128);
constexpr uint32_t IDESC_PV = idesc_bf16_f32(128, 128) | (1u << 16);  // B (V) MN-major
constexpr float kRescaleThreshold = 8.0f;  // log2 units: rescale O only when the max grows by > 2^8

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

struct Bars {
  uint64_t q_full, kv_full[2], kv_free[2], s_full[2], s_free[2], p_full[2], o_done[2];
  uint32_t tmem_base;
  int abort_flag;
  float red[2][128];  // per-row partial max / sum exchanged by the two warps sharing a row
};
static_assert(sizeof(Bars) <= 2048, "barrier block must fit the reserved 2 KB");

__device__ __forceinline__ void named_bar_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

__global__ void __launch_bounds__(THREADS, 2)
    gqa_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                  const __grid_constant__ CUtensorMap tmV, uint16_t* __restrict__ o, long long ldo, int seq, int hq,
                  int hkv, int qcol0, int kcol0, int vcol0, float scale_log2, int* err) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* base = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  uint8_t* sQ = base;
  uint8_t* sK = sQ + TILE;
  uint8_t* sV = sK + 2 * TILE;
  uint8_t* sP = sV + 2 * TILE;
  Bars& bar = *reinterpret_cast<Bars*>(sP + 2 * TILE);

  const int nq = (seq + BQ - 1) / BQ;
  const int qt = nq - 1 - (int)blockIdx.x;  // heaviest (longest causal) tiles first
  const int h = blockIdx.y, b = blockIdx.z;
  const int kvh = h / (hq / hkv);
  const int q0 = qt * BQ;
  const int row_base = b * seq;  // token row of position 0 of this sequence
  const int ntiles = qt + 1;     // causal: key tiles 0 .. qt
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mbar_init(&bar.q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bar.kv_full[i], 1);
      mbar_init(&bar.kv_free[i], 1);
      mbar_init(&bar.s_full[i], 1);
      mbar_init(&bar.s_free[i], 8);
    }
    mbar_init(&bar.p_full[0], 8);
    mbar_init(&bar.p_full[1], 8);
    mbar_init(&bar.o_done[0], 1);
    mbar_init(&bar.o_done[1], 1);
    bar.abort_flag = 0;
    fence_barrier_init();
    fence_proxy_async();
  }
  if (warp == 1) { tmem_alloc(&bar.tmem_base, 512); tmem_relinquish(); }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bar.tmem_base;  // S[0]: cols 0..127, S[1]: 128..255, O: 256..383
  volatile int* abort_flag = &bar.abort_flag;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      mbar_arrive_expect_tx(&bar.q_full, TILE);
      tma_load_2d(sQ, &tmQ, &bar.q_full, qcol0 + h * D, row_base + q0);
      tma_load_2d(sQ + SUB, &tmQ, &bar.q_full, qcol0 + h * D + 64, row_base + q0);
      for (int j = 0; j < ntiles && !*abort_flag; ++j) {
        const int s = j & 1;
        if (!mbar_wait(&bar.kv_free[s], ((j >> 1) & 1) ^ 1u, err)) { *abort_flag = 1; break; }
        mbar_arrive_expect_tx(&bar.kv_full[s], 2 * TILE);
        const int krow = row_base + j * BKV;
        uint8_t* k = sK + s * TILE;
        uint8_t* v = sV + s * TILE;
        tma_load_2d(k, &tmK, &bar.kv_full[s], kcol0 + kvh * D, krow);
        tma_load_2d(k + SUB, &tmK, &bar.kv_full[s], kcol0 + kvh * D + 64, krow);
        tma_load_2d(v, &tmV, &bar.kv_full[s], vcol0 + kvh * D, krow);
        tma_load_2d(v + SUB, &tmV, &bar.kv_full[s], vcol0 + kvh * D + 64, krow);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      bool ok = mbar_wait(&bar.q_full, 0, err);
      const uint32_t qa = smem_u32(sQ), pa = smem_u32(sP);
      auto pv = [&](int j) -> bool {  // O += P(j) V(j)
        if (!mbar_wait(&bar.p_full[j & 1], (j >> 1) & 1, err)) return false;
        tc_fence_after();
        const uint32_t va = smem_u32(sV + (j & 1) * TILE);
        const uint32_t pj = pa + (j & 1) * TILE;
#pragma unroll
        for (int kk = 0; kk < BKV / 16; ++kk)
          umma_f16(tmem + 256, smem_desc_sw128(pj + (kk >> 2) * SUB + (kk & 3) * 32),
                   smem_desc_sw128_mn(va + kk * 2048, SUB), IDESC_PV, (j | kk) != 0);
        umma_commit(&bar.o_done[j & 1]);
        umma_commit(&bar.kv_free[j & 1]);
        return true;
      };
      for (int j = 0; ok && j < ntiles && !*abort_flag; ++j) {
        const int s = j & 1;
        if (!mbar_wait(&bar.kv_full[s], (j >> 1) & 1, err) ||
            !mbar_wait(&bar.s_free[s], ((j >> 1) & 1) ^ 1u, err)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t ka = smem_u32(sK + s * TILE);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          umma_f16(tmem + s * 128, smem_desc_sw128(qa + (kk >> 2) * SUB + (kk & 3) * 32),
                   smem_desc_sw128(ka + (kk >> 2) * SUB + (kk & 3) * 32), IDESC_QK, kk != 0);
        umma_commit(&bar.s_full[s]);
        if (j > 0 && !pv(j - 1)) { ok = false; break; }
      }
      if (ok && !*abort_flag) ok = pv(ntiles - 1);
      if (!ok) *abort_flag = 1;
    }
  } else {
    // softmax warps 2..9: TMEM lane quarter = warp % 4; each row is split between two warps
    const int q = warp & 3;
    const int half = (warp - 2) >> 2;  // columns [64*half, 64*half + 64) of S, O and P
    const int r = q * 32 + lane;
    const int qpos = q0 + r;
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    const int pair_bar = 1 + q;  // named barrier shared with the warp owning the other half of these rows
    float m = -INFINITY, l = 0.0f;
    bool ok = true;
    for (int j = 0; j < ntiles; ++j) {
      const int s = j & 1;
      if (!mbar_wait(&bar.s_full[s], (j >> 1) & 1, err)) { ok = false; break; }
      tc_fence_after();
      const int k0 = j * BKV;
      const bool diag = k0 + BKV - 1 > q0 || k0 + BKV > seq;  // warp-uniform: tile needs the causal / length mask
      // pass 1: row max of the scaled, masked scores (own 64 columns, then the partner's)
      float mt = -INFINITY;
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        const int c = 2 * half + cc;
        uint32_t v[32];
        tmem_ld32(tmem + lane_off + s * 128 + c * 32, v);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int kpos = k0 + c * 32 + i;
          float x = __uint_as_float(v[i]) * scale_log2;
          if (diag && (kpos > qpos || kpos >= seq)) x = -INFINITY;
          mt = fmaxf(mt, x);
        }
      }
      bar.red[half][r] = mt;
      named_bar_sync(pair_bar, 64);
      mt = fmaxf(mt, bar.red[half ^ 1][r]);
      named_bar_sync(pair_bar, 64);  // both read before the next tile overwrites
      const float m_new = fmaxf(m, mt);
      const bool rescale = m == -INFINITY ? true : (m_new > m + kRescaleThreshold);
      const float m_use = rescale ? m_new : m;
      const float alpha = (rescale && m != -INFINITY) ? exp2f(m - m_use) : 1.0f;
      // P buffer (j & 1) is free once PV(j-2) has completed
      if (j > 1 && !mbar_wait(&bar.o_done[j & 1], ((j - 2) >> 1) & 1, err)) { ok = false; break; }
      tc_fence_after();
      // pass 2: probabilities -> bf16 P, keys [64*half, +64) = sub-tile `half` of
      // the swizzled K-major tile (16-byte chunks XOR row % 8)
      float ls = 0.0f;
      const uint32_t prow = smem_u32(sP) + (j & 1) * TILE + half * SUB + r * 128;
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        const int c = 2 * half + cc;
        uint32_t v[32];
        tmem_ld32(tmem + lane_off + s * 128 + c * 32, v);
        tmem_ld_wait();
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int kp = k0 + c * 32 + 2 * i;
          float x0 = __uint_as_float(v[2 * i]) * scale_log2, x1 = __uint_as_float(v[2 * i + 1]) * scale_log2;
          float p0 = (m_use == -INFINITY || (diag && (kp > qpos || kp >= seq))) ? 0.0f : ex2(x0 - m_use);
          float p1 = (m_use == -INFINITY || (diag && (kp + 1 > qpos || kp + 1 >= seq))) ? 0.0f : ex2(x1 - m_use);
          ls += p0 + p1;
          pk[i] = pack_bf16x2(p0, p1);
        }
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          const int cch = cc * 4 + g;  // 16-byte chunk (8 keys) within this 64-key sub-tile row
          const uint32_t addr = prow + ((cch ^ (r & 7)) << 4);
          asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(pk[4 * g]), "r"(pk[4 * g + 1]),
                       "r"(pk[4 * g + 2]), "r"(pk[4 * g + 3])
                       : "memory");
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar.s_free[s]);
      l = l * alpha + ls;
      m = m_use;
      if (j > 0 && __any_sync(0xffffffffu, alpha != 1.0f)) {
        // O must hold PV(j-1) before it is rescaled
        if (!mbar_wait(&bar.o_done[(j - 1) & 1], ((j - 1) >> 1) & 1, err)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
          const int c = 2 * half + cc;
          uint32_t v[32];
          tmem_ld32(tmem + lane_off + 256 + c * 32, v);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = __float_as_uint(__uint_as_float(v[i]) * alpha);
          tmem_st32(tmem + lane_off + 256 + c * 32, v);
        }
        tmem_st_wait();
      }
      fence_proxy_async();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar.p_full[j & 1]);
    }
    // row sum over both halves
    bar.red[half][r] = l;
    named_bar_sync(pair_bar, 64);
    const float l_tot = l + bar.red[half ^ 1][r];
    if (ok && mbar_wait(&bar.o_done[(ntiles - 1) & 1], ((ntiles - 1) >> 1) & 1, err)) {
      tc_fence_after();
      const float inv = l_tot > 0.0f ? 1.0f / l_tot : 0.0f;
      uint16_t* orow = o + (long long)(row_base + qpos) * ldo + h * D;
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        const int c = 2 * half + cc;
        uint32_t v[32];
        tmem_ld32(tmem + lane_off + 256 + c * 32, v);
        tmem_ld_wait();
        if (qpos < seq) {
#pragma unroll
          for (int g = 0; g < 4; ++g)
            st_global_v4(orow + c * 32 + g * 8,
                         pack_bf16x2(__uint_as_float(v[8 * g]) * inv, __uint_as_float(v[8 * g + 1]) * inv),
                         pack_bf16x2(__uint_as_float(v[8 * g + 2]) * inv, __uint_as_float(v[8 * g + 3]) * inv),
                         pack_bf16x2(__uint_as_float(v[8 * g + 4]) * inv, __uint_as_float(v[8 * g + 5]) * inv),
                         pack_bf16x2(__uint_as_float(v[8 * g + 6]) * inv, __uint_as_float(v[8 * g + 7]) * inv));
        }
      }
    } else {
      *abort_flag = 1;
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
  dim3 grid((seq + BQ - 1) / BQ, hq, batch);
  const float scale_log2 = 1.4426950408889634f / sqrtf((float)D);
  gqa_tc_kernel<<<grid, THREADS, SMEM, s>>>(tq, tk, tv, o, ldo, seq, hq, hkv, 0, 0, 0, scale_log2, err);
  ENNX_LAUNCH_CHECK("gqa attention");
  return ENNX_B200_OK;
}

}  // namespace ennx
