// kda.cu -- chunked KDA (gated delta rule with per-key-channel decay) on
// tcgen05 tensor cores.
//
// Recurrence (restated from rust/crates/ennx/src/kda_moe.metal:167-225):
//   S_t = diag(exp g_t) S_{t-1};  u_t = beta_t (v_t - k_t^T S_t);
//   S_t += k_t u_t^T;  o_t = q_t^T S_t / sqrt(dk)
// The reference runs it token by token.  Here it is evaluated in chunks of
// C = 64 tokens (WY form).  With Gc_t the inclusive cumulative log decay of
// the chunk and S0 the state entering it:
//   A'[t,s] = sum_i k_t[i] k_s[i] exp(Gc_t[i] - Gc_s[i])          (s < t)
//   U = (I + diag(beta) A')^-1 diag(beta) (V - (K o e^Gc) S0)
//   O = ((Q o e^Gc) S0 + QK U) / sqrt(dk),  QK[t,s] likewise for s <= t
//   S_C = diag(e^Gc_C) S0 + (K o e^(Gc_C - Gc))^T U
// The per-channel exp(Gc_t - Gc_s) is factored through a reference token r
// (first token of t's 16-token block): both factors stay bounded for s <= t
// because each step decays by at most e^-5.
//
// Two kernels:
//   kda_prep_kernel -- one CTA per (sequence, head, chunk), all in parallel.
//     Builds, straight from registers, the decay-scaled operands
//     K~ = K o e^Gc, Q~ = Q o e^Gc, K^ = K o e^(Gc_C - Gc) (to the chunk
//     record) and, in shared memory, the intra-chunk MMA operands
//       A   = [Q o e^(Gc - Gc_r); K o e^(Gc - Gc_r)]        (128 x 128)
//       B_b = K[0 : 16(b+1)] o e^(Gc_{r_b} - Gc)            (block b = 0..3)
//     and runs the four intra-chunk products D_b = A B_b^T on tcgen05 with
//     fp32 accumulators in TMEM: rows 0..63 of D_b give QK, rows 64..127
//     give A', each read for the rows of block b.  Then
//     T = (I + diag(beta) A')^-1 diag(beta) in fp32 on the CUDA cores
//     (blocked: 16x16 diagonal inverses, then 32x32, then 64x64).
//   kda_scan_kernel -- one CTA per (sequence, head) walks the chunks in order
//     in transposed form, TMEM lane = value column v:
//       X^T = S^T K~^T, O^T = S^T Q~^T              (one MMA, N = 128)
//       X^T = V^T - X^T  -> bf16 smem
//       U^T = X^T T^T                               (MMA)
//       O^T += U^T QK^T;  S^T = S^T diag(e^Gc_C) + U^T K^   (MMAs)
//     The fp32 state S^T lives in TMEM for the whole sequence; a bf16 copy
//     in shared memory is the A operand of the next chunk.  Chunk records
//     and V tiles arrive by TMA (no multicast) through a producer warp; one
//     thread issues the MMAs; eight warps do the element-wise steps.
// Every wait is bounded.
#include "common.cuh"
#include "kernels.cuh"

#include <string.h>

namespace ennx {
namespace {

constexpr int C = 64, DK = 128;
constexpr int LF = C + 1;  // padded fp32 row of [64][64] matrices
constexpr float kLog2e = 1.4426950408889634f;

// Chunk records (workspace), as three arrays so that each is a plain 2-D
// tensor for TMA:
//   BIG   [R * 192][128] bf16 : rows 192r + [0,64) K~, [64,128) Q~, [128,192) K^
//   SMALL [R * 128][64]  bf16 : rows 128r + [0,64) T diag(beta), [64,128) QK
//   DEND  [R][128]       fp32 : e^Gc_C
constexpr size_t kBigRecBytes = 192ull * DK * 2;
constexpr size_t kSmallRecBytes = 128ull * C * 2;
constexpr size_t kDendRecBytes = DK * 4;
constexpr size_t kChunkBytes = kBigRecBytes + kSmallRecBytes + kDendRecBytes;

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

// byte offset of the 16-byte chunk `c` (0..7) of row `r` in a 128-byte-swizzled
// K-major tile (rows of 128 bytes, chunk index XOR row % 8)
__device__ __forceinline__ uint32_t sw128(int r, int c) { return (uint32_t)(r * 128 + ((c ^ (r & 7)) << 4)); }

__device__ __forceinline__ void unpack8(uint4 v, float f[8]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    f[2 * j] = bf16_to_f32((uint16_t)(w[j] & 0xffffu));
    f[2 * j + 1] = bf16_to_f32((uint16_t)(w[j] >> 16));
  }
}
__device__ __forceinline__ uint4 pack8(const float f[8]) {
  return make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]), pack_bf16x2(f[4], f[5]),
                    pack_bf16x2(f[6], f[7]));
}

// ===========================================================================
// prep: one CTA per (sequence, head, chunk)
// ===========================================================================
constexpr int PREP_THREADS = 256;
constexpr int P_XA = 0;                    // A operand, 2 sub-tiles of 128 rows x 128 B
constexpr int P_YB = 32768;                // B_b operands, 16(b+1) rows each, 2 sub-tiles
constexpr int P_GC = P_YB + 40960;         // fp32 [64][128] log2 decay, then in-block products X
constexpr int P_FB = P_GC + C * DK * 4;    // fp32 [4][128] block-to-block decay factors
constexpr int P_EB = P_FB + 4 * DK * 4;    // fp32 [4][128] 2^Gc at each block's reference token
constexpr int P_SB = P_EB + 4 * DK * 4;    // fp32 [4][128] 2^(Gc_C - Gc) at each block's reference token
constexpr int P_BETA = P_SB + 4 * DK * 4;  // fp32 [64]
// scratch of the decay-factor phase, in the B operand region (written later)
constexpr int P_AR = P_YB;                 // fp32 [4][128] per-step factor of each reference token
constexpr int P_XE = P_YB + 4 * DK * 4;    // fp32 [4][128] in-block product at each block's last token
constexpr int P_BAR = P_BETA + C * 4;      // mbarrier + TMEM slot
constexpr int PREP_SMEM = P_BAR + 64 + 1024;
// after the MMAs complete, the A operand region holds L (then T) and the B
// operand region the temporaries of the inverse
constexpr int P_L = P_XA;
static_assert(C * LF * 4 <= P_YB - P_XA, "L must fit the A operand region");
static_assert(2 * (PREP_SMEM + 1024) <= 232448, "two prep CTAs per SM");
static_assert(2 * 16 * 17 * 4 <= 40960 && 32 * 33 * 4 <= 40960, "inverse temporaries must fit the B region");

__host__ __device__ constexpr int yb_off(int b) { return P_YB + 4096 * (b * (b + 1) / 2); }
__host__ __device__ constexpr int yb_rows(int b) { return 16 * (b + 1); }
__host__ __device__ constexpr int d_col(int b) { return 8 * b * (b + 1); }  // TMEM column of D_b

// max(x, 0) + log(1 + e^-|x|) on the SFU (log2 / exp2 approximations)
__device__ __forceinline__ float softplus_stable(float x) { return fmaxf(x, 0.0f) + __logf(1.0f + __expf(-fabsf(x))); }
__device__ __forceinline__ float rcp_approx(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__global__ void __launch_bounds__(PREP_THREADS, 2)
    kda_prep_kernel(const uint16_t* __restrict__ qg, const uint16_t* __restrict__ kg, long long ld,
                    const float* __restrict__ gg, long long ldg, const float* __restrict__ bg, int seq, int heads,
                    int nchunks, KdaRawGate raw, uint16_t* __restrict__ big, uint16_t* __restrict__ small,
                    float* __restrict__ dend, int* err) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* sm = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  float(*Gc)[DK] = reinterpret_cast<float(*)[DK]>(sm + P_GC);
  float(*fb)[DK] = reinterpret_cast<float(*)[DK]>(sm + P_FB);
  float* beta = reinterpret_cast<float*>(sm + P_BETA);
  uint64_t* mma_done = reinterpret_cast<uint64_t*>(sm + P_BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + P_BAR + 8);

  const int ch = blockIdx.x, bh = blockIdx.y, b = bh / heads, h = bh % heads;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const long long tok0 = (long long)b * seq;
  const int t0 = ch * C;
  const size_t rec = (size_t)bh * nchunks + ch;
  uint16_t* bigr = big + rec * (192 * DK);
  uint16_t* smallr = small + rec * (128 * C);

  if (tid == 0) {
    mbar_init(mma_done, 1);
    fence_barrier_init();
  }
  if (warp == 0) { tmem_alloc(tmem_slot, 256); tmem_relinquish(); }

  // ---- gates: log2 decay per (token, channel) and beta ----
  if (raw.active) {
    // g = max(-exp(decay_h) * softplus(f + time_bias), -5) and beta =
    // sigmoid(raw beta) from the raw projections (kda_moe.metal:869-895)
    const bool set0 = b < raw.split_seq;
    const uint16_t* tb = set0 ? raw.tb0 : raw.tb1;
    const float dscale = __expf(bf16_to_f32((set0 ? raw.decay0 : raw.decay1)[h]));
#pragma unroll
    for (int i = tid; i < C * (DK / 8); i += PREP_THREADS) {
      const int r = i >> 4, c = (i & 15) * 8;
      float gv[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      if (t0 + r < seq) {
        float fv[8], bv[8];
        unpack8(*reinterpret_cast<const uint4*>(raw.f + (tok0 + t0 + r) * raw.ldf + h * DK + c), fv);
        unpack8(*reinterpret_cast<const uint4*>(tb + h * DK + c), bv);
#pragma unroll
        for (int j = 0; j < 8; ++j) gv[j] = fmaxf(-dscale * softplus_stable(fv[j] + bv[j]), -5.0f) * kLog2e;
      }
      *reinterpret_cast<float4*>(&Gc[r][c]) = make_float4(gv[0], gv[1], gv[2], gv[3]);
      *reinterpret_cast<float4*>(&Gc[r][c + 4]) = make_float4(gv[4], gv[5], gv[6], gv[7]);
    }
    if (tid < C)
      beta[tid] = t0 + tid < seq ? 1.0f / (1.0f + __expf(-bf16_to_f32(raw.rbeta[(tok0 + t0 + tid) * raw.ldb + h])))
                                 : 0.0f;
  } else {
#pragma unroll
    for (int i = tid; i < C * (DK / 4); i += PREP_THREADS) {
      const int r = i >> 5, c = (i & 31) * 4;
      float4 gv = make_float4(0.f, 0.f, 0.f, 0.f);
      if (t0 + r < seq) gv = *reinterpret_cast<const float4*>(gg + (tok0 + t0 + r) * ldg + h * DK + c);
      *reinterpret_cast<float4*>(&Gc[r][c]) =
          make_float4(gv.x * kLog2e, gv.y * kLog2e, gv.z * kLog2e, gv.w * kLog2e);
    }
    if (tid < C) beta[tid] = t0 + tid < seq ? bg[(tok0 + t0 + tid) * heads + h] : 0.0f;
  }
  __syncthreads();
  // ---- decay factors in product form: per step a_t = 2^(g_t log2 e);
  // within each 16-token block b (reference token r_b = 16b) the running
  // product X_t = 2^(Gc_t - Gc_r) (X_r = 1, >= 2^-108 for g >= -5), and per
  // block the scalars 2^Gc_r (Eb), 2^(Gc_C - Gc_r) (Sb) and the block-to-block
  // factor fb.  Thread (channel, half) owns the two blocks of its half.
  {
    float(*Ar)[DK] = reinterpret_cast<float(*)[DK]>(sm + P_AR);
    float(*Xe)[DK] = reinterpret_cast<float(*)[DK]>(sm + P_XE);
    const int c = tid & 127, half = tid >> 7;
    float x[32];
#pragma unroll
    for (int t = 0; t < 32; ++t) x[t] = ex2(Gc[half * 32 + t][c]);
#pragma unroll
    for (int b2 = 0; b2 < 2; ++b2) {
      Ar[2 * half + b2][c] = x[16 * b2];
      x[16 * b2] = 1.0f;
#pragma unroll
      for (int t = 1; t < 16; ++t) x[16 * b2 + t] = fmaxf(x[16 * b2 + t] * x[16 * b2 + t - 1], 7.52316e-37f);  // >= 2^-120
      Xe[2 * half + b2][c] = x[16 * b2 + 15];
    }
#pragma unroll
    for (int t = 0; t < 32; ++t) Gc[half * 32 + t][c] = x[t];  // Gc now holds X
    __syncthreads();
    if (tid < DK) {
      float(*Eb)[DK] = reinterpret_cast<float(*)[DK]>(sm + P_EB);
      float(*Sb)[DK] = reinterpret_cast<float(*)[DK]>(sm + P_SB);
      float f[4];
#pragma unroll
      for (int bb = 1; bb < 4; ++bb) f[bb] = Xe[bb - 1][tid] * Ar[bb][tid];  // 2^(Gc_r(bb) - Gc_r(bb-1))
      float e = Ar[0][tid];
      Eb[0][tid] = e;
#pragma unroll
      for (int bb = 1; bb < 4; ++bb) { e *= f[bb]; Eb[bb][tid] = e; fb[bb][tid] = f[bb]; }
      dend[rec * DK + tid] = e * Xe[3][tid];
      float sv = Xe[3][tid];
      Sb[3][tid] = sv;
#pragma unroll
      for (int bb = 2; bb >= 0; --bb) { sv *= f[bb + 1]; Sb[bb][tid] = sv; }
    }
    __syncthreads();
  }

  // ---- operands: a half-warp per token row, one 8-channel chunk per lane;
  // the q/k loads of the next row run one iteration ahead ----
  auto load_qk = [&](int it, uint4& qv, uint4& kv) {
    const int t = it * (PREP_THREADS / 16) + (tid >> 4), c0 = (tid & 15) * 8;
    qv = kv = make_uint4(0, 0, 0, 0);
    if (t0 + t < seq) {
      qv = __ldg(reinterpret_cast<const uint4*>(qg + (tok0 + t0 + t) * ld + h * DK + c0));
      kv = __ldg(reinterpret_cast<const uint4*>(kg + (tok0 + t0 + t) * ld + h * DK + c0));
    }
  };
  uint4 qn, kn;
  load_qk(0, qn, kn);
#pragma unroll 1
  for (int it = 0; it < C * 16 / PREP_THREADS; ++it) {
    const int t = it * (PREP_THREADS / 16) + (tid >> 4), cc = tid & 15, c0 = cc * 8;
    const int blk = t >> 4;
    float q[8], k[8];
    unpack8(qn, q);
    unpack8(kn, k);
    if (it + 1 < C * 16 / PREP_THREADS) load_qk(it + 1, qn, kn);
    if (raw.active && !raw.no_l2norm) {
      // per-token L2 normalisation, 1/max(|x|, 1e-6), rounded to bf16 (kda_moe.metal:510-534)
      float sq = 0.0f, sk = 0.0f;
#pragma unroll
      for (int j = 0; j < 8; ++j) { sq += q[j] * q[j]; sk += k[j] * k[j]; }
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) {
        sq += __shfl_xor_sync(0xffffffffu, sq, o);
        sk += __shfl_xor_sync(0xffffffffu, sk, o);
      }
      const float iq = 1.0f / fmaxf(sqrtf(sq), 1e-6f), ik = 1.0f / fmaxf(sqrtf(sk), 1e-6f);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        q[j] = bf16_to_f32(f32_to_bf16_rne(q[j] * iq));
        k[j] = bf16_to_f32(f32_to_bf16_rne(k[j] * ik));
      }
    }
    float X[8], eb[8], sb[8];
    *reinterpret_cast<float4*>(X) = *reinterpret_cast<const float4*>(&Gc[t][c0]);
    *reinterpret_cast<float4*>(X + 4) = *reinterpret_cast<const float4*>(&Gc[t][c0 + 4]);
    *reinterpret_cast<float4*>(eb) = *reinterpret_cast<const float4*>(sm + P_EB + (blk * DK + c0) * 4);
    *reinterpret_cast<float4*>(eb + 4) = *reinterpret_cast<const float4*>(sm + P_EB + (blk * DK + c0 + 4) * 4);
    *reinterpret_cast<float4*>(sb) = *reinterpret_cast<const float4*>(sm + P_SB + (blk * DK + c0) * 4);
    *reinterpret_cast<float4*>(sb + 4) = *reinterpret_cast<const float4*>(sm + P_SB + (blk * DK + c0 + 4) * 4);
    float ks[8], qs[8], ke[8], xq[8], xk[8], y[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float rx = rcp_approx(X[j]);
      const float e = eb[j] * X[j];  // 2^Gc_t
      ks[j] = k[j] * e;
      qs[j] = q[j] * e;
      ke[j] = k[j] * (sb[j] * rx);    // 2^(Gc_C - Gc_t)
      xq[j] = q[j] * X[j];            // 2^(Gc_t - Gc_r)
      xk[j] = k[j] * X[j];
      y[j] = k[j] * rx;               // 2^(Gc_r - Gc_t)
    }
    *reinterpret_cast<uint4*>(bigr + (size_t)t * DK + c0) = pack8(ks);
    *reinterpret_cast<uint4*>(bigr + (size_t)(64 + t) * DK + c0) = pack8(qs);
    *reinterpret_cast<uint4*>(bigr + (size_t)(128 + t) * DK + c0) = pack8(ke);
    const int sub = cc >> 3, chk = cc & 7;
    *reinterpret_cast<uint4*>(sm + P_XA + sub * 16384 + sw128(t, chk)) = pack8(xq);
    *reinterpret_cast<uint4*>(sm + P_XA + sub * 16384 + sw128(64 + t, chk)) = pack8(xk);
#pragma unroll
    for (int bb = 0; bb < 4; ++bb) {
      if (bb < blk) continue;
      if (bb > blk) {
#pragma unroll
        for (int j = 0; j < 8; ++j) y[j] *= fb[bb][c0 + j];
      }
      *reinterpret_cast<uint4*>(sm + yb_off(bb) + sub * (yb_rows(bb) * 128) + sw128(t, chk)) = pack8(y);
    }
  }
  fence_proxy_async();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (tid == 0) {
    const uint32_t xa = smem_u32(sm + P_XA);
#pragma unroll
    for (int bb = 0; bb < 4; ++bb) {
      const uint32_t yb = smem_u32(sm + yb_off(bb));
      const uint32_t idesc = idesc_bf16_f32(128, yb_rows(bb));
#pragma unroll
      for (int kk = 0; kk < DK / 16; ++kk)
        umma_f16(tmem + d_col(bb), smem_desc_sw128(xa + (kk >> 2) * 16384 + (kk & 3) * 32),
                 smem_desc_sw128(yb + (kk >> 2) * (yb_rows(bb) * 128) + (kk & 3) * 32), idesc, kk != 0);
    }
    umma_commit(mma_done);
  }
  const bool ok = mbar_wait(mma_done, 0, err);
  tc_fence_after();

  // ---- read D_b: warp w reads TMEM lanes 32(w%4).., block 2((w%4)&1) + w/4 ----
  float(*L)[LF] = reinterpret_cast<float(*)[LF]>(sm + P_L);
  {
    const int qd = warp & 3, R = qd * 32 + lane;
    const int bl = 2 * (qd & 1) + (warp >> 2);
    const int t = R & 63;
    const bool mine = (t >> 4) == bl;
    const bool is_qk = R < 64;
    const int n = yb_rows(bl);
    float row[64];
#pragma unroll
    for (int s = 0; s < 64; ++s) row[s] = 0.0f;
#pragma unroll
    for (int p = 0; p < 2; ++p) {
      if (p * 32 < n) {  // warp-uniform
        uint32_t v[32];
        tmem_ld32(tmem + ((uint32_t)(qd * 32) << 16) + d_col(bl) + p * 32, v);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (p * 32 + i < n) row[p * 32 + i] = ok ? __uint_as_float(v[i]) : 0.0f;
      }
    }
    if (mine) {
      if (is_qk) {
        uint16_t* dst = smallr + (size_t)(64 + t) * C;
#pragma unroll
        for (int g = 0; g < 8; ++g) {
          float f[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) f[j] = (8 * g + j <= t) ? row[8 * g + j] : 0.0f;
          *reinterpret_cast<uint4*>(dst + 8 * g) = pack8(f);
        }
      } else {
        const float bt = beta[t];
#pragma unroll
        for (int s = 0; s < 64; ++s) L[t][s] = s < t ? bt * row[s] : 0.0f;
      }
    }
  }
  tc_fence_before();
  __syncthreads();

  // ---- T = (I + L)^-1 in place in L, three levels:
  //   (1) the four 16x16 diagonal blocks by forward substitution;
  //   (2) the lower-left 16x16 block of each 32x32 half: T10 = -D1 (L10 D0);
  //   (3) the lower-left 32x32 block: T_BA = -T_B (L_BA T_A).
  // Blocks above the diagonal of L are zero and stay zero, so the products
  // run over full ranges.  Temporaries P live in the dead B operand region.
  float(*P16)[16][17] = reinterpret_cast<float(*)[16][17]>(sm + P_YB);
  float(*P32)[33] = reinterpret_cast<float(*)[33]>(sm + P_YB);
  if (tid < 64) {
    const int d0 = (tid >> 4) * 16, jj = tid & 15;
    float x[16];
#pragma unroll
    for (int t = 0; t < 16; ++t) {
      float v = (t == jj) ? 1.0f : 0.0f;
#pragma unroll
      for (int u = 0; u < t; ++u) v -= L[d0 + t][d0 + u] * x[u];
      x[t] = v;
    }
    __syncwarp();
#pragma unroll
    for (int t = 0; t < 16; ++t) L[d0 + t][d0 + jj] = x[t];
  }
  __syncthreads();
  {  // (2a) P = L10 D0 for both halves: thread -> (half, row, 2 columns)
    const int hb = tid >> 7, rr = (tid >> 3) & 15, c0 = (tid & 7) * 2, o = 32 * hb;
    float a0 = 0.0f, a1 = 0.0f;
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      const float l = L[o + 16 + rr][o + k];
      a0 += l * L[o + k][o + c0];
      a1 += l * L[o + k][o + c0 + 1];
    }
    P16[hb][rr][c0] = a0;
    P16[hb][rr][c0 + 1] = a1;
  }
  __syncthreads();
  {  // (2b) T10 = -D1 P
    const int hb = tid >> 7, rr = (tid >> 3) & 15, c0 = (tid & 7) * 2, o = 32 * hb;
    float a0 = 0.0f, a1 = 0.0f;
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      const float d = L[o + 16 + rr][o + 16 + k];
      a0 += d * P16[hb][k][c0];
      a1 += d * P16[hb][k][c0 + 1];
    }
    L[o + 16 + rr][o + c0] = -a0;
    L[o + 16 + rr][o + c0 + 1] = -a1;
  }
  __syncthreads();
  {  // (3a) P = L_BA T_A: thread -> (row, 4 columns)
    const int rr = tid >> 3, c0 = (tid & 7) * 4;
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll 8
    for (int k = 0; k < 32; ++k) {
      const float l = L[32 + rr][k];
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[j] += l * L[k][c0 + j];
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) P32[rr][c0 + j] = acc[j];
  }
  __syncthreads();
  {  // (3b) T_BA = -T_B P
    const int rr = tid >> 3, c0 = (tid & 7) * 4;
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll 8
    for (int k = 0; k < 32; ++k) {
      const float d = L[32 + rr][32 + k];
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[j] += d * P32[k][c0 + j];
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) L[32 + rr][c0 + j] = -acc[j];
  }
  __syncthreads();
  // T diag(beta) -> record (lower triangle incl. diagonal), 8 columns per thread
  for (int i = tid; i < C * C / 8; i += PREP_THREADS) {
    const int rr = i >> 3, c0 = (i & 7) * 8;
    float f[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int c2 = c0 + u;
      f[u] = c2 <= rr ? L[rr][c2] * beta[c2] : 0.0f;
    }
    *reinterpret_cast<uint4*>(smallr + (size_t)rr * C + c0) = pack8(f);
  }
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

// ===========================================================================
// scan: one CTA per (sequence, head), chunks in order, state in TMEM
// ===========================================================================
constexpr int SCAN_THREADS = 320;  // producer, MMA, 8 element-wise warps
constexpr int S_SB = 0;                 // bf16 state copy S^T [v][i], 2 sub-tiles of 16 KB
constexpr int S_XS = 32768;             // X^T [v][t] bf16, one sub-tile
constexpr int S_US = S_XS + 16384;      // U^T [v][t] bf16
constexpr int S_KQ = S_US + 16384;      // [K~; Q~] as B (128 rows), 2 sub-tiles, x2 buffers
constexpr int S_KE = S_KQ + 2 * 32768;  // K^ [t][i] MN-major B, 2 blocks of 8 KB
constexpr int S_TT = S_KE + 16384;      // T [t][s]
constexpr int S_QK = S_TT + 8192;       // QK [t][s]
constexpr int S_V = S_QK + 8192;        // V [t][v] plain row-major
constexpr int S_D = S_V + 16384;        // e^Gc_C, fp32 [128]
constexpr int S_BAR = S_D + 512;
constexpr int SCAN_SMEM = S_BAR + 256 + 1024;
constexpr uint32_t IDESC_N128 = idesc_bf16_f32(128, 128);
constexpr uint32_t IDESC_N64 = idesc_bf16_f32(128, 64);
constexpr uint32_t IDESC_N128_BMN = idesc_bf16_f32(128, 128) | (1u << 16);  // B MN-major
// TMEM columns
constexpr uint32_t TM_X = 0, TM_O = 64, TM_U = 128, TM_S = 256;

struct ScanBars {
  uint64_t kq_full[2], kq_free[2], t_full, t_free, m3_full, m3_free, v_full, v_free;
  uint64_t s_ready, x_full, xs_ready, u_full, us_ready, o_full;
  uint32_t tmem_base;
  int abort_flag;
};

__global__ void __launch_bounds__(SCAN_THREADS, 1)
    kda_scan_kernel(const __grid_constant__ CUtensorMap tmBig, const __grid_constant__ CUtensorMap tmSmall,
                    const __grid_constant__ CUtensorMap tmV, const float* __restrict__ dend,
                    float* __restrict__ state, uint16_t* __restrict__ og, long long ldo, int seq, int heads,
                    int nchunks, int* err) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* sm = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  ScanBars& bar = *reinterpret_cast<ScanBars*>(sm + S_BAR);
  const int bh = blockIdx.x, b = bh / heads, h = bh % heads;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long tok0 = (long long)b * seq;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) { mbar_init(&bar.kq_full[i], 1); mbar_init(&bar.kq_free[i], 1); }
    mbar_init(&bar.t_full, 1); mbar_init(&bar.t_free, 1);
    mbar_init(&bar.m3_full, 1); mbar_init(&bar.m3_free, 1);
    mbar_init(&bar.v_full, 1); mbar_init(&bar.v_free, 8);
    mbar_init(&bar.s_ready, 8); mbar_init(&bar.x_full, 1); mbar_init(&bar.xs_ready, 8);
    mbar_init(&bar.u_full, 1); mbar_init(&bar.us_ready, 8); mbar_init(&bar.o_full, 1);
    bar.abort_flag = 0;
    fence_barrier_init();
    fence_proxy_async();
  }
  if (warp == 1) { tmem_alloc(&bar.tmem_base, 512); tmem_relinquish(); }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bar.tmem_base;
  volatile int* abort_flag = &bar.abort_flag;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmBig);
      tma_prefetch_desc(&tmSmall);
      tma_prefetch_desc(&tmV);
      for (int c = 0; c < nchunks && !*abort_flag; ++c) {
        const int rec = bh * nchunks + c, bf = c & 1;
        const uint32_t par = (c & 1) ^ 1u;
        if (!mbar_wait(&bar.kq_free[bf], ((c >> 1) & 1) ^ 1u, err)) { *abort_flag = 1; break; }
        mbar_arrive_expect_tx(&bar.kq_full[bf], 32768);
        uint8_t* kq = sm + S_KQ + bf * 32768;
        for (int j = 0; j < 2; ++j) {
          tma_load_2d(kq + j * 16384, &tmBig, &bar.kq_full[bf], 64 * j, 192 * rec);
          tma_load_2d(kq + j * 16384 + 8192, &tmBig, &bar.kq_full[bf], 64 * j, 192 * rec + 64);
        }
        if (!mbar_wait(&bar.t_free, par, err)) { *abort_flag = 1; break; }
        mbar_arrive_expect_tx(&bar.t_full, 8192);
        tma_load_2d(sm + S_TT, &tmSmall, &bar.t_full, 0, 128 * rec);
        if (!mbar_wait(&bar.m3_free, par, err)) { *abort_flag = 1; break; }
        mbar_arrive_expect_tx(&bar.m3_full, 16384 + 8192);
        tma_load_2d(sm + S_KE, &tmBig, &bar.m3_full, 0, 192 * rec + 128);
        tma_load_2d(sm + S_KE + 8192, &tmBig, &bar.m3_full, 64, 192 * rec + 128);
        tma_load_2d(sm + S_QK, &tmSmall, &bar.m3_full, 0, 128 * rec + 64);
        if (!mbar_wait(&bar.v_free, par, err)) { *abort_flag = 1; break; }
        mbar_arrive_expect_tx(&bar.v_full, 16384 + 512);
        tma_load_2d(sm + S_V, &tmV, &bar.v_full, h * DK, (int)(tok0 + c * C));
        bulk_load(sm + S_D, dend + (size_t)rec * DK, 512, &bar.v_full);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t sb = smem_u32(sm + S_SB), xs = smem_u32(sm + S_XS), us = smem_u32(sm + S_US);
      const uint32_t tt = smem_u32(sm + S_TT), qk = smem_u32(sm + S_QK), ke = smem_u32(sm + S_KE);
      bool ok = true;
      for (int c = 0; ok && c < nchunks && !*abort_flag; ++c) {
        const int bf = c & 1;
        const uint32_t par = c & 1;
        // X^T | O1^T = S^T [K~; Q~]^T
        if (!mbar_wait(&bar.kq_full[bf], (c >> 1) & 1, err) || !mbar_wait(&bar.s_ready, par, err)) { ok = false; break; }
        tc_fence_after();
        const uint32_t kq = smem_u32(sm + S_KQ + bf * 32768);
#pragma unroll
        for (int kk = 0; kk < DK / 16; ++kk)
          umma_f16(tmem + TM_X, smem_desc_sw128(sb + (kk >> 2) * 16384 + (kk & 3) * 32),
                   smem_desc_sw128(kq + (kk >> 2) * 16384 + (kk & 3) * 32), IDESC_N128, kk != 0);
        umma_commit(&bar.x_full);
        umma_commit(&bar.kq_free[bf]);
        // U^T = X^T T^T
        if (!mbar_wait(&bar.t_full, par, err) || !mbar_wait(&bar.xs_ready, par, err)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < C / 16; ++kk)
          umma_f16(tmem + TM_U, smem_desc_sw128(xs + kk * 32), smem_desc_sw128(tt + kk * 32), IDESC_N64, kk != 0);
        umma_commit(&bar.u_full);
        umma_commit(&bar.t_free);
        // O^T += U^T QK^T ; S^T += U^T K^
        if (!mbar_wait(&bar.m3_full, par, err) || !mbar_wait(&bar.us_ready, par, err)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < C / 16; ++kk)
          umma_f16(tmem + TM_O, smem_desc_sw128(us + kk * 32), smem_desc_sw128(qk + kk * 32), IDESC_N64, 1);
#pragma unroll
        for (int kk = 0; kk < C / 16; ++kk)
          umma_f16(tmem + TM_S, smem_desc_sw128(us + kk * 32), smem_desc_sw128_mn(ke + kk * 2048, 8192),
                   IDESC_N128_BMN, 1);
        umma_commit(&bar.o_full);
        umma_commit(&bar.m3_free);
      }
      if (!ok) *abort_flag = 1;
    }
  } else {
    // element-wise warps: TMEM lane quarter qd = warp % 4 (value columns
    // v = 32 qd + lane); `half` selects token columns [32 half, +32) of X, U,
    // O and key rows [64 half, +64) of the state
    const int qd = warp & 3, half = (warp - 2) >> 2;
    const int v = qd * 32 + lane;
    const uint32_t lane_off = (uint32_t)(qd * 32) << 16;
    const float qscale = rsqrtf((float)DK);
    float* st_g = state ? state + (size_t)bh * DK * DK : nullptr;
    const uint16_t* sV = reinterpret_cast<const uint16_t*>(sm + S_V);
    const float* sD = reinterpret_cast<const float*>(sm + S_D);
    bool ok = true;
    // initial state: S^T[v][i] = S[i][v]
#pragma unroll
    for (int p = 0; p < 2; ++p) {
      const int i0 = half * 64 + p * 32;
      uint32_t r[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(st_g ? st_g[(size_t)(i0 + i) * DK + v] : 0.0f);
      tmem_st32(tmem + lane_off + TM_S + i0, r);
#pragma unroll
      for (int g = 0; g < 4; ++g)
        *reinterpret_cast<uint4*>(sm + S_SB + half * 16384 + sw128(v, p * 4 + g)) =
            make_uint4(pack_bf16x2(__uint_as_float(r[8 * g]), __uint_as_float(r[8 * g + 1])),
                       pack_bf16x2(__uint_as_float(r[8 * g + 2]), __uint_as_float(r[8 * g + 3])),
                       pack_bf16x2(__uint_as_float(r[8 * g + 4]), __uint_as_float(r[8 * g + 5])),
                       pack_bf16x2(__uint_as_float(r[8 * g + 6]), __uint_as_float(r[8 * g + 7])));
    }
    tmem_st_wait();
    fence_proxy_async();
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(&bar.s_ready);

    for (int c = 0; c < nchunks; ++c) {
      const uint32_t par = c & 1;
      const int t0 = c * C;
      // ---- X^T = V^T - S^T K~^T -> bf16; S^T *= e^Gc_C ----
      if (!mbar_wait(&bar.x_full, par, err) || !mbar_wait(&bar.v_full, par, err)) { ok = false; break; }
      tc_fence_after();
      {
        uint32_t r[32];
        tmem_ld32(tmem + lane_off + TM_X + half * 32, r);
        tmem_ld_wait();
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          uint32_t pk[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int t = half * 32 + 8 * g + 2 * j;
            pk[j] = pack_bf16x2(bf16_to_f32(sV[t * DK + v]) - __uint_as_float(r[8 * g + 2 * j]),
                                bf16_to_f32(sV[(t + 1) * DK + v]) - __uint_as_float(r[8 * g + 2 * j + 1]));
          }
          *reinterpret_cast<uint4*>(sm + S_XS + sw128(v, half * 4 + g)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
        }
      }
      fence_proxy_async();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar.xs_ready);
      // S^T *= e^Gc_C: only the O/S MMAs of this chunk (after us_ready) need
      // it, so it overlaps U^T = X^T T^T
#pragma unroll
      for (int p = 0; p < 2; ++p) {
        const int i0 = half * 64 + p * 32;
        uint32_t r[32];
        tmem_ld32(tmem + lane_off + TM_S + i0, r);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * sD[i0 + i]);
        tmem_st32(tmem + lane_off + TM_S + i0, r);
      }
      tmem_st_wait();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar.v_free);  // V and e^Gc_C consumed
      // ---- U^T -> bf16 ----
      if (!mbar_wait(&bar.u_full, par, err)) { ok = false; break; }
      tc_fence_after();
      {
        uint32_t r[32];
        tmem_ld32(tmem + lane_off + TM_U + half * 32, r);
        tmem_ld_wait();
#pragma unroll
        for (int g = 0; g < 4; ++g)
          *reinterpret_cast<uint4*>(sm + S_US + sw128(v, half * 4 + g)) =
              make_uint4(pack_bf16x2(__uint_as_float(r[8 * g]), __uint_as_float(r[8 * g + 1])),
                         pack_bf16x2(__uint_as_float(r[8 * g + 2]), __uint_as_float(r[8 * g + 3])),
                         pack_bf16x2(__uint_as_float(r[8 * g + 4]), __uint_as_float(r[8 * g + 5])),
                         pack_bf16x2(__uint_as_float(r[8 * g + 6]), __uint_as_float(r[8 * g + 7])));
      }
      fence_proxy_async();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar.us_ready);
      // ---- O out; S^T -> bf16 copy for the next chunk ----
      if (!mbar_wait(&bar.o_full, par, err)) { ok = false; break; }
      tc_fence_after();
      {
        uint32_t r[32];
        tmem_ld32(tmem + lane_off + TM_O + half * 32, r);
        tmem_ld_wait();
        uint16_t* orow = og + (tok0 + t0 + half * 32) * ldo + h * DK + v;
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (t0 + half * 32 + j < seq) orow[(long long)j * ldo] = f32_to_bf16_rne(__uint_as_float(r[j]) * qscale);
      }
      const bool last = c == nchunks - 1;
#pragma unroll
      for (int p = 0; p < 2; ++p) {
        const int i0 = half * 64 + p * 32;
        uint32_t r[32];
        tmem_ld32(tmem + lane_off + TM_S + i0, r);
        tmem_ld_wait();
        if (last) {
          if (st_g)
#pragma unroll
            for (int i = 0; i < 32; ++i) st_g[(size_t)(i0 + i) * DK + v] = __uint_as_float(r[i]);
        } else {
#pragma unroll
          for (int g = 0; g < 4; ++g)
            *reinterpret_cast<uint4*>(sm + S_SB + half * 16384 + sw128(v, p * 4 + g)) =
                make_uint4(pack_bf16x2(__uint_as_float(r[8 * g]), __uint_as_float(r[8 * g + 1])),
                           pack_bf16x2(__uint_as_float(r[8 * g + 2]), __uint_as_float(r[8 * g + 3])),
                           pack_bf16x2(__uint_as_float(r[8 * g + 4]), __uint_as_float(r[8 * g + 5])),
                           pack_bf16x2(__uint_as_float(r[8 * g + 6]), __uint_as_float(r[8 * g + 7])));
        }
      }
      fence_proxy_async();
      tc_fence_before();
      __syncwarp();
      if (lane == 0 && !last) mbar_arrive(&bar.s_ready);
    }
    if (!ok) *abort_flag = 1;
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

bool g_attr[64];

}  // namespace

size_t kda_workspace_bytes(int batch, int seq, int heads) {
  size_t nchunks = (size_t)(seq + C - 1) / C;
  return (size_t)batch * heads * nchunks * kChunkBytes;
}

int32_t launch_kda_chunked(const uint16_t* q, const uint16_t* k, const uint16_t* v, long long ld_qkv, const float* g,
                           const float* beta, float* state, uint16_t* o, long long ldo, int batch, int seq, int heads,
                           void* workspace, size_t workspace_bytes, cudaStream_t s, const KdaRawGate* raw,
                           int* err_word) {
  if (batch <= 0 || seq <= 0 || heads <= 0) return set_error(ENNX_B200_INVALID_ARGUMENT, "kda: empty input");
  if (ld_qkv % 8 || ldo % 2 || (((uintptr_t)q | (uintptr_t)k | (uintptr_t)v) & 15u))
    return set_error(ENNX_B200_INVALID_ARGUMENT, "kda: q/k/v must be 16-byte aligned with ld %% 8 == 0");
  if (((uintptr_t)g & 15u) || ((uintptr_t)workspace & 15u))
    return set_error(ENNX_B200_INVALID_ARGUMENT, "kda: g and workspace must be 16-byte aligned");
  const size_t need = kda_workspace_bytes(batch, seq, heads);
  if (!workspace || workspace_bytes < need)
    return set_error(ENNX_B200_INVALID_ARGUMENT, "kda: workspace of %zu bytes required", need);
  if (!raw && (!g || !beta)) return set_error(ENNX_B200_INVALID_ARGUMENT, "kda: g and beta are required");
  const long long rows = (long long)batch * seq;
  if (rows > 0x7fffffffLL) return set_error(ENNX_B200_UNSUPPORTED, "kda: too many tokens");
  const int nchunks = (seq + C - 1) / C;
  const size_t R = (size_t)batch * heads * nchunks;
  if (R * 192 > 0xffffffffull) return set_error(ENNX_B200_UNSUPPORTED, "kda: too many chunks");
  uint16_t* big = reinterpret_cast<uint16_t*>(workspace);
  uint16_t* small = reinterpret_cast<uint16_t*>(reinterpret_cast<uint8_t*>(workspace) + R * kBigRecBytes);
  float* dend = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(workspace) + R * (kBigRecBytes + kSmallRecBytes));
  CUtensorMap tb, ts, tv;
  ENNX_TRY(make_tmap_2d_bf16(&tb, big, DK, R * 192, DK, 64, 64, true));
  ENNX_TRY(make_tmap_2d_bf16(&ts, small, C, R * 128, C, 64, 64, true));
  ENNX_TRY(make_tmap_2d_bf16(&tv, v, (uint64_t)heads * DK, (uint64_t)rows, (uint64_t)ld_qkv, DK, C, false));
  // A caller-supplied status word (the allocation-free entry point's static
  // one) replaces the lazily allocated per-device word.
  int* err = err_word ? err_word : device_error_word();
  if (!err) return set_error(ENNX_B200_CUDA_ERROR, "kda: no device error word");
  int dev = 0;
  cudaGetDevice(&dev);
  if (!g_attr[dev]) {
    ENNX_CUDA(cudaFuncSetAttribute(kda_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, PREP_SMEM),
              "kda prep smem");
    ENNX_CUDA(cudaFuncSetAttribute(kda_scan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SCAN_SMEM),
              "kda scan smem");
    g_attr[dev] = true;
  }
  KdaRawGate rg;
  memset(&rg, 0, sizeof(rg));
  if (raw) rg = *raw;
  kda_prep_kernel<<<dim3(nchunks, batch * heads), PREP_THREADS, PREP_SMEM, s>>>(
      q, k, ld_qkv, g, (long long)heads * DK, beta, seq, heads, nchunks, rg, big, small, dend, err);
  ENNX_LAUNCH_CHECK("kda prep");
  kda_scan_kernel<<<batch * heads, SCAN_THREADS, SCAN_SMEM, s>>>(tb, ts, tv, dend, state, o, ldo, seq, heads, nchunks,
                                                                 err);
  ENNX_LAUNCH_CHECK("kda scan");
  return ENNX_B200_OK;
}

}  // namespace ennx
