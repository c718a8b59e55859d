// kda.cu -- chunked KDA (gated delta rule with per-key-channel decay).
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
// (first token of t's 16-token sub-block): both factors stay bounded for
// s <= t because each step decays by at most e^-5.
//
// Two kernels:
//   kda_prep_kernel  -- one CTA per (sequence, head, chunk), all in parallel:
//     everything that does not depend on the state: Gc, the intra-chunk
//     products QK and A', T = (I + diag(beta) A')^-1 diag(beta), and the
//     decay-scaled operands K~ = K o e^Gc, Q~ = Q o e^Gc, K^ = K o e^(Gc_C - Gc).
//   kda_scan_kernel  -- one CTA per (sequence, head, 32 value columns) walks
//     the chunks in order with its fp32 state slice resident in shared
//     memory: X = V - K~ S, U = T X, O = (Q~ S + QK U)/sqrt(dk),
//     S = e^Gc_C o S + K^^T U.
// Contractions run on mma.sync m16n8k16 bf16 tensor cores with fp32
// accumulation; decays, triangular inverses and the state stay fp32.
#include "common.cuh"
#include "kernels.cuh"

#include <string.h>

namespace ennx {
namespace {

constexpr int C = 64, DK = 128;
constexpr int LQ = DK + 8;  // padded bf16 row (elements) of [64][128] tiles
constexpr int LS = C + 8;   // padded bf16 row of [64][64] tiles
constexpr int LF = C + 1;   // padded fp32 row of [64][64] matrices
constexpr int SV = 32;      // value columns per scan CTA
constexpr int LV = SV + 8;  // padded bf16 row of [*][32] tiles

// per-chunk operand record produced by the prep kernel (global memory)
constexpr size_t kBigElems = 3ull * C * DK;   // K~, Q~, K^   (bf16)
constexpr size_t kSmallElems = 2ull * C * C;  // T, QK        (bf16)
constexpr size_t kChunkBytes = (kBigElems + kSmallElems) * 2 + DK * 4;  // + e^Gc_C (fp32)

__device__ __forceinline__ void ldsm_x4(const void* p, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x4_t(const void* p, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(smem_u32(p)));
}
__device__ __forceinline__ void mma16816(float c[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;" ::: "memory");
}

// A fragment (16 x 16) at (m0, k0) of a row-major [m][k] bf16 tile.
template <int LD>
__device__ __forceinline__ void frag_a(const uint16_t* base, int m0, int k0, int lane, uint32_t a[4]) {
  ldsm_x4(base + (m0 + (lane & 7) + ((lane >> 3) & 1) * 8) * LD + k0 + (lane >> 4) * 8, a[0], a[1], a[2], a[3]);
}
// A fragment (16 x 16) at (m0, k0) of a tile stored transposed, [k][m].
template <int LD>
__device__ __forceinline__ void frag_a_t(const uint16_t* base, int m0, int k0, int lane, uint32_t a[4]) {
  ldsm_x4_t(base + (k0 + (lane & 7) + (lane >> 4) * 8) * LD + m0 + ((lane >> 3) & 1) * 8, a[0], a[1], a[2], a[3]);
}
// B fragments for n-tiles n0 and n0+8 (k0..k0+15) of a tile stored [n][k].
template <int LD>
__device__ __forceinline__ void frag_b_nk(const uint16_t* base, int n0, int k0, int lane, uint32_t b[4]) {
  ldsm_x4(base + (n0 + (lane & 7) + (lane >> 4) * 8) * LD + k0 + ((lane >> 3) & 1) * 8, b[0], b[1], b[2], b[3]);
}
// B fragments for n-tiles n0 and n0+8 of a tile stored [k][n].
template <int LD>
__device__ __forceinline__ void frag_b_kn(const uint16_t* base, int n0, int k0, int lane, uint32_t b[4]) {
  ldsm_x4_t(base + (k0 + (lane & 7) + ((lane >> 3) & 1) * 8) * LD + n0 + (lane >> 4) * 8, b[0], b[1], b[2], b[3]);
}

// ===========================================================================
// prep: one CTA per (sequence, head, chunk)
// ===========================================================================
struct PrepSmem {
  float Gc[C][DK];
  float L[C][LF];         // beta_t A'[t,s] (strict lower); block rows become T rows
  float Tdiag[4][16][17]; // inverses of the 16x16 diagonal blocks of I + L
  float beta[C];
  uint16_t q[C][LQ], k[C][LQ];
  uint16_t X[32][LQ], Y[C][LQ];
};

__device__ __forceinline__ float softplus_stable(float x) { return fmaxf(x, 0.0f) + log1pf(__expf(-fabsf(x))); }

__global__ void __launch_bounds__(256) kda_prep_kernel(const uint16_t* __restrict__ qg, const uint16_t* __restrict__ kg,
                                                       long long ld, const float* __restrict__ gg, long long ldg,
                                                       const float* __restrict__ bg, int seq, int heads, int nchunks,
                                                       KdaRawGate raw, uint8_t* __restrict__ ops) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  PrepSmem& s = *reinterpret_cast<PrepSmem*>(smem_raw);
  const int ch = blockIdx.x, bh = blockIdx.y, b = bh / heads, h = bh % heads;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const long long tok0 = (long long)b * seq;
  const int t0 = ch * C;
  uint8_t* rec = ops + ((size_t)bh * nchunks + ch) * kChunkBytes;
  uint16_t* big = reinterpret_cast<uint16_t*>(rec);
  uint16_t* small = big + kBigElems;
  float* dend = reinterpret_cast<float*>(small + kSmallElems);

  // ---- loads (independent 16-byte loads from every thread) ----
  for (int i = tid; i < C * (DK / 8); i += 256) {
    int r = i / (DK / 8), c = (i % (DK / 8)) * 8;
    uint4 qv = make_uint4(0, 0, 0, 0), kv = qv;
    if (t0 + r < seq) {
      long long off = (tok0 + t0 + r) * ld + h * DK + c;
      qv = *reinterpret_cast<const uint4*>(qg + off);
      kv = *reinterpret_cast<const uint4*>(kg + off);
    }
    *reinterpret_cast<uint4*>(&s.q[r][c]) = qv;
    *reinterpret_cast<uint4*>(&s.k[r][c]) = kv;
  }
  if (raw.active) {
    // forward path: g = max(-exp(decay_h) * softplus(f + time_bias), -5) and
    // beta = sigmoid(raw beta) from the raw projections (kda_moe.metal:869-895)
    const bool set0 = b < raw.split_seq;
    const uint16_t* tb = set0 ? raw.tb0 : raw.tb1;
    const float dscale = __expf(bf16_to_f32((set0 ? raw.decay0 : raw.decay1)[h]));
    for (int i = tid; i < C * (DK / 8); i += 256) {
      int r = i / (DK / 8), c = (i % (DK / 8)) * 8;
      float gv[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      if (t0 + r < seq) {
        uint4 fv = *reinterpret_cast<const uint4*>(raw.f + (tok0 + t0 + r) * raw.ldf + h * DK + c);
        uint4 bv = *reinterpret_cast<const uint4*>(tb + h * DK + c);
        uint32_t fw[4] = {fv.x, fv.y, fv.z, fv.w}, bw[4] = {bv.x, bv.y, bv.z, bv.w};
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          float x = bf16_to_f32((uint16_t)(fw[j >> 1] >> (16 * (j & 1)))) +
                    bf16_to_f32((uint16_t)(bw[j >> 1] >> (16 * (j & 1))));
          gv[j] = fmaxf(-dscale * softplus_stable(x), -5.0f);
        }
      }
      *reinterpret_cast<float4*>(&s.Gc[r][c]) = make_float4(gv[0], gv[1], gv[2], gv[3]);
      *reinterpret_cast<float4*>(&s.Gc[r][c + 4]) = make_float4(gv[4], gv[5], gv[6], gv[7]);
    }
    if (tid < C)
      s.beta[tid] = t0 + tid < seq
                        ? 1.0f / (1.0f + __expf(-bf16_to_f32(raw.rbeta[(tok0 + t0 + tid) * raw.ldb + h])))
                        : 0.0f;
    __syncthreads();
    // per-token L2 normalisation of q and k, 1/max(|x|, 1e-6) (kda_moe.metal:510-534)
    for (int r = warp; r < 2 * C; r += 8) {
      uint16_t* row = r < C ? &s.q[r][0] : &s.k[r - C][0];
      uint2 rv = *reinterpret_cast<uint2*>(row + lane * 4);
      float f[4] = {bf16_to_f32(rv.x & 0xffffu), bf16_to_f32(rv.x >> 16), bf16_to_f32(rv.y & 0xffffu),
                    bf16_to_f32(rv.y >> 16)};
      float ss = f[0] * f[0] + f[1] * f[1] + f[2] * f[2] + f[3] * f[3];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      float inv = 1.0f / fmaxf(sqrtf(ss), 1e-6f);
      *reinterpret_cast<uint2*>(row + lane * 4) =
          make_uint2(pack_bf16x2(f[0] * inv, f[1] * inv), pack_bf16x2(f[2] * inv, f[3] * inv));
    }
  } else {
    for (int i = tid; i < C * (DK / 4); i += 256) {
      int r = i / (DK / 4), c = (i % (DK / 4)) * 4;
      float4 gv = make_float4(0.f, 0.f, 0.f, 0.f);
      if (t0 + r < seq) gv = *reinterpret_cast<const float4*>(gg + (tok0 + t0 + r) * ldg + h * DK + c);
      *reinterpret_cast<float4*>(&s.Gc[r][c]) = gv;
    }
    if (tid < C) s.beta[tid] = t0 + tid < seq ? bg[(tok0 + t0 + tid) * heads + h] : 0.0f;
  }
  __syncthreads();
  if (tid < DK) {  // inclusive prefix sum of the log decay per key channel
    float acc = 0.0f;
#pragma unroll 8
    for (int t = 0; t < C; ++t) {
      acc += s.Gc[t][tid];
      s.Gc[t][tid] = acc;
    }
  }
  __syncthreads();

  // ---- decay-scaled operands straight to global (K~, Q~, K^, e^Gc_C) ----
  for (int i = tid; i < C * (DK / 8); i += 256) {
    int t = i / (DK / 8), c = (i % (DK / 8)) * 8;
    uint32_t ks[4], qs[4], ke[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float e0 = __expf(s.Gc[t][c + 2 * j]), e1 = __expf(s.Gc[t][c + 2 * j + 1]);
      float d0 = __expf(s.Gc[C - 1][c + 2 * j] - s.Gc[t][c + 2 * j]);
      float d1 = __expf(s.Gc[C - 1][c + 2 * j + 1] - s.Gc[t][c + 2 * j + 1]);
      float k0 = bf16_to_f32(s.k[t][c + 2 * j]), k1 = bf16_to_f32(s.k[t][c + 2 * j + 1]);
      float q0 = bf16_to_f32(s.q[t][c + 2 * j]), q1 = bf16_to_f32(s.q[t][c + 2 * j + 1]);
      ks[j] = pack_bf16x2(k0 * e0, k1 * e1);
      qs[j] = pack_bf16x2(q0 * e0, q1 * e1);
      ke[j] = pack_bf16x2(k0 * d0, k1 * d1);
    }
    *reinterpret_cast<uint4*>(big + t * DK + c) = make_uint4(ks[0], ks[1], ks[2], ks[3]);
    *reinterpret_cast<uint4*>(big + C * DK + t * DK + c) = make_uint4(qs[0], qs[1], qs[2], qs[3]);
    *reinterpret_cast<uint4*>(big + 2 * C * DK + t * DK + c) = make_uint4(ke[0], ke[1], ke[2], ke[3]);
  }
  if (tid < DK) dend[tid] = __expf(s.Gc[C - 1][tid]);

  // ---- intra-chunk products, one 16-row block at a time ----
  uint16_t* QKg = small + C * C;
  for (int blk = 0; blk < 4; ++blk) {
    const int r = blk * 16, ns = r + 16;
    __syncthreads();
    for (int i = tid; i < 32 * DK; i += 256) {  // X rows: 16 q-scaled, 16 k-scaled
      int row = i / DK, c = i % DK;
      int t = r + (row & 15);
      float e = __expf(s.Gc[t][c] - s.Gc[r][c]);
      float src = bf16_to_f32(row < 16 ? s.q[t][c] : s.k[t][c]);
      s.X[row][c] = f32_to_bf16_rne(src * e);
    }
    for (int i = tid; i < ns * DK; i += 256) {
      int t = i / DK, c = i % DK;
      s.Y[t][c] = f32_to_bf16_rne(bf16_to_f32(s.k[t][c]) * __expf(s.Gc[r][c] - s.Gc[t][c]));
    }
    __syncthreads();
    const int npairs = ns / 16;
    for (int task = warp; task < 2 * npairs; task += 8) {
      const int which = task / npairs;  // 0: QK, 1: A'
      const int n0 = (task % npairs) * 16;
      float acc[2][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}};
#pragma unroll
      for (int kk = 0; kk < DK; kk += 16) {
        uint32_t a[4], bb[4];
        frag_a<LQ>(&s.X[0][0], which * 16, kk, lane, a);
        frag_b_nk<LQ>(&s.Y[0][0], n0, kk, lane, bb);
        mma16816(acc[0], a, bb[0], bb[1]);
        mma16816(acc[1], a, bb[2], bb[3]);
      }
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 4; e += 2) {
          int t = r + (lane >> 2) + (e >> 1) * 8;
          int sc = n0 + nt * 8 + (lane & 3) * 2;
          float x0 = acc[nt][e], x1 = acc[nt][e + 1];
          if (which == 0) {
            *reinterpret_cast<uint32_t*>(QKg + t * C + sc) =
                pack_bf16x2(sc <= t ? x0 : 0.0f, sc + 1 <= t ? x1 : 0.0f);
          } else {
            s.L[t][sc] = sc < t ? s.beta[t] * x0 : 0.0f;
            s.L[t][sc + 1] = sc + 1 < t ? s.beta[t] * x1 : 0.0f;
          }
        }
    }
    for (int i = tid; i < 16 * (C - ns); i += 256) {  // zero right of the computed columns
      int t = r + i / (C - ns), sc = ns + i % (C - ns);
      QKg[t * C + sc] = 0;
      s.L[t][sc] = 0.0f;
    }
  }
  __syncthreads();

  // ---- T = (I + L)^-1: 16x16 diagonal inverses, then block rows in order ----
  if (warp < 4 && lane < 16) {
    const int d0 = warp * 16, jj = lane;
    float x[16];
#pragma unroll
    for (int t = 0; t < 16; ++t) {
      float v = (t == jj) ? 1.0f : 0.0f;
#pragma unroll
      for (int u = 0; u < t; ++u) v -= s.L[d0 + t][d0 + u] * x[u];
      x[t] = v;
    }
#pragma unroll
    for (int t = 0; t < 16; ++t) s.Tdiag[warp][t][jj] = x[t];
  }
  __syncthreads();
  // block row bi of T (bj < bi): T_ij = -T_ii sum_{k=j}^{i-1} L_ik T_kj.  Rows
  // < bi of L already hold T; row bi of L still holds L until overwritten.
  for (int bi = 1; bi < 4; ++bi) {
    float mval[3];
    const int n = bi * 256;
#pragma unroll
    for (int q = 0; q < 3; ++q) {
      int i = tid + q * 256;
      mval[q] = 0.0f;
      if (i < n) {
        int bj = i / 256, e = i % 256, rr = e / 16, cc = e % 16;
        float acc = 0.0f;
        for (int kx = bj * 16; kx < bi * 16; ++kx) {
          float tkj = (kx < (bj + 1) * 16) ? s.Tdiag[bj][kx - bj * 16][cc] : s.L[kx][bj * 16 + cc];
          acc += s.L[bi * 16 + rr][kx] * tkj;
        }
        mval[q] = acc;
      }
    }
    __syncthreads();
#pragma unroll
    for (int q = 0; q < 3; ++q) {
      int i = tid + q * 256;
      if (i < n) {
        int bj = i / 256, e = i % 256, rr = e / 16, cc = e % 16;
        s.L[bi * 16 + rr][bj * 16 + cc] = mval[q];  // M_ij, temporarily
      }
    }
    __syncthreads();
#pragma unroll
    for (int q = 0; q < 3; ++q) {
      int i = tid + q * 256;
      mval[q] = 0.0f;
      if (i < n) {
        int bj = i / 256, e = i % 256, rr = e / 16, cc = e % 16;
        float acc = 0.0f;
#pragma unroll 4
        for (int kx = 0; kx < 16; ++kx) acc -= s.Tdiag[bi][rr][kx] * s.L[bi * 16 + kx][bj * 16 + cc];
        mval[q] = acc;
      }
    }
    __syncthreads();
#pragma unroll
    for (int q = 0; q < 3; ++q) {
      int i = tid + q * 256;
      if (i < n) {
        int bj = i / 256, e = i % 256, rr = e / 16, cc = e % 16;
        s.L[bi * 16 + rr][bj * 16 + cc] = mval[q];
      }
    }
    __syncthreads();
  }
  // T diag(beta) -> global (lower incl. diagonal)
  uint16_t* Tg = small;
  for (int i = tid; i < C * C / 2; i += 256) {
    int rr = (2 * i) / C, cc = (2 * i) % C;
    float v[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      int c2 = cc + u;
      float tv = 0.0f;
      if (c2 <= rr) tv = (c2 >> 4) == (rr >> 4) ? s.Tdiag[rr >> 4][rr & 15][c2 & 15] : s.L[rr][c2];
      v[u] = tv * s.beta[c2];
    }
    *reinterpret_cast<uint32_t*>(Tg + rr * C + cc) = pack_bf16x2(v[0], v[1]);
  }
}

// ===========================================================================
// scan: one CTA per (sequence, head, 32 value columns), chunks in order
// ===========================================================================
struct ScanSmem {
  float Sf[DK][SV];      // state slice, fp32 master
  float dend[DK];
  uint16_t Sb[DK][LV];   // bf16 copy of the state slice
  uint16_t Ks[C][LQ], Qs[C][LQ], Ke[C][LQ];
  uint16_t T[C][LS], QK[C][LS];
  uint16_t V[C][LV], XU[C][LV];
};

__global__ void __launch_bounds__(128) kda_scan_kernel(const uint16_t* __restrict__ vg, long long ld,
                                                       const uint8_t* __restrict__ ops, float* __restrict__ state,
                                                       uint16_t* __restrict__ og, long long ldo, int seq, int heads,
                                                       int nchunks) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  ScanSmem& s = *reinterpret_cast<ScanSmem*>(smem_raw);
  // the value slices of one (sequence, head) are adjacent block indices, so
  // they run together and share the chunk records through L2
  const int bh = blockIdx.y, b = bh / heads, h = bh % heads;
  const int j0 = blockIdx.x * SV;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const long long tok0 = (long long)b * seq;
  const float qscale = rsqrtf((float)DK);
  float* st_g = state ? state + (long long)bh * DK * DK : nullptr;

  for (int i = tid; i < DK * SV; i += 128) {
    int r = i / SV, c = i % SV;
    float x = st_g ? st_g[r * DK + j0 + c] : 0.0f;
    s.Sf[r][c] = x;
    s.Sb[r][c] = f32_to_bf16_rne(x);
  }

  const int m0 = warp * 16;  // token rows of this warp for X, U, O
  for (int ch = 0; ch < nchunks; ++ch) {
    const int t0 = ch * C;
    const uint8_t* rec = ops + ((size_t)bh * nchunks + ch) * kChunkBytes;
    const uint16_t* big = reinterpret_cast<const uint16_t*>(rec);
    const uint16_t* small = big + kBigElems;
    const float* dend = reinterpret_cast<const float*>(small + kSmallElems);
    __syncthreads();  // previous chunk done with every buffer
    for (int i = tid; i < 3 * C * (DK / 8); i += 128) {
      int m = i / (C * (DK / 8)), rem = i % (C * (DK / 8));
      int r = rem / (DK / 8), c = (rem % (DK / 8)) * 8;
      uint16_t* dst = m == 0 ? &s.Ks[r][c] : m == 1 ? &s.Qs[r][c] : &s.Ke[r][c];
      cp_async16(dst, big + (size_t)m * C * DK + r * DK + c);
    }
    for (int i = tid; i < 2 * C * (C / 8); i += 128) {
      int m = i / (C * (C / 8)), rem = i % (C * (C / 8));
      int r = rem / (C / 8), c = (rem % (C / 8)) * 8;
      cp_async16(m == 0 ? &s.T[r][c] : &s.QK[r][c], small + (size_t)m * C * C + r * C + c);
    }
    for (int i = tid; i < C * (SV / 8); i += 128) {
      int r = i / (SV / 8), c = (i % (SV / 8)) * 8;
      if (t0 + r < seq) cp_async16(&s.V[r][c], vg + (tok0 + t0 + r) * ld + h * DK + j0 + c);
      else *reinterpret_cast<uint4*>(&s.V[r][c]) = make_uint4(0, 0, 0, 0);
    }
    for (int i = tid; i < DK / 4; i += 128) cp_async16(&s.dend[4 * i], dend + 4 * i);
    cp_async_wait_all();
    __syncthreads();

    // X = V - K~ S and O1 = Q~ S for this warp's 16 rows x 32 columns
    float xacc[4][4], oacc[4][4];
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) xacc[nt][e] = oacc[nt][e] = 0.0f;
#pragma unroll
    for (int kk = 0; kk < DK; kk += 16) {
      uint32_t ak[4], aq[4], b0[4], b1[4];
      frag_a<LQ>(&s.Ks[0][0], m0, kk, lane, ak);
      frag_a<LQ>(&s.Qs[0][0], m0, kk, lane, aq);
      frag_b_kn<LV>(&s.Sb[0][0], 0, kk, lane, b0);
      frag_b_kn<LV>(&s.Sb[0][0], 16, kk, lane, b1);
      mma16816(xacc[0], ak, b0[0], b0[1]);
      mma16816(xacc[1], ak, b0[2], b0[3]);
      mma16816(xacc[2], ak, b1[0], b1[1]);
      mma16816(xacc[3], ak, b1[2], b1[3]);
      mma16816(oacc[0], aq, b0[0], b0[1]);
      mma16816(oacc[1], aq, b0[2], b0[3]);
      mma16816(oacc[2], aq, b1[0], b1[1]);
      mma16816(oacc[3], aq, b1[2], b1[3]);
    }
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
      for (int e = 0; e < 4; e += 2) {
        int t = m0 + (lane >> 2) + (e >> 1) * 8;
        int c = nt * 8 + (lane & 3) * 2;
        uint32_t raw = *reinterpret_cast<const uint32_t*>(&s.V[t][c]);
        *reinterpret_cast<uint32_t*>(&s.XU[t][c]) =
            pack_bf16x2(bf16_to_f32(raw & 0xffffu) - xacc[nt][e], bf16_to_f32(raw >> 16) - xacc[nt][e + 1]);
      }
    __syncthreads();
    // U = T X (T already carries diag(beta))
    float uacc[4][4];
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) uacc[nt][e] = 0.0f;
#pragma unroll
    for (int kk = 0; kk < C; kk += 16) {
      uint32_t a[4], b0[4], b1[4];
      frag_a<LS>(&s.T[0][0], m0, kk, lane, a);
      frag_b_kn<LV>(&s.XU[0][0], 0, kk, lane, b0);
      frag_b_kn<LV>(&s.XU[0][0], 16, kk, lane, b1);
      mma16816(uacc[0], a, b0[0], b0[1]);
      mma16816(uacc[1], a, b0[2], b0[3]);
      mma16816(uacc[2], a, b1[0], b1[1]);
      mma16816(uacc[3], a, b1[2], b1[3]);
    }
    __syncthreads();
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
      for (int e = 0; e < 4; e += 2) {
        int t = m0 + (lane >> 2) + (e >> 1) * 8;
        int c = nt * 8 + (lane & 3) * 2;
        *reinterpret_cast<uint32_t*>(&s.XU[t][c]) = pack_bf16x2(uacc[nt][e], uacc[nt][e + 1]);
      }
    __syncthreads();
    // O = (Q~ S + QK U) / sqrt(dk)
#pragma unroll
    for (int kk = 0; kk < C; kk += 16) {
      uint32_t a[4], b0[4], b1[4];
      frag_a<LS>(&s.QK[0][0], m0, kk, lane, a);
      frag_b_kn<LV>(&s.XU[0][0], 0, kk, lane, b0);
      frag_b_kn<LV>(&s.XU[0][0], 16, kk, lane, b1);
      mma16816(oacc[0], a, b0[0], b0[1]);
      mma16816(oacc[1], a, b0[2], b0[3]);
      mma16816(oacc[2], a, b1[0], b1[1]);
      mma16816(oacc[3], a, b1[2], b1[3]);
    }
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
      for (int e = 0; e < 4; e += 2) {
        int t = m0 + (lane >> 2) + (e >> 1) * 8;
        int c = nt * 8 + (lane & 3) * 2;
        if (t0 + t < seq)
          *reinterpret_cast<uint32_t*>(og + (tok0 + t0 + t) * ldo + h * DK + j0 + c) =
              pack_bf16x2(oacc[nt][e] * qscale, oacc[nt][e + 1] * qscale);
      }
    // S = e^Gc_C o S + K^^T U : this warp owns state rows [32w, 32w + 32)
#pragma unroll
    for (int mt = 0; mt < 2; ++mt) {
      const int mi = warp * 32 + mt * 16;
      float sacc[4][4];
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) sacc[nt][0] = sacc[nt][1] = sacc[nt][2] = sacc[nt][3] = 0.0f;
#pragma unroll
      for (int kk = 0; kk < C; kk += 16) {
        uint32_t a[4], b0[4], b1[4];
        frag_a_t<LQ>(&s.Ke[0][0], mi, kk, lane, a);
        frag_b_kn<LV>(&s.XU[0][0], 0, kk, lane, b0);
        frag_b_kn<LV>(&s.XU[0][0], 16, kk, lane, b1);
        mma16816(sacc[0], a, b0[0], b0[1]);
        mma16816(sacc[1], a, b0[2], b0[3]);
        mma16816(sacc[2], a, b1[0], b1[1]);
        mma16816(sacc[3], a, b1[2], b1[3]);
      }
#pragma unroll
      for (int nt = 0; nt < 4; ++nt)
#pragma unroll
        for (int e = 0; e < 4; e += 2) {
          int i = mi + (lane >> 2) + (e >> 1) * 8;
          int c = nt * 8 + (lane & 3) * 2;
          float d = s.dend[i];
          float n0 = d * s.Sf[i][c] + sacc[nt][e];
          float n1 = d * s.Sf[i][c + 1] + sacc[nt][e + 1];
          s.Sf[i][c] = n0;
          s.Sf[i][c + 1] = n1;
          *reinterpret_cast<uint32_t*>(&s.Sb[i][c]) = pack_bf16x2(n0, n1);
        }
    }
  }
  __syncthreads();
  if (st_g)
    for (int i = tid; i < DK * SV; i += 128) st_g[(i / SV) * DK + j0 + (i % SV)] = s.Sf[i / SV][i % SV];
}

bool g_attr[64];

}  // namespace

size_t kda_workspace_bytes(int batch, int seq, int heads) {
  size_t nchunks = (size_t)(seq + C - 1) / C;
  return (size_t)batch * heads * nchunks * kChunkBytes;
}

int32_t launch_kda_chunked(const uint16_t* q, const uint16_t* k, const uint16_t* v, long long ld_qkv, const float* g,
                           const float* beta, float* state, uint16_t* o, long long ldo, int batch, int seq, int heads,
                           void* workspace, size_t workspace_bytes, cudaStream_t s, const KdaRawGate* raw) {
  if (batch <= 0 || seq <= 0 || heads <= 0) return set_error(ENNX_B200_INVALID_ARGUMENT, "kda: empty input");
  if (ld_qkv % 8 || ldo % 2 || (((uintptr_t)q | (uintptr_t)k | (uintptr_t)v) & 15u))
    return set_error(ENNX_B200_INVALID_ARGUMENT, "kda: q/k/v must be 16-byte aligned with ld %% 8 == 0");
  if (((uintptr_t)g & 15u) || ((uintptr_t)workspace & 15u))
    return set_error(ENNX_B200_INVALID_ARGUMENT, "kda: g and workspace must be 16-byte aligned");
  const size_t need = kda_workspace_bytes(batch, seq, heads);
  if (!workspace || workspace_bytes < need)
    return set_error(ENNX_B200_INVALID_ARGUMENT, "kda: workspace of %zu bytes required", need);
  int dev = 0;
  cudaGetDevice(&dev);
  if (!g_attr[dev]) {
    ENNX_CUDA(cudaFuncSetAttribute(kda_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(PrepSmem)),
              "kda prep smem");
    ENNX_CUDA(cudaFuncSetAttribute(kda_scan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(ScanSmem)),
              "kda scan smem");
    g_attr[dev] = true;
  }
  const int nchunks = (seq + C - 1) / C;
  KdaRawGate rg;
  memset(&rg, 0, sizeof(rg));
  if (raw) rg = *raw;
  if (!raw && (!g || !beta)) return set_error(ENNX_B200_INVALID_ARGUMENT, "kda: g and beta are required");
  kda_prep_kernel<<<dim3(nchunks, batch * heads), 256, sizeof(PrepSmem), s>>>(
      q, k, ld_qkv, g, (long long)heads * DK, beta, seq, heads, nchunks, rg, (uint8_t*)workspace);
  ENNX_LAUNCH_CHECK("kda prep");
  kda_scan_kernel<<<dim3(DK / SV, batch * heads), 128, sizeof(ScanSmem), s>>>(v, ld_qkv, (const uint8_t*)workspace,
                                                                               state, o, ldo, seq, heads, nchunks);
  ENNX_LAUNCH_CHECK("kda scan");
  return ENNX_B200_OK;
}

}  // namespace ennx
