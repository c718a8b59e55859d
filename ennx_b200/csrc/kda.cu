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
// One CTA owns one (sequence, head) and 64 of the 128 value columns; it walks
// the chunks in order with the fp32 state slice resident in shared memory.
// The contractions (7 per chunk) run on mma.sync m16n8k16 bf16 tensor cores
// with fp32 accumulation; cumulative decays, the 16x16 triangular inverses
// and the state update stay fp32.
#include "common.cuh"
#include "kernels.cuh"

namespace ennx {
namespace {

constexpr int C = 64, DK = 128, DVS = 64, THREADS = 256;
constexpr int LQ = DK + 8;   // padded bf16 row (elements) for [64][128] tiles
constexpr int LS = DVS + 8;  // padded bf16 row for [*][64] tiles
constexpr int LF = C + 1;    // padded fp32 row for [64][64] matrices

struct KdaSmem {
  float Sf[DK][DVS];        // state slice, fp32 master
  float Gc[C][DK];          // cumulative log decay of the chunk
  float L[C][LF];           // beta_t * A'[t,s] (strictly lower)
  float Tf[C][LF];          // (I + L)^-1
  float beta[C];
  uint16_t q[C][LQ], k[C][LQ];
  uint16_t X[C][LQ], Y[C][LQ];  // scaled operands
  uint16_t Sb[DK][LS];          // bf16 copy of the state slice
  uint16_t WU[C][LS];           // W, then U
  uint16_t Tb[C][LS];           // bf16 (I + L)^-1
  uint16_t QK[C][LS];           // masked intra-chunk q.k products
};

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

// A fragment (16 x 16) at (m0, k0) of a row-major [m][k] bf16 tile.
template <int LD>
__device__ __forceinline__ void frag_a(const uint16_t* base, int m0, int k0, int lane, uint32_t a[4]) {
  const uint16_t* p = base + (m0 + (lane & 7) + ((lane >> 3) & 1) * 8) * LD + k0 + (lane >> 4) * 8;
  ldsm_x4(p, a[0], a[1], a[2], a[3]);
}
// A fragment (16 x 16) at (m0, k0) of a tile stored transposed, [k][m].
template <int LD>
__device__ __forceinline__ void frag_a_t(const uint16_t* base, int m0, int k0, int lane, uint32_t a[4]) {
  const uint16_t* p = base + (k0 + (lane & 7) + (lane >> 4) * 8) * LD + m0 + ((lane >> 3) & 1) * 8;
  ldsm_x4_t(p, a[0], a[1], a[2], a[3]);
}
// B fragments for n-tiles n0 and n0+8 (k0..k0+15) of a tile stored [n][k].
template <int LD>
__device__ __forceinline__ void frag_b_nk(const uint16_t* base, int n0, int k0, int lane, uint32_t b[4]) {
  const uint16_t* p = base + (n0 + (lane & 7) + (lane >> 4) * 8) * LD + k0 + ((lane >> 3) & 1) * 8;
  ldsm_x4(p, b[0], b[1], b[2], b[3]);
}
// B fragments for n-tiles n0 and n0+8 of a tile stored [k][n].
template <int LD>
__device__ __forceinline__ void frag_b_kn(const uint16_t* base, int n0, int k0, int lane, uint32_t b[4]) {
  const uint16_t* p = base + (k0 + (lane & 7) + ((lane >> 3) & 1) * 8) * LD + n0 + (lane >> 4) * 8;
  ldsm_x4_t(p, b[0], b[1], b[2], b[3]);
}

__global__ void __launch_bounds__(THREADS, 1)
    kda_chunk_kernel(const uint16_t* __restrict__ qg, const uint16_t* __restrict__ kg, const uint16_t* __restrict__ vg,
                     long long ld, const float* __restrict__ gg, long long ldg, const float* __restrict__ bg,
                     float* __restrict__ state, uint16_t* __restrict__ og, long long ldo, int seq, int heads) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  KdaSmem& s = *reinterpret_cast<KdaSmem*>(smem_raw);
  const int bh = blockIdx.x, b = bh / heads, h = bh % heads;
  const int j0 = blockIdx.y * DVS;  // value-column slice
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const long long tok0 = (long long)b * seq;
  const float qscale = rsqrtf((float)DK);
  float* st_g = state ? state + ((long long)bh * DK) * DK : nullptr;  // [DK][DK] per (b, h)

  for (int i = tid; i < DK * DVS; i += THREADS) {
    int r = i / DVS, c = i % DVS;
    float x = st_g ? st_g[r * DK + j0 + c] : 0.0f;
    s.Sf[r][c] = x;
    s.Sb[r][c] = f32_to_bf16_rne(x);
  }
  const int nchunks = (seq + C - 1) / C;

  for (int ch = 0; ch < nchunks; ++ch) {
    const int t0 = ch * C;
    // ---- S1: load q, k (bf16), beta; cumulative decay per channel -----------
    for (int i = tid; i < C * (DK / 8); i += THREADS) {
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
    if (tid < C) s.beta[tid] = t0 + tid < seq ? bg[(tok0 + t0 + tid) * heads + h] : 0.0f;
    if (tid < DK) {
      float acc = 0.0f;
      for (int t = 0; t < C; ++t) {
        if (t0 + t < seq) acc += gg[(tok0 + t0 + t) * ldg + h * DK + tid];
        s.Gc[t][tid] = acc;
      }
    }
    __syncthreads();

    // ---- S2: intra-chunk products, one 16-row block at a time ------------
    for (int blk = 0; blk < 4; ++blk) {
      const int r = blk * 16, ns = r + 16;
      for (int i = tid; i < 32 * DK; i += THREADS) {  // X rows: 16 of q-scaled, 16 of k-scaled
        int row = i / DK, c = i % DK;
        int t = r + (row & 15);
        float e = __expf(s.Gc[t][c] - s.Gc[r][c]);
        float src = bf16_to_f32(row < 16 ? s.q[t][c] : s.k[t][c]);
        s.X[row][c] = f32_to_bf16_rne(src * e);
      }
      for (int i = tid; i < ns * DK; i += THREADS) {
        int t = i / DK, c = i % DK;
        s.Y[t][c] = f32_to_bf16_rne(bf16_to_f32(s.k[t][c]) * __expf(s.Gc[r][c] - s.Gc[t][c]));
      }
      __syncthreads();
      const int ntiles = ns / 8;  // n-tiles of 8 columns, two matrices
      for (int task = warp; task < 2 * (ntiles / 2); task += THREADS / 32) {
        const int which = task / (ntiles / 2);  // 0: QK, 1: A'
        const int n0 = (task % (ntiles / 2)) * 16;
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
          for (int e = 0; e < 4; ++e) {
            int t = r + (lane >> 2) + (e >> 1) * 8;
            int sc = n0 + nt * 8 + (lane & 3) * 2 + (e & 1);
            float x = acc[nt][e];
            if (which == 0) s.QK[t][sc] = f32_to_bf16_rne(sc <= t ? x : 0.0f);
            else s.L[t][sc] = sc < t ? s.beta[t] * x : 0.0f;
          }
      }
      // zero the part of rows [r, r+16) right of the computed columns
      for (int i = tid; i < 16 * (C - ns); i += THREADS) {
        int t = r + i / (C - ns), sc = ns + i % (C - ns);
        s.QK[t][sc] = 0;
        s.L[t][sc] = 0.0f;
      }
      __syncthreads();
    }

    // ---- S3: T = (I + L)^-1 by 16x16 diagonal inverses + block recursion ----
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
      for (int t = 0; t < 16; ++t) s.Tf[d0 + t][d0 + jj] = x[t];
    }
    __syncthreads();
    for (int bi = 1; bi < 4; ++bi) {
      // M[bj] = sum_{bk=bj}^{bi-1} L[bi,bk] T[bk,bj]  -> stored in Tf[bi,bj] temporarily
      float mloc[4];
      int cnt = 0;
      for (int i = tid; i < bi * 256; i += THREADS, ++cnt) {
        int bj = i / 256, e = i % 256, rr = e / 16, cc = e % 16;
        float acc = 0.0f;
        for (int kx = bj * 16; kx < bi * 16; ++kx) acc += s.L[bi * 16 + rr][kx] * s.Tf[kx][bj * 16 + cc];
        mloc[cnt] = acc;
      }
      __syncthreads();
      cnt = 0;
      for (int i = tid; i < bi * 256; i += THREADS, ++cnt) {
        int bj = i / 256, e = i % 256, rr = e / 16, cc = e % 16;
        s.Tf[bi * 16 + rr][bj * 16 + cc] = mloc[cnt];
      }
      __syncthreads();
      cnt = 0;
      for (int i = tid; i < bi * 256; i += THREADS, ++cnt) {
        int bj = i / 256, e = i % 256, rr = e / 16, cc = e % 16;
        float acc = 0.0f;
        for (int kx = 0; kx < 16; ++kx) acc -= s.Tf[bi * 16 + rr][bi * 16 + kx] * s.Tf[bi * 16 + kx][bj * 16 + cc];
        mloc[cnt] = acc;
      }
      __syncthreads();
      cnt = 0;
      for (int i = tid; i < bi * 256; i += THREADS, ++cnt) {
        int bj = i / 256, e = i % 256, rr = e / 16, cc = e % 16;
        s.Tf[bi * 16 + rr][bj * 16 + cc] = mloc[cnt];
      }
      __syncthreads();
    }
    for (int i = tid; i < C * C; i += THREADS) {
      int rr = i / C, cc = i % C;
      s.Tb[rr][cc] = f32_to_bf16_rne(cc <= rr ? s.Tf[rr][cc] : 0.0f);
    }
    // ---- S4: X <- k o e^Gc, Y <- q o e^Gc --------------------------------
    for (int i = tid; i < C * DK; i += THREADS) {
      int t = i / DK, c = i % DK;
      float e = __expf(s.Gc[t][c]);
      s.X[t][c] = f32_to_bf16_rne(bf16_to_f32(s.k[t][c]) * e);
      s.Y[t][c] = f32_to_bf16_rne(bf16_to_f32(s.q[t][c]) * e);
    }
    __syncthreads();
    // warp tile: rows m0 = 16*(warp/2), columns 32*(warp%2) .. +31 (4 n-tiles)
    const int m0 = 16 * (warp >> 1), nb = 32 * (warp & 1);
    float wacc[4][4], oacc[4][4];
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) wacc[nt][e] = oacc[nt][e] = 0.0f;
#pragma unroll
    for (int kk = 0; kk < DK; kk += 16) {
      uint32_t ak[4], aq[4], b0[4], b1[4];
      frag_a<LQ>(&s.X[0][0], m0, kk, lane, ak);
      frag_a<LQ>(&s.Y[0][0], m0, kk, lane, aq);
      frag_b_kn<LS>(&s.Sb[0][0], nb, kk, lane, b0);
      frag_b_kn<LS>(&s.Sb[0][0], nb + 16, kk, lane, b1);
      mma16816(wacc[0], ak, b0[0], b0[1]);
      mma16816(wacc[1], ak, b0[2], b0[3]);
      mma16816(wacc[2], ak, b1[0], b1[1]);
      mma16816(wacc[3], ak, b1[2], b1[3]);
      mma16816(oacc[0], aq, b0[0], b0[1]);
      mma16816(oacc[1], aq, b0[2], b0[3]);
      mma16816(oacc[2], aq, b1[0], b1[1]);
      mma16816(oacc[3], aq, b1[2], b1[3]);
    }
    // W = beta (v - K~ S0)
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
      for (int e = 0; e < 4; e += 2) {
        int t = m0 + (lane >> 2) + (e >> 1) * 8;
        int c = nb + nt * 8 + (lane & 3) * 2;
        float v0 = 0.0f, v1 = 0.0f;
        if (t0 + t < seq) {
          uint32_t raw = *reinterpret_cast<const uint32_t*>(vg + (tok0 + t0 + t) * ld + h * DK + j0 + c);
          v0 = bf16_to_f32(raw & 0xffffu);
          v1 = bf16_to_f32(raw >> 16);
        }
        float bt = s.beta[t];
        *reinterpret_cast<uint32_t*>(&s.WU[t][c]) = pack_bf16x2(bt * (v0 - wacc[nt][e]), bt * (v1 - wacc[nt][e + 1]));
      }
    __syncthreads();
    // ---- S5: U = T W --------------------------------------------------------
    float uacc[4][4];
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) uacc[nt][e] = 0.0f;
#pragma unroll
    for (int kk = 0; kk < C; kk += 16) {
      uint32_t a[4], b0[4], b1[4];
      frag_a<LS>(&s.Tb[0][0], m0, kk, lane, a);
      frag_b_kn<LS>(&s.WU[0][0], nb, kk, lane, b0);
      frag_b_kn<LS>(&s.WU[0][0], nb + 16, kk, lane, b1);
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
        int c = nb + nt * 8 + (lane & 3) * 2;
        *reinterpret_cast<uint32_t*>(&s.WU[t][c]) = pack_bf16x2(uacc[nt][e], uacc[nt][e + 1]);
      }
    __syncthreads();
    // ---- S6: O = (Q~ S0 + QK U) / sqrt(dk) -------------------------------
#pragma unroll
    for (int kk = 0; kk < C; kk += 16) {
      uint32_t a[4], b0[4], b1[4];
      frag_a<LS>(&s.QK[0][0], m0, kk, lane, a);
      frag_b_kn<LS>(&s.WU[0][0], nb, kk, lane, b0);
      frag_b_kn<LS>(&s.WU[0][0], nb + 16, kk, lane, b1);
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
        int c = nb + nt * 8 + (lane & 3) * 2;
        if (t0 + t < seq)
          *reinterpret_cast<uint32_t*>(og + (tok0 + t0 + t) * ldo + h * DK + j0 + c) =
              pack_bf16x2(oacc[nt][e] * qscale, oacc[nt][e + 1] * qscale);
      }
    // ---- S7: state update S = e^Gc_end S + (K o e^(Gc_end - Gc))^T U ------
    for (int i = tid; i < C * DK; i += THREADS) {
      int t = i / DK, c = i % DK;
      s.X[t][c] = f32_to_bf16_rne(bf16_to_f32(s.k[t][c]) * __expf(s.Gc[C - 1][c] - s.Gc[t][c]));
    }
    __syncthreads();
    {
      const int mi = 16 * warp;  // state rows (key channels) of this warp
      float sacc[8][4];
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) sacc[nt][0] = sacc[nt][1] = sacc[nt][2] = sacc[nt][3] = 0.0f;
#pragma unroll
      for (int kk = 0; kk < C; kk += 16) {
        uint32_t a[4];
        frag_a_t<LQ>(&s.X[0][0], mi, kk, lane, a);
#pragma unroll
        for (int np = 0; np < 4; ++np) {
          uint32_t bb[4];
          frag_b_kn<LS>(&s.WU[0][0], np * 16, kk, lane, bb);
          mma16816(sacc[2 * np], a, bb[0], bb[1]);
          mma16816(sacc[2 * np + 1], a, bb[2], bb[3]);
        }
      }
#pragma unroll
      for (int nt = 0; nt < 8; ++nt)
#pragma unroll
        for (int e = 0; e < 4; e += 2) {
          int i = mi + (lane >> 2) + (e >> 1) * 8;
          int c = nt * 8 + (lane & 3) * 2;
          float d = __expf(s.Gc[C - 1][i]);
          float n0 = d * s.Sf[i][c] + sacc[nt][e];
          float n1 = d * s.Sf[i][c + 1] + sacc[nt][e + 1];
          s.Sf[i][c] = n0;
          s.Sf[i][c + 1] = n1;
          *reinterpret_cast<uint32_t*>(&s.Sb[i][c]) = pack_bf16x2(n0, n1);
        }
    }
    __syncthreads();
  }
  if (st_g)
    for (int i = tid; i < DK * DVS; i += THREADS) st_g[(i / DVS) * DK + j0 + (i % DVS)] = s.Sf[i / DVS][i % DVS];
}

bool g_attr[64];

}  // namespace

int32_t launch_kda_chunked(const uint16_t* q, const uint16_t* k, const uint16_t* v, long long ld_qkv, const float* g,
                           const float* beta, float* state, uint16_t* o, long long ldo, int batch, int seq, int heads,
                           cudaStream_t s) {
  if (batch <= 0 || seq <= 0 || heads <= 0) return set_error(ENNX_B200_INVALID_ARGUMENT, "kda: empty input");
  if (ld_qkv % 8 || ldo % 2 || (((uintptr_t)q | (uintptr_t)k | (uintptr_t)v) & 15u))
    return set_error(ENNX_B200_INVALID_ARGUMENT, "kda: q/k/v must be 16-byte aligned with ld %% 8 == 0");
  int dev = 0;
  cudaGetDevice(&dev);
  const int smem = (int)sizeof(KdaSmem);
  if (!g_attr[dev]) {
    ENNX_CUDA(cudaFuncSetAttribute(kda_chunk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem), "kda smem");
    g_attr[dev] = true;
  }
  dim3 grid(batch * heads, DK / DVS);
  kda_chunk_kernel<<<grid, THREADS, smem, s>>>(q, k, v, ld_qkv, g, (long long)heads * DK, beta, state, o, ldo, seq,
                                              heads);
  ENNX_LAUNCH_CHECK("kda chunked");
  return ENNX_B200_OK;
}

}  // namespace ennx
