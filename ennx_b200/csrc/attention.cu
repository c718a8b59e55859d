// attention.cu -- causal grouped-query attention (FlashAttention-2 style).
//
// One CTA = 128 query rows of one (batch, query head); 8 warps x 16 rows.
// K/V tiles of 64 keys stream through a double-buffered, XOR-swizzled
// shared-memory ring (cp.async 16 B), S = Q K^T and O += P V run on
// mma.sync m16n8k16 bf16 with fp32 accumulators, online softmax in fp32
// registers (exp2 domain), causal tiles beyond the diagonal are skipped.
// Head dim 128; Hq/Hkv query heads share one KV head.
//
// No reference counterpart (the reference has no attention).  Inputs may be
// strided views of a fused QKV projection: token (b, s) of head h starts at
// q + (b*seq + s)*ldq + h*128.
#include "common.cuh"
#include "kernels.cuh"

namespace ennx {
namespace {

constexpr int D = 128, BQ = 128, BKV = 64, WARPS = 8;
constexpr int ROWB = D * 2;             // bytes per smem row (256)
constexpr int TILE_BYTES = BKV * ROWB;  // 16 KB

__device__ __forceinline__ uint32_t swz(int row, int chunk) {  // byte offset of 16-B chunk
  return (uint32_t)(row * ROWB + ((chunk ^ (row & 7)) << 4));
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool pred) {
  int sz = pred ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(sz) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
__device__ __forceinline__ void mma16816(float c[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack2(float lo, float hi) { return pack_bf16x2(lo, hi); }

__global__ void __launch_bounds__(WARPS * 32, 1)
    gqa_fwd_kernel(const uint16_t* __restrict__ q, long long ldq, const uint16_t* __restrict__ k, long long ldk,
                   const uint16_t* __restrict__ v, long long ldv, uint16_t* __restrict__ o, long long ldo, int seq,
                   int hq, int hkv, float scale_log2) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* sQ = smem;                        // 128 rows
  uint8_t* sK = smem + BQ * ROWB;            // 2 x 64 rows
  uint8_t* sV = sK + 2 * TILE_BYTES;         // 2 x 64 rows
  const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int kh = h / (hq / hkv);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int q0 = qt * BQ;
  const long long tok0 = (long long)b * seq;

  // Q tile -> smem
  for (int i = tid; i < BQ * 16; i += WARPS * 32) {
    int r = i >> 4, c = i & 15;
    bool ok = q0 + r < seq;
    cp_async16(smem_u32(sQ) + swz(r, c), q + (tok0 + (ok ? q0 + r : 0)) * ldq + h * D + c * 8, ok);
  }
  auto load_kv = [&](int j, int buf) {
    int k0 = j * BKV;
    for (int i = tid; i < BKV * 16; i += WARPS * 32) {
      int r = i >> 4, c = i & 15;
      bool ok = k0 + r < seq;
      long long tok = tok0 + (ok ? k0 + r : 0);
      cp_async16(smem_u32(sK + buf * TILE_BYTES) + swz(r, c), k + tok * ldk + kh * D + c * 8, ok);
      cp_async16(smem_u32(sV + buf * TILE_BYTES) + swz(r, c), v + tok * ldv + kh * D + c * 8, ok);
    }
  };
  const int last_q = min(q0 + BQ, seq) - 1;
  const int nkv = last_q / BKV + 1;  // causal: tiles up to the diagonal
  load_kv(0, 0);
  cp_async_commit();

  uint32_t qf[8][4];
  float oacc[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) oacc[i][0] = oacc[i][1] = oacc[i][2] = oacc[i][3] = 0.0f;
  float m_r[2] = {-INFINITY, -INFINITY}, l_r[2] = {0.0f, 0.0f};
  const int wrow0 = q0 + warp * 16;           // first query row of this warp
  const int qrow_a = wrow0 + (lane >> 2);     // rows owned by this thread
  const int qrow_b = qrow_a + 8;

  for (int j = 0; j < nkv; ++j) {
    if (j + 1 < nkv) load_kv(j + 1, (j + 1) & 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    if (j == 0) {
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        int r = warp * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        int c = kk * 2 + (lane >> 4);
        ldsm_x4(smem_u32(sQ) + swz(r, c), qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3]);
      }
    }
    const int buf = j & 1;
    const uint32_t kb = smem_u32(sK + buf * TILE_BYTES), vb = smem_u32(sV + buf * TILE_BYTES);
    const int k0 = j * BKV;
    if (k0 <= wrow0 + 15) {  // warp has at least one unmasked key in this tile
      float s[8][4];
#pragma unroll
      for (int n = 0; n < 8; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.0f;
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
#pragma unroll
        for (int np = 0; np < 4; ++np) {  // pairs of n-tiles (16 keys)
          int r = np * 16 + (lane & 7) + (lane >> 4) * 8;
          int c = kk * 2 + ((lane >> 3) & 1);
          uint32_t b0, b1, b2, b3;
          ldsm_x4(kb + swz(r, c), b0, b1, b2, b3);
          mma16816(s[2 * np], qf[kk], b0, b1);
          mma16816(s[2 * np + 1], qf[kk], b2, b3);
        }
      }
      // scale, causal mask, online softmax (two rows per thread)
      float mx[2] = {m_r[0], m_r[1]};
#pragma unroll
      for (int n = 0; n < 8; ++n) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          int key = k0 + n * 8 + (lane & 3) * 2 + (e & 1);
          int row = e < 2 ? qrow_a : qrow_b;
          float x = s[n][e] * scale_log2;
          if (key > row || key >= seq) x = -INFINITY;
          s[n][e] = x;
          mx[e >> 1] = fmaxf(mx[e >> 1], x);
        }
      }
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        mx[i] = fmaxf(mx[i], __shfl_xor_sync(0xffffffffu, mx[i], 1));
        mx[i] = fmaxf(mx[i], __shfl_xor_sync(0xffffffffu, mx[i], 2));
      }
      float corr[2], rs[2] = {0.0f, 0.0f};
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        corr[i] = mx[i] == -INFINITY ? 1.0f : exp2f(m_r[i] - mx[i]);
        m_r[i] = mx[i];
      }
#pragma unroll
      for (int n = 0; n < 8; ++n) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float mm = m_r[e >> 1];
          float p = mm == -INFINITY ? 0.0f : exp2f(s[n][e] - mm);
          s[n][e] = p;
          rs[e >> 1] += p;
        }
      }
#pragma unroll
      for (int i = 0; i < 2; ++i) l_r[i] = l_r[i] * corr[i] + rs[i];
#pragma unroll
      for (int n = 0; n < 16; ++n) {
        oacc[n][0] *= corr[0]; oacc[n][1] *= corr[0];
        oacc[n][2] *= corr[1]; oacc[n][3] *= corr[1];
      }
      // O += P V
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {  // 16 keys per k-step
        uint32_t a[4] = {pack2(s[2 * kk][0], s[2 * kk][1]), pack2(s[2 * kk][2], s[2 * kk][3]),
                         pack2(s[2 * kk + 1][0], s[2 * kk + 1][1]), pack2(s[2 * kk + 1][2], s[2 * kk + 1][3])};
#pragma unroll
        for (int np = 0; np < 8; ++np) {  // pairs of d n-tiles
          int r = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
          int c = np * 2 + (lane >> 4);
          uint32_t b0, b1, b2, b3;
          ldsm_x4_t(vb + swz(r, c), b0, b1, b2, b3);
          mma16816(oacc[2 * np], a, b0, b1);
          mma16816(oacc[2 * np + 1], a, b2, b3);
        }
      }
    }
    __syncthreads();
  }

  // normalise and store
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    l_r[i] += __shfl_xor_sync(0xffffffffu, l_r[i], 1);
    l_r[i] += __shfl_xor_sync(0xffffffffu, l_r[i], 2);
  }
  float inv[2] = {l_r[0] > 0.0f ? 1.0f / l_r[0] : 0.0f, l_r[1] > 0.0f ? 1.0f / l_r[1] : 0.0f};
#pragma unroll
  for (int n = 0; n < 16; ++n) {
    int col = h * D + n * 8 + (lane & 3) * 2;
    if (qrow_a < seq)
      *reinterpret_cast<uint32_t*>(o + (tok0 + qrow_a) * ldo + col) = pack2(oacc[n][0] * inv[0], oacc[n][1] * inv[0]);
    if (qrow_b < seq)
      *reinterpret_cast<uint32_t*>(o + (tok0 + qrow_b) * ldo + col) = pack2(oacc[n][2] * inv[1], oacc[n][3] * inv[1]);
  }
}

constexpr int SMEM = BQ * ROWB + 4 * TILE_BYTES;  // 96 KB
bool g_attr[64];

}  // namespace

int32_t launch_gqa_attention(const uint16_t* q, long long ldq, const uint16_t* k, long long ldk, const uint16_t* v,
                             long long ldv, uint16_t* o, long long ldo, int batch, int seq, int hq, int hkv,
                             cudaStream_t s) {
  if (hkv <= 0 || hq % hkv) return set_error(ENNX_B200_INVALID_ARGUMENT, "attention: Hq must be a multiple of Hkv");
  if (seq <= 0 || batch <= 0) return set_error(ENNX_B200_INVALID_ARGUMENT, "attention: empty input");
  if ((ldq | ldk | ldv | ldo) % 8 || (((uintptr_t)q | (uintptr_t)k | (uintptr_t)v | (uintptr_t)o) & 15u))
    return set_error(ENNX_B200_INVALID_ARGUMENT, "attention: operands must be 16-byte aligned");
  int dev = 0;
  cudaGetDevice(&dev);
  if (!g_attr[dev]) {
    ENNX_CUDA(cudaFuncSetAttribute(gqa_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM), "attn smem");
    g_attr[dev] = true;
  }
  dim3 grid((seq + BQ - 1) / BQ, hq, batch);
  const float scale_log2 = 1.4426950408889634f / sqrtf((float)D);
  gqa_fwd_kernel<<<grid, WARPS * 32, SMEM, s>>>(q, ldq, k, ldk, v, ldv, o, ldo, seq, hq, hkv, scale_log2);
  ENNX_LAUNCH_CHECK("gqa attention");
  return ENNX_B200_OK;
}

}  // namespace ennx
