// norm.cu -- memory-bound elementwise/normalisation kernels of the hybrid
// forward: RMSNorm, embedding gather, per-head L2 norm, KDA gate/beta,
// KDA output norm + gate, RoPE.  One warp per row (or per token-head),
// 16-byte loads, warp-shuffle reductions, fp32 math, bf16 RNE stores.
//
// Formulas restate rust/crates/ennx/src/kda_moe.metal:
//   decoder_rms_norm          :536-554
//   kda_normalize_qk          :510-534
//   kda_make_gate_beta_16k    :869-895
//   kda_postprocess_16k       :898-921
//   token_embedding_lookup    :990-1003
// RoPE has no reference counterpart (rotate-half pairing, theta given).
#include "common.cuh"
#include "kernels.cuh"

namespace ennx {

__device__ __forceinline__ void unpack8(uint4 v, float f[8]) {
  uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = bf16_to_f32((uint16_t)(w[i] & 0xffffu));
    f[2 * i + 1] = bf16_to_f32((uint16_t)(w[i] >> 16));
  }
}
__device__ __forceinline__ uint4 pack8(const float f[8]) {
  return make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]), pack_bf16x2(f[4], f[5]),
                    pack_bf16x2(f[6], f[7]));
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
// warp_sum over the 32 values p[2l + e] held as (p0, p1) by lane l of a
// half-warp: the same additions in the same tree order, so the same float
// result (lane 2l + e ^ 16 is half-lane l ^ 8, and so on; the last step adds
// the lane's own pair)
__device__ __forceinline__ float half_warp_pair_sum(float p0, float p1) {
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) {
    p0 += __shfl_xor_sync(0xffffffffu, p0, o);
    p1 += __shfl_xor_sync(0xffffffffu, p1, o);
  }
  return p0 + p1;
}

// y = x * rsqrt(mean(x^2) + eps) * w; rows [0, split) use w0, the rest w1.
__global__ void rmsnorm_kernel(const uint16_t* __restrict__ x, long long ldx, const uint16_t* __restrict__ w0,
                               const uint16_t* __restrict__ w1, long long split, uint16_t* __restrict__ out,
                               long long ldo, long long rows, int width, float eps) {
  long long row = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const uint16_t* w = row < split ? w0 : w1;
  const uint16_t* xr = x + row * ldx;
  float ss = 0.0f;
  for (int c = lane * 8; c < width; c += 256) {
    float f[8];
    unpack8(*reinterpret_cast<const uint4*>(xr + c), f);
#pragma unroll
    for (int i = 0; i < 8; ++i) ss = fmaf(f[i], f[i], ss);
  }
  ss = warp_sum(ss);
  float inv = rsqrtf(ss / (float)width + eps);
  uint16_t* o = out + row * ldo;
  for (int c = lane * 8; c < width; c += 256) {
    float f[8], g[8];
    unpack8(*reinterpret_cast<const uint4*>(xr + c), f);
    unpack8(*reinterpret_cast<const uint4*>(w + c), g);
#pragma unroll
    for (int i = 0; i < 8; ++i) f[i] = f[i] * inv * g[i];
    *reinterpret_cast<uint4*>(o + c) = pack8(f);
  }
}

// hidden[r] = table_s[tokens[r % per_set]] for r in set s (s = r / per_set).
// With `noise` (the pair's bf16 noise step of the table), the rows are formed
// as t0 + noise (set 0) and t0 - noise (set 1), one RNE rounding each: the
// perturbed embedding of the antithetic pair, never stored as a table.
__global__ void embed_kernel(const int* __restrict__ tokens, const uint16_t* __restrict__ t0,
                             const uint16_t* __restrict__ t1, const uint16_t* __restrict__ noise, long long per_set,
                             long long rows, int width, int vocab, uint16_t* __restrict__ out, int* err) {
  long long row = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  int lane = threadIdx.x & 31;
  if (row >= rows) return;
  int tok = tokens[row % per_set];
  if (tok < 0 || tok >= vocab) {
    if (lane == 0) atomicExch(err, ENNX_B200_INVALID_ARGUMENT);
    tok = 0;
  }
  uint16_t* dst = out + row * width;
  if (noise) {
    const uint16_t* src = t0 + (long long)tok * width;
    const uint16_t* nz = noise + (long long)tok * width;
    const bool plus = row < per_set;
    for (int c = lane * 8; c < width; c += 256) {
      const uint4 w = *reinterpret_cast<const uint4*>(src + c), e = *reinterpret_cast<const uint4*>(nz + c);
      *reinterpret_cast<uint4*>(dst + c) =
          plus ? make_uint4(bf16x2_add(w.x, e.x), bf16x2_add(w.y, e.y), bf16x2_add(w.z, e.z), bf16x2_add(w.w, e.w))
               : make_uint4(bf16x2_sub(w.x, e.x), bf16x2_sub(w.y, e.y), bf16x2_sub(w.z, e.z), bf16x2_sub(w.w, e.w));
    }
    return;
  }
  const uint16_t* src = (row < per_set ? t0 : t1) + (long long)tok * width;
  for (int c = lane * 8; c < width; c += 256)
    *reinterpret_cast<uint4*>(dst + c) = *reinterpret_cast<const uint4*>(src + c);
}

// In-place per-head L2 normalisation, 1/max(|x|, 1e-6), head width 128.
// groups = rows * heads; head h of row r starts at base + r*ld + h*128.
__global__ void l2norm_heads_kernel(uint16_t* __restrict__ base, long long ld, int heads, long long groups) {
  long long gidx = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  int lane = threadIdx.x & 31;
  if (gidx >= groups) return;
  uint16_t* p = base + (gidx / heads) * ld + (gidx % heads) * 128 + lane * 4;
  uint2 raw = *reinterpret_cast<uint2*>(p);
  float f[4] = {bf16_to_f32(raw.x & 0xffffu), bf16_to_f32(raw.x >> 16), bf16_to_f32(raw.y & 0xffffu),
                bf16_to_f32(raw.y >> 16)};
  float ss = warp_sum(f[0] * f[0] + f[1] * f[1] + f[2] * f[2] + f[3] * f[3]);
  float inv = 1.0f / fmaxf(sqrtf(ss), 1e-6f);
  *reinterpret_cast<uint2*>(p) = make_uint2(pack_bf16x2(f[0] * inv, f[1] * inv), pack_bf16x2(f[2] * inv, f[3] * inv));
}

__device__ __forceinline__ float softplus_stable(float x) { return fmaxf(x, 0.0f) + log1pf(__expf(-fabsf(x))); }

// g[r, j] = max(-exp(decay[h]) * softplus(raw[r, j] + time_bias[j]), -5)   (fp32 out)
// beta[r, h] = sigmoid(raw_beta[r, h])                                       (fp32 out)
// Parameters (decay, time_bias) are bf16 and per set (rows < split use set 0).
__global__ void kda_gate_kernel(const uint16_t* __restrict__ raw, long long ldraw, const uint16_t* __restrict__ rbeta,
                                long long ldb, const uint16_t* __restrict__ decay0, const uint16_t* __restrict__ decay1,
                                const uint16_t* __restrict__ tb0, const uint16_t* __restrict__ tb1, long long split,
                                long long rows, int heads, int head_width, float* __restrict__ gate,
                                float* __restrict__ beta) {
  int width = heads * head_width;
  long long total = rows * (long long)width;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    long long r = i / width;
    int j = (int)(i % width);
    int h = j / head_width;
    bool s0 = r < split;
    float x = bf16_to_f32(raw[r * ldraw + j]) + bf16_to_f32((s0 ? tb0 : tb1)[j]);
    float g = -__expf(bf16_to_f32((s0 ? decay0 : decay1)[h])) * softplus_stable(x);
    gate[i] = fmaxf(g, -5.0f);
    if (j % head_width == 0) beta[r * heads + h] = 1.0f / (1.0f + __expf(-bf16_to_f32(rbeta[r * ldb + h])));
  }
}

// out = rmsnorm_head(o) * norm * sigmoid(og), head width 128; norm per set.
// Per-head RMSNorm x norm weight x sigmoid(output gate).  A half-warp per
// (row, head): lane l of the half holds elements 8l..8l+7 (16-byte loads).
__global__ void kda_post_kernel(const uint16_t* __restrict__ o, const uint16_t* __restrict__ og, long long ldog,
                                const uint16_t* __restrict__ n0, const uint16_t* __restrict__ n1, long long split,
                                int heads, long long groups, float eps, uint16_t* __restrict__ out) {
  const long long g_raw = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 4;
  const int l = threadIdx.x & 15;
  const bool ok = g_raw < groups;  // no early exit: the shuffles span the whole warp
  const long long gidx = ok ? g_raw : groups - 1;
  const long long r = gidx / heads;
  const int h = (int)(gidx % heads);
  const long long off = r * (long long)heads * 128 + h * 128 + l * 8;
  const uint4 raw = *reinterpret_cast<const uint4*>(o + off);
  const uint4 graw = *reinterpret_cast<const uint4*>(og + r * ldog + h * 128 + l * 8);
  const uint4 nraw = *reinterpret_cast<const uint4*>((r < split ? n0 : n1) + l * 8);
  const uint32_t ow[4] = {raw.x, raw.y, raw.z, raw.w}, gw[4] = {graw.x, graw.y, graw.z, graw.w},
                 nw[4] = {nraw.x, nraw.y, nraw.z, nraw.w};
  float f[8], g[8], n[8];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    f[2 * j] = bf16_to_f32(ow[j] & 0xffffu); f[2 * j + 1] = bf16_to_f32(ow[j] >> 16);
    g[2 * j] = bf16_to_f32(gw[j] & 0xffffu); g[2 * j + 1] = bf16_to_f32(gw[j] >> 16);
    n[2 * j] = bf16_to_f32(nw[j] & 0xffffu); n[2 * j + 1] = bf16_to_f32(nw[j] >> 16);
  }
  // sum of squares over the head: partials of 4 consecutive elements, summed
  // over the head in warp_sum's order
  float p0 = f[0] * f[0] + f[1] * f[1] + f[2] * f[2] + f[3] * f[3];
  float p1 = f[4] * f[4] + f[5] * f[5] + f[6] * f[6] + f[7] * f[7];
  float ss = half_warp_pair_sum(p0, p1);
  const float inv = rsqrtf(ss / 128.0f + eps);
  float y[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) y[i] = f[i] * inv * n[i] / (1.0f + __expf(-g[i]));
  if (ok)
    *reinterpret_cast<uint4*>(out + off) = make_uint4(pack_bf16x2(y[0], y[1]), pack_bf16x2(y[2], y[3]),
                                                      pack_bf16x2(y[4], y[5]), pack_bf16x2(y[6], y[7]));
}

// Rotate-half RoPE in place on `heads` heads of width dim starting at base + r*ld.
// Position of row r is r % seq.  One thread per (row, 8 rotary pairs): the
// eight angles (inv_freq = 2^(-log2(theta) 2k/dim), angle = pos inv_freq,
// the per-element formula) are computed once and applied to that chunk of
// every head, with 16-byte loads of x[k0..k0+7] and x[k0+half..k0+half+7].
__global__ void rope_kernel(uint16_t* __restrict__ base, long long ld, int heads, int dim, long long rows, int seq,
                            float log2_theta) {
  const int half = dim / 2, cpr = half / 8;  // 8-pair chunks per head
  const long long total = rows * cpr;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / cpr;
    const int k0 = (int)(i - r * cpr) * 8;
    const float pos = (float)(r % seq);
    float sn[8], cs[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float inv_freq = exp2f(-log2_theta * (2.0f * (k0 + e) / (float)dim));
      sincosf(pos * inv_freq, &sn[e], &cs[e]);
    }
    uint16_t* row = base + r * ld + k0;
#pragma unroll 4
    for (int h = 0; h < heads; ++h) {
      uint16_t* p = row + (long long)h * dim;
      const uint4 a = *reinterpret_cast<const uint4*>(p), b = *reinterpret_cast<const uint4*>(p + half);
      const uint32_t aw[4] = {a.x, a.y, a.z, a.w}, bw[4] = {b.x, b.y, b.z, b.w};
      uint32_t ya[4], yb[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float o1[2], o2[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float x1 = bf16_to_f32((uint16_t)(aw[j] >> (16 * e))), x2 = bf16_to_f32((uint16_t)(bw[j] >> (16 * e)));
          o1[e] = x1 * cs[2 * j + e] - x2 * sn[2 * j + e];
          o2[e] = x2 * cs[2 * j + e] + x1 * sn[2 * j + e];
        }
        ya[j] = pack_bf16x2(o1[0], o1[1]);
        yb[j] = pack_bf16x2(o2[0], o2[1]);
      }
      *reinterpret_cast<uint4*>(p) = make_uint4(ya[0], ya[1], ya[2], ya[3]);
      *reinterpret_cast<uint4*>(p + half) = make_uint4(yb[0], yb[1], yb[2], yb[3]);
    }
  }
}

// ---------------------------------------------------------------------------
// launchers
// ---------------------------------------------------------------------------
static int warp_rows_grid(long long rows, int warps_per_block) {
  return (int)((rows + warps_per_block - 1) / warps_per_block);
}
static int stride_grid(long long n, int threads) {
  long long b = (n + threads - 1) / threads;
  long long cap = (long long)sm_count() * 16;
  return (int)(b < cap ? (b > 0 ? b : 1) : cap);
}

int32_t launch_rmsnorm(const uint16_t* x, long long ldx, const uint16_t* w0, const uint16_t* w1, long long split,
                       uint16_t* out, long long ldo, long long rows, int width, float eps, cudaStream_t s) {
  if (width % 256 != 0) return set_error(ENNX_B200_UNSUPPORTED, "rmsnorm width %d must be a multiple of 256", width);
  rmsnorm_kernel<<<warp_rows_grid(rows, 8), 256, 0, s>>>(x, ldx, w0, w1 ? w1 : w0, w1 ? split : rows, out, ldo,
                                                          rows, width, eps);
  ENNX_LAUNCH_CHECK("rmsnorm");
  return ENNX_B200_OK;
}

int32_t launch_embed(const int* tokens, const uint16_t* t0, const uint16_t* t1, long long per_set, long long rows,
                     int width, int vocab, uint16_t* out, cudaStream_t s, const uint16_t* noise) {
  if (width % 256 != 0) return set_error(ENNX_B200_UNSUPPORTED, "embedding width must be a multiple of 256");
  embed_kernel<<<warp_rows_grid(rows, 8), 256, 0, s>>>(tokens, t0, t1 ? t1 : t0, noise, per_set, rows, width, vocab,
                                                        out, device_error_word());
  ENNX_LAUNCH_CHECK("embed");
  return ENNX_B200_OK;
}

int32_t launch_l2norm_heads(uint16_t* base, long long ld, int heads, long long rows, cudaStream_t s) {
  long long groups = rows * heads;
  l2norm_heads_kernel<<<warp_rows_grid(groups, 8), 256, 0, s>>>(base, ld, heads, groups);
  ENNX_LAUNCH_CHECK("l2norm_heads");
  return ENNX_B200_OK;
}

int32_t launch_kda_gate(const uint16_t* raw, long long ldraw, const uint16_t* rbeta, long long ldb,
                        const uint16_t* decay0, const uint16_t* decay1, const uint16_t* tb0, const uint16_t* tb1,
                        long long split, long long rows, int heads, int head_width, float* gate, float* beta,
                        cudaStream_t s) {
  long long total = rows * heads * (long long)head_width;
  kda_gate_kernel<<<stride_grid(total, 256), 256, 0, s>>>(raw, ldraw, rbeta, ldb, decay0, decay1 ? decay1 : decay0,
                                                           tb0, tb1 ? tb1 : tb0, decay1 ? split : rows, rows, heads,
                                                           head_width, gate, beta);
  ENNX_LAUNCH_CHECK("kda_gate");
  return ENNX_B200_OK;
}

int32_t launch_kda_post(const uint16_t* o, const uint16_t* og, long long ldog, const uint16_t* n0, const uint16_t* n1,
                        long long split, int heads, long long rows, float eps, uint16_t* out, cudaStream_t s) {
  long long groups = rows * heads;
  if (((uintptr_t)o | (uintptr_t)og | (uintptr_t)out | (uintptr_t)n0 | (uintptr_t)(n1 ? n1 : n0)) & 15u || ldog % 8)
    return set_error(ENNX_B200_INVALID_ARGUMENT, "kda_post: operands must be 16-byte aligned");
  kda_post_kernel<<<(unsigned)((groups + 15) / 16), 256, 0, s>>>(o, og, ldog, n0, n1 ? n1 : n0, n1 ? split : rows,
                                                                  heads, groups, eps, out);
  ENNX_LAUNCH_CHECK("kda_post");
  return ENNX_B200_OK;
}

int32_t launch_rope(uint16_t* base, long long ld, int heads, int dim, long long rows, int seq, float theta,
                    cudaStream_t s) {
  if (dim % 16 || ld % 8 || ((uintptr_t)base & 15u))
    return set_error(ENNX_B200_UNSUPPORTED, "rope: head width must be a multiple of 16 with 16-byte aligned rows");
  long long total = rows * (long long)(dim / 16);
  rope_kernel<<<stride_grid(total, 256), 256, 0, s>>>(base, ld, heads, dim, rows, seq, log2f(theta));
  ENNX_LAUNCH_CHECK("rope");
  return ENNX_B200_OK;
}

}  // namespace ennx
