// decode.cu -- resident single-token KDA-MoE decoder over packed int4/int8
// weights (the NativeKdaModel of the reference, Metal-only there).
//
// Restates KdaMoeMetalModel::decode_token / generate / prepare_candidate
// (rust/crates/ennx/src/forward_metal.rs:1256-1394) and the per-layer order of
// KdaMoeMetalExecutor::encode_decode_layer (:614-810) with the math of the
// Metal kernels it encodes (kda_moe.metal): decoder_rms_norm (:536-554),
// decoder_project_packed_simd (:424-449), kda_short_conv_decode (:481-508),
// kda_split_qkv_16k (:137-153), kda_normalize_qk (:510-534),
// kda_split_control_16k (:847-867), kda_make_gate_beta_16k (:875-896, fused into the step),
// kda_decode_step (:283-338), kda_postprocess_16k (:898-921),
// decoder_residual (:556-565), moe_router_topk_simd (:625-689),
// moe_gate_up_simd / moe_down_simd (:759-834), packed_embedding_lookup
// (:929-946) and decoder_argmax (:948-975).
//
// B200 design: the weights stay packed in HBM (0.5 or 1 byte per weight) and
// every projection is a warp-per-row GEMV that dequantises and perturbs the
// integer codes on the fly -- at one token per step the decoder is bound by
// the bytes of the weights it reads, so reading codes rather than bf16 copies
// is the roofline.  Activations, the recurrent state and the convolution
// history are fp32 (the reference keeps activations in half).  Every kernel of
// a token reads the token id from device memory and the argmax writes the
// next one there, so the whole step is captured once per seed as a CUDA graph
// and generation replays it without host round trips.
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include "common.cuh"
#include "packed.cuh"

namespace ennx {
namespace {

constexpr int kMaxKeyWidth = 128;   // kda_decode_step: min(key_width, 128)
constexpr int kMaxTopK = 8;         // moe_router_topk_simd
constexpr int kMaxExperts = 1 << 16;  // router scores buffer

struct LayerDev {  // device copies of one layer's descriptors
  PackedDesc qkv, control, output, conv, forget_b, gate_b, router;
  const PackedDesc* gate;  // [experts]
  const PackedDesc* up;
  const PackedDesc* down;
  // per-layer state and prepared vectors
  float* conv_history;   // [3][qkv_width]
  float* state;          // [heads][key_width][value_width]
  float* attn_norm;      // [hidden]
  float* moe_norm;       // [hidden]
  float* decay;          // [heads]
  float* time_bias;      // [hidden]
  float* out_norm;       // [head_width]
};

struct Arena {
  const uint8_t* w;
  const float* sc;
  const float* bi;
};

// perturb_code (kda_moe.metal:73-90) on one code
__device__ __forceinline__ uint32_t perturb_one(uint32_t code, const PackedDesc& d, ennx_b200_perturb_seed s,
                                                uint32_t element, uint32_t max_code) {
  const uint32_t random = packed_hash(s.low, s.high, element);
  const uint32_t amount = d.whole + (uint32_t)((random >> 1) < (d.threshold >> 1));
  if (amount == 0u) return code;
  if ((random & 1u) == 0u) return code >= amount ? code - amount : min(code + amount, max_code);
  return code + amount <= max_code ? code + amount : code >= amount ? code - amount : 0u;
}

// Codes of one 64-column chunk as 32-bit words (int4: 8 words, int8: 16),
// all loads issued before any is used; byte assembly where the arena offset
// leaves the chunk unaligned.
template <int kWords>
__device__ __forceinline__ void load_chunk(const uint8_t* p, uint32_t (&cw)[kWords]) {
  if (((uintptr_t)p & 3u) == 0) {
#pragma unroll
    for (int w = 0; w < kWords; ++w) cw[w] = __ldg(reinterpret_cast<const uint32_t*>(p) + w);
  } else {
#pragma unroll
    for (int w = 0; w < kWords; ++w)
      cw[w] = (uint32_t)__ldg(p + 4 * w) | ((uint32_t)__ldg(p + 4 * w + 1) << 8) |
              ((uint32_t)__ldg(p + 4 * w + 2) << 16) | ((uint32_t)__ldg(p + 4 * w + 3) << 24);
  }
}

// One 64-column chunk of a row: 8 runs of 8 columns, one scale/bias per run.
template <bool kInt4>
__device__ __forceinline__ float chunk_dot(const uint8_t* wrow, const float* srow, const float* brow,
                                           const PackedDesc& d, ennx_b200_perturb_seed s, uint32_t elem_row,
                                           uint32_t base, const float* __restrict__ x, float acc) {
  constexpr int kWords = kInt4 ? 8 : 16;
  constexpr uint32_t kMax = kInt4 ? 15u : 255u;
  uint32_t cw[kWords];
  load_chunk<kWords>(wrow + (kInt4 ? base / 2 : base), cw);
#pragma unroll
  for (int r = 0; r < 8; ++r) {
    const uint32_t c0 = base + 8 * r;
    const uint32_t g = min(c0 / d.group_size, (uint32_t)d.groups - 1u);
    const float sc = __ldg(srow + g), bi = __ldg(brow + g);
    float xv[8];
    if (((uintptr_t)(x + c0) & 15u) == 0) {
      const float4 a = __ldg(reinterpret_cast<const float4*>(x + c0));
      const float4 b = __ldg(reinterpret_cast<const float4*>(x + c0 + 4));
      xv[0] = a.x; xv[1] = a.y; xv[2] = a.z; xv[3] = a.w; xv[4] = b.x; xv[5] = b.y; xv[6] = b.z; xv[7] = b.w;
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) xv[j] = __ldg(x + c0 + j);
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      uint32_t code = kInt4 ? (cw[r] >> (4 * j)) & 15u : (cw[2 * r + (j >> 2)] >> (8 * (j & 3))) & 255u;
      if (s.enabled) code = perturb_one(code, d, s, elem_row + c0 + j, kMax);
      acc = fmaf(xv[j], __fmaf_rn((float)code, sc, bi), acc);
    }
  }
  return acc;
}

// Packed dot product of one weight row with x (fp32); the warp sum is
// returned in every lane.  Each lane takes contiguous 64-column chunks
// (stride 2048 columns per warp) so that many independent code loads are in
// flight per lane; chunks that leave the row or straddle a scale group of a
// size that is not a multiple of 8 take the per-element path.
__device__ __forceinline__ float warp_row_dot(const Arena& A, const PackedDesc& d, ennx_b200_perturb_seed seed,
                                              uint64_t row, const float* __restrict__ x, int lane) {
  // the reference enables perturbation for every seed; a descriptor with
  // whole = 0 and threshold < 2 never moves a code, so skip the hash there
  ennx_b200_perturb_seed s = seed;
  if (d.whole == 0 && (d.threshold >> 1) == 0) s.enabled = 0;
  float acc = 0.0f;
  const uint32_t n = (uint32_t)d.input_width;
  const bool fast = (d.group_size & 7u) == 0;
  const uint8_t* wrow = A.w + d.byte_offset + row * d.row_bytes;
  const float* srow = A.sc + d.scale_offset + row * d.groups;
  const float* brow = A.bi + d.bias_offset + row * d.groups;
  const uint32_t elem_row = (uint32_t)d.element_offset + (uint32_t)row * n;  // 32-bit, as the reference
  for (uint32_t base = (uint32_t)lane * 64; base < n; base += 32 * 64) {
    if (fast && base + 64 <= n) {
      acc = d.bits == 4 ? chunk_dot<true>(wrow, srow, brow, d, s, elem_row, base, x, acc)
                        : chunk_dot<false>(wrow, srow, brow, d, s, elem_row, base, x, acc);
    } else {
      for (uint32_t c = base; c < n && c < base + 64; ++c)
        acc = fmaf(__ldg(x + c), packed_weight(A.w, A.sc, A.bi, d, s, row, c), acc);
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  return acc;
}

enum GemvMode : int { kPlain = 0, kResidual = 1, kGateUp = 2, kDown = 3 };

struct GemvArgs {
  Arena A;
  const float* x;
  float* y;
  PackedDesc d;                 // kPlain / kResidual
  const PackedDesc* gate;       // kGateUp
  const PackedDesc* up;
  const PackedDesc* down;       // kDown
  const uint32_t* route_idx;
  const float* route_w;
  uint32_t rows;
  uint32_t top_k;
  uint32_t expert_width;
  float residual_scale;
  ennx_b200_perturb_seed seed;
  int mode;
};

// decoder_project_packed_simd / moe_gate_up_simd / moe_down_simd: one warp
// per output dot, one instantiation per mode.  kResidual adds
// residual_scale * result to y (decoder_residual fused into the projection
// that produces the update); the expert modes give every (rank, row) dot its
// own warp and leave SwiGLU and the rank sum to two short kernels.
template <int kMode>
__global__ void __launch_bounds__(256) dec_gemv_kernel(const __grid_constant__ GemvArgs g) {
  const int lane = threadIdx.x & 31;
  const uint32_t row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= g.rows) return;  // whole warps leave together
  if constexpr (kMode == kPlain || kMode == kResidual) {
    const PackedDesc d = g.d;
    const float v = warp_row_dot(g.A, d, g.seed, row, g.x, lane);
    if (lane == 0) g.y[row] = kMode == kPlain ? v : g.y[row] + g.residual_scale * v;
  } else if constexpr (kMode == kGateUp) {
    // rows [0, k*I): gate dots, [k*I, 2*k*I): up dots, one warp each
    const uint32_t half = g.top_k * g.expert_width;
    const bool up = row >= half;
    const uint32_t rr = up ? row - half : row;
    const uint32_t rank = rr / g.expert_width, feature = rr % g.expert_width;
    const uint32_t e = g.route_idx[rank];
    const PackedDesc d = up ? g.up[e] : g.gate[e];
    const float v = warp_row_dot(g.A, d, g.seed, feature, g.x, lane);
    if (lane == 0) g.y[row] = v;
  } else {  // kDown: rows [r*H, (r+1)*H): w_r * down_e(act_r)[row], summed by dec_down_sum_kernel
    const uint32_t hidden = g.rows / g.top_k;
    const uint32_t r = row / hidden, f = row % hidden;
    const PackedDesc dd = g.down[g.route_idx[r]];
    const float v = warp_row_dot(g.A, dd, g.seed, f, g.x + (uint64_t)r * g.expert_width, lane);
    if (lane == 0) g.y[row] = g.route_w[r] * v;
  }
}

// SwiGLU of the selected experts: act = silu(gate) * up
__global__ void __launch_bounds__(256) dec_swiglu_kernel(const float* __restrict__ gu, float* __restrict__ act,
                                                         uint32_t n) {
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float gv = gu[i];
  act[i] = gv / (1.0f + expf(-gv)) * gu[n + i];
}

// hidden += residual_scale * sum over ranks (in rank order) of the weighted
// expert outputs (moe_down_simd's sum + decoder_residual)
__global__ void __launch_bounds__(256) dec_down_sum_kernel(const float* __restrict__ part,
                                                           float* __restrict__ hidden, uint32_t top_k,
                                                           uint32_t n, float rs) {
  const uint32_t f = blockIdx.x * blockDim.x + threadIdx.x;
  if (f >= n) return;
  float sum = 0.0f;
  for (uint32_t r = 0; r < top_k; ++r) sum += part[(uint64_t)r * n + f];
  hidden[f] = hidden[f] + rs * sum;
}

// decoder_rms_norm: y = x * rsqrt(mean(x^2) + eps) * w; one CTA.
__global__ void __launch_bounds__(1024) dec_rmsnorm_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                                           float* __restrict__ y, uint32_t n, float eps) {
  __shared__ float part[32];
  __shared__ float inv;
  float ss = 0.0f;
  for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) ss = fmaf(x[i], x[i], ss);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.0f;
    for (uint32_t i = 0; i < (blockDim.x + 31) / 32; ++i) t += part[i];
    inv = rsqrtf(t / (float)n + eps);
  }
  __syncthreads();
  for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) y[i] = x[i] * inv * w[i];
}

// packed_embedding_lookup: hidden = W_emb[token] * scale (token from device)
__global__ void __launch_bounds__(256) dec_embed_kernel(Arena A, PackedDesc d, ennx_b200_perturb_seed seed,
                                                        const uint32_t* __restrict__ token, float scale,
                                                        float* __restrict__ hidden) {
  const uint32_t t = *token;
  if (t >= d.output_width) return;
  ennx_b200_perturb_seed s = seed;
  if (d.whole == 0 && (d.threshold >> 1) == 0) s.enabled = 0;
  for (uint64_t c = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; c < d.input_width;
       c += (uint64_t)gridDim.x * blockDim.x)
    hidden[c] = packed_weight(A.w, A.sc, A.bi, d, s, t, c) * scale;
}

// kda_short_conv_decode: 4-tap causal depthwise convolution with a 3-step
// history per feature, then SiLU; the history advances in place.
__global__ void __launch_bounds__(256) dec_conv_kernel(Arena A, PackedDesc conv, ennx_b200_perturb_seed seed,
                                                       float* __restrict__ qkv, float* __restrict__ hist, uint32_t width) {
  const uint32_t f = blockIdx.x * blockDim.x + threadIdx.x;
  if (f >= width) return;
  ennx_b200_perturb_seed s = seed;
  if (conv.whole == 0 && (conv.threshold >> 1) == 0) s.enabled = 0;
  const float cur = qkv[f];
  float v = 0.0f;
  v = fmaf(hist[f], packed_weight(A.w, A.sc, A.bi, conv, s, f, 0), v);
  v = fmaf(hist[width + f], packed_weight(A.w, A.sc, A.bi, conv, s, f, 1), v);
  v = fmaf(hist[2 * width + f], packed_weight(A.w, A.sc, A.bi, conv, s, f, 2), v);
  v = fmaf(cur, packed_weight(A.w, A.sc, A.bi, conv, s, f, 3), v);
  hist[f] = hist[width + f];
  hist[width + f] = hist[2 * width + f];
  hist[2 * width + f] = cur;
  qkv[f] = v / (1.0f + expf(-v));
}

// kda_normalize_qk: per-head L2 normalisation of q and k; warp per (q|k, head)
__global__ void __launch_bounds__(256) dec_l2norm_kernel(float* __restrict__ qkv, uint32_t heads, uint32_t hw) {
  const int lane = threadIdx.x & 31;
  const uint32_t g = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (g >= 2 * heads) return;
  float* v = qkv + (uint64_t)(g / heads) * heads * hw + (uint64_t)(g % heads) * hw;
  float ss = 0.0f;
  for (uint32_t i = lane; i < hw; i += 32) ss = fmaf(v[i], v[i], ss);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  const float inv = 1.0f / fmaxf(sqrtf(ss), 1.0e-6f);
  for (uint32_t i = lane; i < hw; i += 32) v[i] *= inv;
}

__device__ __forceinline__ float softplus_stable(float x) { return fmaxf(x, 0.0f) + log1pf(expf(-fabsf(x))); }

// kda_decode_step: CTA per (head, block of 32 value columns); its 8 warps
// split the key rows (16 each at d_k = 128) and keep their part of each
// column in registers across the two passes (read-out k.S of the decayed
// state, then the delta-rule update and q.S), with fixed-order shared-memory
// sums across the warps.
constexpr int kStepWarps = 8;
constexpr int kStepRows = kMaxKeyWidth / kStepWarps;  // rows per warp at most

// The gates of the step are formed here (kda_make_gate_beta_16k,
// kda_moe.metal:869-896): g = max(-exp(decay_h) * softplus(raw + tb), -5) per
// key row, beta = sigmoid(control[2r + h]).
__global__ void __launch_bounds__(kStepWarps * 32) dec_kda_step_kernel(const float* __restrict__ qkv,
                                                                       const float* __restrict__ raw_gate,
                                                                       const float* __restrict__ control,
                                                                       const float* __restrict__ decay,
                                                                       const float* __restrict__ time_bias,
                                                                       float* __restrict__ state,
                                                                       float* __restrict__ out, uint32_t heads,
                                                                       uint32_t hw, uint32_t rank) {
  __shared__ float red[kStepWarps][32];
  __shared__ float upd_s[32];
  const uint32_t h = blockIdx.x, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t col = blockIdx.y * 32 + lane;
  const uint32_t width = heads * hw;
  const uint32_t kw = hw < (uint32_t)kMaxKeyWidth ? hw : (uint32_t)kMaxKeyWidth;
  const uint32_t per = (kw + kStepWarps - 1) / kStepWarps;
  const uint32_t r0 = warp * per;
  const bool live = col < hw;
  float* S = state + (uint64_t)h * hw * hw + col;
  const float* q = qkv + h * hw;
  const float* k = qkv + width + h * hw;
  const float* rg = raw_gate + h * hw;
  const float* tb = time_bias + h * hw;
  const float ed = expf(decay[h]);
  float sv[kStepRows];
  float part = 0.0f;
#pragma unroll
  for (int j = 0; j < kStepRows; ++j) {
    const uint32_t i = r0 + j;
    sv[j] = 0.0f;
    if ((uint32_t)j < per && i < kw && live) {
      const float gi = fmaxf(-ed * softplus_stable(rg[i] + tb[i]), -5.0f);
      sv[j] = S[(uint64_t)i * hw] * expf(gi);
      part = fmaf(k[i], sv[j], part);
    }
  }
  red[warp][lane] = part;
  __syncthreads();
  if (warp == 0) {
    float read = 0.0f;
#pragma unroll
    for (int w = 0; w < kStepWarps; ++w) read += red[w][lane];
    const float beta = 1.0f / (1.0f + expf(-control[2 * rank + h]));
    upd_s[lane] = live ? beta * (qkv[2 * width + h * hw + col] - read) : 0.0f;
  }
  __syncthreads();
  const float upd = upd_s[lane];
  part = 0.0f;
#pragma unroll
  for (int j = 0; j < kStepRows; ++j) {
    const uint32_t i = r0 + j;
    if ((uint32_t)j < per && i < kw && live) {
      sv[j] = fmaf(k[i], upd, sv[j]);
      part = fmaf(q[i], sv[j], part);
      S[(uint64_t)i * hw] = sv[j];
    }
  }
  __syncthreads();  // every warp has read red[] for the first sum
  red[warp][lane] = part;
  __syncthreads();
  if (warp == 0 && live) {
    float res = 0.0f;
#pragma unroll
    for (int w = 0; w < kStepWarps; ++w) res += red[w][lane];
    out[h * hw + col] = res * rsqrtf((float)kw);
  }
}

// kda_postprocess_16k: per-head RMS norm x output_norm x sigmoid(output gate)
__global__ void __launch_bounds__(256) dec_post_kernel(const float* __restrict__ o, const float* __restrict__ og,
                                                       const float* __restrict__ norm, float* __restrict__ out,
                                                       uint32_t hw, float eps) {
  __shared__ float part[8];
  __shared__ float inv;
  const uint32_t h = blockIdx.x;
  const float* v = o + (uint64_t)h * hw;
  float ss = 0.0f;
  for (uint32_t i = threadIdx.x; i < hw; i += blockDim.x) ss = fmaf(v[i], v[i], ss);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.0f;
    for (uint32_t i = 0; i < blockDim.x / 32; ++i) t += part[i];
    inv = rsqrtf(t / (float)hw + eps);
  }
  __syncthreads();
  for (uint32_t i = threadIdx.x; i < hw; i += blockDim.x) {
    const float x = v[i] * inv * norm[i];
    const float gv = og[(uint64_t)h * hw + i];
    out[(uint64_t)h * hw + i] = x / (1.0f + expf(-gv));
  }
}

// moe_router_topk_simd, second half: the expert scores come from the packed
// GEMV (warp per expert, all SMs); one warp then takes k rounds of "highest
// score, lowest expert index" -- the selection of the reference's insertion
// with strict '>' -- and writes the softmax over the chosen scores.
__global__ void __launch_bounds__(32) dec_topk_kernel(const float* __restrict__ scores, uint32_t experts,
                                                      uint32_t top_k, uint32_t* __restrict__ idx,
                                                      float* __restrict__ wts) {
  __shared__ float val[kMaxTopK];
  __shared__ uint32_t ind[kMaxTopK];
  const uint32_t lane = threadIdx.x;
  for (uint32_t r = 0; r < top_k; ++r) {
    float best = -INFINITY;
    uint32_t bi = 0xffffffffu;
    for (uint32_t e = lane; e < experts; e += 32) {
      bool taken = false;
      for (uint32_t q = 0; q < r; ++q) taken |= ind[q] == e;
      const float v = scores[e];
      if (!taken && (v > best || (v == best && e < bi) || bi == 0xffffffffu)) { best = v; bi = e; }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, off);
      const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, off);
      if (oi != 0xffffffffu && (bi == 0xffffffffu || ob > best || (ob == best && oi < bi))) { best = ob; bi = oi; }
    }
    if (lane == 0) { val[r] = best; ind[r] = bi; }
    __syncwarp();
  }
  if (lane == 0) {
    const float mx = val[0];
    float ex[kMaxTopK], den = 0.0f;
#pragma unroll
    for (int r = 0; r < kMaxTopK; ++r)
      if ((uint32_t)r < top_k) { ex[r] = expf(val[r] - mx); den += ex[r]; }
#pragma unroll
    for (int r = 0; r < kMaxTopK; ++r)
      if ((uint32_t)r < top_k) { idx[r] = ind[r]; wts[r] = ex[r] / den; }
  }
}

// decoder_argmax: 256 lanes scan strided logits (strict '>'), then a tree
// keeps the left value unless the right one is strictly larger.  The token
// is written for the next step and appended to the generation output.
__global__ void __launch_bounds__(256) dec_argmax_kernel(const float* __restrict__ logits, uint32_t vocab,
                                                         uint32_t* __restrict__ token, uint32_t* __restrict__ next,
                                                         uint32_t* __restrict__ out, uint32_t* __restrict__ out_count,
                                                         uint32_t out_cap) {
  __shared__ float val[256];
  __shared__ uint32_t ind[256];
  const uint32_t lane = threadIdx.x;
  float best = -INFINITY;
  uint32_t bi = 0;
  for (uint32_t i = lane; i < vocab; i += 256)
    if (logits[i] > best) { best = logits[i]; bi = i; }
  val[lane] = best;
  ind[lane] = bi;
  __syncthreads();
  for (uint32_t stride = 128; stride > 0; stride >>= 1) {
    if (lane < stride && val[lane + stride] > val[lane]) { val[lane] = val[lane + stride]; ind[lane] = ind[lane + stride]; }
    __syncthreads();
  }
  if (lane == 0) {
    const uint32_t t = ind[0];
    *next = t;
    *token = t;
    const uint32_t k = *out_count;
    if (k < out_cap) out[k] = t;
    *out_count = k + 1;
  }
}

// The perturbed codes of one candidate (seed), written once into a shadow
// arena: integer-code perturbation depends on (seed, element) only, not on
// the token, so every token of that candidate then reads ready codes and no
// GEMV hashes.  One thread per byte (one int8 code or two int4 codes); the
// job of a byte is found by binary search over the cumulative byte starts.
struct ArenaJob {
  PackedDesc d;
  uint64_t first;  // first byte of this linear in the concatenated job range
};

__global__ void __launch_bounds__(256) dec_perturb_arena_kernel(const uint8_t* __restrict__ src,
                                                                uint8_t* __restrict__ dst,
                                                                const ArenaJob* __restrict__ jobs, uint32_t njobs,
                                                                uint64_t total, ennx_b200_perturb_seed seed) {
  constexpr uint64_t kChunkBytes = 64;  // one job search per chunk
  for (uint64_t c0 = ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) * kChunkBytes; c0 < total;
       c0 += (uint64_t)gridDim.x * blockDim.x * kChunkBytes) {
    uint32_t lo = 0, hi = njobs - 1;
    while (lo < hi) {
      const uint32_t mid = (lo + hi + 1) >> 1;
      if (jobs[mid].first <= c0) lo = mid; else hi = mid - 1;
    }
    uint32_t j = lo;
    uint64_t next = j + 1 < njobs ? jobs[j + 1].first : total;
    for (uint64_t i = c0; i < c0 + kChunkBytes && i < total; ++i) {
      while (i >= next) {
        ++j;
        next = j + 1 < njobs ? jobs[j + 1].first : total;
      }
      const PackedDesc& d = jobs[j].d;
      const uint64_t b = i - jobs[j].first;
      uint32_t v = src[d.byte_offset + b];
      if (d.whole != 0 || (d.threshold >> 1) != 0) {
        const uint64_t row = b / d.row_bytes, cb = b % d.row_bytes;
        const uint32_t er = (uint32_t)d.element_offset + (uint32_t)row * (uint32_t)d.input_width;  // 32-bit
        if (d.bits == 8) {
          v = perturb_one(v, d, seed, er + (uint32_t)cb, 255u);
        } else {
          const uint32_t c = 2u * (uint32_t)cb;
          const uint32_t a = perturb_one(v & 15u, d, seed, er + c, 15u);
          const uint32_t z = c + 1 < d.input_width ? perturb_one(v >> 4, d, seed, er + c + 1, 15u) : (v >> 4);
          v = a | (z << 4);
        }
      }
      dst[d.byte_offset + b] = (uint8_t)v;
    }
  }
}

}  // namespace
}  // namespace ennx

using namespace ennx;

struct ennx_b200_kda_decoder {
  int device;
  cudaStream_t stream;
  ennx_b200_kda_decoder_config cfg;
  uint8_t* packed;
  float* scales;
  float* biases;
  size_t packed_bytes, n_scales, n_biases;
  // host descriptors
  ennx_b200_kda_decoder_layer* host_layers;    // copies (expert pointers below)
  ennx_b200_packed_linear* host_experts;       // [layers][3][experts]
  ennx_b200_packed_linear embedding, final_norm;
  LayerDev* layers;                            // host array of device pointers
  PackedDesc* expert_descs;                    // device [layers][3][experts]
  float* final_norm_v;
  // activations
  float *hidden, *normed, *qkv, *control, *raw_gate, *ogate, *post, *gated, *act, *logits, *route_w;
  float* scores;  // router scores [experts]
  float* gu;      // expert gate | up dots [2][top_k][expert_width]
  float* part;    // weighted expert outputs [top_k][hidden]
  uint32_t *route_idx, *token, *next, *out_tokens, *out_count;
  size_t out_cap;
  // graph of one token step
  cudaGraphExec_t graph;
  int have_graph;
  int has_logits;
  int own_stream;
  // per-candidate perturbed codes
  uint8_t* shadow;
  ArenaJob* jobs;
  uint32_t njobs;
  uint64_t job_bytes;
  uint64_t shadow_seed;
  int have_shadow;
};

namespace {

void* dalloc(size_t bytes, int32_t* st) {
  void* p = nullptr;
  if (*st) return nullptr;
  if (cudaMalloc(&p, bytes < 16 ? 16 : bytes) != cudaSuccess) {
    *st = set_error(ENNX_B200_CUDA_ERROR, "decoder device allocation of %zu bytes failed", bytes);
    return nullptr;
  }
  return p;
}

void destroy_decoder(ennx_b200_kda_decoder* h) {
  if (!h) return;
  if (h->have_graph) cudaGraphExecDestroy(h->graph);
  void* ptrs[] = {h->packed,   h->scales,  h->biases,   h->expert_descs, h->final_norm_v, h->hidden,
                  h->normed,   h->qkv,     h->control,  h->raw_gate,     h->ogate,
                  h->post,     h->gated,   h->act,      h->logits,       h->route_w,
                  h->route_idx, h->token,  h->next,     h->out_tokens,   h->out_count, h->scores,
                  h->shadow,   h->jobs,    h->gu,       h->part};
  for (void* p : ptrs)
    if (p) cudaFree(p);
  if (h->layers) {
    for (uint32_t l = 0; l < h->cfg.num_layers; ++l) {
      LayerDev& L = h->layers[l];
      void* lp[] = {L.conv_history, L.state, L.attn_norm, L.moe_norm, L.decay, L.time_bias, L.out_norm};
      for (void* p : lp)
        if (p) cudaFree(p);
    }
    free(h->layers);
  }
  free(h->host_layers);
  free(h->host_experts);
  if (h->own_stream) cudaStreamDestroy(h->stream);
  free(h);
}

// Bounds of a linear against the arenas: every device read stays inside.
int32_t check_linear(const ennx_b200_kda_decoder* h, const ennx_b200_packed_linear* l, const char* name,
                     uint64_t in, uint64_t out) {
  PackedDesc d;
  ENNX_TRY(make_desc(l, &d));
  if ((in && l->input_width != in) || (out && l->output_width != out))
    return set_error(ENNX_B200_INVALID_ARGUMENT, "linear %s must be %llu x %llu, got %llu x %llu", name,
                     (unsigned long long)out, (unsigned long long)in, (unsigned long long)l->output_width,
                     (unsigned long long)l->input_width);
  if (d.byte_offset + d.row_bytes * d.output_width > h->packed_bytes)
    return set_error(ENNX_B200_INVALID_ARGUMENT, "linear %s exceeds weights arena", name);
  if (d.scale_offset + d.groups * d.output_width > h->n_scales || d.bias_offset + d.groups * d.output_width > h->n_biases)
    return set_error(ENNX_B200_INVALID_ARGUMENT, "linear %s exceeds scale or bias arena", name);
  return ENNX_B200_OK;
}

ennx_b200_perturb_seed seed_of(uint64_t s) {
  ennx_b200_perturb_seed p;
  p.low = (uint32_t)s;
  p.high = (uint32_t)(s >> 32);
  p.enabled = 1;  // MetalSeed::from (forward_metal.rs:1494-1503)
  return p;
}

int32_t gemv(ennx_b200_kda_decoder* h, const GemvArgs& g) {
  const unsigned blocks = (g.rows + 7) / 8;
  switch (g.mode) {
    case kPlain: dec_gemv_kernel<kPlain><<<blocks, 256, 0, h->stream>>>(g); break;
    case kResidual: dec_gemv_kernel<kResidual><<<blocks, 256, 0, h->stream>>>(g); break;
    case kGateUp: dec_gemv_kernel<kGateUp><<<blocks, 256, 0, h->stream>>>(g); break;
    default: dec_gemv_kernel<kDown><<<blocks, 256, 0, h->stream>>>(g); break;
  }
  ENNX_LAUNCH_CHECK("decoder gemv");
  return ENNX_B200_OK;
}

GemvArgs plain(ennx_b200_kda_decoder* h, const PackedDesc& d, const float* x, float* y, ennx_b200_perturb_seed s,
               int mode) {
  GemvArgs g;
  memset(&g, 0, sizeof(g));
  g.A = Arena{h->shadow, h->scales, h->biases};
  g.x = x;
  g.y = y;
  g.d = d;
  g.rows = (uint32_t)d.output_width;
  g.residual_scale = h->cfg.residual_scale;
  g.seed = s;
  g.mode = mode;
  return g;
}

// One token through every layer and the head (encode_decode_layer x L +
// decode_token's head), enqueued on the decoder's stream.
int32_t enqueue_step(ennx_b200_kda_decoder* h, uint64_t seed64) {
  const ennx_b200_kda_decoder_config& c = h->cfg;
  cudaStream_t s = h->stream;
  // the codes in the shadow arena are already perturbed for this seed
  ennx_b200_perturb_seed seed = seed_of(seed64);
  seed.enabled = 0;
  const Arena A{h->shadow, h->scales, h->biases};
  const uint32_t W = c.heads * c.head_width;
  PackedDesc emb, fin;
  ENNX_TRY(make_desc(&h->embedding, &emb));
  ENNX_TRY(make_desc(&h->final_norm, &fin));
  dec_embed_kernel<<<(c.hidden + 255) / 256, 256, 0, s>>>(A, emb, seed, h->token, c.embedding_scale, h->hidden);
  ENNX_LAUNCH_CHECK("decoder embed");
  for (uint32_t l = 0; l < c.num_layers; ++l) {
    const LayerDev& L = h->layers[l];
    dec_rmsnorm_kernel<<<1, 1024, 0, s>>>(h->hidden, L.attn_norm, h->normed, c.hidden, c.rms_epsilon);
    ENNX_LAUNCH_CHECK("decoder rmsnorm");
    ENNX_TRY(gemv(h, plain(h, L.qkv, h->normed, h->qkv, seed, kPlain)));
    dec_conv_kernel<<<(3 * W + 255) / 256, 256, 0, s>>>(A, L.conv, seed, h->qkv, L.conv_history, 3 * W);
    ENNX_LAUNCH_CHECK("decoder conv");
    dec_l2norm_kernel<<<(2 * c.heads + 7) / 8, 256, 0, s>>>(h->qkv, c.heads, c.head_width);
    ENNX_LAUNCH_CHECK("decoder l2norm");
    ENNX_TRY(gemv(h, plain(h, L.control, h->normed, h->control, seed, kPlain)));
    ENNX_TRY(gemv(h, plain(h, L.forget_b, h->control, h->raw_gate, seed, kPlain)));
    ENNX_TRY(gemv(h, plain(h, L.gate_b, h->control + c.gate_rank, h->ogate, seed, kPlain)));
    dec_kda_step_kernel<<<dim3(c.heads, (c.head_width + 31) / 32), kStepWarps * 32, 0, s>>>(
        h->qkv, h->raw_gate, h->control, L.decay, L.time_bias, L.state, h->post, c.heads, c.head_width,
        c.gate_rank);
    ENNX_LAUNCH_CHECK("decoder kda step");
    dec_post_kernel<<<c.heads, 256, 0, s>>>(h->post, h->ogate, L.out_norm, h->gated, c.head_width, c.rms_epsilon);
    ENNX_LAUNCH_CHECK("decoder post");
    ENNX_TRY(gemv(h, plain(h, L.output, h->gated, h->hidden, seed, kResidual)));
    dec_rmsnorm_kernel<<<1, 1024, 0, s>>>(h->hidden, L.moe_norm, h->normed, c.hidden, c.rms_epsilon);
    ENNX_LAUNCH_CHECK("decoder rmsnorm");
    ENNX_TRY(gemv(h, plain(h, L.router, h->normed, h->scores, seed, kPlain)));
    dec_topk_kernel<<<1, 32, 0, s>>>(h->scores, c.num_experts, c.top_k, h->route_idx, h->route_w);
    ENNX_LAUNCH_CHECK("decoder router");
    GemvArgs gu = plain(h, L.router, h->normed, h->gu, seed, kGateUp);
    gu.gate = L.gate;
    gu.up = L.up;
    gu.route_idx = h->route_idx;
    gu.rows = 2 * c.top_k * c.expert_width;
    gu.top_k = c.top_k;
    gu.expert_width = c.expert_width;
    ENNX_TRY(gemv(h, gu));
    const uint32_t nact = c.top_k * c.expert_width;
    dec_swiglu_kernel<<<(nact + 255) / 256, 256, 0, s>>>(h->gu, h->act, nact);
    ENNX_LAUNCH_CHECK("decoder swiglu");
    GemvArgs dn = plain(h, L.router, h->act, h->part, seed, kDown);
    dn.down = L.down;
    dn.route_idx = h->route_idx;
    dn.route_w = h->route_w;
    dn.rows = c.top_k * c.hidden;
    dn.top_k = c.top_k;
    dn.expert_width = c.expert_width;
    ENNX_TRY(gemv(h, dn));
    dec_down_sum_kernel<<<(c.hidden + 255) / 256, 256, 0, s>>>(h->part, h->hidden, c.top_k, c.hidden,
                                                               c.residual_scale);
    ENNX_LAUNCH_CHECK("decoder expert sum");
  }
  dec_rmsnorm_kernel<<<1, 1024, 0, s>>>(h->hidden, h->final_norm_v, h->normed, c.hidden, c.rms_epsilon);
  ENNX_LAUNCH_CHECK("decoder final norm");
  ENNX_TRY(gemv(h, plain(h, emb, h->normed, h->logits, seed, kPlain)));
  dec_argmax_kernel<<<1, 256, 0, s>>>(h->logits, (uint32_t)emb.output_width, h->token, h->next, h->out_tokens,
                                      h->out_count, (uint32_t)h->out_cap);
  ENNX_LAUNCH_CHECK("decoder argmax");
  return ENNX_B200_OK;
}

// The step for `seed`, captured once and replayed (the seed is a kernel
// argument, so a new seed recaptures).
int32_t build_shadow(ennx_b200_kda_decoder* h, uint64_t seed) {
  if (h->have_shadow && h->shadow_seed == seed) return ENNX_B200_OK;
  uint64_t blocks = (h->job_bytes / 64 + 255) / 256 + 1;
  const uint64_t cap = (uint64_t)sm_count() * 16;
  if (blocks > cap) blocks = cap;
  dec_perturb_arena_kernel<<<(unsigned)blocks, 256, 0, h->stream>>>(h->packed, h->shadow, h->jobs, h->njobs,
                                                                    h->job_bytes, seed_of(seed));
  ENNX_LAUNCH_CHECK("decoder perturbed arena");
  h->have_shadow = 1;
  h->shadow_seed = seed;
  return ENNX_B200_OK;
}

int32_t run_step(ennx_b200_kda_decoder* h, uint64_t seed) {
  ENNX_TRY(build_shadow(h, seed));
  if (!h->have_graph) {
    if (h->have_graph) {
      cudaGraphExecDestroy(h->graph);
      h->have_graph = 0;
    }
    cudaGraph_t g;
    ENNX_CUDA(cudaStreamBeginCapture(h->stream, cudaStreamCaptureModeThreadLocal), "decoder capture");
    int32_t st = enqueue_step(h, seed);
    cudaError_t e = cudaStreamEndCapture(h->stream, &g);
    if (st != ENNX_B200_OK) {
      if (e == cudaSuccess) cudaGraphDestroy(g);
      return st;
    }
    ENNX_CUDA(e, "decoder capture");
    e = cudaGraphInstantiate(&h->graph, g, 0);
    cudaGraphDestroy(g);
    ENNX_CUDA(e, "decoder graph instantiate");
    h->have_graph = 1;
  }
  ENNX_CUDA(cudaGraphLaunch(h->graph, h->stream), "decoder graph launch");
  note_launch(0);
  h->has_logits = 1;
  return ENNX_B200_OK;
}

int32_t check_current(ennx_b200_kda_decoder* h) {
  if (!h) return set_error(ENNX_B200_INVALID_ARGUMENT, "decoder handle is null");
  int d = -1;
  ENNX_CUDA(cudaGetDevice(&d), "cudaGetDevice");
  if (d != h->device)
    return set_error(ENNX_B200_INVALID_ARGUMENT, "decoder belongs to device %d, current device is %d", h->device, d);
  return ENNX_B200_OK;
}

}  // namespace

extern "C" {

int32_t ennx_b200_kda_decoder_create(const uint8_t* packed, size_t packed_bytes, const float* scales,
                                     size_t num_scales, const float* biases, size_t num_biases,
                                     const ennx_b200_kda_decoder_config* config,
                                     const ennx_b200_kda_decoder_layer* layers,
                                     const ennx_b200_packed_linear* embedding,
                                     const ennx_b200_packed_linear* final_norm, void* stream,
                                     ennx_b200_kda_decoder** out) {
  if (!out) return set_error(ENNX_B200_INVALID_ARGUMENT, "decoder output handle is null");
  *out = nullptr;
  if (!packed || !scales || !biases || !config || !embedding || !final_norm)
    return set_error(ENNX_B200_INVALID_ARGUMENT, "decoder inputs are null");
  const ennx_b200_kda_decoder_config c = *config;
  if (c.num_layers == 0 || !layers) return set_error(ENNX_B200_INVALID_ARGUMENT, "resident KDA-MoE model has no layers");
  if (c.hidden == 0 || c.heads == 0 || c.head_width == 0 || c.gate_rank == 0 || c.num_experts == 0 ||
      c.expert_width == 0)
    return set_error(ENNX_B200_INVALID_ARGUMENT, "decoder dimensions must be positive");
  if (c.heads * c.head_width != c.hidden)
    return set_error(ENNX_B200_INVALID_ARGUMENT, "decoder hidden width must equal heads x head width");
  if (c.head_width > (uint32_t)kMaxKeyWidth)
    return set_error(ENNX_B200_UNSUPPORTED, "decoder head width above %d is not supported", kMaxKeyWidth);
  if (c.top_k == 0 || c.top_k > (uint32_t)kMaxTopK || c.top_k > c.num_experts)
    return set_error(ENNX_B200_INVALID_ARGUMENT, "decoder top_k must be in 1..=%d and at most the expert count",
                     kMaxTopK);
  if (c.num_experts > (uint32_t)kMaxExperts)
    return set_error(ENNX_B200_UNSUPPORTED, "decoder supports at most %d experts", kMaxExperts);
  if (!isfinite(c.embedding_scale)) return set_error(ENNX_B200_INVALID_ARGUMENT, "embedding scale must be finite");
  if (!isfinite(c.residual_scale) || !isfinite(c.rms_epsilon) || c.rms_epsilon < 0.0f)
    return set_error(ENNX_B200_INVALID_ARGUMENT, "decoder residual scale and epsilon must be finite");
  ennx_b200_kda_decoder* h = (ennx_b200_kda_decoder*)calloc(1, sizeof(ennx_b200_kda_decoder));
  if (!h) return set_error(ENNX_B200_CUDA_ERROR, "out of host memory");
  int32_t st = ENNX_B200_OK;
  const uint32_t L = c.num_layers, E = c.num_experts, W = c.heads * c.head_width;
  do {
    if (cudaGetDevice(&h->device) != cudaSuccess) { st = set_error(ENNX_B200_CUDA_ERROR, "cudaGetDevice failed"); break; }
    // An own stream: the token step is captured as a CUDA graph, which the
    // legacy default stream does not allow.  Every public call synchronises
    // it before returning, so no ordering with `stream` is needed.
    if (cudaStreamCreateWithFlags(&h->stream, cudaStreamNonBlocking) != cudaSuccess) {
      st = set_error(ENNX_B200_CUDA_ERROR, "decoder stream creation failed");
      break;
    }
    h->own_stream = 1;
    (void)stream;
    h->cfg = c;
    h->packed_bytes = packed_bytes;
    h->n_scales = num_scales;
    h->n_biases = num_biases;
    h->embedding = *embedding;
    h->final_norm = *final_norm;
    // attach_causal_head checks (forward_metal.rs:1182-1201)
    if ((st = check_linear(h, embedding, "embedding", c.hidden, 0))) {
      if (embedding->input_width != c.hidden) st = set_error(ENNX_B200_INVALID_ARGUMENT, "embedding hidden width does not match decoder");
      break;
    }
    if (final_norm->input_width != c.hidden || final_norm->output_width != 1) {
      st = set_error(ENNX_B200_INVALID_ARGUMENT, "final norm must be a hidden-width vector");
      break;
    }
    if ((st = check_linear(h, final_norm, "final_norm", c.hidden, 1))) break;
    h->host_layers = (ennx_b200_kda_decoder_layer*)calloc(L, sizeof(ennx_b200_kda_decoder_layer));
    h->host_experts = (ennx_b200_packed_linear*)calloc((size_t)L * 3 * E, sizeof(ennx_b200_packed_linear));
    h->layers = (LayerDev*)calloc(L, sizeof(LayerDev));
    if (!h->host_layers || !h->host_experts || !h->layers) { st = set_error(ENNX_B200_CUDA_ERROR, "out of host memory"); break; }
    PackedDesc* hd = (PackedDesc*)calloc((size_t)L * 3 * E, sizeof(PackedDesc));
    if (!hd) { st = set_error(ENNX_B200_CUDA_ERROR, "out of host memory"); break; }
    for (uint32_t l = 0; l < L && !st; ++l) {
      const ennx_b200_kda_decoder_layer& y = layers[l];
      h->host_layers[l] = y;
      if (!y.expert_gate || !y.expert_up || !y.expert_down) { st = set_error(ENNX_B200_INVALID_ARGUMENT, "layer %u has no expert descriptors", l); break; }
      LayerDev& D = h->layers[l];
      if ((st = check_linear(h, &y.qkv, "qkv", c.hidden, 3ull * W)) || (st = make_desc(&y.qkv, &D.qkv))) break;
      if ((st = check_linear(h, &y.control, "control", c.hidden, 2ull * c.gate_rank + c.heads)) ||
          (st = make_desc(&y.control, &D.control))) break;
      if ((st = check_linear(h, &y.output, "output", W, c.hidden)) || (st = make_desc(&y.output, &D.output))) break;
      if ((st = check_linear(h, &y.qkv_conv, "qkv_conv", 4, 3ull * W)) || (st = make_desc(&y.qkv_conv, &D.conv))) break;
      if ((st = check_linear(h, &y.forget_b, "forget_b", c.gate_rank, W)) || (st = make_desc(&y.forget_b, &D.forget_b))) break;
      if ((st = check_linear(h, &y.gate_b, "gate_b", c.gate_rank, W)) || (st = make_desc(&y.gate_b, &D.gate_b))) break;
      if ((st = check_linear(h, &y.router, "router", c.hidden, E)) || (st = make_desc(&y.router, &D.router))) break;
      if ((st = check_linear(h, &y.decay, "decay", c.heads, 1))) break;
      if ((st = check_linear(h, &y.time_bias, "time_bias", W, 1))) break;
      if ((st = check_linear(h, &y.output_norm, "output_norm", c.head_width, 1))) break;
      if ((st = check_linear(h, &y.attention_norm, "attention_norm", c.hidden, 1))) break;
      if ((st = check_linear(h, &y.moe_norm, "moe_norm", c.hidden, 1))) break;
      for (uint32_t e = 0; e < E && !st; ++e) {
        ennx_b200_packed_linear* he = h->host_experts + ((size_t)l * 3) * E;
        he[e] = y.expert_gate[e];
        he[E + e] = y.expert_up[e];
        he[2 * E + e] = y.expert_down[e];
        if ((st = check_linear(h, &he[e], "expert gate", c.hidden, c.expert_width))) break;
        if ((st = check_linear(h, &he[E + e], "expert up", c.hidden, c.expert_width))) break;
        if ((st = check_linear(h, &he[2 * E + e], "expert down", c.expert_width, c.hidden))) break;
        PackedDesc* dd = hd + ((size_t)l * 3) * E;
        make_desc(&he[e], &dd[e]);
        make_desc(&he[E + e], &dd[E + e]);
        make_desc(&he[2 * E + e], &dd[2 * E + e]);
      }
    }
    if (st) { free(hd); break; }
    h->expert_descs = (PackedDesc*)dalloc((size_t)L * 3 * E * sizeof(PackedDesc), &st);
    h->packed = (uint8_t*)dalloc(packed_bytes, &st);
    h->scales = (float*)dalloc(num_scales * sizeof(float), &st);
    h->biases = (float*)dalloc(num_biases * sizeof(float), &st);
    if (!st) {
      cudaError_t e = cudaMemcpyAsync(h->expert_descs, hd, (size_t)L * 3 * E * sizeof(PackedDesc), cudaMemcpyHostToDevice, h->stream);
      if (e == cudaSuccess) e = cudaMemcpyAsync(h->packed, packed, packed_bytes, cudaMemcpyHostToDevice, h->stream);
      if (e == cudaSuccess) e = cudaMemcpyAsync(h->scales, scales, num_scales * sizeof(float), cudaMemcpyHostToDevice, h->stream);
      if (e == cudaSuccess) e = cudaMemcpyAsync(h->biases, biases, num_biases * sizeof(float), cudaMemcpyHostToDevice, h->stream);
      if (e == cudaSuccess) e = cudaStreamSynchronize(h->stream);
      if (e != cudaSuccess) st = check_cuda(e, "decoder upload");
    }
    free(hd);
    if (st) break;
    for (uint32_t l = 0; l < L && !st; ++l) {
      LayerDev& D = h->layers[l];
      D.gate = h->expert_descs + ((size_t)l * 3) * E;
      D.up = D.gate + E;
      D.down = D.gate + 2 * E;
      D.conv_history = (float*)dalloc(3ull * 3 * W * sizeof(float), &st);
      D.state = (float*)dalloc((size_t)c.heads * c.head_width * c.head_width * sizeof(float), &st);
      D.attn_norm = (float*)dalloc(c.hidden * sizeof(float), &st);
      D.moe_norm = (float*)dalloc(c.hidden * sizeof(float), &st);
      D.decay = (float*)dalloc(c.heads * sizeof(float), &st);
      D.time_bias = (float*)dalloc(W * sizeof(float), &st);
      D.out_norm = (float*)dalloc(c.head_width * sizeof(float), &st);
    }
    // jobs of the per-candidate perturbation pass: every linear of the model
    {
      const size_t nj = (size_t)L * (12 + 3 * (size_t)E) + 2;
      ArenaJob* jobs = (ArenaJob*)calloc(nj, sizeof(ArenaJob));
      if (!jobs) { st = set_error(ENNX_B200_CUDA_ERROR, "out of host memory"); break; }
      size_t n = 0;
      uint64_t first = 0;
      auto add = [&](const ennx_b200_packed_linear* l) {
        PackedDesc d;
        make_desc(l, &d);
        jobs[n].d = d;
        jobs[n].first = first;
        first += d.row_bytes * d.output_width;
        ++n;
      };
      add(embedding);
      add(final_norm);
      for (uint32_t l = 0; l < L; ++l) {
        const ennx_b200_kda_decoder_layer& y = h->host_layers[l];
        const ennx_b200_packed_linear* v[] = {&y.qkv,   &y.control,   &y.output,      &y.qkv_conv,
                                              &y.forget_b, &y.gate_b, &y.decay,       &y.time_bias,
                                              &y.output_norm, &y.attention_norm, &y.moe_norm, &y.router};
        for (const ennx_b200_packed_linear* x : v) add(x);
        const ennx_b200_packed_linear* he = h->host_experts + ((size_t)l * 3) * E;
        for (uint32_t e = 0; e < 3 * E; ++e) add(&he[e]);
      }
      h->njobs = (uint32_t)n;
      h->job_bytes = first;
      h->jobs = (ArenaJob*)dalloc(n * sizeof(ArenaJob), &st);
      h->shadow = (uint8_t*)dalloc(packed_bytes, &st);
      if (!st) {
        cudaError_t e = cudaMemcpyAsync(h->jobs, jobs, n * sizeof(ArenaJob), cudaMemcpyHostToDevice, h->stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(h->stream);
        if (e != cudaSuccess) st = check_cuda(e, "decoder jobs");
      }
      free(jobs);
      if (st) break;
    }
    h->final_norm_v = (float*)dalloc(c.hidden * sizeof(float), &st);
    h->hidden = (float*)dalloc(c.hidden * sizeof(float), &st);
    h->normed = (float*)dalloc(c.hidden * sizeof(float), &st);
    h->qkv = (float*)dalloc(3ull * W * sizeof(float), &st);
    h->control = (float*)dalloc((2ull * c.gate_rank + c.heads) * sizeof(float), &st);
    h->raw_gate = (float*)dalloc(W * sizeof(float), &st);
    h->ogate = (float*)dalloc(W * sizeof(float), &st);
    h->post = (float*)dalloc(W * sizeof(float), &st);
    h->gated = (float*)dalloc(W * sizeof(float), &st);
    h->act = (float*)dalloc((size_t)c.top_k * c.expert_width * sizeof(float), &st);
    h->gu = (float*)dalloc(2ull * c.top_k * c.expert_width * sizeof(float), &st);
    h->part = (float*)dalloc((size_t)c.top_k * c.hidden * sizeof(float), &st);
    h->logits = (float*)dalloc(embedding->output_width * sizeof(float), &st);
    h->route_w = (float*)dalloc(kMaxTopK * sizeof(float), &st);
    h->scores = (float*)dalloc(c.num_experts * sizeof(float), &st);
    h->route_idx = (uint32_t*)dalloc(kMaxTopK * sizeof(uint32_t), &st);
    h->token = (uint32_t*)dalloc(sizeof(uint32_t), &st);
    h->next = (uint32_t*)dalloc(sizeof(uint32_t), &st);
    h->out_count = (uint32_t*)dalloc(sizeof(uint32_t), &st);
    h->out_cap = 1;
    h->out_tokens = (uint32_t*)dalloc(sizeof(uint32_t), &st);
    if (st) break;
    if (cudaMemsetAsync(h->out_count, 0, sizeof(uint32_t), h->stream) != cudaSuccess ||
        cudaMemsetAsync(h->token, 0, sizeof(uint32_t), h->stream) != cudaSuccess) {
      st = set_error(ENNX_B200_CUDA_ERROR, "decoder init failed");
      break;
    }
  } while (0);
  if (st) {
    if (h->own_stream) cudaStreamSynchronize(h->stream);
    destroy_decoder(h);
    return st;
  }
  *out = h;
  // the reference's constructor resets nothing and prepares candidate 0
  if ((st = ennx_b200_kda_decoder_reset(h)) || (st = ennx_b200_kda_decoder_prepare(h, 0))) {
    destroy_decoder(h);
    *out = nullptr;
    return st;
  }
  return ENNX_B200_OK;
}

int32_t ennx_b200_kda_decoder_destroy(ennx_b200_kda_decoder* h) {
  if (!h) return ENNX_B200_OK;
  int prev = -1;
  cudaGetDevice(&prev);
  cudaSetDevice(h->device);
  cudaStreamSynchronize(h->stream);
  destroy_decoder(h);
  if (prev >= 0) cudaSetDevice(prev);
  return ENNX_B200_OK;
}

int32_t ennx_b200_kda_decoder_reset(ennx_b200_kda_decoder* h) {
  ENNX_TRY(check_current(h));
  const ennx_b200_kda_decoder_config& c = h->cfg;
  const size_t W = (size_t)c.heads * c.head_width;
  for (uint32_t l = 0; l < c.num_layers; ++l) {
    ENNX_CUDA(cudaMemsetAsync(h->layers[l].state, 0, W * c.head_width * sizeof(float), h->stream), "reset");
    ENNX_CUDA(cudaMemsetAsync(h->layers[l].conv_history, 0, 9 * W * sizeof(float), h->stream), "reset");
  }
  ENNX_CUDA(cudaStreamSynchronize(h->stream), "reset");
  return ENNX_B200_OK;
}

int32_t ennx_b200_kda_decoder_prepare(ennx_b200_kda_decoder* h, uint64_t seed) {
  ENNX_TRY(check_current(h));
  const ennx_b200_perturb_seed s = seed_of(seed);
  for (uint32_t l = 0; l < h->cfg.num_layers; ++l) {
    const ennx_b200_kda_decoder_layer& y = h->host_layers[l];
    LayerDev& D = h->layers[l];
    ENNX_TRY(ennx_b200_packed_dequantize_f32(h->packed, h->scales, h->biases, &y.attention_norm, s, D.attn_norm, h->stream));
    ENNX_TRY(ennx_b200_packed_dequantize_f32(h->packed, h->scales, h->biases, &y.moe_norm, s, D.moe_norm, h->stream));
    ENNX_TRY(ennx_b200_packed_dequantize_f32(h->packed, h->scales, h->biases, &y.decay, s, D.decay, h->stream));
    ENNX_TRY(ennx_b200_packed_dequantize_f32(h->packed, h->scales, h->biases, &y.time_bias, s, D.time_bias, h->stream));
    ENNX_TRY(ennx_b200_packed_dequantize_f32(h->packed, h->scales, h->biases, &y.output_norm, s, D.out_norm, h->stream));
  }
  ENNX_TRY(ennx_b200_packed_dequantize_f32(h->packed, h->scales, h->biases, &h->final_norm, s, h->final_norm_v, h->stream));
  ENNX_CUDA(cudaStreamSynchronize(h->stream), "prepare");
  return ENNX_B200_OK;
}

int32_t ennx_b200_kda_decoder_decode_token(ennx_b200_kda_decoder* h, uint32_t token, uint64_t seed,
                                           uint32_t* next_token) {
  ENNX_TRY(check_current(h));
  if (token >= h->embedding.output_width)
    return set_error(ENNX_B200_INVALID_ARGUMENT, "token %u exceeds the model vocabulary", token);
  ENNX_CUDA(cudaMemcpyAsync(h->token, &token, sizeof(token), cudaMemcpyHostToDevice, h->stream), "token");
  ENNX_TRY(run_step(h, seed));
  uint32_t nx = 0;
  ENNX_CUDA(cudaMemcpyAsync(&nx, h->next, sizeof(nx), cudaMemcpyDeviceToHost, h->stream), "next token");
  ENNX_CUDA(cudaStreamSynchronize(h->stream), "decode");
  if (next_token) *next_token = nx;
  return consume_device_error(h->stream);
}

int32_t ennx_b200_kda_decoder_generate(ennx_b200_kda_decoder* h, const uint32_t* prompt, size_t prompt_len,
                                       size_t max_new_tokens, uint64_t seed, uint32_t* out) {
  ENNX_TRY(check_current(h));
  if (!prompt || prompt_len == 0) return set_error(ENNX_B200_INVALID_ARGUMENT, "generation prompt cannot be empty");
  if (!out) return set_error(ENNX_B200_INVALID_ARGUMENT, "generation output is null");
  for (size_t i = 0; i < prompt_len; ++i)
    if (prompt[i] >= h->embedding.output_width)
      return set_error(ENNX_B200_INVALID_ARGUMENT, "token %u exceeds the model vocabulary", prompt[i]);
  if (max_new_tokens > h->out_cap) {
    ENNX_CUDA(cudaStreamSynchronize(h->stream), "generate");
    cudaFree(h->out_tokens);
    h->out_tokens = nullptr;
    int32_t st = ENNX_B200_OK;
    h->out_tokens = (uint32_t*)dalloc(max_new_tokens * sizeof(uint32_t), &st);
    if (st) return st;
    h->out_cap = max_new_tokens;
    // the captured step holds the old output pointer
    if (h->have_graph) {
      cudaGraphExecDestroy(h->graph);
      h->have_graph = 0;
    }
  }
  // generate (forward_metal.rs:1372-1394): the prompt through decode_token,
  // then each prediction fed back; on the device the argmax of one step is
  // the token of the next, and its output slot counts the generated tokens.
  for (size_t i = 0; i < prompt_len; ++i) {
    ENNX_CUDA(cudaMemcpyAsync(h->token, &prompt[i], sizeof(uint32_t), cudaMemcpyHostToDevice, h->stream), "prompt");
    if (i + 1 == prompt_len) ENNX_CUDA(cudaMemsetAsync(h->out_count, 0, sizeof(uint32_t), h->stream), "count");
    ENNX_TRY(run_step(h, seed));
    ENNX_CUDA(cudaStreamSynchronize(h->stream), "prompt");  // the pageable prompt token is consumed
  }
  for (size_t i = 1; i < max_new_tokens; ++i) ENNX_TRY(run_step(h, seed));
  for (size_t i = 0; i < prompt_len; ++i) out[i] = prompt[i];
  if (max_new_tokens)
    ENNX_CUDA(cudaMemcpyAsync(out + prompt_len, h->out_tokens, max_new_tokens * sizeof(uint32_t),
                              cudaMemcpyDeviceToHost, h->stream),
              "generated tokens");
  ENNX_CUDA(cudaStreamSynchronize(h->stream), "generate");
  return consume_device_error(h->stream);
}

int32_t ennx_b200_kda_decoder_logits(ennx_b200_kda_decoder* h, float* out, size_t vocab) {
  ENNX_TRY(check_current(h));
  if (!out || vocab != h->embedding.output_width)
    return set_error(ENNX_B200_INVALID_ARGUMENT, "logits need %llu elements",
                     (unsigned long long)h->embedding.output_width);
  ENNX_CUDA(cudaMemcpyAsync(out, h->logits, vocab * sizeof(float), cudaMemcpyDeviceToHost, h->stream), "logits");
  ENNX_CUDA(cudaStreamSynchronize(h->stream), "logits");
  if (!h->has_logits)
    for (size_t i = 0; i < vocab; ++i) out[i] = 0.0f;
  return ENNX_B200_OK;
}

}  // extern "C"
