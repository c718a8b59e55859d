// moe.cu -- MoE routing (bit-exact router + top-k), expert-major
// permutation, row gather and weighted combine.
//
// Router math restates rust/crates/ennx/src/kda_moe.metal:570-621
// (moe_router_topk): fp32 logits x.W_r^T, top-k by insertion with strict '>'
// so ties keep the lower expert index, gates = max-subtracted softmax over the
// k kept logits.  The logits use a FIXED reduction order so that they -- and
// the routing indices -- are bit-identical to the CPU oracle
// (oracle/ennx_oracle.c eo_router_logits): lane l of a warp owns elements
// {256*j + 8*l + u}, runs a serial fma chain over j then u, and the 32
// partials meet in an xor butterfly (16, 8, 4, 2, 1).
#include "common.cuh"
#include "kernels.cuh"

namespace ennx {

// Router: a block owns up to TPB consecutive tokens of one weight set and
// walks the experts in chunks whose weights are staged in shared memory
// (EC experts x H bf16 <= 32 KB), so W_r is read from L2 once per block
// instead of once per token.  A warp handles one token at a time with x in
// registers; the per-lane element ownership and the fma/butterfly order are
// the fixed reduction order described above.
constexpr int kRouterTPB = 32;
constexpr int kRouterSmem = 32768;

template <int NJ, int SLOTS>
__global__ void __launch_bounds__(256) router_topk_kernel(
    const uint16_t* __restrict__ x, long long ldx, const uint16_t* __restrict__ w0, const uint16_t* __restrict__ w1,
    long long split, long long tokens, int experts, int top_k, float* __restrict__ logits, int* __restrict__ idx,
    float* __restrict__ gate) {
  constexpr int H = NJ * 256;
  constexpr int EC = kRouterSmem / (H * 2);
  constexpr int TPW = kRouterTPB / 8;  // tokens per warp
  __shared__ __align__(16) uint16_t ws[EC * H];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long nb0 = (split + kRouterTPB - 1) / kRouterTPB;
  long long tb, te;
  const uint16_t* w;
  if ((long long)blockIdx.x < nb0) {
    tb = (long long)blockIdx.x * kRouterTPB; te = min(split, tb + kRouterTPB); w = w0;
  } else {
    tb = split + ((long long)blockIdx.x - nb0) * kRouterTPB; te = min(tokens, tb + kRouterTPB); w = w1;
  }
  float mine[TPW][SLOTS];
#pragma unroll
  for (int tt = 0; tt < TPW; ++tt)
#pragma unroll
    for (int s = 0; s < SLOTS; ++s) mine[tt][s] = -INFINITY;

  for (int e0 = 0; e0 < experts; e0 += EC) {
    const int ne = min(EC, experts - e0);
    __syncthreads();
    for (int i = threadIdx.x; i < ne * H / 8; i += blockDim.x)
      reinterpret_cast<uint4*>(ws)[i] = __ldg(reinterpret_cast<const uint4*>(w + (long long)e0 * H) + i);
    __syncthreads();
#pragma unroll
    for (int tt = 0; tt < TPW; ++tt) {
      const long long t = tb + warp + 8 * tt;
      if (t >= te) break;
      uint4 xs[NJ];
#pragma unroll
      for (int j = 0; j < NJ; ++j) xs[j] = *reinterpret_cast<const uint4*>(x + t * ldx + 256 * j + 8 * lane);
      // four experts at a time: independent fma chains and butterflies give
      // the warp instruction-level parallelism; each logit keeps its own
      // fixed reduction order.
      int el = 0;
      for (; el + 4 <= ne; el += 4) {
        float p[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
        for (int j = 0; j < NJ; ++j) {
          uint32_t xw[4] = {xs[j].x, xs[j].y, xs[j].z, xs[j].w};
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            uint4 wv = *reinterpret_cast<const uint4*>(ws + (el + g) * H + 256 * j + 8 * lane);
            uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
            for (int h = 0; h < 4; ++h) {
              p[g] = __fmaf_rn(bf16_to_f32((uint16_t)(xw[h] & 0xffffu)), bf16_to_f32((uint16_t)(ww[h] & 0xffffu)), p[g]);
              p[g] = __fmaf_rn(bf16_to_f32((uint16_t)(xw[h] >> 16)), bf16_to_f32((uint16_t)(ww[h] >> 16)), p[g]);
            }
          }
        }
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1)
#pragma unroll
          for (int g = 0; g < 4; ++g) p[g] = __fadd_rn(p[g], __shfl_xor_sync(0xffffffffu, p[g], o));
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          const int e = e0 + el + g;
#pragma unroll
          for (int s2 = 0; s2 < SLOTS; ++s2)
            if (e >> 5 == s2 && lane == (e & 31)) mine[tt][s2] = p[g];
          if (logits && lane == 0) logits[t * experts + e] = p[g];
        }
      }
      for (; el < ne; ++el) {
        const uint16_t* wr = ws + el * H;
        float p = 0.0f;
#pragma unroll
        for (int j = 0; j < NJ; ++j) {
          uint4 wv = *reinterpret_cast<const uint4*>(wr + 256 * j + 8 * lane);
          uint32_t xw[4] = {xs[j].x, xs[j].y, xs[j].z, xs[j].w};
          uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
          for (int h = 0; h < 4; ++h) {
            p = __fmaf_rn(bf16_to_f32((uint16_t)(xw[h] & 0xffffu)), bf16_to_f32((uint16_t)(ww[h] & 0xffffu)), p);
            p = __fmaf_rn(bf16_to_f32((uint16_t)(xw[h] >> 16)), bf16_to_f32((uint16_t)(ww[h] >> 16)), p);
          }
        }
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) p = __fadd_rn(p, __shfl_xor_sync(0xffffffffu, p, o));
        const int e = e0 + el;
#pragma unroll
        for (int s2 = 0; s2 < SLOTS; ++s2)
          if (e >> 5 == s2 && lane == (e & 31)) mine[tt][s2] = p;
        if (logits && lane == 0) logits[t * experts + e] = p;
      }
    }
  }

#pragma unroll
  for (int tt = 0; tt < TPW; ++tt) {
    const long long t = tb + warp + 8 * tt;
    if (t >= te) break;
    float val[8];
    int ids[8];
    unsigned used = 0;
    for (int r = 0; r < top_k; ++r) {
      float bv = -INFINITY;
      int bi = 0x7fffffff;
#pragma unroll
      for (int s = 0; s < SLOTS; ++s) {
        int e = s * 32 + lane;
        if (e < experts && !(used >> s & 1u)) {
          if (mine[tt][s] > bv || (mine[tt][s] == bv && e < bi)) { bv = mine[tt][s]; bi = e; }
        }
      }
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) {
        float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
      }
      if (bi == 0x7fffffff) bi = 0;  // fewer finite logits than k: keep index 0 like the reference
      val[r] = bv;
      ids[r] = bi;
      if ((bi & 31) == lane) used |= 1u << (bi >> 5);
    }
    if (lane == 0) {
      float ex[8], den = 0.0f;
      for (int r = 0; r < top_k; ++r) { ex[r] = expf(val[r] - val[0]); den += ex[r]; }
      for (int r = 0; r < top_k; ++r) {
        idx[t * top_k + r] = ids[r];
        gate[t * top_k + r] = ex[r] / den;
      }
    }
  }
}

__global__ void moe_count_kernel(const int* __restrict__ idx, long long tokens, int top_k, int experts,
                                 long long split, int* __restrict__ counts) {
  long long n = tokens * top_k;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    long long t = i / top_k;
    int g = (t >= split ? experts : 0) + idx[i];
    atomicAdd(&counts[g], 1);
  }
}

// single block: exclusive scan of counts into offsets, reset cursors
__global__ void moe_scan_kernel(const int* __restrict__ counts, int groups, int* __restrict__ offsets,
                                int* __restrict__ cursor) {
  __shared__ int buf[1024];
  int tid = threadIdx.x;
  int v = tid < groups ? counts[tid] : 0;
  buf[tid] = v;
  __syncthreads();
  for (int o = 1; o < blockDim.x; o <<= 1) {
    int add = tid >= o ? buf[tid - o] : 0;
    __syncthreads();
    buf[tid] += add;
    __syncthreads();
  }
  if (tid < groups) {
    offsets[tid] = buf[tid] - v;
    cursor[tid] = 0;
  }
  if (tid == groups - 1) offsets[groups] = buf[tid];
}

__global__ void moe_scatter_kernel(const int* __restrict__ idx, const float* __restrict__ gate, long long tokens,
                                   int top_k, int experts, long long split, const int* __restrict__ offsets,
                                   int* __restrict__ cursor, int* __restrict__ perm_pos, int* __restrict__ src_row,
                                   float* __restrict__ perm_gate) {
  long long n = tokens * top_k;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    long long t = i / top_k;
    int g = (t >= split ? experts : 0) + idx[i];
    int pos = offsets[g] + atomicAdd(&cursor[g], 1);
    perm_pos[i] = pos;
    src_row[pos] = (int)t;
    perm_gate[pos] = gate[i];
  }
}

__global__ void gather_rows_kernel(const uint16_t* __restrict__ x, long long ldx, const int* __restrict__ src,
                                   long long rows, int width, uint16_t* __restrict__ out) {
  long long r = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  int lane = threadIdx.x & 31;
  if (r >= rows) return;
  const uint16_t* s = x + (long long)src[r] * ldx;
  uint16_t* d = out + r * width;
  for (int c = lane * 8; c < width; c += 256)
    *reinterpret_cast<uint4*>(d + c) = *reinterpret_cast<const uint4*>(s + c);
}

__global__ void moe_combine_kernel(const uint16_t* __restrict__ y, const int* __restrict__ perm_pos, long long tokens,
                                   int top_k, int width, const uint16_t* __restrict__ residual,
                                   uint16_t* __restrict__ out) {
  long long t = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  int lane = threadIdx.x & 31;
  if (t >= tokens) return;
  int pos[8];
  for (int r = 0; r < top_k; ++r) pos[r] = perm_pos[t * top_k + r];
  for (int c = lane * 8; c < width; c += 256) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    if (residual) {
      uint4 rv = *reinterpret_cast<const uint4*>(residual + t * width + c);
      uint32_t w[4] = {rv.x, rv.y, rv.z, rv.w};
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        acc[2 * h] = bf16_to_f32((uint16_t)(w[h] & 0xffffu));
        acc[2 * h + 1] = bf16_to_f32((uint16_t)(w[h] >> 16));
      }
    }
    for (int r = 0; r < top_k; ++r) {
      uint4 yv = *reinterpret_cast<const uint4*>(y + (long long)pos[r] * width + c);
      uint32_t w[4] = {yv.x, yv.y, yv.z, yv.w};
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        acc[2 * h] += bf16_to_f32((uint16_t)(w[h] & 0xffffu));
        acc[2 * h + 1] += bf16_to_f32((uint16_t)(w[h] >> 16));
      }
    }
    *reinterpret_cast<uint4*>(out + t * width + c) =
        make_uint4(pack_bf16x2(acc[0], acc[1]), pack_bf16x2(acc[2], acc[3]), pack_bf16x2(acc[4], acc[5]),
                   pack_bf16x2(acc[6], acc[7]));
  }
}

static int stride_grid(long long n, int threads) {
  long long b = (n + threads - 1) / threads;
  long long cap = (long long)sm_count() * 16;
  return (int)(b < cap ? (b > 0 ? b : 1) : cap);
}

template <int NJ>
static void launch_router_nj(int slots, dim3 g, dim3 b, cudaStream_t s, const uint16_t* x, long long ldx,
                             const uint16_t* w0, const uint16_t* w1, long long split, long long tokens, int experts,
                             int top_k, float* logits, int* idx, float* gate) {
  switch (slots) {
    case 1: router_topk_kernel<NJ, 1><<<g, b, 0, s>>>(x, ldx, w0, w1, split, tokens, experts, top_k, logits, idx, gate); break;
    case 2: router_topk_kernel<NJ, 2><<<g, b, 0, s>>>(x, ldx, w0, w1, split, tokens, experts, top_k, logits, idx, gate); break;
    case 4: router_topk_kernel<NJ, 4><<<g, b, 0, s>>>(x, ldx, w0, w1, split, tokens, experts, top_k, logits, idx, gate); break;
    default: router_topk_kernel<NJ, 8><<<g, b, 0, s>>>(x, ldx, w0, w1, split, tokens, experts, top_k, logits, idx, gate); break;
  }
}

int32_t launch_router_topk(const uint16_t* x, long long ldx, const uint16_t* w0, const uint16_t* w1, long long split,
                           long long tokens, int hidden, int experts, int top_k, float* logits, int* idx,
                           float* gate, cudaStream_t s) {
  if (top_k < 1 || top_k > 8 || top_k > experts)
    return set_error(ENNX_B200_INVALID_ARGUMENT, "router: top_k must be in [1, min(8, experts)]");  // forward_program.rs:428
  if (experts > 256) return set_error(ENNX_B200_UNSUPPORTED, "router: at most 256 experts");
  if (ldx % 8 || ((uintptr_t)x & 15u) || ((uintptr_t)w0 & 15u) || (w1 && ((uintptr_t)w1 & 15u)))
    return set_error(ENNX_B200_INVALID_ARGUMENT, "router: operands must be 16-byte aligned");
  int slots = (experts + 31) / 32;
  slots = slots <= 1 ? 1 : slots <= 2 ? 2 : slots <= 4 ? 4 : 8;
  if (!w1) { w1 = w0; split = tokens; }
  long long blocks = (split + kRouterTPB - 1) / kRouterTPB + (tokens - split + kRouterTPB - 1) / kRouterTPB;
  dim3 g((unsigned)blocks), b(256);
  switch (hidden) {
    case 256: launch_router_nj<1>(slots, g, b, s, x, ldx, w0, w1, split, tokens, experts, top_k, logits, idx, gate); break;
    case 512: launch_router_nj<2>(slots, g, b, s, x, ldx, w0, w1, split, tokens, experts, top_k, logits, idx, gate); break;
    case 1024: launch_router_nj<4>(slots, g, b, s, x, ldx, w0, w1, split, tokens, experts, top_k, logits, idx, gate); break;
    case 2048: launch_router_nj<8>(slots, g, b, s, x, ldx, w0, w1, split, tokens, experts, top_k, logits, idx, gate); break;
    case 4096: launch_router_nj<16>(slots, g, b, s, x, ldx, w0, w1, split, tokens, experts, top_k, logits, idx, gate); break;
    default: return set_error(ENNX_B200_UNSUPPORTED, "router: hidden %d not in {256,512,1024,2048,4096}", hidden);
  }
  ENNX_LAUNCH_CHECK("router_topk");
  return ENNX_B200_OK;
}

int32_t launch_moe_permute(const int* idx, const float* gate, long long tokens, int top_k, int experts, long long split,
                           int sets, int* counters, int* group_offsets, int* perm_pos, int* src_row,
                           float* perm_gate, cudaStream_t s) {
  int groups = sets * experts;
  if (groups > 1024) return set_error(ENNX_B200_UNSUPPORTED, "moe: at most 1024 (set, expert) groups");
  if (sets == 1) split = tokens;
  ENNX_CUDA(cudaMemsetAsync(counters, 0, sizeof(int) * groups, s), "moe counters");
  long long n = tokens * top_k;
  moe_count_kernel<<<stride_grid(n, 256), 256, 0, s>>>(idx, tokens, top_k, experts, split, counters);
  moe_scan_kernel<<<1, 1024, 0, s>>>(counters, groups, group_offsets, counters + groups);
  moe_scatter_kernel<<<stride_grid(n, 256), 256, 0, s>>>(idx, gate, tokens, top_k, experts, split, group_offsets,
                                                          counters + groups, perm_pos, src_row, perm_gate);
  note_launch(2);
  ENNX_LAUNCH_CHECK("moe_permute");
  return ENNX_B200_OK;
}

int32_t launch_gather_rows(const uint16_t* x, long long ldx, const int* src_row, long long rows, int width,
                           uint16_t* out, cudaStream_t s) {
  if (width % 256) return set_error(ENNX_B200_UNSUPPORTED, "gather: width must be a multiple of 256");
  gather_rows_kernel<<<(unsigned)((rows + 7) / 8), 256, 0, s>>>(x, ldx, src_row, rows, width, out);
  ENNX_LAUNCH_CHECK("gather_rows");
  return ENNX_B200_OK;
}

int32_t launch_moe_combine(const uint16_t* y, const int* perm_pos, long long tokens, int top_k, int width,
                           const uint16_t* residual, uint16_t* out, cudaStream_t s) {
  if (width % 256) return set_error(ENNX_B200_UNSUPPORTED, "combine: width must be a multiple of 256");
  moe_combine_kernel<<<(unsigned)((tokens + 7) / 8), 256, 0, s>>>(y, perm_pos, tokens, top_k, width, residual, out);
  ENNX_LAUNCH_CHECK("moe_combine");
  return ENNX_B200_OK;
}

}  // namespace ennx
