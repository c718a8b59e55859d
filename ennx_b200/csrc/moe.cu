// moe.cu -- MoE routing (bit-exact router + top-k), expert-major
// permutation, row gather and weighted combine.
//
// Router math restates rust/crates/ennx/src/kda_moe.metal:570-621
// (moe_router_topk): fp32 logits x.W_r^T, top-k by insertion with strict '>'
// so ties keep the lower expert index, gates = max-subtracted softmax over the
// k kept logits.  Each logit is one serial fma chain over the hidden index,
// the order of the reference's per-token loop, so the logits -- and the
// routing indices -- are bit-identical to the CPU oracle
// (oracle/ennx_oracle.c eo_router_logits).
#include "common.cuh"
#include "kernels.cuh"

namespace ennx {

// Router: a register-blocked fp32 SIMT GEMM.  A block owns RT consecutive
// tokens of one weight set and all experts (in tiles of RE); K is staged
// through shared memory in chunks of RK, converted from bf16 to fp32 once.
// Thread (ty, tx) accumulates tokens 8*ty..8*ty+7 x experts 4*tx..4*tx+3,
// each logit one serial fma chain over k = 0, 1, ..., H-1 starting from 0 --
// the order of the reference's per-token loop (kda_moe.metal:589-595) and of
// the CPU oracle, so logits are bit-identical.  The serial chain rules out
// splitting K; the parallelism comes from 32 independent chains per thread,
// issued as 16 packed fma.rn.f32x2 per k-step (two independent IEEE fma.rn
// each), with operands loaded one k-step ahead.  The logits of the block's tokens
// are kept in shared memory; one thread per token then runs the insertion
// top-k and the gate softmax.
//
// Sizes: 56 tokens per block (7 rows of 16 threads), so that one weight set
// of 4096 tokens -- half of a pair's rows -- is 74 blocks and a pair fills
// the 148 SMs exactly.  Each K chunk (64 k) is copied into a bf16 staging
// area with cp.async before the previous chunk's FMAs run, so the copies are
// in flight meanwhile.  (A dedicated feed warp converting for the other four
// measured slower: one warp's conversion outlasts a chunk of FMAs.)
constexpr int RT = 56, RE = 64, RK = 64, kRouterThreads = 112;
static_assert(RT == 8 * (kRouterThreads / 16) && RE == 4 * 16, "thread (tx, ty) owns 8 tokens x 4 experts");

__device__ __forceinline__ uint64_t pack_f32x2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
// two independent IEEE fma.rn in one instruction (sm_100)
__device__ __forceinline__ uint64_t fma_f32x2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
constexpr int kXLoads = RK * RT / 8, kWLoads = RK * RE / 8;     // uint4 per chunk (x rows, expert rows)
constexpr int kXPer = (kXLoads + kRouterThreads - 1) / kRouterThreads;
constexpr int kWPer = (kWLoads + kRouterThreads - 1) / kRouterThreads;
// 16-byte global -> shared copy (zero fill when !ok)
__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool ok) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(ok ? 16 : 0)
               : "memory");
}

// The router weights of both sets as fp32, k-major per tile of RE experts:
// wt[set][tile][k][RE] (experts past the end are zero).  One conversion per
// call, so the router blocks copy their expert operand chunks (RK x RE fp32,
// 16 KB, contiguous) straight into shared memory instead of each converting
// the same rows.
__global__ void router_wt_kernel(const uint16_t* __restrict__ w0, const uint16_t* __restrict__ w1, int hidden,
                                 int experts, int tiles, float* __restrict__ wt) {
  const long long per_set = (long long)tiles * hidden * RE;
  const long long total = 2 * per_set;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const int set = (int)(i / per_set);
    const long long j = i - set * per_set;
    const int tile = (int)(j / ((long long)hidden * RE));
    const int k = (int)((j / RE) % hidden), e = tile * RE + (int)(j % RE);
    wt[i] = e < experts ? bf16_to_f32((set ? w1 : w0)[(long long)e * hidden + k]) : 0.0f;
  }
}

__global__ void __launch_bounds__(kRouterThreads, 2) router_topk_kernel(
    const uint16_t* __restrict__ x, long long ldx, const uint16_t* __restrict__ w0, const uint16_t* __restrict__ w1,
    long long split, long long tokens, int hidden, int experts, int top_k, float* __restrict__ logits,
    int* __restrict__ idx, float* __restrict__ gate, int* __restrict__ counts, const float* __restrict__ wt) {
  extern __shared__ __align__(16) float rsm[];
  __shared__ int hist[256];  // picks per expert of this block's tokens (counts != nullptr)
  float* As = rsm;                  // [2][RK][RT]
  float* Bs = As + 2 * RK * RT;     // [2][RK][RE]
  float* Ls = Bs + 2 * RK * RE;     // [RT][lds]
  const int lds = ((experts + RE - 1) / RE) * RE + 1;
  uint16_t* xst = reinterpret_cast<uint16_t*>(Ls + (RT * lds + 3) / 4 * 4);  // [kXLoads][8] bf16 staging
  uint16_t* wst = xst + kXLoads * 8;                                         // [kWLoads][8]
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const long long nb0 = (split + RT - 1) / RT;
  long long tb, te;
  const uint16_t* w;
  const int set = (long long)blockIdx.x < nb0 ? 0 : 1;
  const int tiles = (experts + RE - 1) / RE;
  if ((long long)blockIdx.x < nb0) {
    tb = (long long)blockIdx.x * RT; te = min(split, tb + RT); w = w0;
  } else {
    tb = split + ((long long)blockIdx.x - nb0) * RT; te = min(tokens, tb + RT); w = w1;
  }
  const int nchunks = hidden / RK;
  for (int e0 = 0; e0 < experts; e0 += RE) {
    // chunk c's copies (16 B = 8 k of one token or expert each); each thread
    // later converts exactly the pieces it copied, so the staging needs no
    // barrier of its own
    auto fetch = [&](int c) {
#pragma unroll
      for (int i = 0; i < kXPer; ++i) {
        const int li = tid + i * kRouterThreads, t = li % RT, q = li / RT;
        if (li < kXLoads) {
          const bool ok = tb + t < te;
          cp_async16(xst + li * 8, x + (ok ? (tb + t) * ldx + c * RK + 8 * q : 0), ok);
        }
      }
      if (wt) {  // fp32 operand chunk, copied straight into Bs[c & 1]
        const float* src = wt + (((long long)set * tiles + e0 / RE) * hidden + (long long)c * RK) * RE;
        float* dst = Bs + (c & 1) * RK * RE;
        for (int li = tid; li < RK * RE / 4; li += kRouterThreads) cp_async16(dst + 4 * li, src + 4 * li, true);
      } else {
#pragma unroll
        for (int i = 0; i < kWPer; ++i) {
          const int li = tid + i * kRouterThreads, e = e0 + li % RE, qe = li / RE;
          if (li < kWLoads) {
            const bool ok = e < experts;
            cp_async16(wst + li * 8, w + (ok ? (long long)e * hidden + c * RK + 8 * qe : 0), ok);
          }
        }
      }
      asm volatile("cp.async.commit_group;" ::: "memory");
    };
    // the staged chunk into the fp32 operands As/Bs[buf]
    auto stash = [&](int buf) {
      asm volatile("cp.async.wait_group 0;" ::: "memory");
      float* a = As + buf * RK * RT;
      float* bb = Bs + buf * RK * RE;
#pragma unroll
      for (int i = 0; i < kXPer; ++i) {
        const int li = tid + i * kRouterThreads, t = li % RT, q = li / RT;
        if (li >= kXLoads) break;
        const uint4 v = *reinterpret_cast<const uint4*>(xst + li * 8);
        const uint32_t xv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          a[(8 * q + 2 * h) * RT + t] = bf16_to_f32((uint16_t)(xv[h] & 0xffffu));
          a[(8 * q + 2 * h + 1) * RT + t] = bf16_to_f32((uint16_t)(xv[h] >> 16));
        }
      }
#pragma unroll
      for (int i = 0; i < kWPer; ++i) {
        const int li = tid + i * kRouterThreads, e = li % RE, qe = li / RE;
        if (wt || li >= kWLoads) break;
        const uint4 v = *reinterpret_cast<const uint4*>(wst + li * 8);
        const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          bb[(8 * qe + 2 * h) * RE + e] = bf16_to_f32((uint16_t)(wv[h] & 0xffffu));
          bb[(8 * qe + 2 * h + 1) * RE + e] = bf16_to_f32((uint16_t)(wv[h] >> 16));
        }
      }
    };
    uint64_t accp[4][4];  // accp[i][j] = (logit of token 8ty+2i, of token 8ty+2i+1) for expert 4tx+j
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) accp[i][j] = 0ull;
    __syncthreads();  // previous expert tile's readers are done with the buffers
    fetch(0);
    stash(0);
    __syncthreads();
    for (int c = 0; c < nchunks; ++c) {
      if (c + 1 < nchunks) fetch(c + 1);
      const float* a = As + (c & 1) * RK * RT + 8 * ty;
      const float* bb = Bs + (c & 1) * RK * RE + 4 * tx;
      // operands one k-step ahead; the FMAs run as packed pairs over tokens
      // (fma.rn.f32x2: two independent fma.rn per instruction)
      float4 a0 = *reinterpret_cast<const float4*>(a), a1 = *reinterpret_cast<const float4*>(a + 4);
      float4 b0 = *reinterpret_cast<const float4*>(bb);
#pragma unroll
      for (int k = 0; k < RK; ++k) {
        float4 na0, na1, nb0v;
        if (k + 1 < RK) {
          na0 = *reinterpret_cast<const float4*>(a + (k + 1) * RT);
          na1 = *reinterpret_cast<const float4*>(a + (k + 1) * RT + 4);
          nb0v = *reinterpret_cast<const float4*>(bb + (k + 1) * RE);
        }
        const uint64_t ap[4] = {pack_f32x2(a0.x, a0.y), pack_f32x2(a0.z, a0.w), pack_f32x2(a1.x, a1.y),
                                pack_f32x2(a1.z, a1.w)};
        const float br[4] = {b0.x, b0.y, b0.z, b0.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint64_t bj = pack_f32x2(br[j], br[j]);
#pragma unroll
          for (int i = 0; i < 4; ++i) accp[i][j] = fma_f32x2(ap[i], bj, accp[i][j]);
        }
        if (k + 1 < RK) { a0 = na0; a1 = na1; b0 = nb0v; }
      }
      if (c + 1 < nchunks) stash((c + 1) & 1);
      __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        Ls[(8 * ty + 2 * i) * lds + e0 + 4 * tx + j] = __uint_as_float((uint32_t)accp[i][j]);
        Ls[(8 * ty + 2 * i + 1) * lds + e0 + 4 * tx + j] = __uint_as_float((uint32_t)(accp[i][j] >> 32));
      }
  }
  for (int e = tid; e < experts; e += kRouterThreads) hist[e] = 0;
  __syncthreads();
  if (logits) {
    for (int i = tid; i < RT * experts; i += kRouterThreads) {
      const int r = i / experts, e = i % experts;
      if (tb + r < te) logits[(tb + r) * experts + e] = Ls[r * lds + e];
    }
  }
  if (tid < RT && tb + tid < te) {
    // insertion with strict '>': once a score is inserted at rank r every
    // lower rank shifts down by one (branch-free over constant indices)
    float val[8];
    int ids[8];
#pragma unroll
    for (int r = 0; r < 8; ++r) { val[r] = -INFINITY; ids[r] = 0; }
    const float* row = Ls + tid * lds;
    for (int e = 0; e < experts; ++e) {
      float v = row[e];
      int id = e;
      bool shifting = false;
#pragma unroll
      for (int r = 0; r < 8; ++r) {
        if (r < top_k) {
          const bool take = shifting || v > val[r];
          if (take) {
            const float tv = val[r];
            const int ti = ids[r];
            val[r] = v; ids[r] = id; v = tv; id = ti;
          }
          shifting = take;
        }
      }
    }
    float ex[8], den = 0.0f;
#pragma unroll
    for (int r = 0; r < 8; ++r)
      if (r < top_k) { ex[r] = expf(val[r] - val[0]); den += ex[r]; }
    const long long t = tb + tid;
#pragma unroll
    for (int r = 0; r < 8; ++r)
      if (r < top_k) {
        idx[t * top_k + r] = ids[r];
        gate[t * top_k + r] = ex[r] / den;
        if (counts) atomicAdd(&hist[ids[r]], 1);
      }
  }
  if (counts) {  // group = (weight set, expert); this block's tokens all use one set
    __syncthreads();
    const int set = (long long)blockIdx.x < nb0 ? 0 : 1;
    for (int e = tid; e < experts; e += kRouterThreads)
      if (hist[e]) atomicAdd(&counts[set * experts + e], hist[e]);
  }
}

// Expert-major permutation and row copy in one pass.  Every block rebuilds the
// exclusive scan of the per-group pick counts in shared memory (block 0 also
// publishes it for the grouped GEMM); a warp per token claims one slot per
// pick in its group (order inside a group is arbitrary, results are not:
// each slot is a whole row) and copies the token's row, read once, into all
// of its slots.
__global__ void __launch_bounds__(256) moe_scatter_gather_kernel(
    const int* __restrict__ idx, const float* __restrict__ gate, float gate_scale, long long tokens, int top_k,
    int experts, long long split, int groups, const int* __restrict__ counts, int* __restrict__ offsets,
    int* __restrict__ cursor, int* __restrict__ perm_pos, float* __restrict__ perm_gate,
    const uint16_t* __restrict__ x, long long ldx, int width, uint16_t* __restrict__ xperm) {
  __shared__ int off[257];
  __shared__ int wsum[8];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  {  // exclusive scan of counts[0 .. groups) (groups <= 256)
    int v = tid < groups ? counts[tid] : 0;
    int incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int n = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += n;
    }
    if (lane == 31) wsum[warp] = incl;
    __syncthreads();
    int base = 0;
    for (int w = 0; w < warp; ++w) base += wsum[w];
    off[tid] = base + incl - v;
    if (tid == 255) off[256] = base + incl;
    __syncthreads();
    if (blockIdx.x == 0) {
      if (tid < groups) offsets[tid] = off[tid];
      if (tid == 0) offsets[groups] = off[groups];  // total (counts past `groups` read as 0)
    }
  }
  const long long t = (long long)blockIdx.x * 8 + warp;
  if (t >= tokens) return;
  int pos = 0;
  if (lane < top_k) {
    const int g = (t >= split ? experts : 0) + idx[t * top_k + lane];
    pos = off[g] + atomicAdd(&cursor[g], 1);
    perm_pos[t * top_k + lane] = pos;
    perm_gate[pos] = gate_scale * gate[t * top_k + lane];
  }
  // the row goes through this warp's 4 KB of shared memory in segments of
  // 2048 elements: eight 16-byte loads per lane (all in flight), one store
  // to shared memory, then one bulk copy (TMA engine) per slot
  __shared__ __align__(128) uint4 seg_buf[8][256];
  uint4* buf = seg_buf[warp];
  const uint32_t buf_s = smem_u32(buf);
  const uint16_t* src = x + t * ldx;
  int slot[8];
#pragma unroll
  for (int r = 0; r < 8; ++r) slot[r] = __shfl_sync(0xffffffffu, pos, r);
  for (int s0 = 0; s0 < width; s0 += 2048) {
    const int seg = min(2048, width - s0);
    uint4 v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (lane * 8 + j * 256 < seg) v[j] = ldg_stream_v4(src + s0 + lane * 8 + j * 256);
    if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");  // previous segment read out
    __syncwarp();
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (lane * 8 + j * 256 < seg) buf[lane + 32 * j] = v[j];
    fence_proxy_async();
    __syncwarp();
    if (lane == 0) {
      for (int r = 0; r < top_k; ++r) {
        uint16_t* dst = xperm + (long long)slot[r] * width + s0;
        asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst), "r"(buf_s),
                     "r"(seg * 2)
                     : "memory");
      }
      asm volatile("cp.async.bulk.commit_group;" ::: "memory");
    }
  }
  if (lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
  __syncwarp();
}

// out = residual + sum_r y[perm_pos[t, r]] (fp32 sum in pick order, one
// rounding).  A warp per token; each lane keeps two 16-byte chunks of all
// top_k rows in flight before it sums.
__global__ void moe_combine_kernel(const uint16_t* __restrict__ y, const int* __restrict__ perm_pos, long long tokens,
                                   int top_k, int width, const uint16_t* __restrict__ residual,
                                   uint16_t* __restrict__ out) {
  long long t = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  int lane = threadIdx.x & 31;
  if (t >= tokens) return;
  int pos[8];
#pragma unroll
  for (int r = 0; r < 8; ++r) pos[r] = r < top_k ? perm_pos[t * top_k + r] : 0;
  for (int c0 = lane * 8; c0 < width; c0 += 2 * 256) {
    float acc[2][8];
    uint4 yv[2][8];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int c = c0 + u * 256;
#pragma unroll
      for (int h = 0; h < 8; ++h) acc[u][h] = 0.0f;
      if (c < width && residual) {
        const uint4 rv = *reinterpret_cast<const uint4*>(residual + t * width + c);
        const uint32_t w[4] = {rv.x, rv.y, rv.z, rv.w};
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          acc[u][2 * h] = bf16_to_f32((uint16_t)(w[h] & 0xffffu));
          acc[u][2 * h + 1] = bf16_to_f32((uint16_t)(w[h] >> 16));
        }
      }
#pragma unroll
      for (int r = 0; r < 8; ++r)
        if (r < top_k && c < width) yv[u][r] = ldg_stream_v4(y + (long long)pos[r] * width + c);
    }
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int c = c0 + u * 256;
      if (c >= width) break;
#pragma unroll
      for (int r = 0; r < 8; ++r) {
        if (r >= top_k) break;
        const uint32_t w[4] = {yv[u][r].x, yv[u][r].y, yv[u][r].z, yv[u][r].w};
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          acc[u][2 * h] += bf16_to_f32((uint16_t)(w[h] & 0xffffu));
          acc[u][2 * h + 1] += bf16_to_f32((uint16_t)(w[h] >> 16));
        }
      }
      *reinterpret_cast<uint4*>(out + t * width + c) =
          make_uint4(pack_bf16x2(acc[u][0], acc[u][1]), pack_bf16x2(acc[u][2], acc[u][3]),
                     pack_bf16x2(acc[u][4], acc[u][5]), pack_bf16x2(acc[u][6], acc[u][7]));
    }
  }
}

int32_t launch_router_topk(const uint16_t* x, long long ldx, const uint16_t* w0, const uint16_t* w1, long long split,
                           long long tokens, int hidden, int experts, int top_k, float* logits, int* idx,
                           float* gate, cudaStream_t s, int* counts, float* wt) {
  if (top_k < 1 || top_k > 8 || top_k > experts)
    return set_error(ENNX_B200_INVALID_ARGUMENT, "router: top_k must be in [1, min(8, experts)]");  // forward_program.rs:428
  if (experts > 256) return set_error(ENNX_B200_UNSUPPORTED, "router: at most 256 experts");
  if (hidden <= 0 || hidden % RK) return set_error(ENNX_B200_UNSUPPORTED, "router: hidden %d must be a multiple of %d", hidden, RK);
  if (ldx % 8 || ((uintptr_t)x & 15u) || ((uintptr_t)w0 & 15u) || (w1 && ((uintptr_t)w1 & 15u)))
    return set_error(ENNX_B200_INVALID_ARGUMENT, "router: operands must be 16-byte aligned");
  if (tokens <= 0) return ENNX_B200_OK;
  if (!w1) { w1 = w0; split = tokens; }
  const long long blocks = (split + RT - 1) / RT + (tokens - split + RT - 1) / RT;
  const int lds = ((experts + RE - 1) / RE) * RE + 1;
  const size_t smem = sizeof(float) * (2 * RK * RT + 2 * RK * RE + ((size_t)RT * lds + 3) / 4 * 4) +
                      16 * (kXLoads + kWLoads);
  static bool attr[64];
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr[dev]) {
    ENNX_CUDA(cudaFuncSetAttribute(router_topk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)(sizeof(float) * (2 * RK * RT + 2 * RK * RE + (RT * (256 + 1) + 3) / 4 * 4) +
                                         16 * (kXLoads + kWLoads))),
              "router smem");
    attr[dev] = true;
  }
  if (wt) {
    if ((uintptr_t)wt & 15u) return set_error(ENNX_B200_INVALID_ARGUMENT, "router: fp32 weight scratch must be 16-byte aligned");
    const long long n = 2LL * ((experts + RE - 1) / RE) * hidden * RE;
    router_wt_kernel<<<(unsigned)((n + 255) / 256 < 4LL * sm_count() ? (n + 255) / 256 : 4LL * sm_count()), 256, 0, s>>>(
        w0, w1, hidden, experts, (experts + RE - 1) / RE, wt);
    ENNX_LAUNCH_CHECK("router_wt");
  }
  router_topk_kernel<<<(unsigned)blocks, kRouterThreads, smem, s>>>(x, ldx, w0, w1, split, tokens, hidden, experts,
                                                                      top_k, logits, idx, gate, counts, wt);
  ENNX_LAUNCH_CHECK("router_topk");
  return ENNX_B200_OK;
}

int32_t launch_moe_scatter_gather(const int* idx, const float* gate, float gate_scale, long long tokens, int top_k,
                                  int experts, long long split, int sets, const int* counts, int* offsets, int* cursor,
                                  int* perm_pos, float* perm_gate, const uint16_t* x, long long ldx, int width,
                                  uint16_t* xperm, cudaStream_t s) {
  const int groups = sets * experts;
  if (groups > 256) return set_error(ENNX_B200_UNSUPPORTED, "moe: at most 256 (set, expert) groups");
  if (width % 256 || ldx % 8) return set_error(ENNX_B200_UNSUPPORTED, "moe: width must be a multiple of 256");
  if (sets == 1) split = tokens;
  moe_scatter_gather_kernel<<<(unsigned)((tokens + 7) / 8), 256, 0, s>>>(idx, gate, gate_scale, tokens, top_k, experts,
                                                                       split, groups, counts, offsets, cursor,
                                                                       perm_pos, perm_gate, x, ldx, width, xperm);
  ENNX_LAUNCH_CHECK("moe_scatter_gather");
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
