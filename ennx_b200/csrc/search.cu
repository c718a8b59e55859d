// search.cu -- resident BF16 TuRBO search: candidate scoring against the
// trust-region history, per-region selection, materialisation of the chosen
// candidates and the device-side tell (history, incumbent, trust region).
//
// Restates the ennx-cuda Bf16SearchEngine (cuda/src/bf16_search.rs:129-1067)
// and its kernels (cuda/kernels/src/lib.rs:1310-1480, 1657-1745, 2050-2308;
// cuda/kernels/src/bf16.rs:160-330, lib.rs:409-535).  Layout and kernel split
// are this library's own:
//
//   * rows [slots][stride] bf16 (stride = len rounded up to 128 elements,
//     256-byte aligned rows), slot 0 = incumbent, 1..capacity = history,
//     the rest = pending trials; batch [regions][len] = the last proposals.
//   * search_distance_kernel: one CTA per element tile computes every
//     candidate's BF16 values for its tile once (in registers, packed bf16
//     pairs) and streams each history row once, accumulating the weighted
//     squared distances of 8 candidates x 2 history rows per pass with
//     packed f32x2 arithmetic.  The reference's CTA per (candidate, tile)
//     re-reads every history row once per candidate.  Distances are direct
//     differences: |c|^2 + |h|^2 - 2 c.h on tensor cores would cancel
//     catastrophically, since candidates and history rows all lie within a
//     trust region around the same base.
//   * search_score_pick_kernel: per candidate, sums the tile partials in a
//     fixed tree order with the whole CTA, runs the k-nearest-neighbour
//     acquisition (the float order of acquisition_score, bf16.rs:224-275);
//     the region's last CTA to finish picks its best candidate (lower index
//     on ties, lib.rs:1660-1744) -- score and pick in one launch.
//   * search_write_kernel: materialises the selected candidates (bf16_seed).
//   * search_tell_plan_kernel + search_tell_copy_kernel: the sequential
//     bookkeeping of tell_bf16 on one thread, then the row copies it decides
//     (best -> slot 0, trials -> history slots, restart -> slot 1) as one
//     grid-wide pass instead of a single CTA.
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include "common.cuh"

extern "C" int32_t ennx_b200_check_bf16(const uint16_t* v, size_t n, int32_t* all_finite, void* stream);

namespace ennx {
namespace {

constexpr int kThreads = 256;
constexpr int kTileElems = kThreads * 8;  // one 16-byte vector per thread
constexpr int kMaxHistory = 128;          // MAX_HISTORY, cuda/kernels/src/lib.rs:18
constexpr int kMaxPending = 32;           // BF16_MAX_PENDING, bf16_search.rs:7
constexpr int kChunk = 8;                 // candidates per register pass
constexpr int kGroup = 32;                // candidates sharing one pass over the history

struct SearchLeaf {  // Bf16Leaf with mix64(key ^ K) precomputed
  uint64_t key_mix;
  uint64_t offset;
  uint64_t length;
  float scale;
  float weight;
};

struct SearchStateDev {  // SearchState, cuda/kernels/src/bf16.rs:41-58
  double length, length_init, length_min, length_max, trust_best, hist_min, hist_max;
  float best, best_variance;
  uint64_t prev_obs;
  uint32_t successes, failures, restarts, history, status;
};

struct CopyPlan {  // row copies decided by one tell
  uint32_t valid, best_slot, restarted, count;
  uint32_t src[kMaxPending], dst[kMaxPending];
};

struct AskArgs {
  const uint16_t* rows;
  uint64_t stride;
  uint64_t len;
  uint32_t base_slot;
  uint32_t history;       // host value; the device state's when resident
  uint32_t hstride;       // partial / distance stride over history rows
  uint32_t candidates;
  uint32_t cpr;           // candidates per region
  uint32_t regions;
  uint32_t parts;         // CTAs of the distance kernel
  uint32_t nl;
  uint32_t neighbors;
  uint32_t acquisition;
  int32_t resident;
  float coefficient;
  float epistemic_scale, aleatoric_scale, y_scale, beta;
  uint64_t seed_root;
  uint64_t draw_seed;
  const uint64_t* seeds;
  const SearchLeaf* leaves;
  const uint32_t* history_slots;
  const float* outcomes;
  const float* variances;
  const SearchStateDev* state;
  float* partials;        // [parts][candidates][hstride]
  uint32_t* invalid;      // [candidates]
  float* distances;       // [candidates][hstride]
  float* scores;          // [candidates]
  ennx_b200_selection* selection;  // [regions]
  const uint32_t* trial_slots;     // [regions]
  uint16_t* rows_out;
  uint16_t* batch;
  uint32_t* region_status;         // [regions]
  uint32_t* region_done;           // [regions] tickets of the score kernel
};

// trial_hash, cuda/kernels/src/lib.rs:150-158
__host__ __device__ __forceinline__ uint32_t trial_hash(uint32_t lo, uint32_t hi, uint32_t element) {
  uint32_t v = lo ^ (element * 0x9e3779b9u);
  v ^= v >> 16;
  v *= 0x7feb352du;
  v ^= hi;
  v *= 0x846ca68bu;
  return v ^ (v >> 15);
}

// Candidate seed: host-provided, or derived from the round's root as
// seed_bf16 does (lib.rs:1466-1480).
__device__ __forceinline__ uint64_t candidate_seed(const AskArgs& a, uint32_t c) {
  if (!a.resident) return a.seeds[c];
  uint32_t lo = (uint32_t)a.seed_root, hi = (uint32_t)(a.seed_root >> 32);
  uint32_t s_lo = trial_hash(lo, hi, c);
  uint32_t s_hi = trial_hash(hi, lo, c ^ 0x9e3779b9u);
  return (uint64_t)s_lo | ((uint64_t)s_hi << 32);
}

__device__ __forceinline__ float step_coefficient(const AskArgs& a) {
  return a.resident ? (float)a.state->length : a.coefficient;
}
__device__ __forceinline__ uint32_t history_rows(const AskArgs& a) {
  return a.resident ? min(a.state->history, (uint32_t)kMaxHistory) : a.history;
}

// bf16_seed (cuda/kernels/src/bf16.rs:160-176): v + scale*coef*sign rounded
// to BF16, or one ulp toward the step if that leaves v unchanged.  The
// products and the sum round separately, as in the reference.
// Bit 0 of mix64(x), the sign of dense_sign (lib.rs:345-353): the last
// xor-shift makes it bit0 ^ bit31 of the last product, whose low 32 bits only
// need the low 32 bits of its operands -- one 32-bit multiply instead of a
// 64-bit one.
__device__ __forceinline__ uint32_t mix64_bit0(uint64_t x) {
  uint64_t v = x + 0x9e3779b97f4a7c15ull;
  v = (v ^ (v >> 30)) * 0xbf58476d1ce4e5b9ull;
  const uint32_t lo = (uint32_t)(v ^ (v >> 27)) * 0x133111ebu;  // low word of 0x94d049bb133111eb
  return (lo ^ (lo >> 31)) & 1u;
}

__device__ __forceinline__ uint16_t bf16_seed(uint16_t v, uint64_t key_mix, uint64_t emix, float scale,
                                              uint64_t seed, float coef) {
  float dir = mix64_bit0(seed ^ key_mix ^ emix) ? 1.0f : -1.0f;
  float x = __fadd_rn(bf16_to_f32(v), __fmul_rn(__fmul_rn(scale, coef), dir));
  uint16_t cand = f32_to_bf16_rne(x);
  if (coef == 0.0f || cand == v) return bf16_next(v, (coef > 0.0f) == (dir > 0.0f));
  return cand;
}

__device__ __forceinline__ bool bf16_is_finite(uint16_t v) { return (v & 0x7f80u) != 0x7f80u; }

__device__ __forceinline__ int find_leaf(const SearchLeaf* leaves, int nl, uint64_t i) {
  int lo = 0, hi = nl - 1;
  while (lo < hi) {
    int mid = (lo + hi + 1) >> 1;
    if (__ldg(&leaves[mid].offset) <= i) lo = mid; else hi = mid - 1;
  }
  return lo;
}

__device__ __forceinline__ uint4 ld_row16(const uint16_t* p) { return __ldg(reinterpret_cast<const uint4*>(p)); }

// packed f32x2 helpers (two independent IEEE operations per instruction)
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t f2_sub(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
// bf16 pair (low half = even element) -> packed f32x2
__device__ __forceinline__ uint64_t bf2_to_f2(uint32_t p) {
  return f2_pack(__uint_as_float(p << 16), __uint_as_float(p & 0xffff0000u));
}

// Warp transpose-reduction of 16 values: lane pair (2k, 2k+1) returns the
// warp sum of value k.  16 shuffles instead of 80 for a butterfly per value.
__device__ __forceinline__ float xpose_reduce16(float (&v)[16], int lane) {
  bool up = lane & 16;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    float send = up ? v[i] : v[i + 8], keep = up ? v[i + 8] : v[i];
    v[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
  }
  up = lane & 8;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float send = up ? v[i] : v[i + 4], keep = up ? v[i + 4] : v[i];
    v[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
  }
  up = lane & 4;
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    float send = up ? v[i] : v[i + 2], keep = up ? v[i + 2] : v[i];
    v[i] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
  }
  up = lane & 2;
  {
    float send = up ? v[0] : v[1], keep = up ? v[1] : v[0];
    v[0] = keep + __shfl_xor_sync(0xffffffffu, send, 2);
  }
  return v[0] + __shfl_xor_sync(0xffffffffu, v[0], 1);
}

// ---------------------------------------------------------------------------
// distances: partials[part][c][h] = sum over the part's tiles of
// w * (cand_c - hist_h)^2.  CTA `part` takes tiles part, part + grid, ...;
// per tile every thread owns one 16-byte vector (8 elements).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kThreads) search_distance_kernel(const __grid_constant__ AskArgs a) {
  __shared__ float red[2][kThreads / 32][16];
  __shared__ float part_sum[kGroup][kMaxHistory];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint32_t H = history_rows(a);
  const float coef = step_coefficient(a);
  const uint64_t tiles = (a.len + kTileElems - 1) / kTileElems;
  int rbuf = 0;
  // Candidates in groups of kGroup: per tile, every chunk of the group reads
  // the same history tiles, so HBM sees each history row once per group.
  for (uint32_t g0 = 0; g0 < a.candidates; g0 += kGroup) {
    for (int i = tid; i < kGroup * kMaxHistory; i += kThreads) part_sum[i / kMaxHistory][i % kMaxHistory] = 0.0f;
    __syncthreads();
    for (uint64_t tile = blockIdx.x; tile < tiles; tile += gridDim.x)
    for (uint32_t c0 = g0; c0 < g0 + kGroup && c0 < a.candidates; c0 += kChunk) {
      uint64_t seed[kChunk];
#pragma unroll
      for (int c = 0; c < kChunk; ++c) seed[c] = c0 + c < a.candidates ? candidate_seed(a, c0 + c) : 0;
      const uint64_t e0 = tile * kTileElems + (uint64_t)tid * 8;
      const bool active = e0 < a.len;
      // history rows 0 and 1 in flight while the candidates are generated
      uint4 nxt[2];
#pragma unroll
      for (int hh = 0; hh < 2; ++hh)
        nxt[hh] = active && (uint32_t)hh < H
                      ? ld_row16(a.rows + (uint64_t)__ldg(&a.history_slots[hh]) * a.stride + e0)
                      : make_uint4(0, 0, 0, 0);
      // candidate values of this chunk for the thread's vector, packed bf16 pairs
      uint32_t cand[kChunk][4];
      uint64_t w2[4];
      uint32_t bad = 0;
      if (active) {
        uint4 b = ld_row16(a.rows + (uint64_t)a.base_slot * a.stride + e0);
        const uint32_t bw[4] = {b.x, b.y, b.z, b.w};
        int leaf = find_leaf(a.leaves, a.nl, e0);
        float wgt[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const uint64_t e = e0 + j;
          while (leaf + 1 < (int)a.nl && __ldg(&a.leaves[leaf + 1].offset) <= e) ++leaf;
          const SearchLeaf* L = a.leaves + leaf;
          const bool in = e < a.len;
          const uint64_t km = __ldg(&L->key_mix);
          const uint64_t em = mix64((e - __ldg(&L->offset)) ^ 0xa0761d6478bd642full);
          const float sc = __ldg(&L->scale);
          wgt[j] = in ? __ldg(&L->weight) : 0.0f;
          const uint16_t v = (uint16_t)(bw[j >> 1] >> ((j & 1) * 16));
#pragma unroll
          for (int c = 0; c < kChunk; ++c) {
            uint16_t r = v;
            if (in && c0 + c < a.candidates) {
              r = bf16_seed(v, km, em, sc, seed[c], coef);
              if (!bf16_is_finite(r)) { bad |= 1u << c; r = v; }
            }
            if (j & 1) cand[c][j >> 1] |= (uint32_t)r << 16; else cand[c][j >> 1] = r;
          }
        }
#pragma unroll
        for (int p = 0; p < 4; ++p) w2[p] = f2_pack(wgt[2 * p], wgt[2 * p + 1]);
      } else {
#pragma unroll
        for (int c = 0; c < kChunk; ++c)
#pragma unroll
          for (int p = 0; p < 4; ++p) cand[c][p] = 0;
#pragma unroll
        for (int p = 0; p < 4; ++p) w2[p] = 0;
      }
      bad = __reduce_or_sync(0xffffffffu, bad);
      if (lane == 0 && bad) {
        for (int c = 0; c < kChunk; ++c)
          if ((bad >> c) & 1u) atomicOr(&a.invalid[c0 + c], 1u);
      }

      for (uint32_t h0 = 0; h0 < H; h0 += 2) {
        uint64_t acc[kChunk][2];
#pragma unroll
        for (int c = 0; c < kChunk; ++c) { acc[c][0] = 0; acc[c][1] = 0; }
        if (active) {
          const uint4 hv[2] = {nxt[0], nxt[1]};
          // next pair in flight during this pair's arithmetic
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            const uint32_t h = h0 + 2 + hh;
            nxt[hh] = h < H ? ld_row16(a.rows + (uint64_t)__ldg(&a.history_slots[h]) * a.stride + e0)
                            : make_uint4(0, 0, 0, 0);
          }
#pragma unroll
          for (int p = 0; p < 4; ++p) {
            uint64_t h2[2];
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
              const uint32_t word = p == 0 ? hv[hh].x : p == 1 ? hv[hh].y : p == 2 ? hv[hh].z : hv[hh].w;
              h2[hh] = bf2_to_f2(word);
            }
#pragma unroll
            for (int c = 0; c < kChunk; ++c) {
              const uint64_t c2 = bf2_to_f2(cand[c][p]);
#pragma unroll
              for (int hh = 0; hh < 2; ++hh) {
                const uint64_t d = f2_sub(c2, h2[hh]);
                acc[c][hh] = f2_fma(f2_mul(d, w2[p]), d, acc[c][hh]);
              }
            }
          }
        }
        float v[16];
#pragma unroll
        for (int c = 0; c < kChunk; ++c)
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            float lo, hi;
            f2_unpack(acc[c][hh], lo, hi);
            v[c * 2 + hh] = lo + hi;
          }
        const float s = xpose_reduce16(v, lane);
        if ((lane & 1) == 0) red[rbuf][warp][lane >> 1] = s;
        __syncthreads();
        if (tid < 16) {
          float t = 0.0f;
#pragma unroll
          for (int w = 0; w < kThreads / 32; ++w) t += red[rbuf][w][tid];
          const uint32_t h = h0 + (tid & 1);
          if (h < H) part_sum[c0 - g0 + (tid >> 1)][h] += t;
        }
        rbuf ^= 1;
      }
    }
    __syncthreads();
    for (int i = tid; i < kGroup * kMaxHistory; i += kThreads) {
      const uint32_t c = g0 + i / kMaxHistory, h = i % kMaxHistory;
      if (c < a.candidates && h < H)
        a.partials[((uint64_t)blockIdx.x * a.candidates + c) * a.hstride + h] = part_sum[i / kMaxHistory][h];
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// score + pick, one CTA per region
// ---------------------------------------------------------------------------
// draw_normal (cuda/kernels/src/lib.rs:316-343): two splitmix64 outputs ->
// Box-Muller in double precision.
__device__ double draw_normal(uint64_t seed, uint32_t index, uint32_t metric) {
  const uint64_t prime = 1000003ull;
  uint64_t base = (seed * prime + (uint64_t)index) * prime;
  uint64_t combined = base + (uint64_t)metric;
  uint64_t first = mix64(combined), second = mix64(combined ^ 0xd2b74407b1ce6e93ull);
  const double inv = 1.0 / 9007199254740992.0;
  double raw = (double)(first >> 11) * inv;
  double u1 = raw < 1.0e-12 ? 1.0e-12 : (raw > 1.0 - 1.0e-12 ? 1.0 - 1.0e-12 : raw);
  double u2 = (double)(second >> 11) * inv;
  return sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2);
}

// acquisition_score (cuda/kernels/src/bf16.rs:224-275) on one thread, same
// insertion order and float rounding.
__device__ float acquisition(const AskArgs& a, const float* dist, uint32_t H, uint32_t K, uint32_t candidate,
                             float* nd, uint32_t* ni) {
  for (uint32_t k = 0; k < K; ++k) { nd[k] = INFINITY; ni[k] = 0; }
  for (uint32_t o = 0; o < H; ++o) {
    float d = dist[o];
    uint32_t at = K;
    for (uint32_t k = 0; k < K; ++k)
      if (d < nd[k] || (d == nd[k] && o < ni[k])) { at = k; break; }
    if (at >= K) continue;
    for (uint32_t m = K - 1; m > at; --m) { nd[m] = nd[m - 1]; ni[m] = ni[m - 1]; }
    nd[at] = d;
    ni[at] = o;
  }
  float wsum = 0.0f, wval = 0.0f;
  for (uint32_t k = 0; k < K; ++k) {
    uint32_t idx = ni[k];
    float var = __fadd_rn(__fadd_rn(__fadd_rn(1.0e-9f, __fmul_rn(a.epistemic_scale, nd[k])), a.aleatoric_scale),
                          a.variances[idx]);
    float w = __fdiv_rn(1.0f, fmaxf(var, 1.0e-12f));
    wsum = __fadd_rn(wsum, w);
    wval = __fadd_rn(wval, __fmul_rn(w, a.outcomes[idx]));
  }
  float mean = __fdiv_rn(wval, fmaxf(wsum, 1.0e-12f));
  float se = __fmul_rn(__fsqrt_rn(__fdiv_rn(1.0f, fmaxf(wsum, 1.0e-12f))), a.y_scale);
  if (a.acquisition == 1) return __fadd_rn(mean, __fmul_rn(se, (float)draw_normal(a.draw_seed, candidate, 0)));
  if (a.acquisition == 2) return __fadd_rn(mean, se);
  return __fadd_rn(mean, __fmul_rn(a.beta, se));
}

__device__ __forceinline__ bool better(float s, uint32_t i, float bs, uint32_t bi) {
  return s > bs || (s == bs && i < bi);
}

// One CTA per candidate: the tile partials are summed by all threads in a
// fixed tree order (deterministic for a given history length), thread 0
// scores, and the last CTA of each region to finish -- found with an atomic
// ticket, nothing waits -- picks the region's best (pick_trial order: higher
// score, then lower index).
__global__ void __launch_bounds__(kThreads) search_score_pick_kernel(const __grid_constant__ AskArgs a) {
  __shared__ float red[kThreads];
  __shared__ float dist[kMaxHistory];
  __shared__ float nd[kMaxHistory];
  __shared__ uint32_t ni[kMaxHistory];
  __shared__ uint32_t last;
  const int tid = threadIdx.x;
  const uint32_t c = blockIdx.x;
  const uint32_t region = c / a.cpr;
  const uint32_t H = history_rows(a);
  const uint32_t K = min(a.neighbors, H);
  uint32_t hp = 1;
  while (hp < H) hp <<= 1;                  // history lanes (power of two <= 128)
  const uint32_t slices = kThreads / hp;    // >= 2
  const uint32_t h = tid % hp, sl = tid / hp;
  float s0 = 0.0f, s1 = 0.0f, s2 = 0.0f, s3 = 0.0f;
  if (h < H) {
    const float* p = a.partials + (uint64_t)c * a.hstride + h;
    const uint64_t step = (uint64_t)a.candidates * a.hstride;
    uint32_t t = sl;
    for (; t + 3 * slices < a.parts; t += 4 * slices) {
      s0 += __ldcg(p + (uint64_t)t * step);
      s1 += __ldcg(p + (uint64_t)(t + slices) * step);
      s2 += __ldcg(p + (uint64_t)(t + 2 * slices) * step);
      s3 += __ldcg(p + (uint64_t)(t + 3 * slices) * step);
    }
    for (; t < a.parts; t += slices) s0 += __ldcg(p + (uint64_t)t * step);
  }
  red[tid] = (s0 + s1) + (s2 + s3);
  __syncthreads();
  for (uint32_t half = slices / 2; half > 0; half >>= 1) {
    if (sl < half) red[tid] += red[tid + half * hp];
    __syncthreads();
  }
  if (tid < (int)H) {
    dist[tid] = red[tid];
    a.distances[(uint64_t)c * kMaxHistory + tid] = red[tid];
  }
  __syncthreads();
  if (tid == 0) {
    const float sc = (a.invalid[c] || !isfinite(dist[0])) ? -INFINITY : acquisition(a, dist, H, K, c, nd, ni);
    a.scores[c] = sc;
    __threadfence();
    const uint32_t ticket = atomicAdd(&a.region_done[region], 1u);
    last = ticket == a.cpr - 1;
  }
  __syncthreads();
  if (!last || tid >= 32) return;
  __threadfence();
  const uint32_t first = region * a.cpr, end = first + a.cpr;
  float bs = -INFINITY;
  uint32_t bi = 0xffffffffu;
  for (uint32_t q = first + tid; q < end; q += 32) {
    const float sq = __ldcg(&a.scores[q]);
    if (better(sq, q, bs, bi)) { bs = sq; bi = q; }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const float os = __shfl_xor_sync(0xffffffffu, bs, off);
    const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, off);
    if (better(os, oi, bs, bi)) { bs = os; bi = oi; }
  }
  if (tid == 0) {
    // all-NaN regions keep index 0xffffffff: the host check or the write
    // kernel treats it as invalid
    a.selection[region].index = bi;
    a.selection[region].score = bs;
    a.region_done[region] = 0;
  }
}

// ---------------------------------------------------------------------------
// materialise the selected candidates (write_bf16, lib.rs:2050-2130)
// ---------------------------------------------------------------------------
__device__ void materialise_vector(const AskArgs& a, uint32_t region, uint64_t e0, uint32_t pick, bool& invalid);

__global__ void __launch_bounds__(kThreads) search_write_kernel(const __grid_constant__ AskArgs a) {
  const uint32_t region = blockIdx.y;
  const uint64_t e0 = ((uint64_t)blockIdx.x * kThreads + threadIdx.x) * 8;
  const uint32_t pick = a.selection[region].index;
  bool invalid = (a.resident && a.state->status != 0) || pick >= a.candidates;
  if (e0 < a.len) materialise_vector(a, region, e0, pick, invalid);
  invalid = __any_sync(0xffffffffu, invalid);
  if ((threadIdx.x & 31) == 0 && invalid) atomicOr(&a.region_status[region], 1u);
}

__device__ void materialise_vector(const AskArgs& a, uint32_t region, uint64_t e0, uint32_t pick, bool& invalid) {
  const uint64_t seed = pick < a.candidates ? candidate_seed(a, pick) : 0;
  const float coef = step_coefficient(a);
  uint4 b = ld_row16(a.rows + (uint64_t)a.base_slot * a.stride + e0);
  uint32_t in[4] = {b.x, b.y, b.z, b.w}, out[4];
  int leaf = find_leaf(a.leaves, a.nl, e0);
  uint16_t* brow = a.batch + (uint64_t)region * a.len;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    uint64_t e = e0 + j;
    uint16_t v = (uint16_t)(in[j >> 1] >> ((j & 1) * 16));
    uint16_t r = v;
    if (e < a.len) {
      while (leaf + 1 < (int)a.nl && __ldg(&a.leaves[leaf + 1].offset) <= e) ++leaf;
      const SearchLeaf& L = a.leaves[leaf];
      r = bf16_seed(v, __ldg(&L.key_mix), mix64((e - __ldg(&L.offset)) ^ 0xa0761d6478bd642full), __ldg(&L.scale),
                    seed, coef);
      invalid |= !bf16_is_finite(r);
      brow[e] = r;
    }
    if (j & 1) out[j >> 1] |= (uint32_t)r << 16; else out[j >> 1] = r;
  }
  // rows beyond len stay as they were (zero padding), so a full vector store
  // writes back the base's padding values there
  *reinterpret_cast<uint4*>(a.rows_out + (uint64_t)a.trial_slots[region] * a.stride + e0) =
      make_uint4(out[0], out[1], out[2], out[3]);
}

// ---------------------------------------------------------------------------
// tell: bookkeeping on one thread, then the row copies as a grid pass
// ---------------------------------------------------------------------------
struct TellArgs {
  uint32_t* history_slots;
  float* outcomes;
  float* variances;
  SearchStateDev* state;
  ennx_b200_tell_summary* summary;
  uint32_t* accepted;
  const float* values;
  const float* trial_variances;
  const uint32_t* region_status;
  CopyPlan* plan;
  uint32_t trial_slots[kMaxPending];
  uint32_t trials;
  uint32_t capacity;
  uint32_t failure_tolerance;
};

// tell_bf16 + tell_validate / tell_history / tell_adapt
// (cuda/kernels/src/lib.rs:409-535, 2135-2258), same order of updates.
__global__ void search_tell_plan_kernel(const __grid_constant__ TellArgs t) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  uint32_t status = 0;
  for (uint32_t i = 0; i < t.trials; ++i) {
    float v = t.values[i], var = t.trial_variances[i];
    if (!isfinite(v) || !isfinite(var) || var < 0.0f) status = 1;
    t.accepted[i] = 0;
    status |= t.region_status[i];
  }
  SearchStateDev s = *t.state;
  CopyPlan* plan = t.plan;
  plan->valid = 0;
  // a history longer than this call's capacity cannot be extended in place
  if (s.history == 0 || s.history > t.capacity || t.capacity > (uint32_t)kMaxHistory) status |= 2;
  if (status != 0) {
    s.status = status;
    *t.state = s;
    *t.summary = ennx_b200_tell_summary{s.length, s.best, s.best_variance, s.history, s.restarts, 0u, status};
    return;
  }
  uint32_t best_slot = 0xffffffffu;
  for (uint32_t i = 0; i < t.trials; ++i) {
    float v = t.values[i], var = t.trial_variances[i];
    uint32_t slot = t.trial_slots[i];
    if (v > s.best) {
      s.best = v;
      s.best_variance = var;
      best_slot = slot;
      t.accepted[i] = 1;
    }
    uint32_t dest;
    if (s.history == t.capacity) {
      dest = t.history_slots[0];
      for (uint32_t k = 1; k < s.history; ++k) {
        t.history_slots[k - 1] = t.history_slots[k];
        t.outcomes[k - 1] = t.outcomes[k];
        t.variances[k - 1] = t.variances[k];
      }
      s.history -= 1;
    } else {
      dest = s.history + 1;
    }
    plan->src[i] = slot;
    plan->dst[i] = dest;
    t.history_slots[s.history] = dest;
    t.outcomes[s.history] = v;
    t.variances[s.history] = var;
    s.history += 1;
  }
  // tell_adapt
  double prev = s.trust_best;
  if (isfinite(prev)) {
    double scale = s.prev_obs >= 2 ? fmax(s.hist_max - s.hist_min, 1.0e-6) : 0.0;
    if ((double)s.best > prev + 1.0e-3 * scale) {
      s.successes += 1;
      s.failures = 0;
    } else {
      s.failures += 1;
      s.successes = 0;
    }
    if (s.successes >= 3) {
      s.length = fmin(s.length * 2.0, s.length_max);
      s.successes = 0;
    } else if (s.failures >= t.failure_tolerance) {
      s.length *= 0.5;
      s.failures = 0;
    }
  }
  s.trust_best = (double)s.best;
  for (uint32_t i = 0; i < t.trials; ++i) {
    double v = (double)t.values[i];
    s.hist_min = fmin(s.hist_min, v);
    s.hist_max = fmax(s.hist_max, v);
  }
  s.prev_obs += t.trials;
  uint32_t restarted = 0;
  if (s.length < s.length_min) {
    s.length = s.length_init;
    s.successes = 0;
    s.failures = 0;
    s.trust_best = -INFINITY;
    s.hist_min = INFINITY;
    s.hist_max = -INFINITY;
    s.history = 1;
    s.restarts += 1;
    t.history_slots[0] = 1;
    t.outcomes[0] = s.best;
    t.variances[0] = s.best_variance;
    restarted = 1;
  }
  s.status = 0;
  *t.state = s;
  *t.summary = ennx_b200_tell_summary{s.length, s.best, s.best_variance, s.history, s.restarts, restarted, 0u};
  plan->best_slot = best_slot;
  plan->restarted = restarted;
  plan->count = t.trials;
  plan->valid = 1;
}

// Per element: incumbent <- best trial; history slots <- trials; slot 1 <-
// incumbent on a restart.  The order per element is the reference's order
// over whole rows, so one pass over the elements does all copies.
__global__ void __launch_bounds__(kThreads) search_tell_copy_kernel(uint16_t* rows, uint64_t stride, uint64_t len,
                                                                    const CopyPlan* plan) {
  if (!plan->valid) return;
  const uint32_t best = plan->best_slot, restarted = plan->restarted, count = plan->count;
  const uint64_t vecs = (stride) / 8;  // whole 16-byte vectors per row (padding included)
  const uint64_t used = (len + 7) / 8;
  for (uint64_t v = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; v < used && v < vecs;
       v += (uint64_t)gridDim.x * blockDim.x) {
    uint4* r = reinterpret_cast<uint4*>(rows);
    uint64_t rs = stride / 8;
    if (best != 0xffffffffu) r[v] = r[(uint64_t)best * rs + v];
    for (uint32_t i = 0; i < count; ++i) r[(uint64_t)plan->dst[i] * rs + v] = r[(uint64_t)plan->src[i] * rs + v];
    if (restarted) r[rs + v] = r[v];
  }
}

}  // namespace
}  // namespace ennx

using namespace ennx;

struct ennx_b200_bf16_search {
  int device;
  cudaStream_t stream;
  size_t len, stride, slots;
  uint16_t* rows;
  uint16_t* batch;
  size_t batch_rows;
  SearchLeaf* leaves;
  uint32_t nl;
  uint32_t* history_slots;
  float* outcomes;
  float* variances;
  SearchStateDev* state;
  ennx_b200_tell_summary* summary;
  uint32_t* accepted;
  float* tell_values;
  float* tell_variances;
  uint32_t* region_status;
  CopyPlan* plan;
  ennx_b200_selection* selection;
  uint32_t* trial_slots;
  // per-ask scratch, grown on demand
  uint64_t* seeds;
  uint32_t* invalid;
  float* scores;
  float* distances;
  size_t cand_cap;
  float* partials;
  size_t partial_cap;
  // last ask
  uint32_t last_candidates;
  int initialized;
  // profiling
  int profiling;
  int have_profile;
  cudaEvent_t ev[4];
  float profile[4];
  cudaEvent_t handoff;
};

namespace {

int32_t dev_alloc(void** p, size_t bytes, const char* what) {
  ENNX_CUDA(cudaMalloc(p, bytes < 16 ? 16 : bytes), what);
  return ENNX_B200_OK;
}

void release(ennx_b200_bf16_search* h) {
  if (!h) return;
  void* ptrs[] = {h->rows,         h->batch,      h->leaves,    h->history_slots, h->outcomes,
                  h->variances,    h->state,      h->summary,   h->accepted,      h->tell_values,
                  h->tell_variances, h->region_status, h->plan, h->selection,     h->trial_slots,
                  h->seeds,        h->invalid,    h->scores,    h->distances,     h->partials};
  for (void* p : ptrs)
    if (p) cudaFree(p);
  for (int i = 0; i < 4; ++i)
    if (h->ev[i]) cudaEventDestroy(h->ev[i]);
  if (h->handoff) cudaEventDestroy(h->handoff);
  free(h);
}

// Calls run on the caller's current device, which must be the handle's.
int32_t check_handle(ennx_b200_bf16_search* h) {
  if (!h) return set_error(ENNX_B200_INVALID_ARGUMENT, "BF16 search handle is null");
  int d = -1;
  ENNX_CUDA(cudaGetDevice(&d), "cudaGetDevice");
  if (d != h->device)
    return set_error(ENNX_B200_INVALID_ARGUMENT, "BF16 search handle belongs to device %d, current device is %d",
                     h->device, d);
  return ENNX_B200_OK;
}

int32_t check_slot(const ennx_b200_bf16_search* h, size_t slot) {
  if (slot >= h->slots)
    return set_error(ENNX_B200_INVALID_ARGUMENT, "CUDA BF16 row slot %zu exceeds capacity %zu", slot, h->slots);
  return ENNX_B200_OK;
}

uint16_t* row_ptr(const ennx_b200_bf16_search* h, size_t slot) { return h->rows + slot * h->stride; }

int32_t grow_scratch(ennx_b200_bf16_search* h, size_t candidates, size_t partials) {
  if (candidates > h->cand_cap) {
    size_t cap = 1;
    while (cap < candidates) cap <<= 1;
    void* p[4] = {h->seeds, h->invalid, h->scores, h->distances};
    for (void* q : p)
      if (q) cudaFree(q);
    h->seeds = nullptr; h->invalid = nullptr; h->scores = nullptr; h->distances = nullptr;
    h->cand_cap = 0;
    ENNX_TRY(dev_alloc((void**)&h->seeds, cap * sizeof(uint64_t), "search seeds"));
    ENNX_TRY(dev_alloc((void**)&h->invalid, cap * sizeof(uint32_t), "search flags"));
    ENNX_TRY(dev_alloc((void**)&h->scores, cap * sizeof(float), "search scores"));
    ENNX_TRY(dev_alloc((void**)&h->distances, cap * kMaxHistory * sizeof(float), "search distances"));
    h->cand_cap = cap;
  }
  if (partials > h->partial_cap) {
    size_t cap = 1;
    while (cap < partials) cap <<= 1;
    if (h->partials) cudaFree(h->partials);
    h->partials = nullptr;
    h->partial_cap = 0;
    ENNX_TRY(dev_alloc((void**)&h->partials, cap * sizeof(float), "search partials"));
    h->partial_cap = cap;
  }
  return ENNX_B200_OK;
}

int32_t check_config(const ennx_b200_ask_config* c) {
  if (!c) return set_error(ENNX_B200_INVALID_ARGUMENT, "CUDA BF16 acquisition configuration is invalid");
  if (c->acquisition > 2 || !isfinite(c->epistemic_scale) || c->epistemic_scale < 0.0f ||
      !isfinite(c->aleatoric_scale) || c->aleatoric_scale < 0.0f || !isfinite(c->y_scale) || c->y_scale < 0.0f ||
      !isfinite(c->beta))
    return set_error(ENNX_B200_INVALID_ARGUMENT, "CUDA BF16 acquisition configuration is invalid");
  return ENNX_B200_OK;
}

// check_ask (bf16_search.rs:596-644) + the launch sequence of launch()
int32_t run_ask(ennx_b200_bf16_search* h, size_t base_slot, size_t history, const uint32_t* trial_slots,
                size_t regions, const uint64_t* seeds, size_t cpr, uint64_t seed_root, bool resident,
                float coefficient, uint64_t draw_seed, const ennx_b200_ask_config* config) {
  if (!h->initialized) return set_error(ENNX_B200_INVALID_ARGUMENT, "CUDA BF16 search state is not initialised");
  ENNX_TRY(check_slot(h, base_slot));
  if (history == 0 || history > (size_t)kMaxHistory)
    return set_error(ENNX_B200_INVALID_ARGUMENT, "CUDA BF16 history must contain 1..=%d rows", kMaxHistory);
  if (regions == 0 || cpr == 0 || !trial_slots)
    return set_error(ENNX_B200_INVALID_ARGUMENT, "CUDA BF16 search requires regions and candidates");
  if (regions > (size_t)kMaxPending)
    return set_error(ENNX_B200_INVALID_ARGUMENT, "CUDA BF16 search supports at most %d regions", kMaxPending);
  if (cpr > (size_t)UINT32_MAX / regions)
    return set_error(ENNX_B200_INVALID_ARGUMENT, "CUDA BF16 candidate count overflow");
  const size_t candidates = regions * cpr;
  if (!resident && !seeds) return set_error(ENNX_B200_INVALID_ARGUMENT, "CUDA BF16 seeds do not match the search shape");
  if (!config) return set_error(ENNX_B200_INVALID_ARGUMENT, "CUDA BF16 acquisition configuration is invalid");
  if (config->neighbors == 0 || config->neighbors > history)
    return set_error(ENNX_B200_INVALID_ARGUMENT, "CUDA BF16 neighbor count exceeds resident history");
  if (!isfinite(coefficient) || coefficient <= 0.0f)
    return set_error(ENNX_B200_INVALID_ARGUMENT, "CUDA BF16 perturbation coefficient must be positive");
  ENNX_TRY(check_config(config));
  for (size_t r = 0; r < regions; ++r) {
    ENNX_TRY(check_slot(h, trial_slots[r]));
    bool dup = trial_slots[r] == base_slot;
    for (size_t q = 0; q < r; ++q) dup |= trial_slots[q] == trial_slots[r];
    if (dup) return set_error(ENNX_B200_INVALID_ARGUMENT, "CUDA BF16 trial slots must be distinct from live rows");
  }
  const size_t tiles = (h->len + kTileElems - 1) / kTileElems;
  const size_t max_parts = (size_t)sm_count() * 4;
  const uint32_t parts = (uint32_t)(tiles < max_parts ? tiles : max_parts);
  const size_t hstride = resident ? (size_t)kMaxHistory : history;
  ENNX_TRY(grow_scratch(h, candidates, (size_t)parts * candidates * hstride));
  if (regions > h->batch_rows) {
    if (h->batch) cudaFree(h->batch);
    h->batch = nullptr;
    h->batch_rows = 0;
    ENNX_TRY(dev_alloc((void**)&h->batch, regions * h->len * sizeof(uint16_t), "search batch"));
    h->batch_rows = regions;
  }
  cudaStream_t s = h->stream;
  if (!resident)
    ENNX_CUDA(cudaMemcpyAsync(h->seeds, seeds, candidates * sizeof(uint64_t), cudaMemcpyHostToDevice, s), "seeds");
  // trial slots ride in the argument block of the kernels; the device copy
  // serves the tell of this round
  ENNX_CUDA(cudaMemcpyAsync(h->trial_slots, trial_slots, regions * sizeof(uint32_t), cudaMemcpyHostToDevice, s),
            "trial slots");
  ENNX_CUDA(cudaMemsetAsync(h->invalid, 0, candidates * sizeof(uint32_t), s), "flags");
  // region status words and the score kernel's tickets
  ENNX_CUDA(cudaMemsetAsync(h->region_status, 0, 2 * kMaxPending * sizeof(uint32_t), s), "status");

  AskArgs a;
  memset(&a, 0, sizeof(a));
  a.rows = h->rows;
  a.stride = h->stride;
  a.len = h->len;
  a.base_slot = (uint32_t)base_slot;
  a.history = (uint32_t)history;
  a.hstride = (uint32_t)hstride;
  a.candidates = (uint32_t)candidates;
  a.cpr = (uint32_t)cpr;
  a.regions = (uint32_t)regions;
  a.parts = parts;
  a.nl = h->nl;
  a.neighbors = config->neighbors;
  a.acquisition = config->acquisition;
  a.resident = resident ? 1 : 0;
  a.coefficient = coefficient;
  a.epistemic_scale = config->epistemic_scale;
  a.aleatoric_scale = config->aleatoric_scale;
  a.y_scale = config->y_scale;
  a.beta = config->beta;
  a.seed_root = seed_root;
  a.draw_seed = draw_seed;
  a.seeds = h->seeds;
  a.leaves = h->leaves;
  a.history_slots = h->history_slots;
  a.outcomes = h->outcomes;
  a.variances = h->variances;
  a.state = h->state;
  a.partials = h->partials;
  a.invalid = h->invalid;
  a.distances = h->distances;
  a.scores = h->scores;
  a.selection = h->selection;
  a.trial_slots = h->trial_slots;
  a.rows_out = h->rows;
  a.batch = h->batch;
  a.region_status = h->region_status;
  a.region_done = h->region_status + kMaxPending;

  if (h->profiling) ENNX_CUDA(cudaEventRecord(h->ev[0], s), "event");
  search_distance_kernel<<<parts, kThreads, 0, s>>>(a);
  ENNX_LAUNCH_CHECK("search_distance launch");
  search_score_pick_kernel<<<(unsigned)candidates, kThreads, 0, s>>>(a);
  ENNX_LAUNCH_CHECK("search_score_pick launch");
  if (h->profiling) ENNX_CUDA(cudaEventRecord(h->ev[1], s), "event");
  dim3 wgrid((unsigned)((h->len + kTileElems - 1) / kTileElems), (unsigned)regions);
  search_write_kernel<<<wgrid, kThreads, 0, s>>>(a);
  ENNX_LAUNCH_CHECK("search_write launch");
  if (h->profiling) {
    ENNX_CUDA(cudaEventRecord(h->ev[2], s), "event");
    ENNX_CUDA(cudaEventSynchronize(h->ev[2]), "event");
    float score = 0.0f, write = 0.0f;
    ENNX_CUDA(cudaEventElapsedTime(&score, h->ev[0], h->ev[1]), "event");
    ENNX_CUDA(cudaEventElapsedTime(&write, h->ev[1], h->ev[2]), "event");
    h->profile[0] = score;  // distances + score + pick (one fused launch pair)
    h->profile[1] = 0.0f;   // pick runs inside the score launch
    h->profile[2] = write;
    h->profile[3] = score + write;
    h->have_profile = 1;
  } else {
    h->have_profile = 0;
  }
  h->last_candidates = (uint32_t)candidates;
  return ENNX_B200_OK;
}

int32_t copy_rows(ennx_b200_bf16_search* h, size_t src, size_t dst) {
  if (src == dst) return ENNX_B200_OK;
  ENNX_CUDA(cudaMemcpyAsync(row_ptr(h, dst), row_ptr(h, src), h->len * sizeof(uint16_t), cudaMemcpyDeviceToDevice,
                            h->stream),
            "row copy");
  return ENNX_B200_OK;
}

}  // namespace

extern "C" {

int32_t ennx_b200_bf16_search_create(const uint16_t* base, size_t len, const ennx_b200_bf16_leaf* leaves,
                                     size_t nl, size_t slots, void* stream, ennx_b200_bf16_search** out) {
  if (!out) return set_error(ENNX_B200_INVALID_ARGUMENT, "BF16 search output handle is null");
  *out = nullptr;
  if (!base) return set_error(ENNX_B200_INVALID_ARGUMENT, "CUDA BF16 search requires a device base");
  if (len == 0 || !leaves || nl == 0)
    return set_error(ENNX_B200_INVALID_ARGUMENT, "CUDA BF16 search requires base values and leaves");
  if (slots < 2) return set_error(ENNX_B200_INVALID_ARGUMENT, "CUDA BF16 search requires at least two row slots");
  if (nl > UINT32_MAX) return set_error(ENNX_B200_INVALID_ARGUMENT, "CUDA BF16 leaf count exceeds u32");
  uint64_t expected = 0;
  for (size_t i = 0; i < nl; ++i) {
    if (leaves[i].offset != expected || leaves[i].length == 0)
      return set_error(ENNX_B200_INVALID_ARGUMENT, "CUDA BF16 leaves must form a contiguous non-empty layout");
    if (!isfinite(leaves[i].scale) || leaves[i].scale <= 0.0f || !isfinite(leaves[i].weight) ||
        leaves[i].weight <= 0.0f)
      return set_error(ENNX_B200_INVALID_ARGUMENT, "CUDA BF16 leaf scales and weights must be positive");
    if (leaves[i].length > UINT32_MAX) return set_error(ENNX_B200_INVALID_ARGUMENT, "CUDA BF16 leaf length exceeds u32");
    expected += leaves[i].length;
  }
  if (expected != (uint64_t)len)
    return set_error(ENNX_B200_INVALID_ARGUMENT, "CUDA BF16 leaf layout covers %llu values, expected %zu",
                     (unsigned long long)expected, len);
  ennx_b200_bf16_search* h = (ennx_b200_bf16_search*)calloc(1, sizeof(ennx_b200_bf16_search));
  if (!h) return set_error(ENNX_B200_CUDA_ERROR, "out of host memory");
  int32_t st = ENNX_B200_OK;
  do {
    if (cudaGetDevice(&h->device) != cudaSuccess) { st = set_error(ENNX_B200_CUDA_ERROR, "cudaGetDevice failed"); break; }
    h->stream = (cudaStream_t)stream;
    h->len = len;
    h->stride = (len + 127) & ~(size_t)127;
    h->slots = slots;
    if ((st = dev_alloc((void**)&h->rows, slots * h->stride * sizeof(uint16_t), "search rows"))) break;
    if (cudaMemsetAsync(h->rows, 0, slots * h->stride * sizeof(uint16_t), h->stream) != cudaSuccess) {
      st = set_error(ENNX_B200_CUDA_ERROR, "row clear failed");
      break;
    }
    SearchLeaf* host = (SearchLeaf*)malloc(nl * sizeof(SearchLeaf));
    if (!host) { st = set_error(ENNX_B200_CUDA_ERROR, "out of host memory"); break; }
    for (size_t i = 0; i < nl; ++i)
      host[i] = SearchLeaf{mix64(leaves[i].key ^ 0xd6e8feb86659fd93ull), leaves[i].offset, leaves[i].length,
                           leaves[i].scale, leaves[i].weight};
    h->nl = (uint32_t)nl;
    if ((st = dev_alloc((void**)&h->leaves, nl * sizeof(SearchLeaf), "search leaves"))) { free(host); break; }
    cudaError_t e = cudaMemcpyAsync(h->leaves, host, nl * sizeof(SearchLeaf), cudaMemcpyHostToDevice, h->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(h->stream);
    free(host);
    if (e != cudaSuccess) { st = check_cuda(e, "leaf upload"); break; }
    if ((st = dev_alloc((void**)&h->history_slots, kMaxHistory * sizeof(uint32_t), "history"))) break;
    if ((st = dev_alloc((void**)&h->outcomes, kMaxHistory * sizeof(float), "history"))) break;
    if ((st = dev_alloc((void**)&h->variances, kMaxHistory * sizeof(float), "history"))) break;
    if ((st = dev_alloc((void**)&h->state, sizeof(SearchStateDev), "state"))) break;
    if ((st = dev_alloc((void**)&h->summary, sizeof(ennx_b200_tell_summary), "summary"))) break;
    if ((st = dev_alloc((void**)&h->accepted, kMaxPending * sizeof(uint32_t), "accepted"))) break;
    if ((st = dev_alloc((void**)&h->tell_values, kMaxPending * sizeof(float), "tell values"))) break;
    if ((st = dev_alloc((void**)&h->tell_variances, kMaxPending * sizeof(float), "tell variances"))) break;
    if ((st = dev_alloc((void**)&h->region_status, 2 * kMaxPending * sizeof(uint32_t), "status"))) break;
    if ((st = dev_alloc((void**)&h->plan, sizeof(CopyPlan), "plan"))) break;
    if ((st = dev_alloc((void**)&h->selection, kMaxPending * sizeof(ennx_b200_selection), "selection"))) break;
    if ((st = dev_alloc((void**)&h->trial_slots, kMaxPending * sizeof(uint32_t), "trial slots"))) break;
    e = cudaMemsetAsync(h->state, 0, sizeof(SearchStateDev), h->stream);
    if (e == cudaSuccess) e = cudaMemsetAsync(h->region_status, 0, 2 * kMaxPending * sizeof(uint32_t), h->stream);
    if (e == cudaSuccess) e = cudaMemsetAsync(h->plan, 0, sizeof(CopyPlan), h->stream);
    if (e == cudaSuccess)
      e = cudaMemcpyAsync(h->rows, base, len * sizeof(uint16_t), cudaMemcpyDeviceToDevice, h->stream);
    if (e != cudaSuccess) { st = check_cuda(e, "search init"); break; }
    for (int i = 0; i < 4 && st == ENNX_B200_OK; ++i)
      if (cudaEventCreate(&h->ev[i]) != cudaSuccess) st = set_error(ENNX_B200_CUDA_ERROR, "event create failed");
    if (st) break;
    if (cudaEventCreateWithFlags(&h->handoff, cudaEventDisableTiming) != cudaSuccess) {
      st = set_error(ENNX_B200_CUDA_ERROR, "event create failed");
      break;
    }
    int32_t finite = 0;
    if ((st = ennx_b200_check_bf16(h->rows, len, &finite, h->stream))) break;
    if (!finite) { st = set_error(ENNX_B200_INVALID_ARGUMENT, "CUDA BF16 search base values must be finite"); break; }
  } while (0);
  if (st != ENNX_B200_OK) {
    cudaStreamSynchronize((cudaStream_t)stream);
    release(h);
    return st;
  }
  *out = h;
  return ENNX_B200_OK;
}

int32_t ennx_b200_bf16_search_destroy(ennx_b200_bf16_search* h) {
  if (!h) return ENNX_B200_OK;
  int prev = -1;
  cudaGetDevice(&prev);
  cudaSetDevice(h->device);
  cudaStreamSynchronize(h->stream);
  release(h);
  if (prev >= 0) cudaSetDevice(prev);
  return ENNX_B200_OK;
}

int32_t ennx_b200_bf16_search_init(ennx_b200_bf16_search* h, float base_value, float base_variance,
                                   size_t capacity, double length_init, double length_min, double length_max) {
  ENNX_TRY(check_handle(h));
  if (capacity == 0 || capacity > (size_t)kMaxHistory || !isfinite(base_value) || !isfinite(base_variance) ||
      base_variance < 0.0f || !isfinite(length_init) || !isfinite(length_min) || !isfinite(length_max) ||
      length_min <= 0.0 || length_init < length_min || length_init > length_max)
    return set_error(ENNX_B200_INVALID_ARGUMENT, "CUDA BF16 search state is invalid");
  if (capacity + 1 > h->slots)
    return set_error(ENNX_B200_INVALID_ARGUMENT, "CUDA BF16 history capacity exceeds the row slots");
  SearchStateDev s;
  memset(&s, 0, sizeof(s));
  s.length = length_init;
  s.length_init = length_init;
  s.length_min = length_min;
  s.length_max = length_max;
  s.best = base_value;
  s.best_variance = base_variance;
  s.trust_best = (double)base_value;
  s.hist_min = (double)base_value;
  s.hist_max = (double)base_value;
  s.prev_obs = 1;
  s.history = 1;
  uint32_t one = 1;
  // pageable sources: the copies complete before these calls return
  ENNX_CUDA(cudaMemcpyAsync(h->history_slots, &one, sizeof(one), cudaMemcpyHostToDevice, h->stream), "init");
  ENNX_CUDA(cudaMemcpyAsync(h->outcomes, &base_value, sizeof(float), cudaMemcpyHostToDevice, h->stream), "init");
  ENNX_CUDA(cudaMemcpyAsync(h->variances, &base_variance, sizeof(float), cudaMemcpyHostToDevice, h->stream), "init");
  ENNX_CUDA(cudaMemcpyAsync(h->state, &s, sizeof(s), cudaMemcpyHostToDevice, h->stream), "init");
  ENNX_CUDA(cudaStreamSynchronize(h->stream), "init");
  h->initialized = 1;
  return ENNX_B200_OK;
}

int32_t ennx_b200_bf16_search_copy_row(ennx_b200_bf16_search* h, size_t source, size_t destination) {
  ENNX_TRY(check_handle(h));
  ENNX_TRY(check_slot(h, source));
  ENNX_TRY(check_slot(h, destination));
  return copy_rows(h, source, destination);
}

int32_t ennx_b200_bf16_search_ask(ennx_b200_bf16_search* h, size_t base_slot, size_t history,
                                  const uint32_t* trial_slots, size_t regions, const uint64_t* seeds, size_t cpr,
                                  float coefficient, uint64_t draw_seed, const ennx_b200_ask_config* config,
                                  ennx_b200_selection* selections) {
  ENNX_TRY(check_handle(h));
  if (!selections) return set_error(ENNX_B200_INVALID_ARGUMENT, "BF16 ask needs a selection output");
  ENNX_TRY(run_ask(h, base_slot, history, trial_slots, regions, seeds, cpr, 0, false, coefficient, draw_seed, config));
  uint32_t status[kMaxPending];
  ENNX_CUDA(cudaMemcpyAsync(selections, h->selection, regions * sizeof(ennx_b200_selection), cudaMemcpyDeviceToHost,
                            h->stream),
            "selection read");
  ENNX_CUDA(cudaMemcpyAsync(status, h->region_status, regions * sizeof(uint32_t), cudaMemcpyDeviceToHost, h->stream),
            "status read");
  ENNX_CUDA(cudaStreamSynchronize(h->stream), "ask");
  // collect (bf16_search.rs:868-887): index inside its region, no overflow
  for (size_t r = 0; r < regions; ++r) {
    size_t first = r * cpr, end = first + cpr;
    if (selections[r].index < first || selections[r].index >= end) {
      for (size_t q = 0; q < regions; ++q) ENNX_TRY(copy_rows(h, base_slot, trial_slots[q]));
      ENNX_CUDA(cudaStreamSynchronize(h->stream), "reset");
      return set_error(ENNX_B200_INVALID_ARGUMENT, "CUDA BF16 region %zu selected invalid trial index %u", r,
                       selections[r].index);
    }
  }
  for (size_t r = 0; r < regions; ++r)
    if (status[r]) {
      for (size_t q = 0; q < regions; ++q) ENNX_TRY(copy_rows(h, base_slot, trial_slots[q]));
      ENNX_CUDA(cudaStreamSynchronize(h->stream), "reset");
      return set_error(ENNX_B200_OVERFLOW, "CUDA BF16 search perturbation overflowed FP32");
    }
  return ENNX_B200_OK;
}

int32_t ennx_b200_bf16_search_ask_seeded(ennx_b200_bf16_search* h, size_t base_slot, const uint32_t* trial_slots,
                                         size_t regions, size_t cpr, uint64_t seed_root, uint64_t draw_seed,
                                         const ennx_b200_ask_config* config) {
  ENNX_TRY(check_handle(h));
  return run_ask(h, base_slot, kMaxHistory, trial_slots, regions, nullptr, cpr, seed_root, true, 1.0f, draw_seed,
                 config);
}

int32_t ennx_b200_bf16_search_tell(ennx_b200_bf16_search* h, const uint32_t* trial_slots, size_t count,
                                   const float* values, const float* variances, int32_t on_device, size_t capacity,
                                   size_t failure_tolerance) {
  ENNX_TRY(check_handle(h));
  if (!trial_slots || count == 0 || count > (size_t)kMaxPending || capacity == 0 || capacity > (size_t)kMaxHistory)
    return set_error(ENNX_B200_INVALID_ARGUMENT, "CUDA BF16 tell shape is invalid");
  if (!values) return set_error(ENNX_B200_INVALID_ARGUMENT, "CUDA BF16 tell requires valid device rewards");
  if (!h->initialized) return set_error(ENNX_B200_INVALID_ARGUMENT, "CUDA BF16 search state is not initialised");
  for (size_t i = 0; i < count; ++i) ENNX_TRY(check_slot(h, trial_slots[i]));
  cudaStream_t s = h->stream;
  cudaMemcpyKind kind = on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice;
  ENNX_CUDA(cudaMemcpyAsync(h->tell_values, values, count * sizeof(float), kind, s), "tell values");
  if (variances)
    ENNX_CUDA(cudaMemcpyAsync(h->tell_variances, variances, count * sizeof(float), kind, s), "tell variances");
  else
    ENNX_CUDA(cudaMemsetAsync(h->tell_variances, 0, count * sizeof(float), s), "tell variances");
  TellArgs t;
  memset(&t, 0, sizeof(t));
  t.history_slots = h->history_slots;
  t.outcomes = h->outcomes;
  t.variances = h->variances;
  t.state = h->state;
  t.summary = h->summary;
  t.accepted = h->accepted;
  t.values = h->tell_values;
  t.trial_variances = h->tell_variances;
  t.region_status = h->region_status;
  t.plan = h->plan;
  for (size_t i = 0; i < count; ++i) t.trial_slots[i] = trial_slots[i];
  t.trials = (uint32_t)count;
  t.capacity = (uint32_t)capacity;
  t.failure_tolerance = (uint32_t)(failure_tolerance > UINT32_MAX ? UINT32_MAX : (failure_tolerance ? failure_tolerance : 1));
  search_tell_plan_kernel<<<1, 32, 0, s>>>(t);
  ENNX_LAUNCH_CHECK("search_tell_plan launch");
  size_t vecs = (h->len + 7) / 8;
  unsigned blocks = (unsigned)((vecs + kThreads - 1) / kThreads);
  unsigned cap = (unsigned)sm_count() * 4;
  if (blocks > cap) blocks = cap;
  if (blocks == 0) blocks = 1;
  search_tell_copy_kernel<<<blocks, kThreads, 0, s>>>(h->rows, h->stride, h->len, h->plan);
  ENNX_LAUNCH_CHECK("search_tell_copy launch");
  // the proposals of this round are consumed
  ENNX_CUDA(cudaMemsetAsync(h->region_status, 0, kMaxPending * sizeof(uint32_t), s), "status");
  return ENNX_B200_OK;
}

int32_t ennx_b200_bf16_search_collect(ennx_b200_bf16_search* h, size_t count, uint8_t* accepted,
                                      ennx_b200_tell_summary* summary) {
  ENNX_TRY(check_handle(h));
  if (count == 0 || count > (size_t)kMaxPending || !summary)
    return set_error(ENNX_B200_INVALID_ARGUMENT, "CUDA BF16 summary count is invalid");
  uint32_t acc[kMaxPending];
  ENNX_CUDA(cudaMemcpyAsync(summary, h->summary, sizeof(*summary), cudaMemcpyDeviceToHost, h->stream), "summary");
  ENNX_CUDA(cudaMemcpyAsync(acc, h->accepted, count * sizeof(uint32_t), cudaMemcpyDeviceToHost, h->stream), "accepted");
  ENNX_CUDA(cudaStreamSynchronize(h->stream), "collect");
  if (summary->status != 0) return set_error(ENNX_B200_INVALID_ARGUMENT, "CUDA BF16 proposal or rewards are invalid");
  if (accepted)
    for (size_t i = 0; i < count; ++i) accepted[i] = acc[i] ? 1 : 0;
  return ENNX_B200_OK;
}

int32_t ennx_b200_bf16_search_row(ennx_b200_bf16_search* h, size_t slot, const uint16_t** row) {
  ENNX_TRY(check_handle(h));
  ENNX_TRY(check_slot(h, slot));
  if (!row) return set_error(ENNX_B200_INVALID_ARGUMENT, "BF16 row output is null");
  *row = row_ptr(h, slot);
  return ENNX_B200_OK;
}

int32_t ennx_b200_bf16_search_round(ennx_b200_bf16_search* h, size_t rows, const uint16_t** batch) {
  ENNX_TRY(check_handle(h));
  if (!batch || rows == 0 || rows > h->batch_rows)
    return set_error(ENNX_B200_INVALID_ARGUMENT, "CUDA BF16 round shape is invalid");
  *batch = h->batch;
  return ENNX_B200_OK;
}

int32_t ennx_b200_bf16_search_gather(ennx_b200_bf16_search* h, const uint32_t* slots, size_t count,
                                     const uint16_t** batch) {
  ENNX_TRY(check_handle(h));
  if (!slots || !batch || count == 0 || count > (size_t)kMaxPending)
    return set_error(ENNX_B200_INVALID_ARGUMENT, "CUDA BF16 batch shape is invalid");
  for (size_t i = 0; i < count; ++i) ENNX_TRY(check_slot(h, slots[i]));
  if (count > h->batch_rows) {
    ENNX_CUDA(cudaStreamSynchronize(h->stream), "batch");
    if (h->batch) cudaFree(h->batch);
    h->batch = nullptr;
    h->batch_rows = 0;
    ENNX_TRY(dev_alloc((void**)&h->batch, count * h->len * sizeof(uint16_t), "search batch"));
    h->batch_rows = count;
  }
  for (size_t i = 0; i < count; ++i)
    ENNX_CUDA(cudaMemcpyAsync(h->batch + i * h->len, row_ptr(h, slots[i]), h->len * sizeof(uint16_t),
                              cudaMemcpyDeviceToDevice, h->stream),
              "batch gather");
  *batch = h->batch;
  return ENNX_B200_OK;
}

int32_t ennx_b200_bf16_search_handoff(ennx_b200_bf16_search* h, void* consumer, int32_t mode) {
  ENNX_TRY(check_handle(h));
  if (mode == 0) {
    ENNX_CUDA(cudaStreamSynchronize(h->stream), "handoff");
  } else if (mode == 2) {
    ENNX_CUDA(cudaEventRecord(h->handoff, h->stream), "handoff");
    ENNX_CUDA(cudaStreamWaitEvent((cudaStream_t)consumer, h->handoff, 0), "handoff");
  } else if (mode != 1) {
    return set_error(ENNX_B200_INVALID_ARGUMENT, "invalid stream hand-off mode %d", mode);
  }
  return ENNX_B200_OK;
}

int32_t ennx_b200_bf16_search_last_scores(ennx_b200_bf16_search* h, float* scores, size_t ns, float* distances,
                                          size_t nd) {
  ENNX_TRY(check_handle(h));
  size_t c = h->last_candidates;
  if (ns > c || nd > c * (size_t)kMaxHistory)
    return set_error(ENNX_B200_INVALID_ARGUMENT, "the last ask scored %zu candidates", c);
  if (scores && ns)
    ENNX_CUDA(cudaMemcpyAsync(scores, h->scores, ns * sizeof(float), cudaMemcpyDeviceToHost, h->stream), "scores");
  if (distances && nd)
    ENNX_CUDA(cudaMemcpyAsync(distances, h->distances, nd * sizeof(float), cudaMemcpyDeviceToHost, h->stream),
              "distances");
  ENNX_CUDA(cudaStreamSynchronize(h->stream), "scores");
  return ENNX_B200_OK;
}

int32_t ennx_b200_bf16_search_set_profiling(ennx_b200_bf16_search* h, int32_t enabled) {
  ENNX_TRY(check_handle(h));
  h->profiling = enabled ? 1 : 0;
  if (!enabled) h->have_profile = 0;
  return ENNX_B200_OK;
}

int32_t ennx_b200_bf16_search_last_profile(ennx_b200_bf16_search* h, float* out, int32_t* available) {
  ENNX_TRY(check_handle(h));
  if (!out || !available) return set_error(ENNX_B200_INVALID_ARGUMENT, "profile output is null");
  *available = h->have_profile;
  for (int i = 0; i < 4; ++i) out[i] = h->have_profile ? h->profile[i] : 0.0f;
  return ENNX_B200_OK;
}

}  // extern "C"
