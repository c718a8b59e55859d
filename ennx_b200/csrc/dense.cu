// dense.cu -- seeded dense perturbation (fp32 and BF16), finiteness check,
// fused perturbed GEMV and the Philox population noise generator.
//
// Bit-exact restatements of rust/crates/ennx/src/dense.rs:361-433 (fp32),
// dense/bf16.rs:228-292 and cuda/kernels/src/bf16.rs:91-158 (BF16), and
// cuda/kernels/src/lib.rs:308-406 (device copies).  Every add and multiply of
// the perturbation uses the round-to-nearest intrinsics so that nvcc cannot
// contract "value + scale*sum" into an FMA: the reference rounds twice.
#include <string.h>

#include "common.cuh"
#include "kernels.cuh"

namespace ennx {
namespace {

struct DevLeaf {  // leaf with its key pre-mixed (mix64(key ^ K) is per-leaf)
  uint64_t key_mix;
  uint64_t offset;
  uint64_t len;
  float scale;
  uint32_t pad;
};
struct DevTerm {
  uint64_t seed;
  float coefficient;
  uint32_t pad;
};

// dense.rs:367-379: sum of c*sign and the dominant term's direction.
__device__ __forceinline__ float term_sum(const DevTerm* terms, int nt, uint64_t key_mix, uint64_t element,
                                          bool& positive) {
  uint64_t emix = mix64(element ^ 0xa0761d6478bd642full);
  float sum = 0.0f, strongest = 0.0f;
  positive = true;
  for (int t = 0; t < nt; ++t) {
    float c = terms[t].coefficient;
    if (c == 0.0f) continue;
    float dir = (mix64(terms[t].seed ^ key_mix ^ emix) & 1ull) ? 1.0f : -1.0f;
    sum = __fadd_rn(sum, __fmul_rn(c, dir));
    if (fabsf(c) > strongest) {
      strongest = fabsf(c);
      positive = (c > 0.0f) == (dir > 0.0f);
    }
  }
  return sum;
}

__device__ __forceinline__ float dense_next(float value, bool positive) {
  if (value == 0.0f) return __uint_as_float(positive ? 1u : 0x80000001u);
  bool grows = (value > 0.0f) == positive;
  uint32_t b = __float_as_uint(value);
  float cand = __uint_as_float(grows ? b + 1u : b - 1u);
  if (isfinite(cand)) return cand;
  return __uint_as_float(grows ? b - 1u : b + 1u);
}

// Leaf lookup by binary search over the (contiguous) leaf offsets.
__device__ __forceinline__ int find_leaf(const DevLeaf* leaves, int nl, uint64_t i) {
  int lo = 0, hi = nl - 1;
  while (lo < hi) {
    int mid = (lo + hi + 1) >> 1;
    if (leaves[mid].offset <= i) lo = mid; else hi = mid - 1;
  }
  return lo;
}

constexpr int kMaxSmemLeaves = 256;
constexpr int kMaxSmemTerms = 128;

template <typename T>
__device__ __forceinline__ void stage_to_smem(T* dst, const T* src, int n) {
  for (int i = threadIdx.x; i < n; i += blockDim.x) dst[i] = src[i];
}

__global__ void apply_dense_f32_kernel(const float* __restrict__ base, float* __restrict__ out, uint64_t n,
                                       const DevLeaf* __restrict__ gleaves, int nl,
                                       const DevTerm* __restrict__ gterms, int nt, int* bad) {
  __shared__ DevLeaf leaves[kMaxSmemLeaves];
  __shared__ DevTerm terms[kMaxSmemTerms];
  stage_to_smem(leaves, gleaves, nl);
  stage_to_smem(terms, gterms, nt);
  __syncthreads();
  int invalid = 0;
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x) {
    const DevLeaf& L = leaves[find_leaf(leaves, nl, i)];
    uint64_t local = i - L.offset;
    bool positive;
    float sum = term_sum(terms, nt, L.key_mix, local, positive);
    float v = base[i];
    float cand = __fadd_rn(v, __fmul_rn(L.scale, sum));
    float r = (sum == 0.0f || cand == v) ? dense_next(v, positive) : cand;
    invalid |= !isfinite(r);
    out[i] = r;
  }
  if (__syncthreads_or(invalid) && threadIdx.x == 0) atomicOr(bad, 1);
}

__global__ void apply_dense_bf16_kernel(const uint16_t* __restrict__ base, uint16_t* __restrict__ out,
                                        uint64_t n, const DevLeaf* __restrict__ gleaves, int nl,
                                        const DevTerm* __restrict__ gterms, int nt, int* bad) {
  __shared__ DevLeaf leaves[kMaxSmemLeaves];
  __shared__ DevTerm terms[kMaxSmemTerms];
  stage_to_smem(leaves, gleaves, nl);
  stage_to_smem(terms, gterms, nt);
  __syncthreads();
  int invalid = 0;
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x) {
    const DevLeaf& L = leaves[find_leaf(leaves, nl, i)];
    uint64_t local = i - L.offset;
    bool positive;
    float sum = term_sum(terms, nt, L.key_mix, local, positive);
    uint16_t v = base[i];
    uint16_t cand = f32_to_bf16_rne(__fadd_rn(bf16_to_f32(v), __fmul_rn(L.scale, sum)));
    uint16_t r = (sum == 0.0f || cand == v) ? bf16_next(v, positive) : cand;
    invalid |= ((r & 0x7f80u) == 0x7f80u);  // bf16_finite, kernels bf16.rs:96-99
    out[i] = r;
  }
  if (__syncthreads_or(invalid) && threadIdx.x == 0) atomicOr(bad, 1);
}

__global__ void check_bf16_kernel(const uint16_t* __restrict__ v, uint64_t n, int* bad) {
  int invalid = 0;
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x)
    invalid |= ((v[i] & 0x7f80u) == 0x7f80u);
  if (__syncthreads_or(invalid) && threadIdx.x == 0) atomicOr(bad, 1);
}

// One block per output row (cuda/kernels/src/lib.rs:2359-2423): each thread
// runs an fma chain over its strided columns, then warp and block reduction.
__global__ void dense_linear_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                    const float* __restrict__ bias, float* __restrict__ out, uint64_t columns,
                                    uint64_t rows, DevLeaf wv, DevLeaf bv, const DevTerm* __restrict__ gterms,
                                    int nt) {
  __shared__ DevTerm terms[kMaxSmemTerms];
  __shared__ float warp_sums[32];
  stage_to_smem(terms, gterms, nt);
  __syncthreads();
  uint64_t row = blockIdx.x;
  if (row >= rows) return;
  float sum = 0.0f;
  uint64_t start = row * columns;
  for (uint64_t c = threadIdx.x; c < columns; c += blockDim.x) {
    uint64_t idx = start + c;
    bool positive;
    float s = term_sum(terms, nt, wv.key_mix, wv.offset + idx, positive);
    float v = w[idx];
    float cand = __fadd_rn(v, __fmul_rn(wv.scale, s));
    float pw = (s == 0.0f || cand == v) ? dense_next(v, positive) : cand;
    sum = __fmaf_rn(x[c], pw, sum);
  }
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) warp_sums[warp] = sum;
  __syncthreads();
  if (warp == 0) {
    float t = lane < (int)(blockDim.x >> 5) ? warp_sums[lane] : 0.0f;
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (lane == 0) {
      if (bias) {
        bool positive;
        float s = term_sum(terms, nt, bv.key_mix, bv.offset + row, positive);
        float v = bias[row];
        float cand = __fadd_rn(v, __fmul_rn(bv.scale, s));
        t += (s == 0.0f || cand == v) ? dense_next(v, positive) : cand;
      }
      out[row] = t;
    }
  }
}

// Population noise: each thread owns 8 consecutive elements (one Philox
// block) per step, 16-byte loads and stores.  The noise step is
// e = bf16(sigma * z) (RNE) and the perturbed weights are W +/- e, each
// rounded once (RNE of the exact sum) -- the same values the perturbed GEMM
// forms in its operand path from W and e.  With w == nullptr only e is
// written (to `plus`): the noise operand of that GEMM.  Blocks of 128 threads cover a fixed 4096-element span and
// retire quickly, so the block scheduler can interleave them with the compute
// stream's kernels on the same SMs (this kernel runs on a low-priority
// stream); the batched form covers every tensor of a layer in one launch.
constexpr int kPerturbGroupsPerThread = 4;
constexpr int kPerturbThreads = 128;
// One 8-element group span of a perturbation: block `blk` of the tensor.
// cols == 0: outputs are contiguous like the input; otherwise element e of the
// row-major [n / cols, cols] tensor goes to (e / cols) * dld + e % cols of the
// outputs (a block of a wider matrix; cols % 8 == 0).
__device__ __forceinline__ void perturb_block(const uint16_t* __restrict__ w, uint64_t n, uint64_t seed,
                                              uint32_t pair, uint32_t tensor, float sigma,
                                              uint16_t* __restrict__ plus, uint16_t* __restrict__ minus,
                                              uint32_t cols, uint64_t dld, uint64_t blk) {
  const uint64_t groups = (n + 7) / 8, full = n / 8;
  const uint64_t g0 = blk * (kPerturbThreads * kPerturbGroupsPerThread) + threadIdx.x;
  // all of this thread's loads first (streaming: the base weights are read
  // once per pair and do not fit in L2), then the noise and the stores
  uint4 raw[kPerturbGroupsPerThread];
#pragma unroll
  for (int it = 0; it < kPerturbGroupsPerThread; ++it) {
    const uint64_t g = g0 + (uint64_t)it * kPerturbThreads;
    raw[it] = (w && g < full) ? __ldcs(reinterpret_cast<const uint4*>(w) + g) : make_uint4(0, 0, 0, 0);
  }
#pragma unroll
  for (int it = 0; it < kPerturbGroupsPerThread; ++it) {
    const uint64_t g = g0 + (uint64_t)it * kPerturbThreads;
    if (g >= groups) return;
    const uint64_t e0 = g * 8;
    float z[8];
    noise8(seed, pair, tensor, g, z);
    if (g < full) {
      uint32_t ev[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) ev[j] = pack_bf16x2(__fmul_rn(sigma, z[2 * j]), __fmul_rn(sigma, z[2 * j + 1]));
      const uint64_t d = cols ? (e0 / cols) * dld + e0 % cols : e0;
      if (!w) {
        __stcs(reinterpret_cast<uint4*>(plus + d), make_uint4(ev[0], ev[1], ev[2], ev[3]));
        continue;
      }
      const uint32_t in[4] = {raw[it].x, raw[it].y, raw[it].z, raw[it].w};
      uint32_t p[4], m[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        p[j] = bf16x2_add(in[j], ev[j]);
        m[j] = bf16x2_sub(in[j], ev[j]);
      }
      __stcs(reinterpret_cast<uint4*>(plus + d), make_uint4(p[0], p[1], p[2], p[3]));
      if (minus) __stcs(reinterpret_cast<uint4*>(minus + d), make_uint4(m[0], m[1], m[2], m[3]));
    } else {
      for (uint64_t e = e0; e < n; ++e) {
        const uint16_t step = f32_to_bf16_rne(__fmul_rn(sigma, z[e - e0]));
        const uint64_t d = cols ? (e / cols) * dld + e % cols : e;
        if (!w) {
          plus[d] = step;
          continue;
        }
        const float a = bf16_to_f32(w[e]), sg = bf16_to_f32(step);
        plus[d] = f32_to_bf16_rne(__fadd_rn(a, sg));
        if (minus) minus[d] = f32_to_bf16_rne(__fsub_rn(a, sg));
      }
    }
  }
}

__global__ void __launch_bounds__(kPerturbThreads) perturb_bf16_kernel(const uint16_t* __restrict__ w, uint64_t n,
                                                                       uint64_t seed, uint32_t pair, uint32_t tensor,
                                                                       float sigma, uint16_t* __restrict__ plus,
                                                                       uint16_t* __restrict__ minus, uint32_t cols,
                                                                       uint64_t dld) {
  perturb_block(w, n, seed, pair, tensor, sigma, plus, minus, cols, dld, blockIdx.x);
}

// Several tensors of one antithetic pair in one launch (a layer's weights):
// block b belongs to the job j with block0[j] <= b < block0[j + 1].
__global__ void __launch_bounds__(kPerturbThreads) perturb_batch_kernel(const __grid_constant__ PerturbBatch batch) {
  int j = 0;
  while (j + 1 < batch.count && blockIdx.x >= batch.block0[j + 1]) ++j;
  const PerturbJob& jb = batch.job[j];
  perturb_block(jb.w, jb.n, batch.seed, batch.pair, jb.tensor, batch.sigma, jb.plus, jb.minus, jb.cols, jb.dld,
                blockIdx.x - batch.block0[j]);
}

// ---------------------------------------------------------------------------
// host helpers
// ---------------------------------------------------------------------------
int32_t validate_leaves(const ennx_b200_dense_leaf* leaves, size_t nl, size_t n) {
  if (!leaves || nl == 0) return set_error(ENNX_B200_INVALID_ARGUMENT, "at least one dense leaf is required");
  if (nl > (size_t)kMaxSmemLeaves)
    return set_error(ENNX_B200_UNSUPPORTED, "at most %d dense leaves per call", kMaxSmemLeaves);
  size_t end = 0;
  for (size_t i = 0; i < nl; ++i) {
    if (leaves[i].offset != end)
      return set_error(ENNX_B200_INVALID_ARGUMENT, "dense leaf offset %zu does not continue parameter offset %zu",
                       leaves[i].offset, end);
    if (leaves[i].len == 0 || !isfinite(leaves[i].scale) || leaves[i].scale <= 0.0f)
      return set_error(ENNX_B200_INVALID_ARGUMENT, "dense leaves require positive lengths and scales");
    end += leaves[i].len;
  }
  if (end != n)
    return set_error(ENNX_B200_INVALID_ARGUMENT, "dense leaves cover %zu parameters, expected %zu", end, n);
  return ENNX_B200_OK;
}

static double coefficient_of(const ennx_b200_dense_term* t, size_t nt, uint64_t seed) {
  double c = 0.0;
  for (size_t i = 0; i < nt; ++i) if (t[i].seed == seed) c += (double)t[i].coefficient;
  return c;
}

int32_t validate_terms(const ennx_b200_dense_term* terms, size_t nt, const char* what) {
  if (!terms || nt == 0) return set_error(ENNX_B200_INVALID_ARGUMENT, "%s requires perturbation terms", what);
  if (nt > (size_t)kMaxSmemTerms) return set_error(ENNX_B200_UNSUPPORTED, "at most %d terms per call", kMaxSmemTerms);
  for (size_t i = 0; i < nt; ++i)
    if (!isfinite(terms[i].coefficient))
      return set_error(ENNX_B200_INVALID_ARGUMENT, "dense coefficients must be finite");
  for (size_t i = 0; i < nt; ++i) {  // has_direction, dense.rs:258-265
    bool seen = false;
    for (size_t j = 0; j < i; ++j) seen |= terms[j].seed == terms[i].seed;
    if (!seen && coefficient_of(terms, nt, terms[i].seed) != 0.0) return ENNX_B200_OK;
  }
  return set_error(ENNX_B200_INVALID_ARGUMENT, "%s terms cancel to zero", what);
}

// Copies leaves + terms + a zeroed status word into the staging area.
int32_t stage(const ennx_b200_dense_leaf* leaves, size_t nl, const ennx_b200_dense_term* terms, size_t nt,
              cudaStream_t s, DevLeaf** dl, DevTerm** dt, int** status) {
  size_t lb = nl * sizeof(DevLeaf), tb = nt * sizeof(DevTerm);
  size_t bytes = 64 + lb + tb;
  char* base = (char*)staging(bytes);
  if (!base) return set_error(ENNX_B200_CUDA_ERROR, "staging allocation failed");
  DevLeaf hl[kMaxSmemLeaves];
  DevTerm ht[kMaxSmemTerms];
  for (size_t i = 0; i < nl; ++i)
    hl[i] = DevLeaf{mix64(leaves[i].key ^ 0xd6e8feb86659fd93ull), leaves[i].offset, leaves[i].len, leaves[i].scale, 0};
  for (size_t i = 0; i < nt; ++i) ht[i] = DevTerm{terms[i].seed, terms[i].coefficient, 0};
  *status = (int*)base;
  *dl = (DevLeaf*)(base + 64);
  *dt = (DevTerm*)(base + 64 + lb);
  ENNX_CUDA(cudaMemsetAsync(base, 0, 64, s), "status reset");
  if (nl) ENNX_CUDA(cudaMemcpyAsync(*dl, hl, lb, cudaMemcpyHostToDevice, s), "stage leaves");
  ENNX_CUDA(cudaMemcpyAsync(*dt, ht, tb, cudaMemcpyHostToDevice, s), "stage terms");
  return ENNX_B200_OK;
}

int grid_for(uint64_t n, int threads) {
  uint64_t blocks = (n + threads - 1) / threads;
  uint64_t cap = (uint64_t)sm_count() * 16;
  return (int)(blocks < cap ? (blocks ? blocks : 1) : cap);
}

}  // namespace
}  // namespace ennx

using namespace ennx;

namespace ennx {
int32_t launch_perturb_bf16(const uint16_t* w, size_t n, uint64_t seed, uint32_t pair, uint32_t tensor, float sigma,
                            uint16_t* plus, uint16_t* minus, uint32_t cols, uint64_t dld, cudaStream_t s) {
  if (!plus || n == 0) return set_error(ENNX_B200_INVALID_ARGUMENT, "perturb_bf16 needs an output");
  if (!w && minus) return set_error(ENNX_B200_INVALID_ARGUMENT, "perturb_bf16: the noise step has one output");
  if (((uintptr_t)w | (uintptr_t)plus | (uintptr_t)minus) & 15u)
    return set_error(ENNX_B200_INVALID_ARGUMENT, "perturb_bf16 buffers must be 16-byte aligned");
  if (!isfinite(sigma)) return set_error(ENNX_B200_INVALID_ARGUMENT, "sigma must be finite");
  if (cols && (cols % 8 || n % cols || dld % 8 || dld < cols))
    return set_error(ENNX_B200_INVALID_ARGUMENT, "perturb_bf16: strided output needs cols %% 8 == 0 and dld >= cols");
  uint64_t groups = (n + 7) / 8;
  uint64_t per_block = kPerturbThreads * kPerturbGroupsPerThread;
  uint64_t blocks = (groups + per_block - 1) / per_block;
  if (blocks > 0x7fffffffull) return set_error(ENNX_B200_UNSUPPORTED, "perturb_bf16: tensor too large");
  perturb_bf16_kernel<<<(unsigned)blocks, kPerturbThreads, 0, s>>>(w, n, seed, pair, tensor, sigma, plus, minus,
                                                                    cols, dld);
  ENNX_LAUNCH_CHECK("perturb_bf16 launch");
  return ENNX_B200_OK;
}

int32_t launch_perturb_batch(const PerturbBatch& batch, cudaStream_t s) {
  if (batch.count <= 0) return ENNX_B200_OK;
  if (batch.count > kMaxPerturbJobs) return set_error(ENNX_B200_UNSUPPORTED, "perturb batch: too many tensors");
  if (!isfinite(batch.sigma)) return set_error(ENNX_B200_INVALID_ARGUMENT, "sigma must be finite");
  PerturbBatch b = batch;
  const uint64_t per_block = kPerturbThreads * kPerturbGroupsPerThread;
  uint64_t blocks = 0;
  for (int j = 0; j < b.count; ++j) {
    const PerturbJob& jb = b.job[j];
    if (!jb.plus || jb.n == 0) return set_error(ENNX_B200_INVALID_ARGUMENT, "perturb batch: empty job %d", j);
    if (((uintptr_t)jb.w | (uintptr_t)jb.plus | (uintptr_t)jb.minus) & 15u)
      return set_error(ENNX_B200_INVALID_ARGUMENT, "perturb batch: buffers must be 16-byte aligned");
    if (jb.cols && (jb.cols % 8 || jb.n % jb.cols || jb.dld % 8 || jb.dld < jb.cols))
      return set_error(ENNX_B200_INVALID_ARGUMENT, "perturb batch: bad strided output");
    b.block0[j] = (uint32_t)blocks;
    blocks += ((jb.n + 7) / 8 + per_block - 1) / per_block;
  }
  if (blocks > 0x7fffffffull) return set_error(ENNX_B200_UNSUPPORTED, "perturb batch: too many blocks");
  b.block0[b.count] = (uint32_t)blocks;
  perturb_batch_kernel<<<(unsigned)blocks, kPerturbThreads, 0, s>>>(b);
  ENNX_LAUNCH_CHECK("perturb batch launch");
  return ENNX_B200_OK;
}

}  // namespace ennx

extern "C" {

int32_t ennx_b200_dense_apply_f32(const float* base, size_t n, const ennx_b200_dense_leaf* leaves, size_t nl,
                                  const ennx_b200_dense_term* terms, size_t nt, float* out, size_t* changed,
                                  void* stream) {
  cudaStream_t s = (cudaStream_t)stream;
  if (!base || !out || n == 0) return set_error(ENNX_B200_INVALID_ARGUMENT, "dense base cannot be empty");
  ENNX_TRY(validate_leaves(leaves, nl, n));
  ENNX_TRY(validate_terms(terms, nt, "dense"));
  DevLeaf* dl; DevTerm* dt; int* status;
  ENNX_TRY(stage(leaves, nl, terms, nt, s, &dl, &dt, &status));
  apply_dense_f32_kernel<<<grid_for(n, 256), 256, 0, s>>>(base, out, n, dl, (int)nl, dt, (int)nt, status);
  ENNX_LAUNCH_CHECK("apply_dense_f32 launch");
  int host = 0;
  ENNX_CUDA(cudaMemcpyAsync(&host, status, sizeof(int), cudaMemcpyDeviceToHost, s), "status read");
  ENNX_CUDA(cudaStreamSynchronize(s), "apply_dense_f32");
  if (host) return set_error(ENNX_B200_OVERFLOW, "dense perturbation overflowed FP32");
  if (changed) *changed = n;
  return ENNX_B200_OK;
}

int32_t ennx_b200_dense_apply_bf16(const uint16_t* base, size_t n, const ennx_b200_dense_leaf* leaves, size_t nl,
                                   const ennx_b200_dense_term* terms, size_t nt, uint16_t* out, void* stream) {
  cudaStream_t s = (cudaStream_t)stream;
  if (!base || !out || n == 0) return set_error(ENNX_B200_INVALID_ARGUMENT, "BF16 pytree base cannot be empty");
  ENNX_TRY(validate_leaves(leaves, nl, n));
  ENNX_TRY(validate_terms(terms, nt, "BF16 pytree"));
  DevLeaf* dl; DevTerm* dt; int* status;
  ENNX_TRY(stage(leaves, nl, terms, nt, s, &dl, &dt, &status));
  apply_dense_bf16_kernel<<<grid_for(n, 256), 256, 0, s>>>(base, out, n, dl, (int)nl, dt, (int)nt, status);
  ENNX_LAUNCH_CHECK("apply_dense_bf16 launch");
  int host = 0;
  ENNX_CUDA(cudaMemcpyAsync(&host, status, sizeof(int), cudaMemcpyDeviceToHost, s), "status read");
  ENNX_CUDA(cudaStreamSynchronize(s), "apply_dense_bf16");
  if (host) {  // roll back to the base, cuda/src/lib.rs:1247-1250
    ENNX_CUDA(cudaMemcpyAsync(out, base, n * 2, cudaMemcpyDeviceToDevice, s), "rollback");
    ENNX_CUDA(cudaStreamSynchronize(s), "rollback");
    return set_error(ENNX_B200_OVERFLOW, "BF16 pytree perturbation overflowed FP32");
  }
  return ENNX_B200_OK;
}

int32_t ennx_b200_check_bf16(const uint16_t* v, size_t n, int32_t* all_finite, void* stream) {
  cudaStream_t s = (cudaStream_t)stream;
  if (!v || n == 0 || !all_finite) return set_error(ENNX_B200_INVALID_ARGUMENT, "check_bf16 needs a non-empty buffer");
  int* status = (int*)staging(64);
  if (!status) return set_error(ENNX_B200_CUDA_ERROR, "staging allocation failed");
  ENNX_CUDA(cudaMemsetAsync(status, 0, 4, s), "status reset");
  check_bf16_kernel<<<grid_for(n, 256), 256, 0, s>>>(v, n, status);
  ENNX_LAUNCH_CHECK("check_bf16 launch");
  int host = 0;
  ENNX_CUDA(cudaMemcpyAsync(&host, status, sizeof(int), cudaMemcpyDeviceToHost, s), "status read");
  ENNX_CUDA(cudaStreamSynchronize(s), "check_bf16");
  *all_finite = host ? 0 : 1;
  return ENNX_B200_OK;
}

int32_t ennx_b200_dense_linear_f32(const float* input, size_t columns, const float* weight, size_t rows,
                                   const float* bias, ennx_b200_dense_view wv, ennx_b200_dense_view bv,
                                   const ennx_b200_dense_term* terms, size_t nt, float* out, void* stream) {
  cudaStream_t s = (cudaStream_t)stream;
  if (!input || !weight || !out || columns == 0 || rows == 0)
    return set_error(ENNX_B200_INVALID_ARGUMENT, "dense linear weight must contain complete non-empty rows");
  if (!isfinite(wv.scale) || wv.scale <= 0.0f)
    return set_error(ENNX_B200_INVALID_ARGUMENT, "dense linear weight scale must be finite and positive");
  if (bias && (!isfinite(bv.scale) || bv.scale <= 0.0f))
    return set_error(ENNX_B200_INVALID_ARGUMENT, "dense linear bias scale must be finite and positive");
  if (rows > 0x7fffffffull) return set_error(ENNX_B200_UNSUPPORTED, "dense linear rows exceed 2^31");
  ENNX_TRY(validate_terms(terms, nt, "dense linear"));
  DevLeaf* dl; DevTerm* dt; int* status;
  ENNX_TRY(stage(nullptr, 0, terms, nt, s, &dl, &dt, &status));
  DevLeaf w{mix64(wv.key ^ 0xd6e8feb86659fd93ull), wv.start, 0, wv.scale, 0};
  DevLeaf b{mix64(bv.key ^ 0xd6e8feb86659fd93ull), bv.start, 0, bv.scale, 0};
  dense_linear_kernel<<<(unsigned)rows, 256, 0, s>>>(input, weight, bias, out, columns, rows, w, b, dt, (int)nt);
  ENNX_LAUNCH_CHECK("dense_linear launch");
  return ENNX_B200_OK;
}

// Host arithmetic only: energy (sum of len * scale^2 over the leaves) times the
// squared distance between the two coefficient vectors, each seed counted once,
// left seeds first, then right-only seeds (zig/src/dense.zig:124-167).
int32_t ennx_b200_dense_dist2(const ennx_b200_dense_leaf* leaves, size_t nl, const ennx_b200_dense_term* left,
                              size_t nleft, const ennx_b200_dense_term* right, size_t nright, double* out) {
  if (!out) return set_error(ENNX_B200_INVALID_ARGUMENT, "dense distance needs an output");
  if (!leaves || nl == 0) return set_error(ENNX_B200_INVALID_ARGUMENT, "at least one dense leaf is required");
  if ((nleft && !left) || (nright && !right))
    return set_error(ENNX_B200_INVALID_ARGUMENT, "dense distance terms are null");
  size_t end = 0;
  double energy = 0.0;
  for (size_t i = 0; i < nl; ++i) {
    if (leaves[i].offset != end)
      return set_error(ENNX_B200_INVALID_ARGUMENT, "dense leaf offset %zu does not continue parameter offset %zu",
                       leaves[i].offset, end);
    if (leaves[i].len == 0 || !isfinite(leaves[i].scale) || leaves[i].scale <= 0.0f)
      return set_error(ENNX_B200_INVALID_ARGUMENT, "dense leaves require positive lengths and scales");
    if (leaves[i].len > SIZE_MAX - end) return set_error(ENNX_B200_INVALID_ARGUMENT, "dense parameter count overflow");
    end += leaves[i].len;
    double sc = (double)leaves[i].scale;
    energy += (double)leaves[i].len * sc * sc;
  }
  for (size_t i = 0; i < nleft; ++i)
    if (!isfinite(left[i].coefficient))
      return set_error(ENNX_B200_INVALID_ARGUMENT, "dense coefficients must be finite");
  for (size_t i = 0; i < nright; ++i)
    if (!isfinite(right[i].coefficient))
      return set_error(ENNX_B200_INVALID_ARGUMENT, "dense coefficients must be finite");
  auto seen = [](const ennx_b200_dense_term* t, size_t n, uint64_t seed) {
    for (size_t i = 0; i < n; ++i) if (t[i].seed == seed) return true;
    return false;
  };
  double d2 = 0.0;
  for (size_t i = 0; i < nleft; ++i) {
    if (seen(left, i, left[i].seed)) continue;
    double d = coefficient_of(left, nleft, left[i].seed) - coefficient_of(right, nright, left[i].seed);
    d2 += d * d;
  }
  for (size_t i = 0; i < nright; ++i) {
    if (seen(right, i, right[i].seed) || seen(left, nleft, right[i].seed)) continue;
    double c = coefficient_of(right, nright, right[i].seed);
    d2 += c * c;
  }
  *out = energy * d2;
  return ENNX_B200_OK;
}

int32_t ennx_b200_perturb_bf16(const uint16_t* w, size_t n, uint64_t seed, uint32_t pair, uint32_t tensor,
                               float sigma, uint16_t* plus, uint16_t* minus, void* stream) {
  return ennx::launch_perturb_bf16(w, n, seed, pair, tensor, sigma, plus, minus, 0, 0, (cudaStream_t)stream);
}

}  // extern "C"
