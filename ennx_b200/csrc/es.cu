// es.cu -- the zeroth-order update: every rank regenerates the population's
// noise from (seed, pair, tensor, element) and moves its replica of the base
// weights by the broadcast coefficients,
//   W <- bf16( W + sum_p c_p * eps_p )      (fp32 sum over pairs in order)
// so no weight or gradient ever crosses the interconnect: only the scalar
// fitness vector (gather) and the coefficients (broadcast).
//
// The coefficients of the antithetic estimator are
//   c_p = -lr * (f(W + sigma eps_p) - f(W - sigma eps_p)) / (2 sigma P)
// (f = mean cross-entropy, minimised).  This is the tell of the population
// round: the reference's device tell moves the incumbent from the rewards of
// the round (rust/crates/ennx/src/bf16_search.rs:319-407 tell_device ->
// finish_round; cuda/kernels/src/lib.rs:409-535), here for a Gaussian
// population instead of one picked trial.
//
// HBM- and ALU-bound: 4 B per weight (read, write) and P normals per weight
// (one Philox4x32-10 call per 8 elements per pair).
#include <string.h>

#include "common.cuh"
#include "kernels.cuh"

namespace ennx {
namespace {

constexpr int kUpdThreads = 256;
constexpr int kMaxPairs = 256;

__global__ void es_coef_kernel(const float* __restrict__ fitness, int pairs, float scale, float* __restrict__ coef) {
  const int p = blockIdx.x * blockDim.x + threadIdx.x;
  if (p < pairs) coef[p] = scale * (fitness[2 * p] - fitness[2 * p + 1]);
}

// Blocks of the batch: block b belongs to job j with block0[j] <= b < block0[j + 1];
// each thread updates groups of 8 consecutive elements (one Philox block).
__global__ void __launch_bounds__(kUpdThreads) es_update_kernel(const __grid_constant__ EsUpdateBatch batch,
                                                                const float* __restrict__ coef) {
  __shared__ float c[kMaxPairs];
  for (int i = threadIdx.x; i < batch.pairs; i += blockDim.x) c[i] = coef[i];
  __syncthreads();
  int j = 0;
  while (j + 1 < batch.count && blockIdx.x >= batch.block0[j + 1]) ++j;
  const EsUpdateJob& jb = batch.job[j];
  const uint64_t groups = (jb.n + 7) / 8, full = jb.n / 8;
  const uint64_t g = (uint64_t)(blockIdx.x - batch.block0[j]) * kUpdThreads + threadIdx.x;
  if (g >= groups) return;
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  for (int p = 0; p < batch.pairs; ++p) {
    float z[8];
    noise8(batch.seed, batch.first_pair + (uint32_t)p, jb.tensor, g, z);
    const float cp = c[p];
#pragma unroll
    for (int k = 0; k < 8; ++k) acc[k] = __fmaf_rn(cp, z[k], acc[k]);
  }
  uint16_t* w = jb.w;
  if (g < full) {
    uint4 v = *reinterpret_cast<const uint4*>(w + g * 8);
    uint32_t in[4] = {v.x, v.y, v.z, v.w}, out[4];
#pragma unroll
    for (int k = 0; k < 4; ++k)
      out[k] = pack_bf16x2(__fadd_rn(bf16_to_f32((uint16_t)(in[k] & 0xffffu)), acc[2 * k]),
                           __fadd_rn(bf16_to_f32((uint16_t)(in[k] >> 16)), acc[2 * k + 1]));
    *reinterpret_cast<uint4*>(w + g * 8) = make_uint4(out[0], out[1], out[2], out[3]);
  } else {
    for (uint64_t e = g * 8; e < jb.n; ++e) w[e] = f32_to_bf16_rne(__fadd_rn(bf16_to_f32(w[e]), acc[e - g * 8]));
  }
}

}  // namespace

int32_t launch_es_coefficients(const float* fitness, int pairs, float sigma, float lr, int total_pairs, float* coef,
                               cudaStream_t s) {
  if (!fitness || !coef || pairs <= 0) return set_error(ENNX_B200_INVALID_ARGUMENT, "es_coefficients: empty input");
  if (!(sigma > 0.0f) || !isfinite(sigma) || !isfinite(lr))
    return set_error(ENNX_B200_INVALID_ARGUMENT, "es_coefficients: sigma must be positive and finite, lr finite");
  if (total_pairs < pairs) return set_error(ENNX_B200_INVALID_ARGUMENT, "es_coefficients: total_pairs < pairs");
  const float scale = -lr / (2.0f * sigma * (float)total_pairs);
  es_coef_kernel<<<(pairs + 255) / 256, 256, 0, s>>>(fitness, pairs, scale, coef);
  ENNX_LAUNCH_CHECK("es_coefficients");
  return ENNX_B200_OK;
}

int32_t launch_es_update(const EsUpdateBatch& batch, const float* coef, cudaStream_t s) {
  if (batch.count <= 0) return ENNX_B200_OK;
  if (batch.count > kMaxEsJobs) return set_error(ENNX_B200_UNSUPPORTED, "es_update: too many tensors per launch");
  if (!coef || batch.pairs <= 0 || batch.pairs > kMaxPairs)
    return set_error(ENNX_B200_INVALID_ARGUMENT, "es_update: 1..%d pairs and their coefficients required", kMaxPairs);
  EsUpdateBatch b = batch;
  uint64_t blocks = 0;
  for (int j = 0; j < b.count; ++j) {
    if (!b.job[j].w || b.job[j].n == 0) return set_error(ENNX_B200_INVALID_ARGUMENT, "es_update: empty tensor %d", j);
    if ((uintptr_t)b.job[j].w & 15u) return set_error(ENNX_B200_INVALID_ARGUMENT, "es_update: 16-byte aligned weights");
    b.block0[j] = (uint32_t)blocks;
    blocks += ((b.job[j].n + 7) / 8 + kUpdThreads - 1) / kUpdThreads;
  }
  if (blocks > 0x7fffffffull) return set_error(ENNX_B200_UNSUPPORTED, "es_update: too many blocks");
  b.block0[b.count] = (uint32_t)blocks;
  es_update_kernel<<<(unsigned)blocks, kUpdThreads, 0, s>>>(b, coef);
  ENNX_LAUNCH_CHECK("es_update");
  return ENNX_B200_OK;
}

}  // namespace ennx

extern "C" {

int32_t ennx_b200_es_coefficients(const float* fitness, int32_t pairs, int32_t total_pairs, float sigma, float lr,
                                  float* coef, void* stream) {
  return ennx::launch_es_coefficients(fitness, pairs, sigma, lr, total_pairs, coef, (cudaStream_t)stream);
}

int32_t ennx_b200_es_update_bf16(uint16_t* w, size_t n, uint64_t seed, uint32_t tensor, const float* coef,
                                 uint32_t first_pair, uint32_t pairs, void* stream) {
  using namespace ennx;
  EsUpdateBatch b;
  memset(&b, 0, sizeof(b));
  b.seed = seed;
  b.first_pair = first_pair;
  b.pairs = (int)pairs;
  b.count = 1;
  b.job[0].w = w;
  b.job[0].n = n;
  b.job[0].tensor = tensor;
  return launch_es_update(b, coef, (cudaStream_t)stream);
}

}  // extern "C"
