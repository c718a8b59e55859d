// loss.cu -- LM-head cross-entropy reduction.  The vocabulary GEMM
// (gemm.cu, EPI_LSE) leaves one (max, sum exp) pair per 256-column tile and
// the target logit per row; logits are never materialised.  Here each row's
// partials are merged into logsumexp - target, then each candidate's rows are
// averaged in a fixed order (deterministic fitness).  No reference
// counterpart: the reference scores candidates with a composite objective
// (kda_moe.metal:1011-1032), BASELINE asks for mean cross-entropy.
#include "common.cuh"
#include "kernels.cuh"

namespace ennx {

__global__ void lse_loss_kernel(const float2* __restrict__ part, int n_tiles, const float* __restrict__ tl,
                                long long rows, float* __restrict__ loss) {
  long long r = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  int lane = threadIdx.x & 31;
  if (r >= rows) return;
  const float2* p = part + r * n_tiles;
  float m = -INFINITY;
  for (int i = lane; i < n_tiles; i += 32) m = fmaxf(m, p[i].x);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  float s = 0.0f;
  for (int i = lane; i < n_tiles; i += 32) s += p[i].y * expf(p[i].x - m);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (lane == 0) loss[r] = m + logf(s) - tl[r];
}

__global__ void mean_per_set_kernel(const float* __restrict__ v, long long per_set, float* __restrict__ out) {
  __shared__ double buf[1024];
  const float* p = v + blockIdx.x * per_set;
  double acc = 0.0;
  for (long long i = threadIdx.x; i < per_set; i += blockDim.x) acc += (double)p[i];
  buf[threadIdx.x] = acc;
  __syncthreads();
  for (int o = blockDim.x / 2; o > 0; o >>= 1) {
    if ((int)threadIdx.x < o) buf[threadIdx.x] += buf[threadIdx.x + o];
    __syncthreads();
  }
  if (threadIdx.x == 0) out[blockIdx.x] = (float)(buf[0] / (double)per_set);
}

int32_t launch_lse_loss(const float* lse_partial, int n_tiles, const float* target_logit, long long rows,
                        float* row_loss, cudaStream_t s) {
  lse_loss_kernel<<<(unsigned)((rows + 7) / 8), 256, 0, s>>>((const float2*)lse_partial, n_tiles, target_logit, rows,
                                                              row_loss);
  ENNX_LAUNCH_CHECK("lse_loss");
  return ENNX_B200_OK;
}

int32_t launch_mean_per_set(const float* row_loss, long long rows_per_set, int sets, float* out, cudaStream_t s) {
  mean_per_set_kernel<<<sets, 1024, 0, s>>>(row_loss, rows_per_set, out);
  ENNX_LAUNCH_CHECK("mean_per_set");
  return ENNX_B200_OK;
}

}  // namespace ennx
