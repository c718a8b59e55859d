// packed.cu -- packed int4/int8 affine weights with integer-code perturbation.
//
// Restates the reference's native packed projection path (Metal only there):
// packed_code_device / packed_weight_device / perturb_hash
// (rust/crates/ennx/src/kda_moe.metal:63-96, 351-395), the row dequantisers
// packed_dequantize_row_half/_float (:451-476) and the packed projection
// decoder_project_packed (:399-420).  On B200 the projection for M tokens is
// a dequantise(+perturb) pass into a bf16 weight matrix followed by the
// tcgen05 GEMM, the same materialise-then-GEMM structure as the bf16 forward.
#include <string.h>

#include "common.cuh"
#include "kernels.cuh"
#include "packed.cuh"

namespace ennx {
namespace {

// one thread per (row, 8 consecutive columns)
template <typename T>
__global__ void __launch_bounds__(256) packed_dequant_kernel(const uint8_t* __restrict__ w,
                                                             const float* __restrict__ sc,
                                                             const float* __restrict__ bi, PackedDesc d,
                                                             ennx_b200_perturb_seed seed, T* __restrict__ out) {
  const uint64_t per_row = (d.input_width + 7) / 8;
  const uint64_t total = per_row * d.output_width;
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t row = i / per_row, c0 = (i % per_row) * 8;
    T* o = out + row * d.input_width + c0;
    if (c0 + 8 <= d.input_width && d.input_width % 8 == 0) {
      float f[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) f[j] = packed_weight(w, sc, bi, d, seed, row, c0 + j);
      if constexpr (sizeof(T) == 2) {
        *reinterpret_cast<uint4*>(o) = make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]),
                                                  pack_bf16x2(f[4], f[5]), pack_bf16x2(f[6], f[7]));
      } else {
        *reinterpret_cast<float4*>(o) = make_float4(f[0], f[1], f[2], f[3]);
        *reinterpret_cast<float4*>(o + 4) = make_float4(f[4], f[5], f[6], f[7]);
      }
    } else {
      for (uint64_t c = c0; c < d.input_width && c < c0 + 8; ++c) {
        const float v = packed_weight(w, sc, bi, d, seed, row, c);
        if constexpr (sizeof(T) == 2) o[c - c0] = f32_to_bf16_rne(v);
        else o[c - c0] = v;
      }
    }
  }
}

template <typename T>
int32_t dequant(const uint8_t* w, const float* sc, const float* bi, const ennx_b200_packed_linear* l,
                ennx_b200_perturb_seed seed, T* out, cudaStream_t s) {
  PackedDesc d;
  ENNX_TRY(make_desc(l, &d));
  if (!w || !sc || !bi || !out) return set_error(ENNX_B200_INVALID_ARGUMENT, "packed dequantize: null buffer");
  if ((uintptr_t)out & 15u) return set_error(ENNX_B200_INVALID_ARGUMENT, "packed dequantize: out must be 16-byte aligned");
  const uint64_t work = (d.input_width + 7) / 8 * d.output_width;
  uint64_t blocks = (work + 255) / 256;
  const uint64_t cap = (uint64_t)sm_count() * 32;
  if (blocks > cap) blocks = cap;
  packed_dequant_kernel<T><<<(unsigned)blocks, 256, 0, s>>>(w, sc, bi, d, seed, out);
  ENNX_LAUNCH_CHECK("packed dequantize");
  return ENNX_B200_OK;
}

}  // namespace
}  // namespace ennx

using namespace ennx;

extern "C" {

int32_t ennx_b200_packed_dequantize_bf16(const uint8_t* weights, const float* scales, const float* biases,
                                         const ennx_b200_packed_linear* linear, ennx_b200_perturb_seed seed,
                                         uint16_t* out, void* stream) {
  return dequant<uint16_t>(weights, scales, biases, linear, seed, out, (cudaStream_t)stream);
}

int32_t ennx_b200_packed_dequantize_f32(const uint8_t* weights, const float* scales, const float* biases,
                                        const ennx_b200_packed_linear* linear, ennx_b200_perturb_seed seed,
                                        float* out, void* stream) {
  return dequant<float>(weights, scales, biases, linear, seed, out, (cudaStream_t)stream);
}

size_t ennx_b200_packed_linear_workspace_size(const ennx_b200_packed_linear* linear) {
  if (!linear) return 0;
  return (size_t)linear->input_width * linear->output_width * sizeof(uint16_t);
}

int32_t ennx_b200_packed_linear_bf16(const uint16_t* x, int64_t tokens, const uint8_t* weights, const float* scales,
                                     const float* biases, const ennx_b200_packed_linear* linear,
                                     ennx_b200_perturb_seed seed, uint16_t* out, void* workspace,
                                     size_t workspace_bytes, void* stream) {
  cudaStream_t s = (cudaStream_t)stream;
  PackedDesc d;
  ENNX_TRY(make_desc(linear, &d));
  if (!x || !out || tokens <= 0) return set_error(ENNX_B200_INVALID_ARGUMENT, "packed linear: empty input");
  if (d.input_width % 64 || d.input_width > 0x7fffffffull || d.output_width > 0x7fffffffull || tokens > 0x7fffffffLL)
    return set_error(ENNX_B200_UNSUPPORTED, "packed linear: input_width must be a multiple of 64 (widths < 2^31)");
  if (d.output_width % 8) return set_error(ENNX_B200_UNSUPPORTED, "packed linear: output_width must be a multiple of 8");
  const size_t need = ennx_b200_packed_linear_workspace_size(linear);
  if (!workspace || workspace_bytes < need)
    return set_error(ENNX_B200_INVALID_ARGUMENT, "packed linear: workspace of %zu bytes required", need);
  ENNX_TRY(dequant<uint16_t>(weights, scales, biases, linear, seed, (uint16_t*)workspace, s));
  ennx_b200_gemm_params p;
  memset(&p, 0, sizeof(p));
  p.m = (int)tokens; p.n = (int)d.output_width; p.k = (int)d.input_width;
  p.lda = (int64_t)d.input_width; p.ldb = (int64_t)d.input_width; p.ldc = (int64_t)d.output_width;
  p.groups = 1; p.epilogue = ENNX_B200_EPI_BF16; p.alpha = 1.0f;
  return gemm_bf16(&p, x, (const uint16_t*)workspace, out, s);
}

}  // extern "C"
