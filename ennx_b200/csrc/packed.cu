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

namespace ennx {
namespace {

// Metal perturb_hash (kda_moe.metal:63-71): note the XOR of seed.high comes
// after the last multiply, unlike the CUDA trial_hash (cuda/kernels/src/lib.rs:150-158).
__device__ __forceinline__ uint32_t packed_hash(uint32_t low, uint32_t high, uint32_t element) {
  uint32_t v = low ^ (element * 0x9E3779B9u);
  v ^= v >> 16;
  v *= 0x7FEB352Du;
  v ^= v >> 15;
  v *= 0x846CA68Bu;
  v ^= v >> 15;
  return v ^ high;
}

struct PackedDesc {
  uint64_t byte_offset, scale_offset, bias_offset, input_width, output_width, element_offset, row_bytes, groups;
  uint32_t bits, group_size, whole, threshold;
};

__device__ __forceinline__ float packed_weight(const uint8_t* __restrict__ w, const float* __restrict__ sc,
                                               const float* __restrict__ bi, const PackedDesc& d,
                                               ennx_b200_perturb_seed seed, uint64_t row, uint64_t col) {
  const uint32_t epb = d.bits == 4 ? 2u : 1u;
  const uint32_t shift = d.bits == 4 ? (uint32_t)(col & 1u) * 4u : 0u;
  const uint32_t max_code = (1u << d.bits) - 1u;
  uint32_t code = ((uint32_t)w[d.byte_offset + row * d.row_bytes + col / epb] >> shift) & max_code;
  if (seed.enabled) {
    // 32-bit element index, as the reference's uint arithmetic
    const uint32_t element = (uint32_t)d.element_offset + (uint32_t)row * (uint32_t)d.input_width + (uint32_t)col;
    const uint32_t random = packed_hash(seed.low, seed.high, element);
    const uint32_t amount = d.whole + (uint32_t)((random >> 1) < (d.threshold >> 1));
    if (amount != 0u) {
      if ((random & 1u) == 0u)
        code = code >= amount ? code - amount : min(code + amount, max_code);
      else
        code = code + amount <= max_code ? code + amount : code >= amount ? code - amount : 0u;
    }
  }
  const uint64_t group = min(col / d.group_size, d.groups - 1);
  const uint64_t si = row * d.groups + group;
  return __fmaf_rn((float)code, sc[d.scale_offset + si], bi[d.bias_offset + si]);
}

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

int32_t make_desc(const ennx_b200_packed_linear* l, PackedDesc* d) {
  if (!l) return set_error(ENNX_B200_INVALID_ARGUMENT, "packed linear descriptor is null");
  // KdaPackedLinear::validate (forward_program.rs:238-249)
  if (l->input_width == 0 || l->output_width == 0 || l->group_size == 0)
    return set_error(ENNX_B200_INVALID_ARGUMENT, "packed KDA linear dimensions must be positive");
  if (l->bits != 4 && l->bits != 8)
    return set_error(ENNX_B200_INVALID_ARGUMENT, "packed KDA linear bits must be 4 or 8, got %u", l->bits);
  d->byte_offset = l->byte_offset; d->scale_offset = l->scale_offset; d->bias_offset = l->bias_offset;
  d->input_width = l->input_width; d->output_width = l->output_width; d->element_offset = l->element_offset;
  d->row_bytes = (l->input_width * l->bits + 7) / 8;
  d->groups = (l->input_width + l->group_size - 1) / l->group_size;
  d->bits = l->bits; d->group_size = l->group_size; d->whole = l->perturb_whole; d->threshold = l->perturb_threshold;
  return ENNX_B200_OK;
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
