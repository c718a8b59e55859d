// packed.cuh -- packed int4/int8 affine weights with integer-code
// perturbation, shared by the packed projection (packed.cu) and the packed
// single-token decoder (decode.cu).
//
// Restates packed_code_device / packed_weight_device / perturb_hash
// (rust/crates/ennx/src/kda_moe.metal:63-96, 351-395) and
// KdaPackedLinear::validate (forward_program.rs:238-249).
#pragma once

#include "common.cuh"

namespace ennx {

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

// KdaPackedLinear -> device descriptor (validates the dimensions and bits).
inline int32_t make_desc(const ennx_b200_packed_linear* l, PackedDesc* d) {
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

}  // namespace ennx
