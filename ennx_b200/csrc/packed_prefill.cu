// packed_prefill.cu -- the KDA attention block of the packed (int4/int8)
// model over whole sequences: the counterpart of the reference's 16k prefill
// KdaMoeMetalExecutor::kda (rust/crates/ennx/src/forward_metal.rs:997-1129),
// which chains kda_project_packed_16k (qkv, control), kda_split_qkv_16k,
// kda_split_control_16k, the forget / output-gate projections,
// kda_make_gate_beta_16k, kda_recurrence_16k, kda_postprocess_16k, the
// output projection and decoder_residual (kda_moe.metal:167-225, 847-921,
// 556-565) -- with no short convolution and no q/k L2 norm, as that path
// has none -- for any sequence length instead of only 16384.
//
// B200 form: every projection's packed codes (with the candidate's integer-
// code perturbation) are dequantised once per call into bf16 and the
// projections run as tcgen05 GEMMs over all tokens; the gates, beta and the
// recurrence run in the chunked KDA kernels (gate formation fused into the
// chunk preparation); the output projection adds s * update to the residual
// stream in its epilogue.
#include <string.h>

#include "common.cuh"
#include "kernels.cuh"

namespace ennx {
namespace {

constexpr int HD = 128;

struct PrefillLayout {
  size_t w_qkv, w_ctl, w_f, w_og, w_out, decay, tb, onorm;  // dequantised weights (element offsets)
  size_t qkv, ctl, f, og, o, post;                         // activations
  size_t kda_ws;                                           // byte offset of the KDA chunk records
  size_t kda_bytes, total;
  long long ldc;
};

size_t al(size_t elems) { return (elems + 127) / 128 * 128; }  // 256-byte granules of bf16

int32_t layout(const ennx_b200_packed_kda_block* b, int batch, int seq, int hidden, PrefillLayout* L) {
  if (!b || batch <= 0 || seq <= 0 || hidden <= 0)
    return set_error(ENNX_B200_INVALID_ARGUMENT, "packed_kda_prefill: empty problem");
  const long long heads = b->heads, r = b->gate_rank, hw = heads * HD, H = hidden, T = (long long)batch * seq;
  if (heads <= 0 || r <= 0 || r % 64 || H % 64)
    return set_error(ENNX_B200_UNSUPPORTED, "packed_kda_prefill: gate_rank and hidden must be multiples of 64");
  struct Want { const ennx_b200_packed_linear* l; long long out, in; const char* name; } want[] = {
      {&b->qkv, 3 * hw, H, "qkv"}, {&b->control, 2 * r + heads, H, "control"}, {&b->forget_b, hw, r, "forget_b"},
      {&b->gate_b, hw, r, "gate_b"}, {&b->output, H, hw, "output"}, {&b->decay, 1, heads, "decay"},
      {&b->time_bias, 1, hw, "time_bias"}, {&b->output_norm, 1, HD, "output_norm"}};
  for (const Want& w : want)
    if ((long long)w.l->output_width != w.out || (long long)w.l->input_width != w.in)
      return set_error(ENNX_B200_INVALID_ARGUMENT, "packed_kda_prefill: %s must be [%lld, %lld], got [%llu, %llu]",
                       w.name, w.out, w.in, (unsigned long long)w.l->output_width,
                       (unsigned long long)w.l->input_width);
  size_t off = 0;
  auto take = [&](size_t n) { size_t o = off; off += al(n); return o; };
  L->ldc = (2 * r + heads + 7) / 8 * 8;
  L->w_qkv = take(3 * hw * H);
  L->w_ctl = take((2 * r + heads) * H);
  L->w_f = take(hw * r);
  L->w_og = take(hw * r);
  L->w_out = take(H * hw);
  L->decay = take(heads);
  L->tb = take(hw);
  L->onorm = take(HD);
  L->qkv = take(T * 3 * hw);
  L->ctl = take(T * L->ldc);
  L->f = take(T * hw);
  L->og = take(T * hw);
  L->o = take(T * hw);
  L->post = take(T * hw);
  L->kda_ws = off * 2;
  L->kda_bytes = kda_workspace_bytes(batch, seq, (int)heads);
  L->total = L->kda_ws + (L->kda_bytes + 255) / 256 * 256;
  return ENNX_B200_OK;
}

int32_t gemm(const uint16_t* a, long long lda, const uint16_t* w, long long n, long long k, uint16_t* c, long long ldc,
             long long rows, const uint16_t* residual, float alpha, cudaStream_t s) {
  ennx_b200_gemm_params p;
  memset(&p, 0, sizeof(p));
  p.m = (int)rows; p.n = (int)n; p.k = (int)k;
  p.lda = lda; p.ldb = k; p.ldc = ldc;
  p.groups = 1; p.epilogue = ENNX_B200_EPI_BF16; p.alpha = alpha;
  p.residual = residual; p.ldr = ldc;
  ProfScope ps("gemm", s, 2.0 * rows * n * k, 2.0 * (rows * k + n * k + rows * n * (residual ? 2 : 1)));
  return gemm_bf16(&p, a, w, c, s);
}

}  // namespace
}  // namespace ennx

using namespace ennx;

extern "C" {

size_t ennx_b200_packed_kda_prefill_workspace_size(const ennx_b200_packed_kda_block* block, int32_t batch, int32_t seq,
                                                   int32_t hidden) {
  PrefillLayout L;
  if (layout(block, batch, seq, hidden, &L) != ENNX_B200_OK) return 0;
  return L.total;
}

int32_t ennx_b200_packed_kda_prefill(const uint8_t* weights, const float* scales, const float* biases,
                                     const ennx_b200_packed_kda_block* block, ennx_b200_perturb_seed seed,
                                     const uint16_t* normalized, uint16_t* hidden, float* state, int32_t batch,
                                     int32_t seq, int32_t hidden_width, void* workspace, size_t workspace_bytes,
                                     void* stream) {
  cudaStream_t s = (cudaStream_t)stream;
  PrefillLayout L;
  ENNX_TRY(layout(block, batch, seq, hidden_width, &L));
  if (!weights || !scales || !biases || !normalized || !hidden)
    return set_error(ENNX_B200_INVALID_ARGUMENT, "packed_kda_prefill: null argument");
  if (!workspace || workspace_bytes < L.total || ((uintptr_t)workspace & 255u))
    return set_error(ENNX_B200_INVALID_ARGUMENT, "packed_kda_prefill: 256-byte aligned workspace of %zu bytes required",
                     L.total);
  if (!isfinite(block->rms_eps) || !isfinite(block->residual_scale))
    return set_error(ENNX_B200_INVALID_ARGUMENT, "packed_kda_prefill: epsilon and residual scale must be finite");
  uint16_t* ws = (uint16_t*)workspace;
  const long long heads = block->heads, r = block->gate_rank, hw = heads * HD, H = hidden_width;
  const long long T = (long long)batch * seq;
  // 1. the candidate's weights: dequantised (integer-code perturbation
  //    included) once per call
  const struct { const ennx_b200_packed_linear* l; size_t off; } deq[] = {
      {&block->qkv, L.w_qkv}, {&block->control, L.w_ctl}, {&block->forget_b, L.w_f}, {&block->gate_b, L.w_og},
      {&block->output, L.w_out}, {&block->decay, L.decay}, {&block->time_bias, L.tb},
      {&block->output_norm, L.onorm}};
  for (const auto& d : deq)
    ENNX_TRY(ennx_b200_packed_dequantize_bf16(weights, scales, biases, d.l, seed, ws + d.off, stream));
  // 2. projections over all tokens (kda_project_packed_16k, then the splits:
  //    q | k | v and forget state | output state | beta are column ranges)
  uint16_t *qkv = ws + L.qkv, *ctl = ws + L.ctl, *f = ws + L.f, *og = ws + L.og, *o = ws + L.o, *post = ws + L.post;
  ENNX_TRY(gemm(normalized, H, ws + L.w_qkv, 3 * hw, H, qkv, 3 * hw, T, nullptr, 1.0f, s));
  ENNX_TRY(gemm(normalized, H, ws + L.w_ctl, 2 * r + heads, H, ctl, L.ldc, T, nullptr, 1.0f, s));
  ENNX_TRY(gemm(ctl, L.ldc, ws + L.w_f, hw, r, f, hw, T, nullptr, 1.0f, s));
  ENNX_TRY(gemm(ctl + r, L.ldc, ws + L.w_og, hw, r, og, hw, T, nullptr, 1.0f, s));
  // 3. gate / beta (kda_make_gate_beta_16k) inside the chunk preparation, and
  //    the recurrence (kda_recurrence_16k) on q and k as projected
  KdaRawGate rg;
  memset(&rg, 0, sizeof(rg));
  rg.f = f; rg.ldf = hw;
  rg.rbeta = ctl + 2 * r; rg.ldb = L.ldc;
  rg.decay0 = rg.decay1 = ws + L.decay;
  rg.tb0 = rg.tb1 = ws + L.tb;
  rg.split_seq = batch;
  rg.active = 1;
  rg.no_l2norm = 1;
  {
    ProfScope ps("kda", s, (double)T * heads * (6.0 * HD * HD + 6.0 * 64 * HD), (double)T * heads * HD * 12.0);
    ENNX_TRY(launch_kda_chunked(qkv, qkv + hw, qkv + 2 * hw, 3 * hw, nullptr, nullptr, state, o, hw, batch, seq,
                                (int)heads, (uint8_t*)workspace + L.kda_ws, L.kda_bytes, s, &rg));
  }
  // 4. per-head RMSNorm x output norm x sigmoid(output gate) (kda_postprocess_16k)
  ENNX_TRY(launch_kda_post(o, og, hw, ws + L.onorm, nullptr, T, (int)heads, T, block->rms_eps, post, s));
  // 5. output projection and decoder_residual: hidden += s * (post . W_out^T)
  return gemm(post, hw, ws + L.w_out, H, hw, hidden, H, T, hidden, block->residual_scale, s);
}

}  // extern "C"
