// forward.cu -- public operator entry points and the population forward.
//
// The population forward is the B200 replacement of the reference's
// evaluation seam: ForwardEvaluator::evaluate (rust/crates/ennx/src/
// forward_program.rs:210-212) driven by ResidentBoState::ask_evaluate
// (:706-720), with the decoder layer order of
// KdaMoeMetalExecutor::encode_decode_layer (forward_metal.rs:614-810):
//   rms_norm -> qkv proj -> split -> L2 norm q,k -> control proj -> split ->
//   forget / output-gate proj -> gate, beta -> KDA -> post-norm * gate ->
//   out proj -> residual -> rms_norm -> router top-k -> gate_up -> down ->
//   residual
// generalised to prefill over whole sequences, GQA layers every
// `attn_period` layers, and a fused LM-head cross-entropy at the end.
//
// Work is organised per antithetic pair: the pair's perturbation of one layer
// is generated into a scratch area (streaming kernel on a second stream)
// while the previous layer runs, then both candidates' tokens run through
// the layer as one batch.  Two perturbation modes
// (ennx_b200_set_perturbation_mode):
//   materialised (default): the noise kernel writes W + e and W - e
//     (e = bf16(sigma*eps)) for every tensor; every GEMM is a 2-group tcgen05
//     launch on those copies (MoE: 2*E groups);
//   fused: the noise kernel writes only the noise step e of the matrices, and
//     every GEMM is one perturbed launch that forms W + e and W - e inside its
//     operand path, so no perturbed matrix is stored.  Small per-layer vectors
//     and the router matrix are W +/- e copies in both modes.
// Both modes compute the same perturbed weights bit for bit.
#include <string.h>

#include <algorithm>
#include <vector>

#include <stdlib.h>

#include "common.cuh"
#include "kernels.cuh"

namespace ennx {
namespace {

constexpr int HD = 128;  // head dim of both attention kinds

struct Carver {
  uint8_t* base;
  size_t off = 0, cap;
  bool measure;
  template <typename T>
  T* take(size_t count) {
    size_t bytes = (count * sizeof(T) + 255) & ~(size_t)255;
    T* p = measure ? nullptr : reinterpret_cast<T*>(base + off);
    off += bytes;
    return p;
  }
};

__global__ void targets_kernel(const int* __restrict__ tokens, int batch, int seq, int* __restrict__ inp,
                               int* __restrict__ tgt2) {
  int n = batch * seq;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    int b = i / seq, t = i % seq;
    inp[i] = tokens[b * (seq + 1) + t];
    int y = tokens[b * (seq + 1) + t + 1];
    tgt2[i] = y;
    tgt2[i + n] = y;
  }
}

// ---------------------------------------------------------------------------
// MoE layer body shared by ennx_b200_moe_layer and the population forward
// ---------------------------------------------------------------------------
struct MoeBuffers {
  float* logits;
  int *idx, *counters, *offsets, *perm_pos;
  float *gate, *perm_gate;
  uint16_t *xperm, *act, *yperm;
  float* router_wt;  // both router weight sets as fp32, k-major per 64-expert tile
};

void carve_moe(Carver& c, long long tokens, int hidden, int experts, int top_k, int width, int sets, MoeBuffers& m) {
  long long rows = tokens * top_k;
  m.idx = c.take<int>(rows);
  m.gate = c.take<float>(rows);
  m.counters = c.take<int>(2 * sets * experts);
  m.offsets = c.take<int>(sets * experts + 1);
  m.perm_pos = c.take<int>(rows);
  m.perm_gate = c.take<float>(rows);
  m.xperm = c.take<uint16_t>(rows * hidden);
  m.act = c.take<uint16_t>(rows * width);
  m.yperm = c.take<uint16_t>(rows * hidden);
  m.router_wt = c.take<float>(2 * (size_t)((experts + 63) / 64) * hidden * 64);
  m.logits = nullptr;
}

// x [tokens, hidden] -> out = residual + MoE(x).  Sets: rows < split use
// expert block 0 of the weights, the rest block 1 (block stride = experts).
int32_t run_moe(const uint16_t* x, const uint16_t* wr0, const uint16_t* wr1, const uint16_t* wgu, const uint16_t* wd,
                long long tokens, long long split, int sets, int hidden, int experts, int top_k, int width,
                const uint16_t* residual, uint16_t* out, MoeBuffers& m, cudaStream_t s, float residual_scale = 1.0f,
                const uint16_t* gu_noise = nullptr, const uint16_t* down_noise = nullptr) {
  if (width % 128) return set_error(ENNX_B200_UNSUPPORTED, "moe: expert width %d must be a multiple of 128", width);
  long long rows = tokens * top_k;
  {
    ProfScope ps("moe_routing", s, 2.0 * tokens * hidden * experts,
                 2.0 * tokens * hidden + 2.0 * sets * experts * hidden + 4.0 * rows * hidden);
    // pick counts (router) -> slots and row copies in expert-major order (one pass)
    ENNX_CUDA(cudaMemsetAsync(m.counters, 0, sizeof(int) * 2 * sets * experts, s), "moe counters");
    ENNX_TRY(launch_router_topk(x, hidden, wr0, sets > 1 ? wr1 : nullptr, split, tokens, hidden, experts, top_k,
                                m.logits, m.idx, m.gate, s, m.counters, m.router_wt));
    ENNX_TRY(launch_moe_scatter_gather(m.idx, m.gate, residual_scale, tokens, top_k, experts, split, sets, m.counters,
                                       m.offsets, m.counters + sets * experts, m.perm_pos, m.perm_gate, x, hidden,
                                       hidden, m.xperm, s));
  }
  ennx_b200_gemm_params p;
  memset(&p, 0, sizeof(p));
  p.m = (int)rows; p.n = 2 * width; p.k = hidden;
  p.lda = hidden; p.ldb = hidden; p.ldc = width;
  p.groups = sets * experts; p.b_group_rows = 2 * width; p.group_offsets = m.offsets;
  p.epilogue = ENNX_B200_EPI_SWIGLU; p.alpha = 1.0f;
  {
    ProfScope ps("gemm", s, 2.0 * rows * 2 * width * hidden,
                 2.0 * (rows * hidden + (double)sets * experts * 2 * width * hidden + rows * width));
    // sets == 2 with noise: expert e of set 0 uses W + e, of set 1 W - e
    if (gu_noise) ENNX_TRY(gemm_bf16_perturbed(&p, m.xperm, wgu, gu_noise, m.act, s));
    else ENNX_TRY(gemm_bf16(&p, m.xperm, wgu, m.act, s));
  }
  memset(&p, 0, sizeof(p));
  p.m = (int)rows; p.n = hidden; p.k = width;
  p.lda = width; p.ldb = width; p.ldc = hidden;
  p.groups = sets * experts; p.b_group_rows = hidden; p.group_offsets = m.offsets;
  p.epilogue = ENNX_B200_EPI_ROWSCALE; p.row_scale = m.perm_gate; p.alpha = 1.0f;
  {
    ProfScope ps("gemm", s, 2.0 * rows * hidden * width,
                 2.0 * (rows * width + (double)sets * experts * hidden * width + rows * hidden));
    if (down_noise) ENNX_TRY(gemm_bf16_perturbed(&p, m.act, wd, down_noise, m.yperm, s));
    else ENNX_TRY(gemm_bf16(&p, m.act, wd, m.yperm, s));
  }
  {
    ProfScope ps("moe_combine", s, 0, 2.0 * (rows * hidden + 2.0 * tokens * hidden));
    ENNX_TRY(launch_moe_combine(m.yperm, m.perm_pos, tokens, top_k, hidden, residual, out, s));
  }
  return ENNX_B200_OK;
}

// ---------------------------------------------------------------------------
// population forward
// ---------------------------------------------------------------------------
enum Field { F_ATTN_NORM, F_QKV, F_CTL, F_FORGET, F_OGATE, F_DECAY, F_TB, F_OUT_NORM, F_WO, F_MOE_NORM, F_ROUTER,
             F_GATE_UP, F_DOWN, F_COUNT };

struct Shapes {
  long long rows[F_COUNT], cols[F_COUNT];
};

bool is_gqa(const ennx_b200_model_config& c, int l) {
  return c.attn_period > 0 && (l % c.attn_period) == c.attn_period - 1;
}

Shapes layer_shapes(const ennx_b200_model_config& c, bool gqa) {
  Shapes s;
  memset(&s, 0, sizeof(s));
  const long long H = c.hidden, I = c.expert_width, E = c.experts;
  const long long heads = gqa ? c.q_heads : c.kda_heads;
  s.rows[F_ATTN_NORM] = 1; s.cols[F_ATTN_NORM] = H;
  s.rows[F_QKV] = gqa ? (long long)(c.q_heads + 2 * c.kv_heads) * HD : 3LL * c.kda_heads * HD; s.cols[F_QKV] = H;
  if (!gqa) {
    s.rows[F_CTL] = 2LL * c.gate_rank + c.kda_heads; s.cols[F_CTL] = H;
    s.rows[F_FORGET] = (long long)c.kda_heads * HD; s.cols[F_FORGET] = c.gate_rank;
    s.rows[F_OGATE] = (long long)c.kda_heads * HD; s.cols[F_OGATE] = c.gate_rank;
    s.rows[F_DECAY] = 1; s.cols[F_DECAY] = c.kda_heads;
    s.rows[F_TB] = 1; s.cols[F_TB] = (long long)c.kda_heads * HD;
    s.rows[F_OUT_NORM] = 1; s.cols[F_OUT_NORM] = HD;
  }
  s.rows[F_WO] = H; s.cols[F_WO] = heads * HD;
  s.rows[F_MOE_NORM] = 1; s.cols[F_MOE_NORM] = H;
  s.rows[F_ROUTER] = E; s.cols[F_ROUTER] = H;
  s.rows[F_GATE_UP] = E * 2 * I; s.cols[F_GATE_UP] = H;
  s.rows[F_DOWN] = E * H; s.cols[F_DOWN] = I;
  return s;
}

size_t align_elems(long long n) { return (size_t)((n + 127) / 128 * 128); }  // 256-byte granules of bf16

// Scratch layout of the perturbed copies of one layer.  On KDA layers the
// QKV projection and the control projection share one region, [W_qkv; W_ctl]
// per sign, so one GEMM of N = rows(qkv) + rows(ctl) computes both; the
// forget and output-gate projections share a block-diagonal [2*hw, 2*r]
// matrix [[W_f, 0], [0, W_o]] per sign, so one GEMM with K = 2r over
// ctl[:, 0:2r] computes [f | og].  The off-diagonal blocks are zeroed once
// per call and never written.
long long field_elems(const Shapes& sh, int f) {
  switch (f) {
    case F_QKV: return (sh.rows[F_QKV] + sh.rows[F_CTL]) * sh.cols[F_QKV];
    case F_CTL: return 0;
    case F_FORGET: return 4 * sh.rows[F_FORGET] * sh.cols[F_FORGET];
    case F_OGATE: return 0;
    default: return sh.rows[f] * sh.cols[f];
  }
}
// Matrices consumed by the perturbed GEMM: only their noise step e is
// generated (one copy); the other fields get materialised W + e and W - e.
bool gemm_field(int f, bool fused) {
  return fused && (f == F_QKV || f == F_CTL || f == F_FORGET || f == F_OGATE || f == F_WO || f == F_GATE_UP || f == F_DOWN);
}
int g_fused_mode = 0;  // ennx_b200_set_perturbation_mode
int kda_ordinal(const ennx_b200_model_config& c, int l) {  // index of KDA layer l among the KDA layers
  int n = 0;
  for (int i = 0; i < l; ++i) n += is_gqa(c, i) ? 0 : 1;
  return n;
}
// leading dimension of the fused QKV(+control) GEMM output
long long qkv_ld(const Shapes& sh) { return (sh.rows[F_QKV] + sh.rows[F_CTL] + 7) / 8 * 8; }

struct Work {
  const int* tokens;       // caller's [batch, seq + 1] token ids
  bool fused;              // perturbation mode of this call
  uint16_t *emb_scr[2];    // two slots of [2][V*H] (plus, minus), or the noise step [V*H] (fused)
  uint16_t *fnorm_scr[2];  // two slots of [2][H] (final norm plus, minus)
  uint16_t *layer_scr[2];  // two slots of per-field areas: [n] noise (GEMM fields) or [2][n] (plus, minus)
  size_t field_off[F_COUNT];  // element offsets into layer_scr
  uint16_t* base_fused;    // per KDA layer: [W_qkv; W_ctl] then [[W_f, 0], [0, W_o]] (base weights)
  size_t base_stride;      // elements per KDA layer in base_fused
  uint16_t *hidden, *xn, *qkv, *fg, *o, *post;
  float *gate, *beta;
  int *inp, *tgt;
  float *lse, *tlogit, *row_loss;
  void* kda_ws;
  size_t kda_ws_bytes;
  MoeBuffers moe;
  size_t bytes;
};

int32_t validate_config(const ennx_b200_model_config* c, int batch, int seq) {
  if (!c) return set_error(ENNX_B200_INVALID_ARGUMENT, "null model config");
  if (c->layers <= 0 || c->hidden <= 0 || c->vocab <= 0 || batch <= 0 || seq <= 0)
    return set_error(ENNX_B200_INVALID_ARGUMENT, "model config and token batch must be non-empty");
  if (c->hidden % 256) return set_error(ENNX_B200_UNSUPPORTED, "hidden must be a multiple of 256");
  if (c->expert_width % 128) return set_error(ENNX_B200_UNSUPPORTED, "expert_width must be a multiple of 128");
  if (c->gate_rank % 64 || c->gate_rank <= 0) return set_error(ENNX_B200_UNSUPPORTED, "gate_rank must be a multiple of 64");
  if (c->attn_period > 0 && (c->kv_heads <= 0 || c->q_heads % c->kv_heads))
    return set_error(ENNX_B200_INVALID_ARGUMENT, "q_heads must be a multiple of kv_heads");
  if (c->top_k < 1 || c->top_k > 8 || c->top_k > c->experts)
    return set_error(ENNX_B200_INVALID_ARGUMENT, "top_k must be in [1, min(8, experts)]");
  if (2 * c->experts > 256) return set_error(ENNX_B200_UNSUPPORTED, "at most 128 experts");
  if (!isfinite(c->residual_scale) || !isfinite(c->rms_eps))  // KdaMoeLayerRequest::validate, forward_program.rs:431
    return set_error(ENNX_B200_INVALID_ARGUMENT, "residual scale and RMS epsilon must be finite");
  if (c->residual_scale == 0.0f)
    return set_error(ENNX_B200_INVALID_ARGUMENT, "residual scale 0 would drop every layer update");
  return ENNX_B200_OK;
}

void carve_work(const ennx_b200_model_config& c, int batch, int seq, uint8_t* base, Work& w) {
  Carver cv{base, 0, 0, base == nullptr};
  w.fused = g_fused_mode != 0;
  const long long Tc = (long long)batch * seq, T = 2 * Tc, H = c.hidden;
  for (int k = 0; k < 2; ++k) {
    w.emb_scr[k] = cv.take<uint16_t>(2 * align_elems((long long)c.vocab * H));
    w.fnorm_scr[k] = cv.take<uint16_t>(2 * align_elems(H));
  }
  size_t per_field_max[F_COUNT] = {0};
  for (int g = 0; g < 2; ++g) {
    Shapes sh = layer_shapes(c, g == 1);
    for (int f = 0; f < F_COUNT; ++f) {
      size_t n = align_elems(field_elems(sh, f));
      if (n > per_field_max[f]) per_field_max[f] = n;
    }
  }
  size_t off = 0;
  for (int f = 0; f < F_COUNT; ++f) { w.field_off[f] = off; off += 2 * per_field_max[f]; }  // room for both modes
  for (int k = 0; k < 2; ++k) w.layer_scr[k] = cv.take<uint16_t>(off);
  {
    const Shapes sk = layer_shapes(c, false);
    w.base_stride = align_elems(field_elems(sk, F_QKV)) + align_elems(field_elems(sk, F_FORGET));
    long long kda_layers = 0;
    for (int l = 0; l < c.layers; ++l) kda_layers += is_gqa(c, l) ? 0 : 1;
    w.base_fused = cv.take<uint16_t>(w.base_stride * kda_layers);
  }
  const long long qkv_cols = std::max(qkv_ld(layer_shapes(c, false)), qkv_ld(layer_shapes(c, true)));
  const long long heads_max = std::max(c.kda_heads, c.q_heads);
  w.hidden = cv.take<uint16_t>(T * H);
  w.xn = cv.take<uint16_t>(T * H);
  w.qkv = cv.take<uint16_t>(T * qkv_cols);
  w.fg = cv.take<uint16_t>(T * 2 * c.kda_heads * HD);  // [forget | output gate]
  w.o = cv.take<uint16_t>(T * heads_max * HD);
  w.post = cv.take<uint16_t>(T * c.kda_heads * HD);
  w.gate = cv.take<float>(T * c.kda_heads * HD);
  w.beta = cv.take<float>(T * c.kda_heads);
  w.inp = cv.take<int>(Tc);
  w.tgt = cv.take<int>(T);
  const long long ntiles = 2 * ((c.vocab + 255) / 256);  // LSE partials per row
  w.lse = cv.take<float>(T * ntiles * 2);
  w.tlogit = cv.take<float>(T);
  w.row_loss = cv.take<float>(T);
  carve_moe(cv, T, c.hidden, c.experts, c.top_k, c.expert_width, 2, w.moe);
  w.kda_ws_bytes = kda_workspace_bytes(2 * batch, seq, std::max(c.kda_heads, 1));
  w.kda_ws = cv.take<uint8_t>(w.kda_ws_bytes);
  w.bytes = cv.off;
}

const uint16_t* field_ptr(const ennx_b200_layer_weights& L, int f) {
  switch (f) {
    case F_ATTN_NORM: return L.attn_norm;
    case F_QKV: return L.w_qkv;
    case F_CTL: return L.w_ctl;
    case F_FORGET: return L.w_forget;
    case F_OGATE: return L.w_ogate;
    case F_DECAY: return L.decay;
    case F_TB: return L.time_bias;
    case F_OUT_NORM: return L.out_norm;
    case F_WO: return L.w_o;
    case F_MOE_NORM: return L.moe_norm;
    case F_ROUTER: return L.w_router;
    case F_GATE_UP: return L.w_gate_up;
    default: return L.w_down;
  }
}

// One antithetic pair's projection: rows [0, rows/2) against W + e, the rest
// against W - e, bf16 out (+ residual).  w == nullptr: e points at the stored
// copies [W + e; W - e] ([2n, k]); otherwise W and e are [n, k] and the
// perturbed GEMM forms both signs in its operand path.
int32_t gemm2(const uint16_t* a, long long lda, const uint16_t* w, const uint16_t* e, long long n, long long k,
              void* c, long long ldc, long long rows, const uint16_t* residual, cudaStream_t s,
              double useful_flops = 0.0, float alpha = 1.0f) {
  ennx_b200_gemm_params p;
  memset(&p, 0, sizeof(p));
  p.m = (int)rows; p.n = (int)n; p.k = (int)k;
  p.lda = lda; p.ldb = k; p.ldc = ldc;
  p.groups = 2; p.b_group_rows = (int)n;
  p.epilogue = ENNX_B200_EPI_BF16; p.alpha = alpha;
  p.residual = residual; p.ldr = ldc;
  ProfScope ps("gemm", s, useful_flops > 0.0 ? useful_flops : 2.0 * rows * n * k,
               2.0 * (rows * k + 2.0 * n * k + rows * n * (residual ? 2 : 1)));
  return w ? gemm_bf16_perturbed(&p, a, w, e, c, s) : gemm_bf16(&p, a, e, c, s);
}

// Per-device streams of the pipelined population forward: `compute` runs the
// layers (highest priority), `noise` generates the next layer's perturbed
// weights (lowest priority) into the other half of a double buffer, so the
// HBM-streaming noise kernel fills the issue slots and bandwidth the tensor-
// core GEMMs leave free.
struct PipeStreams {
  cudaStream_t compute = nullptr, noise = nullptr;
  cudaEvent_t ev[8] = {};
};
PipeStreams g_pipe[64];

int32_t pipe_streams(PipeStreams** out) {
  int dev = 0;
  cudaGetDevice(&dev);
  PipeStreams& p = g_pipe[dev];
  if (!p.compute) {
    int least = 0, greatest = 0;
    ENNX_CUDA(cudaDeviceGetStreamPriorityRange(&least, &greatest), "stream priorities");
    ENNX_CUDA(cudaStreamCreateWithPriority(&p.compute, cudaStreamNonBlocking, greatest), "compute stream");
    ENNX_CUDA(cudaStreamCreateWithPriority(&p.noise, cudaStreamNonBlocking, least), "noise stream");
    for (auto& e : p.ev) ENNX_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "pipe events");
  }
  *out = &p;
  return ENNX_B200_OK;
}

struct LayerPtrs {
  uint16_t* P[F_COUNT];
  uint16_t* M[F_COUNT];
};

LayerPtrs layer_ptrs(const ennx_b200_model_config& c, int l, const Work& w, int slot) {
  LayerPtrs lp;
  Shapes sh = layer_shapes(c, is_gqa(c, l));
  for (int f = 0; f < F_COUNT; ++f) {
    long long n = sh.rows[f] * sh.cols[f];
    lp.P[f] = lp.M[f] = nullptr;
    if (n == 0 || f == F_CTL || f == F_OGATE) continue;
    lp.P[f] = w.layer_scr[slot] + w.field_off[f];  // GEMM fields: the noise step e
    // minus copy directly after plus; GEMM operands (n % 64 == 0) keep the B
    // row-block stride between the two signs at exactly `rows`
    const long long fn = field_elems(sh, f);
    if (!gemm_field(f, w.fused)) lp.M[f] = lp.P[f] + (fn % 8 == 0 ? (size_t)fn : align_elems(fn));
  }
  if (sh.rows[F_CTL]) {  // control rows follow the QKV rows of each sign
    lp.P[F_CTL] = lp.P[F_QKV] + sh.rows[F_QKV] * sh.cols[F_QKV];
    if (lp.M[F_QKV]) lp.M[F_CTL] = lp.M[F_QKV] + sh.rows[F_QKV] * sh.cols[F_QKV];
  }
  if (sh.rows[F_OGATE]) {  // output-gate block: rows [hw, 2hw), columns [r, 2r)
    const long long hw = sh.rows[F_FORGET], r = sh.cols[F_FORGET];
    lp.P[F_OGATE] = lp.P[F_FORGET] + hw * 2 * r + r;
    if (lp.M[F_FORGET]) lp.M[F_OGATE] = lp.M[F_FORGET] + hw * 2 * r + r;
  }
  return lp;
}

// noise stream: W +/- sigma*eps of every tensor of layer l into scratch `slot`
// (appended to `batch`; one launch per layer)
int32_t add_layer_jobs(const ennx_b200_model_config& c, const ennx_b200_model_weights& W, int l, const Work& w,
                       int slot, PerturbBatch& batch) {
  const ennx_b200_layer_weights& L = W.layers[l];
  Shapes sh = layer_shapes(c, is_gqa(c, l));
  LayerPtrs lp = layer_ptrs(c, l, w, slot);
  for (int f = 0; f < F_COUNT; ++f) {
    long long n = sh.rows[f] * sh.cols[f];
    if (n == 0) continue;
    const uint16_t* src = field_ptr(L, f);
    if (!src) return set_error(ENNX_B200_INVALID_ARGUMENT, "missing weight tensor %d of layer %d", f, l);
    if (batch.count == kMaxPerturbJobs) return set_error(ENNX_B200_UNSUPPORTED, "too many tensors per layer");
    // forget / output-gate weights land as blocks of the block-diagonal matrix
    const bool blk = f == F_FORGET || f == F_OGATE;
    PerturbJob& j = batch.job[batch.count++];
    j.w = gemm_field(f, w.fused) ? nullptr : src;  // fused GEMM fields: noise step only
    j.plus = lp.P[f]; j.minus = lp.M[f]; j.n = (uint64_t)n;
    j.tensor = 16u + 16u * (uint32_t)l + (uint32_t)f;
    j.cols = blk ? (uint32_t)sh.cols[f] : 0u;
    j.dld = blk ? 2 * (uint64_t)sh.cols[f] : 0u;
  }
  return ENNX_B200_OK;
}

// compute stream: one decoder layer for both candidates of a pair (T rows).
// L: the caller's base weights of the layer; lp: the pair's noise steps and
// small perturbed vectors.
int32_t compute_layer(const ennx_b200_model_config& c, int l, const ennx_b200_layer_weights& L, const LayerPtrs& lp,
                      int batch, int seq, Work& w, cudaStream_t s) {
  const long long Tc = (long long)batch * seq, T = 2 * Tc, H = c.hidden;
  const bool gqa = is_gqa(c, l);
  Shapes sh = layer_shapes(c, gqa);
  uint16_t* const* P = lp.P;
  uint16_t* const* M = lp.M;
  ENNX_TRY(launch_rmsnorm(w.hidden, H, P[F_ATTN_NORM], M[F_ATTN_NORM], Tc, w.xn, H, T, (int)H, c.rms_eps, s));
  // one GEMM: [q | k | v] (and on KDA layers the control projection after them)
  const long long qkv_cols = qkv_ld(sh);
  const uint16_t* base_qkv =
      !w.fused ? nullptr : gqa ? L.w_qkv : w.base_fused + (size_t)kda_ordinal(c, l) * w.base_stride;
  ENNX_TRY(gemm2(w.xn, H, base_qkv, P[F_QKV], sh.rows[F_QKV] + sh.rows[F_CTL], H, w.qkv, qkv_cols, T, nullptr, s));
  if (gqa) {
    const long long kd = (long long)c.q_heads * HD, vd = kd + (long long)c.kv_heads * HD;
    // q heads then k heads, adjacent in each qkv row: one launch
    ENNX_TRY(launch_rope(w.qkv, qkv_cols, c.q_heads + c.kv_heads, HD, T, seq, c.rope_theta, s));
    {
      ProfScope ps("attention", s, 2.0 * batch * c.q_heads * (double)seq * (seq + 1) * HD * 2.0,
                   2.0 * T * (2.0 * kd + 2.0 * c.kv_heads * HD));
      ENNX_TRY(launch_gqa_attention(w.qkv, qkv_cols, w.qkv + kd, qkv_cols, w.qkv + vd, qkv_cols, w.o, kd, 2 * batch,
                                    seq, c.q_heads, c.kv_heads, s));
    }
    ENNX_TRY(gemm2(w.o, kd, w.fused ? L.w_o : nullptr, P[F_WO], H, kd, w.hidden, H, T, w.hidden, s, 0.0, c.residual_scale));
  } else {
    const long long hw = (long long)c.kda_heads * HD, r = c.gate_rank;
    const uint16_t* ctl = w.qkv + sh.rows[F_QKV];  // [forget state | output state | beta], row stride qkv_cols
    // [f | og] = ctl[:, 0:2r] . [[W_f, 0], [0, W_o]]^T
    const uint16_t* base_fo = w.fused ? base_qkv + align_elems(field_elems(sh, F_QKV)) : nullptr;
    ENNX_TRY(gemm2(ctl, qkv_cols, base_fo, P[F_FORGET], 2 * hw, 2 * r, w.fg, 2 * hw, T, nullptr, s,
                   2.0 * 2.0 * T * hw * r));  // the zero blocks are not counted as work
    {
      KdaRawGate rg;
      rg.f = w.fg; rg.ldf = 2 * hw;
      rg.rbeta = ctl + 2 * r; rg.ldb = qkv_cols;
      rg.decay0 = P[F_DECAY]; rg.decay1 = M[F_DECAY];
      rg.tb0 = P[F_TB]; rg.tb1 = M[F_TB];
      rg.split_seq = batch;
      rg.active = 1;
      ProfScope ps("kda", s, (double)T * c.kda_heads * (6.0 * HD * HD + 6.0 * 64 * HD),
                   (double)T * c.kda_heads * HD * (2.0 * 4 + 4.0) + 4.0 * T * c.kda_heads);
      ENNX_TRY(launch_kda_chunked(w.qkv, w.qkv + hw, w.qkv + 2 * hw, qkv_cols, nullptr, nullptr, nullptr, w.o, hw,
                                  2 * batch, seq, c.kda_heads, w.kda_ws, w.kda_ws_bytes, s, &rg));
    }
    ENNX_TRY(launch_kda_post(w.o, w.fg + hw, 2 * hw, P[F_OUT_NORM], M[F_OUT_NORM], Tc, c.kda_heads, T, c.rms_eps,
                             w.post, s));
    ENNX_TRY(gemm2(w.post, hw, w.fused ? L.w_o : nullptr, P[F_WO], H, hw, w.hidden, H, T, w.hidden, s, 0.0, c.residual_scale));
  }
  ENNX_TRY(launch_rmsnorm(w.hidden, H, P[F_MOE_NORM], M[F_MOE_NORM], Tc, w.xn, H, T, (int)H, c.rms_eps, s));
  if (w.fused)
    ENNX_TRY(run_moe(w.xn, P[F_ROUTER], M[F_ROUTER], L.w_gate_up, L.w_down, T, Tc, 2, (int)H, c.experts, c.top_k,
                     c.expert_width, w.hidden, w.hidden, w.moe, s, c.residual_scale, P[F_GATE_UP], P[F_DOWN]));
  else  // stored copies: expert e of set 1 is block E + e of [W + e; W - e]
    ENNX_TRY(run_moe(w.xn, P[F_ROUTER], M[F_ROUTER], P[F_GATE_UP], P[F_DOWN], T, Tc, 2, (int)H, c.experts, c.top_k,
                     c.expert_width, w.hidden, w.hidden, w.moe, s, c.residual_scale));
  return ENNX_B200_OK;
}

// Pipelined population forward.  Job j = (pair i, layer l), j = i*L + l.
// The noise stream perturbs job j+1 into layer slot (j+1)%2 while the compute
// stream runs job j; a pair's embedding (= LM head) and final norm are
// perturbed with its layer 0 into embedding slot i%2.
// hidden_out (nullable): run only the first `stop_layers` layers of each pair
// and copy the residual stream [2][batch*seq][hidden] there instead of the
// LM head (per-layer parity checks).
int32_t run_population(const ennx_b200_model_config& c, const ennx_b200_model_weights& W, uint64_t seed, float sigma,
                       int first_pair, int num_pairs, int batch, int seq, Work& w, float* fitness,
                       cudaStream_t caller, int stop_layers = -1, uint16_t* hidden_out = nullptr,
                       int* index_out = nullptr) {
  PipeStreams* ps = nullptr;
  ENNX_TRY(pipe_streams(&ps));
  cudaStream_t cs = ps->compute, ns = ps->noise;
  // ENNX_B200_NOISE_STREAM=0 runs the perturbation on the compute stream
  // (serialised with the layers) instead of overlapping it on its own stream
  static const bool noise_overlap = [] {
    const char* e = getenv("ENNX_B200_NOISE_STREAM");
    return !(e && e[0] == '0');
  }();
  if (!noise_overlap) ns = cs;
  cudaEvent_t ev_start = ps->ev[0], ev_done_noise = ps->ev[1];
  cudaEvent_t ready[2] = {ps->ev[2], ps->ev[3]}, freed[2] = {ps->ev[4], ps->ev[5]};
  cudaEvent_t emb_freed[2] = {ps->ev[6], ps->ev[7]};
  const long long Tc = (long long)batch * seq, T = 2 * Tc, H = c.hidden, V = c.vocab;
  const int L = hidden_out ? stop_layers : c.layers;
  const int jobs = num_pairs * L;

  ENNX_CUDA(cudaEventRecord(ev_start, caller), "fork");
  ENNX_CUDA(cudaStreamWaitEvent(cs, ev_start, 0), "fork compute");
  ENNX_CUDA(cudaStreamWaitEvent(ns, ev_start, 0), "fork noise");
  {  // zero the block-diagonal forget/output-gate noise areas; the noise kernel fills only the diagonal blocks
    const long long blkdiag = field_elems(layer_shapes(c, false), F_FORGET);
    if (blkdiag > 0)
      for (int k = 0; k < 2; ++k)
        ENNX_CUDA(cudaMemsetAsync(w.layer_scr[k] + w.field_off[F_FORGET], 0, 2 * (size_t)blkdiag * sizeof(uint16_t), ns),
                  "zero gate blocks");
  }
  // Base operands of the fused KDA projections, once per call: [W_qkv; W_ctl]
  // (one GEMM computes both) and the block-diagonal [[W_f, 0], [0, W_o]].
  for (int l = 0; l < L && w.fused; ++l) {
    if (is_gqa(c, l)) continue;
    const ennx_b200_layer_weights& Lw = W.layers[l];
    if (!Lw.w_qkv || !Lw.w_ctl || !Lw.w_forget || !Lw.w_ogate)
      return set_error(ENNX_B200_INVALID_ARGUMENT, "missing KDA projection weights of layer %d", l);
    const Shapes sk = layer_shapes(c, false);
    uint16_t* bq = w.base_fused + (size_t)kda_ordinal(c, l) * w.base_stride;
    uint16_t* bfo = bq + align_elems(field_elems(sk, F_QKV));
    const size_t nq = (size_t)(sk.rows[F_QKV] * sk.cols[F_QKV]), nc = (size_t)(sk.rows[F_CTL] * sk.cols[F_CTL]);
    const size_t hw = (size_t)sk.rows[F_FORGET], r = (size_t)sk.cols[F_FORGET];
    ENNX_CUDA(cudaMemcpyAsync(bq, Lw.w_qkv, nq * 2, cudaMemcpyDeviceToDevice, cs), "base qkv");
    ENNX_CUDA(cudaMemcpyAsync(bq + nq, Lw.w_ctl, nc * 2, cudaMemcpyDeviceToDevice, cs), "base ctl");
    ENNX_CUDA(cudaMemsetAsync(bfo, 0, 4 * hw * r * 2, cs), "base gate blocks");
    ENNX_CUDA(cudaMemcpy2DAsync(bfo, 4 * r, Lw.w_forget, 2 * r, 2 * r, hw, cudaMemcpyDeviceToDevice, cs), "base W_f");
    ENNX_CUDA(cudaMemcpy2DAsync(bfo + hw * 2 * r + r, 4 * r, Lw.w_ogate, 2 * r, 2 * r, hw, cudaMemcpyDeviceToDevice, cs),
              "base W_o gate");
  }
  targets_kernel<<<(unsigned)((Tc + 255) / 256), 256, 0, cs>>>(w.tokens, batch, seq, w.inp, w.tgt);
  ENNX_LAUNCH_CHECK("targets");

  bool freed_recorded[2] = {false, false}, emb_freed_recorded[2] = {false, false};
  auto noise_job = [&](int j) -> int32_t {
    const int i = j / L, l = j % L, slot = j % 2;
    const uint32_t pair = (uint32_t)(first_pair + i);
    if (freed_recorded[slot]) ENNX_CUDA(cudaStreamWaitEvent(ns, freed[slot], 0), "wait slot");
    if (l == 0) {
      const int es = i % 2;
      if (emb_freed_recorded[es]) ENNX_CUDA(cudaStreamWaitEvent(ns, emb_freed[es], 0), "wait emb slot");
    }
    PerturbBatch batch;
    memset(&batch, 0, sizeof(batch));
    batch.seed = seed; batch.pair = pair; batch.sigma = sigma;
    if (l == 0) {
      const int es = i % 2;
      PerturbJob& je = batch.job[batch.count++];
      je.w = w.fused ? nullptr : W.embedding;  // fused: noise step only
      je.plus = w.emb_scr[es]; je.minus = w.fused ? nullptr : w.emb_scr[es] + V * H; je.n = (uint64_t)(V * H);
      je.tensor = 0;
      PerturbJob& jn = batch.job[batch.count++];
      jn.w = W.final_norm; jn.plus = w.fnorm_scr[es]; jn.minus = w.fnorm_scr[es] + H; jn.n = (uint64_t)H;
      jn.tensor = 1;
      if (!W.embedding || !W.final_norm) return set_error(ENNX_B200_INVALID_ARGUMENT, "missing embedding / final norm");
    }
    ENNX_TRY(add_layer_jobs(c, W, l, w, slot, batch));
    {
      double elems = 0;
      for (int q = 0; q < batch.count; ++q) elems += (double)batch.job[q].n;
      double bytes = 0;  // noise steps: 2 B written per element; W +/- e copies: 2 read + 4 written
      for (int q = 0; q < batch.count; ++q) bytes += (batch.job[q].w ? 6.0 : 2.0) * (double)batch.job[q].n;
      (void)elems;
      ProfScope pp("noise", ns, 0, bytes);
      ENNX_TRY(launch_perturb_batch(batch, ns));
    }
    ENNX_CUDA(cudaEventRecord(ready[slot], ns), "ready");
    return ENNX_B200_OK;
  };

  ENNX_TRY(noise_job(0));
  for (int j = 0; j < jobs; ++j) {
    if (j + 1 < jobs) ENNX_TRY(noise_job(j + 1));
    const int i = j / L, l = j % L, slot = j % 2, es = i % 2;
    ENNX_CUDA(cudaStreamWaitEvent(cs, ready[slot], 0), "wait ready");
    if (l == 0)
      ENNX_TRY(w.fused ? launch_embed(w.inp, W.embedding, nullptr, Tc, T, (int)H, (int)V, w.hidden, cs, w.emb_scr[es])
                       : launch_embed(w.inp, w.emb_scr[es], w.emb_scr[es] + V * H, Tc, T, (int)H, (int)V, w.hidden, cs));
    ENNX_TRY(compute_layer(c, l, W.layers[l], layer_ptrs(c, l, w, slot), batch, seq, w, cs));
    ENNX_CUDA(cudaEventRecord(freed[slot], cs), "freed");
    freed_recorded[slot] = true;
    if (l == L - 1 && hidden_out) {
      ENNX_CUDA(cudaMemcpyAsync(hidden_out + (size_t)i * T * H, w.hidden, sizeof(uint16_t) * (size_t)T * H,
                                cudaMemcpyDeviceToDevice, cs),
                "copy hidden state");
      if (index_out)
        ENNX_CUDA(cudaMemcpyAsync(index_out, w.moe.idx, sizeof(int) * (size_t)T * c.top_k, cudaMemcpyDeviceToDevice,
                                  cs),
                  "copy routing");
      ENNX_CUDA(cudaEventRecord(emb_freed[es], cs), "emb freed");
      emb_freed_recorded[es] = true;
    } else if (l == L - 1) {
      uint16_t* fn = w.fnorm_scr[es];
      ENNX_TRY(launch_rmsnorm(w.hidden, H, fn, fn + H, Tc, w.xn, H, T, (int)H, c.rms_eps, cs));
      ennx_b200_gemm_params p;
      memset(&p, 0, sizeof(p));
      p.m = (int)T; p.n = (int)V; p.k = (int)H;
      p.lda = H; p.ldb = H;
      p.groups = 2; p.b_group_rows = (int)V;
      p.epilogue = ENNX_B200_EPI_LSE; p.alpha = 1.0f;
      p.targets = w.tgt; p.lse_partial = w.lse; p.target_logit = w.tlogit;
      {
        ProfScope pf("gemm", cs, 2.0 * T * V * H, 2.0 * (T * H + 2.0 * V * H));
        ENNX_TRY(w.fused ? gemm_bf16_perturbed(&p, w.xn, W.embedding, w.emb_scr[es], nullptr, cs)
                         : gemm_bf16(&p, w.xn, w.emb_scr[es], nullptr, cs));
      }
      ENNX_CUDA(cudaEventRecord(emb_freed[es], cs), "emb freed");
      emb_freed_recorded[es] = true;
      ENNX_TRY(launch_lse_loss(w.lse, (int)(2 * ((V + 255) / 256)), w.tlogit, T, w.row_loss, cs));
      ENNX_TRY(launch_mean_per_set(w.row_loss, Tc, 2, fitness + 2 * i, cs));
    }
  }
  // join both streams back into the caller's stream
  ENNX_CUDA(cudaEventRecord(ev_done_noise, ns), "join noise");
  ENNX_CUDA(cudaStreamWaitEvent(cs, ev_done_noise, 0), "join noise into compute");
  ENNX_CUDA(cudaEventRecord(ev_start, cs), "join compute");
  ENNX_CUDA(cudaStreamWaitEvent(caller, ev_start, 0), "join into caller");
  return ENNX_B200_OK;
}

}  // namespace
}  // namespace ennx

using namespace ennx;

extern "C" {

int32_t ennx_b200_rmsnorm_bf16(const uint16_t* x, const uint16_t* w, int64_t rows, int32_t width, float eps,
                               uint16_t* out, void* stream) {
  if (!x || !w || !out || rows <= 0) return set_error(ENNX_B200_INVALID_ARGUMENT, "rmsnorm: empty input");
  if ((((uintptr_t)x | (uintptr_t)w | (uintptr_t)out) & 15u))
    return set_error(ENNX_B200_INVALID_ARGUMENT, "rmsnorm: buffers must be 16-byte aligned");
  return launch_rmsnorm(x, width, w, nullptr, rows, out, width, rows, width, eps, (cudaStream_t)stream);
}

int32_t ennx_b200_moe_route(const uint16_t* x, const uint16_t* w_router, int64_t tokens, int32_t hidden,
                            int32_t experts, int32_t top_k, float* logits, int32_t* index, float* gate, void* stream) {
  if (!x || !w_router || !index || !gate || tokens <= 0)
    return set_error(ENNX_B200_INVALID_ARGUMENT, "moe_route: null or empty argument");
  return launch_router_topk(x, hidden, w_router, nullptr, tokens, tokens, hidden, experts, top_k, logits, index, gate,
                            (cudaStream_t)stream);
}

size_t ennx_b200_moe_workspace_size(int64_t tokens, int32_t hidden, int32_t experts, int32_t top_k,
                                    int32_t expert_width) {
  Carver c{nullptr, 0, 0, true};
  MoeBuffers m;
  carve_moe(c, tokens, hidden, experts, top_k, expert_width, 1, m);
  return c.off;
}

int32_t ennx_b200_moe_layer(const uint16_t* x, const uint16_t* w_router, const uint16_t* w_gate_up,
                            const uint16_t* w_down, int64_t tokens, int32_t hidden, int32_t experts, int32_t top_k,
                            int32_t expert_width, const uint16_t* residual, uint16_t* y, int32_t* index, float* gate,
                            void* workspace, size_t workspace_bytes, void* stream) {
  if (!x || !w_router || !w_gate_up || !w_down || !y || tokens <= 0)
    return set_error(ENNX_B200_INVALID_ARGUMENT, "moe_layer: null or empty argument");
  size_t need = ennx_b200_moe_workspace_size(tokens, hidden, experts, top_k, expert_width);
  if (!workspace || workspace_bytes < need)
    return set_error(ENNX_B200_INVALID_ARGUMENT, "moe_layer: workspace of %zu bytes required", need);
  Carver c{(uint8_t*)workspace, 0, workspace_bytes, false};
  MoeBuffers m;
  carve_moe(c, tokens, hidden, experts, top_k, expert_width, 1, m);
  cudaStream_t s = (cudaStream_t)stream;
  ENNX_TRY(run_moe(x, w_router, nullptr, w_gate_up, w_down, tokens, tokens, 1, hidden, experts, top_k, expert_width,
                   residual, y, m, s));
  if (index) ENNX_CUDA(cudaMemcpyAsync(index, m.idx, sizeof(int) * tokens * top_k, cudaMemcpyDeviceToDevice, s), "idx");
  if (gate) ENNX_CUDA(cudaMemcpyAsync(gate, m.gate, sizeof(float) * tokens * top_k, cudaMemcpyDeviceToDevice, s), "gate");
  return ENNX_B200_OK;
}

int32_t ennx_b200_gqa_attention(uint16_t* q, uint16_t* k, const uint16_t* v, uint16_t* o, int32_t batch, int32_t seq,
                                int32_t hq, int32_t hkv, float rope_theta, void* stream) {
  if (!q || !k || !v || !o) return set_error(ENNX_B200_INVALID_ARGUMENT, "attention: null argument");
  cudaStream_t s = (cudaStream_t)stream;
  long long T = (long long)batch * seq;
  if (rope_theta > 0.0f) {
    ENNX_TRY(launch_rope(q, (long long)hq * HD, hq, HD, T, seq, rope_theta, s));
    ENNX_TRY(launch_rope(k, (long long)hkv * HD, hkv, HD, T, seq, rope_theta, s));
  }
  return launch_gqa_attention(q, (long long)hq * HD, k, (long long)hkv * HD, v, (long long)hkv * HD, o,
                              (long long)hq * HD, batch, seq, hq, hkv, s);
}

size_t ennx_b200_kda_workspace_size(int32_t batch, int32_t seq, int32_t heads) {
  if (batch <= 0 || seq <= 0 || heads <= 0) return 0;
  return kda_workspace_bytes(batch, seq, heads);
}

int32_t ennx_b200_kda_chunked(const uint16_t* q, const uint16_t* k, const uint16_t* v, const float* g,
                              const float* beta, float* state, uint16_t* o, int32_t batch, int32_t seq, int32_t heads,
                              void* workspace, size_t workspace_bytes, void* stream) {
  if (!q || !k || !v || !g || !beta || !o) return set_error(ENNX_B200_INVALID_ARGUMENT, "kda: null argument");
  return launch_kda_chunked(q, k, v, (long long)heads * HD, g, beta, state, o, (long long)heads * HD, batch, seq,
                            heads, workspace, workspace_bytes, (cudaStream_t)stream);
}

size_t ennx_b200_population_workspace_size(const ennx_b200_model_config* cfg, int32_t batch, int32_t seq) {
  if (!cfg || validate_config(cfg, batch, seq) != ENNX_B200_OK) return 0;
  Work w;
  carve_work(*cfg, batch, seq, nullptr, w);
  return w.bytes;
}

int32_t ennx_b200_population_forward(const ennx_b200_model_config* cfg, const ennx_b200_model_weights* weights,
                                     uint64_t seed, float sigma, int32_t first_pair, int32_t num_pairs,
                                     const int32_t* tokens, int32_t batch, int32_t seq, float* fitness,
                                     void* workspace, size_t workspace_bytes, void* stream) {
  ENNX_TRY(validate_config(cfg, batch, seq));
  if (!weights || !weights->embedding || !weights->final_norm || !weights->layers || !tokens || !fitness)
    return set_error(ENNX_B200_INVALID_ARGUMENT, "population_forward: null argument");
  if (num_pairs <= 0 || first_pair < 0) return set_error(ENNX_B200_INVALID_ARGUMENT, "population_forward: empty pair range");
  if (!isfinite(sigma) || sigma < 0.0f) return set_error(ENNX_B200_INVALID_ARGUMENT, "sigma must be finite and >= 0");
  Work w;
  carve_work(*cfg, batch, seq, nullptr, w);
  if (!workspace || workspace_bytes < w.bytes)
    return set_error(ENNX_B200_INVALID_ARGUMENT, "population_forward: workspace of %zu bytes required", w.bytes);
  carve_work(*cfg, batch, seq, (uint8_t*)workspace, w);
  w.tokens = tokens;
  if ((size_t)cfg->vocab * cfg->hidden != align_elems((long long)cfg->vocab * cfg->hidden))
    return set_error(ENNX_B200_UNSUPPORTED, "vocab*hidden must be a multiple of 128");
  ENNX_TRY(run_population(*cfg, *weights, seed, sigma, first_pair, num_pairs, batch, seq, w, fitness,
                          (cudaStream_t)stream));
  return ENNX_B200_OK;
}

int32_t ennx_b200_population_hidden(const ennx_b200_model_config* cfg, const ennx_b200_model_weights* weights,
                                    uint64_t seed, float sigma, int32_t pair, int32_t layers, const int32_t* tokens,
                                    int32_t batch, int32_t seq, uint16_t* hidden, int32_t* index, void* workspace,
                                    size_t workspace_bytes, void* stream) {
  ENNX_TRY(validate_config(cfg, batch, seq));
  if (!weights || !weights->embedding || !weights->final_norm || !weights->layers || !tokens || !hidden)
    return set_error(ENNX_B200_INVALID_ARGUMENT, "population_hidden: null argument");
  if (pair < 0 || layers < 1 || layers > cfg->layers)
    return set_error(ENNX_B200_INVALID_ARGUMENT, "population_hidden: layers must be in [1, %d]", cfg->layers);
  if (!isfinite(sigma) || sigma < 0.0f) return set_error(ENNX_B200_INVALID_ARGUMENT, "sigma must be finite and >= 0");
  Work w;
  carve_work(*cfg, batch, seq, nullptr, w);
  if (!workspace || workspace_bytes < w.bytes)
    return set_error(ENNX_B200_INVALID_ARGUMENT, "population_hidden: workspace of %zu bytes required", w.bytes);
  carve_work(*cfg, batch, seq, (uint8_t*)workspace, w);
  w.tokens = tokens;
  return run_population(*cfg, *weights, seed, sigma, pair, 1, batch, seq, w, nullptr, (cudaStream_t)stream, layers,
                        hidden, index);
}

int32_t ennx_b200_population_update(const ennx_b200_model_config* cfg, const ennx_b200_model_weights* weights,
                                    uint64_t seed, const float* coef, int32_t first_pair, int32_t num_pairs,
                                    void* stream) {
  if (!cfg || cfg->layers <= 0) return set_error(ENNX_B200_INVALID_ARGUMENT, "population_update: bad config");
  if (!weights || !weights->embedding || !weights->final_norm || !weights->layers || !coef)
    return set_error(ENNX_B200_INVALID_ARGUMENT, "population_update: null argument");
  if (num_pairs <= 0 || first_pair < 0)
    return set_error(ENNX_B200_INVALID_ARGUMENT, "population_update: empty pair range");
  cudaStream_t s = (cudaStream_t)stream;
  const ennx_b200_model_config& c = *cfg;
  // The weights are updated in place through the caller's device pointers;
  // the tensor ids are those of the forward's perturbation.
  EsUpdateBatch b;
  memset(&b, 0, sizeof(b));
  b.seed = seed; b.first_pair = (uint32_t)first_pair; b.pairs = num_pairs;
  b.job[b.count++] = EsUpdateJob{const_cast<uint16_t*>(weights->embedding), (uint64_t)c.vocab * c.hidden, 0u};
  b.job[b.count++] = EsUpdateJob{const_cast<uint16_t*>(weights->final_norm), (uint64_t)c.hidden, 1u};
  for (int l = 0; l < c.layers; ++l) {
    const Shapes sh = layer_shapes(c, is_gqa(c, l));
    for (int f = 0; f < F_COUNT; ++f) {
      const long long n = sh.rows[f] * sh.cols[f];
      if (n == 0) continue;
      const uint16_t* src = field_ptr(weights->layers[l], f);
      if (!src) return set_error(ENNX_B200_INVALID_ARGUMENT, "missing weight tensor %d of layer %d", f, l);
      b.job[b.count++] = EsUpdateJob{const_cast<uint16_t*>(src), (uint64_t)n, 16u + 16u * (uint32_t)l + (uint32_t)f};
    }
    {
      ProfScope ps("es_update", s, 0, 0);
      ENNX_TRY(launch_es_update(b, coef, s));
    }
    b.count = 0;
  }
  return ENNX_B200_OK;
}

int32_t ennx_b200_set_perturbation_mode(int32_t mode) {
  if (mode != 0 && mode != 1) return set_error(ENNX_B200_INVALID_ARGUMENT, "perturbation mode must be 0 or 1");
  g_fused_mode = mode;
  return ENNX_B200_OK;
}

int32_t ennx_b200_l2norm_heads_bf16(uint16_t* x, int64_t rows, int32_t heads, int64_t ld, void* stream) {
  if (!x || rows <= 0 || heads <= 0) return set_error(ENNX_B200_INVALID_ARGUMENT, "l2norm_heads: empty input");
  if (ld < (int64_t)heads * HD || ld % 4 || ((uintptr_t)x & 7u))
    return set_error(ENNX_B200_INVALID_ARGUMENT, "l2norm_heads: 8-byte aligned rows with ld >= heads*128 required");
  return launch_l2norm_heads(x, ld, heads, rows, (cudaStream_t)stream);
}

int32_t ennx_b200_kda_gate_beta(const uint16_t* raw_gate, int64_t ld_gate, const uint16_t* raw_beta, int64_t ld_beta,
                                const uint16_t* decay, const uint16_t* time_bias, int64_t tokens, int32_t heads,
                                float* gate, float* beta, void* stream) {
  if (!raw_gate || !raw_beta || !decay || !time_bias || !gate || !beta || tokens <= 0 || heads <= 0)
    return set_error(ENNX_B200_INVALID_ARGUMENT, "kda_gate_beta: null or empty argument");
  if (ld_gate < (int64_t)heads * HD || ld_beta < heads)
    return set_error(ENNX_B200_INVALID_ARGUMENT, "kda_gate_beta: row strides too small");
  return launch_kda_gate(raw_gate, ld_gate, raw_beta, ld_beta, decay, nullptr, time_bias, nullptr, tokens, tokens,
                         heads, HD, gate, beta, (cudaStream_t)stream);
}

int32_t ennx_b200_kda_postprocess(const uint16_t* o, const uint16_t* gate, int64_t ld_gate, const uint16_t* norm,
                                  int64_t tokens, int32_t heads, float eps, uint16_t* out, void* stream) {
  if (!o || !gate || !norm || !out || tokens <= 0 || heads <= 0)
    return set_error(ENNX_B200_INVALID_ARGUMENT, "kda_postprocess: null or empty argument");
  if (ld_gate < (int64_t)heads * HD || ld_gate % 4 || (((uintptr_t)o | (uintptr_t)gate | (uintptr_t)out) & 7u))
    return set_error(ENNX_B200_INVALID_ARGUMENT, "kda_postprocess: 8-byte aligned rows with ld >= heads*128 required");
  return launch_kda_post(o, gate, ld_gate, norm, nullptr, tokens, heads, tokens, eps, out, (cudaStream_t)stream);
}

int32_t ennx_b200_kda_gated(const uint16_t* qkv, int64_t ld_qkv, const uint16_t* raw_gate, int64_t ld_gate,
                            const uint16_t* raw_beta, int64_t ld_beta, const uint16_t* decay, const uint16_t* time_bias,
                            float* state, uint16_t* o, int32_t batch, int32_t seq, int32_t heads, void* workspace,
                            size_t workspace_bytes, void* stream) {
  if (!qkv || !raw_gate || !raw_beta || !decay || !time_bias || !o)
    return set_error(ENNX_B200_INVALID_ARGUMENT, "kda_gated: null argument");
  const long long hw = (long long)heads * HD;
  if (ld_qkv < 3 * hw || ld_gate < hw || ld_beta < heads || ld_gate % 8)
    return set_error(ENNX_B200_INVALID_ARGUMENT, "kda_gated: row strides too small or unaligned");
  KdaRawGate rg;
  memset(&rg, 0, sizeof(rg));
  rg.f = raw_gate; rg.ldf = ld_gate;
  rg.rbeta = raw_beta; rg.ldb = ld_beta;
  rg.decay0 = rg.decay1 = decay;
  rg.tb0 = rg.tb1 = time_bias;
  rg.split_seq = batch;
  rg.active = 1;
  return launch_kda_chunked(qkv, qkv + hw, qkv + 2 * hw, ld_qkv, nullptr, nullptr, state, o, hw, batch, seq, heads,
                            workspace, workspace_bytes, (cudaStream_t)stream, &rg);
}

}  // extern "C"
