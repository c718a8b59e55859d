// kernels.cuh -- internal launchers shared by the C-ABI entry points and the
// population-forward orchestrator.  All launch on `s`, validate their own
// shape contract, and return an ENNX_B200_* status.
#pragma once
#include "common.cuh"

namespace ennx {

// norm.cu
int32_t launch_rmsnorm(const uint16_t* x, long long ldx, const uint16_t* w0, const uint16_t* w1, long long split,
                       uint16_t* out, long long ldo, long long rows, int width, float eps, cudaStream_t s);
// noise (nullable): rows of set 0 are t0 + noise, set 1 t0 - noise
int32_t launch_embed(const int* tokens, const uint16_t* t0, const uint16_t* t1, long long per_set, long long rows,
                     int width, int vocab, uint16_t* out, cudaStream_t s, const uint16_t* noise = nullptr);
int32_t launch_l2norm_heads(uint16_t* base, long long ld, int heads, long long rows, cudaStream_t s);
int32_t launch_kda_gate(const uint16_t* raw, long long ldraw, const uint16_t* rbeta, long long ldb,
                        const uint16_t* decay0, const uint16_t* decay1, const uint16_t* tb0, const uint16_t* tb1,
                        long long split, long long rows, int heads, int head_width, float* gate, float* beta,
                        cudaStream_t s);
int32_t launch_kda_post(const uint16_t* o, const uint16_t* og, long long ldog, const uint16_t* n0, const uint16_t* n1,
                        long long split, int heads, long long rows, float eps, uint16_t* out, cudaStream_t s);
int32_t launch_rope(uint16_t* base, long long ld, int heads, int dim, long long rows, int seq, float theta,
                    cudaStream_t s);

// moe.cu
int32_t launch_router_topk(const uint16_t* x, long long ldx, const uint16_t* w0, const uint16_t* w1, long long split,
                           long long tokens, int hidden, int experts, int top_k, float* logits, int* idx,
                           float* gate, cudaStream_t s,
                           int* counts = nullptr,
                           // optional scratch of 2 * ceil(experts / 64) * hidden * 64 floats: the
                           // router weights converted once per call instead of once per block
                           float* wt = nullptr);
// Expert-major permutation and row copy in one pass.  Group of (token t,
// rank r) is set(t) * experts + idx[t, r] (set = t >= split); `counts` are the
// per-group picks (launch_router_topk with counts), `cursor` int[groups]
// zeroed.  Writes offsets[groups + 1], perm_pos[t*k + r] (row of (t, r) in
// permuted order), perm_gate[pos] = gate_scale * gate (the residual scale of
// the layer folded into the combine weights) and xperm[pos] = x[t].
int32_t launch_moe_scatter_gather(const int* idx, const float* gate, float gate_scale, long long tokens, int top_k,
                                  int experts, long long split, int sets, const int* counts, int* offsets, int* cursor,
                                  int* perm_pos, float* perm_gate, const uint16_t* x, long long ldx, int width,
                                  uint16_t* xperm, cudaStream_t s);
// hidden[t] = residual[t] + sum_r y[perm_pos[t*k + r]]
int32_t launch_moe_combine(const uint16_t* y, const int* perm_pos, long long tokens, int top_k, int width,
                           const uint16_t* residual, uint16_t* out, cudaStream_t s);

// loss.cu
int32_t launch_lse_loss(const float* lse_partial, int n_tiles, const float* target_logit, long long rows,
                        float* row_loss, cudaStream_t s);
int32_t launch_mean_per_set(const float* row_loss, long long rows_per_set, int sets, float* out, cudaStream_t s);

// attention.cu / kda.cu
int32_t launch_gqa_attention(const uint16_t* q, long long ldq, const uint16_t* k, long long ldk, const uint16_t* v,
                             long long ldv, uint16_t* o, long long ldo, int batch, int seq, int hq, int hkv,
                             cudaStream_t s);
size_t kda_workspace_bytes(int batch, int seq, int heads);
// Forward-path inputs of the chunked KDA: gates from the raw projections and
// in-kernel L2 normalisation of q and k (sequences < split_seq use set 0).
struct KdaRawGate {
  const uint16_t* f = nullptr;      // raw forget logits [T, heads*128]
  long long ldf = 0;
  const uint16_t* rbeta = nullptr;  // raw beta logits, column h of row t
  long long ldb = 0;
  const uint16_t *decay0 = nullptr, *decay1 = nullptr;  // [heads]
  const uint16_t *tb0 = nullptr, *tb1 = nullptr;        // [heads*128]
  long long split_seq = 0;
  int active = 0;
  int no_l2norm = 0;  // q and k used as given (the 16k prefill block applies no L2 norm)
};
int32_t launch_kda_chunked(const uint16_t* q, const uint16_t* k, const uint16_t* v, long long ld_qkv,
                           const float* g, const float* beta, float* state, uint16_t* o, long long ldo, int batch,
                           int seq, int heads, void* workspace, size_t workspace_bytes, cudaStream_t s,
                           const KdaRawGate* raw = nullptr, int* err_word = nullptr);

// dense.cu: W +/- sigma*eps; cols > 0 writes the [n/cols, cols] result as a
// block of a matrix with row stride dld (noise indexed by the source element)
int32_t launch_perturb_bf16(const uint16_t* w, size_t n, uint64_t seed, uint32_t pair, uint32_t tensor, float sigma,
                            uint16_t* plus, uint16_t* minus, uint32_t cols, uint64_t dld, cudaStream_t s);

// several tensors of one antithetic pair in one launch
constexpr int kMaxPerturbJobs = 16;
struct PerturbJob {
  const uint16_t* w;
  uint16_t *plus, *minus;
  uint64_t n, dld;
  uint32_t tensor, cols;
};
struct PerturbBatch {
  int count;
  uint32_t pair;
  uint64_t seed;
  float sigma;
  PerturbJob job[kMaxPerturbJobs];
  uint32_t block0[kMaxPerturbJobs + 1];  // filled by launch_perturb_batch
};
int32_t launch_perturb_batch(const PerturbBatch& batch, cudaStream_t s);

// es.cu: the zeroth-order update W <- bf16(W + sum_p coef[p] * eps_{first_pair + p})
constexpr int kMaxEsJobs = 16;
struct EsUpdateJob {
  uint16_t* w;
  uint64_t n;
  uint32_t tensor;
};
struct EsUpdateBatch {
  int count, pairs;
  uint32_t first_pair;
  uint64_t seed;
  EsUpdateJob job[kMaxEsJobs];
  uint32_t block0[kMaxEsJobs + 1];  // filled by launch_es_update
};
int32_t launch_es_update(const EsUpdateBatch& batch, const float* coef, cudaStream_t s);
int32_t launch_es_coefficients(const float* fitness, int pairs, float sigma, float lr, int total_pairs, float* coef,
                               cudaStream_t s);

// gemm.cu (internal form of ennx_b200_gemm_bf16)
int32_t gemm_bf16(const ennx_b200_gemm_params* p, const uint16_t* a, const uint16_t* b, void* c, cudaStream_t s);
// gemm.cu: W +/- E formed in the operand path (ennx_b200_gemm_bf16_perturbed)
int32_t gemm_bf16_perturbed(const ennx_b200_gemm_params* p, const uint16_t* a, const uint16_t* w, const uint16_t* e,
                            void* c, cudaStream_t s);

}  // namespace ennx
