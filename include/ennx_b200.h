/*
 * ennx_b200.h -- C ABI of the B200-native (sm_100a) model-evaluation hot path.
 *
 * Drop-in boundary for the GPU path of Kvutza/ennx.  Conventions follow the
 * reference's existing C ABI (zig/include/ennx.h:11-65: int32 status, POD
 * structs, size_t counts) and the public surface of its `ennx-cuda` crate
 * (cuda/src/lib.rs:13-27, 1084-1430).  Each entry point names the reference
 * interface it replaces.  Citations are file:line inside Kvutza/ennx.
 *
 * Common rules
 *   - Every pointer argument documented "device" is a CUDA device pointer on
 *     the current device; the caller owns it (zero copy).  Pointers documented
 *     "host" are read before the call returns.
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default stream).
 *     Calls are asynchronous on `stream` unless documented "synchronises".
 *   - Status codes below; on failure a description is available from
 *     ennx_b200_last_error() (thread-local).  Nothing aborts the process.
 *   - Device kernels never trap or spin forever: every wait is bounded and a
 *     timeout is reported as ENNX_B200_TIMEOUT by the next synchronising call
 *     or by ennx_b200_device_status().
 *   - Handles / workspaces are not thread-safe; use one per thread and device.
 */
#ifndef ENNX_B200_H
#define ENNX_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ENNX_B200_ABI_VERSION 1u

#if defined(__GNUC__)
#define ENNX_B200_API __attribute__((visibility("default")))
#else
#define ENNX_B200_API
#endif

enum {
    ENNX_B200_OK = 0,               /* == ENNX_OK (zig/include/ennx.h:12) */
    ENNX_B200_INVALID_ARGUMENT = 1, /* == ENNX_INVALID_ARGUMENT (zig/include/ennx.h:13) */
    ENNX_B200_OVERFLOW = 2,         /* "perturbation overflowed" (dense/bf16.rs:254) */
    ENNX_B200_CUDA_ERROR = 3,
    ENNX_B200_TIMEOUT = 4,          /* a bounded device wait expired */
    ENNX_B200_UNSUPPORTED = 5       /* device is not sm_100 or shape outside the kernels' contract */
};

/* Same layout as ennx_dense_leaf / ennx_dense_term / ennx_dense_view
 * (zig/include/ennx.h:16-32) and DenseLeaf/DenseTerm/DenseView
 * (rust/crates/ennx/src/dense.rs:24-48, dense/linear.rs:14-20). */
typedef struct { uint64_t key; size_t offset; size_t len; float scale; } ennx_b200_dense_leaf;
typedef struct { uint64_t seed; float coefficient; } ennx_b200_dense_term;
typedef struct { uint64_t key; uint64_t start; float scale; } ennx_b200_dense_view;

/* ---- library ---------------------------------------------------------- */

/* Replaces ennx_abi_version (zig/include/ennx.h:34). Returns ENNX_B200_ABI_VERSION. */
ENNX_B200_API uint32_t ennx_b200_abi_version(void);
/* Thread-local description of the last failure ("" if none). */
ENNX_B200_API const char* ennx_b200_last_error(void);
/* ENNX_B200_OK if the current device is an sm_100 part this library was built for. */
ENNX_B200_API int32_t ennx_b200_device_check(void);
/* Synchronises `stream`, then returns and clears the device error word
 * (ENNX_B200_TIMEOUT if any kernel gave up on a bounded wait). */
ENNX_B200_API int32_t ennx_b200_device_status(void* stream);

/* ---- seeded dense perturbation (the existing CUDA drop-in) ------------- */

/* out = base + scale * sum(c_i * sign_i), with the one-ulp rule.  Replaces
 * `dense_apply` (cuda/src/lib.rs:1084-1124; CPU ennx_dense_apply_f32,
 * zig/include/ennx.h:36-44).  base/out: device float[num_values];
 * leaves/terms: host.  out_changed (host, nullable) receives num_values on
 * success.  Synchronises; ENNX_B200_OVERFLOW if any output is non-finite. */
ENNX_B200_API int32_t ennx_b200_dense_apply_f32(const float* base, size_t num_values,
                                  const ennx_b200_dense_leaf* leaves, size_t num_leaves,
                                  const ennx_b200_dense_term* terms, size_t num_terms,
                                  float* out, size_t* out_changed, void* stream);

/* BF16 materialisation with per-tile overflow status and rollback to base.
 * Replaces Bf16Engine::materialize (cuda/src/lib.rs:1211-1252).
 * base/out: device uint16 (bf16 bits)[num_values].  Synchronises; on
 * overflow out is restored to base and ENNX_B200_OVERFLOW is returned. */
ENNX_B200_API int32_t ennx_b200_dense_apply_bf16(const uint16_t* base, size_t num_values,
                                   const ennx_b200_dense_leaf* leaves, size_t num_leaves,
                                   const ennx_b200_dense_term* terms, size_t num_terms,
                                   uint16_t* out, void* stream);

/* *out_distance = (sum over leaves of len * scale^2) * sum over seeds of
 * (c_left(seed) - c_right(seed))^2: the squared L2 distance between the two
 * perturbations.  Replaces ennx_dense_dist2 (zig/include/ennx.h:46-53), same
 * argument order; host memory only, no device work.  Empty term lists are
 * allowed; leaves must be contiguous from offset 0. */
ENNX_B200_API int32_t ennx_b200_dense_dist2(const ennx_b200_dense_leaf* leaves, size_t num_leaves,
                              const ennx_b200_dense_term* left, size_t num_left,
                              const ennx_b200_dense_term* right, size_t num_right, double* out_distance);

/* *all_finite (host) = 1 iff every bf16 value is finite.  Replaces the
 * check_bf16 kernel path (cuda/kernels/src/lib.rs:2311-2354).  Synchronises. */
ENNX_B200_API int32_t ennx_b200_check_bf16(const uint16_t* values, size_t num_values, int32_t* all_finite,
                             void* stream);

/* Fused perturbed GEMV y = W~ x (+ b~).  Replaces DenseLinearEngine::eval
 * (cuda/src/lib.rs:1339-1429) and ennx_dense_linear_f32
 * (zig/include/ennx.h:55-65), same argument order.  input/weight/bias/out:
 * device (bias nullable); terms: host.  Asynchronous. */
ENNX_B200_API int32_t ennx_b200_dense_linear_f32(const float* input, size_t columns, const float* weight,
                                   size_t rows, const float* bias,
                                   ennx_b200_dense_view weight_view, ennx_b200_dense_view bias_view,
                                   const ennx_b200_dense_term* terms, size_t num_terms, float* out,
                                   void* stream);

/* ---- population noise (no reference counterpart: the reference draws
 *      Rademacher signs; BASELINE asks for Philox Gaussian noise) --------- */

/* Noise step e = bf16(sigma*eps) (RNE), eps = Philox4x32-10 Box-Muller
 * normal of (seed, pair, tensor, element); out_plus = bf16(W + e), out_minus =
 * bf16(W - e) (nullable), each one RNE rounding of the exact sum -- the
 * values ennx_b200_gemm_bf16_perturbed forms from W and e.  w == NULL:
 * out_plus receives e itself (out_minus must be NULL).  w/out_*: device bf16
 * bits[n].  Asynchronous. */
ENNX_B200_API int32_t ennx_b200_perturb_bf16(const uint16_t* w, size_t n, uint64_t seed, uint32_t pair,
                               uint32_t tensor, float sigma, uint16_t* out_plus,
                               uint16_t* out_minus, void* stream);

/* ---- dense contractions ------------------------------------------------ */

enum {
    ENNX_B200_EPI_BF16 = 0,     /* C[bf16] = alpha*acc (+ residual)               */
    ENNX_B200_EPI_F32 = 1,      /* C[f32]  = alpha*acc                            */
    ENNX_B200_EPI_SWIGLU = 2,   /* C[bf16, N/2 cols] = silu(gate) * up, see below */
    ENNX_B200_EPI_ROWSCALE = 3, /* C[bf16] = row_scale[r] * acc                   */
    ENNX_B200_EPI_LSE = 4       /* per-row logsumexp partials + target logit      */
};

/* C = A . B^T with A [M, K] and B [N, K] bf16 row-major (K contiguous), fp32
 * accumulation on tcgen05 tensor cores (TMEM accumulators, TMA-fed).
 * The reference has no GEMM; the nearest operator is the fused linear
 * (dense/linear.rs:484-519: C[m,:] = linear(A[m,:], B)).
 *
 * Grouping: rows of A/C are split into `groups` contiguous segments; group g
 * uses rows [g*b_group_rows, g*b_group_rows + N) of B (b_group_rows = 0: all
 * groups share rows [0, N)).
 * Segment bounds come from `group_offsets` (device int32[groups+1]) or, when
 * it is NULL, from equal segments of M/groups rows.
 *
 * Epilogues: EPI_SWIGLU expects B's rows in blocks of 256 = [128 gate rows |
 * 128 up rows]; output column j of block b is silu(g)*u of row 128b+j.
 * EPI_LSE writes lse_partial[r * 2*ceil(N/256) + j] = (max, sum exp(x - max))
 * over columns [128j, 128j + 128) as float2 ((-inf, 0) for an empty range),
 * and target_logit[r] = acc[r, targets[r]].
 * Requirements: K % 64 == 0, K >= 64, lda/ldb % 8 == 0, 16-byte aligned A/B. */
typedef struct {
    int32_t m, n, k;
    int64_t lda, ldb, ldc;   /* elements */
    int32_t groups;          /* >= 1 */
    int32_t b_group_rows;    /* B row stride between groups (0: shared B) */
    const int32_t* group_offsets; /* device, nullable */
    int32_t epilogue;
    float alpha;
    const uint16_t* residual; /* EPI_BF16: device bf16 [M, ldr] added after alpha*acc; nullable */
    int64_t ldr;
    const float* row_scale;   /* EPI_ROWSCALE: device float[M] */
    const int32_t* targets;   /* EPI_LSE: device int32[M] */
    float* lse_partial;       /* EPI_LSE: device float2[M, 2*ceil(N/256)] */
    float* target_logit;      /* EPI_LSE: device float[M] */
} ennx_b200_gemm_params;

ENNX_B200_API int32_t ennx_b200_gemm_bf16(const ennx_b200_gemm_params* params, const uint16_t* a,
                            const uint16_t* b, void* c, void* stream);

/* The antithetic perturbed GEMM: the weights of candidate +/- are W + E and
 * W - E, each rounded once to bf16 (RNE of the exact sum), formed tile by tile
 * inside the GEMM's operand path and never written to memory.  E is the
 * noise operand sigma*eps (bf16, same shape and row stride ldb as W).  groups
 * = 2P: groups [0, P) hold the `+` rows and groups [P, 2P) the `-` rows;
 * groups e and P + e both use row block e of W and E (rows
 * [e*b_group_rows, e*b_group_rows + N)).  Other parameters and epilogues as
 * ennx_b200_gemm_bf16.  The fused counterpart of the reference's perturbed
 * contraction, linear_cpu / perturbed (rust/crates/ennx/src/dense/linear.rs:
 * 484-548) and dense_linear (cuda/kernels/src/lib.rs:2359-2423), which form
 * each perturbed weight inside the dot product. */
ENNX_B200_API int32_t ennx_b200_gemm_bf16_perturbed(const ennx_b200_gemm_params* params, const uint16_t* a,
                                                    const uint16_t* w, const uint16_t* e, void* c, void* stream);

/* ---- forward-path operators (no reference counterpart unless cited) ---- */

/* out = x * rsqrt(mean(x^2) + eps) * w per row; x/out bf16 [rows, width],
 * w bf16 [width]; width % 256 == 0.  Restates decoder_rms_norm
 * (rust/crates/ennx/src/kda_moe.metal:536-554). */
ENNX_B200_API int32_t ennx_b200_rmsnorm_bf16(const uint16_t* x, const uint16_t* w, int64_t rows, int32_t width,
                                             float eps, uint16_t* out, void* stream);

/* Router logits (fp32, one serial fma chain over the hidden index per logit,
 * the reference's loop order, bit-identical to the CPU oracle), top-k with
 * strict '>' (ties keep the lower expert index) and softmax over the kept
 * logits.  Replaces moe_router_topk (kda_moe.metal:570-621); top_k <= 8 as
 * KdaMoeLayerRequest::validate (forward_program.rs:428).  x bf16 [tokens,
 * hidden], w_router bf16 [experts, hidden], hidden % 32 == 0, experts <= 256.
 * logits (nullable) f32 [tokens, experts]; index i32 / gate f32 [tokens, top_k]. */
ENNX_B200_API int32_t ennx_b200_moe_route(const uint16_t* x, const uint16_t* w_router, int64_t tokens,
                                          int32_t hidden, int32_t experts, int32_t top_k, float* logits,
                                          int32_t* index, float* gate, void* stream);

/* Full MoE layer y = sum_r gate_r * W_d[e_r] (silu(W_g[e_r] x) * W_u[e_r] x):
 * router + expert-major permutation + grouped tcgen05 gate/up GEMM with a
 * SwiGLU epilogue + grouped down GEMM + weighted combine (+ residual).
 * Restates moe_gate_up / moe_down (kda_moe.metal:691-755).
 * w_gate_up bf16 [experts, 2*I, hidden] in blocks of 256 rows =
 * [128 gate rows | 128 up rows]; w_down bf16 [experts, hidden, I]; I % 128 == 0.
 * residual (nullable) is added to y.  index/gate outputs (nullable) receive the
 * routing.  workspace >= ennx_b200_moe_workspace_size(tokens, hidden, experts,
 * top_k, I) bytes of device memory. */
ENNX_B200_API size_t ennx_b200_moe_workspace_size(int64_t tokens, int32_t hidden, int32_t experts, int32_t top_k,
                                                  int32_t expert_width);
ENNX_B200_API int32_t ennx_b200_moe_layer(const uint16_t* x, const uint16_t* w_router, const uint16_t* w_gate_up,
                                          const uint16_t* w_down, int64_t tokens, int32_t hidden, int32_t experts,
                                          int32_t top_k, int32_t expert_width, const uint16_t* residual,
                                          uint16_t* y, int32_t* index, float* gate, void* workspace,
                                          size_t workspace_bytes, void* stream);

/* Causal GQA attention, head_dim 128, softmax scale 1/sqrt(128), fp32
 * softmax statistics.  q bf16 [batch, seq, hq, 128], k/v [batch, seq, hkv,
 * 128], o [batch, seq, hq, 128].  If rope_theta > 0, rotary embedding
 * (rotate-half pairing, position = sequence index) is applied to q and k IN
 * PLACE first. */
ENNX_B200_API int32_t ennx_b200_gqa_attention(uint16_t* q, uint16_t* k, const uint16_t* v, uint16_t* o,
                                              int32_t batch, int32_t seq, int32_t hq, int32_t hkv,
                                              float rope_theta, void* stream);

/* Chunked KDA (gated delta rule, per-key-channel decay, chunk 64, d_k = d_v =
 * 128), equivalent to the serial recurrence of kda_recurrence_16k
 * (kda_moe.metal:167-225).  q, k, v bf16 [batch, seq, heads, 128]; g f32
 * [batch, seq, heads, 128] (log decay per step); beta f32 [batch, seq, heads];
 * state f32 [batch, heads, 128, 128] (nullable: zero initial state, final
 * state discarded; otherwise read as the initial state and overwritten with
 * the final state); o bf16 [batch, seq, heads, 128], scaled by 1/sqrt(128).
 * workspace (device, 16-byte aligned) >= ennx_b200_kda_workspace_size(batch,
 * seq, heads) bytes holds the per-chunk operands of the two-phase scheme. */
ENNX_B200_API size_t ennx_b200_kda_workspace_size(int32_t batch, int32_t seq, int32_t heads);
ENNX_B200_API int32_t ennx_b200_kda_chunked(const uint16_t* q, const uint16_t* k, const uint16_t* v, const float* g,
                                            const float* beta, float* state, uint16_t* o, int32_t batch,
                                            int32_t seq, int32_t heads, void* workspace, size_t workspace_bytes,
                                            void* stream);

/* Same operation as ennx_b200_kda_chunked for callers that cannot allocate
 * device memory (code inside a CUDA graph being captured, hosts that reserve
 * all device memory for their own pool, latency-critical embedders).  No
 * counterpart exists in the reference.  The per-chunk scratch comes from one
 * 32 MiB static device array that every GPU loading this library holds until
 * exit, so batch * heads * ceil(seq / 64) must stay <= 508 (66 048 bytes per
 * chunk record); larger problems are rejected with ENNX_B200_INVALID_ARGUMENT.
 * Calls allocate nothing (no cudaMalloc/cudaFree, no allocating library
 * call, and no lazily allocated status word either: a device wait that
 * gives up writes ENNX_B200_TIMEOUT to a static status word of this path).
 * The first call on a device looks up the addresses of the array and of that
 * word (cudaGetSymbolAddress) with that device current; make that first call
 * before any stream capture.  Every call shares the one array: calls that
 * overlap on the GPU (different streams, or threads) race on it.  A call
 * that returned early leaves a partial o/state; ennx_b200_device_status(stream)
 * (outside any capture: it synchronises the stream) reports it and clears
 * the word, and itself allocates nothing when no regular entry point ran. */
ENNX_B200_API int32_t ennx_b200_kda_chunked_noalloc(const uint16_t* q, const uint16_t* k, const uint16_t* v,
                                                    const float* g, const float* beta, float* state,
                                                    uint16_t* o, int32_t batch, int32_t seq, int32_t heads,
                                                    void* stream);

/* ---- population forward: the hybrid KDA/GQA-MoE decoder --------------- */

typedef struct {
    int32_t layers, hidden, vocab;
    int32_t attn_period;   /* layer l is GQA iff l % attn_period == attn_period - 1 (0: no GQA) */
    int32_t q_heads, kv_heads;       /* GQA, head_dim 128 */
    int32_t kda_heads, gate_rank;    /* KDA, head_dim 128 */
    int32_t experts, top_k, expert_width;
    float rms_eps, rope_theta;
    float residual_scale;  /* h + s*u at both residual adds of a layer (decoder_residual,
                              kda_moe.metal:556-565); finite; 1 for the plain residual */
} ennx_b200_model_config;

/* Device pointers, bf16.  KDA layers use every field; GQA layers use
 * attn_norm, w_qkv, w_o and the MoE fields. */
typedef struct {
    const uint16_t* attn_norm;   /* [H] */
    const uint16_t* w_qkv;       /* KDA [3*Hk*128, H]; GQA [(Hq + 2*Hkv)*128, H] */
    const uint16_t* w_ctl;       /* KDA [2*rank + Hk, H] = forget state | output state | beta,
                                    the control layout of kda_split_control_16k (kda_moe.metal:847-867) */
    const uint16_t* w_forget;    /* KDA [Hk*128, rank] */
    const uint16_t* w_ogate;     /* KDA [Hk*128, rank] */
    const uint16_t* decay;       /* KDA [Hk] */
    const uint16_t* time_bias;   /* KDA [Hk*128] */
    const uint16_t* out_norm;    /* KDA [128] */
    const uint16_t* w_o;         /* [H, heads*128] */
    const uint16_t* moe_norm;    /* [H] */
    const uint16_t* w_router;    /* [E, H] */
    const uint16_t* w_gate_up;   /* [E, 2*I, H], blocks of [128 gate | 128 up] rows */
    const uint16_t* w_down;      /* [E, H, I] */
} ennx_b200_layer_weights;

typedef struct {
    const uint16_t* embedding;   /* [V, H]; also the (tied) LM head */
    const uint16_t* final_norm;  /* [H] */
    const ennx_b200_layer_weights* layers; /* host array [layers] */
} ennx_b200_model_weights;

/* Evaluates antithetic pairs [first_pair, first_pair + num_pairs) of a
 * zeroth-order population: candidate 2p+0 uses W + sigma*eps_p, 2p+1 uses
 * W - sigma*eps_p (every weight tensor t, eps = Philox normal of (seed, p, t,
 * element), tensor ids: embedding 0, final_norm 1, field f of layer l
 * 16 + 16*l + f).  Each candidate is scored by the mean next-token
 * cross-entropy on tokens (device int32 [batch, seq + 1]: inputs [:, :seq],
 * targets [:, 1:]).  fitness (device f32 [2*num_pairs]) receives candidate
 * 2i+s of the range at index 2i+s.  This is the ForwardEvaluator seam of
 * the reference (forward_program.rs:210-212) for a whole population.
 * workspace >= ennx_b200_population_workspace_size(cfg, batch, seq). */
ENNX_B200_API size_t ennx_b200_population_workspace_size(const ennx_b200_model_config* cfg, int32_t batch,
                                                         int32_t seq);
ENNX_B200_API int32_t ennx_b200_population_forward(const ennx_b200_model_config* cfg,
                                                   const ennx_b200_model_weights* weights, uint64_t seed,
                                                   float sigma, int32_t first_pair, int32_t num_pairs,
                                                   const int32_t* tokens, int32_t batch, int32_t seq,
                                                   float* fitness, void* workspace, size_t workspace_bytes,
                                                   void* stream);

/* ---- the zeroth-order update (the population's tell) ------------------- */

/* coef[p] = -lr * (fitness[2p] - fitness[2p+1]) / (2 * sigma * total_pairs),
 * p < pairs: the antithetic estimator of the mean cross-entropy's gradient,
 * as a step that lowers it.  fitness, coef: device f32. */
ENNX_B200_API int32_t ennx_b200_es_coefficients(const float* fitness, int32_t pairs, int32_t total_pairs,
                                                float sigma, float lr, float* coef, void* stream);
/* In place: w[i] = bf16(w[i] + sum_{p < pairs} coef[p] * eps(seed, first_pair + p,
 * tensor, i)) with the fp32 sum taken over p in order and one RNE rounding;
 * eps is the forward's Philox normal.  pairs <= 256.  Counterpart of the
 * reference's device tell that moves the incumbent from a round's rewards
 * (rust/crates/ennx/src/bf16_search.rs:319-407, cuda/kernels/src/lib.rs:409-535). */
ENNX_B200_API int32_t ennx_b200_es_update_bf16(uint16_t* w, size_t n, uint64_t seed, uint32_t tensor,
                                               const float* coef, uint32_t first_pair, uint32_t pairs,
                                               void* stream);
/* ennx_b200_es_update_bf16 over every tensor of the model (the forward's
 * tensor ids), writing through the device pointers of `weights`; one launch
 * per layer.  Every rank applies it with the same broadcast coefficients, so
 * the replicas stay identical without moving any weight. */
ENNX_B200_API int32_t ennx_b200_population_update(const ennx_b200_model_config* cfg,
                                                  const ennx_b200_model_weights* weights, uint64_t seed,
                                                  const float* coef, int32_t first_pair, int32_t num_pairs,
                                                  void* stream);

/* Process-wide choice of how the population forward applies each pair's
 * perturbation (both give the same perturbed weights bit for bit):
 * 0 (default) materialised -- the noise kernel writes bf16(W + e) and
 * bf16(W - e) copies of every tensor and the GEMMs read them; 1 fused --
 * only the noise step e of the matrices is written and every GEMM forms
 * W + e and W - e in its operand path (ennx_b200_gemm_bf16_perturbed).  The
 * workspace size does not depend on the mode.  Not thread-safe against
 * concurrent forward calls. */
ENNX_B200_API int32_t ennx_b200_set_perturbation_mode(int32_t mode);

/* Per-layer parity probe of the population forward: runs antithetic pair
 * `pair` through the first `layers` decoder layers only and copies the
 * residual stream after them to hidden (device bf16 [2][batch*seq][hidden],
 * sign + first), instead of the LM head; index (nullable, device int32
 * [2][batch*seq][top_k]) receives the expert choices of the last of those
 * layers.  Same arguments and workspace as
 * ennx_b200_population_forward.  No counterpart in the reference (its
 * Metal executor exposes per-layer outputs only through its own buffers,
 * forward_metal.rs:614-810). */
ENNX_B200_API int32_t ennx_b200_population_hidden(const ennx_b200_model_config* cfg,
                                                  const ennx_b200_model_weights* weights, uint64_t seed,
                                                  float sigma, int32_t pair, int32_t layers,
                                                  const int32_t* tokens, int32_t batch, int32_t seq,
                                                  uint16_t* hidden, int32_t* index, void* workspace,
                                                  size_t workspace_bytes, void* stream);

/* ---- KDA element-wise stages (the 16k-prefill kernels of kda_moe.metal) --- */

/* In-place per-head L2 normalisation of bf16 rows (x[r, h*128 .. +127] /=
 * max(|x|, 1e-6)), kda_normalize_qk (kda_moe.metal:510-534). */
ENNX_B200_API int32_t ennx_b200_l2norm_heads_bf16(uint16_t* x, int64_t rows, int32_t heads, int64_t ld,
                                                  void* stream);
/* gate[t, j] = max(-exp(decay[j/128]) * softplus(raw_gate[t, j] + time_bias[j]), -5),
 * beta[t, h] = sigmoid(raw_beta[t, h]); f32 outputs [tokens, heads*128] and
 * [tokens, heads]; kda_make_gate_beta_16k + softplus_stable
 * (kda_moe.metal:869-895). */
ENNX_B200_API int32_t ennx_b200_kda_gate_beta(const uint16_t* raw_gate, int64_t ld_gate, const uint16_t* raw_beta,
                                              int64_t ld_beta, const uint16_t* decay, const uint16_t* time_bias,
                                              int64_t tokens, int32_t heads, float* gate, float* beta,
                                              void* stream);
/* out[t, h, :] = o[t, h, :] * rsqrt(mean(o[t, h, :]^2) + eps) * norm * sigmoid(gate[t, h*128 + :]),
 * kda_postprocess_16k (kda_moe.metal:898-921). */
ENNX_B200_API int32_t ennx_b200_kda_postprocess(const uint16_t* o, const uint16_t* gate, int64_t ld_gate,
                                                const uint16_t* norm, int64_t tokens, int32_t heads, float eps,
                                                uint16_t* out, void* stream);
/* The forward's fused KDA: q, k, v are columns [0, hw), [hw, 2hw), [2hw, 3hw)
 * of qkv rows (hw = heads*128, q and k NOT yet normalised); the chunk
 * preparation applies the per-head L2 norm of q and k (rounded to bf16) and
 * forms g and beta from the raw projections exactly as
 * ennx_b200_l2norm_heads_bf16 / ennx_b200_kda_gate_beta define them, then
 * runs the chunked recurrence of ennx_b200_kda_chunked. */
ENNX_B200_API int32_t ennx_b200_kda_gated(const uint16_t* qkv, int64_t ld_qkv, const uint16_t* raw_gate,
                                          int64_t ld_gate, const uint16_t* raw_beta, int64_t ld_beta,
                                          const uint16_t* decay, const uint16_t* time_bias, float* state,
                                          uint16_t* o, int32_t batch, int32_t seq, int32_t heads,
                                          void* workspace, size_t workspace_bytes, void* stream);

/* ---- packed int4/int8 linear (KdaPackedLinear) ------------------------- */

/* Packed affine weights of the reference's native KDA-MoE model: field order
 * of KdaPackedLinear (rust/crates/ennx/src/forward_program.rs:224-235); the
 * arenas (`weights` u8, `scales`/`biases` f32) are indexed by the offsets.
 * Code of (row, column): bits 4 -> two codes per byte, low nibble first;
 * bits 8 -> one byte; rows start every ceil(input_width * bits / 8) bytes.
 * Weight = code' * scale[row, group] + bias[row, group] (one fused
 * multiply-add), group = min(column / group_size, groups - 1). */
typedef struct {
    uint64_t byte_offset, scale_offset, bias_offset;
    uint64_t input_width, output_width;
    uint32_t bits;          /* 4 or 8 */
    uint32_t group_size;
    uint64_t element_offset;
    uint32_t perturb_whole, perturb_threshold;
} ennx_b200_packed_linear;

/* PerturbSeed of kda_moe.metal:56-61: when `enabled`, code' is the integer
 * code moved by whole (+1 with probability threshold/2^32) with reflection at
 * the code range, driven by the Metal perturb_hash of (seed, element_offset +
 * row * input_width + column) in 32-bit arithmetic (kda_moe.metal:63-96). */
typedef struct {
    uint32_t low, high, enabled;
} ennx_b200_perturb_seed;

/* Dequantise (and perturb) all rows into out[output_width, input_width]:
 * packed_dequantize_row_half / _float (kda_moe.metal:451-476) for every row.
 * Errors as KdaPackedLinear::validate (forward_program.rs:238-249). */
ENNX_B200_API int32_t ennx_b200_packed_dequantize_bf16(const uint8_t* weights, const float* scales,
                                                       const float* biases, const ennx_b200_packed_linear* linear,
                                                       ennx_b200_perturb_seed seed, uint16_t* out, void* stream);
ENNX_B200_API int32_t ennx_b200_packed_dequantize_f32(const uint8_t* weights, const float* scales,
                                                      const float* biases, const ennx_b200_packed_linear* linear,
                                                      ennx_b200_perturb_seed seed, float* out, void* stream);

/* out[t, r] = sum_c x[t, c] * W'[r, c] for tokens x bf16 [tokens,
 * input_width]: decoder_project_packed (kda_moe.metal:399-420) for M
 * tokens, as dequantise-into-workspace + tcgen05 GEMM (fp32 accumulation,
 * bf16 out).  input_width % 64 == 0.  workspace >=
 * ennx_b200_packed_linear_workspace_size(linear) bytes. */
ENNX_B200_API size_t ennx_b200_packed_linear_workspace_size(const ennx_b200_packed_linear* linear);
ENNX_B200_API int32_t ennx_b200_packed_linear_bf16(const uint16_t* x, int64_t tokens, const uint8_t* weights,
                                                   const float* scales, const float* biases,
                                                   const ennx_b200_packed_linear* linear,
                                                   ennx_b200_perturb_seed seed, uint16_t* out, void* workspace,
                                                   size_t workspace_bytes, void* stream);

/* ---- packed KDA attention block over whole sequences (16k prefill) ------ */

/* Descriptors of one layer's KDA block in a package (names as in the
 * package: layers.<i>.attention.{qkv, control, forget_b, gate_b, output,
 * decay, time_bias, output_norm}); the vectors are one-row linears. */
typedef struct {
    ennx_b200_packed_linear qkv;          /* [3*heads*128, hidden] */
    ennx_b200_packed_linear control;      /* [2*rank + heads, hidden]: forget state | output state | beta */
    ennx_b200_packed_linear forget_b;     /* [heads*128, rank] */
    ennx_b200_packed_linear gate_b;       /* [heads*128, rank] */
    ennx_b200_packed_linear output;       /* [hidden, heads*128] */
    ennx_b200_packed_linear decay;        /* [1, heads] */
    ennx_b200_packed_linear time_bias;    /* [1, heads*128] */
    ennx_b200_packed_linear output_norm;  /* [1, 128] */
    int32_t heads, gate_rank;
    float rms_eps, residual_scale;
} ennx_b200_packed_kda_block;

/* The KDA attention update of KdaMoeMetalExecutor::kda (forward_metal.rs:
 * 997-1129: packed qkv and control projections, splits, forget / output-gate
 * projections, gate and beta, the gated delta recurrence, per-head norm x
 * sigmoid(output gate), output projection, residual) for `batch` sequences
 * of any length `seq` (the reference requires 16384): hidden (device bf16
 * [batch*seq, hidden_width]) += residual_scale * update, computed from
 * `normalized` (the RMS-normalised input, same shape).  Like that path it
 * applies no short convolution and no q/k L2 norm.  `seed` is the integer-
 * code perturbation of every projection (PerturbSeed).  state (nullable,
 * f32 [batch, heads, 128, 128]) is the recurrent state in and out.  heads*128
 * key/value width, gate_rank and hidden_width multiples of 64.  workspace:
 * 256-byte aligned, >= ennx_b200_packed_kda_prefill_workspace_size bytes. */
ENNX_B200_API size_t ennx_b200_packed_kda_prefill_workspace_size(const ennx_b200_packed_kda_block* block,
                                                                 int32_t batch, int32_t seq, int32_t hidden_width);
ENNX_B200_API int32_t ennx_b200_packed_kda_prefill(const uint8_t* weights, const float* scales, const float* biases,
                                                   const ennx_b200_packed_kda_block* block,
                                                   ennx_b200_perturb_seed seed, const uint16_t* normalized,
                                                   uint16_t* hidden, float* state, int32_t batch, int32_t seq,
                                                   int32_t hidden_width, void* workspace, size_t workspace_bytes,
                                                   void* stream);

/* ---- resident BF16 TuRBO search (replaces the Bf16SearchEngine of the
 *      ennx-cuda crate, cuda/src/bf16_search.rs:129-1067, and its kernels
 *      distance_bf16 / score_bf16 / draw_bf16 / seed_bf16 / pick_trial /
 *      write_bf16 / tell_bf16 / check_search, cuda/kernels/src/lib.rs:1310-2308)
 *
 * A handle owns `slots` device rows of the model (slot 0 = incumbent, slots
 * 1..capacity = trust-region history, the rest = pending trials), the
 * history outcomes and the trust-region state, all in device memory, so
 * that ask -> evaluate -> tell rounds need no host round trip.  Calls are
 * enqueued on the stream given at creation; those documented as
 * synchronising wait for it.  A handle is not thread-safe. ---------------- */

/* Same layout as Bf16Leaf (cuda/kernels/src/bf16.rs:5-13). */
typedef struct {
    uint64_t key;
    uint64_t offset;
    uint64_t length;
    float scale;
    float weight;   /* multiplies the squared distance of this leaf's elements */
} ennx_b200_bf16_leaf;

/* Same layout as Selection (cuda/kernels/src/lib.rs:41-47). */
typedef struct {
    uint32_t index;   /* candidate index over all regions */
    float score;
} ennx_b200_selection;

/* Acquisition settings of one ask (ennx_cuda::Ask, cuda/src/lib.rs).
 * acquisition: 0 = UCB (mean + beta*se), 1 = Thompson (mean + se*N(0,1)),
 * 2 = Pareto (mean + se). */
typedef struct {
    uint32_t neighbors;
    uint32_t acquisition;
    float epistemic_scale;
    float aleatoric_scale;
    float y_scale;
    float beta;
} ennx_b200_ask_config;

/* Same fields as TellSummary (cuda/kernels/src/bf16.rs:63-72). */
typedef struct {
    double length;
    float best;
    float best_variance;
    uint32_t history;
    uint32_t restarts;
    uint32_t restarted;
    uint32_t status;   /* nonzero: the proposals or rewards were invalid */
} ennx_b200_tell_summary;

typedef struct ennx_b200_bf16_search ennx_b200_bf16_search;

/* Copy `len` BF16 values from device memory `base` into slot 0 of a new
 * handle with `slots` rows (>= 2).  Leaves must tile [0, len) contiguously,
 * with positive finite scales and weights; base values must be finite.
 * Bf16SearchEngine::from_device (cuda/src/bf16_search.rs:166-188).
 * Synchronises. */
ENNX_B200_API int32_t ennx_b200_bf16_search_create(const uint16_t* base, size_t len,
                                                   const ennx_b200_bf16_leaf* leaves, size_t num_leaves,
                                                   size_t slots, void* stream, ennx_b200_bf16_search** out);
ENNX_B200_API int32_t ennx_b200_bf16_search_destroy(ennx_b200_bf16_search* search);
/* Trust-region state and a one-row history (slot 1, value base_value);
 * init_search (bf16_search.rs:243-293).  capacity <= 128. */
ENNX_B200_API int32_t ennx_b200_bf16_search_init(ennx_b200_bf16_search* search, float base_value,
                                                 float base_variance, size_t capacity, double length_init,
                                                 double length_min, double length_max);
/* Device copy of one row slot onto another (copy_row, bf16_search.rs:889-904). */
ENNX_B200_API int32_t ennx_b200_bf16_search_copy_row(ennx_b200_bf16_search* search, size_t source,
                                                     size_t destination);
/* Score regions*candidates_per_region seeded candidates (host `seeds`)
 * around row `base_slot` with step `coefficient` against the first
 * `history` rows of the history, pick the best per region and write it
 * into `trial_slots[r]` and row r of the batch.  Writes `regions`
 * selections (host).  On an overflowing candidate the trial rows are reset
 * to the base row and ENNX_B200_OVERFLOW is returned.  Bf16SearchEngine::ask
 * (bf16_search.rs:518-556).  Synchronises. */
ENNX_B200_API int32_t ennx_b200_bf16_search_ask(ennx_b200_bf16_search* search, size_t base_slot, size_t history,
                                                const uint32_t* trial_slots, size_t regions,
                                                const uint64_t* seeds, size_t candidates_per_region,
                                                float coefficient, uint64_t draw_seed,
                                                const ennx_b200_ask_config* config,
                                                ennx_b200_selection* selections);
/* Resident round: seeds derived on the device from `seed_root`, step and
 * history taken from the device state.  Asynchronous; errors of the
 * candidates surface at the next tell.  ask_seeded (bf16_search.rs:558-594). */
ENNX_B200_API int32_t ennx_b200_bf16_search_ask_seeded(ennx_b200_bf16_search* search, size_t base_slot,
                                                       const uint32_t* trial_slots, size_t regions,
                                                       size_t candidates_per_region, uint64_t seed_root,
                                                       uint64_t draw_seed, const ennx_b200_ask_config* config);
/* Record `count` rewards (host or device float arrays; variances nullable =
 * zeros) for the trials in `trial_slots`, update the history, the incumbent
 * row and the trust region on the device.  Asynchronous; read the outcome
 * with ennx_b200_bf16_search_collect.  tell / queue_tell
 * (bf16_search.rs:295-492). */
ENNX_B200_API int32_t ennx_b200_bf16_search_tell(ennx_b200_bf16_search* search, const uint32_t* trial_slots,
                                                 size_t count, const float* values, const float* variances,
                                                 int32_t values_on_device, size_t capacity,
                                                 size_t failure_tolerance);
/* Synchronise and read the last tell: accepted[count] (host, 0/1) and the
 * summary.  collect_tell (bf16_search.rs:494-516). */
ENNX_B200_API int32_t ennx_b200_bf16_search_collect(ennx_b200_bf16_search* search, size_t count,
                                                    uint8_t* accepted, ennx_b200_tell_summary* summary);
/* Device pointer of one row slot (device_row) and of the batch of the last
 * ask, `rows` x len contiguous (device_round). */
ENNX_B200_API int32_t ennx_b200_bf16_search_row(ennx_b200_bf16_search* search, size_t slot,
                                                const uint16_t** row);
ENNX_B200_API int32_t ennx_b200_bf16_search_round(ennx_b200_bf16_search* search, size_t rows,
                                                  const uint16_t** batch);
/* Gather row slots into the batch, `count` x len (device_batch). */
ENNX_B200_API int32_t ennx_b200_bf16_search_gather(ennx_b200_bf16_search* search, const uint32_t* slots,
                                                   size_t count, const uint16_t** batch);
/* Make `consumer` see all enqueued work: mode 0 synchronises, 1 does
 * nothing, 2 makes `consumer` wait on an event (sync_stream,
 * cuda/src/lib.rs:1014-1033). */
ENNX_B200_API int32_t ennx_b200_bf16_search_handoff(ennx_b200_bf16_search* search, void* consumer,
                                                    int32_t mode);
/* Copy the per-candidate scores and summed distances (history stride 128)
 * of the last ask to host memory; test and tracing aid. */
ENNX_B200_API int32_t ennx_b200_bf16_search_last_scores(ennx_b200_bf16_search* search, float* scores,
                                                        size_t num_scores, float* distances,
                                                        size_t num_distances);
/* CUDA-event timing of asks (AskProfile): out[0..3] = score, pick,
 * materialize, total milliseconds of the last ask; *available = 0 when
 * profiling was off.  Synchronises. */
ENNX_B200_API int32_t ennx_b200_bf16_search_set_profiling(ennx_b200_bf16_search* search, int32_t enabled);
ENNX_B200_API int32_t ennx_b200_bf16_search_last_profile(ennx_b200_bf16_search* search, float* out,
                                                         int32_t* available);

/* ---- resident single-token KDA-MoE decoder on packed weights (replaces
 *      NativeKdaModel / KdaMoeMetalModel, rust/crates/ennx-py/src/
 *      py_experimental.rs:163-315, rust/crates/ennx/src/forward_metal.rs:
 *      614-810, 1140-1394; Metal-only there) ---------------------------- */

/* The packed linears of one layer, named as the reference's model package
 * names them: layers.{i}.attention.{qkv, control, output, qkv_conv,
 * forget_b, gate_b, decay, time_bias, output_norm},
 * layers.{i}.{attention_norm, moe_norm}, layers.{i}.moe.router and
 * layers.{i}.moe.experts.{e}.{gate, up, down} (host arrays of num_experts). */
typedef struct {
    ennx_b200_packed_linear qkv, control, output, qkv_conv, forget_b, gate_b;
    ennx_b200_packed_linear decay, time_bias, output_norm, attention_norm, moe_norm, router;
    const ennx_b200_packed_linear* expert_gate;
    const ennx_b200_packed_linear* expert_up;
    const ennx_b200_packed_linear* expert_down;
} ennx_b200_kda_decoder_layer;

typedef struct {
    uint32_t num_layers, hidden, heads, head_width, gate_rank, num_experts, top_k, expert_width;
    float residual_scale, rms_epsilon, embedding_scale;
} ennx_b200_kda_decoder_config;

typedef struct ennx_b200_kda_decoder ennx_b200_kda_decoder;

/* Copy the host arenas (packed u8 codes, f32 scales and biases) to the
 * device, validate every linear's shape and arena bounds, reset the decode
 * state and prepare candidate 0 (the reference constructor's order).
 * `embedding` is tied: token lookup and LM head.  hidden = heads x
 * head_width, head_width <= 128, top_k <= 8.  The decoder runs on its own
 * stream; every call below synchronises before returning. */
ENNX_B200_API int32_t ennx_b200_kda_decoder_create(const uint8_t* packed, size_t packed_bytes, const float* scales,
                                                   size_t num_scales, const float* biases, size_t num_biases,
                                                   const ennx_b200_kda_decoder_config* config,
                                                   const ennx_b200_kda_decoder_layer* layers,
                                                   const ennx_b200_packed_linear* embedding,
                                                   const ennx_b200_packed_linear* final_norm, void* stream,
                                                   ennx_b200_kda_decoder** out);
ENNX_B200_API int32_t ennx_b200_kda_decoder_destroy(ennx_b200_kda_decoder* decoder);
/* Zero the recurrent state and the convolution history of every layer. */
ENNX_B200_API int32_t ennx_b200_kda_decoder_reset(ennx_b200_kda_decoder* decoder);
/* Dequantise the norm / decay / time-bias vectors under `seed`
 * (prepare_candidate, forward_metal.rs:1262-1283). */
ENNX_B200_API int32_t ennx_b200_kda_decoder_prepare(ennx_b200_kda_decoder* decoder, uint64_t seed);
/* One greedy step: embed `token`, run every layer, LM head, argmax. */
ENNX_B200_API int32_t ennx_b200_kda_decoder_decode_token(ennx_b200_kda_decoder* decoder, uint32_t token,
                                                         uint64_t seed, uint32_t* next_token);
/* out[0..prompt_len) = prompt, then max_new_tokens greedy tokens; the token
 * step is one CUDA graph replayed per token with the token fed back on the
 * device. */
ENNX_B200_API int32_t ennx_b200_kda_decoder_generate(ennx_b200_kda_decoder* decoder, const uint32_t* prompt,
                                                     size_t prompt_len, size_t max_new_tokens, uint64_t seed,
                                                     uint32_t* out);
/* fp32 logits of the last step (host, vocab entries). */
ENNX_B200_API int32_t ennx_b200_kda_decoder_logits(ennx_b200_kda_decoder* decoder, float* out, size_t vocab);

/* ---- measurement (CUDA-event timing per kernel class, the counterpart of
 *      the reference's AskProfile / ENNX_CUDA_PROFILE, cuda/src/lib.rs:165-171,
 *      977-1005) --------------------------------------------------------- */

typedef struct {
    char name[32];
    int64_t launches;
    double total_ms;   /* sum of CUDA-event durations on the launching stream */
    double flops;      /* algorithmic FLOPs of the timed launches */
    double bytes;      /* algorithmic HBM bytes of the timed launches */
} ennx_b200_profile_entry;

/* Start recording CUDA events around every launch of the population forward
 * (and the operators it uses) on the calling thread's device. */
ENNX_B200_API int32_t ennx_b200_profile_begin(void);
/* Synchronise, stop recording and return one entry per kernel class. */
ENNX_B200_API int32_t ennx_b200_profile_end(ennx_b200_profile_entry* out, int32_t max_entries,
                                            int32_t* num_entries);
/* Number of kernels this library has launched in this process. */
ENNX_B200_API uint64_t ennx_b200_launch_count(void);

#ifdef __cplusplus
}
#endif
#endif /* ENNX_B200_H */
