/*
 * ennx_oracle.h -- CPU restatement of the reference's model-evaluation math.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker that the CUDA path
 * in ennx_b200 is compared against.  Nothing in the product links it: only
 * tests/, __graft_entry__.smoke() and the cpu_baseline leg of bench.py load
 * it.  Every function cites the reference file:line it restates (paths are
 * relative to the Kvutza/ennx repository root).
 *
 * Parity pinning:
 *   - mix64 / dense_sign / tensor_key / dense_next / bf16 encode+next / dense
 *     apply / dense linear / trial_hash+perturb_code are pinned against the
 *     reference's own golden vectors (rust/crates/ennx/src/dense.rs:470-505,
 *     dense/bf16.rs:321-390) and against fixtures produced by executing the
 *     reference's pure-Python restatement (ops/bf16_parity.py:18-106), see
 *     tests/golden/make_golden.py.
 *   - The KDA serial recurrence is pinned by the decode known-answer test of
 *     buck2/tests/metal.rs:371-414.
 *   - RMSNorm, router top-k, SwiGLU, KDA gate/beta, post-norm and the packed
 *     int4/int8 dequantisation with its Metal perturb_hash restate
 *     kda_moe.metal; the reference has no CPU test of them (unpinned).
 *   - Philox noise, RoPE, GQA attention, chunked KDA, LM-head cross-entropy
 *     have no reference implementation at all: parity unpinned, the functions
 *     here are builder-written fp32/fp64 definitions.
 */
#ifndef ENNX_ORACLE_H
#define ENNX_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { EO_OK = 0, EO_INVALID_ARGUMENT = 1, EO_OVERFLOW = 2 };

typedef struct { uint64_t key; size_t offset; size_t len; float scale; } eo_leaf;
typedef struct { uint64_t seed; float coefficient; } eo_term;
typedef struct { uint64_t key; uint64_t start; float scale; } eo_view;

/* ---- perturbation family (bit-exact restatements) ---- */
uint64_t eo_mix64(uint64_t x);
float eo_dense_sign(uint64_t seed, uint64_t key, uint64_t element);
uint64_t eo_tensor_key(const char* name);
float eo_dense_next(float value, int positive);
float eo_bf16_decode(uint16_t v);
uint16_t eo_bf16_encode(float v);
uint16_t eo_bf16_next(uint16_t v, int positive);
int32_t eo_dense_apply_f32(const float* base, size_t n, const eo_leaf* leaves, size_t nl,
                           const eo_term* terms, size_t nt, float* out, size_t* changed);
int32_t eo_dense_apply_bf16(const uint16_t* base, size_t n, const eo_leaf* leaves, size_t nl,
                            const eo_term* terms, size_t nt, uint16_t* out);
int32_t eo_dense_dist2(const eo_leaf* leaves, size_t nl, const eo_term* left, size_t nleft,
                       const eo_term* right, size_t nright, double* out);
int32_t eo_dense_linear_f32(const float* input, size_t columns, const float* weight, size_t rows,
                            const float* bias, eo_view weight_view, eo_view bias_view,
                            const eo_term* terms, size_t nt, float* out);
uint32_t eo_trial_hash(uint32_t seed_low, uint32_t seed_high, uint32_t element);
/* resident BF16 search */
typedef struct { uint64_t key; uint64_t offset; uint64_t length; float scale; float weight; } eo_bf16_leaf;
uint16_t eo_bf16_seed(uint16_t v, uint64_t key, uint64_t element, uint64_t seed, float scale, float coef);
int32_t eo_search_candidate(const uint16_t* base, size_t len, const eo_bf16_leaf* leaves, size_t nl,
                            uint64_t seed, float coef, uint16_t* out);
int32_t eo_search_distances(const uint16_t* rows, size_t stride, size_t base_slot, const uint32_t* history_slots,
                            size_t history, const eo_bf16_leaf* leaves, size_t nl, size_t len, uint64_t seed,
                            float coef, double* out);
double eo_draw_normal(uint64_t seed, uint32_t index, uint32_t metric);
uint32_t eo_perturb_code(uint32_t code, uint32_t seed_low, uint32_t seed_high, uint32_t element,
                         uint32_t bits, uint32_t whole, uint32_t threshold);

/* ---- packed int4/int8 weights (kda_moe.metal, Metal only in the reference) ---- */
typedef struct {
    uint64_t byte_offset, scale_offset, bias_offset, input_width, output_width;
    uint32_t bits, group_size;
    uint64_t element_offset;
    uint32_t perturb_whole, perturb_threshold;
} eo_packed_linear;
uint32_t eo_packed_hash(uint32_t low, uint32_t high, uint32_t element);
void eo_packed_dequantize(const uint8_t* weights, const float* scales, const float* biases,
                          const eo_packed_linear* l, uint32_t seed_low, uint32_t seed_high,
                          uint32_t enabled, float* out);

/* ---- population noise (builder-defined; no reference counterpart) ---- */
void eo_philox4x32_10(const uint32_t ctr[4], const uint32_t key[2], uint32_t out[4]);
void eo_noise8(uint64_t seed, uint32_t pair, uint32_t tensor, uint64_t block, float out[8]);
void eo_perturb_bf16_at(const uint16_t* w, size_t n, size_t start, uint64_t seed, uint32_t pair, uint32_t tensor,
                        float sigma, int sign, uint16_t* out);
void eo_es_update(const uint16_t* w, size_t n, uint64_t seed, uint32_t tensor, const float* coef,
                  uint32_t first_pair, uint32_t pairs, uint16_t* out);
void eo_perturb_bf16(const uint16_t* w, size_t n, uint64_t seed, uint32_t pair, uint32_t tensor,
                     float sigma, int sign, uint16_t* out);

/* ---- forward math ---- */
void eo_rmsnorm(const float* x, const float* w, size_t rows, size_t width, float eps, float* out);
void eo_router_logits(const uint16_t* x, const uint16_t* w, size_t tokens, size_t hidden,
                      size_t experts, float* logits);
void eo_router_topk(const float* logits, size_t tokens, size_t experts, size_t k,
                    int32_t* index, float* gate);
void eo_kda_gate_beta(const float* raw_gate, const float* raw_beta, const float* decay,
                      const float* time_bias, size_t tokens, size_t heads, size_t head_width,
                      float* gate, float* beta);
void eo_l2norm_heads(float* x, size_t groups, size_t width);
void eo_kda_recurrence(const float* q, const float* k, const float* v, const float* g,
                       const float* beta, size_t batch, size_t length, size_t heads,
                       size_t dk, size_t dv, float* state, float* out);
void eo_kda_postprocess(const float* o, const float* gate, const float* norm, size_t tokens,
                        size_t heads, size_t width, float eps, float* out);
void eo_rope(float* x, size_t batch, size_t seq, size_t heads, size_t dim, double theta);
void eo_gqa_attention(const float* q, const float* k, const float* v, size_t batch, size_t seq,
                      size_t hq, size_t hkv, size_t dim, float* out);
void eo_cross_entropy_rows(const float* logits, const int32_t* targets, size_t rows,
                           size_t vocab, double* loss);

#ifdef __cplusplus
}
#endif
#endif
