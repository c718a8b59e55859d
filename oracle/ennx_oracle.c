/*
 * ennx_oracle.c -- CPU restatement of the reference's model-evaluation math.
 *
 * TEST INFRASTRUCTURE ONLY: the checker for the CUDA path, never the product.
 * Compiled with -ffp-contract=off so that every "a + b*c" rounds twice, as the
 * reference's Rust code does (Rust never contracts to FMA unless mul_add is
 * written out).  Citations are file:line inside the Kvutza/ennx repository.
 */
#include "ennx_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------------ */
/* Perturbation family                                                      */
/* ------------------------------------------------------------------------ */

/* splitmix64 finaliser; rust/crates/ennx/src/dense.rs:428-433 */
uint64_t eo_mix64(uint64_t x) {
    uint64_t v = x + 0x9e3779b97f4a7c15ull;
    v = (v ^ (v >> 30)) * 0xbf58476d1ce4e5b9ull;
    v = (v ^ (v >> 27)) * 0x94d049bb133111ebull;
    return v ^ (v >> 31);
}

/* Rademacher direction of (seed, leaf key, element); dense.rs:397-405 */
float eo_dense_sign(uint64_t seed, uint64_t key, uint64_t element) {
    uint64_t leaf = eo_mix64(key ^ 0xd6e8feb86659fd93ull);
    uint64_t coord = eo_mix64(element ^ 0xa0761d6478bd642full);
    return (eo_mix64(seed ^ leaf ^ coord) & 1ull) ? 1.0f : -1.0f;
}

/* FNV-1a 64 over the tensor name bytes; dense.rs:51-58 */
uint64_t eo_tensor_key(const char* name) {
    uint64_t key = 1469598103934665603ull;
    for (const unsigned char* p = (const unsigned char*)name; *p; ++p)
        key = (key ^ (uint64_t)*p) * 1099511628211ull;
    return key;
}

static uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* one-ulp step toward the dominant direction, kept finite; dense.rs:407-426 */
float eo_dense_next(float value, int positive) {
    if (value == 0.0f) return u2f(positive ? 1u : 0x80000001u);
    int grows = (value > 0.0f) == (positive != 0);
    float cand = u2f(grows ? f2u(value) + 1u : f2u(value) - 1u);
    if (isfinite(cand)) return cand;
    return u2f(grows ? f2u(value) - 1u : f2u(value) + 1u);
}

/* dense/bf16.rs:266-268 */
float eo_bf16_decode(uint16_t v) { return u2f((uint32_t)v << 16); }

/* round-to-nearest-even encode; dense/bf16.rs:270-273 */
uint16_t eo_bf16_encode(float v) {
    uint32_t bits = f2u(v);
    return (uint16_t)((bits + 0x7fffu + ((bits >> 16) & 1u)) >> 16);
}

/* dense/bf16.rs:275-292 */
uint16_t eo_bf16_next(uint16_t v, int positive) {
    if ((v & 0x7fffu) == 0) return positive ? 1u : 0x8001u;
    int grows = ((v & 0x8000u) == 0) == (positive != 0);
    uint16_t cand = grows ? (uint16_t)(v + 1u) : (uint16_t)(v - 1u);
    if (isfinite(eo_bf16_decode(cand))) return cand;
    return grows ? (uint16_t)(v - 1u) : (uint16_t)(v + 1u);
}

/* Sum of coefficient*direction plus the dominant term's direction; the inner
 * loop shared by dense.rs:367-379, dense/bf16.rs:239-251, linear.rs:530-541. */
static float term_sum(const eo_term* terms, size_t nt, uint64_t key, uint64_t element,
                      int* positive) {
    float sum = 0.0f, strongest = 0.0f;
    *positive = 1;
    for (size_t t = 0; t < nt; ++t) {
        float c = terms[t].coefficient;
        if (c == 0.0f) continue;
        float dir = eo_dense_sign(terms[t].seed, key, element);
        float prod = c * dir;
        sum = sum + prod;
        if (fabsf(c) > strongest) {
            strongest = fabsf(c);
            *positive = (c > 0.0f) == (dir > 0.0f);
        }
    }
    return sum;
}

/* dense.rs:191-240 (validate_leaves / dense_validate) */
static int leaves_valid(const eo_leaf* leaves, size_t nl, size_t n) {
    if (!leaves || nl == 0) return 0;
    size_t end = 0;
    for (size_t i = 0; i < nl; ++i) {
        if (leaves[i].offset != end || leaves[i].len == 0) return 0;
        if (!isfinite(leaves[i].scale) || leaves[i].scale <= 0.0f) return 0;
        end += leaves[i].len;
    }
    return end == n;
}

static double coefficient_of(const eo_term* terms, size_t nt, uint64_t seed) {
    double c = 0.0;
    for (size_t i = 0; i < nt; ++i)
        if (terms[i].seed == seed) c += (double)terms[i].coefficient;
    return c;
}

/* dense.rs:258-265 (has_direction) */
static int has_direction(const eo_term* terms, size_t nt) {
    for (size_t i = 0; i < nt; ++i) {
        int seen = 0;
        for (size_t j = 0; j < i; ++j) if (terms[j].seed == terms[i].seed) seen = 1;
        if (!seen && coefficient_of(terms, nt, terms[i].seed) != 0.0) return 1;
    }
    return 0;
}

static int terms_valid(const eo_term* terms, size_t nt) {
    for (size_t i = 0; i < nt; ++i) if (!isfinite(terms[i].coefficient)) return 0;
    return 1;
}

/* fp32 dense perturbation; dense.rs:361-395 */
int32_t eo_dense_apply_f32(const float* base, size_t n, const eo_leaf* leaves, size_t nl,
                           const eo_term* terms, size_t nt, float* out, size_t* changed) {
    if (!base || !out || n == 0) return EO_INVALID_ARGUMENT;
    for (size_t i = 0; i < n; ++i) if (!isfinite(base[i])) return EO_INVALID_ARGUMENT;
    if (!leaves_valid(leaves, nl, n) || !terms_valid(terms, nt) || !has_direction(terms, nt))
        return EO_INVALID_ARGUMENT;
    size_t count = 0;
    for (size_t l = 0; l < nl; ++l) {
        for (size_t local = 0; local < leaves[l].len; ++local) {
            size_t idx = leaves[l].offset + local;
            int positive;
            float sum = term_sum(terms, nt, leaves[l].key, local, &positive);
            float step = leaves[l].scale * sum;
            float cand = base[idx] + step;
            float v;
            if (sum == 0.0f || cand == base[idx]) v = eo_dense_next(base[idx], positive);
            else if (isfinite(cand)) v = cand;
            else return EO_OVERFLOW;
            out[idx] = v;
            count += (v != base[idx]);
        }
    }
    if (changed) *changed = count;
    return EO_OK;
}

/* BF16 dense perturbation; dense/bf16.rs:228-264 */
int32_t eo_dense_apply_bf16(const uint16_t* base, size_t n, const eo_leaf* leaves, size_t nl,
                            const eo_term* terms, size_t nt, uint16_t* out) {
    if (!base || !out || n == 0) return EO_INVALID_ARGUMENT;
    for (size_t i = 0; i < n; ++i) if (!isfinite(eo_bf16_decode(base[i]))) return EO_INVALID_ARGUMENT;
    if (!leaves_valid(leaves, nl, n) || !terms_valid(terms, nt) || !has_direction(terms, nt))
        return EO_INVALID_ARGUMENT;
    for (size_t l = 0; l < nl; ++l) {
        for (size_t local = 0; local < leaves[l].len; ++local) {
            size_t idx = leaves[l].offset + local;
            int positive;
            float sum = term_sum(terms, nt, leaves[l].key, local, &positive);
            float step = leaves[l].scale * sum;
            float value = eo_bf16_decode(base[idx]) + step;
            if (!isfinite(value)) {
                memcpy(out, base, n * sizeof(uint16_t)); /* roll back, bf16.rs:139-142 */
                return EO_OVERFLOW;
            }
            uint16_t cand = eo_bf16_encode(value);
            out[idx] = (sum == 0.0f || cand == base[idx]) ? eo_bf16_next(base[idx], positive) : cand;
        }
    }
    return EO_OK;
}

/* closed-form squared distance between two term sets; dense.rs:341-358 */
int32_t eo_dense_dist2(const eo_leaf* leaves, size_t nl, const eo_term* left, size_t nleft,
                       const eo_term* right, size_t nright, double* out) {
    if (!out || !leaves || nl == 0) return EO_INVALID_ARGUMENT;
    double energy = 0.0;
    for (size_t i = 0; i < nl; ++i) {
        if (leaves[i].len == 0 || !(leaves[i].scale > 0.0f)) return EO_INVALID_ARGUMENT;
        energy += (double)leaves[i].len * (double)leaves[i].scale * (double)leaves[i].scale;
    }
    double dist = 0.0;
    size_t total = nleft + nright;
    for (size_t i = 0; i < total; ++i) {
        uint64_t seed = i < nleft ? left[i].seed : right[i - nleft].seed;
        int seen = 0;
        for (size_t j = 0; j < i; ++j) {
            uint64_t s = j < nleft ? left[j].seed : right[j - nleft].seed;
            if (s == seed) seen = 1;
        }
        if (seen) continue;
        double d = coefficient_of(left, nleft, seed) - coefficient_of(right, nright, seed);
        dist += d * d;
    }
    *out = energy * dist;
    return EO_OK;
}

/* per-element perturbation used by the fused linear; linear.rs:522-548 */
static int perturbed_value(float base, eo_view view, uint64_t element, const eo_term* terms,
                           size_t nt, float* out) {
    int positive;
    float sum = term_sum(terms, nt, view.key, view.start + element, &positive);
    float step = view.scale * sum;
    float cand = base + step;
    if (sum == 0.0f || cand == base) *out = eo_dense_next(base, positive);
    else if (isfinite(cand)) *out = cand;
    else return 0;
    return 1;
}

/* fused perturbed GEMV with a serial fma chain per row; linear.rs:484-519 */
int32_t eo_dense_linear_f32(const float* input, size_t columns, const float* weight, size_t rows,
                            const float* bias, eo_view weight_view, eo_view bias_view,
                            const eo_term* terms, size_t nt, float* out) {
    if (!input || !weight || !out || columns == 0 || rows == 0 || nt == 0) return EO_INVALID_ARGUMENT;
    if (!terms_valid(terms, nt) || !has_direction(terms, nt)) return EO_INVALID_ARGUMENT;
    if (!(weight_view.scale > 0.0f) || !isfinite(weight_view.scale)) return EO_INVALID_ARGUMENT;
    if (bias && (!(bias_view.scale > 0.0f) || !isfinite(bias_view.scale))) return EO_INVALID_ARGUMENT;
    for (size_t r = 0; r < rows; ++r) {
        float sum = 0.0f;
        for (size_t c = 0; c < columns; ++c) {
            size_t idx = r * columns + c;
            float w;
            if (!perturbed_value(weight[idx], weight_view, idx, terms, nt, &w)) return EO_OVERFLOW;
            sum = fmaf(input[c], w, sum);
        }
        if (bias) {
            float b;
            if (!perturbed_value(bias[r], bias_view, r, terms, nt, &b)) return EO_OVERFLOW;
            sum = sum + b;
        }
        if (!isfinite(sum)) return EO_OVERFLOW;
        out[r] = sum;
    }
    return EO_OK;
}

/* packed-code hash of the CUDA trial path; cuda/kernels/src/lib.rs:150-158 */
uint32_t eo_trial_hash(uint32_t seed_low, uint32_t seed_high, uint32_t element) {
    uint32_t v = seed_low ^ (element * 0x9e3779b9u);
    v ^= v >> 16;
    v *= 0x7feb352du;
    v ^= seed_high;
    v *= 0x846ca68bu;
    return v ^ (v >> 15);
}

/* integer-code step with reflection at the code range; lib.rs:230-258 */
uint32_t eo_perturb_code(uint32_t code, uint32_t seed_low, uint32_t seed_high, uint32_t element,
                         uint32_t bits, uint32_t whole, uint32_t threshold) {
    uint32_t random = eo_trial_hash(seed_low, seed_high, element);
    uint32_t amount = whole + (uint32_t)((random >> 1) < (threshold >> 1));
    if (amount == 0) return code;
    uint32_t max_code = (1u << bits) - 1u;
    if ((random & 1u) == 0) {
        if (code >= amount) return code - amount;
        uint32_t up = code + amount;
        return up < max_code ? up : max_code;
    }
    if (code + amount <= max_code) return code + amount;
    return code >= amount ? code - amount : 0u;
}

/* ------------------------------------------------------------------------ */
/* Packed int4/int8 affine weights (Metal only in the reference).            */
/* ------------------------------------------------------------------------ */

/* Metal perturb_hash, kda_moe.metal:63-71 (seed.high XORed last). */
uint32_t eo_packed_hash(uint32_t low, uint32_t high, uint32_t element) {
    uint32_t v = low ^ (element * 0x9E3779B9u);
    v ^= v >> 16;
    v *= 0x7FEB352Du;
    v ^= v >> 15;
    v *= 0x846CA68Bu;
    v ^= v >> 15;
    return v ^ high;
}

/* packed_weight_device (kda_moe.metal:351-395) for every (row, column):
 * code from the byte arena (int4: low nibble first), integer-code step when
 * the seed is enabled (kda_moe.metal:73-96, 32-bit element index), then
 * code * scale + bias as one fused multiply-add. */
void eo_packed_dequantize(const uint8_t* weights, const float* scales, const float* biases,
                          const eo_packed_linear* l, uint32_t seed_low, uint32_t seed_high,
                          uint32_t enabled, float* out) {
    uint64_t row_bytes = (l->input_width * l->bits + 7) / 8;
    uint64_t groups = (l->input_width + l->group_size - 1) / l->group_size;
    uint32_t max_code = (1u << l->bits) - 1u;
    for (uint64_t r = 0; r < l->output_width; ++r) {
        for (uint64_t c = 0; c < l->input_width; ++c) {
            uint32_t epb = l->bits == 4 ? 2u : 1u;
            uint32_t shift = l->bits == 4 ? (uint32_t)(c & 1u) * 4u : 0u;
            uint32_t code = ((uint32_t)weights[l->byte_offset + r * row_bytes + c / epb] >> shift) & max_code;
            if (enabled) {
                uint32_t element = (uint32_t)l->element_offset + (uint32_t)r * (uint32_t)l->input_width +
                                   (uint32_t)c;
                uint32_t random = eo_packed_hash(seed_low, seed_high, element);
                uint32_t amount = l->perturb_whole + (uint32_t)((random >> 1) < (l->perturb_threshold >> 1));
                if (amount != 0u) {
                    if ((random & 1u) == 0u) {
                        if (code >= amount) code -= amount;
                        else code = code + amount < max_code ? code + amount : max_code;
                    } else if (code + amount <= max_code) {
                        code += amount;
                    } else {
                        code = code >= amount ? code - amount : 0u;
                    }
                }
            }
            uint64_t g = c / l->group_size;
            if (g > groups - 1) g = groups - 1;
            uint64_t si = r * groups + g;
            out[r * l->input_width + c] = fmaf((float)code, scales[l->scale_offset + si], biases[l->bias_offset + si]);
        }
    }
}

/* ------------------------------------------------------------------------ */
/* Population noise: Philox4x32-10 (Salmon, Moraes, Dror, Shaw, SC'11) with  */
/* Box-Muller.  Builder-defined -- the reference draws Rademacher signs.     */
/* ------------------------------------------------------------------------ */

void eo_philox4x32_10(const uint32_t ctr[4], const uint32_t key[2], uint32_t out[4]) {
    uint32_t c0 = ctr[0], c1 = ctr[1], c2 = ctr[2], c3 = ctr[3];
    uint32_t k0 = key[0], k1 = key[1];
    for (int round = 0; round < 10; ++round) {
        uint64_t p0 = (uint64_t)0xD2511F53u * c0;
        uint64_t p1 = (uint64_t)0xCD9E8D57u * c2;
        uint32_t n0 = (uint32_t)(p1 >> 32) ^ c1 ^ k0;
        uint32_t n1 = (uint32_t)p1;
        uint32_t n2 = (uint32_t)(p0 >> 32) ^ c3 ^ k1;
        uint32_t n3 = (uint32_t)p0;
        c0 = n0; c1 = n1; c2 = n2; c3 = n3;
        k0 += 0x9E3779B9u;
        k1 += 0xBB67AE85u;
    }
    out[0] = c0; out[1] = c1; out[2] = c2; out[3] = c3;
}

/* Box-Muller on the two 16-bit halves of one Philox word: u1 = (lo + 1/2) / 2^16 in (0,1),
 * angle 2 pi (hi / 2^16 - 1/2); computed in double so the oracle is the exactly rounded
 * value the device approximates. */
static void box_muller16(uint32_t w, float* z0, float* z1) {
    float u1 = ((float)(w & 0xffffu) + 0.5f) * 1.52587890625e-05f; /* 2^-16: exact, < 1 */
    float u2 = (float)(w >> 16) * 1.52587890625e-05f;
    double r = sqrt(-2.0 * log((double)u1));
    double th = 2.0 * M_PI * ((double)u2 - 0.5);
    *z0 = (float)(r * cos(th));
    *z1 = (float)(r * sin(th));
}

/* Eight N(0,1) draws for element block `block` (elements 8*block .. 8*block+7)
 * of tensor `tensor`, antithetic pair `pair`, population seed `seed`: one
 * Philox4x32-10 call, counter {lo(block), hi(block), tensor, pair}, key
 * {lo(seed), hi(seed)}; word j gives draws 2j and 2j+1. */
void eo_noise8(uint64_t seed, uint32_t pair, uint32_t tensor, uint64_t block, float out[8]) {
    uint32_t ctr[4] = {(uint32_t)block, (uint32_t)(block >> 32), tensor, pair};
    uint32_t key[2] = {(uint32_t)seed, (uint32_t)(seed >> 32)};
    uint32_t x[4];
    eo_philox4x32_10(ctr, key, x);
    for (int j = 0; j < 4; ++j) box_muller16(x[j], &out[2 * j], &out[2 * j + 1]);
}

/* Noise step e = bf16(sigma * eps) (fp32 product, RNE) and the perturbed
 * weight W~ = bf16(W + sign * e): the float sum of two bf16 values is exact
 * (or, for exponents more than 16 apart, rounds to a value whose RNE
 * encoding equals that of the exact sum), so this is one RNE rounding of the
 * exact sum.  Elements [start, start + n) of a tensor (w and out point at
 * element start; start % 8 == 0).  w == NULL: out receives e itself. */
void eo_perturb_bf16_at(const uint16_t* w, size_t n, size_t start, uint64_t seed, uint32_t pair, uint32_t tensor,
                        float sigma, int sign, uint16_t* out) {
    float z[8];
    for (size_t i = 0; i < n; ++i) {
        if ((i & 7) == 0) eo_noise8(seed, pair, tensor, (start + i) >> 3, z);
        uint16_t e = eo_bf16_encode(sigma * z[i & 7]);
        if (!w) {
            out[i] = e;
            continue;
        }
        float step = eo_bf16_decode(e);
        float v = sign >= 0 ? eo_bf16_decode(w[i]) + step : eo_bf16_decode(w[i]) - step;
        out[i] = eo_bf16_encode(v);
    }
}

/* The zeroth-order update (the ES tell): out[i] = bf16(w[i] + sum_p coef[p] *
 * eps(seed, first_pair + p, tensor, i)), the sum in fp32 with one fused
 * multiply-add per pair in pair order, one RNE rounding at the end. */
void eo_es_update(const uint16_t* w, size_t n, uint64_t seed, uint32_t tensor, const float* coef,
                  uint32_t first_pair, uint32_t pairs, uint16_t* out) {
    for (size_t g = 0; g < (n + 7) / 8; ++g) {
        float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (uint32_t p = 0; p < pairs; ++p) {
            float z[8];
            eo_noise8(seed, first_pair + p, tensor, g, z);
            for (int k = 0; k < 8; ++k) acc[k] = fmaf(coef[p], z[k], acc[k]);
        }
        for (size_t e = g * 8; e < n && e < g * 8 + 8; ++e) out[e] = eo_bf16_encode(eo_bf16_decode(w[e]) + acc[e - g * 8]);
    }
}

void eo_perturb_bf16(const uint16_t* w, size_t n, uint64_t seed, uint32_t pair, uint32_t tensor,
                     float sigma, int sign, uint16_t* out) {
    eo_perturb_bf16_at(w, n, 0, seed, pair, tensor, sigma, sign, out);
}

/* ------------------------------------------------------------------------ */
/* Forward math                                                             */
/* ------------------------------------------------------------------------ */

/* x * rsqrt(mean(x^2) + eps) * w; kda_moe.metal:536-554 (fp64 accumulate). */
void eo_rmsnorm(const float* x, const float* w, size_t rows, size_t width, float eps, float* out) {
    for (size_t r = 0; r < rows; ++r) {
        double ss = 0.0;
        for (size_t i = 0; i < width; ++i) ss += (double)x[r * width + i] * x[r * width + i];
        double inv = 1.0 / sqrt(ss / (double)width + (double)eps);
        for (size_t i = 0; i < width; ++i)
            out[r * width + i] = (float)((double)x[r * width + i] * inv * (double)w[i]);
    }
}

/* Router logits: one serial fmaf chain per (token, expert) over the hidden
 * index 0..H-1 starting from 0, the loop order of kda_moe.metal:589-595
 * (score += input * weight, contracted to a fused multiply-add).  The CUDA
 * router keeps exactly this order, so the logits -- and therefore the routing
 * indices -- are bit-identical. */
void eo_router_logits(const uint16_t* x, const uint16_t* w, size_t tokens, size_t hidden,
                      size_t experts, float* logits) {
    for (size_t t = 0; t < tokens; ++t) {
        for (size_t e = 0; e < experts; ++e) {
            float acc = 0.0f;
            for (size_t i = 0; i < hidden; ++i)
                acc = fmaf(eo_bf16_decode(x[t * hidden + i]), eo_bf16_decode(w[e * hidden + i]), acc);
            logits[t * experts + e] = acc;
        }
    }
}

/* Top-k by insertion with strict '>' (ties keep the lower expert index), then
 * a max-subtracted softmax over the k kept logits; kda_moe.metal:596-621. */
void eo_router_topk(const float* logits, size_t tokens, size_t experts, size_t k,
                    int32_t* index, float* gate) {
    for (size_t t = 0; t < tokens; ++t) {
        float val[64];
        int32_t idx[64];
        for (size_t r = 0; r < k; ++r) { val[r] = -INFINITY; idx[r] = 0; }
        for (size_t e = 0; e < experts; ++e) {
            float s = logits[t * experts + e];
            for (size_t r = 0; r < k; ++r) {
                if (s > val[r]) {
                    for (size_t m = k - 1; m > r; --m) { val[m] = val[m - 1]; idx[m] = idx[m - 1]; }
                    val[r] = s; idx[r] = (int32_t)e;
                    break;
                }
            }
        }
        double den = 0.0, ex[64];
        for (size_t r = 0; r < k; ++r) { ex[r] = exp((double)val[r] - (double)val[0]); den += ex[r]; }
        for (size_t r = 0; r < k; ++r) {
            index[t * k + r] = idx[r];
            gate[t * k + r] = (float)(ex[r] / den);
        }
    }
}

static double softplus_d(double x) { return (x > 0 ? x : 0.0) + log1p(exp(-fabs(x))); }

/* g = max(-exp(decay_h) * softplus(raw + time_bias), -5), beta = sigmoid(raw_beta);
 * kda_moe.metal:869-895. */
void eo_kda_gate_beta(const float* raw_gate, const float* raw_beta, const float* decay,
                      const float* time_bias, size_t tokens, size_t heads, size_t head_width,
                      float* gate, float* beta) {
    size_t width = heads * head_width;
    for (size_t t = 0; t < tokens; ++t) {
        for (size_t j = 0; j < width; ++j) {
            size_t h = j / head_width;
            double raw = (double)raw_gate[t * width + j] + (double)time_bias[j];
            double g = -exp((double)decay[h]) * softplus_d(raw);
            gate[t * width + j] = (float)(g < -5.0 ? -5.0 : g);
        }
        for (size_t h = 0; h < heads; ++h)
            beta[t * heads + h] = (float)(1.0 / (1.0 + exp(-(double)raw_beta[t * heads + h])));
    }
}

/* per-head L2 normalisation with max(|x|, 1e-6); kda_moe.metal:510-534 */
void eo_l2norm_heads(float* x, size_t groups, size_t width) {
    for (size_t gi = 0; gi < groups; ++gi) {
        double ss = 0.0;
        for (size_t i = 0; i < width; ++i) ss += (double)x[gi * width + i] * x[gi * width + i];
        double n = sqrt(ss);
        double inv = 1.0 / (n > 1e-6 ? n : 1e-6);
        for (size_t i = 0; i < width; ++i) x[gi * width + i] = (float)(x[gi * width + i] * inv);
    }
}

/* Serial gated delta rule with per-key-channel decay, fp32 state, in the
 * reference's operation order; kda_moe.metal:167-225.  q,k: [B,T,H,dk],
 * v: [B,T,H,dv], g: [B,T,H,dk], beta: [B,T,H], state: [B,H,dk,dv] in/out,
 * out: [B,T,H,dv] scaled by 1/sqrt(dk). */
void eo_kda_recurrence(const float* q, const float* k, const float* v, const float* g,
                       const float* beta, size_t batch, size_t length, size_t heads,
                       size_t dk, size_t dv, float* state, float* out) {
    float scale = 1.0f / sqrtf((float)dk);
    for (size_t b = 0; b < batch; ++b)
        for (size_t h = 0; h < heads; ++h) {
            float* S = state + (b * heads + h) * dk * dv;
            for (size_t t = 0; t < length; ++t) {
                size_t qk = ((b * length + t) * heads + h) * dk;
                size_t vo = ((b * length + t) * heads + h) * dv;
                float rate = beta[(b * length + t) * heads + h];
                for (size_t i = 0; i < dk; ++i) {
                    float d = expf(g[qk + i]);
                    for (size_t j = 0; j < dv; ++j) S[i * dv + j] *= d;
                }
                for (size_t j = 0; j < dv; ++j) {
                    float read = 0.0f;
                    for (size_t i = 0; i < dk; ++i) read += k[qk + i] * S[i * dv + j];
                    float upd = rate * (v[vo + j] - read);
                    for (size_t i = 0; i < dk; ++i) S[i * dv + j] += k[qk + i] * upd;
                    float res = 0.0f;
                    for (size_t i = 0; i < dk; ++i) res += q[qk + i] * S[i * dv + j];
                    out[vo + j] = res * scale;
                }
            }
        }
}

/* per-head RMSNorm * norm, then * sigmoid(gate); kda_moe.metal:898-921 */
void eo_kda_postprocess(const float* o, const float* gate, const float* norm, size_t tokens,
                        size_t heads, size_t width, float eps, float* out) {
    for (size_t t = 0; t < tokens; ++t)
        for (size_t h = 0; h < heads; ++h) {
            const float* x = o + (t * heads + h) * width;
            double ss = 0.0;
            for (size_t i = 0; i < width; ++i) ss += (double)x[i] * x[i];
            double inv = 1.0 / sqrt(ss / (double)width + (double)eps);
            for (size_t i = 0; i < width; ++i) {
                size_t j = (t * heads + h) * width + i;
                double val = (double)x[i] * inv * (double)norm[i];
                out[j] = (float)(val / (1.0 + exp(-(double)gate[j])));
            }
        }
}

/* Rotary embedding, rotate-half (NeoX) pairing (i, i + dim/2), position = s.
 * No reference counterpart.  x: [B, S, H, dim], in place. */
void eo_rope(float* x, size_t batch, size_t seq, size_t heads, size_t dim, double theta) {
    size_t half = dim / 2;
    for (size_t b = 0; b < batch; ++b)
        for (size_t s = 0; s < seq; ++s)
            for (size_t h = 0; h < heads; ++h) {
                float* p = x + ((b * seq + s) * heads + h) * dim;
                for (size_t i = 0; i < half; ++i) {
                    double inv = pow(theta, -2.0 * (double)i / (double)dim);
                    double a = (double)s * inv, c = cos(a), sn = sin(a);
                    double x1 = p[i], x2 = p[i + half];
                    p[i] = (float)(x1 * c - x2 * sn);
                    p[i + half] = (float)(x2 * c + x1 * sn);
                }
            }
}

/* Causal grouped-query attention, softmax scale 1/sqrt(dim), fp64 accumulate.
 * q: [B,S,Hq,dim], k,v: [B,S,Hkv,dim], out: [B,S,Hq,dim].  No reference
 * counterpart. */
void eo_gqa_attention(const float* q, const float* k, const float* v, size_t batch, size_t seq,
                      size_t hq, size_t hkv, size_t dim, float* out) {
    double scale = 1.0 / sqrt((double)dim);
    double* p = (double*)malloc(seq * sizeof(double));
    size_t group = hq / hkv;
    for (size_t b = 0; b < batch; ++b)
        for (size_t h = 0; h < hq; ++h) {
            size_t kh = h / group;
            for (size_t t = 0; t < seq; ++t) {
                const float* qr = q + ((b * seq + t) * hq + h) * dim;
                double mx = -INFINITY;
                for (size_t s = 0; s <= t; ++s) {
                    const float* kr = k + ((b * seq + s) * hkv + kh) * dim;
                    double dot = 0.0;
                    for (size_t i = 0; i < dim; ++i) dot += (double)qr[i] * kr[i];
                    p[s] = dot * scale;
                    if (p[s] > mx) mx = p[s];
                }
                double den = 0.0;
                for (size_t s = 0; s <= t; ++s) { p[s] = exp(p[s] - mx); den += p[s]; }
                float* orow = out + ((b * seq + t) * hq + h) * dim;
                for (size_t i = 0; i < dim; ++i) {
                    double acc = 0.0;
                    for (size_t s = 0; s <= t; ++s) acc += p[s] * v[((b * seq + s) * hkv + kh) * dim + i];
                    orow[i] = (float)(acc / den);
                }
            }
        }
    free(p);
}

/* per-row logsumexp(logits) - logits[target]; no reference counterpart. */
void eo_cross_entropy_rows(const float* logits, const int32_t* targets, size_t rows,
                           size_t vocab, double* loss) {
    for (size_t r = 0; r < rows; ++r) {
        const float* x = logits + r * vocab;
        double mx = -INFINITY;
        for (size_t i = 0; i < vocab; ++i) if (x[i] > mx) mx = x[i];
        double s = 0.0;
        for (size_t i = 0; i < vocab; ++i) s += exp((double)x[i] - mx);
        loss[r] = mx + log(s) - (double)x[targets[r]];
    }
}

/* ------------------------------------------------------------------------ */
/* Resident BF16 search (cuda/kernels/src/bf16.rs:160-330, lib.rs:316-343)  */
/* ------------------------------------------------------------------------ */

/* bf16_seed: v + (scale*coef)*sign rounded to BF16, or one ulp toward the
 * step when that leaves v unchanged; cuda/kernels/src/bf16.rs:160-176 */
uint16_t eo_bf16_seed(uint16_t v, uint64_t key, uint64_t element, uint64_t seed, float scale, float coef) {
    float dir = eo_dense_sign(seed, key, element);
    float step = (scale * coef) * dir;
    uint16_t cand = eo_bf16_encode(eo_bf16_decode(v) + step);
    if (coef == 0.0f || cand == v) return eo_bf16_next(v, (coef > 0.0f) == (dir > 0.0f));
    return cand;
}

static size_t search_leaf_of(const eo_bf16_leaf* leaves, size_t nl, size_t e) {
    size_t l = 0;
    while (l + 1 < nl && leaves[l + 1].offset <= e) ++l;
    return l;
}

/* The candidate row of one seed around `base`; returns 1 if any value is
 * not finite (write_bf16, lib.rs:2053-2130). */
int32_t eo_search_candidate(const uint16_t* base, size_t len, const eo_bf16_leaf* leaves, size_t nl,
                            uint64_t seed, float coef, uint16_t* out) {
    int32_t invalid = 0;
    size_t l = 0;
    for (size_t e = 0; e < len; ++e) {
        while (l + 1 < nl && leaves[l + 1].offset <= e) ++l;
        uint16_t r = eo_bf16_seed(base[e], leaves[l].key, (uint64_t)(e - leaves[l].offset), seed,
                                  leaves[l].scale, coef);
        if ((r & 0x7f80u) == 0x7f80u) invalid = 1;
        out[e] = r;
    }
    return invalid;
}

/* Weighted squared distances of one seeded candidate to `history` rows,
 * accumulated in double (tile_distances, bf16.rs:278-330, restated without
 * its fp32 summation order).  Returns 1 (and +inf distances) if the
 * candidate has a non-finite value. */
int32_t eo_search_distances(const uint16_t* rows, size_t stride, size_t base_slot, const uint32_t* history_slots,
                            size_t history, const eo_bf16_leaf* leaves, size_t nl, size_t len, uint64_t seed,
                            float coef, double* out) {
    for (size_t h = 0; h < history; ++h) out[h] = 0.0;
    const uint16_t* base = rows + base_slot * stride;
    for (size_t e = 0; e < len; ++e) {
        size_t l = search_leaf_of(leaves, nl, e);
        uint16_t c = eo_bf16_seed(base[e], leaves[l].key, (uint64_t)(e - leaves[l].offset), seed,
                                  leaves[l].scale, coef);
        if ((c & 0x7f80u) == 0x7f80u) {
            for (size_t h = 0; h < history; ++h) out[h] = INFINITY;
            return 1;
        }
        float cv = eo_bf16_decode(c);
        for (size_t h = 0; h < history; ++h) {
            float d = cv - eo_bf16_decode(rows[(size_t)history_slots[h] * stride + e]);
            out[h] += (double)d * (double)d * (double)leaves[l].weight;
        }
    }
    return 0;
}

/* draw_normal: Box-Muller over two splitmix64 outputs; lib.rs:316-343 */
double eo_draw_normal(uint64_t seed, uint32_t index, uint32_t metric) {
    const uint64_t prime = 1000003ull;
    uint64_t base = (seed * prime + (uint64_t)index) * prime;
    uint64_t combined = base + (uint64_t)metric;
    uint64_t first = eo_mix64(combined), second = eo_mix64(combined ^ 0xd2b74407b1ce6e93ull);
    const double inv = 1.0 / 9007199254740992.0;
    double raw = (double)(first >> 11) * inv;
    double u1 = raw < 1.0e-12 ? 1.0e-12 : (raw > 1.0 - 1.0e-12 ? 1.0 - 1.0e-12 : raw);
    double u2 = (double)(second >> 11) * inv;
    return sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2);
}
