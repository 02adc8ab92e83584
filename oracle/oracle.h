/* Test infrastructure only: plain-C restatement of the reference's per-token
 * decode step, used as the checker for the CUDA engine. It is never linked into
 * the product library. Every function cites the reference file:line it follows.
 * Arithmetic order follows the reference's scalar kernel so that, compiled with
 * -ffp-contract=off, results are bit-identical to `Kernel::scalar`. */
#ifndef ORACLE_H
#define ORACLE_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
    const int8_t *q, *k, *v, *o, *gate, *up, *down;
    const float *q_scales, *k_scales, *v_scales, *o_scales, *gate_scales, *up_scales, *down_scales;
    const float *input_norm, *post_norm, *q_bias, *k_bias, *v_bias;
} orc_layer;

typedef struct {
    size_t hidden, intermediate, layers, heads, kv_heads, dim, vocab;
    float epsilon, theta;
    const int8_t* embed;
    const float* embed_scales;
    const float* final_norm;
    const orc_layer* layer; /* [layers] */
} orc_model;

void orc_matvec_i8(const int8_t* w, const float* scales, size_t rows, size_t cols,
                   const float* x, float* y, int threads);
void orc_rmsnorm(const float* x, const float* w, float* out, size_t n, float eps);
void orc_inverse_frequency(float* inv, size_t dim, float theta);
void orc_rope_direct(float* x, size_t heads, size_t dim, size_t pos, float theta);
void orc_rope_cached(float* x, size_t heads, size_t dim, size_t pos, const float* inv_freq);
int orc_attention(const float* q, const float* keys, const float* values, float* out, float* scores,
                  size_t length, size_t heads, size_t kv_heads, size_t dim, int threads);
void orc_silu_mul(float* gate, const float* up, size_t n);
int orc_argmax(const float* x, size_t n);
float orc_f16_round(float x);
void orc_f16_round_array(float* x, size_t n);
void orc_quantize_row(const float* src, size_t n, int8_t* out, float* scale);

/* One decode step over a caller-owned KV cache laid out per layer as
 * [capacity][kv_heads*dim] floats, K and V separately, layer-major. With
 * kv_f16 != 0 the new K/V are rounded to binary16 before they are stored,
 * which is what a half-precision cache holds. Returns 0 or an error code. */
int orc_step(const orc_model* m, float* kcache, float* vcache, size_t capacity, int kv_f16,
             size_t pos, int token, int head, int cached_rope, float* logits, int threads);

#ifdef __cplusplus
}
#endif
#endif
