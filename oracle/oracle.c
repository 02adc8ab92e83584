/* Test infrastructure only (see oracle.h): the CPU checker for the CUDA engine.
 * Citations are to the reference project mottopanikeiku/cpu-decode. */
#include "oracle.h"
#include <math.h>
#include <stdlib.h>
#include <string.h>

/* src/kernels.cpp:24-28 (dot_scalar) and :107-120 (matvec): sequential FP32
 * sum of float(w)*x, then one multiply by the row scale. */
void orc_matvec_i8(const int8_t* w, const float* scales, size_t rows, size_t cols,
                   const float* x, float* y, int threads) {
    long r;
#pragma omp parallel for num_threads(threads) schedule(static) if (threads > 1)
    for (r = 0; r < (long)rows; ++r) {
        const int8_t* row = w + (size_t)r * cols;
        float sum = 0;
        for (size_t j = 0; j < cols; ++j) sum += (float)row[j] * x[j];
        y[r] = sum * scales[r];
    }
}

/* src/kernels.cpp:132-137 */
void orc_rmsnorm(const float* x, const float* w, float* out, size_t n, float eps) {
    float sum = 0;
    for (size_t j = 0; j < n; ++j) sum += x[j] * x[j];
    float inv = 1.0f / sqrtf(sum / (float)n + eps);
    for (size_t j = 0; j < n; ++j) out[j] = x[j] * inv * w[j];
}

/* src/model.cpp:222-224 */
void orc_inverse_frequency(float* inv, size_t dim, float theta) {
    for (size_t j = 0; j < dim / 2; ++j) inv[j] = 1.0f / powf(theta, (float)(2 * j) / (float)dim);
}

/* src/kernels.cpp:138-149 (direct split-half rotation) */
void orc_rope_direct(float* x, size_t heads, size_t dim, size_t pos, float theta) {
    for (size_t j = 0; j < dim / 2; ++j) {
        float angle = (float)pos / powf(theta, (float)(2 * j) / (float)dim);
        float c = cosf(angle), s = sinf(angle);
        for (size_t h = 0; h < heads; ++h) {
            float* v = x + h * dim;
            float a = v[j], b = v[j + dim / 2];
            v[j] = a * c - b * s;
            v[j + dim / 2] = b * c + a * s;
        }
    }
}

/* src/model.cpp:269-274 (cos/sin per step) and :288-297 (rotate) */
void orc_rope_cached(float* x, size_t heads, size_t dim, size_t pos, const float* inv_freq) {
    for (size_t h = 0; h < heads; ++h)
        for (size_t j = 0; j < dim / 2; ++j) {
            float angle = (float)pos * inv_freq[j];
            float c = cosf(angle), s = sinf(angle);
            size_t a = h * dim + j, b = a + dim / 2;
            float first = x[a], second = x[b];
            x[a] = first * c - second * s;
            x[b] = second * c + first * s;
        }
}

/* src/kernels.cpp:150-179: per query head, scaled dot scores, max-subtracted
 * exp, then p/total times V accumulated over positions. */
int orc_attention(const float* q, const float* keys, const float* values, float* out, float* scores,
                  size_t length, size_t heads, size_t kv_heads, size_t dim, int threads) {
    if (!length || !kv_heads || heads % kv_heads || !dim || threads < 1) return 1;
    const size_t stride = kv_heads * dim;
    const float scale = 1.0f / sqrtf((float)dim);
    long hh;
#pragma omp parallel for num_threads(threads) schedule(static) if (threads > 1)
    for (hh = 0; hh < (long)heads; ++hh) {
        size_t h = (size_t)hh, kv = h / (heads / kv_heads);
        float* p = scores + h * length;
        float maximum = -INFINITY;
        for (size_t t = 0; t < length; ++t) {
            float dot = 0;
            for (size_t j = 0; j < dim; ++j) dot += q[h * dim + j] * keys[t * stride + kv * dim + j];
            p[t] = dot * scale;
            if (maximum < p[t]) maximum = p[t];
        }
        float total = 0;
        for (size_t t = 0; t < length; ++t) {
            p[t] = expf(p[t] - maximum);
            total += p[t];
        }
        for (size_t j = 0; j < dim; ++j) out[h * dim + j] = 0.0f;
        for (size_t t = 0; t < length; ++t) {
            float pt = p[t] / total;
            for (size_t j = 0; j < dim; ++j) out[h * dim + j] += pt * values[t * stride + kv * dim + j];
        }
    }
    return 0;
}

/* src/model.cpp:308 */
void orc_silu_mul(float* gate, const float* up, size_t n) {
    for (size_t j = 0; j < n; ++j) gate[j] = (gate[j] / (1.0f + expf(-gate[j]))) * up[j];
}

/* src/main.cpp:35-37: std::max_element, the first maximal index wins. */
int orc_argmax(const float* x, size_t n) {
    size_t best = 0;
    for (size_t i = 1; i < n; ++i)
        if (x[best] < x[i]) best = i;
    return (int)best;
}

/* IEEE binary16 round-to-nearest-even, returned widened back to float. */
float orc_f16_round(float x) {
    _Float16 h = (_Float16)x;
    return (float)h;
}
void orc_f16_round_array(float* x, size_t n) {
    for (size_t i = 0; i < n; ++i) x[i] = orc_f16_round(x[i]);
}

/* src/kernels.cpp:121-131: scale = max|x|/127 (1 for an all-zero row),
 * q = clamp(round_half_away(x/scale), -127, 127). */
void orc_quantize_row(const float* src, size_t n, int8_t* out, float* scale) {
    float maximum = 0;
    for (size_t j = 0; j < n; ++j) maximum = fmaxf(maximum, fabsf(src[j]));
    *scale = maximum == 0 ? 1.0f : maximum / 127.0f;
    for (size_t j = 0; j < n; ++j) {
        float r = roundf(src[j] / *scale);
        out[j] = (int8_t)(r < -127.0f ? -127.0f : r > 127.0f ? 127.0f : r);
    }
}

/* src/model.cpp:258-329 (Engine::Impl::step) over caller-owned KV. */
int orc_step(const orc_model* m, float* kcache, float* vcache, size_t capacity, int kv_f16,
             size_t pos, int token, int head, int cached_rope, float* logits, int threads) {
    if (token < 0 || (size_t)token >= m->vocab) return 2;
    if (pos >= capacity) return 3;
    const size_t H = m->hidden, I = m->intermediate, kvd = m->kv_heads * m->dim;
    float* buf = (float*)calloc(6 * H + 2 * kvd + 2 * I + m->heads * (pos + 1) + m->dim, sizeof(float));
    if (!buf) return 4;
    float *x = buf, *norm = x + H, *q = norm + H, *attn = q + H, *proj = attn + H, *spare = proj + H;
    float *k = spare + H, *v = k + kvd, *gate = v + kvd, *up = gate + I, *scores = up + I;
    float* inv = scores + m->heads * (pos + 1);
    (void)spare;
    orc_inverse_frequency(inv, m->dim, m->theta);
    /* src/model.cpp:261-267 */
    for (size_t j = 0; j < H; ++j)
        x[j] = (float)m->embed[(size_t)token * H + j] * m->embed_scales[token];
    for (size_t l = 0; l < m->layers; ++l) {
        const orc_layer* L = &m->layer[l];
        float* kc = kcache + l * capacity * kvd;
        float* vc = vcache + l * capacity * kvd;
        orc_rmsnorm(x, L->input_norm, norm, H, m->epsilon);
        orc_matvec_i8(L->q, L->q_scales, H, H, norm, q, threads);
        orc_matvec_i8(L->k, L->k_scales, kvd, H, norm, k, threads);
        orc_matvec_i8(L->v, L->v_scales, kvd, H, norm, v, threads);
        for (size_t j = 0; j < H; ++j) q[j] += L->q_bias[j];
        for (size_t j = 0; j < kvd; ++j) { k[j] += L->k_bias[j]; v[j] += L->v_bias[j]; }
        if (cached_rope) {
            orc_rope_cached(q, m->heads, m->dim, pos, inv);
            orc_rope_cached(k, m->kv_heads, m->dim, pos, inv);
        } else {
            orc_rope_direct(q, m->heads, m->dim, pos, m->theta);
            orc_rope_direct(k, m->kv_heads, m->dim, pos, m->theta);
        }
        if (kv_f16) { orc_f16_round_array(k, kvd); orc_f16_round_array(v, kvd); }
        memcpy(kc + pos * kvd, k, kvd * sizeof(float));
        memcpy(vc + pos * kvd, v, kvd * sizeof(float));
        orc_attention(q, kc, vc, attn, scores, pos + 1, m->heads, m->kv_heads, m->dim, threads);
        orc_matvec_i8(L->o, L->o_scales, H, H, attn, proj, threads);
        for (size_t j = 0; j < H; ++j) x[j] += proj[j];
        orc_rmsnorm(x, L->post_norm, norm, H, m->epsilon);
        orc_matvec_i8(L->gate, L->gate_scales, I, H, norm, gate, threads);
        orc_matvec_i8(L->up, L->up_scales, I, H, norm, up, threads);
        orc_silu_mul(gate, up, I);
        orc_matvec_i8(L->down, L->down_scales, H, I, gate, proj, threads);
        for (size_t j = 0; j < H; ++j) x[j] += proj[j];
    }
    if (head) {
        orc_rmsnorm(x, m->final_norm, norm, H, m->epsilon);
        orc_matvec_i8(m->embed, m->embed_scales, m->vocab, H, norm, logits, threads);
    }
    free(buf);
    return 0;
}
