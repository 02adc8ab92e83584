// Test infrastructure only: a C shim over the reference library so the parity
// tests can call the reference's own public functions (include/decode.hpp:15-59
// of the reference) in-process through ctypes. It is linked with the reference's
// src/kernels.cpp and src/model.cpp, compiled in place by oracle/Makefile.
#include "decode.hpp"
#include <cstring>
#include <exception>
#include <string>

namespace {
thread_local std::string last_error;
template <class F> int guarded(F&& fn) {
    try { fn(); return 0; }
    catch (const std::exception& e) { last_error = e.what(); return 1; }
}
decode::Kernel kernel_of(int k) {
    switch (k) {
    case 1: return decode::Kernel::simd256;
    case 2: return decode::Kernel::simd512;
    case 3: return decode::Kernel::simd512x4;
    default: return decode::Kernel::scalar;
    }
}
}

extern "C" {
const char* ref_last_error() { return last_error.c_str(); }

// kernel: 0 scalar, 1 simd256, 2 simd512, 3 simd512x4; dtype: 0 bf16, 1 f32, 2 i8.
int ref_matvec(const void* data, const float* scales, size_t rows, size_t cols, int dtype,
               const float* x, float* y, int kernel, int threads) {
    return guarded([&] {
        decode::Matrix m{data, scales, rows, cols,
                         dtype == 0 ? decode::DType::bf16 : dtype == 1 ? decode::DType::f32 : decode::DType::i8};
        decode::matvec(m, x, y, decode::parse_kernel(decode::kernel_name(kernel_of(kernel))), threads);
    });
}
int ref_quantize_row(const float* src, size_t n, int8_t* out, float* scale) {
    return guarded([&] { decode::quantize_row(src, n, out, *scale); });
}
int ref_rmsnorm(const float* x, const float* w, float* out, size_t n, float eps) {
    return guarded([&] { decode::rmsnorm(x, w, out, n, eps); });
}
int ref_rope(float* x, size_t heads, size_t dim, size_t pos, float theta) {
    return guarded([&] { decode::rope(x, heads, dim, pos, theta); });
}
int ref_attention(const float* q, const float* k, const float* v, float* out, float* scores,
                  size_t length, size_t heads, size_t kv_heads, size_t dim, int threads) {
    return guarded([&] { decode::attention(q, k, v, out, scores, length, heads, kv_heads, dim, threads); });
}
int ref_quantize_model(const char* src, const char* dst) {
    return guarded([&] { decode::quantize_model(src, dst); });
}

int ref_engine_create(const char* dir, int kernel, int threads, size_t capacity, int cached_rope, void** out) {
    return guarded([&] {
        *out = new decode::Engine(dir, kernel_of(kernel), threads, capacity, cached_rope != 0);
    });
}
int ref_engine_step(void* e, int token, int head, float* logits_out, size_t vocab) {
    return guarded([&] {
        const auto& logits = static_cast<decode::Engine*>(e)->step(token, head != 0);
        if (head && logits_out) std::memcpy(logits_out, logits.data(), vocab * sizeof(float));
    });
}
int ref_engine_step_profiled(void* e, int token, int head, float* logits_out, size_t vocab,
                             unsigned long long* bytes /* 11 counters */) {
    return guarded([&] {
        decode::Profile p;
        const auto& logits = static_cast<decode::Engine*>(e)->step(token, head != 0, &p);
        if (head && logits_out) std::memcpy(logits_out, logits.data(), vocab * sizeof(float));
        unsigned long long v[11] = {p.matrix_weight_bytes, p.scale_bytes, p.norm_bias_bytes, p.embedding_bytes,
                                    p.kv_write_bytes, p.kv_read_min_bytes, p.kv_read_logical_bytes,
                                    p.lm_head_weight_bytes, p.lm_head_scale_bytes, p.steps, p.head_steps};
        std::memcpy(bytes, v, sizeof(v));
    });
}
int ref_engine_rewind(void* e, size_t pos) { return guarded([&] { static_cast<decode::Engine*>(e)->rewind(pos); }); }
int ref_engine_reset(void* e) { return guarded([&] { static_cast<decode::Engine*>(e)->reset(); }); }
size_t ref_engine_position(void* e) { return static_cast<decode::Engine*>(e)->position(); }
void ref_engine_destroy(void* e) { delete static_cast<decode::Engine*>(e); }
}
