// Device helpers shared by the decode-step kernel and the isolated operators.
// sm_100a only: inline PTX for cache-hinted loads, L2 bulk prefetch, acquire
// loads and release reductions.
#pragma once
#include <cstdint>
#include <cuda_fp16.h>

namespace dcb {

constexpr unsigned FULL = 0xffffffffu;

__device__ __forceinline__ int4 ld_stream(const void* p) {
    // Weights are read exactly once per token: bypass L1, normal L2 policy.
    int4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.s32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
    return v;
}

__device__ __forceinline__ float ld_cg(const float* p) { return __ldcg(p); }
__device__ __forceinline__ int ld_cg(const int* p) { return __ldcg(p); }

__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ int ld_volatile(const int* p) { return *reinterpret_cast<const volatile int*>(p); }

__device__ __forceinline__ void red_release_add(unsigned* p, unsigned v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" :: "l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint64_t globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Fire-and-forget prefetch of [p, p+bytes) into L2. p and bytes must be
// multiples of 16; callers round inward.
__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" :: "l"(p), "r"(bytes) : "memory");
}

// Prefetch this block's 1/nblocks slice of [base, base+bytes), 16-byte aligned.
__device__ __forceinline__ void prefetch_slice(const void* base, size_t bytes, int block, int nblocks) {
    if (!base || bytes < 16) return;
    uintptr_t b = reinterpret_cast<uintptr_t>(base);
    uintptr_t lo = b + bytes * (size_t)block / nblocks;
    uintptr_t hi = b + bytes * (size_t)(block + 1) / nblocks;
    lo = (lo + 15) & ~uintptr_t(15);
    hi = hi & ~uintptr_t(15);
    constexpr uintptr_t piece = 32768;
    for (uintptr_t p = lo; p < hi; p += piece) {
        uintptr_t n = hi - p < piece ? hi - p : piece;
        prefetch_l2(reinterpret_cast<const void*>(p), (uint32_t)n);
    }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(FULL, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(FULL, v, o));
    return v;
}

// Exact int8 -> FP32 without the I2F pipe: the biased byte (b + 128) is placed
// in the low mantissa byte of 2^23, giving 2^23 + b + 128 exactly; subtracting
// 2^23 + 128 leaves b. Checked against a plain conversion for all 256 values.
__device__ __forceinline__ float i8_lane(uint32_t biased, int k) {
    return __uint_as_float(__byte_perm(biased, 0x4B000000u, 0x7440u + (uint32_t)k)) - 8388736.0f;
}

// acc += dot(4 int8 in w, x) with the int8 widened exactly to FP32, as two
// packed FP32 lanes (Blackwell f32x2 add/fma: half the FP32 instructions).
__device__ __forceinline__ float2 dot4(uint32_t w, float4 x, float2 acc) {
    const uint32_t u = w ^ 0x80808080u;
    const float2 bias = make_float2(-8388736.0f, -8388736.0f);
    float2 lo = make_float2(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7440u)),
                            __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7441u)));
    float2 hi = make_float2(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7442u)),
                            __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7443u)));
    lo = __fadd2_rn(lo, bias);
    hi = __fadd2_rn(hi, bias);
    acc = __ffma2_rn(lo, make_float2(x.x, x.y), acc);
    acc = __ffma2_rn(hi, make_float2(x.z, x.w), acc);
    return acc;
}

// An activation vector staged in shared memory for 16-byte weight chunks:
// chunk c (weights 16c..16c+15) multiplies xs4[k*nch + c] for k = 0..3, so a
// warp reading consecutive chunks reads consecutive float4s (no bank conflicts).
__device__ __forceinline__ float2 dot16(int4 w, const float4* xs4, int nch, int c, float2 acc) {
    acc = dot4((uint32_t)w.x, xs4[c], acc);
    acc = dot4((uint32_t)w.y, xs4[nch + c], acc);
    acc = dot4((uint32_t)w.z, xs4[2 * nch + c], acc);
    acc = dot4((uint32_t)w.w, xs4[3 * nch + c], acc);
    return acc;
}

// Index of element j of the logical vector inside the chunk-interleaved layout.
__device__ __forceinline__ int xs_index(int j, int nch) {
    const int c = j >> 4, r = j & 15;
    return ((r >> 2) * nch + c) * 4 + (r & 3);
}

// R rows of `nch` 16-byte chunks each, dotted with the staged vector; the
// result of row r is returned (warp-reduced) in out[r] on every lane. Rows
// whose pointer is null contribute 0. MAXC = chunks per lane, fully unrolled
// so all of a lane's loads are in flight together.
template <int R, int MAXC>
__device__ __forceinline__ void rows_dot_unrolled(const int8_t* const (&rows)[R], const float4* xs4, int nch,
                                                  int lane, float (&out)[R]) {
    int4 w[R][MAXC];
#pragma unroll
    for (int c = 0; c < MAXC; ++c) {
        const int ch = lane + 32 * c;
#pragma unroll
        for (int r = 0; r < R; ++r)
            w[r][c] = (ch < nch && rows[r]) ? ld_stream(rows[r] + (size_t)ch * 16) : make_int4(0, 0, 0, 0);
    }
    float2 acc[R];
#pragma unroll
    for (int r = 0; r < R; ++r) acc[r] = make_float2(0.f, 0.f);
#pragma unroll
    for (int c = 0; c < MAXC; ++c) {
        const int ch = lane + 32 * c;
        if (ch < nch) {
#pragma unroll
            for (int r = 0; r < R; ++r) acc[r] = dot16(w[r][c], xs4, nch, ch, acc[r]);
        }
    }
#pragma unroll
    for (int r = 0; r < R; ++r) out[r] = warp_sum(acc[r].x + acc[r].y);
}

// Same for long rows: loop over groups of U chunks per lane.
template <int R, int U>
__device__ __forceinline__ void rows_dot_loop(const int8_t* const (&rows)[R], const float4* xs4, int nch, int lane,
                                              float (&out)[R]) {
    float2 acc[R];
#pragma unroll
    for (int r = 0; r < R; ++r) acc[r] = make_float2(0.f, 0.f);
    for (int base = 0; base < nch; base += 32 * U) {
        int4 w[R][U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int ch = base + lane + 32 * u;
#pragma unroll
            for (int r = 0; r < R; ++r)
                w[r][u] = (ch < nch && rows[r]) ? ld_stream(rows[r] + (size_t)ch * 16) : make_int4(0, 0, 0, 0);
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int ch = base + lane + 32 * u;
            if (ch < nch) {
#pragma unroll
                for (int r = 0; r < R; ++r) acc[r] = dot16(w[r][u], xs4, nch, ch, acc[r]);
            }
        }
    }
#pragma unroll
    for (int r = 0; r < R; ++r) out[r] = warp_sum(acc[r].x + acc[r].y);
}

__device__ __forceinline__ float kv_load(const float* p) { return __ldcg(p); }
__device__ __forceinline__ float kv_load(const __half* p) {
    unsigned short bits = __ldcg(reinterpret_cast<const unsigned short*>(p));
    return __half2float(__ushort_as_half(bits));
}
__device__ __forceinline__ void kv_store(float* p, float v) { *p = v; }
__device__ __forceinline__ void kv_store(__half* p, float v) { *p = __float2half_rn(v); }

}  // namespace dcb
