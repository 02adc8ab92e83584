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

// One 128-byte line at p into L2 (no register, nothing to wait for).
__device__ __forceinline__ void prefetch_line_l2(const void* p) {
    asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
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

// ---- 24-bit fixed point for exact dp4a dot products --------------------------------
// A vector v is staged with scale s = max|v| / FIX_MAX as q_j = rint(v_j / s) =
// hi*2^16 + mid*2^8 + lo (hi, mid, lo signed bytes) in three byte planes, so
// 4 int8 weights times 4 staged values are three exact dp4a. The error is
// below 2^-23 * max|v| per element.
constexpr float FIX_MAX = 8323072.0f;  // 2^23 - 2^16: keeps hi within [-127, 127]

// Four values times rs (= FIX_MAX / max|v|) into the packed hi, mid, lo bytes.
__device__ __forceinline__ void fix_pack4(float4 v4, float rs, uint32_t& ph, uint32_t& pm, uint32_t& pl) {
    const float vv[4] = {v4.x, v4.y, v4.z, v4.w};
    ph = pm = pl = 0;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const int q = __float2int_rn(vv[e] * rs);
        const int lo = (int)(int8_t)(q & 0xff);
        const int q1 = (q - lo) >> 8;
        const int md = (int)(int8_t)(q1 & 0xff);
        const int hi = (q1 - md) >> 8;
        ph |= (uint32_t)(hi & 0xff) << (8 * e);
        pm |= (uint32_t)(md & 0xff) << (8 * e);
        pl |= (uint32_t)(lo & 0xff) << (8 * e);
    }
}

// 16 int8 weights times 16 staged activations, exact in three int32 planes.
__device__ __forceinline__ void dp4a16(const int4& w, const int4& h, const int4& m, const int4& l, int& ah, int& am,
                                       int& al) {
    ah = __dp4a(w.x, h.x, ah);
    am = __dp4a(w.x, m.x, am);
    al = __dp4a(w.x, l.x, al);
    ah = __dp4a(w.y, h.y, ah);
    am = __dp4a(w.y, m.y, am);
    al = __dp4a(w.y, l.y, al);
    ah = __dp4a(w.z, h.z, ah);
    am = __dp4a(w.z, m.z, am);
    al = __dp4a(w.z, l.z, al);
    ah = __dp4a(w.w, h.w, ah);
    am = __dp4a(w.w, m.w, am);
    al = __dp4a(w.w, l.w, al);
}
// sum_j w_j q_j from the three plane sums (each exact; one rounding per step).
__device__ __forceinline__ float planes_to_float(int ah, int am, int al) {
    return fmaf(65536.0f, (float)ah, fmaf(256.0f, (float)am, (float)al));
}
__device__ __forceinline__ void load_planes(const int8_t* xq, int plane, int c, int4& h, int4& m, int4& l) {
    h = reinterpret_cast<const int4*>(xq)[c];
    m = reinterpret_cast<const int4*>(xq + plane)[c];
    l = reinterpret_cast<const int4*>(xq + 2 * plane)[c];
}

__device__ __forceinline__ float kv_load(const float* p) { return __ldcg(p); }
__device__ __forceinline__ float kv_load(const __half* p) {
    unsigned short bits = __ldcg(reinterpret_cast<const unsigned short*>(p));
    return __half2float(__ushort_as_half(bits));
}
__device__ __forceinline__ void kv_store(float* p, float v) { *p = v; }
__device__ __forceinline__ void kv_store(__half* p, float v) { *p = __float2half_rn(v); }

}  // namespace dcb
