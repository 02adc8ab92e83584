// Isolated operators behind the C ABI: int8 GEMV (+bias), split-KV GQA
// attention, RMSNorm, RoPE and argmax, each on caller-provided device memory.
// They share the device code of the fused step kernel, so the GEMV sweep and
// the attention sweep measure the same inner loops.
#include "decode_b200.h"
#include "attention.cuh"
#include "device.cuh"

#include <cuda_runtime.h>
#include <algorithm>
#include <cmath>
#include <string>

namespace dcb {
void set_last_error(const std::string& msg);
}

namespace {
using namespace dcb;

int fail(int code, const std::string& msg) {
    dcb::set_last_error(msg);
    return code;
}
int cuda_fail(cudaError_t e, const char* what) {
    return fail(DCB_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

constexpr int GEMV_THREADS = 256;
constexpr int GEMV_WARPS = GEMV_THREADS / 32;

// y[r] = scale[r] * dot(w[r], x) (+ bias[r]); R rows per warp, rows 16-byte aligned.
template <int R, int MAXC>
__global__ void __launch_bounds__(GEMV_THREADS) gemv_i8_kernel(const int8_t* __restrict__ w,
                                                               const float* __restrict__ scales,
                                                               const float* __restrict__ bias,
                                                               const float* __restrict__ x, float* __restrict__ y,
                                                               int rows, int cols) {
    extern __shared__ __align__(16) float4 xs4[];
    const int nch = cols / 16;
    float* xs = reinterpret_cast<float*>(xs4);
    for (int j = threadIdx.x; j < cols; j += blockDim.x) xs[xs_index(j, nch)] = x[j];
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int r0 = (blockIdx.x * GEMV_WARPS + warp) * R;
    if (r0 >= rows) return;
    const int8_t* rp[R];
#pragma unroll
    for (int r = 0; r < R; ++r) rp[r] = r0 + r < rows ? w + (size_t)(r0 + r) * cols : nullptr;
    float dot[R];
    if (MAXC > 0) rows_dot_unrolled<R, (MAXC > 0 ? MAXC : 1)>(rp, xs4, nch, lane, dot);
    else rows_dot_loop<R, 2>(rp, xs4, nch, lane, dot);
    if (lane < R && r0 + lane < rows) {
        float v = 0.f;
#pragma unroll
        for (int r = 0; r < R; ++r)
            if (r == lane) v = dot[r];
        v *= scales[r0 + lane];
        if (bias) v += bias[r0 + lane];
        y[r0 + lane] = v;
    }
}

// Rows whose length is a multiple of 4 but not of 16: 4-byte loads.
__global__ void __launch_bounds__(GEMV_THREADS) gemv_i8_narrow_kernel(const int8_t* __restrict__ w,
                                                                      const float* __restrict__ scales,
                                                                      const float* __restrict__ bias,
                                                                      const float* __restrict__ x,
                                                                      float* __restrict__ y, int rows, int cols) {
    const int lane = threadIdx.x & 31;
    const int r = blockIdx.x * GEMV_WARPS + (threadIdx.x >> 5);
    if (r >= rows) return;
    const uint32_t* row = reinterpret_cast<const uint32_t*>(w + (size_t)r * cols);
    float2 acc2 = make_float2(0.f, 0.f);
    for (int c = lane; c < cols / 4; c += 32) {
        const float4 xv = make_float4(x[4 * c], x[4 * c + 1], x[4 * c + 2], x[4 * c + 3]);
        acc2 = dot4(__ldg(row + c), xv, acc2);
    }
    const float acc = warp_sum(acc2.x + acc2.y);
    if (lane == 0) y[r] = acc * scales[r] + (bias ? bias[r] : 0.f);
}

template <typename KV>
__global__ void __launch_bounds__(512) attention_kernel(AttnIO io) {
    extern __shared__ __align__(16) float att_sm[];
    const int u = blockIdx.x;
    attention_unit<KV>(io, u / io.nsplit, u % io.nsplit, att_sm);
}

__global__ void rope_inv_kernel(float* inv, int dim, float theta) {
    const int j = threadIdx.x;
    if (j < dim / 2) inv[j] = 1.0f / powf(theta, (float)(2 * j) / (float)dim);
}

__global__ void rmsnorm_kernel(const float* x, const float* w, float* out, int n, float eps) {
    __shared__ float red[33];
    float ss = 0.f;
    for (int j = threadIdx.x; j < n; j += blockDim.x) ss = fmaf(x[j], x[j], ss);
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x < 32) {
        float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
        t = warp_sum(t);
        if (threadIdx.x == 0) red[32] = 1.0f / sqrtf(t / (float)n + eps);
    }
    __syncthreads();
    const float inv = red[32];
    for (int j = threadIdx.x; j < n; j += blockDim.x) out[j] = x[j] * inv * w[j];
}

// Split-half rotation (src/kernels.cpp:138-149 direct, src/model.cpp:269-297 cached).
__global__ void rope_kernel(float* x, int heads, int dim, int pos, float theta, int direct) {
    const int half = dim / 2;
    for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < heads * half; e += gridDim.x * blockDim.x) {
        const int h = e / half, j = e % half;
        const float p = powf(theta, (float)(2 * j) / (float)dim);
        const float angle = direct ? __fdiv_rn((float)pos, p) : __fmul_rn((float)pos, 1.0f / p);
        float sn, cs;
        sincosf(angle, &sn, &cs);
        float* v = x + (size_t)h * dim;
        const float a = v[j], b = v[j + half];
        v[j] = __fsub_rn(__fmul_rn(a, cs), __fmul_rn(b, sn));
        v[j + half] = __fadd_rn(__fmul_rn(b, cs), __fmul_rn(a, sn));
    }
}

// First index of the maximum, one block.
__global__ void __launch_bounds__(1024) argmax_kernel(const float* x, int n, int* out) {
    __shared__ float sv[32];
    __shared__ int si[32];
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float v = x[i];
        if (v > bv || (v == bv && i < bi)) { bv = v; bi = i; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(FULL, bv, o);
        const int oi = __shfl_xor_sync(FULL, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    if ((threadIdx.x & 31) == 0) { sv[threadIdx.x >> 5] = bv; si[threadIdx.x >> 5] = bi; }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
            if (sv[w] > bv || (sv[w] == bv && si[w] < bi)) { bv = sv[w]; bi = si[w]; }
        *out = bi == 0x7fffffff ? 0 : bi;
    }
}

template <int R>
int launch_gemv(const int8_t* w, const float* s, const float* b, const float* x, float* y, int rows, int cols,
                cudaStream_t st) {
    const int blocks = (rows + GEMV_WARPS * R - 1) / (GEMV_WARPS * R);
    const size_t smem = (size_t)cols * sizeof(float);
    const int nch = cols / 16;
    const void* k;
    if (nch <= 32) k = (const void*)gemv_i8_kernel<R, 1>;
    else if (nch <= 64) k = (const void*)gemv_i8_kernel<R, 2>;
    else if (nch <= 128) k = (const void*)gemv_i8_kernel<R, 4>;
    else k = (const void*)gemv_i8_kernel<R, 0>;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return cuda_fail(e, "gemv shared memory");
    }
    void* args[] = {(void*)&w, (void*)&s, (void*)&b, (void*)&x, (void*)&y, (void*)&rows, (void*)&cols};
    cudaError_t e = cudaLaunchKernel(k, dim3(blocks), dim3(GEMV_THREADS), args, smem, st);
    return e == cudaSuccess ? 0 : cuda_fail(e, "gemv launch");
}

}  // namespace

extern "C" {

int dcb_gemv_i8(const int8_t* w, const float* scales, const float* bias, const float* x, float* y, int rows,
                int cols, void* stream) {
    if (!w || !scales || !x || !y || rows <= 0 || cols <= 0) return fail(DCB_ERR_ARGUMENT, "invalid matvec arguments");
    if (cols % 4) return fail(DCB_ERR_ARGUMENT, "int8 matrices must contain a multiple of four elements");
    if ((size_t)cols * sizeof(float) > 200 * 1024) return fail(DCB_ERR_UNSUPPORTED, "matvec input longer than 51200");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const bool aligned = cols % 16 == 0 && (reinterpret_cast<uintptr_t>(w) & 15) == 0;
    if (!aligned) {
        const int blocks = (rows + GEMV_WARPS - 1) / GEMV_WARPS;
        gemv_i8_narrow_kernel<<<blocks, GEMV_THREADS, 0, st>>>(w, scales, bias, x, y, rows, cols);
        cudaError_t e = cudaGetLastError();
        return e == cudaSuccess ? 0 : cuda_fail(e, "gemv launch");
    }
    // Four rows per warp once there are enough rows to fill the GPU twice over.
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (rows >= 2 * sms * GEMV_WARPS * 4) return launch_gemv<4>(w, scales, bias, x, y, rows, cols, st);
    return launch_gemv<1>(w, scales, bias, x, y, rows, cols, st);
}

int dcb_attention(const float* q_in, const void* keys, const void* values, int kv_dtype, float* out, int length,
                  int heads, int kv_heads, int dim, float rope_theta, void* stream) {
    if (!q_in || !keys || !values || !out || length <= 0 || kv_heads <= 0 || heads % kv_heads || dim <= 0 ||
        dim % 2 || dim > 128)
        return fail(DCB_ERR_ARGUMENT, "invalid attention dimensions");
    if (kv_dtype != DCB_KV_F32 && kv_dtype != DCB_KV_F16) return fail(DCB_ERR_ARGUMENT, "invalid KV dtype");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int chunks = (length + KV_CHUNK - 1) / KV_CHUNK;
    const int want = std::max(1, 2 * sms / kv_heads);
    const int n = std::min(chunks, want);
    const int split_len = ((chunks + n - 1) / n) * KV_CHUNK;
    const int nsplit = (length + split_len - 1) / split_len;
    const int gq = heads / kv_heads;
    // Scratch: rope table, partials, per-group counters (stream-ordered).
    const size_t inv_bytes = 256 * sizeof(float);
    const size_t part_bytes = (size_t)heads * nsplit * (dim + 2) * sizeof(float);
    const size_t cnt_bytes = (size_t)kv_heads * sizeof(unsigned);
    char* scratch = nullptr;
    cudaError_t e = cudaMallocAsync((void**)&scratch, inv_bytes + part_bytes + cnt_bytes, st);
    if (e != cudaSuccess) return cuda_fail(e, "attention scratch");
    float* inv = reinterpret_cast<float*>(scratch);
    float* part = reinterpret_cast<float*>(scratch + inv_bytes);
    unsigned* cnt = reinterpret_cast<unsigned*>(scratch + inv_bytes + part_bytes);
    cudaMemsetAsync(cnt, 0, cnt_bytes, st);
    AttnIO io;
    io.q = q_in;
    io.rope_inv = nullptr;
    io.rope_pos = length - 1;
    if (rope_theta > 0) {
        rope_inv_kernel<<<1, 64, 0, st>>>(inv, dim, rope_theta);
        io.rope_inv = inv;
    }
    io.keys = keys;
    io.values = values;
    io.out = out;
    io.part = part;
    io.group_done = cnt;
    io.heads = heads;
    io.kv_heads = kv_heads;
    io.d = dim;
    io.length = length;
    io.nsplit = nsplit;
    io.split_len = split_len;
    const size_t smem = attention_smem_floats(dim, gq) * sizeof(float);
    const int threads = std::min(512, std::max(128, ((gq + 3) / 4) * 128));
    if (kv_dtype == DCB_KV_F16) {
        cudaFuncSetAttribute(attention_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        attention_kernel<__half><<<kv_heads * nsplit, threads, smem, st>>>(io);
    } else {
        cudaFuncSetAttribute(attention_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        attention_kernel<float><<<kv_heads * nsplit, threads, smem, st>>>(io);
    }
    e = cudaGetLastError();
    cudaFreeAsync(scratch, st);
    return e == cudaSuccess ? 0 : cuda_fail(e, "attention launch");
}

int dcb_rmsnorm(const float* x, const float* w, float* out, int n, float eps, void* stream) {
    if (!x || !w || !out || n <= 0) return fail(DCB_ERR_ARGUMENT, "invalid rmsnorm arguments");
    rmsnorm_kernel<<<1, 1024, 0, static_cast<cudaStream_t>(stream)>>>(x, w, out, n, eps);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : cuda_fail(e, "rmsnorm launch");
}

int dcb_rope(float* x, int heads, int dim, int pos, float theta, int direct, void* stream) {
    if (!x || heads <= 0 || dim <= 0 || dim % 2 || pos < 0) return fail(DCB_ERR_ARGUMENT, "invalid rope arguments");
    const int n = heads * dim / 2;
    rope_kernel<<<(n + 255) / 256, 256, 0, static_cast<cudaStream_t>(stream)>>>(x, heads, dim, pos, theta, direct);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : cuda_fail(e, "rope launch");
}

int dcb_argmax(const float* x, int n, int* out, void* stream) {
    if (!x || !out || n <= 0) return fail(DCB_ERR_ARGUMENT, "invalid argmax arguments");
    argmax_kernel<<<1, 1024, 0, static_cast<cudaStream_t>(stream)>>>(x, n, out);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : cuda_fail(e, "argmax launch");
}

}  // extern "C"

// ---- attention with its scratch in a static device array --------------------------
// dcb_attention_noalloc is dcb_attention with the cudaMallocAsync scratch
// replaced by one fixed array per device, for callers that must not allocate
// device memory per call. Layout: [0, 1 KiB) RoPE inverse frequencies (256
// floats), [1 KiB, 2 KiB) per-group arrival counters (up to 256 unsigned), then
// the split partials (heads x splits x (dim + 2) floats).
#include <mutex>

namespace {
constexpr size_t NOALLOC_BYTES = DCB_ATTENTION_NOALLOC_SCRATCH_BYTES;
constexpr size_t NOALLOC_CNT_OFF = 1024, NOALLOC_PART_OFF = 2048;
constexpr int NOALLOC_MAX_KV_HEADS = 256;
constexpr int NOALLOC_MAX_DEVICES = 64;

__device__ __align__(256) unsigned char g_attention_scratch[NOALLOC_BYTES];

struct NoallocDevice {
    std::once_flag once;
    cudaError_t status = cudaSuccess;
    const char* what = "";
    char* scratch = nullptr;
    int sms = 0;
    int max_dynamic[2] = {0, 0};  // dynamic shared memory cap of attention_kernel<float>, <__half>
};
NoallocDevice g_noalloc[NOALLOC_MAX_DEVICES];

template <typename KV>
cudaError_t raise_smem_cap(int optin, int& cap) {
    cudaFuncAttributes fa;
    cudaError_t e = cudaFuncGetAttributes(&fa, attention_kernel<KV>);
    if (e != cudaSuccess) return e;
    cap = optin - (int)fa.sharedSizeBytes;
    return cudaFuncSetAttribute(attention_kernel<KV>, cudaFuncAttributeMaxDynamicSharedMemorySize, cap);
}

// Once per device, with that device current: the scratch's device address and
// the kernel attributes (the dynamic shared memory cap raised to what the
// device allows next to the kernel's static shared memory, so later calls set
// nothing).
void noalloc_setup(NoallocDevice& d, int dev) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_attention_scratch);
    if (e != cudaSuccess) {
        d.status = e;
        d.what = "attention scratch address";
        return;
    }
    d.scratch = static_cast<char*>(p);
    int optin = 0;
    if ((e = cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess ||
        (e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev)) != cudaSuccess) {
        d.status = e;
        d.what = "device attributes";
        return;
    }
    if ((e = raise_smem_cap<float>(optin, d.max_dynamic[0])) != cudaSuccess ||
        (e = raise_smem_cap<__half>(optin, d.max_dynamic[1])) != cudaSuccess) {
        d.status = e;
        d.what = "attention kernel attributes";
    }
}
}  // namespace

extern "C" int dcb_attention_noalloc(const float* q_in, const void* keys, const void* values, int kv_dtype,
                                     float* out, int length, int heads, int kv_heads, int dim, float rope_theta,
                                     void* stream) {
    if (!q_in || !keys || !values || !out || length <= 0 || kv_heads <= 0 || heads % kv_heads || dim <= 0 ||
        dim % 2 || dim > 128)
        return fail(DCB_ERR_ARGUMENT, "invalid attention dimensions");
    if (kv_dtype != DCB_KV_F32 && kv_dtype != DCB_KV_F16) return fail(DCB_ERR_ARGUMENT, "invalid KV dtype");
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "current device");
    if (dev < 0 || dev >= NOALLOC_MAX_DEVICES)
        return fail(DCB_ERR_UNSUPPORTED, "dcb_attention_noalloc supports device ordinals below 64");
    NoallocDevice& d = g_noalloc[dev];
    std::call_once(d.once, noalloc_setup, std::ref(d), dev);
    if (d.status != cudaSuccess) return cuda_fail(d.status, d.what);

    // The split of dcb_attention, so both produce the same partials.
    const int chunks = (length + KV_CHUNK - 1) / KV_CHUNK;
    const int want = std::max(1, 2 * d.sms / kv_heads);
    const int n = std::min(chunks, want);
    const int split_len = ((chunks + n - 1) / n) * KV_CHUNK;
    const int nsplit = (length + split_len - 1) / split_len;
    const int gq = heads / kv_heads;
    const size_t part_bytes = (size_t)heads * nsplit * (dim + 2) * sizeof(float);
    if (kv_heads > NOALLOC_MAX_KV_HEADS || NOALLOC_PART_OFF + part_bytes > NOALLOC_BYTES)
        return fail(DCB_ERR_ARGUMENT,
                    "dcb_attention_noalloc: needs " + std::to_string(NOALLOC_PART_OFF + part_bytes) +
                        " bytes of scratch (" + std::to_string(kv_heads) + " KV heads, " + std::to_string(heads) +
                        " heads x " + std::to_string(nsplit) + " splits x " + std::to_string(dim + 2) +
                        " floats); the static scratch holds " + std::to_string(NOALLOC_BYTES) +
                        " bytes and at most 256 KV heads");
    const size_t smem = attention_smem_floats(dim, gq) * sizeof(float);
    if (smem > (size_t)d.max_dynamic[kv_dtype == DCB_KV_F16 ? 1 : 0])
        return fail(DCB_ERR_UNSUPPORTED, "attention needs more shared memory than a block has");

    cudaStream_t st = static_cast<cudaStream_t>(stream);
    float* inv = reinterpret_cast<float*>(d.scratch);
    unsigned* cnt = reinterpret_cast<unsigned*>(d.scratch + NOALLOC_CNT_OFF);
    float* part = reinterpret_cast<float*>(d.scratch + NOALLOC_PART_OFF);
    // The arrival counters must be zero when the kernel starts.
    if ((e = cudaMemsetAsync(cnt, 0, (size_t)kv_heads * sizeof(unsigned), st)) != cudaSuccess)
        return cuda_fail(e, "attention counters");
    AttnIO io;
    io.q = q_in;
    io.rope_inv = nullptr;
    io.rope_pos = length - 1;
    if (rope_theta > 0) {
        rope_inv_kernel<<<1, 64, 0, st>>>(inv, dim, rope_theta);
        io.rope_inv = inv;
    }
    io.keys = keys;
    io.values = values;
    io.out = out;
    io.part = part;
    io.group_done = cnt;
    io.heads = heads;
    io.kv_heads = kv_heads;
    io.d = dim;
    io.length = length;
    io.nsplit = nsplit;
    io.split_len = split_len;
    const int threads = std::min(512, std::max(128, ((gq + 3) / 4) * 128));
    if (kv_dtype == DCB_KV_F16)
        attention_kernel<__half><<<kv_heads * nsplit, threads, smem, st>>>(io);
    else
        attention_kernel<float><<<kv_heads * nsplit, threads, smem, st>>>(io);
    e = cudaGetLastError();
    return e == cudaSuccess ? 0 : cuda_fail(e, "attention launch");
}
