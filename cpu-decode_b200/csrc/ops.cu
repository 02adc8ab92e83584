// Isolated operators behind the C ABI: int8 GEMV (+bias), split-KV GQA
// attention, RMSNorm, RoPE and argmax, each on caller-provided device memory.
// They share the device code of the fused step kernel, so the GEMV sweep and
// the attention sweep measure the same inner loops.
#include <mutex>
#include <set>
#include <utility>
#include "decode_b200.h"
#include "attention.cuh"
#include "device.cuh"

#include <cuda_runtime.h>
#include <algorithm>
#include <atomic>
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

constexpr int GEMV_NT = 512, GEMV_NW = GEMV_NT / 32;

// y[r] = scale[r] * dot(w[r], x) (+ bias[r]) for rows of a multiple of 16
// int8 (16-byte aligned). Persistent: every block stages x once as three
// fixed-point byte planes (scale max|x| / FIX_MAX), then its warps take row
// groups of R in turn, each lane streaming 16-byte chunks lane, lane + 32, ...
// with U chunks of all R rows in flight, three exact dp4a per 4 weights.
template <int R, int U>
__global__ void __launch_bounds__(GEMV_NT) gemv_dp4a_kernel(const int8_t* __restrict__ w,
                                                          const float* __restrict__ scales,
                                                          const float* __restrict__ bias,
                                                          const float* __restrict__ x, float* __restrict__ y,
                                                          int rows, int cols) {
    extern __shared__ __align__(16) int8_t xq[];  // planes hi | mid | lo, cols bytes each
    __shared__ float red[GEMV_NW];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    float mx = 0.f;
    for (int j = tid; j < cols; j += GEMV_NT) mx = fmaxf(mx, fabsf(__ldg(x + j)));
    mx = warp_max(mx);
    if (lane == 0) red[warp] = mx;
    __syncthreads();
    float M = 0.f;
#pragma unroll
    for (int k = 0; k < GEMV_NW; ++k) M = fmaxf(M, red[k]);
    const float rs = M > 0.f ? FIX_MAX * __frcp_rn(M) : 0.f;
    const float xs = M > 0.f ? __frcp_rn(rs) : 1.f;
    for (int quad = tid; quad < cols / 4; quad += GEMV_NT) {
        const float4 v = make_float4(__ldg(x + 4 * quad), __ldg(x + 4 * quad + 1), __ldg(x + 4 * quad + 2),
                                     __ldg(x + 4 * quad + 3));
        uint32_t ph, pm, pl;
        fix_pack4(v, rs, ph, pm, pl);
        reinterpret_cast<uint32_t*>(xq)[quad] = ph;
        reinterpret_cast<uint32_t*>(xq + cols)[quad] = pm;
        reinterpret_cast<uint32_t*>(xq + 2 * cols)[quad] = pl;
    }
    __syncthreads();
    const int nch = cols / 16;
    const int stride = gridDim.x * GEMV_NW * R;
    for (int r0 = (blockIdx.x * GEMV_NW + warp) * R; r0 < rows; r0 += stride) {
        int ah[R], am[R], al[R];
#pragma unroll
        for (int r = 0; r < R; ++r) ah[r] = am[r] = al[r] = 0;
        for (int c0 = lane; c0 < nch; c0 += 32 * U) {
            int4 wv[U][R];
#pragma unroll
            for (int u = 0; u < U; ++u)
#pragma unroll
                for (int r = 0; r < R; ++r) {
                    const int c = c0 + 32 * u;
                    wv[u][r] = (c < nch && r0 + r < rows) ? ld_stream(w + (size_t)(r0 + r) * cols + (size_t)c * 16)
                                                          : make_int4(0, 0, 0, 0);
                }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int c = c0 + 32 * u;
                if (c < nch) {
                    int4 h, m, l;
                    load_planes(xq, cols, c, h, m, l);
#pragma unroll
                    for (int r = 0; r < R; ++r) dp4a16(wv[u][r], h, m, l, ah[r], am[r], al[r]);
                }
            }
        }
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const float t = warp_sum(planes_to_float(ah[r], am[r], al[r]));
            if (lane == 0 && r0 + r < rows) {
                const float v = t * xs * scales[r0 + r];
                y[r0 + r] = bias ? v + bias[r0 + r] : v;
            }
        }
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

// ---- read-bandwidth probe ---------------------------------------------------------
constexpr int PROBE_NT = 512, PROBE_BLOCKS_PER_SM = 4, PROBE_ILP = 4;

// Word i = i * 6364136223846793005 + 1 (tools/bandwidth.cpp:83-84).
__global__ void fill_probe_kernel(uint64_t* p, size_t n) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        p[i] = i * 6364136223846793005ull + 1ull;
}

// `passes` sweeps of n 16-byte pieces, PROBE_ILP streaming loads in flight per
// thread, XOR-folded so nothing is skipped; one XOR per warp into *sum.
__global__ void __launch_bounds__(PROBE_NT) read_probe_kernel(const int4* __restrict__ p, size_t n, int passes,
                                                           unsigned long long* sum) {
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    uint64_t acc = 0;
    for (int pass = 0; pass < passes; ++pass) {
        size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
        for (; i + (PROBE_ILP - 1) * stride < n; i += PROBE_ILP * stride) {
            int4 v[PROBE_ILP];
#pragma unroll
            for (int k = 0; k < PROBE_ILP; ++k) v[k] = ld_stream(p + i + k * stride);
#pragma unroll
            for (int k = 0; k < PROBE_ILP; ++k)
                acc ^= (((uint64_t)(uint32_t)v[k].y << 32) | (uint32_t)v[k].x) ^
                       (((uint64_t)(uint32_t)v[k].w << 32) | (uint32_t)v[k].z);
        }
        for (; i < n; i += stride) {
            const int4 v = ld_stream(p + i);
            acc ^= (((uint64_t)(uint32_t)v.y << 32) | (uint32_t)v.x) ^ (((uint64_t)(uint32_t)v.w << 32) | (uint32_t)v.z);
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc ^= __shfl_xor_sync(FULL, acc, o);
    if ((threadIdx.x & 31) == 0 && acc) atomicXor(sum, (unsigned long long)acc);
}

// Multiprocessor count of each device, looked up once.
std::atomic<int> g_sm_count[64];
int sm_count() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    int n = g_sm_count[dev].load(std::memory_order_relaxed);
    if (!n) {
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        g_sm_count[dev].store(n, std::memory_order_relaxed);
    }
    return n;
}

// Raise kernel k's dynamic shared-memory cap, once per device, to what the
// device allows next to the kernel's static shared memory. Only ever raised:
// threads launching the same kernel with different sizes cannot lower it
// under one another, and later calls touch no attribute.
std::mutex g_cap_mutex;
std::set<std::pair<int, const void*>> g_cap_done;
cudaError_t ensure_smem_cap(const void* k) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    std::lock_guard<std::mutex> lock(g_cap_mutex);
    if (g_cap_done.count({dev, k})) return cudaSuccess;
    int optin = 0;
    cudaFuncAttributes fa;
    if ((e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev)) != cudaSuccess ||
        (e = cudaFuncGetAttributes(&fa, k)) != cudaSuccess ||
        (e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, optin - (int)fa.sharedSizeBytes)) !=
            cudaSuccess)
        return e;
    g_cap_done.insert({dev, k});
    return cudaSuccess;
}

template <int R, int U>
int launch_gemv(const int8_t* w, const float* s, const float* b, const float* x, float* y, int rows, int cols,
                cudaStream_t st) {
    const int groups = (rows + R - 1) / R;
    const int blocks = std::max(1, std::min(2 * sm_count(), (groups + GEMV_NW - 1) / GEMV_NW));
    const size_t smem = 3 * (size_t)cols;
    const void* k = (const void*)gemv_dp4a_kernel<R, U>;
    if (smem > 48 * 1024) {
        cudaError_t e = ensure_smem_cap(k);
        if (e != cudaSuccess) return cuda_fail(e, "gemv shared memory");
    }
    void* args[] = {(void*)&w, (void*)&s, (void*)&b, (void*)&x, (void*)&y, (void*)&rows, (void*)&cols};
    cudaError_t e = cudaLaunchKernel(k, dim3(blocks), dim3(GEMV_NT), args, smem, st);
    return e == cudaSuccess ? 0 : cuda_fail(e, "gemv launch");
}

// Split plan of the isolated attention: about two blocks per SM across the KV
// heads, whole 64-position chunks per split.
void attention_plan(int length, int kv_heads, int sms, int* nsplit, int* split_len) {
    const int chunks = (length + AT_T - 1) / AT_T;
    const int want = std::max(1, 2 * sms / kv_heads);
    const int n = std::min(chunks, want);
    *split_len = ((chunks + n - 1) / n) * AT_T;
    *nsplit = (length + *split_len - 1) / *split_len;
}

template <typename KV, int DT>
cudaError_t launch_split(const AttnIO& io, size_t smem, cudaStream_t st) {
    const void* k = (const void*)attention_split_kernel<KV, DT>;
    if (smem > 48 * 1024) {
        cudaError_t e = ensure_smem_cap(k);
        if (e != cudaSuccess) return e;
    }
    AttnIO a = io;
    void* args[] = {(void*)&a};
    return cudaLaunchKernel(k, dim3(io.kv_heads * io.nsplit), dim3(AT_NT), args, smem, st);
}

template <typename KV>
cudaError_t launch_group(const AttnIO& io, size_t smem, cudaStream_t st) {
    const void* k = (const void*)attention_group_kernel<KV>;
    if (smem > 48 * 1024) {
        cudaError_t e = ensure_smem_cap(k);
        if (e != cudaSuccess) return e;
    }
    AttnIO a = io;
    void* args[] = {(void*)&a};
    return cudaLaunchKernel(k, dim3(io.kv_heads * io.nsplit), dim3(AT_NT), args, smem, st);
}

// The split kernel, then (several splits) the combine kernel, on stream st.
int launch_attention(const AttnIO& io, int kv_dtype, cudaStream_t st) {
    const int es = kv_dtype == DCB_KV_F16 ? 2 : 4;
    const size_t smem = attention_smem_bytes(io.d, es, io.heads / io.kv_heads);
    int dev = 0, optin = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (smem + 1024 > (size_t)optin)
        return fail(DCB_ERR_UNSUPPORTED, "attention needs more shared memory than a block has");
    cudaError_t e;
    if (io.d == 64 && io.heads / io.kv_heads <= AT_GH) {
        // head_dim 64, up to AT_GH query heads per KV head: the group kernel.
        const size_t gs = attention_group_smem_bytes(es, io.heads / io.kv_heads);
        e = kv_dtype == DCB_KV_F16 ? launch_group<__half>(io, gs, st) : launch_group<float>(io, gs, st);
    } else if (kv_dtype == DCB_KV_F16) {
        e = io.d == 64 ? launch_split<__half, 64>(io, smem, st) : launch_split<__half, 0>(io, smem, st);
    } else {
        e = io.d == 64 ? launch_split<float, 64>(io, smem, st) : launch_split<float, 0>(io, smem, st);
    }
    if (e != cudaSuccess) return cuda_fail(e, "attention launch");
    if (io.nsplit > 1) {
        AttnIO a = io;
        void* args[] = {(void*)&a};
        e = cudaLaunchKernel((const void*)attention_combine_kernel, dim3(io.heads), dim3(AT_NT), args, 0, st);
        if (e != cudaSuccess) return cuda_fail(e, "attention combine launch");
    }
    return 0;
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
    // Rows per warp: as many (up to 4) as every warp of two blocks per SM gets.
    const int warps = 2 * sm_count() * GEMV_NW;
    if (rows >= 4 * warps) return launch_gemv<4, 2>(w, scales, bias, x, y, rows, cols, st);
    if (rows >= 2 * warps) return launch_gemv<2, 2>(w, scales, bias, x, y, rows, cols, st);
    return launch_gemv<1, 4>(w, scales, bias, x, y, rows, cols, st);
}

int dcb_attention(const float* q_in, const void* keys, const void* values, int kv_dtype, float* out, int length,
                  int heads, int kv_heads, int dim, float rope_theta, void* stream) {
    if (!q_in || !keys || !values || !out || length <= 0 || kv_heads <= 0 || heads % kv_heads || dim <= 0 ||
        dim % 2 || dim > 128)
        return fail(DCB_ERR_ARGUMENT, "invalid attention dimensions");
    if (kv_dtype != DCB_KV_F32 && kv_dtype != DCB_KV_F16) return fail(DCB_ERR_ARGUMENT, "invalid KV dtype");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    AttnIO io;
    io.q = q_in;
    io.keys = keys;
    io.values = values;
    io.out = out;
    io.part = nullptr;
    io.rope_theta = rope_theta;
    io.heads = heads;
    io.kv_heads = kv_heads;
    io.d = dim;
    io.length = length;
    attention_plan(length, kv_heads, sm_count(), &io.nsplit, &io.split_len);
    // Scratch: the split partials (stream-ordered).
    float* part = nullptr;
    if (io.nsplit > 1) {
        const size_t part_bytes = (size_t)heads * io.nsplit * (dim + 2) * sizeof(float);
        cudaError_t e = cudaMallocAsync((void**)&part, part_bytes, st);
        if (e != cudaSuccess) return cuda_fail(e, "attention scratch");
        io.part = part;
    }
    const int rc = launch_attention(io, kv_dtype, st);
    if (part) cudaFreeAsync(part, st);
    return rc;
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

int dcb_read_bandwidth(int device, size_t mib, int passes, int repeats, double* gb_per_s, uint64_t* checksum) {
    if (mib < 32 || mib > 65536 || passes < 1 || repeats < 1 || !gb_per_s)
        return fail(DCB_ERR_ARGUMENT, "invalid sweep parameters");
    int caller_device = 0;
    cudaError_t e = cudaGetDevice(&caller_device);
    if (e != cudaSuccess) return cuda_fail(e, "current device");
    e = cudaSetDevice(device);
    if (e != cudaSuccess) return cuda_fail(e, "read probe device");
    const size_t bytes = mib << 20, words = bytes / sizeof(uint64_t);
    int sms = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    uint64_t* data = nullptr;
    unsigned long long* sum = nullptr;
    cudaStream_t st = nullptr;
    cudaEvent_t t0 = nullptr, t1 = nullptr;
    int rc = 0;
    auto check = [&](cudaError_t err, const char* what) {
        if (err != cudaSuccess && !rc) rc = cuda_fail(err, what);
        return rc == 0;
    };
    const int grid = std::max(1, sms) * PROBE_BLOCKS_PER_SM;
    auto sweep = [&](int count) {
        read_probe_kernel<<<grid, PROBE_NT, 0, st>>>(reinterpret_cast<const int4*>(data), bytes / 16, count, sum);
        return check(cudaGetLastError(), "read probe launch");
    };
    if (check(cudaMalloc(&data, bytes), "read probe array") && check(cudaMalloc(&sum, sizeof(*sum)), "read probe sum") &&
        check(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking), "read probe stream") &&
        check(cudaEventCreate(&t0), "read probe event") && check(cudaEventCreate(&t1), "read probe event")) {
        fill_probe_kernel<<<grid, PROBE_NT, 0, st>>>(data, words);
        if (check(cudaGetLastError(), "read probe fill") && sweep(3)) {
            for (int r = 0; r < repeats && rc == 0; ++r) {
                float ms = 0.f;
                if (check(cudaEventRecord(t0, st), "read probe event") && sweep(passes) &&
                    check(cudaEventRecord(t1, st), "read probe event") &&
                    check(cudaEventSynchronize(t1), "read probe sweep") &&
                    check(cudaEventElapsedTime(&ms, t0, t1), "read probe time"))
                    gb_per_s[r] = (double)bytes * passes / (ms / 1000.0) / 1e9;
            }
            // The checksum of one sweep (an odd count: repeated sweeps would cancel).
            unsigned long long host = 0;
            if (rc == 0 && check(cudaMemsetAsync(sum, 0, sizeof(*sum), st), "read probe sum") && sweep(1) &&
                check(cudaMemcpyAsync(&host, sum, sizeof(host), cudaMemcpyDeviceToHost, st), "read probe sum") &&
                check(cudaStreamSynchronize(st), "read probe sum") && checksum)
                *checksum = host;
        }
    }
    if (st) cudaStreamSynchronize(st);
    if (t0) cudaEventDestroy(t0);
    if (t1) cudaEventDestroy(t1);
    if (st) cudaStreamDestroy(st);
    if (data) cudaFree(data);
    if (sum) cudaFree(sum);
    cudaSetDevice(caller_device);  // the calling thread keeps its device
    return rc;
}

}  // extern "C"

namespace {
// One warp per row of BF16 weights: the reference's per-row rule
// (src/kernels.cpp:121-131) in IEEE FP32: the largest magnitude, scale =
// max / 127 (1 for an all-zero row), each weight / scale rounded half away
// from zero (roundf) and clamped to [-127, 127]. A non-finite weight raises
// *bad (the row's output is then not used).
constexpr int QZ_ROWS = 8;  // rows (warps) per block
__global__ void __launch_bounds__(32 * QZ_ROWS) quantize_rows_kernel(const uint16_t* __restrict__ w, size_t rows,
                                                                      size_t cols, int8_t* __restrict__ q,
                                                                      float* __restrict__ scales, int* bad) {
    const size_t r = (size_t)blockIdx.x * QZ_ROWS + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (r >= rows) return;
    const uint16_t* row = w + r * cols;
    float peak = 0.f;
    bool finite = true;
    for (size_t j = lane; j < cols; j += 32) {
        const float v = __uint_as_float((uint32_t)row[j] << 16);
        finite = finite && isfinite(v);
        peak = fmaxf(peak, fabsf(v));
    }
    peak = warp_max(peak);
    if (!__all_sync(FULL, finite)) {
        if (lane == 0) atomicExch(bad, 1);
        return;
    }
    const float scale = peak > 0.f ? __fdiv_rn(peak, 127.0f) : 1.0f;
    int8_t* out = q + r * cols;
    for (size_t j = lane; j < cols; j += 32) {
        const float v = __uint_as_float((uint32_t)row[j] << 16);
        const float x = roundf(__fdiv_rn(v, scale));
        out[j] = (int8_t)(x > 127.f ? 127.f : (x < -127.f ? -127.f : x));
    }
    if (lane == 0) scales[r] = scale;
}
}  // namespace

extern "C" int dcb_quantize_rows_bf16(const uint16_t* weights, size_t rows, size_t cols, int8_t* out, float* scales,
                                      int device) {
    if (!weights || !out || !scales) return fail(DCB_ERR_ARGUMENT, "null argument");
    if (!rows) return 0;
    if (!cols) return fail(DCB_ERR_ARGUMENT, "empty quantization row");
    int caller_device = 0;
    cudaError_t e = cudaGetDevice(&caller_device);
    if (e != cudaSuccess) return cuda_fail(e, "current device");
    e = cudaSetDevice(device);
    if (e != cudaSuccess) return cuda_fail(e, "quantiser device");
    uint16_t* dw = nullptr;
    int8_t* dq = nullptr;
    float* ds = nullptr;
    int* dbad = nullptr;
    int bad = 0, rc = 0;
    auto check = [&](cudaError_t err, const char* what) {
        if (err != cudaSuccess && !rc) rc = cuda_fail(err, what);
        return rc == 0;
    };
    const size_t n = rows * cols;
    if (check(cudaMalloc(&dw, n * 2), "quantiser input") && check(cudaMalloc(&dq, n), "quantiser output") &&
        check(cudaMalloc(&ds, rows * 4), "quantiser scales") && check(cudaMalloc(&dbad, 4), "quantiser flag") &&
        check(cudaMemset(dbad, 0, 4), "quantiser flag") &&
        check(cudaMemcpy(dw, weights, n * 2, cudaMemcpyHostToDevice), "quantiser upload")) {
        quantize_rows_kernel<<<(unsigned)((rows + QZ_ROWS - 1) / QZ_ROWS), 32 * QZ_ROWS>>>(dw, rows, cols, dq, ds,
                                                                                           dbad);
        if (check(cudaGetLastError(), "quantiser launch") && check(cudaMemcpy(&bad, dbad, 4, cudaMemcpyDeviceToHost),
                                                                    "quantiser flag") && !bad) {
            check(cudaMemcpy(out, dq, n, cudaMemcpyDeviceToHost), "quantiser download");
            check(cudaMemcpy(scales, ds, rows * 4, cudaMemcpyDeviceToHost), "quantiser download");
        }
    }
    if (dw) cudaFree(dw);
    if (dq) cudaFree(dq);
    if (ds) cudaFree(ds);
    if (dbad) cudaFree(dbad);
    cudaSetDevice(caller_device);
    if (!rc && bad) rc = fail(DCB_ERR_ARGUMENT, "nonfinite model weight");
    return rc;
}

// ---- attention with its scratch in a static device array --------------------------
// dcb_attention_noalloc is dcb_attention with the cudaMallocAsync scratch
// replaced by one fixed array per device, for callers that must not allocate
// device memory per call. The array holds the split partials (heads x splits
// x (dim + 2) floats); a call writes every word it reads, so nothing in it has
// to start at zero.

namespace {
constexpr size_t NOALLOC_BYTES = DCB_ATTENTION_NOALLOC_SCRATCH_BYTES;
constexpr int NOALLOC_MAX_DEVICES = 64;

__device__ __align__(256) unsigned char g_attention_scratch[NOALLOC_BYTES];

struct NoallocDevice {
    std::once_flag once;
    cudaError_t status = cudaSuccess;
    const char* what = "";
    char* scratch = nullptr;
    int sms = 0;
};
NoallocDevice g_noalloc[NOALLOC_MAX_DEVICES];

// Once per device, with that device current: the scratch's device address
// (the kernels' shared-memory caps are raised once per device by the launch
// helpers, as for dcb_attention).
void noalloc_setup(NoallocDevice& d, int dev) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_attention_scratch);
    if (e != cudaSuccess) {
        d.status = e;
        d.what = "attention scratch address";
        return;
    }
    d.scratch = static_cast<char*>(p);
    if ((e = cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) {
        d.status = e;
        d.what = "device attributes";
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

    AttnIO io;
    io.q = q_in;
    io.keys = keys;
    io.values = values;
    io.out = out;
    io.part = reinterpret_cast<float*>(d.scratch);
    io.rope_theta = rope_theta;
    io.heads = heads;
    io.kv_heads = kv_heads;
    io.d = dim;
    io.length = length;
    // The split of dcb_attention, so both produce the same partials.
    attention_plan(length, kv_heads, d.sms, &io.nsplit, &io.split_len);
    const size_t part_bytes = io.nsplit > 1 ? (size_t)heads * io.nsplit * (dim + 2) * sizeof(float) : 0;
    if (part_bytes > NOALLOC_BYTES)
        return fail(DCB_ERR_ARGUMENT,
                    "dcb_attention_noalloc: needs " + std::to_string(part_bytes) + " bytes of scratch (" +
                        std::to_string(heads) + " heads x " + std::to_string(io.nsplit) + " splits x " +
                        std::to_string(dim + 2) + " floats); the static scratch holds " +
                        std::to_string(NOALLOC_BYTES) + " bytes");
    return launch_attention(io, kv_dtype, static_cast<cudaStream_t>(stream));
}
