// The decode step as one persistent cooperative kernel (one block per SM) and
// the host engine behind the C ABI in include/decode_b200.h.
//
// One launch runs the reference's Engine::Impl::step (src/model.cpp:258-329)
// for one token: embedding, then per layer five phases separated by grid-wide
// barriers
//   QKV  : RMSNorm prologue, fused Q/K/V int8 GEMV + bias + split-half RoPE,
//          K/V written to the cache at `pos`
//   ATTN : split-KV flash-decoding attention (one block per KV head x split)
//   O    : O GEMV, residual added into x
//   GU   : RMSNorm prologue, fused gate/up GEMV, SiLU(gate)*up
//   DOWN : down GEMV, residual added into x
// and finally the final RMSNorm, the tied LM head and a device argmax.
// While a block waits at a barrier, the weights of later phases are already
// streaming into L2 (cp.async.bulk.prefetch.L2), so HBM stays busy across the
// dependency chain.
#include "decode_b200.h"
#include "attention.cuh"
#include "device.cuh"

#include <cuda_runtime.h>
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

namespace dcb {

void set_last_error(const std::string& msg);

constexpr int NT = 512;
constexpr int NW = NT / 32;
constexpr int MAX_KV_HEADS = 64;
constexpr uint64_t WAIT_LIMIT_NS = 1000000000ull;  // one second
constexpr int ERR_BARRIER = 1;
constexpr int ERR_TOKEN = 2;

struct LayerW {
    const int8_t* qkv;  // [qkv_rows][Kh], RoPE pairs (j, j+d/2) adjacent
    const float* qkv_scale;
    const float* qkv_bias;
    const int8_t* o;  // [H][Kh]
    const float* o_scale;
    const int8_t* gu;  // [2I][Kh], rows (gate_j, up_j) adjacent
    const float* gu_scale;
    const int8_t* down;  // [H][Ki]
    const float* down_scale;
    const float* in_norm;
    const float* post_norm;
};

struct Sync {
    unsigned arrive;
    unsigned done;
    unsigned amax_done;
    int error;
    unsigned group_done[MAX_KV_HEADS];
};

struct ArgBest {
    float v;
    int i;
};

struct Params {
    int H, I, L, NH, NKV, D, V, Kh, Ki, qkv_rows;
    float eps;
    int cached_rope;
    size_t capacity;
    const LayerW* layers;
    const int8_t* embed;  // [V][Kh]
    const float* embed_scale;
    const float* final_norm;
    const float* rope_inv;  // [D/2] 1/theta^(2j/D)      (cached formula)
    const float* rope_den;  // [D/2] theta^(2j/D)        (direct formula)
    void* kcache;           // [L][capacity][kvd]
    void* vcache;
    float* x;       // [Kh] residual stream
    float* q;       // [H] rotated queries
    float* attn;    // [Kh]
    float* hbuf;    // [Ki]
    float* logits;  // [V]
    float* part;    // attention partials
    ArgBest* amax;  // [grid]
    Sync* sync;
    int* result;    // [0] argmax of the last head step
    int xs_floats;  // staged-activation floats in shared memory
    int prefetch_ahead;
    int head_prefetch_rows;
};

struct StepArgs {
    int token;
    const int* token_dev;
    int pos;
    int head;
    int* argmax_dev;
    int nsplit;
    int split_len;
};

__device__ __forceinline__ bool better(float v, int i, float bv, int bi) {
    return v > bv || (v == bv && i < bi);
}

// Grid barrier with a bounded wait. Returns false when the step must abort.
__device__ bool grid_sync(Sync* s, unsigned target, int* s_abort) {
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        red_release_add(&s->arrive, 1u);
        const uint64_t t0 = globaltimer();
        unsigned spins = 0;
        while (ld_acquire(&s->arrive) < target) {
            if ((++spins & 15u) == 0) {
                if (ld_volatile(&s->error)) { *s_abort = 1; break; }
                if (globaltimer() - t0 > WAIT_LIMIT_NS) {
                    atomicCAS(&s->error, 0, ERR_BARRIER);
                    *s_abort = 1;
                    break;
                }
            }
        }
        __threadfence();
    }
    __syncthreads();
    return *s_abort == 0;
}

// Stage the activation for a GEMV phase into shared memory (chunk-interleaved,
// zero padded to nch*16), optionally RMS-normalised (src/kernels.cpp:132-137).
// Source: the residual stream `src`, or the embedding row of `token` when
// `embed` is set (src/model.cpp:261-267), in which case block 0 also writes
// the row to `x_out`.
__device__ void stage_vector(float4* xs4, const float* src, int n, int nch, const float* norm_w, float eps,
                             const int8_t* embed, const float* embed_scale, int token, int Kh, float* x_out,
                             float* red) {
    float* xs = reinterpret_cast<float*>(xs4);
    float ss = 0.f;
    const float es = embed ? embed_scale[token] : 0.f;
    for (int j = threadIdx.x; j < nch * 16; j += blockDim.x) {
        float v = 0.f;
        if (j < n) {
            if (embed) {
                v = (float)embed[(size_t)token * Kh + j] * es;
                if (blockIdx.x == 0) x_out[j] = v;
            } else {
                v = __ldcg(src + j);
            }
        }
        ss = fmaf(v, v, ss);
        xs[xs_index(j, nch)] = v;
    }
    if (!norm_w) {
        __syncthreads();
        return;
    }
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
    for (int j = threadIdx.x; j < n; j += blockDim.x) {
        const int ix = xs_index(j, nch);
        xs[ix] = xs[ix] * inv * norm_w[j];
    }
    __syncthreads();
}

__device__ void prefetch_phase(const Params& P, const StepArgs& A, int ph) {
    if (threadIdx.x != 0 || ph < 0) return;
    const int G = gridDim.x, b = blockIdx.x;
    if (ph >= 5 * P.L) {
        if (ph == 5 * P.L && A.head)
            prefetch_slice(P.embed, (size_t)min(P.V, P.head_prefetch_rows) * P.Kh, b, G);
        return;
    }
    const LayerW& W = P.layers[ph / 5];
    switch (ph % 5) {
    case 0: prefetch_slice(W.qkv, (size_t)P.qkv_rows * P.Kh, b, G); break;
    case 1: break;  // the KV rows are prefetched by prefetch_kv in the QKV phase
    case 2: prefetch_slice(W.o, (size_t)P.H * P.Kh, b, G); break;
    case 3: prefetch_slice(W.gu, (size_t)2 * P.I * P.Kh, b, G); break;
    case 4: prefetch_slice(W.down, (size_t)P.H * P.Ki, b, G); break;
    }
}

template <typename KV>
__device__ void prefetch_kv(const Params& P, int layer, int rows) {
    if (threadIdx.x != 0 || rows <= 0) return;
    const size_t kvd = (size_t)P.NKV * P.D;
    const size_t off = (size_t)layer * P.capacity * kvd;
    const size_t bytes = (size_t)rows * kvd * sizeof(KV);
    prefetch_slice(static_cast<const KV*>(P.kcache) + off, bytes, blockIdx.x, gridDim.x);
    prefetch_slice(static_cast<const KV*>(P.vcache) + off, bytes, blockIdx.x, gridDim.x);
}

template <int MAXC, typename KV>
__global__ void __launch_bounds__(NT, 1) decode_step_kernel(const Params P, const StepArgs A) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    float4* xs4 = reinterpret_cast<float4*>(smem_raw);
    float* att_sm = reinterpret_cast<float*>(smem_raw) + P.xs_floats;
    __shared__ float red[40];
    __shared__ int s_abort;
    __shared__ ArgBest s_best[NW];

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int G = gridDim.x, TW = G * NW, gw = blockIdx.x * NW + warp;
    const int kvd = P.NKV * P.D, half = P.D / 2;
    const int nch_h = P.Kh / 16, nch_i = P.Ki / 16;
    unsigned nbar = 0;
    if (threadIdx.x == 0) s_abort = 0;
    int token = A.token_dev ? __ldcg(A.token_dev) : A.token;
    if ((unsigned)token >= (unsigned)P.V) {  // a device-supplied token out of range
        if (threadIdx.x == 0) atomicCAS(&P.sync->error, 0, ERR_TOKEN);
        token = 0;
    }
    const float posf = (float)A.pos;

    for (int ph = 0; ph < P.prefetch_ahead; ++ph) prefetch_phase(P, A, ph);
    __syncthreads();

    for (int l = 0; l < P.L; ++l) {
        const LayerW W = P.layers[l];
        KV* kc = static_cast<KV*>(P.kcache) + (size_t)l * P.capacity * kvd;
        KV* vc = static_cast<KV*>(P.vcache) + (size_t)l * P.capacity * kvd;

        // ---- QKV: RMSNorm, Q/K/V rows + bias, RoPE, KV write (src/model.cpp:276-302)
        prefetch_phase(P, A, 5 * l + P.prefetch_ahead);
        prefetch_kv<KV>(P, l, A.pos);
        stage_vector(xs4, P.x, P.H, nch_h, W.in_norm, P.eps, l == 0 ? P.embed : nullptr, P.embed_scale, token,
                     P.Kh, P.x, red);
        {
            const int pairs = P.qkv_rows / 2, qpairs = P.NH * half, kpairs = P.NKV * half;
            for (int u = gw; u < pairs; u += TW) {
                const int8_t* rows[2] = {W.qkv + (size_t)(2 * u) * P.Kh, W.qkv + (size_t)(2 * u + 1) * P.Kh};
                float dot[2];
                rows_dot_unrolled<2, MAXC>(rows, xs4, nch_h, lane, dot);
                if (lane == 0) {
                    float y0 = dot[0] * W.qkv_scale[2 * u] + W.qkv_bias[2 * u];
                    float y1 = dot[1] * W.qkv_scale[2 * u + 1] + W.qkv_bias[2 * u + 1];
                    const int kind = u < qpairs ? 0 : (u < qpairs + kpairs ? 1 : 2);
                    const int pu = kind == 0 ? u : (kind == 1 ? u - qpairs : u - qpairs - kpairs);
                    const int head = pu / half, j = pu % half;
                    if (kind < 2) {
                        const float angle = P.cached_rope ? __fmul_rn(posf, P.rope_inv[j]) : __fdiv_rn(posf, P.rope_den[j]);
                        float sn, cs;
                        sincosf(angle, &sn, &cs);
                        const float a = y0, b = y1;
                        y0 = __fsub_rn(__fmul_rn(a, cs), __fmul_rn(b, sn));
                        y1 = __fadd_rn(__fmul_rn(b, cs), __fmul_rn(a, sn));
                    }
                    const int idx = head * P.D + j;
                    if (kind == 0) {
                        P.q[idx] = y0;
                        P.q[idx + half] = y1;
                    } else {
                        KV* dst = (kind == 1 ? kc : vc) + (size_t)A.pos * kvd;
                        kv_store(dst + idx, y0);
                        kv_store(dst + idx + half, y1);
                    }
                }
            }
        }
        if (!grid_sync(P.sync, (unsigned)G * ++nbar, &s_abort)) return;

        // ---- ATTN over positions [0, pos] (src/kernels.cpp:150-179)
        prefetch_phase(P, A, 5 * l + 1 + P.prefetch_ahead);
        {
            AttnIO io;
            io.q = P.q;
            io.rope_inv = nullptr;
            io.rope_pos = 0;
            io.keys = kc;
            io.values = vc;
            io.out = P.attn;
            io.part = P.part;
            io.group_done = P.sync->group_done;
            io.heads = P.NH;
            io.kv_heads = P.NKV;
            io.d = P.D;
            io.length = A.pos + 1;
            io.nsplit = A.nsplit;
            io.split_len = A.split_len;
            const int units = P.NKV * A.nsplit;
            for (int u = blockIdx.x; u < units; u += G) attention_unit<KV>(io, u / A.nsplit, u % A.nsplit, att_sm);
        }
        if (!grid_sync(P.sync, (unsigned)G * ++nbar, &s_abort)) return;

        // ---- O projection + residual (src/model.cpp:304-305)
        prefetch_phase(P, A, 5 * l + 2 + P.prefetch_ahead);
        stage_vector(xs4, P.attn, P.H, nch_h, nullptr, 0.f, nullptr, nullptr, 0, P.Kh, nullptr, red);
        for (int u = gw; u < (P.H + 1) / 2; u += TW) {
            const int r0 = 2 * u, r1 = 2 * u + 1;
            const int8_t* rows[2] = {W.o + (size_t)r0 * P.Kh, r1 < P.H ? W.o + (size_t)r1 * P.Kh : nullptr};
            float dot[2];
            rows_dot_unrolled<2, MAXC>(rows, xs4, nch_h, lane, dot);
            if (lane == 0) {
                P.x[r0] = __ldcg(P.x + r0) + dot[0] * W.o_scale[r0];
                if (r1 < P.H) P.x[r1] = __ldcg(P.x + r1) + dot[1] * W.o_scale[r1];
            }
        }
        if (!grid_sync(P.sync, (unsigned)G * ++nbar, &s_abort)) return;

        // ---- gate/up + SiLU (src/model.cpp:306-308)
        prefetch_phase(P, A, 5 * l + 3 + P.prefetch_ahead);
        stage_vector(xs4, P.x, P.H, nch_h, W.post_norm, P.eps, nullptr, nullptr, 0, P.Kh, nullptr, red);
        for (int u = gw; u < P.I; u += TW) {
            const int8_t* rows[2] = {W.gu + (size_t)(2 * u) * P.Kh, W.gu + (size_t)(2 * u + 1) * P.Kh};
            float dot[2];
            rows_dot_unrolled<2, MAXC>(rows, xs4, nch_h, lane, dot);
            if (lane == 0) {
                const float g = dot[0] * W.gu_scale[2 * u];
                const float up = dot[1] * W.gu_scale[2 * u + 1];
                P.hbuf[u] = (g / (1.0f + expf(-g))) * up;
            }
        }
        if (!grid_sync(P.sync, (unsigned)G * ++nbar, &s_abort)) return;

        // ---- down + residual (src/model.cpp:309-310)
        prefetch_phase(P, A, 5 * l + 4 + P.prefetch_ahead);
        if (l + 1 < P.L) prefetch_kv<KV>(P, l + 1, 0);
        stage_vector(xs4, P.hbuf, P.I, nch_i, nullptr, 0.f, nullptr, nullptr, 0, P.Kh, nullptr, red);
        for (int u = gw; u < (P.H + 1) / 2; u += TW) {
            const int r0 = 2 * u, r1 = 2 * u + 1;
            const int8_t* rows[2] = {W.down + (size_t)r0 * P.Ki, r1 < P.H ? W.down + (size_t)r1 * P.Ki : nullptr};
            float dot[2];
            rows_dot_loop<2, 2>(rows, xs4, nch_i, lane, dot);
            if (lane == 0) {
                P.x[r0] = __ldcg(P.x + r0) + dot[0] * W.down_scale[r0];
                if (r1 < P.H) P.x[r1] = __ldcg(P.x + r1) + dot[1] * W.down_scale[r1];
            }
        }
        if (!grid_sync(P.sync, (unsigned)G * ++nbar, &s_abort)) return;
    }

    if (A.head) {
        // ---- final RMSNorm + tied LM head + argmax (src/model.cpp:318-326, src/main.cpp:35-37)
        stage_vector(xs4, P.x, P.H, nch_h, P.final_norm, P.eps, nullptr, nullptr, 0, P.Kh, nullptr, red);
        float best_v = -INFINITY;
        int best_i = 0x7fffffff;
        const int quads = (P.V + 3) / 4;
        // Keep L2 a few iterations ahead of this block's stream of rows: in
        // iteration k the block reads rows [4*(k*TW + blockIdx.x*NW), +4*NW).
        constexpr int HEAD_AHEAD = 3;
        auto prefetch_iter = [&](int k) {
            const long r = 4L * ((long)k * TW + (long)blockIdx.x * NW);
            if (r < P.V) prefetch_l2(P.embed + (size_t)r * P.Kh, (uint32_t)(min(4 * NW, P.V - (int)r) * P.Kh));
        };
        if (threadIdx.x == 0)
            for (int k = 0; k < HEAD_AHEAD; ++k) prefetch_iter(k);
        for (int u = gw, k = 0; u < quads; u += TW, ++k) {
            const int r0 = 4 * u;
            if (threadIdx.x == 0) prefetch_iter(k + HEAD_AHEAD);
            const int8_t* rows[4];
#pragma unroll
            for (int r = 0; r < 4; ++r) rows[r] = r0 + r < P.V ? P.embed + (size_t)(r0 + r) * P.Kh : nullptr;
            float dot[4];
            rows_dot_unrolled<4, MAXC>(rows, xs4, nch_h, lane, dot);
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                if (r0 + r < P.V) {
                    const float v = dot[r] * P.embed_scale[r0 + r];
                    if (lane == r) P.logits[r0 + r] = v;
                    if (better(v, r0 + r, best_v, best_i)) { best_v = v; best_i = r0 + r; }
                }
            }
        }
        if (lane == 0) s_best[warp] = {best_v, best_i};
        __syncthreads();
        if (threadIdx.x == 0) {
            ArgBest b = s_best[0];
            for (int w = 1; w < NW; ++w)
                if (better(s_best[w].v, s_best[w].i, b.v, b.i)) b = s_best[w];
            P.amax[blockIdx.x] = b;
            __threadfence();
            const unsigned prev = atomicAdd(&P.sync->amax_done, 1u);
            if (prev == (unsigned)G - 1) {
                __threadfence();
                ArgBest r = {-INFINITY, 0x7fffffff};
                for (int c = 0; c < G; ++c) {
                    ArgBest t;
                    t.v = __ldcg(&P.amax[c].v);
                    t.i = __ldcg(&P.amax[c].i);
                    if (better(t.v, t.i, r.v, r.i)) r = t;
                }
                if (r.i == 0x7fffffff) r.i = 0;
                P.result[0] = r.i;
                if (A.argmax_dev) *A.argmax_dev = r.i;
                P.sync->amax_done = 0;
            }
        }
    }

    // The last block out resets the barrier for the next launch.
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        const unsigned prev = atomicAdd(&P.sync->done, 1u);
        if (prev == (unsigned)G - 1) {
            P.sync->arrive = 0;
            P.sync->done = 0;
            __threadfence();
        }
    }
}

}  // namespace dcb

// ============================================================================
// Host engine
// ============================================================================
using namespace dcb;

namespace {
thread_local std::string g_last_error;
}  // namespace

void dcb::set_last_error(const std::string& msg) { g_last_error = msg; }

namespace {
int fail(int code, const std::string& msg) {
    g_last_error = msg;
    return code;
}
#define DCB_CUDA(call)                                                                              \
    do {                                                                                            \
        cudaError_t e_ = (call);                                                                    \
        if (e_ != cudaSuccess) return fail(DCB_ERR_CUDA, std::string(#call ": ") + cudaGetErrorString(e_)); \
    } while (0)

size_t round_up(size_t v, size_t m) { return (v + m - 1) / m * m; }
}  // namespace

struct dcb_engine {
    int device = 0;
    cudaStream_t stream = nullptr;
    bool own_stream = false;
    Params P{};
    int H, I, L, NH, NKV, D, V, Kh, Ki;
    int kv_dtype = DCB_KV_F32;
    size_t capacity = 0, pos = 0;
    std::vector<void*> allocations;
    LayerW* d_layers = nullptr;
    int grid = 0, smem = 0, sms = 0;
    void* kernel = nullptr;
    int* h_result = nullptr;  // pinned [2]
    uint64_t launches = 0;

    ~dcb_engine() {
        if (device >= 0) cudaSetDevice(device);
        if (stream) cudaStreamSynchronize(stream);
        for (void* p : allocations) cudaFree(p);
        if (h_result) cudaFreeHost(h_result);
        if (stream && own_stream) cudaStreamDestroy(stream);
    }
    template <class T>
    int alloc(T** out, size_t count) {
        void* p = nullptr;
        size_t bytes = round_up(std::max<size_t>(count * sizeof(T), 16), 256);
        cudaError_t e = cudaMalloc(&p, bytes);
        if (e != cudaSuccess) return fail(DCB_ERR_CUDA, std::string("cudaMalloc: ") + cudaGetErrorString(e));
        allocations.push_back(p);
        e = cudaMemset(p, 0, bytes);
        if (e != cudaSuccess) return fail(DCB_ERR_CUDA, std::string("cudaMemset: ") + cudaGetErrorString(e));
        *out = static_cast<T*>(p);
        return 0;
    }
};

namespace {

template <int MAXC>
void* pick_kernel(int kv_dtype) {
    return kv_dtype == DCB_KV_F16 ? (void*)decode_step_kernel<MAXC, __half> : (void*)decode_step_kernel<MAXC, float>;
}

// Upload a [rows][cols] int8 matrix into [rows][ld] (zero padded) at row order
// `order` (row i of the device matrix is source row order[i]).
int upload_rows(dcb_engine* e, int8_t** out, const std::vector<const int8_t*>& src_rows, int cols, int ld) {
    int8_t* d = nullptr;
    if (int rc = e->alloc(&d, src_rows.size() * (size_t)ld)) return rc;
    std::vector<int8_t> staging(src_rows.size() * (size_t)ld, 0);
    for (size_t i = 0; i < src_rows.size(); ++i) std::memcpy(&staging[i * ld], src_rows[i], cols);
    DCB_CUDA(cudaMemcpy(d, staging.data(), staging.size(), cudaMemcpyHostToDevice));
    *out = d;
    return 0;
}
int upload_floats(dcb_engine* e, float** out, const std::vector<float>& v) {
    float* d = nullptr;
    if (int rc = e->alloc(&d, v.size())) return rc;
    DCB_CUDA(cudaMemcpy(d, v.data(), v.size() * sizeof(float), cudaMemcpyHostToDevice));
    *out = d;
    return 0;
}

int validate(const dcb_model_desc* m) {
    if (!m || !m->layer || !m->embed || !m->embed_scales || !m->final_norm)
        return fail(DCB_ERR_ARGUMENT, "null model description");
    if (m->hidden <= 0 || m->intermediate <= 0 || m->layers <= 0 || m->heads <= 0 || m->kv_heads <= 0 ||
        m->head_dim <= 0 || m->vocab <= 0)
        return fail(DCB_ERR_ARGUMENT, "invalid Qwen dimensions or constants");
    if (m->hidden != m->heads * m->head_dim || m->heads % m->kv_heads || m->head_dim % 2)
        return fail(DCB_ERR_ARGUMENT, "invalid Qwen dimensions or constants");
    if (m->head_dim > 128) return fail(DCB_ERR_UNSUPPORTED, "head_dim above 128 is not supported");
    if (m->kv_heads > MAX_KV_HEADS) return fail(DCB_ERR_UNSUPPORTED, "more than 64 KV heads is not supported");
    if (!(m->epsilon > 0) || !std::isfinite(m->epsilon) || !(m->theta > 0) || !std::isfinite(m->theta))
        return fail(DCB_ERR_ARGUMENT, "invalid Qwen dimensions or constants");
    for (int l = 0; l < m->layers; ++l) {
        const dcb_layer_desc& L = m->layer[l];
        const void* ps[] = {L.q, L.k, L.v, L.o, L.gate, L.up, L.down, L.q_scales, L.k_scales, L.v_scales,
                            L.o_scales, L.gate_scales, L.up_scales, L.down_scales, L.input_norm, L.post_norm,
                            L.q_bias, L.k_bias, L.v_bias};
        for (const void* p : ps)
            if (!p) return fail(DCB_ERR_ARGUMENT, "null layer tensor");
    }
    return 0;
}

void choose_split(const dcb_engine* e, int length, int* nsplit, int* split_len) {
    const int chunks = (length + KV_CHUNK - 1) / KV_CHUNK;
    int want = std::max(1, e->grid / e->NKV);
    int n = std::min(chunks, want);
    int per = (chunks + n - 1) / n;  // chunks per split
    *split_len = per * KV_CHUNK;
    *nsplit = (length + *split_len - 1) / *split_len;
}

int launch(dcb_engine* e, int token, const int* token_dev, int head, int* argmax_dev) {
    StepArgs A{};
    A.token = token;
    A.token_dev = token_dev;
    A.pos = (int)e->pos;
    A.head = head;
    A.argmax_dev = argmax_dev;
    choose_split(e, (int)e->pos + 1, &A.nsplit, &A.split_len);
    void* args[] = {(void*)&e->P, (void*)&A};
    DCB_CUDA(cudaLaunchCooperativeKernel(e->kernel, dim3(e->grid), dim3(NT), args, (size_t)e->smem, e->stream));
    ++e->launches;
    return 0;
}

int device_error(dcb_engine* e, int err) {
    if (!err) return 0;
    DCB_CUDA(cudaMemset(e->P.sync, 0, sizeof(Sync)));
    if (err == ERR_TOKEN) return fail(DCB_ERR_TOKEN, "token ID outside vocabulary");
    return fail(DCB_ERR_DEVICE_WAIT, "a device-side wait ran out of time; the step was abandoned");
}

int check_device_error(dcb_engine* e) {
    int err = 0;
    DCB_CUDA(cudaMemcpy(&err, &e->P.sync->error, sizeof(int), cudaMemcpyDeviceToHost));
    return device_error(e, err);
}

}  // namespace

extern "C" {

const char* dcb_last_error(void) { return g_last_error.c_str(); }
void dcb_set_error(const char* message) { g_last_error = message ? message : ""; }

int dcb_create(const dcb_model_desc* m, size_t capacity, int kv_dtype, int cached_rope, int device,
               dcb_engine** out) {
    if (!out) return fail(DCB_ERR_ARGUMENT, "null output handle");
    *out = nullptr;
    if (int rc = validate(m)) return rc;
    if (!capacity || capacity > (size_t)0x7fffffff) return fail(DCB_ERR_ARGUMENT, "invalid thread count or context capacity");
    if (kv_dtype != DCB_KV_F32 && kv_dtype != DCB_KV_F16) return fail(DCB_ERR_ARGUMENT, "invalid KV dtype");
    DCB_CUDA(cudaSetDevice(device));
    auto* e = new dcb_engine();
    e->device = device;
    auto bail = [&](int rc) { delete e; return rc; };
    e->H = m->hidden; e->I = m->intermediate; e->L = m->layers; e->NH = m->heads; e->NKV = m->kv_heads;
    e->D = m->head_dim; e->V = m->vocab;
    e->Kh = (int)round_up(e->H, 16);
    e->Ki = (int)round_up(e->I, 16);
    e->kv_dtype = kv_dtype;
    e->capacity = capacity;
    const int H = e->H, I = e->I, D = e->D, half = D / 2, kvd = e->NKV * D;
    Params& P = e->P;
    P.H = H; P.I = I; P.L = e->L; P.NH = e->NH; P.NKV = e->NKV; P.D = D; P.V = e->V; P.Kh = e->Kh; P.Ki = e->Ki;
    P.qkv_rows = H + 2 * kvd;
    P.eps = m->epsilon;
    P.cached_rope = cached_rope ? 1 : 0;
    P.capacity = capacity;

    int dev_sms = 0;
    if (cudaDeviceGetAttribute(&dev_sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) return bail(fail(DCB_ERR_CUDA, "device query failed"));
    e->sms = dev_sms;

    // Weights, in the engine's layout.
    std::vector<LayerW> lw(e->L);
    for (int l = 0; l < e->L; ++l) {
        const dcb_layer_desc& S = m->layer[l];
        LayerW& W = lw[l];
        std::vector<const int8_t*> rows;
        std::vector<float> sc, bias;
        auto add_pairs = [&](const int8_t* w, const float* s, const float* b, int heads) {
            for (int h = 0; h < heads; ++h)
                for (int j = 0; j < half; ++j)
                    for (int r : {h * D + j, h * D + j + half}) {
                        rows.push_back(w + (size_t)r * H);
                        sc.push_back(s[r]);
                        bias.push_back(b[r]);
                    }
        };
        add_pairs(S.q, S.q_scales, S.q_bias, e->NH);
        add_pairs(S.k, S.k_scales, S.k_bias, e->NKV);
        add_pairs(S.v, S.v_scales, S.v_bias, e->NKV);
        int8_t* d8;
        float* df;
        if (int rc = upload_rows(e, &d8, rows, H, e->Kh)) return bail(rc);
        W.qkv = d8;
        if (int rc = upload_floats(e, &df, sc)) return bail(rc);
        W.qkv_scale = df;
        if (int rc = upload_floats(e, &df, bias)) return bail(rc);
        W.qkv_bias = df;

        rows.clear();
        for (int r = 0; r < H; ++r) rows.push_back(S.o + (size_t)r * H);
        if (int rc = upload_rows(e, &d8, rows, H, e->Kh)) return bail(rc);
        W.o = d8;
        if (int rc = upload_floats(e, &df, std::vector<float>(S.o_scales, S.o_scales + H))) return bail(rc);
        W.o_scale = df;

        rows.clear();
        sc.clear();
        for (int j = 0; j < I; ++j) {
            rows.push_back(S.gate + (size_t)j * H);
            rows.push_back(S.up + (size_t)j * H);
            sc.push_back(S.gate_scales[j]);
            sc.push_back(S.up_scales[j]);
        }
        if (int rc = upload_rows(e, &d8, rows, H, e->Kh)) return bail(rc);
        W.gu = d8;
        if (int rc = upload_floats(e, &df, sc)) return bail(rc);
        W.gu_scale = df;

        rows.clear();
        for (int r = 0; r < H; ++r) rows.push_back(S.down + (size_t)r * I);
        if (int rc = upload_rows(e, &d8, rows, I, e->Ki)) return bail(rc);
        W.down = d8;
        if (int rc = upload_floats(e, &df, std::vector<float>(S.down_scales, S.down_scales + H))) return bail(rc);
        W.down_scale = df;
        if (int rc = upload_floats(e, &df, std::vector<float>(S.input_norm, S.input_norm + H))) return bail(rc);
        W.in_norm = df;
        if (int rc = upload_floats(e, &df, std::vector<float>(S.post_norm, S.post_norm + H))) return bail(rc);
        W.post_norm = df;
    }
    if (int rc = e->alloc(&e->d_layers, lw.size())) return bail(rc);
    if (cudaMemcpy(e->d_layers, lw.data(), lw.size() * sizeof(LayerW), cudaMemcpyHostToDevice) != cudaSuccess)
        return bail(fail(DCB_ERR_CUDA, "layer table upload failed"));
    P.layers = e->d_layers;
    {
        std::vector<const int8_t*> rows;
        for (int r = 0; r < e->V; ++r) rows.push_back(m->embed + (size_t)r * H);
        int8_t* d8;
        float* df;
        if (int rc = upload_rows(e, &d8, rows, H, e->Kh)) return bail(rc);
        P.embed = d8;
        if (int rc = upload_floats(e, &df, std::vector<float>(m->embed_scales, m->embed_scales + e->V))) return bail(rc);
        P.embed_scale = df;
        if (int rc = upload_floats(e, &df, std::vector<float>(m->final_norm, m->final_norm + H))) return bail(rc);
        P.final_norm = df;
        // RoPE tables with the reference's float expressions (src/model.cpp:223-224, src/kernels.cpp:140).
        std::vector<float> inv(half), den(half);
        for (int j = 0; j < half; ++j) {
            den[j] = std::pow(m->theta, float(2 * j) / float(D));
            inv[j] = 1.0f / std::pow(m->theta, float(2 * j) / float(D));
        }
        if (int rc = upload_floats(e, &df, inv)) return bail(rc);
        P.rope_inv = df;
        if (int rc = upload_floats(e, &df, den)) return bail(rc);
        P.rope_den = df;
    }
    const size_t esz = kv_dtype == DCB_KV_F16 ? 2 : 4;
    {
        unsigned char* kc;
        unsigned char* vc;
        const size_t bytes = (size_t)e->L * capacity * kvd * esz;
        if (int rc = e->alloc(&kc, bytes)) return bail(rc);
        if (int rc = e->alloc(&vc, bytes)) return bail(rc);
        P.kcache = kc;
        P.vcache = vc;
    }

    // Launch shape: one 512-thread block per SM, all co-resident.
    const int maxc = (e->Kh / 16 + 31) / 32;
    if (maxc <= 1) e->kernel = pick_kernel<1>(kv_dtype);
    else if (maxc <= 2) e->kernel = pick_kernel<2>(kv_dtype);
    else if (maxc <= 4) e->kernel = pick_kernel<4>(kv_dtype);
    else return bail(fail(DCB_ERR_UNSUPPORTED, "hidden size above 2048 is not supported"));
    P.xs_floats = (int)round_up(std::max(e->Kh, e->Ki), 16);
    const int gq = e->NH / e->NKV;
    e->smem = (P.xs_floats + attention_smem_floats(D, gq)) * (int)sizeof(float);
    if (cudaFuncSetAttribute(e->kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, e->smem) != cudaSuccess)
        return bail(fail(DCB_ERR_UNSUPPORTED, "model too large for shared memory staging"));
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, e->kernel, NT, e->smem) != cudaSuccess || per_sm < 1)
        return bail(fail(DCB_ERR_UNSUPPORTED, "step kernel cannot be resident"));
    e->grid = dev_sms;

    float* f;
    if (int rc = e->alloc(&f, e->Kh)) return bail(rc);
    P.x = f;
    if (int rc = e->alloc(&f, e->Kh)) return bail(rc);
    P.q = f;
    if (int rc = e->alloc(&f, e->Kh)) return bail(rc);
    P.attn = f;
    if (int rc = e->alloc(&f, e->Ki)) return bail(rc);
    P.hbuf = f;
    if (int rc = e->alloc(&f, e->V)) return bail(rc);
    P.logits = f;
    if (int rc = e->alloc(&f, (size_t)e->NH * (e->grid + 1) * (D + 2))) return bail(rc);
    P.part = f;
    ArgBest* ab;
    if (int rc = e->alloc(&ab, e->grid)) return bail(rc);
    P.amax = ab;
    Sync* s;
    if (int rc = e->alloc(&s, 1)) return bail(rc);
    P.sync = s;
    int* res;
    if (int rc = e->alloc(&res, 4)) return bail(rc);
    P.result = res;
    P.prefetch_ahead = 2;
    P.head_prefetch_rows = 16384;
    if (cudaMallocHost(&e->h_result, 4 * sizeof(int)) != cudaSuccess) return bail(fail(DCB_ERR_CUDA, "cudaMallocHost failed"));
    if (cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking) != cudaSuccess)
        return bail(fail(DCB_ERR_CUDA, "stream creation failed"));
    e->own_stream = true;
    if (cudaDeviceSynchronize() != cudaSuccess) return bail(fail(DCB_ERR_CUDA, "device synchronize failed"));
    *out = e;
    return 0;
}

void dcb_destroy(dcb_engine* e) { delete e; }

int dcb_step(dcb_engine* e, int token, int head, float* host_logits, int* argmax_out) {
    if (!e) return fail(DCB_ERR_ARGUMENT, "null engine");
    if (token < 0 || token >= e->V) return fail(DCB_ERR_TOKEN, "token ID outside vocabulary");
    if (e->pos >= e->capacity) return fail(DCB_ERR_CAPACITY, "context capacity exceeded");
    DCB_CUDA(cudaSetDevice(e->device));
    if (int rc = launch(e, token, nullptr, head, nullptr)) return rc;
    if (head && host_logits)
        DCB_CUDA(cudaMemcpyAsync(host_logits, e->P.logits, (size_t)e->V * sizeof(float), cudaMemcpyDeviceToHost, e->stream));
    DCB_CUDA(cudaMemcpyAsync(e->h_result, e->P.result, sizeof(int), cudaMemcpyDeviceToHost, e->stream));
    DCB_CUDA(cudaMemcpyAsync(e->h_result + 1, &e->P.sync->error, sizeof(int), cudaMemcpyDeviceToHost, e->stream));
    DCB_CUDA(cudaStreamSynchronize(e->stream));
    if (int rc = device_error(e, e->h_result[1])) return rc;
    if (head && argmax_out) *argmax_out = e->h_result[0];
    ++e->pos;
    return 0;
}

int dcb_step_async(dcb_engine* e, int token, const int* token_dev, int head, int* argmax_dev) {
    if (!e) return fail(DCB_ERR_ARGUMENT, "null engine");
    if (!token_dev && (token < 0 || token >= e->V)) return fail(DCB_ERR_TOKEN, "token ID outside vocabulary");
    if (e->pos >= e->capacity) return fail(DCB_ERR_CAPACITY, "context capacity exceeded");
    DCB_CUDA(cudaSetDevice(e->device));
    if (int rc = launch(e, token, token_dev, head, argmax_dev)) return rc;
    ++e->pos;
    return 0;
}

int dcb_synchronize(dcb_engine* e) {
    if (!e) return fail(DCB_ERR_ARGUMENT, "null engine");
    DCB_CUDA(cudaSetDevice(e->device));
    DCB_CUDA(cudaStreamSynchronize(e->stream));
    return check_device_error(e);
}

int dcb_rewind(dcb_engine* e, size_t position) {
    if (!e) return fail(DCB_ERR_ARGUMENT, "null engine");
    if (position > e->pos) return fail(DCB_ERR_REWIND, "cannot rewind forward");
    e->pos = position;
    return 0;
}
int dcb_reset(dcb_engine* e) {
    if (!e) return fail(DCB_ERR_ARGUMENT, "null engine");
    e->pos = 0;
    return 0;
}
size_t dcb_position(const dcb_engine* e) { return e ? e->pos : 0; }

int dcb_set_position(dcb_engine* e, size_t position) {
    if (!e) return fail(DCB_ERR_ARGUMENT, "null engine");
    if (position > e->capacity) return fail(DCB_ERR_CAPACITY, "context capacity exceeded");
    e->pos = position;
    return 0;
}

int dcb_set_stream(dcb_engine* e, void* stream) {
    if (!e) return fail(DCB_ERR_ARGUMENT, "null engine");
    DCB_CUDA(cudaSetDevice(e->device));
    DCB_CUDA(cudaStreamSynchronize(e->stream));
    if (e->own_stream) cudaStreamDestroy(e->stream);
    if (stream) {
        e->stream = static_cast<cudaStream_t>(stream);
        e->own_stream = false;
    } else {
        DCB_CUDA(cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking));
        e->own_stream = true;
    }
    return 0;
}
void* dcb_stream(const dcb_engine* e) { return e ? (void*)e->stream : nullptr; }
const float* dcb_logits_device(const dcb_engine* e) { return e ? e->P.logits : nullptr; }

int dcb_kv_write(dcb_engine* e, int layer, size_t start, size_t count, const float* keys, const float* values) {
    if (!e || !keys || !values) return fail(DCB_ERR_ARGUMENT, "null argument");
    if (layer < 0 || layer >= e->L || start + count > e->capacity) return fail(DCB_ERR_ARGUMENT, "KV rows out of range");
    DCB_CUDA(cudaSetDevice(e->device));
    const size_t kvd = (size_t)e->NKV * e->D, n = count * kvd;
    const size_t off = ((size_t)layer * e->capacity + start) * kvd;
    if (e->kv_dtype == DCB_KV_F32) {
        DCB_CUDA(cudaMemcpy(static_cast<float*>(e->P.kcache) + off, keys, n * 4, cudaMemcpyHostToDevice));
        DCB_CUDA(cudaMemcpy(static_cast<float*>(e->P.vcache) + off, values, n * 4, cudaMemcpyHostToDevice));
    } else {
        std::vector<__half> hk(n), hv(n);
        for (size_t i = 0; i < n; ++i) {
            hk[i] = __float2half_rn(keys[i]);
            hv[i] = __float2half_rn(values[i]);
        }
        DCB_CUDA(cudaMemcpy(static_cast<__half*>(e->P.kcache) + off, hk.data(), n * 2, cudaMemcpyHostToDevice));
        DCB_CUDA(cudaMemcpy(static_cast<__half*>(e->P.vcache) + off, hv.data(), n * 2, cudaMemcpyHostToDevice));
    }
    return 0;
}

int dcb_kv_read(const dcb_engine* e, int layer, size_t start, size_t count, float* keys, float* values) {
    if (!e || !keys || !values) return fail(DCB_ERR_ARGUMENT, "null argument");
    if (layer < 0 || layer >= e->L || start + count > e->capacity) return fail(DCB_ERR_ARGUMENT, "KV rows out of range");
    DCB_CUDA(cudaSetDevice(e->device));
    DCB_CUDA(cudaStreamSynchronize(e->stream));
    const size_t kvd = (size_t)e->NKV * e->D, n = count * kvd;
    const size_t off = ((size_t)layer * e->capacity + start) * kvd;
    if (e->kv_dtype == DCB_KV_F32) {
        DCB_CUDA(cudaMemcpy(keys, static_cast<const float*>(e->P.kcache) + off, n * 4, cudaMemcpyDeviceToHost));
        DCB_CUDA(cudaMemcpy(values, static_cast<const float*>(e->P.vcache) + off, n * 4, cudaMemcpyDeviceToHost));
    } else {
        std::vector<__half> hk(n), hv(n);
        DCB_CUDA(cudaMemcpy(hk.data(), static_cast<const __half*>(e->P.kcache) + off, n * 2, cudaMemcpyDeviceToHost));
        DCB_CUDA(cudaMemcpy(hv.data(), static_cast<const __half*>(e->P.vcache) + off, n * 2, cudaMemcpyDeviceToHost));
        for (size_t i = 0; i < n; ++i) {
            keys[i] = __half2float(hk[i]);
            values[i] = __half2float(hv[i]);
        }
    }
    return 0;
}

int dcb_launch_info(const dcb_engine* e, int* blocks, int* threads, int* smem_bytes, int* sms) {
    if (!e) return fail(DCB_ERR_ARGUMENT, "null engine");
    if (blocks) *blocks = e->grid;
    if (threads) *threads = NT;
    if (smem_bytes) *smem_bytes = e->smem;
    if (sms) *sms = e->sms;
    return 0;
}

uint64_t dcb_launch_count(const dcb_engine* e) { return e ? e->launches : 0; }

}  // extern "C"
