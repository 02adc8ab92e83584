// The decode step as one persistent cooperative kernel (one block per SM).
//
// One launch runs the reference's Engine::Impl::step (src/model.cpp:258-329)
// for one token: embedding, then per layer
//   QKV  : RMSNorm prologue, Q/K/V int8 GEMV + bias + split-half RoPE, K/V row
//          written to the cache at `pos`
//   ATTN : GQA attention over positions 0..pos (one block per query head and
//          KV split; split 0 merges the splits' (max, sum, output))
//   O    : split-K over the heads: the block that finishes head h's attention
//          multiplies it by W_o's columns of head h and adds the products into
//          exact fixed-point sums; the gate/up phase reads x_a + sums
//   GU   : RMSNorm prologue, gate/up GEMV, SiLU(gate)*up
//   DOWN : split-K over the blocks: each block multiplies its own SiLU(gate)*up
//          values by its columns of W_down and adds the products into exact
//          fixed-point sums; the next layer reads x_b + sums
// then the final RMSNorm, the tied LM head and the argmax.
//
// Data movement, B200-first:
//  * Weights never wait on activations. Each block owns fixed row ranges of
//    every projection; its rows (int8 + FP32 scale + bias, packed per row) are
//    brought into shared memory by TMA bulk copies (cp.async.bulk + mbarrier)
//    one layer ahead, so a GEMV phase only waits for its input vector.
//  * No grid barriers. Activations travel between blocks as 64-bit words
//    {value, tag}: a producer stores each element once with its tag, consumers
//    poll exactly the elements they need until the tag of this step and layer
//    shows. One L2 round trip per dependency; a stale value is never used.
//    The O and down projections' outputs are sums over blocks instead:
//    64-bit integer reductions into L2 words that count their own additions.
//  * The LM head (136 MB at the Qwen shape) streams straight from HBM: every
//    warp keeps the 16-byte chunks of its next row group in flight while it
//    reduces the current one.
// Every wait is bounded in time; on expiry the block records an error, drains
// its own copies in flight and returns.
#pragma once
#include "device.cuh"

#include <cuda_fp16.h>
#include <cstdint>

namespace dcb {

constexpr int NT = 512;
constexpr int NW = NT / 32;
constexpr uint64_t WAIT_LIMIT_NS = 1000000000ull;  // one second
constexpr int ERR_WAIT = 1;
constexpr int ERR_TOKEN = 2;
constexpr int ATT_CHUNK = 64;  // KV positions per staged chunk
constexpr int ATT_PER_WARP = ATT_CHUNK / NW;
constexpr int ATT_MAX_BUFS = 6;  // staged chunk ring (the host picks how many fit)
constexpr int MAX_WORLD = 8;     // GPUs that split one stream's KV sequence
constexpr int HEAD_R = 4;           // LM-head rows a warp reduces per group (the next group in flight)
constexpr int HEAD_L2_ROWS = 256;   // LM-head rows per block prefetched into L2 during the last layer
constexpr int HEAD_MAXC = 2;        // 16-byte chunks per lane of a hidden-size row (hidden <= 1024)
constexpr int TRACE_MAX_PHASES = 512;
constexpr int DOWN_RPT = 2;    // down output rows per thread (H <= DOWN_RPT * NT)
constexpr int MAXD = 4;        // head_dim <= 128: lane owns dims lane + 32k
constexpr int GQA_MAX = 8;     // query heads per KV group of a group attention unit, at most
constexpr int GQA_PASS = 3;    // resident chunks a group attention unit takes per pass, at most
constexpr int GQA_MERGE_MAX = 160;  // splits a group unit's merge weighs (misc holds the weights)

// Per-layer weights, packed rows: [K int8 | FP32 scale | FP32 bias | 8 pad].
struct LayerW {
    const uint8_t* qkv;   // 2*qkv_pairs rows (RoPE pairs (j, j+d/2) adjacent), stride SH
    const uint8_t* o;     // H rows, stride SH
    const uint8_t* gu;    // 2I rows (gate_j, up_j adjacent), stride SH
    const uint8_t* down;  // H rows, stride SI
};

struct Sync {
    unsigned amax_done;
    int error;   // first error of the step (ERR_*), 0 if none
    int result;  // argmax of the logits; follows `error` so one 8-byte copy reads both
};

struct ArgBest {
    float v;
    int i;
};

struct Params {
    int H, I, L, NH, NKV, D, V, Kh, Ki, SH, SI, qkv_pairs;
    float eps;
    int cached_rope;
    int capacity;
    // KV-sequence split over GPUs: this engine keeps positions [kv_base, kv_end)
    // (local cache row t - kv_base) and attends over them; rank `rank` of
    // `world` engines exchanges per-head partials through exch (its own
    // buffer, [2][NH][world][D+2] tagged words) and peers[q] (rank q's buffer).
    int kv_base, kv_end, world, rank;
    uint64_t* exch;
    uint64_t* const* peers;
    const LayerW* layers;
    const uint8_t* embed;   // V packed rows, stride SH (the tied LM head)
    const float* norms;     // [L+1][2][Kh]: (input, post-attention) RMSNorm gains per layer, then (final, 0)
    const float* rope_inv;  // [D/2] 1/theta^(2j/D)  (cached angle formula)
    const float* rope_den;  // [D/2] theta^(2j/D)    (direct angle formula)
    void* kcache;           // [L][NKV][capacity][D], head-major
    void* vcache;
    uint64_t* ll_q;     // [H]   rotated queries
    uint64_t* ll_kv;    // [2*NKV*D] the new K and V rows
    uint64_t* ll_part;    // [NH][nsplit][D+2] tagged attention split partials (m, l, o)
    float* logits;        // [V]
    ArgBest* amax;        // [grid]
    Sync* sync;
    uint64_t* trace;  // [2][TRACE_MAX_PHASES][grid] ready/done ns, or null
    // shared memory layout (bytes)
    int off_gu, off_down, off_qkv, off_att, off_xs, off_xq, off_gpart, off_xr, off_misc;
    int xq_plane;      // bytes per fixed-point plane of a hidden-sized vector (>= Kh)
    int gpart_floats;  // floats per block-GEMV partial buffer (NW * max rows of a phase)
    int att_chunk_bytes;
    int att_bufs;     // chunk buffers in the attention ring (2..ATT_MAX_BUFS)
    int trace_layer;  // layer whose phases get detailed marks when tracing
    // Down projection as split-K over the blocks: block b holds columns
    // [b*I/G, (b+1)*I/G) of W_down for all H rows, DW int8 per row (zero
    // padded), one down_slice-byte region per block and layer. Its products
    // with the block's own SiLU(gate)*up values are added, scaled per row, into
    // the self-counting sum words of the layer.
    const uint8_t* down_cols;  // [L][G][down_slice]
    const float* down_scale;   // [L][H] per-row scales of W_down
    // O projection as split-K over the heads: W_o's columns of head h for all
    // H rows, o_dw int8 per row (zero past D), o_slice bytes per (layer, head),
    // copied into the end of the attention buffers (offset wo_off) of the
    // block that finishes head h (split 0).
    const uint8_t* o_cols;     // [L][NH][o_slice]
    const float* o_scale;      // [L][H] per-row scales of W_o
    // Sum words [2 halves][L][2: O, down][Hp].
    uint64_t* dacc;
    int down_dw, down_slice, Hp, off_h, o_dw, o_slice, wo_off;
    int gqa_pass;  // resident chunks a group attention unit takes per pass (<= GQA_PASS, < att_bufs when possible)
};

struct StepArgs {
    int token;
    const int* token_dev;
    int pos;
    int head;
    int* argmax_dev;
    int nsplit;
    int split_len;
    unsigned seq;
    float* host_logits;  // mapped pinned host memory the LM head also writes, or null
    int par;             // which half of dacc this step sums into (the other half is cleared for the next)
    int group;           // attention units are (KV group, split) instead of (query head, split)
    int head_follows;    // (two-role kernel) an LM-head kernel follows this launch: warm L2 with its rows
};

__device__ __forceinline__ bool better(float v, int i, float bv, int bi) { return v > bv || (v == bv && i < bi); }

__device__ __forceinline__ int part_lo(int b, int G, int n) { return (int)((long long)b * n / G); }

// The grid's argmax once every block has a candidate (its best value and
// first index): each block stores its own into amax[block]; the last block to
// count itself in sync->amax_done merges all of them with every thread (one
// load pair each, warp shuffles, one shared-memory step; the first index wins
// ties, as std::max_element), publishes the result and re-arms the counter.
// The merge is block-parallel: one thread walking the candidates would pay an
// L2 round trip per candidate. scratch: T/32 entries; flag: one shared int.
// Every thread of the block calls it.
template <int T>
__device__ void grid_argmax(ArgBest best, ArgBest* amax, Sync* sync, int* argmax_dev, ArgBest* scratch, int* flag) {
    const int tid = threadIdx.x, G = gridDim.x, lane = tid & 31;
    if (tid == 0) {
        amax[blockIdx.x] = best;
        __threadfence();
        *flag = atomicAdd(&sync->amax_done, 1u) == (unsigned)G - 1;
    }
    __syncthreads();
    if (!*flag) return;
    __threadfence();
    ArgBest r = {-INFINITY, 0x7fffffff};
    for (int k = tid; k < G; k += T) {
        ArgBest t;
        t.v = __ldcg(&amax[k].v);
        t.i = __ldcg(&amax[k].i);
        if (better(t.v, t.i, r.v, r.i)) r = t;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        ArgBest t;
        t.v = __shfl_xor_sync(FULL, r.v, o);
        t.i = __shfl_xor_sync(FULL, r.i, o);
        if (better(t.v, t.i, r.v, r.i)) r = t;
    }
    if (lane == 0) scratch[tid >> 5] = r;
    __syncthreads();
    if (tid == 0) {
        for (int w = 0; w < T / 32; ++w)
            if (better(scratch[w].v, scratch[w].i, r.v, r.i)) r = scratch[w];
        if (r.i == 0x7fffffff) r.i = 0;
        sync->result = r.i;
        if (argmax_dev) *argmax_dev = r.i;
        sync->amax_done = 0;
    }
}

// ---- mbarrier + bulk copy ------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t* m, unsigned count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(m)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* m) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(m)) : "memory");
}
__device__ __forceinline__ void mbar_expect(uint64_t* m, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(m)), "r"(bytes) : "memory");
}
// Phase `parity` of m complete? test_wait answers at once (a completed phase
// costs about a shared-memory load); try_wait may first suspend the thread
// for a while, which suits a phase that is still running.
__device__ __forceinline__ bool mbar_test(uint64_t* m, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{ .reg .pred p; mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
        : "=r"(ok)
        : "r"(smem_u32(m)), "r"(parity)
        : "memory");
    if (ok) return true;
    asm volatile(
        "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
        : "=r"(ok)
        : "r"(smem_u32(m)), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* m) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(m))
                 : "memory");
}
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// One thread: fill a shared slot with `bytes` (16-byte aligned, multiple of 16).
// `*fills` counts the fills issued on `m` (used to drain them on abort).
__device__ __forceinline__ void fill_slot(void* dst, const void* src, uint32_t bytes, uint64_t* m, unsigned* fills) {
    ++*fills;
    mbar_expect(m, bytes);
    constexpr uint32_t piece = 32768;
#pragma unroll 1
    for (uint32_t o = 0; o < bytes; o += piece) {
        const uint32_t n = bytes - o < piece ? bytes - o : piece;
        bulk_load(static_cast<char*>(dst) + o, static_cast<const char*>(src) + o, n, m);
    }
}

// ---- tagged activation words -----------------------------------------------------
__device__ __forceinline__ void ll_store(uint64_t* p, float v, uint32_t tag) {
    const uint64_t w = ((uint64_t)tag << 32) | (uint64_t)__float_as_uint(v);
    asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ uint64_t ll_load(const uint64_t* p) {
    uint64_t w;
    asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    return w;
}

// Tagged words another GPU reads or writes (NVLink peer memory): system scope.
__device__ __forceinline__ void ll_store_sys(uint64_t* p, float v, uint32_t tag) {
    const uint64_t w = ((uint64_t)tag << 32) | (uint64_t)__float_as_uint(v);
    asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ uint64_t ll_load_sys(const uint64_t* p) {
    uint64_t w;
    asm volatile("ld.relaxed.sys.global.b64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    return w;
}

struct BlockState {
    int* abort;  // shared flag
    Sync* sync;
};

__device__ __forceinline__ bool should_abort(const BlockState& st) {
    return *reinterpret_cast<volatile int*>(st.abort) != 0;
}
__device__ __forceinline__ void raise_abort(const BlockState& st, int code) {
    atomicCAS(&st.sync->error, 0, code);
    *reinterpret_cast<volatile int*>(st.abort) = 1;
}
// Periodic check inside a wait loop: true when the wait must end.
__device__ __forceinline__ bool wait_expired(const BlockState& st, uint64_t& t0) {
    if (should_abort(st) || ld_volatile(&st.sync->error)) {
        *reinterpret_cast<volatile int*>(st.abort) = 1;
        return true;
    }
    const uint64_t now = globaltimer();
    if (!t0) {
        t0 = now;
    } else if (now - t0 > WAIT_LIMIT_NS) {
        raise_abort(st, ERR_WAIT);
        return true;
    }
    return false;
}

// Block-wide wait until mbarrier `m` completes phase `parity`. Bounded.
// Thread 0 alone tests the barrier (512 threads testing one shared word
// serialise on it); the closing __syncthreads orders the completed copies
// before every thread's reads and lets all threads take the same decision.
static __device__ bool mbar_wait(uint64_t* m, uint32_t parity, const BlockState& st) {
    if (threadIdx.x == 0) {
        uint64_t t0 = 0;
        unsigned spins = 0;
        while (!mbar_test(m, parity))
            if ((++spins & 63u) == 0 && wait_expired(st, t0)) break;
    }
    __syncthreads();
    return !should_abort(st);
}

// ---- staged activation vectors and the block GEMV ----------------------------------
// A GEMV input is staged once per phase as 24-bit fixed point: with
// scale = max|v| / 8323072, q_j = rint(v_j / scale) = hi*2^16 + mid*2^8 + lo
// with hi, mid, lo signed bytes, kept as three byte planes (16*nch bytes each),
// so that 4 int8 weights times 4 activations are three exact dp4a operations
// (6 issue cycles per 4 weights on sm_100 against about 17 for widening each
// byte to FP32). The quantisation error is below 2^-23 * max|v| per element,
// the order of the FP32 rounding in the reference's own sums.

// Element j arrived with value v: raw to xr (when set), v * gain (the RMSNorm
// gain of element j folded in; 1 where there is none) to xf.
__device__ __forceinline__ void accept(int j, float v, float* xr, float* xf, float gain, float& ss, float& mx) {
    if (xr) xr[j] = v;
    const float g = v * gain;
    xf[j] = g;
    ss = fmaf(v, v, ss);
    mx = fmaxf(mx, fabsf(g));
}

struct Staged {
    float scale;  // value of one unit of q
    float inv;    // RMSNorm factor 1/sqrt(mean(v^2) + eps) of the raw values (src/kernels.cpp:132-137)
};

// All elements accepted: reduce (sum v^2, max |v*gain|) and quantise xf into
// the planes (padding n..16*nch as zeros). Two barriers.
static __device__ Staged finish_stage(int n, int nch, const float* xf, int8_t* xq, int plane, float ss, float mx, float* red,
                               float eps) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        ss += __shfl_xor_sync(FULL, ss, o);
        mx = fmaxf(mx, __shfl_xor_sync(FULL, mx, o));
    }
    if ((threadIdx.x & 31) == 0) {
        red[threadIdx.x >> 5] = ss;
        red[NW + (threadIdx.x >> 5)] = mx;
    }
    __syncthreads();
    float t = 0.f, m = 0.f;
#pragma unroll
    for (int w = 0; w < NW; w += 4) {
        const float4 a = *reinterpret_cast<const float4*>(red + w);
        const float4 b = *reinterpret_cast<const float4*>(red + NW + w);
        t += (a.x + a.y) + (a.z + a.w);
        m = fmaxf(fmaxf(m, fmaxf(b.x, b.y)), fmaxf(b.z, b.w));
    }
    Staged out;
    out.inv = __frsqrt_rn(t / (float)n + eps);
    const float rs = m > 0.f ? FIX_MAX * __frcp_rn(m) : 0.f;
    out.scale = m > 0.f ? __frcp_rn(rs) : 1.0f;
    for (int quad = threadIdx.x; quad < nch * 4; quad += NT) {
        uint32_t ph = 0, pm = 0, pl = 0;
        const float4 v4 = 4 * quad + 3 < n ? *reinterpret_cast<const float4*>(xf + 4 * quad)
                                           : make_float4(4 * quad < n ? xf[4 * quad] : 0.f,
                                                         4 * quad + 1 < n ? xf[4 * quad + 1] : 0.f,
                                                         4 * quad + 2 < n ? xf[4 * quad + 2] : 0.f, 0.f);
        fix_pack4(v4, rs, ph, pm, pl);
        reinterpret_cast<uint32_t*>(xq)[quad] = ph;
        reinterpret_cast<uint32_t*>(xq + plane)[quad] = pm;
        reinterpret_cast<uint32_t*>(xq + 2 * plane)[quad] = pl;
    }
    __syncthreads();
    return out;
}

// ---- per-warp staging of a GEMV input ---------------------------------------------
// Warp w owns K-chunks [w*nch/NW, (w+1)*nch/NW) of the input (16 elements
// each), the same chunks block_gemv gives it. warp_stage waits for exactly
// those elements (tagged words, or int8 row values times row_sc when `row` is
// set), keeps the raw values in xr (when set), folds in the RMSNorm gain and
// quantises them into the planes with the warp's own scale max|v|/FIX_MAX
// (returned in wscale). Its share of sum v^2 goes to ss_out[warp] (when set).
// No block barrier: every warp starts its share of the GEMV as soon as its own
// inputs are in. Returns false when the wait ran out (the abort flag is set).
template <int W, bool GAIN>
__device__ bool warp_stage(const uint64_t* src, const uint8_t* row, float row_sc, int n, uint32_t tag, float* xr,
                           float* xf, int8_t* xq, int plane, int nch, const float* gain, float* ss_out, float& wscale,
                           const BlockState& st) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int c0 = warp * nch / NW, c1 = (warp + 1) * nch / NW;
    const int e0 = 16 * c0, e1 = min(16 * c1, n);
    bool okw = true;
    float ss = 0.f, mx = 0.f;
    uint64_t t0 = 0;
    unsigned rounds = 0;
    for (int base = e0; base < e1; base += 32 * W) {
        float v[W], g[W];
        uint64_t w[W];
        unsigned pending = 0;
#pragma unroll
        for (int k = 0; k < W; ++k) {
            const int j = base + lane + 32 * k;
            v[k] = 0.f;
            g[k] = 1.f;
            if (j < e1) {
                if (GAIN) g[k] = __ldg(gain + j);
                if (row) {
                    v[k] = (float)(int8_t)row[j] * row_sc;
                } else {
                    w[k] = ll_load(src + j);
                    pending |= 1u << k;
                }
            }
        }
        while (pending) {
#pragma unroll
            for (int k = 0; k < W; ++k)
                if (((pending >> k) & 1u) && (uint32_t)(w[k] >> 32) == tag) {
                    v[k] = __uint_as_float((uint32_t)w[k]);
                    pending &= ~(1u << k);
                }
            if (!pending) break;
            if ((++rounds & 7u) == 0 && wait_expired(st, t0)) {
                okw = false;
                break;
            }
#pragma unroll
            for (int k = 0; k < W; ++k)
                if ((pending >> k) & 1u) w[k] = ll_load(src + base + lane + 32 * k);
        }
#pragma unroll
        for (int k = 0; k < W; ++k) {
            const int j = base + lane + 32 * k;
            if (j < e1) {
                if (xr) xr[j] = v[k];
                const float gv = v[k] * g[k];
                xf[j] = gv;
                ss = fmaf(v[k], v[k], ss);
                mx = fmaxf(mx, fabsf(gv));
            }
        }
        if (!okw) break;
    }
    // Lanes with nothing left to wait for leave the loop with okw true while
    // others time out; the callers' warp-wide steps (warp_slot_wait, the GEMV's
    // shuffles) need one decision per warp, or half a warp waits forever in a
    // __syncwarp that the other half never reaches.
    okw = __all_sync(FULL, okw);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        ss += __shfl_xor_sync(FULL, ss, o);
        mx = fmaxf(mx, __shfl_xor_sync(FULL, mx, o));
    }
    if (ss_out && lane == 0) ss_out[warp] = ss;
    const float rs = mx > 0.f ? FIX_MAX * __frcp_rn(mx) : 0.f;
    wscale = mx > 0.f ? __frcp_rn(rs) : 1.0f;
    __syncwarp();
    for (int quad = 4 * c0 + lane; quad < 4 * c1; quad += 32) {
        const int j = 4 * quad;
        const float4 v4 = j + 3 < n ? *reinterpret_cast<const float4*>(xf + j)
                                    : make_float4(j < n ? xf[j] : 0.f, j + 1 < n ? xf[j + 1] : 0.f,
                                                  j + 2 < n ? xf[j + 2] : 0.f, 0.f);
        uint32_t ph, pm, pl;
        fix_pack4(v4, rs, ph, pm, pl);
        reinterpret_cast<uint32_t*>(xq)[quad] = ph;
        reinterpret_cast<uint32_t*>(xq + plane)[quad] = pm;
        reinterpret_cast<uint32_t*>(xq + 2 * plane)[quad] = pl;
    }
    __syncwarp();
    return okw;
}

// One warp waits for phase `parity` of mbarrier m: lane 0 tests, then the
// warp synchronises (ordering the completed copies before every lane's reads).
// Bounded; false when the wait ran out (the abort flag is set).
static __device__ bool warp_slot_wait(uint64_t* m, uint32_t parity, const BlockState& st) {
    bool okw = true;
    if ((threadIdx.x & 31) == 0) {
        uint64_t t0 = 0;
        unsigned spins = 0;
        while (!mbar_test(m, parity))
            if ((++spins & 63u) == 0 && wait_expired(st, t0)) {
                okw = false;
                break;
            }
    }
    __syncwarp();
    return __shfl_sync(FULL, okw, 0);
}

// ---- split-K down projection: self-counting fixed-point sums over blocks ------------
// Each output row of the down projection is one 64-bit word in L2 that every
// block adds its share v into with one fire-and-forget reduction:
//   2^56 + (rint(v * 2^26) + 2^47)      (|v| < 2^21 = 2097152, clamped)
// The top 8 bits count the blocks added so far; the low 56 bits hold the sum
// in offset fixed point (no carry reaches the count for up to 255 blocks).
// Integer addition is exact, so the total does not depend on the order in
// which the additions reach L2 (every run, and every GPU of a KV split, gets
// the same bits), and a reader knows the word is complete when its count
// equals the number of blocks: no fence, no flag.
constexpr int DACC_CNT_SHIFT = 56;
constexpr double DACC_ONE = 67108864.0;  // 2^26: one unit of the sum
constexpr long long DACC_BIAS = 1LL << 47;
constexpr uint64_t DACC_LOW = (1ull << DACC_CNT_SHIFT) - 1;

__device__ __forceinline__ void dacc_add(uint64_t* p, float v) {
    // v * 2^26 is exact in FP32 (a power-of-two scaling), so rounding it to
    // an integer here equals rounding the double product.
    long long q = __float2ll_rn(v * (float)DACC_ONE);
    q = q > DACC_BIAS - 1 ? DACC_BIAS - 1 : (q < 1 - DACC_BIAS ? 1 - DACC_BIAS : q);
    const uint64_t c = (1ull << DACC_CNT_SHIFT) + (uint64_t)(q + DACC_BIAS);
    asm volatile("red.relaxed.gpu.global.add.u64 [%0], %1;" ::"l"(p), "l"(c) : "memory");
}
__device__ __forceinline__ unsigned dacc_count(uint64_t w) { return (unsigned)(w >> DACC_CNT_SHIFT); }
__device__ __forceinline__ float dacc_value(uint64_t w) {
    const long long q = (long long)(w & DACC_LOW) - (long long)dacc_count(w) * DACC_BIAS;
    // One rounding of q (|q| < 2^53 here) to FP32, then an exact power-of-two scaling.
    return (float)q * (float)(1.0 / DACC_ONE);
}

// Per-warp staging of x = xr + down sums (the residual stream entering a
// layer): warp w takes the same K-chunks as in warp_stage, polls their sum
// words until every block (`expect`) has added its share, keeps the new raw
// values in xr, folds in the RMSNorm gain, quantises with its own scale
// (wscale) and leaves its share of sum x^2 in ss_out[warp]. Returns false
// when the wait ran out (the abort flag is set); one decision per warp.
// ADD false: the sums are the whole vector (x = sums; xr only receives it).
template <bool ADD = true>
static __device__ bool warp_stage_sum(const uint64_t* acc, unsigned expect, int n, float* xr, float* xf, int8_t* xq,
                                      int plane, int nch, const float* gain, float* ss_out, float& wscale,
                                      const BlockState& st) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int c0 = warp * nch / NW, c1 = (warp + 1) * nch / NW;
    const int e0 = 16 * c0, e1 = min(16 * c1, n);
    bool okw = true;
    float ss = 0.f, mx = 0.f;
    uint64_t t0 = 0;
    unsigned rounds = 0;
    for (int base = e0; base < e1; base += 64) {
        uint64_t w[2];
        float g[2];
        unsigned pending = 0;
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const int j = base + lane + 32 * k;
            g[k] = 0.f;
            w[k] = 0;
            if (j < e1) {
                w[k] = ll_load(acc + j);
                g[k] = __ldg(gain + j);
                pending |= 1u << k;
            }
        }
        while (true) {
#pragma unroll
            for (int k = 0; k < 2; ++k)
                if (((pending >> k) & 1u) && dacc_count(w[k]) == expect) pending &= ~(1u << k);
            if (!pending) break;
            if ((++rounds & 7u) == 0 && wait_expired(st, t0)) {
                okw = false;
                break;
            }
#pragma unroll
            for (int k = 0; k < 2; ++k)
                if ((pending >> k) & 1u) w[k] = ll_load(acc + base + lane + 32 * k);
        }
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const int j = base + lane + 32 * k;
            if (j < e1) {
                const float v = ADD ? xr[j] + dacc_value(w[k]) : dacc_value(w[k]);
                xr[j] = v;
                const float gv = v * g[k];
                xf[j] = gv;
                ss = fmaf(v, v, ss);
                mx = fmaxf(mx, fabsf(gv));
            }
        }
        if (!okw) break;
    }
    okw = __all_sync(FULL, okw);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        ss += __shfl_xor_sync(FULL, ss, o);
        mx = fmaxf(mx, __shfl_xor_sync(FULL, mx, o));
    }
    if (lane == 0) ss_out[warp] = ss;
    const float rs = mx > 0.f ? FIX_MAX * __frcp_rn(mx) : 0.f;
    wscale = mx > 0.f ? __frcp_rn(rs) : 1.0f;
    __syncwarp();
    for (int quad = 4 * c0 + lane; quad < 4 * c1; quad += 32) {
        const int j = 4 * quad;
        const float4 v4 = j + 3 < n ? *reinterpret_cast<const float4*>(xf + j)
                                    : make_float4(j < n ? xf[j] : 0.f, j + 1 < n ? xf[j + 1] : 0.f,
                                                  j + 2 < n ? xf[j + 2] : 0.f, 0.f);
        uint32_t ph, pm, pl;
        fix_pack4(v4, rs, ph, pm, pl);
        reinterpret_cast<uint32_t*>(xq)[quad] = ph;
        reinterpret_cast<uint32_t*>(xq + plane)[quad] = pm;
        reinterpret_cast<uint32_t*>(xq + 2 * plane)[quad] = pl;
    }
    __syncwarp();
    return okw;
}

// A block's share of a projection split over K (the matvec of
// src/kernels.cpp:107-120 by columns): for every output row r < H,
// scale_r * sum_{j < DW} w[r][j] * h[j] with the block's column slice (H rows
// of DW int8 in shared memory, zero past its columns) and its input values h
// (DW floats, zero past its columns), added into the sum word acc[r] by a
// fire-and-forget reduction. Thread t owns rows t + i*NT; scale[i] is row
// t + i*NT's scale, loaded by the caller well ahead.
static __device__ void slice_partial(const uint8_t* slice, int DW, int H, const float* h, const float (&scale)[DOWN_RPT],
                                    uint64_t* acc) {
#pragma unroll
    for (int i = 0; i < DOWN_RPT; ++i) {
        const int r = threadIdx.x + i * NT;
        if (r < H) {
            const uint32_t* w = reinterpret_cast<const uint32_t*>(slice + (size_t)r * DW);
            float2 a = make_float2(0.f, 0.f);
            for (int k = 0; k < DW / 4; ++k) a = dot4(w[k], *reinterpret_cast<const float4*>(h + 4 * k), a);
            dacc_add(acc + r, (a.x + a.y) * scale[i]);
        }
    }
}

// Block-wide staging of x = xr + down sums (the final norm's input): thread t
// polls the sum words t, t + NT (H <= 2*NT) until `expect` blocks have added,
// then the vector is reduced and quantised as in finish_stage. Returns false
// when the step must abort. ADD false: x = sums (xr is not read).
template <bool ADD = true>
static __device__ bool stage_sum(const uint64_t* acc, unsigned expect, int n, int nch, const float* xr, float* xf,
                                 int8_t* xq, int plane, const float* gain, float* red, float eps, Staged& out,
                                 const BlockState& st) {
    float ss = 0.f, mx = 0.f;
    uint64_t w[2];
    unsigned pending = 0;
#pragma unroll
    for (int k = 0; k < 2; ++k) {
        const int j = threadIdx.x + k * NT;
        w[k] = 0;
        if (j < n) {
            w[k] = ll_load(acc + j);
            pending |= 1u << k;
        }
    }
    uint64_t t0 = 0;
    unsigned rounds = 0;
    while (true) {
#pragma unroll
        for (int k = 0; k < 2; ++k)
            if (((pending >> k) & 1u) && dacc_count(w[k]) == expect) pending &= ~(1u << k);
        if (!pending) break;
        if ((++rounds & 7u) == 0 && wait_expired(st, t0)) break;
#pragma unroll
        for (int k = 0; k < 2; ++k)
            if ((pending >> k) & 1u) w[k] = ll_load(acc + threadIdx.x + k * NT);
    }
#pragma unroll
    for (int k = 0; k < 2; ++k) {
        const int j = threadIdx.x + k * NT;
        if (j < n) accept(j, (ADD ? xr[j] : 0.f) + dacc_value(w[k]), nullptr, xf, __ldg(gain + j), ss, mx);
    }
    out = finish_stage(n, nch, xf, xq, plane, ss, mx, red, eps);
    return !should_abort(st);
}

// 1/sqrt(mean(v^2) + eps) from the warps' shares of sum v^2 (src/kernels.cpp:132-137).
__device__ __forceinline__ float rms_inv(const float* ss, int n, float eps) {
    float t = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) t += ss[w];
    return __frsqrt_rn(t / (float)n + eps);
}

// Partial dot products sum_j w_rj q_j of R packed rows in shared memory (stride
// S bytes, nch chunks of 16 int8 each) with the staged vector. Warp w covers
// chunks [w*nch/NW, (w+1)*nch/NW); in a warp, LPR consecutive lanes share a row
// slot and split its chunks, and each lane keeps up to P rows (slot,
// slot + 32/LPR, ...) in flight with independent accumulators, reusing each
// activation chunk for all of them. No per-row warp reduction: partial[w*R + r]
// is written and the caller sums over w after the closing barrier (and scales
// by Staged::scale). Rows are 912 or 4880 bytes apart, so the lanes' 16-byte
// reads of different rows fall in distinct banks.
template <int LPR, int P>
__device__ __noinline__ void block_gemv(const uint8_t* rows, int S, int R, int nch, const int8_t* xq, int plane,
                                        float* partial, float wscale = 1.0f, bool run = true) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int c0 = warp * nch / NW, c1 = (warp + 1) * nch / NW;
    const int sub = lane % LPR, slot = lane / LPR;
    constexpr int RPP = 32 / LPR;
    for (int r0 = 0; run && r0 < R; r0 += RPP * P) {
        int ah[P], am[P], al[P];
#pragma unroll
        for (int p = 0; p < P; ++p) ah[p] = am[p] = al[p] = 0;
        for (int c = c0 + sub; c < c1; c += LPR) {
            int4 h, m, l;
            load_planes(xq, plane, c, h, m, l);
#pragma unroll
            for (int p = 0; p < P; ++p) {
                const int r = r0 + p * RPP + slot;
                if (r < R)
                    dp4a16(*reinterpret_cast<const int4*>(rows + (size_t)r * S + (size_t)c * 16), h, m, l, ah[p], am[p],
                           al[p]);
            }
        }
#pragma unroll
        for (int p = 0; p < P; ++p) {
            const int r = r0 + p * RPP + slot;
            float t = planes_to_float(ah[p], am[p], al[p]);
#pragma unroll
            for (int o = LPR / 2; o > 0; o >>= 1) t += __shfl_xor_sync(FULL, t, o);
            if (sub == 0 && r < R) partial[warp * R + r] = t * wscale;
        }
    }
    __syncthreads();
}

// Sum of row r's partials over the warps.
__device__ __forceinline__ float gemv_row(const float* partial, int R, int r) {
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) s += partial[w * R + r];
    return s;
}

__device__ __forceinline__ float row_scale(const uint8_t* row, int K) {
    return *reinterpret_cast<const float*>(row + K);
}
__device__ __forceinline__ float row_bias(const uint8_t* row, int K) {
    return *reinterpret_cast<const float*>(row + K + 4);
}

__device__ __forceinline__ void trace_mark(const Params& P, int which, int phase) {
    if (P.trace && threadIdx.x == 0)
        P.trace[((size_t)which * TRACE_MAX_PHASES + phase) * gridDim.x + blockIdx.x] = globaltimer();
}
// SM clock counter next to the kernel start (which = 0) and end (1) marks:
// rows 500 + which of the done record, so a trace also yields the SM clock rate.
__device__ __forceinline__ void trace_clock(const Params& P, int which) {
    if (P.trace && threadIdx.x == 0)
        P.trace[((size_t)TRACE_MAX_PHASES + 500 + which) * gridDim.x + blockIdx.x] = clock64();
}
// Detailed marks inside phase k (0..4, or 5 for the LM head) of the traced
// layer: slot TRACE_DETAIL + 8k + m of the ready record.
constexpr int TRACE_DETAIL = 400;
__device__ __forceinline__ void trace_detail(const Params& P, int layer, int k, int m) {
    if (P.trace && layer == P.trace_layer && threadIdx.x == 0)
        P.trace[((size_t)TRACE_DETAIL + 8 * k + m) * gridDim.x + blockIdx.x] = globaltimer();
}

__device__ __forceinline__ float kv_to_float(float v) { return v; }
__device__ __forceinline__ float kv_to_float(__half v) { return __half2float(v); }
// Two adjacent KV elements (8- or 4-byte aligned) as FP32.
__device__ __forceinline__ float2 kv_to_float2(const float* p) { return *reinterpret_cast<const float2*>(p); }
__device__ __forceinline__ float2 kv_to_float2(const __half* p) {
    return __half22float2(*reinterpret_cast<const __half2*>(p));
}
__device__ __forceinline__ float round_to(float v, float) { return v; }
__device__ __forceinline__ float round_to(float v, __half) { return __half2float(__float2half_rn(v)); }

__device__ __forceinline__ void load4(const float* p, float (&out)[4]) {
    const float4 v = *reinterpret_cast<const float4*>(p);
    out[0] = v.x;
    out[1] = v.y;
    out[2] = v.z;
    out[3] = v.w;
}
__device__ __forceinline__ void load4(const __half* p, float (&out)[4]) {
    const uint2 v = *reinterpret_cast<const uint2*>(p);
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&v.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&v.y));
    out[0] = a.x;
    out[1] = a.y;
    out[2] = b.x;
    out[3] = b.y;
}

// ---- attention unit: query head h over positions [t0, t1) --------------------------
// The cached rows of the block's range come in 64-position chunks through a
// ring of att_bufs buffers ([K rows | V rows] each), the first att_bufs issued
// when the layer starts. The new row (position pos) is not copied: it arrives
// as tagged words and is read from shared memory where t == pos.
struct AttnPlan {
    int h, g, t0, t1, nchunks;
    int nissued;  // chunks holding cached rows (start below pos): the ones copied
    bool bulk;    // rows are multiples of 16 bytes: bulk copies, else plain loads
};

template <typename KV>
__device__ __forceinline__ const KV* kv_rows(const Params& P, const void* base, int l, int g, int t) {
    return static_cast<const KV*>(base) + (((size_t)l * P.NKV + g) * P.capacity + (t - P.kv_base)) * P.D;
}

// Thread 0: copy the cached rows (positions below pos) of chunk c into buffer c % att_bufs.
template <typename KV>
__device__ void att_issue(const Params& P, const StepArgs& A, const AttnPlan& ap, int l, int c, uint8_t* att,
                          uint64_t* mb_att, unsigned* fills) {
    const int c0 = ap.t0 + c * ATT_CHUNK;
    const int cend = min(min(ap.t1, c0 + ATT_CHUNK), A.pos);
    if (cend <= c0 || !ap.bulk) return;
    const int buf = c % P.att_bufs;
    const uint32_t rows = (uint32_t)(cend - c0), rb = (uint32_t)(P.D * sizeof(KV));
    KV* kdst = reinterpret_cast<KV*>(att + (size_t)buf * P.att_chunk_bytes);
    KV* vdst = kdst + (size_t)ATT_CHUNK * P.D;
    ++fills[buf];
    mbar_expect(mb_att + buf, 2 * rows * rb);
    bulk_load(kdst, kv_rows<KV>(P, P.kcache, l, ap.g, c0), rows * rb, mb_att + buf);
    bulk_load(vdst, kv_rows<KV>(P, P.vcache, l, ap.g, c0), rows * rb, mb_att + buf);
}

__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Softmax in base 2: scores are scaled by log2(e)/sqrt(D) and exponentiated
// with ex2, so that exp(s - m) = 2^((s - m) * log2(e)).
constexpr float LOG2E = 1.4426950408889634f;

// KV sequence split over GPUs: this GPU's (m, l, o) of head h (threads
// j < D hold own_m, own_l and dimension j of own_acc) goes to every rank's
// exchange buffer (system-scope tagged words over NVLink); then all ranks'
// partials are polled from the local buffer and merged in rank order, so every
// GPU ends with the same attention output, left in misc[0..D). Slots alternate
// with the global layer count: a rank one layer ahead writes the other slot.
// The start of att is used as scratch.
static __device__ bool exchange_head(const Params& P, const StepArgs& A, int h, int D, int l, uint32_t tag, uint8_t* att,
                                     float own_m, float own_l, float own_acc, float* misc, const BlockState& st) {
    {
        __syncthreads();  // the split tables above are consumed
        float* own = reinterpret_cast<float*>(att);  // [D+2]: m, l, o
        float* tab = own + (D + 2);                   // [world][D+2]
        if ((int)threadIdx.x < D) {
            own[2 + threadIdx.x] = own_acc;
            if (threadIdx.x == 0) {
                own[0] = own_m;
                own[1] = own_l;
            }
        }
        __syncthreads();
        const int slot = (int)((A.seq * (unsigned)P.L + (unsigned)l) & 1u);
        const int nw = P.world * (D + 2);
        for (int i = threadIdx.x; i < nw; i += NT) {
            const int q = i / (D + 2), k = i - q * (D + 2);
            ll_store_sys(P.peers[q] + (((size_t)slot * P.NH + h) * P.world + P.rank) * (D + 2) + k, own[k], tag);
        }
        const uint64_t* src = P.exch + ((size_t)slot * P.NH + h) * P.world * (D + 2);
        constexpr int WT = 4;  // world * (D+2) <= 8 * 130 < 4 * NT
        uint64_t w[WT];
        unsigned pending = 0;
#pragma unroll
        for (int k = 0; k < WT; ++k) {
            const int i = threadIdx.x + k * NT;
            if (i < nw) {
                w[k] = ll_load_sys(src + i);
                pending |= 1u << k;
            }
        }
        uint64_t t0 = 0;
        unsigned rounds = 0;
        while (pending) {
#pragma unroll
            for (int k = 0; k < WT; ++k)
                if (((pending >> k) & 1u) && (uint32_t)(w[k] >> 32) == tag) {
                    tab[threadIdx.x + k * NT] = __uint_as_float((uint32_t)w[k]);
                    pending &= ~(1u << k);
                }
            if (!pending) break;
            if ((++rounds & 7u) == 0 && wait_expired(st, t0)) break;
#pragma unroll
            for (int k = 0; k < WT; ++k)
                if ((pending >> k) & 1u) w[k] = ll_load_sys(src + threadIdx.x + k * NT);
        }
        __syncthreads();
        if (should_abort(st)) return false;
        if ((int)threadIdx.x < D) {
            const int j = threadIdx.x;
            float Mx = -INFINITY;
            for (int q = 0; q < P.world; ++q) Mx = fmaxf(Mx, tab[q * (D + 2)]);
            float num = 0.f, den = 0.f;
            for (int q = 0; q < P.world; ++q) {
                const float mq = tab[q * (D + 2)];
                const float f = mq > -INFINITY ? ex2_approx(mq - Mx) : 0.f;
                num = fmaf(f, tab[q * (D + 2) + 2 + j], num);
                den = fmaf(f, tab[q * (D + 2) + 1], den);
            }
            misc[j] = num / den;
        }
    }
    return true;
}

// DT: head_dim known at compile time (64), or 0 for any even head_dim <= 128.
// The block's attention output (split 0 of a head, after the merges) is left
// in misc[0..D). wo_src (split 0, when W_o's columns were not copied at the
// start of the layer): copied to att + wo_off once the chunks are consumed.
template <typename KV, int DT>
__device__ bool attention_block(const Params& P, const StepArgs& A, const AttnPlan& ap, int l, uint32_t tag,
                                uint8_t* att, uint64_t* mb_att, unsigned* issued, float* misc,
                                const uint8_t* wo_src, uint64_t* mb_wo, unsigned* wo_fills, const BlockState& st) {
    constexpr int MD = DT ? (DT + 31) / 32 : MAXD;  // 32-dim groups a lane covers
    const int D = DT ? DT : P.D, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int kvd = P.NKV * D, NB = P.att_bufs;
    float* sq = misc;                      // [D]
    float* s_new = misc + 128;             // [2][D] new K and V rows of group g (rounded to KV)
    float* wpart = misc + 384;             // [NW][D+2]: m, l, o of each warp
    const bool has_new = ap.t0 <= A.pos && A.pos < ap.t1;
    trace_detail(P, l, 1, 0);
    {
        // One round trip for the query and, where needed, the new K/V row:
        // thread t < D polls q[t], D <= t < 3D the new K then V rows.
        const int t = threadIdx.x, nwords = has_new ? 3 * D : D;
        if (t < nwords) {
            const uint64_t* src = t < D ? P.ll_q + (size_t)ap.h * D + t
                                        : P.ll_kv + (t < 2 * D ? 0 : kvd) + (size_t)ap.g * D + (t % D);
            uint64_t t0 = 0;
            unsigned rounds = 0;
            uint64_t w = ll_load(src);
            while ((uint32_t)(w >> 32) != tag) {
                if ((++rounds & 7u) == 0 && wait_expired(st, t0)) break;
                w = ll_load(src);
            }
            const float v = __uint_as_float((uint32_t)w);
            if (t < D) sq[t] = v;
            else s_new[t - D] = round_to(v, KV());
        }
        __syncthreads();
        if (should_abort(st)) return false;
    }
    trace_detail(P, l, 1, 1);
    const float qscale = LOG2E / sqrtf((float)D);
    // Scores: the 8 lanes of group `grp` take position warp*4+grp of a chunk;
    // lane part p owns dims 32k + 4p + e (e < 4), read as one vector.
    const int grp = lane >> 3, part = lane & 7;
    float qv[MD][4];
#pragma unroll
    for (int k = 0; k < MD; ++k)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int j = 32 * k + 4 * part + e;
            qv[k][e] = j < D ? sq[j] * qscale : 0.f;
        }
    float m_run = -INFINITY, l_run = 0.f, o[MD];
#pragma unroll
    for (int k = 0; k < MD; ++k) o[k] = 0.f;

    // Fill number of buffer b before this layer: every layer issues the same chunks.
    const int nissued = ap.nissued;
    for (int c = 0; c < ap.nchunks; ++c) {
        const int c0 = ap.t0 + c * ATT_CHUNK;
        const int n = min(ATT_CHUNK, ap.t1 - c0);
        const int ncache = max(0, min(n, A.pos - c0));
        const int buf = c % NB;
        const KV* kb = reinterpret_cast<const KV*>(att + (size_t)buf * P.att_chunk_bytes);
        const KV* vb = kb + (size_t)ATT_CHUNK * D;
        if (ncache > 0) {
            if (ap.bulk) {
                const int per_layer = (nissued - buf + NB - 1) / NB;  // fills of this buffer per layer
                const uint32_t parity = (uint32_t)(l * per_layer + c / NB) & 1u;
                if (!mbar_wait(mb_att + buf, parity, st)) return false;
            } else {
                KV* kw = const_cast<KV*>(kb);
                KV* vw = const_cast<KV*>(vb);
                for (int e = threadIdx.x; e < ncache * D; e += NT) {
                    const int t = e / D, j = e % D;
                    kw[(size_t)t * D + j] = *(kv_rows<KV>(P, P.kcache, l, ap.g, c0 + t) + j);
                    vw[(size_t)t * D + j] = *(kv_rows<KV>(P, P.vcache, l, ap.g, c0 + t) + j);
                }
                __syncthreads();
            }
            trace_detail(P, l, 1, c == 0 ? 2 : 4);
        }
        const int t = warp * ATT_PER_WARP + grp;
        float sc = 0.f;
        if (t < n) {
            const bool is_new = c0 + t == A.pos;
#pragma unroll
            for (int k = 0; k < MD; ++k) {
                const int j0 = 32 * k + 4 * part;
                float kk[4];
                if (j0 + 3 < D && (D & 3) == 0) {
                    if (is_new) load4(s_new + j0, kk);
                    else load4(kb + (size_t)t * D + j0, kk);
                } else {
#pragma unroll
                    for (int e = 0; e < 4; ++e)
                        kk[e] = j0 + e < D ? (is_new ? s_new[j0 + e] : kv_to_float(kb[(size_t)t * D + j0 + e])) : 0.f;
                }
#pragma unroll
                for (int e = 0; e < 4; ++e) sc = fmaf(qv[k][e], kk[e], sc);
            }
        }
        sc += __shfl_xor_sync(FULL, sc, 4);
        sc += __shfl_xor_sync(FULL, sc, 2);
        sc += __shfl_xor_sync(FULL, sc, 1);
        sc = t < n ? sc : -INFINITY;
        float cmax = fmaxf(sc, __shfl_xor_sync(FULL, sc, 8));
        cmax = fmaxf(cmax, __shfl_xor_sync(FULL, cmax, 16));
        if (cmax > -INFINITY) {
            const float m_new = fmaxf(m_run, cmax);
            const float alpha = ex2_approx(m_run - m_new);
            const float p = ex2_approx(sc - m_new);
            float psum = p + __shfl_xor_sync(FULL, p, 8);
            psum += __shfl_xor_sync(FULL, psum, 16);
            l_run = fmaf(l_run, alpha, psum);
#pragma unroll
            for (int k = 0; k < MD; ++k) o[k] *= alpha;
#pragma unroll
            for (int i = 0; i < ATT_PER_WARP; ++i) {
                const float pi = __shfl_sync(FULL, p, 8 * i);
                const int ti = warp * ATT_PER_WARP + i;
                if (ti < n) {
                    if (c0 + ti == A.pos) {
#pragma unroll
                        for (int k = 0; k < MD; ++k)
                            if (lane + 32 * k < D) o[k] = fmaf(pi, s_new[D + lane + 32 * k], o[k]);
                    } else {
#pragma unroll
                        for (int k = 0; k < MD; ++k)
                            if (lane + 32 * k < D) o[k] = fmaf(pi, kv_to_float(vb[(size_t)ti * D + lane + 32 * k]), o[k]);
                    }
                }
            }
            m_run = m_new;
        }
        trace_detail(P, l, 1, c == 0 ? 3 : 5);
        if (c + NB < ap.nchunks || !ap.bulk) {
            __syncthreads();  // buffer `buf` consumed by every warp
            if (threadIdx.x == 0 && c + NB < ap.nchunks) {
                fence_proxy_async();
                att_issue<KV>(P, A, ap, l, c + NB, att, mb_att, issued);
            }
        }
    }
    // Merge the warps' softmax states: warp w's (m, l, o) to shared memory;
    // lanes of warps 0..ceil(D/32)-1 then weight warp w by 2^(m_w - M).
    if (lane == 0) {
        wpart[warp * (D + 2)] = m_run;
        wpart[warp * (D + 2) + 1] = l_run;
    }
#pragma unroll
    for (int k = 0; k < MD; ++k)
        if (lane + 32 * k < D) wpart[warp * (D + 2) + 2 + lane + 32 * k] = o[k];
    __syncthreads();
    // Every warp is done with the chunk buffers: split 0 brings in W_o's
    // columns of this head now unless they came at the start of the layer.
    if (threadIdx.x == 0 && wo_src) {
        fence_proxy_async();
        fill_slot(att + P.wo_off, wo_src, (uint32_t)P.o_slice, mb_wo, wo_fills);
    }
    const int split = blockIdx.x % A.nsplit;
    float own_m = 0.f, own_l = 0.f, own_acc = 0.f;  // split 0 of several: its own partial (threads j < D)
    if (threadIdx.x < ((D + 31) & ~31)) {
        const int j = threadIdx.x;
        const float mw = lane < NW ? wpart[lane * (D + 2)] : -INFINITY;
        float M = mw;
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(FULL, M, off));
        const float f = (lane < NW && mw > -INFINITY) ? ex2_approx(mw - M) : 0.f;
        float Lsum = lane < NW ? f * wpart[lane * (D + 2) + 1] : 0.f;
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) Lsum += __shfl_xor_sync(FULL, Lsum, off);
        float acc = 0.f;
#pragma unroll
        for (int w = 0; w < NW; ++w) {
            const float fw = __shfl_sync(FULL, f, w);
            if (j < D) acc = fmaf(fw, wpart[w * (D + 2) + 2 + j], acc);
        }
        if (j < D) {
            if (A.nsplit == 1 && P.world == 1) {
                misc[j] = acc / Lsum;
            } else if (split == 0) {
                own_m = M;
                own_l = Lsum;
                own_acc = acc;
            } else {
                // (m, l, unnormalised o) of this split as tagged words for split 0.
                uint64_t* pw = P.ll_part + ((size_t)ap.h * A.nsplit + split) * (D + 2);
                ll_store(pw + 2 + j, acc, tag);
                if (j == 0) {
                    ll_store(pw, M, tag);
                    ll_store(pw + 1, Lsum, tag);
                }
            }
        }
    }
    trace_detail(P, l, 1, 6);
    if (split != 0 || (A.nsplit == 1 && P.world == 1)) return true;
    if (A.nsplit > 1) {
    // Split 0 merges the others (m in base 2): thread t polls words t, t + NT,
    // ... of their (nsplit-1)*(D+2)-word table, all loads in flight, into the
    // chunk buffers (consumed by now); then thread j < D combines dimension j
    // in split order.
    {
        const int nwords = (A.nsplit - 1) * (D + 2);
        const uint64_t* src = P.ll_part + ((size_t)ap.h * A.nsplit + 1) * (D + 2);
        float* table = reinterpret_cast<float*>(att);
        constexpr int WT = 4;
        for (int base = 0; base < nwords; base += WT * NT) {
            uint64_t w[WT];
            unsigned pending = 0;
#pragma unroll
            for (int k = 0; k < WT; ++k) {
                const int i = base + threadIdx.x + k * NT;
                if (i < nwords) {
                    w[k] = ll_load(src + i);
                    pending |= 1u << k;
                }
            }
            uint64_t t0 = 0;
            unsigned rounds = 0;
            while (true) {
#pragma unroll
                for (int k = 0; k < WT; ++k)
                    if (((pending >> k) & 1u) && (uint32_t)(w[k] >> 32) == tag) {
                        table[base + threadIdx.x + k * NT] = __uint_as_float((uint32_t)w[k]);
                        pending &= ~(1u << k);
                    }
                if (!pending) break;
                if ((++rounds & 7u) == 0 && wait_expired(st, t0)) break;
#pragma unroll
                for (int k = 0; k < WT; ++k)
                    if ((pending >> k) & 1u) w[k] = ll_load(src + base + threadIdx.x + k * NT);
            }
        }
        __syncthreads();
        if (should_abort(st)) return false;
        if ((int)threadIdx.x < D) {
            const int j = threadIdx.x;
            float Mx = own_m;
            for (int i = 0; i + 1 < A.nsplit; ++i) Mx = fmaxf(Mx, table[i * (D + 2)]);
            const float f0 = ex2_approx(own_m - Mx);
            float num = f0 * own_acc, den = f0 * own_l;
            for (int i = 0; i + 1 < A.nsplit; ++i) {
                const float f = ex2_approx(table[i * (D + 2)] - Mx);
                num = fmaf(f, table[i * (D + 2) + 2 + j], num);
                den = fmaf(f, table[i * (D + 2) + 1], den);
            }
            if (P.world == 1) {
                misc[j] = num / den;
            } else {
                own_m = Mx;
                own_l = den;
                own_acc = num;
            }
        }
    }
    }
    if (P.world == 1) return true;
    return exchange_head(P, A, ap.h, D, l, tag, att, own_m, own_l, own_acc, misc, st);
}


// ---- attention unit of a whole KV group (long contexts, head_dim 64) -------------
// Block (g, split) reads each cached chunk of its range once for all hpg query
// heads of KV group g (hpg <= GQA_MAX), in passes of up to GQA_PASS resident
// chunks:
//   A: a warp takes 32 positions and 4 of the heads; lane = position, its
//      64-dim dot products walk the K row in a lane-rotated order (no bank
//      conflicts); q is pre-scaled by log2(e)/8 in shared memory (qt);
//   B: warp h turns head h's scores of the pass into 2^(s - m) with the running
//      max m and adds them to the running sum;
//   C: thread (h, d) rescales and accumulates o_h[d] += p_t * V[t][d].
// The new row (position pos) is first written into its chunk buffer, so every
// position is read the same way. Each split publishes (m, l, o) of every head
// as tagged words; block (g, j), j < hpg, then merges head g*hpg + j over all
// splits in split order and leaves the result in misc[0..64). stile: the
// [GQA_MAX][GQA_PASS*64] score tile.
template <typename KV>
__device__ bool attention_group(const Params& P, const StepArgs& A, const AttnPlan& ap, int l, uint32_t tag,
                                uint8_t* att, uint64_t* mb_att, unsigned* issued, float* misc, float* qt,
                                float* stile, const uint8_t* wo_src, uint64_t* mb_wo, unsigned* wo_fills,
                                const BlockState& st) {
    constexpr int D = 64, SROW = GQA_PASS * ATT_CHUNK;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, tid = threadIdx.x;
    const int hpg = P.NH / P.NKV, NB = P.att_bufs, split = blockIdx.x % A.nsplit;
    float* s_new = misc + 128;   // [2][D] new K and V rows (rounded to KV)
    float* hm = misc + 384;      // [GQA_MAX] running max per head
    float* hl = hm + GQA_MAX;    // running sum
    float* ha = hl + GQA_MAX;    // rescale of the current pass
    trace_detail(P, l, 1, 0);
    {
        // q of the group's heads and the new K/V rows of the group: one round trip.
        const int nq = hpg * D, nwords = nq + 2 * D;
        uint64_t w[2];
        unsigned pending = 0;
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const int i = tid + k * NT;
            w[k] = 0;
            if (i < nwords) {
                w[k] = ll_load(i < nq ? P.ll_q + (size_t)ap.g * nq + i
                                      : P.ll_kv + (i < nq + D ? 0 : P.NKV * D) + (size_t)ap.g * D + (i - nq) % D);
                pending |= 1u << k;
            }
        }
        uint64_t t0 = 0;
        unsigned rounds = 0;
        while (true) {
#pragma unroll
            for (int k = 0; k < 2; ++k)
                if (((pending >> k) & 1u) && (uint32_t)(w[k] >> 32) == tag) pending &= ~(1u << k);
            if (!pending) break;
            if ((++rounds & 7u) == 0 && wait_expired(st, t0)) break;
#pragma unroll
            for (int k = 0; k < 2; ++k)
                if ((pending >> k) & 1u) {
                    const int i = tid + k * NT;
                    w[k] = ll_load(i < nq ? P.ll_q + (size_t)ap.g * nq + i
                                          : P.ll_kv + (i < nq + D ? 0 : P.NKV * D) + (size_t)ap.g * D + (i - nq) % D);
                }
        }
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const int i = tid + k * NT;
            if (i < nwords) {
                const float v = __uint_as_float((uint32_t)w[k]);
                if (i < nq) qt[i] = v * (LOG2E / 8.0f);
                else s_new[i - nq] = round_to(v, KV());
            }
        }
        if (tid < GQA_MAX) {
            hm[tid] = -INFINITY;
            hl[tid] = 0.f;
        }
        __syncthreads();
        if (should_abort(st)) return false;
    }
    trace_detail(P, l, 1, 1);
    float2 o0 = make_float2(0.f, 0.f), o1 = o0;  // thread (h, d2) = (tid / 32, tid % 32), tid < hpg * 32: dims 2d2, 2d2+1
    const int nissued = ap.nissued;
    const int pass = P.gqa_pass;
    for (int c = 0; c < ap.nchunks; c += pass) {
        const int cb = min(pass, ap.nchunks - c);
        __syncthreads();  // the previous pass is done with the buffers and the score tile
        for (int u = 0; u < cb; ++u) {
            const int cu = c + u, c0 = ap.t0 + cu * ATT_CHUNK;
            const int ncache = max(0, min(min(ATT_CHUNK, ap.t1 - c0), A.pos - c0));
            if (ncache <= 0) continue;
            const int buf = cu % NB;
            const int per_layer = (nissued - buf + NB - 1) / NB;  // fills of this buffer per layer
            if (!mbar_wait(mb_att + buf, (uint32_t)(l * per_layer + cu / NB) & 1u, st)) return false;
        }
        trace_detail(P, l, 1, c == 0 ? 2 : 4);
        {
            // The new row into its chunk buffer, where the cached rows end.
            const int pc = (A.pos - ap.t0) / ATT_CHUNK - c;
            if (A.pos >= ap.t0 && A.pos < ap.t1 && pc >= 0 && pc < cb && tid < 2 * D) {
                KV* kb = reinterpret_cast<KV*>(att + (size_t)((c + pc) % NB) * P.att_chunk_bytes);
                const int t = (A.pos - ap.t0) % ATT_CHUNK;
                kv_store(kb + (tid < D ? 0 : (size_t)ATT_CHUNK * D) + (size_t)t * D + tid % D, s_new[tid]);
            }
        }
        __syncthreads();
        // A: scores of the pass into the tile (-inf past a chunk's last position).
        // Warp w takes positions 4w..4w+3 of every chunk of the pass: the 8 lanes
        // of group grp own dims 4*part .. +3 and 32 + 4*part .. +3 of position
        // 4w+grp (8 lanes read 128 contiguous bytes: no bank conflicts), read them
        // once, and for each head add q_h over those dims and reduce over the 8
        // lanes (q is read from shared memory, the same dims by 4 lanes).
        {
            const int grp = lane >> 3, part = lane & 7, t = warp * 4 + grp;
            for (int u = 0; u < cb; ++u) {
                const int c0 = ap.t0 + (c + u) * ATT_CHUNK;
                const int n = min(ATT_CHUNK, ap.t1 - c0);
                float kk[8];
                if (t < n) {
                    const KV* kr = reinterpret_cast<const KV*>(att + (size_t)((c + u) % NB) * P.att_chunk_bytes) +
                                   (size_t)t * D + 4 * part;
                    float a[4], bq[4];
                    load4(kr, a);
                    load4(kr + 32, bq);
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        kk[e] = a[e];
                        kk[4 + e] = bq[e];
                    }
                } else {
#pragma unroll
                    for (int e = 0; e < 8; ++e) kk[e] = 0.f;
                }
                for (int h = 0; h < hpg; ++h) {
                    const float4 q0 = *reinterpret_cast<const float4*>(qt + h * D + 4 * part);
                    const float4 q1 = *reinterpret_cast<const float4*>(qt + h * D + 32 + 4 * part);
                    float sc = q0.x * kk[0];
                    sc = fmaf(q0.y, kk[1], sc);
                    sc = fmaf(q0.z, kk[2], sc);
                    sc = fmaf(q0.w, kk[3], sc);
                    sc = fmaf(q1.x, kk[4], sc);
                    sc = fmaf(q1.y, kk[5], sc);
                    sc = fmaf(q1.z, kk[6], sc);
                    sc = fmaf(q1.w, kk[7], sc);
                    sc += __shfl_xor_sync(FULL, sc, 4);
                    sc += __shfl_xor_sync(FULL, sc, 2);
                    sc += __shfl_xor_sync(FULL, sc, 1);
                    if (part == 0) stile[h * SROW + u * ATT_CHUNK + t] = t < n ? sc : -INFINITY;
                }
            }
        }
        __syncthreads();
        // B: per head, 2^(s - m) with the running max, and the running sum.
        if (warp < hpg) {
            float* row = stile + warp * SROW;
            const int np = cb * ATT_CHUNK;
            float mx = -INFINITY;
            for (int q = lane; q < np; q += 32) mx = fmaxf(mx, row[q]);
            mx = warp_max(mx);
            const float mo = hm[warp], mn = fmaxf(mo, mx);
            float sum = 0.f;
            for (int q = lane; q < np; q += 32) {
                const float e = ex2_approx(row[q] - mn);
                row[q] = e;
                sum += e;
            }
            sum = warp_sum(sum);
            if (lane == 0) {
                const float al = ex2_approx(mo - mn);
                ha[warp] = al;
                hl[warp] = fmaf(hl[warp], al, sum);
                hm[warp] = mn;
            }
        }
        __syncthreads();
        // C: o_h[2d2..2d2+1] += p_t * V[t][2d2..2d2+1] over the pass's positions
        // (one 8-byte V load per two FMAs).
        if (tid < hpg * 32) {
            const int h = tid >> 5, d2 = tid & 31;
            const float al = ha[h];
            o0.x *= al;
            o0.y *= al;
            o1.x *= al;
            o1.y *= al;
            const float* prow = stile + h * SROW;
            for (int u = 0; u < cb; ++u) {
                const int c0 = ap.t0 + (c + u) * ATT_CHUNK;
                const int n = min(ATT_CHUNK, ap.t1 - c0);
                const KV* vb = reinterpret_cast<const KV*>(att + (size_t)((c + u) % NB) * P.att_chunk_bytes) +
                               (size_t)ATT_CHUNK * D + 2 * d2;
                const float* pu = prow + u * ATT_CHUNK;
                int t = 0;
#pragma unroll 2
                for (; t + 4 <= n; t += 4) {
                    const float4 pv = *reinterpret_cast<const float4*>(pu + t);
                    const float2 v0 = kv_to_float2(vb + (size_t)t * D), v1 = kv_to_float2(vb + (size_t)(t + 1) * D);
                    const float2 v2 = kv_to_float2(vb + (size_t)(t + 2) * D), v3 = kv_to_float2(vb + (size_t)(t + 3) * D);
                    o0.x = fmaf(pv.x, v0.x, o0.x);
                    o0.y = fmaf(pv.x, v0.y, o0.y);
                    o1.x = fmaf(pv.y, v1.x, o1.x);
                    o1.y = fmaf(pv.y, v1.y, o1.y);
                    o0.x = fmaf(pv.z, v2.x, o0.x);
                    o0.y = fmaf(pv.z, v2.y, o0.y);
                    o1.x = fmaf(pv.w, v3.x, o1.x);
                    o1.y = fmaf(pv.w, v3.y, o1.y);
                }
                for (; t < n; ++t) {
                    const float2 vt = kv_to_float2(vb + (size_t)t * D);
                    o0.x = fmaf(pu[t], vt.x, o0.x);
                    o0.y = fmaf(pu[t], vt.y, o0.y);
                }
            }
        }
        trace_detail(P, l, 1, c == 0 ? 3 : 5);
        if (c + NB < ap.nchunks) {
            __syncthreads();  // the pass's buffers are consumed by every warp
            if (tid == 0)
                for (int u = 0; u < cb; ++u)
                    if (c + u + NB < ap.nchunks) {
                        if (u == 0) fence_proxy_async();
                        att_issue<KV>(P, A, ap, l, c + u + NB, att, mb_att, issued);
                    }
        }
    }
    // (m, l, unnormalised o) of every head of the group for this split.
    if (tid < hpg * 32) {
        const int h = tid >> 5, d = 2 * (tid & 31);
        uint64_t* pw = P.ll_part + ((size_t)(ap.g * hpg + h) * A.nsplit + split) * (D + 2);
        ll_store(pw + 2 + d, o0.x + o1.x, tag);
        ll_store(pw + 3 + d, o0.y + o1.y, tag);
        if (d == 0) {
            ll_store(pw, hm[h], tag);
            ll_store(pw + 1, hl[h], tag);
        }
    }
    trace_detail(P, l, 1, 6);
    if (split >= hpg) return true;
    // Block (g, j) merges head g*hpg + j over all splits: W_o's columns of that
    // head come into the end of the chunk buffers now (unless they came at the
    // start of the layer), the splits' partials into their start.
    __syncthreads();
    if (tid == 0 && wo_src) {
        fence_proxy_async();
        fill_slot(att + P.wo_off, wo_src, (uint32_t)P.o_slice, mb_wo, wo_fills);
    }
    {
        const int nwords = A.nsplit * (D + 2);
        const uint64_t* src = P.ll_part + (size_t)(ap.g * hpg + split) * A.nsplit * (D + 2);
        float* table = reinterpret_cast<float*>(att);
        constexpr int WT = 4;
        for (int base = 0; base < nwords; base += WT * NT) {
            uint64_t w[WT];
            unsigned pending = 0;
#pragma unroll
            for (int k = 0; k < WT; ++k) {
                const int i = base + tid + k * NT;
                if (i < nwords) {
                    w[k] = ll_load(src + i);
                    pending |= 1u << k;
                }
            }
            uint64_t t0 = 0;
            unsigned rounds = 0;
            while (true) {
#pragma unroll
                for (int k = 0; k < WT; ++k)
                    if (((pending >> k) & 1u) && (uint32_t)(w[k] >> 32) == tag) {
                        table[base + tid + k * NT] = __uint_as_float((uint32_t)w[k]);
                        pending &= ~(1u << k);
                    }
                if (!pending) break;
                if ((++rounds & 7u) == 0 && wait_expired(st, t0)) break;
#pragma unroll
                for (int k = 0; k < WT; ++k)
                    if ((pending >> k) & 1u) w[k] = ll_load(src + base + tid + k * NT);
            }
        }
        __syncthreads();
        if (should_abort(st)) return false;
        // Merge in split order, spread over the block: the largest m (warp 0),
        // each split's weight 2^(m_s - M) once, then thread (d, q) sums splits
        // q, q + 8, ... of dimension d (and q's share of the weights' sum), and
        // thread d adds the 8 shares in order.
        float* wgt = misc + 384;           // [nsplit <= GQA_MERGE_MAX] weights
        float* part = wgt + GQA_MERGE_MAX; // [8][D + 1] shares of num (D) and den (1)
        float* smx = part + 8 * (D + 1);   // the largest m
        if (warp == 0) {
            float mx = -INFINITY;
            for (int i = lane; i < A.nsplit; i += 32) mx = fmaxf(mx, table[i * (D + 2)]);
            mx = warp_max(mx);
            if (lane == 0) *smx = mx;
            for (int i = lane; i < A.nsplit; i += 32) wgt[i] = ex2_approx(table[i * (D + 2)] - mx);
        }
        __syncthreads();
        {
            const int d = tid & 63, q = tid >> 6;  // q < 8
            float num = 0.f, den = 0.f;
            for (int i = q; i < A.nsplit; i += 8) {
                num = fmaf(wgt[i], table[i * (D + 2) + 2 + d], num);
                if (d == 0) den = fmaf(wgt[i], table[i * (D + 2) + 1], den);
            }
            part[q * (D + 1) + d] = num;
            if (d == 0) part[q * (D + 1) + D] = den;
        }
        __syncthreads();
        float num = 0.f, den = 0.f;
        if (tid < D) {
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                num += part[q * (D + 1) + tid];
                den += part[q * (D + 1) + D];
            }
            if (P.world == 1) misc[tid] = num / den;
        }
        if (P.world > 1) return exchange_head(P, A, ap.g * hpg + split, D, l, tag, att, *smx, den, num, misc, st);
    }
    return true;
}

template <typename KV>
__global__ void __launch_bounds__(NT, 1) decode_step_kernel(const Params P, const StepArgs A) {
    extern __shared__ __align__(128) uint8_t sm[];
    uint8_t* s_gu = sm + P.off_gu;
    uint8_t* s_down = sm + P.off_down;
    uint8_t* s_qkv = sm + P.off_qkv;
    uint8_t* s_att = sm + P.off_att;
    float* xf = reinterpret_cast<float*>(sm + P.off_xs);       // staged values before quantisation
    int8_t* xq = reinterpret_cast<int8_t*>(sm + P.off_xq);     // fixed-point planes of the staged vector
    const int QP = P.xq_plane;
    float* gpart = reinterpret_cast<float*>(sm + P.off_gpart);  // block-GEMV partial sums, two buffers
    float* xr = reinterpret_cast<float*>(sm + P.off_xr);
    float* misc = reinterpret_cast<float*>(sm + P.off_misc);
    // mbarriers: three weight slots and W_o's head columns, then the attention
    // chunk ring (one arrival + bytes each).
    constexpr int MB_ATT = 4;
    constexpr int NMB = MB_ATT + ATT_MAX_BUFS;
    __shared__ __align__(8) uint64_t mb[NMB];
    uint64_t* mb_gu = mb + 0;
    uint64_t* mb_down = mb + 1;
    uint64_t* mb_qkv = mb + 2;
    uint64_t* mb_wo = mb + 3;
    uint64_t* mb_att = mb + MB_ATT;
    __shared__ float s_cos[64], s_sin[64];
    __shared__ __align__(16) float red[2 * NW + 8];  // read as float4 in finish_stage
    __shared__ float s_ss[NW];  // the warps' shares of sum x^2 for the RMSNorm of a phase
    __shared__ int s_abort;
    __shared__ unsigned s_fills[NMB];  // fills issued per mbarrier (thread 0)
    __shared__ ArgBest s_best;
    __shared__ int s_last;

    const int G = gridDim.x, b = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int H = P.H, I = P.I, D = P.D, half = D / 2, kvd = P.NKV * D;
    const int nch_h = P.Kh / 16;
    const BlockState st{&s_abort, P.sync};

    // This block's rows in every phase.
    const int qa = part_lo(b, G, P.qkv_pairs), qn = part_lo(b + 1, G, P.qkv_pairs) - qa;
    const int ga = part_lo(b, G, I), gn = part_lo(b + 1, G, I) - ga;
    const int ha = part_lo(b, G, P.V), hn = part_lo(b + 1, G, P.V) - ha;
    // This step's sum words (the other half is cleared at the end): per layer
    // the O sums, complete when every head has added, then the down sums,
    // complete when every block that holds down columns has added.
    uint64_t* const dacc = P.dacc + (size_t)A.par * P.L * 2 * P.Hp;
    auto osum = [&](int l) { return dacc + (size_t)(2 * l) * P.Hp; };
    auto dsum = [&](int l) { return dacc + (size_t)(2 * l + 1) * P.Hp; };
    const unsigned dblocks = (unsigned)min(G, I);
    float* const s_h = reinterpret_cast<float*>(sm + P.off_h);  // [down_dw] this block's SiLU(gate)*up

    // This block's attention unit (at most one).
    // Units are (query head, split), or (KV group, split) when A.group.
    AttnPlan ap{};
    const int hpg = P.NH / P.NKV;
    const bool has_att = b < (A.group ? P.NKV : P.NH) * A.nsplit;
    if (has_att) {
        const int unit = b / A.nsplit, usplit = b % A.nsplit;
        ap.g = A.group ? unit : unit / hpg;
        ap.h = A.group ? ap.g * hpg + min(usplit, hpg - 1) : unit;
        ap.t0 = P.kv_base + (b % A.nsplit) * A.split_len;
        ap.t1 = min(min(A.pos + 1, P.kv_end), ap.t0 + A.split_len);
        ap.nchunks = (ap.t1 - ap.t0 + ATT_CHUNK - 1) / ATT_CHUNK;
        ap.nissued = min(ap.nchunks, max(0, (A.pos - ap.t0 + ATT_CHUNK - 1) / ATT_CHUNK));
        ap.bulk = ((size_t)D * sizeof(KV)) % 16 == 0;
    }
    // Split 0 of a head finishes it and adds its O share. W_o's columns come at
    // the start of a layer when this layer's chunks leave the buffers at
    // wo_off free, else once the chunks are consumed.
    const bool o_head = has_att && (A.group ? b % A.nsplit < hpg : b % A.nsplit == 0);
    const bool wo_early = o_head && (size_t)ap.nchunks * P.att_chunk_bytes <= (size_t)P.wo_off;

    if (tid == 0) {
        s_abort = 0;
        for (int i = 0; i < NMB; ++i) {
            mbar_init(mb + i, 1);
            s_fills[i] = 0;
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        const LayerW& W = P.layers[0];
        if (qn) fill_slot(s_qkv, W.qkv + (size_t)qa * 2 * P.SH, (uint32_t)qn * 2 * P.SH, mb_qkv, s_fills + 2);
        if (gn) fill_slot(s_gu, W.gu + (size_t)ga * 2 * P.SH, (uint32_t)gn * 2 * P.SH, mb_gu, s_fills + 0);
        if (gn) fill_slot(s_down, P.down_cols + (size_t)b * P.down_slice, (uint32_t)P.down_slice, mb_down, s_fills + 1);
    }
    // RoPE cos/sin of this position, once per step (src/model.cpp:269-274).
    if (tid < half) {
        const float angle = P.cached_rope ? __fmul_rn((float)A.pos, P.rope_inv[tid]) : __fdiv_rn((float)A.pos, P.rope_den[tid]);
        sincosf(angle, &s_sin[tid], &s_cos[tid]);
    }
    __syncthreads();
    trace_mark(P, 0, 0);
    trace_mark(P, 1, 0);
    trace_clock(P, 0);

    int token = A.token_dev ? __ldcg(A.token_dev) : A.token;
    if ((unsigned)token >= (unsigned)P.V) {  // a device-supplied token out of range
        if (tid == 0) atomicCAS(&P.sync->error, 0, ERR_TOKEN);
        token = 0;
    }
    const uint32_t seq_tag = A.seq << 8;  // tag of layer l's outputs: seq_tag | (l + 1)
    bool ok = true;
    KV* const kc = static_cast<KV*>(P.kcache);
    KV* const vc = static_cast<KV*>(P.vcache);

    for (int l = 0; l < P.L; ++l) {
        const LayerW& W = P.layers[l];
        const uint32_t tag = seq_tag | (uint32_t)(l + 1);
        const int ph = 5 * l;

        // RMSNorm gains of layer l (global memory; read while the words are polled).
        const float* in_norm = P.norms + (size_t)l * 2 * P.Kh;
        const float* post_norm = in_norm + P.Kh;
        // Row scales of this layer's O and down projections for the rows this
        // thread adds (tid + i*NT): loaded now, used after attention and gate/up.
        float oscale[DOWN_RPT], dscale[DOWN_RPT];
#pragma unroll
        for (int i = 0; i < DOWN_RPT; ++i) {
            const int r = tid + i * NT;
            oscale[i] = o_head && r < H ? __ldg(P.o_scale + (size_t)l * H + r) : 0.f;
            dscale[i] = gn && r < H ? __ldg(P.down_scale + (size_t)l * H + r) : 0.f;
        }
        const uint8_t* wo_src = o_head ? P.o_cols + ((size_t)l * P.NH + ap.h) * P.o_slice : nullptr;

        // HBM has slack during the last layer: start this block's first LM-head rows into L2.
        if (tid == 0 && A.head && l == P.L - 1 && hn)
            prefetch_slice(P.embed + (size_t)ha * P.SH, (size_t)min(hn, HEAD_L2_ROWS) * P.SH, 0, 1);

        // The cached KV rows do not depend on this step: start their copies now.
        if (has_att && tid == 0) {
            fence_proxy_async();  // the previous layer read and wrote these buffers
            for (int c = 0; c < min(P.att_bufs, ap.nchunks); ++c)
                att_issue<KV>(P, A, ap, l, c, s_att, mb_att, s_fills + MB_ATT);
            if (wo_early) fill_slot(s_att + P.wo_off, wo_src, (uint32_t)P.o_slice, mb_wo, s_fills + 3);
        }

        // ---- QKV (src/model.cpp:276-302). x entering layer 0 is the embedding
        // row; entering layer l > 0 it is x_b of layer l-1 (xr) plus the down
        // sums of layer l-1, read once every block has added its share.
        // Each warp stages its own chunks of x (RMSNorm gain folded in) and
        // starts its share of the GEMV; 1/rms scales the row totals. Every
        // block keeps x in xr: x_b = xr + O sums.
        trace_detail(P, l, 0, 0);
        {
            float wsc = 1.f;
            bool okw;
            if (l == 0) {
                const uint8_t* er = P.embed + (size_t)token * P.SH;
                okw = warp_stage<2, true>(nullptr, er, row_scale(er, P.Kh), H, tag, xr, xf, xq, QP, nch_h, in_norm,
                                          s_ss, wsc, st);
            } else {
                okw = warp_stage_sum(dsum(l - 1), dblocks, H, xr, xf, xq, QP, nch_h, in_norm, s_ss, wsc, st);
            }
            trace_detail(P, l, 0, 1);
            if (!qn) {
                __syncthreads();
                if (should_abort(st)) {
                    ok = false;
                    break;
                }
            } else {
                trace_detail(P, l, 0, 2);
                const bool okg = okw && warp_slot_wait(mb_qkv, (uint32_t)l & 1u, st);
                trace_mark(P, 0, ph + 1);
                trace_detail(P, l, 0, 3);
                const int qpairs = P.NH * half, kpairs = P.NKV * half;
                block_gemv<8, 2>(s_qkv, P.SH, 2 * qn, nch_h, xq, QP, gpart, wsc, okg);
                if (should_abort(st)) {
                    ok = false;
                    break;
                }
                // One thread per RoPE pair (rows j, j + d/2 of a head).
                if (tid < qn) {
                    const float inv = rms_inv(s_ss, H, P.eps);
                    const int w = tid, u = qa + w;
                    const uint8_t* r0 = s_qkv + (size_t)w * 2 * P.SH;
                    float y0 = gemv_row(gpart, 2 * qn, 2 * w) * inv * row_scale(r0, P.Kh) + row_bias(r0, P.Kh);
                    float y1 = gemv_row(gpart, 2 * qn, 2 * w + 1) * inv * row_scale(r0 + P.SH, P.Kh) +
                               row_bias(r0 + P.SH, P.Kh);
                    const int kind = u < qpairs ? 0 : (u < qpairs + kpairs ? 1 : 2);
                    const int pu = kind == 0 ? u : (kind == 1 ? u - qpairs : u - qpairs - kpairs);
                    const int hd = pu / half, j = pu % half;
                    if (kind < 2) {
                        const float sn = s_sin[j], cs = s_cos[j];
                        const float a = y0, bb = y1;
                        y0 = __fsub_rn(__fmul_rn(a, cs), __fmul_rn(bb, sn));
                        y1 = __fadd_rn(__fmul_rn(bb, cs), __fmul_rn(a, sn));
                    }
                    if (kind == 0) {
                        ll_store(P.ll_q + hd * D + j, y0, tag);
                        ll_store(P.ll_q + hd * D + j + half, y1, tag);
                    } else {
                        if (A.pos >= P.kv_base && A.pos < P.kv_end) {  // this engine keeps position pos
                            KV* cache = (kind == 1 ? kc : vc) +
                                        (((size_t)l * P.NKV + hd) * P.capacity + (A.pos - P.kv_base)) * D;
                            kv_store(cache + j, y0);
                            kv_store(cache + j + half, y1);
                        }
                        uint64_t* nw = P.ll_kv + (kind == 1 ? 0 : kvd) + hd * D;
                        ll_store(nw + j, round_to(y0, KV()), tag);
                        ll_store(nw + j + half, round_to(y1, KV()), tag);
                    }
                }
                trace_detail(P, l, 0, 4);
                __syncthreads();
                trace_detail(P, l, 0, 5);
                if (tid == 0 && l + 1 < P.L) {
                    fence_proxy_async();
                    fill_slot(s_qkv, P.layers[l + 1].qkv + (size_t)qa * 2 * P.SH, (uint32_t)qn * 2 * P.SH, mb_qkv,
                              s_fills + 2);
                }
                trace_detail(P, l, 0, 6);
            }
        }
        trace_mark(P, 1, ph + 1);

        // ---- ATTN over positions 0..pos (src/kernels.cpp:150-179), then the
        // O projection (src/model.cpp:304) split over heads: the block that
        // finishes head h adds W_o[:, h*D .. h*D+D) times the head's output into
        // the O sums of layer l.
        if (has_att) {
            trace_mark(P, 0, ph + 2);
            const uint8_t* late = wo_early ? nullptr : wo_src;
            const bool att_ok =
                A.group   ? attention_group<KV>(P, A, ap, l, tag, s_att, mb_att, s_fills + MB_ATT, misc, xf, gpart, late,
                                                mb_wo, s_fills + 3, st)
                : D == 64 ? attention_block<KV, 64>(P, A, ap, l, tag, s_att, mb_att, s_fills + MB_ATT, misc, late,
                                                    mb_wo, s_fills + 3, st)
                          : attention_block<KV, 0>(P, A, ap, l, tag, s_att, mb_att, s_fills + MB_ATT, misc, late, mb_wo,
                                                   s_fills + 3, st);
            if (!att_ok) {
                ok = false;
                break;
            }
        }
        trace_mark(P, 1, ph + 2);
        if (o_head) {
            trace_mark(P, 0, ph + 3);
            trace_detail(P, l, 2, 0);
            if (tid >= D && tid < P.o_dw) misc[tid] = 0.f;  // the head's output, zero past D
            if (!mbar_wait(mb_wo, (uint32_t)l & 1u, st)) {
                ok = false;
                break;
            }
            trace_detail(P, l, 2, 1);
            slice_partial(s_att + P.wo_off, P.o_dw, H, misc, oscale, osum(l));
            trace_detail(P, l, 2, 2);
        }
        trace_mark(P, 1, ph + 3);

        // ---- gate/up + SiLU (src/model.cpp:305-308; x_b = x_a + O sums, kept raw
        // in xr by every block), then this block's share of down
        // (src/model.cpp:309-310): its columns of W_down times its own
        // SiLU(gate)*up values, for all H rows, into the down sums of layer l.
        // x entering layer l+1, and the final norm's input, is xr plus those sums.
        {
            trace_detail(P, l, 3, 0);
            float wsc = 1.f;
            const bool okw =
                warp_stage_sum(osum(l), (unsigned)P.NH, H, xr, xf, xq, QP, nch_h, post_norm, s_ss, wsc, st);
            trace_detail(P, l, 3, 1);
            if (gn) {
                trace_detail(P, l, 3, 2);
                const bool okg = okw && warp_slot_wait(mb_gu, (uint32_t)l & 1u, st);
                trace_mark(P, 0, ph + 4);
                trace_detail(P, l, 3, 3);
                block_gemv<1, 3>(s_gu, P.SH, 2 * gn, nch_h, xq, QP, gpart, wsc, okg);
                if (should_abort(st)) {
                    ok = false;
                    break;
                }
                if (tid < P.down_dw) {
                    float hv = 0.f;  // zero past this block's columns
                    if (tid < gn) {
                        const float inv = rms_inv(s_ss, H, P.eps);
                        const uint8_t* r0 = s_gu + (size_t)tid * 2 * P.SH;
                        const float g = gemv_row(gpart, 2 * gn, 2 * tid) * inv * row_scale(r0, P.Kh);
                        const float u = gemv_row(gpart, 2 * gn, 2 * tid + 1) * inv * row_scale(r0 + P.SH, P.Kh);
                        hv = (g / (1.0f + expf(-g))) * u;
                    }
                    s_h[tid] = hv;
                }
                trace_detail(P, l, 3, 4);
                __syncthreads();
                trace_detail(P, l, 3, 5);
                if (tid == 0) {
                    fence_proxy_async();
                    if (l + 1 < P.L)
                        fill_slot(s_gu, P.layers[l + 1].gu + (size_t)ga * 2 * P.SH, (uint32_t)gn * 2 * P.SH, mb_gu,
                                  s_fills + 0);
                }
                trace_detail(P, l, 3, 6);
            } else {
                __syncthreads();
                if (should_abort(st)) {
                    ok = false;
                    break;
                }
            }
        }
        trace_mark(P, 1, ph + 4);

        {
            trace_mark(P, 0, ph + 5);
            trace_detail(P, l, 4, 0);
            if (gn) {
                if (!mbar_wait(mb_down, (uint32_t)l & 1u, st)) {
                    ok = false;
                    break;
                }
                trace_detail(P, l, 4, 1);
                slice_partial(s_down, P.down_dw, H, s_h, dscale, dsum(l));
            }
            trace_detail(P, l, 4, 2);
            __syncthreads();  // the down slot is consumed
            if (tid == 0) {
                if (gn && l + 1 < P.L) {
                    fence_proxy_async();
                    fill_slot(s_down, P.down_cols + ((size_t)(l + 1) * G + b) * P.down_slice, (uint32_t)P.down_slice,
                              mb_down, s_fills + 1);
                }
            }
            trace_detail(P, l, 4, 3);
        }
        trace_mark(P, 1, ph + 5);
    }

    if (ok && A.head) {
        // ---- final RMSNorm + tied LM head + argmax (src/model.cpp:318-326, src/main.cpp:35-37)
        float best_v = -INFINITY;
        int best_i = 0x7fffffff;
        if (hn) {
            Staged sf{1.f, 1.f};
            if (!stage_sum(dsum(P.L - 1), dblocks, H, nch_h, xr, xf, xq, QP,
                           P.norms + (size_t)P.L * 2 * P.Kh, red, P.eps, sf, st))
                ok = false;
            const float inv = sf.inv * sf.scale;
            if (ok) {
                // The lane's activation chunks (lane + 32k) stay in registers.
                int4 xv[HEAD_MAXC][3];
#pragma unroll
                for (int k = 0; k < HEAD_MAXC; ++k) {
                    const int ch = lane + 32 * k;
                    if (ch < nch_h) {
                        load_planes(xq, QP, ch, xv[k][0], xv[k][1], xv[k][2]);
                    } else {
                        xv[k][0] = xv[k][1] = xv[k][2] = make_int4(0, 0, 0, 0);
                    }
                }
                trace_mark(P, 0, 5 * P.L + 1);
                // Each warp streams row groups of HEAD_R (groups warp, warp + NW,
                // ...) straight from HBM, with the next group's 16-byte chunks and
                // row scales in flight while the current group is reduced.
                const int ngroups = (hn + HEAD_R - 1) / HEAD_R;
                int4 wc[HEAD_R][HEAD_MAXC], wn[HEAD_R][HEAD_MAXC];
                float sc[HEAD_R], sn[HEAD_R];
                auto load_group = [&](int gi, int4 (&wv)[HEAD_R][HEAD_MAXC], float (&sv)[HEAD_R]) {
#pragma unroll
                    for (int rr = 0; rr < HEAD_R; ++rr) {
                        const int r = ha + gi * HEAD_R + rr;
                        const bool valid = r < ha + hn;
                        const uint8_t* row = P.embed + (size_t)(valid ? r : ha) * P.SH;
#pragma unroll
                        for (int k = 0; k < HEAD_MAXC; ++k) {
                            const int ch = lane + 32 * k;
                            wv[rr][k] = (valid && ch < nch_h) ? ld_stream(row + (size_t)ch * 16) : make_int4(0, 0, 0, 0);
                        }
                        sv[rr] = valid ? __ldg(reinterpret_cast<const float*>(row + P.Kh)) : 0.f;
                    }
                };
                if (warp < ngroups) load_group(warp, wc, sc);
                const int lines = (P.SH + 127) / 128;  // 128-byte lines per row
                for (int gi = warp; gi < ngroups; gi += NW) {
                    if (gi + NW < ngroups) load_group(gi + NW, wn, sn);
                    // The group after next into L2, one line per lane.
                    if (gi + 2 * NW < ngroups && lane < HEAD_R * lines) {
                        const int r = ha + (gi + 2 * NW) * HEAD_R + lane / lines;
                        if (r < ha + hn) prefetch_line_l2(P.embed + (size_t)r * P.SH + (size_t)(lane % lines) * 128);
                    }
                    float vmine = 0.f;  // lane rr keeps row rr's logit: one store per group
#pragma unroll
                    for (int rr = 0; rr < HEAD_R; ++rr) {
                        int ah = 0, am = 0, al = 0;
#pragma unroll
                        for (int k = 0; k < HEAD_MAXC; ++k) dp4a16(wc[rr][k], xv[k][0], xv[k][1], xv[k][2], ah, am, al);
                        const float d = warp_sum(planes_to_float(ah, am, al));
                        const int r = ha + gi * HEAD_R + rr;
                        if (r < ha + hn) {
                            const float v = d * sc[rr] * inv;
                            if (lane == rr) vmine = v;
                            if (better(v, r, best_v, best_i)) {
                                best_v = v;
                                best_i = r;
                            }
                        }
                    }
                    {
                        const int r = ha + gi * HEAD_R + lane;
                        if (lane < HEAD_R && r < ha + hn) {
                            P.logits[r] = vmine;
                            if (A.host_logits) A.host_logits[r] = vmine;
                        }
                    }
#pragma unroll
                    for (int rr = 0; rr < HEAD_R; ++rr) {
                        sc[rr] = sn[rr];
#pragma unroll
                        for (int k = 0; k < HEAD_MAXC; ++k) wc[rr][k] = wn[rr][k];
                    }
                }
                __syncthreads();
                if (should_abort(st)) ok = false;
            }
        }
        if (ok) {
            // Each warp's best is uniform across its lanes; merge the warps.
            if (lane == 0) {
                red[warp] = best_v;
                reinterpret_cast<int*>(red)[NW + warp] = best_i;
            }
            __syncthreads();
            if (tid == 0) {
                for (int w = 0; w < NW; ++w) {
                    const float v = red[w];
                    const int i = reinterpret_cast<const int*>(red)[NW + w];
                    if (better(v, i, best_v, best_i)) {
                        best_v = v;
                        best_i = i;
                    }
                }
                s_best = {best_v, best_i};
            }
            __syncthreads();
            grid_argmax<NT>(s_best, P.amax, P.sync, A.argmax_dev, reinterpret_cast<ArgBest*>(misc), &s_last);
        }
        trace_mark(P, 1, 5 * P.L + 1);
    }
    if (ok && tid == 0) {
        // Warm L2 with this block's first-layer rows for the next token.
        const LayerW& W0 = P.layers[0];
        if (qn) prefetch_l2(W0.qkv + (size_t)qa * 2 * P.SH, (uint32_t)qn * 2 * P.SH);
    }

    // Clear the other half of the down sums for the next step (this step's
    // half is cleared by the next one). Done on abort too.
    {
        uint64_t* z = P.dacc + (size_t)(A.par ^ 1) * P.L * 2 * P.Hp;
        const int n = P.L * 2 * P.Hp;
        for (int i = part_lo(b, G, n) + tid; i < part_lo(b + 1, G, n); i += NT) z[i] = 0ull;
    }

    // On abort, wait (bounded) for this block's copies in flight before the
    // shared memory they target is released.
    __syncthreads();
    if (!ok && tid == 0) {
        const uint64_t t0 = globaltimer();
        for (int i = 0; i < NMB; ++i) {
            // Fill number k completes phase k of its mbarrier (parity k & 1).
            if (!s_fills[i]) continue;
            const uint32_t parity = (s_fills[i] - 1) & 1u;
            while (!mbar_test(mb + i, parity) && globaltimer() - t0 < WAIT_LIMIT_NS) {
            }
        }
    }
    trace_mark(P, 0, 5 * P.L + 2);
    trace_mark(P, 1, 5 * P.L + 2);
    trace_clock(P, 1);
}

}  // namespace dcb
