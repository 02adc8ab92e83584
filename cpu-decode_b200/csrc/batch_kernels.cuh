// Batched decode of independent sequences on one GPU: one step advances every
// active sequence (slot) by one token. Per sequence it is the reference's
// Engine::Impl::step (src/model.cpp:258-329); batching is this project's own.
//
// With up to 64 sequences a projection is a GEMM, not a GEMV, so it runs on
// the 5th-generation tensor cores (tcgen05, kind::i8, accumulators in TMEM):
//   D[rows x 3*slots] = W[rows x K] (int8, the packed weight rows in place)
//                       * X[3*slots x K]^T (int8)
// where X holds every sequence's activation vector as the three byte planes of
// its 24-bit fixed-point form (q = hi*2^16 + mid*2^8 + lo, scale max|v|/FIX_MAX,
// the same staging as the batch-1 step kernel). The three int32 accumulators
// of (row, sequence) are exact; the epilogue folds them into one FP32 sum,
// scales by the row's and the sequence's scale and applies the fused
// operation of the projection (bias + RoPE + KV write, residual, SiLU*up, LM
// head + argmax).
//
// Both operands arrive by TMA (cp.async.bulk.tensor, 128-byte swizzle) into a
// 4-stage shared-memory ring; one thread issues the MMAs, one the loads, and
// every warp reads TMEM in the epilogue (16 warps, four per 32 TMEM lanes, each
// a share of the sequences). Every wait is bounded.
//
// Attention is split-KV over each sequence's own cache (head-major rows, one
// contiguous block per split), every staged K/V byte serving all query heads
// of its group; a combine kernel merges the splits of one sequence and stages
// the result for the O projection.
#pragma once
#include "attention.cuh"
#include "step_kernel.cuh"
#include "tcgen05.cuh"

#include <cuda.h>

#include <climits>

namespace dcb {
namespace batch {

constexpr int GM = 128;        // weight rows per GEMM tile (UMMA M)
constexpr int GK = 128;        // reduction bytes per pipeline stage (one 128-byte swizzle row)
constexpr int GSTAGES = 4;     // pipeline depth of the layer projections (one CTA per SM)
constexpr int HEAD_STAGES = 2; // LM head: two CTAs per SM, one's loads under the other's prologue and epilogue
constexpr int GT = 512;        // GEMM threads of a layer projection: 16 warps, four per 32 TMEM lanes
constexpr int GT_HEAD = 256;   // LM head: 8 warps, two per 32 TMEM lanes (two CTAs per SM)
constexpr int MAX_SLOTS = 64;  // sequences per batch: N = 3 * slots <= 192
constexpr uint32_t TMEM_COLS = 256;
constexpr int A_BYTES = GM * GK;  // 16 KB per stage
constexpr int ST_NT = 512;        // threads of the staging kernels
constexpr int ARG_NT = 256;       // threads of the argmax kernel

enum Epi { EPI_PLAIN = 0, EPI_QKV = 1, EPI_RESID = 2, EPI_GU = 3, EPI_HEAD = 4 };
template <int EPI>
__host__ __device__ constexpr int gemm_threads() {
    return EPI == EPI_HEAD ? GT_HEAD : GT;
}

__host__ __device__ constexpr int b_bytes(int slots) { return 3 * slots * GK; }
// Dynamic shared memory of the GEMM: 1 KB alignment slack, then the A and B rings.
__host__ __device__ constexpr int gemm_smem_bytes(int slots, int stages = GSTAGES) {
    return 1024 + stages * (A_BYTES + b_bytes(slots));
}

struct GemmArgs {
    int M;      // weight rows
    int nk;     // reduction stages (ceil(K / GK))
    int ksplit; // CTAs of a cluster sharing one row tile, each a slice of the stages (1 = no split)
    int nseq;   // active sequences (slots 0..nseq-1)
    int slots;  // sequence slots per plane (multiple of 16)
    const float* wscale;  // row r's scale at wscale[r * wstride]
    int wstride;
    const float* bias;  // row r's bias at bias[r * bstride], or null
    int bstride;
    const float* xsc;   // [slots] scale of each sequence's staged planes
    const float* xinv;  // [slots] RMSNorm factor of each sequence, or null
    float* out;         // PLAIN/HEAD: out[s*ldo + r]; RESID: out[s*ldo + r] += y; GU: out[s*ldo + r/2]; QKV: queries
    int ldo;
    // QKV: rows are RoPE pairs (j, j + D/2) of q heads, then k heads, then v heads
    int NH, NKV, D, L, layer, capacity, cached_rope;
    int kv_seq;  // 1: slot s owns cache s; 0: every slot is a position of one sequence (cache 0)
    const float* rope_inv;  // [D/2]
    const float* rope_den;  // [D/2]
    const int* pos;         // [slots] position of each sequence's new token
    const float2* rope;     // [slots][D/2] (cos, sin) of each sequence's position
    void* kcache;           // [slots or 1][L][NKV][capacity][D]
    void* vcache;
    ArgBest* amax;  // HEAD: [tiles][slots] best (value, row) of each tile and sequence
    int* kpart;     // split-K: [grid][3 * slots][GM] int32 partials, CTA-major
    int* err;       // set to ERR_WAIT when a wait runs out
    // Staging of the next projection's input once every tile is written (the
    // STAGE instantiation): a grid barrier (all CTAs co-resident), then CTA c
    // stages sequences c, c + grid, ... (RMSNorm factor, planes, scale).
    int* gbar;  // [2]: arrivals, generation
    const float* st_src;  // [slots][st_lds]
    int st_lds, st_n, st_kp;
    const float* st_gain;  // RMSNorm gains, or null
    int8_t* st_planes;     // [3][slots][st_kp]
    float* st_xsc;
    float* st_xinv;  // or null
    float st_eps;
};

// ---- tcgen05 / TMA primitives ------------------------------------------------------
// Shared-memory matrix descriptor of a K-major tile written by TMA with the
// 128-byte swizzle: rows of 128 bytes, 8-row atoms 1024 bytes apart (stride
// byte offset), version 1 (sm_100), layout type 2 (SWIZZLE_128B). The tile
// must be 1024-byte aligned. Moving along K inside the atom adds the byte
// offset to the start address (16-byte units).
__device__ __forceinline__ uint64_t sw128_desc(const void* tile) {
    const uint32_t a = smem_u32(tile);
    return (uint64_t)((a >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) | ((uint64_t)1 << 46) |
           ((uint64_t)2 << 61);
}
__device__ __forceinline__ void tma2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* m) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
            "r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(m))
        : "memory");
}
// Programmatic dependent launch: a kernel may start while its predecessor in
// the stream still runs; griddep_wait() returns once the predecessor has
// completed and its writes are visible. Work before it may only touch data
// that no kernel of the same step writes (weights, earlier steps' KV rows).
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
// Expected transaction bytes without an arrival (the phase cannot complete
// before the arrival that comes with the rest of the stage).
__device__ __forceinline__ void mbar_expect_tx(uint64_t* m, uint32_t bytes) {
    asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(m)), "r"(bytes) : "memory");
}
// Thread-block cluster: rank and barrier.
__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// One thread waits for phase `parity` of m, at most WAIT_LIMIT_NS.
static __device__ bool wait_phase(uint64_t* m, uint32_t parity, int* err) {
    uint64_t t0 = 0;
    unsigned spins = 0;
    while (!mbar_test(m, parity)) {
        if ((++spins & 63u) == 0) {
            const uint64_t now = globaltimer();
            if (!t0) {
                t0 = now;
            } else if (now - t0 > WAIT_LIMIT_NS) {
                atomicExch(err, ERR_WAIT);
                return false;
            }
        }
    }
    return true;
}

__device__ __forceinline__ void block_sum_max(float& ss, float& mx, float* red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        ss += __shfl_xor_sync(FULL, ss, o);
        mx = fmaxf(mx, __shfl_xor_sync(FULL, mx, o));
    }
    const int w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    __syncthreads();
    if ((threadIdx.x & 31) == 0) {
        red[w] = ss;
        red[32 + w] = mx;
    }
    __syncthreads();
    ss = 0.f;
    mx = 0.f;
    for (int i = 0; i < nw; ++i) {
        ss += red[i];
        mx = fmaxf(mx, red[32 + i]);
    }
}

__device__ __forceinline__ int ld_acquire_int(const int* p) {
    int v;
    asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_int(int* p, int v) {
    asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// Every CTA of the grid (all co-resident) arrives; the last one resets the
// count and publishes a new generation. Bounded: false when the wait ran out.
static __device__ bool grid_barrier(int* bar, int nblocks, int* err, int* s_flag) {
    __syncthreads();
    if (threadIdx.x == 0) {
        int ok = 1;
        const int gen = ld_acquire_int(bar + 1);
        __threadfence();  // this block's writes before its arrival
        if (atomicAdd(bar, 1) == nblocks - 1) {
            atomicExch(bar, 0);
            __threadfence();
            st_release_int(bar + 1, gen + 1);
        } else {
            uint64_t t0 = 0;
            unsigned spins = 0;
            while (ld_acquire_int(bar + 1) == gen) {
                if ((++spins & 63u) == 0) {
                    const uint64_t now = globaltimer();
                    if (!t0) {
                        t0 = now;
                    } else if (now - t0 > WAIT_LIMIT_NS) {
                        atomicExch(err, ERR_WAIT);
                        ok = 0;
                        break;
                    }
                }
            }
        }
        *s_flag = ok;
    }
    __syncthreads();
    return *s_flag != 0;
}

// The whole block stages sequence s: v = src[0..n) (read through L2), the
// RMSNorm factor of v (src/kernels.cpp:132-137), v*gain as planes.
static __device__ void stage_vec(const float* src, int n, int kp, const float* gain, float eps, int8_t* planes, int slots,
                          int s, float* xsc, float* xinv, float* buf, float* red) {
    float ss = 0.f, mx = 0.f;
    for (int j = threadIdx.x; j < n; j += blockDim.x) {
        const float v = __ldcg(src + j);
        ss = fmaf(v, v, ss);
        const float g = gain ? v * gain[j] : v;
        buf[j] = g;
        mx = fmaxf(mx, fabsf(g));
    }
    block_sum_max(ss, mx, red);
    const float rs = mx > 0.f ? FIX_MAX * __frcp_rn(mx) : 0.f;
    if (threadIdx.x == 0) {
        xsc[s] = mx > 0.f ? __frcp_rn(rs) : 1.0f;
        if (xinv) xinv[s] = __frsqrt_rn(ss / (float)n + eps);
    }
    int8_t* ph = planes + (size_t)s * kp;
    int8_t* pm = ph + (size_t)slots * kp;
    int8_t* pl = pm + (size_t)slots * kp;
    for (int quad = threadIdx.x; quad < kp / 4; quad += blockDim.x) {
        const int j = 4 * quad;
        const float4 v4 = make_float4(j < n ? buf[j] : 0.f, j + 1 < n ? buf[j + 1] : 0.f, j + 2 < n ? buf[j + 2] : 0.f,
                                      j + 3 < n ? buf[j + 3] : 0.f);
        uint32_t h, m, l;
        fix_pack4(v4, rs, h, m, l);
        reinterpret_cast<uint32_t*>(ph)[quad] = h;
        reinterpret_cast<uint32_t*>(pm)[quad] = m;
        reinterpret_cast<uint32_t*>(pl)[quad] = l;
    }
    __syncthreads();  // buf and red are reused by the next sequence
}

// Order-preserving integer key of a logit for a warp max (redux.sync): finite
// values and infinities in float order, -0 equal to +0, NaN below everything
// (a NaN is never the better candidate, as in better()).
__device__ __forceinline__ int argmax_key(float v) {
    if (v != v) return INT_MIN;
    const int b = __float_as_int(v + 0.0f);
    return b >= 0 ? b : b ^ 0x7fffffff;
}
__device__ __forceinline__ float argmax_key_value(int k) { return __int_as_float(k >= 0 ? k : k ^ 0x7fffffff); }

// ---- the GEMM ----------------------------------------------------------------------
template <int EPI, typename KV, int GSTAGES, bool STAGE = false>
__global__ void __launch_bounds__(gemm_threads<EPI>(), 1)
    gemm_i8_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, const GemmArgs a) {
    constexpr int NTH = gemm_threads<EPI>();
    constexpr int NWG = NTH / 128;  // warps per 32 TMEM lanes
    extern __shared__ uint8_t g_sm_raw[];
    uint8_t* g_sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(g_sm_raw) + 1023) & ~uintptr_t(1023));
    const int BB = b_bytes(a.slots), N = 3 * a.slots;
    uint8_t* sA = g_sm;
    uint8_t* sB = g_sm + GSTAGES * A_BYTES;
    __shared__ __align__(8) uint64_t full[GSTAGES], empty[GSTAGES], done;
    __shared__ uint32_t s_tmem;
    __shared__ float s_xsc[MAX_SLOTS], s_xinv[MAX_SLOTS];
    __shared__ float s_bv[4][MAX_SLOTS];
    __shared__ int s_bi[4][MAX_SLOTS];
    __shared__ int s_pos[MAX_SLOTS];
    __shared__ int s_flag;
    __shared__ float s_red[64];

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // Epilogue: warp w reads TMEM lanes 32*(w % 4).. (weight rows) and takes
    // every NWG-th group of 4 sequences from group w / 4 on.
    const int quad = warp & 3, wg = warp >> 2;
    // Split-K: the S CTAs of a cluster share row tile blockIdx.x / S; rank r
    // takes stages [r*nk/S, (r+1)*nk/S) and, after the exact integer sums
    // over the cluster, sequences [r*per, (r+1)*per) of the epilogue (per a
    // multiple of 4).
    const int S = a.ksplit;
    const int rank = S > 1 ? (int)cluster_rank() : 0;
    const int m0 = (blockIdx.x / S) * GM;
    const int kb = rank * a.nk / S, nkl = (rank + 1) * a.nk / S - kb;
    const int per = ((a.slots + S - 1) / S + 3) & ~3;
    const int s_first = rank * per, s_last = min(a.nseq, s_first + per);
    // This thread's weight row, its scale and bias: weights, which no kernel
    // of the step writes, so they load before the wait for the previous one.
    const int r = m0 + 32 * quad + lane;
    const bool rv = r < a.M;
    const float wsc = rv ? __ldg(a.wscale + (size_t)r * a.wstride) : 0.f;
    const float bia = (rv && a.bias) ? __ldg(a.bias + (size_t)r * a.bstride) : 0.f;

    if (tid == 0) {
        for (int s = 0; s < GSTAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(&done, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmA)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmB)) : "memory");
    }
    if (warp == 2) {
        tmem_alloc(&s_tmem, TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_tmem;
    griddep_launch_dependents();

    if (warp == 0) {
        if (lane == 0) {
            // Producer. The first stages' weight tiles do not depend on the
            // previous kernel: they are requested before waiting for it.
            const int npre = min(GSTAGES, nkl);
            for (int i = 0; i < npre; ++i) {
                mbar_expect_tx(&full[i], A_BYTES);
                tma2d(sA + i * A_BYTES, &tmA, (kb + i) * GK, m0, &full[i]);
            }
            griddep_wait();
            for (int i = 0; i < npre; ++i) {
                mbar_expect(&full[i], (uint32_t)BB);
                tma2d(sB + i * BB, &tmB, (kb + i) * GK, 0, &full[i]);
            }
            const uint32_t bytes = (uint32_t)(A_BYTES + BB);
            for (int i = npre; i < nkl; ++i) {
                const int s = i % GSTAGES;
                if (!wait_phase(&empty[s], (uint32_t)((i / GSTAGES) - 1) & 1u, a.err)) break;
                mbar_expect(&full[s], bytes);
                tma2d(sA + s * A_BYTES, &tmA, (kb + i) * GK, m0, &full[s]);
                tma2d(sB + s * BB, &tmB, (kb + i) * GK, 0, &full[s]);
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0) {
            // MMA issuer: 4 MMAs of K = 32 per stage, accumulating in TMEM.
            const uint32_t idesc = idesc_i8(GM, N);
            for (int i = 0; i < nkl; ++i) {
                const int s = i % GSTAGES;
                if (!wait_phase(&full[s], (uint32_t)(i / GSTAGES) & 1u, a.err)) break;
                tc_fence_after();
                const uint64_t da = sw128_desc(sA + s * A_BYTES), db = sw128_desc(sB + s * BB);
#pragma unroll
                for (int kk = 0; kk < GK / 32; ++kk)
                    umma_i8(tmem, da + 2 * kk, db + 2 * kk, idesc, (i | kk) != 0 ? 1u : 0u);
                umma_commit(&empty[s]);
            }
            umma_commit(&done);
        }
        __syncwarp();
    }
    griddep_wait();
    for (int s = tid; s < a.slots; s += NTH) {
        s_xsc[s] = s < a.nseq ? a.xsc[s] : 0.f;
        s_xinv[s] = (a.xinv && s < a.nseq) ? a.xinv[s] : 1.f;
        if (EPI == EPI_QKV) s_pos[s] = s < a.nseq ? a.pos[s] : 0;
    }
    if (tid == 0) {
        wait_phase(&done, 0, a.err);
        // Every load issued must have landed before the block may exit (only
        // relevant after an expired wait; otherwise these phases are complete).
        for (int s = 0; s < GSTAGES && s < nkl; ++s) {
            const int last = s + ((nkl - 1 - s) / GSTAGES) * GSTAGES;  // last local stage using slot s
            wait_phase(&full[s], (uint32_t)(last / GSTAGES) & 1u, a.err);
        }
    }
    __syncthreads();
    tc_fence_after();

    const uint32_t trow = tmem + ((uint32_t)(32 * quad) << 16);
    // Split-K: this CTA's int32 partials (all N columns) to its block of the
    // L2 scratch, column-major (a warp's 32 rows of one column are 128
    // contiguous bytes), then visible to the cluster. Warp (quad, wg) moves
    // the 4-column groups wg, wg + NWG, ... of its 32 rows.
    const int* kpart_tile = a.kpart + (size_t)(blockIdx.x - rank) * N * GM + 32 * quad + lane;
    if (S > 1) {
        int* mine = a.kpart + (size_t)blockIdx.x * N * GM + 32 * quad + lane;
        for (int c0 = 4 * wg; c0 < N; c0 += 16 * NWG) {
            uint32_t v[4][4];
#pragma unroll
            for (int u = 0; u < 4; ++u)
                if (c0 + 4 * NWG * u < N) tmem_ld4(trow + (uint32_t)(c0 + 4 * NWG * u), v[u]);
            tmem_wait_ld();
#pragma unroll
            for (int u = 0; u < 4; ++u)
                if (c0 + 4 * NWG * u < N)
#pragma unroll
                    for (int k = 0; k < 4; ++k) __stcg(mine + (size_t)(c0 + 4 * NWG * u + k) * GM, (int)v[u][k]);
        }
        cluster_sync();
    }

    // ---- epilogue: thread = weight row r, 4 sequences at a time. Every
    // global value a group needs is loaded before its stores, so the loads of
    // a group are in flight together.
    float* __restrict__ out = a.out;
    // QKV: this row's RoPE pair index and frequency (src/model.cpp:222-224,269-274).
    int q_kind = 0, q_hd = 0, q_j = 0;
    if (EPI == EPI_QKV && rv) {
        const int half = a.D >> 1, u = r >> 1;
        const int qpairs = a.NH * half, kpairs = a.NKV * half;
        q_kind = u < qpairs ? 0 : (u < qpairs + kpairs ? 1 : 2);
        const int pu = q_kind == 0 ? u : (q_kind == 1 ? u - qpairs : u - qpairs - kpairs);
        q_hd = pu / half;
        q_j = pu - q_hd * half;
    }
    for (int s0 = s_first + 4 * wg; s0 < s_last; s0 += 4 * NWG) {
        uint32_t hi[4], md[4], lo[4];
        if (S == 1) {
            tmem_ld4(trow + (uint32_t)s0, hi);
            tmem_ld4(trow + (uint32_t)(a.slots + s0), md);
            tmem_ld4(trow + (uint32_t)(2 * a.slots + s0), lo);
        } else {
            // Exact sums of the cluster's partials (integers: any order).
#pragma unroll
            for (int i = 0; i < 4; ++i) hi[i] = md[i] = lo[i] = 0u;
#pragma unroll 2
            for (int q = 0; q < S; ++q) {
                const int* pq = kpart_tile + (size_t)q * N * GM;
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    hi[i] += (uint32_t)__ldcg(pq + (size_t)(s0 + i) * GM);
                    md[i] += (uint32_t)__ldcg(pq + (size_t)(a.slots + s0 + i) * GM);
                    lo[i] += (uint32_t)__ldcg(pq + (size_t)(2 * a.slots + s0 + i) * GM);
                }
            }
        }
        float xo[4];
        float2 cs4[4];
        if (EPI == EPI_RESID) {
#pragma unroll
            for (int i = 0; i < 4; ++i) xo[i] = (rv && s0 + i < s_last) ? out[(size_t)(s0 + i) * a.ldo + r] : 0.f;
        }
        if (EPI == EPI_QKV) {
#pragma unroll
            for (int i = 0; i < 4; ++i)
                cs4[i] = (rv && q_kind < 2 && s0 + i < s_last) ? a.rope[(size_t)(s0 + i) * (a.D >> 1) + q_j]
                                                               : make_float2(1.f, 0.f);
        }
        if (S == 1) tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int s = s0 + i;
            const bool sv = s < s_last;
            const int si = sv ? s : 0;
            const float acc = planes_to_float((int)hi[i], (int)md[i], (int)lo[i]);
            float y = acc * s_xsc[si] * s_xinv[si] * wsc + bia;
            if (EPI == EPI_PLAIN) {
                if (rv && sv) out[(size_t)s * a.ldo + r] = y;
            } else if (EPI == EPI_RESID) {
                if (rv && sv) out[(size_t)s * a.ldo + r] = xo[i] + y;
            } else if (EPI == EPI_GU) {
                // rows (2j, 2j+1) = (gate_j, up_j) in adjacent lanes (src/model.cpp:306-308)
                const float u = __shfl_xor_sync(FULL, y, 1);
                if (rv && sv && !(lane & 1)) out[(size_t)s * a.ldo + (r >> 1)] = (y / (1.0f + expf(-y))) * u;
            } else if (EPI == EPI_QKV) {
                // rows (2u, 2u+1) = (j, j + D/2) of one head in adjacent lanes (src/model.cpp:277-302)
                const float other = __shfl_xor_sync(FULL, y, 1);
                if (rv && sv) {
                    const int half = a.D >> 1;
                    const bool second = lane & 1;
                    const float y0 = second ? other : y, y1 = second ? y : other;
                    float val = second ? y1 : y0;
                    const int p = s_pos[si];
                    if (q_kind < 2) {
                        const float cs = cs4[i].x, sn = cs4[i].y;
                        val = second ? __fadd_rn(__fmul_rn(y1, cs), __fmul_rn(y0, sn))
                                     : __fsub_rn(__fmul_rn(y0, cs), __fmul_rn(y1, sn));
                    }
                    const int idx = q_j + (second ? half : 0);
                    if (q_kind == 0) {
                        out[(size_t)s * a.ldo + q_hd * a.D + idx] = val;
                    } else {
                        KV* cache = static_cast<KV*>(q_kind == 1 ? a.kcache : a.vcache) +
                                    ((((size_t)s * a.kv_seq * a.L + a.layer) * a.NKV + q_hd) * a.capacity + p) * a.D;
                        kv_store(cache + idx, val);
                    }
                }
            } else if (EPI == EPI_HEAD) {
                if (rv && sv && out) out[(size_t)s * a.ldo + r] = y;
                // The warp's best row for sequence s: the largest key, then the
                // lowest lane holding it (rows ascend with the lane: the first
                // maximum, src/main.cpp:35-37).
                const int key = argmax_key((rv && sv) ? y : -INFINITY);
                const int kmax = __reduce_max_sync(FULL, key);
                const unsigned hit = __ballot_sync(FULL, key == kmax);
                if (lane == 0 && sv) {
                    s_bv[quad][s] = argmax_key_value(kmax);
                    s_bi[quad][s] = m0 + 32 * quad + __ffs(hit) - 1;
                }
            }
        }
    }
    if (EPI == EPI_HEAD) {
        __syncthreads();
        if (tid < a.nseq) {
            float v = s_bv[0][tid];
            int vi = s_bi[0][tid];
            for (int w = 1; w < 4; ++w)
                if (better(s_bv[w][tid], s_bi[w][tid], v, vi)) {
                    v = s_bv[w][tid];
                    vi = s_bi[w][tid];
                }
            a.amax[(size_t)blockIdx.x * a.slots + tid] = {v, vi};
        }
    }
    if (STAGE && grid_barrier(a.gbar, gridDim.x, a.err, &s_flag)) {
        float* buf = reinterpret_cast<float*>(g_sm);
        for (int s = blockIdx.x; s < a.nseq; s += gridDim.x)
            stage_vec(a.st_src + (size_t)s * a.st_lds, a.st_n, a.st_kp, a.st_gain, a.st_eps, a.st_planes, a.slots, s,
                      a.st_xsc, a.st_xinv, buf, s_red);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 2) {
        tc_fence_after();
        tmem_dealloc(tmem, TMEM_COLS);
    }
}

// ---- the LM head: persistent -------------------------------------------------------
// One CTA per SM works through row tiles blockIdx.x, + gridDim.x, ... of the
// tied head, its loads one stream of (weight tile from HBM, plane tile from
// L2) stages through a 5-slot ring, so 80 KB of weights are in flight per SM.
// Two TMEM accumulators (columns 0 and 256) alternate between tiles: the
// epilogue of one tile (argmax candidates, optional logits) runs under the
// MMAs of the next. Warps: 0 loads, 1 issues the MMAs, 2 owns TMEM, 4..19 read
// TMEM (four per 32 lanes, every fourth group of 4 sequences).
constexpr int HB_A = 5;     // stages in the ring
constexpr int HB_NT = 640;  // threads
constexpr int HB_EW = 16;   // epilogue warps (4..19)
__host__ __device__ constexpr int head_smem_bytes(int slots) { return 1024 + HB_A * (A_BYTES + b_bytes(slots)); }

__global__ void __launch_bounds__(HB_NT, 1)
    head_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, const GemmArgs a) {
    extern __shared__ uint8_t hb_raw[];
    uint8_t* hm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(hb_raw) + 1023) & ~uintptr_t(1023));
    const int BB = b_bytes(a.slots), N = 3 * a.slots, nk = a.nk;
    uint8_t* sA = hm;                   // HB_A weight tiles
    uint8_t* sB = hm + HB_A * A_BYTES;  // HB_A plane tiles (BB is a multiple of 1024)
    __shared__ __align__(8) uint64_t full[HB_A], empty[HB_A], accf[2], acce[2];
    __shared__ uint32_t s_tmem;
    __shared__ float s_xsc[MAX_SLOTS], s_xinv[MAX_SLOTS];
    __shared__ float s_bv[4][MAX_SLOTS];
    __shared__ int s_bi[4][MAX_SLOTS];
    __shared__ int s_abort;  // an epilogue wait ran out: the epilogue warps skip the remaining tiles' work
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int ntiles = (a.M + GM - 1) / GM;
    const int my = (int)blockIdx.x < ntiles ? (ntiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
    const int total = my * nk;

    if (tid == 0) {
        s_abort = 0;
        for (int s = 0; s < HB_A; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int s = 0; s < 2; ++s) {
            mbar_init(&accf[s], 1);
            mbar_init(&acce[s], HB_EW);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmA)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmB)) : "memory");
    }
    if (warp == 2) {
        tmem_alloc(&s_tmem, 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_tmem;
    griddep_launch_dependents();

    int issued = 0;  // thread 0: weight tiles requested
    if (warp == 0) {
        if (lane == 0) {
            // Weight tiles do not depend on the previous kernel: the first
            // ones are requested before waiting for it.
            const int npre = min(HB_A, total);
            for (int g = 0; g < npre; ++g) {
                const int m0 = ((int)blockIdx.x + (g / nk) * (int)gridDim.x) * GM;
                mbar_expect_tx(&full[g], A_BYTES);
                tma2d(sA + g * A_BYTES, &tmA, (g % nk) * GK, m0, &full[g]);
            }
            issued = npre;
            griddep_wait();
            for (int g = 0; g < npre; ++g) {
                mbar_expect(&full[g], (uint32_t)BB);
                tma2d(sB + g * BB, &tmB, (g % nk) * GK, 0, &full[g]);
            }
            for (int g = npre; g < total; ++g) {
                const int slot = g % HB_A;
                if (!wait_phase(&empty[slot], (uint32_t)((g / HB_A) - 1) & 1u, a.err)) break;
                const int m0 = ((int)blockIdx.x + (g / nk) * (int)gridDim.x) * GM;
                mbar_expect(&full[slot], (uint32_t)(A_BYTES + BB));
                tma2d(sA + slot * A_BYTES, &tmA, (g % nk) * GK, m0, &full[slot]);
                tma2d(sB + slot * BB, &tmB, (g % nk) * GK, 0, &full[slot]);
                issued = g + 1;
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0 && my > 0) {
            const uint32_t idesc = idesc_i8(GM, N);
            bool ok = true;
            for (int j = 0; ok && j < my; ++j) {
                const int acc = j & 1;
                if (j >= 2 && !(ok = wait_phase(&acce[acc], (uint32_t)((j >> 1) - 1) & 1u, a.err))) break;
                tc_fence_after();
                const uint32_t td = tmem + (uint32_t)(acc * 256);
                for (int k = 0; k < nk; ++k) {
                    const int g = j * nk + k, slot = g % HB_A;
                    if (!(ok = wait_phase(&full[slot], (uint32_t)(g / HB_A) & 1u, a.err))) break;
                    tc_fence_after();
                    const uint64_t da = sw128_desc(sA + slot * A_BYTES), db = sw128_desc(sB + slot * BB);
#pragma unroll
                    for (int kk = 0; kk < GK / 32; ++kk)
                        umma_i8(td, da + 2 * kk, db + 2 * kk, idesc, (k | kk) != 0 ? 1u : 0u);
                    umma_commit(&empty[slot]);
                }
                if (ok) umma_commit(&accf[acc]);
            }
        }
        __syncwarp();
    } else if (warp >= 4) {
        const int ew = warp - 4, quad = warp & 3, wg = ew >> 2;
        griddep_wait();
        for (int s = ew * 32 + lane; s < a.slots; s += HB_EW * 32) {
            s_xsc[s] = s < a.nseq ? a.xsc[s] : 0.f;
            s_xinv[s] = (a.xinv && s < a.nseq) ? a.xinv[s] : 1.f;
        }
        asm volatile("bar.sync 1, %0;" ::"r"(HB_EW * 32) : "memory");
        float* __restrict__ out = a.out;
        // Row scales one tile ahead (they sit in the weight rows, in HBM).
        auto row_scale = [&](int j) {
            const int r = ((int)blockIdx.x + j * (int)gridDim.x) * GM + 32 * quad + lane;
            return r < a.M ? __ldg(a.wscale + (size_t)r * a.wstride) : 0.f;
        };
        float wsc_next = my > 0 ? row_scale(0) : 0.f;
        for (int j = 0; j < my; ++j) {
            const int acc = j & 1, tile = (int)blockIdx.x + j * (int)gridDim.x, m0 = tile * GM;
            const int r = m0 + 32 * quad + lane;
            const bool rv = r < a.M;
            const float wsc = wsc_next;
            if (j + 1 < my) wsc_next = row_scale(j + 1);
            // Every epilogue warp takes the same barrier steps for every
            // tile, also after a wait ran out (then without the work).
            int ok = 1;
            if (lane == 0) {
                ok = !*reinterpret_cast<volatile int*>(&s_abort) &&
                     wait_phase(&accf[acc], (uint32_t)(j >> 1) & 1u, a.err);
                if (!ok) atomicExch(&s_abort, 1);
            }
            ok = __shfl_sync(FULL, ok, 0);
            tc_fence_after();
            const uint32_t trow = tmem + (uint32_t)(acc * 256) + ((uint32_t)(32 * quad) << 16);
            for (int s0 = 4 * wg; ok && s0 < a.nseq; s0 += 4 * (HB_EW / 4)) {
                uint32_t hi[4], md[4], lo[4];
                tmem_ld4(trow + (uint32_t)s0, hi);
                tmem_ld4(trow + (uint32_t)(a.slots + s0), md);
                tmem_ld4(trow + (uint32_t)(2 * a.slots + s0), lo);
                tmem_wait_ld();
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int s = s0 + i;
                    const bool sv = s < a.nseq;
                    const int si = sv ? s : 0;
                    const float y = planes_to_float((int)hi[i], (int)md[i], (int)lo[i]) * s_xsc[si] * s_xinv[si] * wsc + 0.f;
                    if (rv && sv && out) out[(size_t)s * a.ldo + r] = y;
                    // The warp's best row for sequence s (first maximum, src/main.cpp:35-37).
                    const int key = argmax_key((rv && sv) ? y : -INFINITY);
                    const int kmax = __reduce_max_sync(FULL, key);
                    const unsigned hit = __ballot_sync(FULL, key == kmax);
                    if (lane == 0 && sv) {
                        s_bv[quad][s] = argmax_key_value(kmax);
                        s_bi[quad][s] = m0 + 32 * quad + __ffs(hit) - 1;
                    }
                }
            }
            // The accumulator is read: the MMAs of tile j + 2 may reuse it.
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acce[acc]);
            asm volatile("bar.sync 1, %0;" ::"r"(HB_EW * 32) : "memory");
            for (int t = ew * 32 + lane; t < a.nseq; t += HB_EW * 32) {
                float v = s_bv[0][t];
                int vi = s_bi[0][t];
                for (int w = 1; w < 4; ++w)
                    if (better(s_bv[w][t], s_bi[w][t], v, vi)) {
                        v = s_bv[w][t];
                        vi = s_bi[w][t];
                    }
                a.amax[(size_t)tile * a.slots + t] = {v, vi};
            }
            asm volatile("bar.sync 1, %0;" ::"r"(HB_EW * 32) : "memory");
        }
    }
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
        // Every load issued must land before the block exits (only relevant
        // after an expired wait; otherwise these phases are complete).
        for (int s = 0; s < HB_A && s < issued; ++s) {
            const int last = s + ((issued - 1 - s) / HB_A) * HB_A;
            wait_phase(&full[s], (uint32_t)(last / HB_A) & 1u, a.err);
        }
    }
    __syncthreads();
    if (warp == 2) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

// ---- staging: RMSNorm factor and fixed-point planes of one vector per sequence -----
struct StageArgs {
    int n;           // vector length
    int kp;          // bytes per plane row (>= n, multiple of 16; zero padded)
    int slots, nseq;
    const float* src;  // [slots][lds] input vectors, or null with `embed`
    int lds;
    const uint8_t* embed;  // packed embedding rows (stride SE, FP32 scale at byte eoff) read for tokens[s]
    int SE, eoff, vocab;
    const int* tokens;
    float* x_out;        // embed mode: the embedded vector is written here ([slots][lds])
    const float* gain;   // RMSNorm gains (folded into the staged values), or null
    float eps;
    int8_t* planes;      // [3][slots][kp]
    float* xsc;          // [slots]
    float* xinv;         // [slots] RMSNorm factor (null: not a normalised input)
    int* err;
    // embed mode: each sequence's RoPE (cos, sin) table for this step
    const int* pos;
    const float* rope_inv;  // [D/2] (cached angle formula) or
    const float* rope_den;  // [D/2] (direct formula)
    int cached_rope, half;
    float2* rope;           // [slots][half]
};

// One block per sequence: v (embedded token row or src), sum v^2 for the
// RMSNorm factor (src/kernels.cpp:132-137), v*gain quantised into the planes.
__global__ void __launch_bounds__(ST_NT) stage_kernel(const StageArgs a) {
    extern __shared__ float st_v[];  // [n] gained values
    __shared__ float red[64];
    griddep_launch_dependents();
    griddep_wait();
    const int s = blockIdx.x;
    if (s >= a.nseq) return;
    const uint8_t* row = nullptr;
    float rsc = 0.f;
    if (a.embed && a.rope && threadIdx.x < a.half) {
        // RoPE angles of this sequence's position (src/model.cpp:269-274), once per step.
        const int j = threadIdx.x;
        const float p = (float)a.pos[s];
        const float angle = a.cached_rope ? __fmul_rn(p, a.rope_inv[j]) : __fdiv_rn(p, a.rope_den[j]);
        float sn, cs;
        sincosf(angle, &sn, &cs);
        a.rope[(size_t)s * a.half + j] = make_float2(cs, sn);
    }
    if (a.embed) {
        int t = a.tokens[s];
        if ((unsigned)t >= (unsigned)a.vocab) {  // a device-supplied token out of range (src/model.cpp:259)
            if (threadIdx.x == 0) atomicCAS(a.err, 0, ERR_TOKEN);
            t = 0;
        }
        row = a.embed + (size_t)t * a.SE;
        rsc = *reinterpret_cast<const float*>(row + a.eoff);
    }
    float ss = 0.f, mx = 0.f;
    if (!row && !(a.n & 3) && !(a.lds & 3)) {
        // Rows of the previous projection: four values per load.
        const float4* src4 = reinterpret_cast<const float4*>(a.src + (size_t)s * a.lds);
        const float4* gain4 = reinterpret_cast<const float4*>(a.gain);
        for (int q = threadIdx.x; q < a.n / 4; q += ST_NT) {
            const float4 v = src4[q];
            ss = fmaf(v.x, v.x, ss);
            ss = fmaf(v.y, v.y, ss);
            ss = fmaf(v.z, v.z, ss);
            ss = fmaf(v.w, v.w, ss);
            float4 g = v;
            if (gain4) {
                const float4 w = gain4[q];
                g = make_float4(v.x * w.x, v.y * w.y, v.z * w.z, v.w * w.w);
            }
            reinterpret_cast<float4*>(st_v)[q] = g;
            mx = fmaxf(mx, fmaxf(fmaxf(fabsf(g.x), fabsf(g.y)), fmaxf(fabsf(g.z), fabsf(g.w))));
        }
    } else {
        for (int j = threadIdx.x; j < a.n; j += ST_NT) {
            float v;
            if (row) {
                v = (float)(int8_t)row[j] * rsc;
                a.x_out[(size_t)s * a.lds + j] = v;
            } else {
                v = a.src[(size_t)s * a.lds + j];
            }
            ss = fmaf(v, v, ss);
            const float g = a.gain ? v * a.gain[j] : v;
            st_v[j] = g;
            mx = fmaxf(mx, fabsf(g));
        }
    }
    block_sum_max(ss, mx, red);
    const float rs = mx > 0.f ? FIX_MAX * __frcp_rn(mx) : 0.f;
    if (threadIdx.x == 0) {
        a.xsc[s] = mx > 0.f ? __frcp_rn(rs) : 1.0f;
        if (a.xinv) a.xinv[s] = __frsqrt_rn(ss / (float)a.n + a.eps);
    }
    int8_t* ph = a.planes + (size_t)s * a.kp;
    int8_t* pm = ph + (size_t)a.slots * a.kp;
    int8_t* pl = pm + (size_t)a.slots * a.kp;
    for (int quad = threadIdx.x; quad < a.kp / 4; quad += ST_NT) {
        const int j = 4 * quad;
        const float4 v4 = j + 3 < a.n ? reinterpret_cast<const float4*>(st_v)[quad]
                                      : make_float4(j < a.n ? st_v[j] : 0.f, j + 1 < a.n ? st_v[j + 1] : 0.f,
                                                    j + 2 < a.n ? st_v[j + 2] : 0.f, j + 3 < a.n ? st_v[j + 3] : 0.f);
        uint32_t h, m, l;
        fix_pack4(v4, rs, h, m, l);
        reinterpret_cast<uint32_t*>(ph)[quad] = h;
        reinterpret_cast<uint32_t*>(pm)[quad] = m;
        reinterpret_cast<uint32_t*>(pl)[quad] = l;
    }
}

// ---- attention ---------------------------------------------------------------------
struct AttnArgs {
    const float* q;  // [slots][NH*D] rotated queries
    const void* kcache;  // [slots or 1][L][NKV][capacity][D]
    const void* vcache;
    float* part;  // [slots][NH][max_splits][D+2]: (max, sum, unnormalised output) of each split
    const int* pos;
    int NH, NKV, D, L, layer, capacity, split_len, max_splits;
    int kv_seq;  // as GemmArgs::kv_seq
};

// Block (split, kv head g, sequence s): positions [split*split_len, ...) up to
// pos[s] (inclusive) of sequence s, all query heads of group g.
template <typename KV, int DT>
__global__ void __launch_bounds__(AT_NT) attention_kernel(const AttnArgs a) {
    extern __shared__ __align__(16) unsigned char at_sm[];
    griddep_launch_dependents();
    griddep_wait();
    const int sp = blockIdx.x, g = blockIdx.y, s = blockIdx.z;
    const int D = DT ? DT : a.D;
    const int length = a.pos[s] + 1;
    const int t0 = sp * a.split_len;
    if (t0 >= length) return;
    const int t1 = min(length, t0 + a.split_len);
    const int gq = a.NH / a.NKV;
    const size_t head = (((size_t)s * a.kv_seq * a.L + a.layer) * a.NKV + g) * (size_t)a.capacity * D;
    const KV* kg = static_cast<const KV*>(a.kcache) + head;
    const KV* vg = static_cast<const KV*>(a.vcache) + head;
    float* sq = reinterpret_cast<float*>(at_sm + 2 * 2 * (size_t)AT_T * D * sizeof(KV));
    const float qscale = 1.4426950408889634f / sqrtf((float)D);
    const float* qs = a.q + ((size_t)s * a.NH + (size_t)g * gq) * D;
    for (int e = threadIdx.x; e < gq * D; e += AT_NT) sq[e] = qs[e] * qscale;
    float* part = a.part + (((size_t)s * a.NH + (size_t)g * gq) * a.max_splits + sp) * (D + 2);
    const size_t hstride = (size_t)a.max_splits * (D + 2);
    attention_split_body<KV, DT>(at_sm, kg, vg, D, D, t0, t1, gq, [&](int hl, int j, float M, float L, float acc) {
        float* pp = part + (size_t)hl * hstride;
        if (j == 0) {
            pp[0] = M;
            pp[1] = L;
        }
        pp[2 + j] = acc;
    });
}

// Merge the splits of every head of sequence s (in split order) and stage the
// attention output (NH*D values) as planes for the O projection. Run by one
// whole block; partials are read through L2 (other blocks of the same kernel
// may have written them). smem: (NH*D + 2*NH*max_splits) floats; red: 64 floats.
struct CombineArgs {
    const float* part;
    const int* pos;
    int NH, D, split_len, max_splits, slots, kp;
    int8_t* planes;  // [3][slots][kp]
    float* xsc;
};
constexpr int CB_SPL = 12;  // splits whose values one warp requests at once
static __device__ __noinline__ void combine_seq(const CombineArgs& a, int s, float* cb_sm, float* red) {
    const int n = a.NH * a.D, D = a.D, W = D + 2;
    float* outv = cb_sm;
    float* wts = cb_sm + n;
    float* lsp = wts + a.NH * a.max_splits;  // [NH][max_splits] the splits' sums
    const int ns = (a.pos[s] + a.split_len) / a.split_len;  // splits covering positions 0..pos
    const float* base = a.part + (size_t)s * a.NH * a.max_splits * W;
    const int nt = blockDim.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = nt / 32;
    float mx = 0.f, ss = 0.f;
    // Warp per head: weight of split i = 2^(m_i - M) / sum_i 2^(m_i - M) l_i
    // (lanes over splits), then lanes over dimensions j = lane + 32k with the
    // loads of CB_SPL splits in flight, summed in split order.
    for (int h = warp; h < a.NH; h += nw) {
        const float* hb = base + (size_t)h * a.max_splits * W;
        float* hw = wts + h * a.max_splits;
        float* hl = lsp + h * a.max_splits;
        float M = -INFINITY;
        for (int i = lane; i < ns; i += 32) {  // (m_i, l_i) requested together, once
            const float mi = __ldcg(hb + (size_t)i * W), li = __ldcg(hb + (size_t)i * W + 1);
            hw[i] = mi;
            hl[i] = li;
            M = fmaxf(M, mi);
        }
        M = warp_max(M);
        __syncwarp();
        float Ls = 0.f;
        for (int i = lane; i < ns; i += 32) {
            const float mi = hw[i];
            const float f = mi > -INFINITY ? at_ex2(mi - M) : 0.f;
            hw[i] = f;
            Ls = fmaf(f, hl[i], Ls);
        }
        Ls = warp_sum(Ls);
        __syncwarp();
        const float invL = 1.0f / Ls;
        float acc[AT_MAXD] = {0.f, 0.f, 0.f, 0.f};
        for (int i0 = 0; i0 < ns; i0 += CB_SPL) {
            float v[CB_SPL][AT_MAXD];
#pragma unroll
            for (int u = 0; u < CB_SPL; ++u)
#pragma unroll
                for (int k = 0; k < AT_MAXD; ++k)
                    v[u][k] = (i0 + u < ns && lane + 32 * k < D) ? __ldcg(hb + (size_t)(i0 + u) * W + 2 + lane + 32 * k)
                                                                 : 0.f;
#pragma unroll
            for (int u = 0; u < CB_SPL; ++u) {
                const float f = i0 + u < ns ? hw[i0 + u] : 0.f;
#pragma unroll
                for (int k = 0; k < AT_MAXD; ++k) acc[k] = fmaf(f, v[u][k], acc[k]);
            }
        }
#pragma unroll
        for (int k = 0; k < AT_MAXD; ++k) {
            const int j = lane + 32 * k;
            if (j < D) {
                const float o = acc[k] * invL;
                outv[h * D + j] = o;
                mx = fmaxf(mx, fabsf(o));
            }
        }
    }
    block_sum_max(ss, mx, red);
    const float rs = mx > 0.f ? FIX_MAX * __frcp_rn(mx) : 0.f;
    if (threadIdx.x == 0) a.xsc[s] = mx > 0.f ? __frcp_rn(rs) : 1.0f;
    int8_t* ph = a.planes + (size_t)s * a.kp;
    int8_t* pm = ph + (size_t)a.slots * a.kp;
    int8_t* pl = pm + (size_t)a.slots * a.kp;
    for (int quad = threadIdx.x; quad < a.kp / 4; quad += nt) {
        const int j = 4 * quad;
        const float4 v4 = make_float4(j < n ? outv[j] : 0.f, j + 1 < n ? outv[j + 1] : 0.f,
                                      j + 2 < n ? outv[j + 2] : 0.f, j + 3 < n ? outv[j + 3] : 0.f);
        uint32_t h, m, l;
        fix_pack4(v4, rs, h, m, l);
        reinterpret_cast<uint32_t*>(ph)[quad] = h;
        reinterpret_cast<uint32_t*>(pm)[quad] = m;
        reinterpret_cast<uint32_t*>(pl)[quad] = l;
    }
}

constexpr int CB_NT = 512;  // combine threads: one warp per head (up to 16 heads per pass)
__global__ void __launch_bounds__(CB_NT) combine_stage_kernel(const CombineArgs a) {
    extern __shared__ float cb_sm[];  // [NH*D] outputs, then [NH][max_splits] weights
    __shared__ float red[64];
    griddep_launch_dependents();
    griddep_wait();
    combine_seq(a, blockIdx.x, cb_sm, red);
}

// ---- attention for head_dim 64: shared geometry ----------------------------------------
// Block (split, KV head g, sequence s) over positions [split*split_len, ...)
// up to pos[s], all gq <= 8 query heads of group g, in 64-position chunks that
// TMA brings into a ring of shared-memory slots (K and V tiles with the
// 128-byte swizzle: 16-byte chunk c of row r sits at c ^ (r % 8) within its
// 128-byte row segment, so rows read without bank conflicts).
constexpr int A64_NT = 256;
constexpr int A64_NW = A64_NT / 32;
constexpr int A64_T = 64;    // positions per chunk
constexpr int A64_HP = 8;    // query heads per group, padded

template <typename KV>
__host__ __device__ constexpr int a64_tile_bytes() { return A64_T * 64 * (int)sizeof(KV); }  // one K or V chunk

struct Attn64Args {
    const float* q;  // [slots][NH*64] rotated queries
    float* part;     // [slots][NH][max_splits][66]
    const int* pos;
    int NH, NKV, L, layer, capacity, split_len, max_splits;
    int kv_seq;  // as GemmArgs::kv_seq
    int* err;
    // Split merge in the kernel (FUSE): the last block to finish for a
    // sequence (seq_done[s] counts them; it resets it) merges its splits.
    int* seq_done;  // [slots]
    CombineArgs cb;
};

// Byte offset of element (row r, dim d) in a swizzled chunk tile.
template <typename KV>
__device__ __forceinline__ int a64_off(int r, int d) {
    if (sizeof(KV) == 4) {  // two 128-byte boxes per row: dims 0..31, then 32..63 (8 KB each)
        const int c = (d & 31) >> 2;
        return (d >> 5) * (A64_T * 128) + r * 128 + ((c ^ (r & 7)) << 4) + ((d & 3) << 2);
    } else {  // one 128-byte box per row
        const int c = d >> 3;
        return r * 128 + ((c ^ (r & 7)) << 4) + ((d & 7) << 1);
    }
}
// ---- attention for head_dim 64 on the tensor cores ----------------------------------
// Block = split x KV head x sequence, 64-position chunks by TMA into a
// swizzled ring; QK and PV are mma.sync m16n8k16 products (FP16 operands,
// FP32 accumulators). An FP32
// operand x is split as hi = f16(x), lo = f16(x - hi); the products
// hi*hi + hi*lo + lo*hi keep about 22 bits (F16 K/V need no split: two
// products). Per chunk:
//   QK: warp w: positions 16(w%4).., dims 32(w/4)..+31 (two k-steps), all heads
//       as the MMA's 8 columns; the two dim halves' partial scores in S
//   SM: warp h < gq: online softmax of head h over the chunk (base 2) -> P
//   PV: warp w: dims 16(w%4).., positions 32(w/4)..+31; O^T[dim][head]
//       accumulates across chunks in the MMA fragments (rescaled per head)
constexpr int TC_RING_F32 = 2 * 32768;  // two FP32 chunk slots (four F16): three blocks per SM
constexpr int TC_SS = 9;                 // S row stride (floats): [half][64 positions][9]
constexpr int TC_PS = 12;                // P row stride (floats): [64 positions][12], conflict-free B loads
__host__ __device__ constexpr int tc_smem_bytes() {
    return 1024 + TC_RING_F32 + 2 * A64_T * TC_SS * 4 + A64_T * TC_PS * 4 + 64;
}
template <typename KV>
__host__ __device__ constexpr int tc_slots() { return TC_RING_F32 / (2 * a64_tile_bytes<KV>()); }

__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], const uint32_t (&b)[2]) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}
// (x0, x1) -> packed f16 hi and lo parts (low half = x0).
__device__ __forceinline__ void split2(float x0, float x1, uint32_t& hi, uint32_t& lo) {
    const __half2 h = __floats2half2_rn(x0, x1);
    const float2 hf = __half22float2(h);
    const __half2 l = __floats2half2_rn(x0 - hf.x, x1 - hf.y);
    hi = *reinterpret_cast<const uint32_t*>(&h);
    lo = *reinterpret_cast<const uint32_t*>(&l);
}
__device__ __forceinline__ uint32_t pack2(float x0, float x1) {
    const __half2 h = __floats2half2_rn(x0, x1);
    return *reinterpret_cast<const uint32_t*>(&h);
}
// K/V element pair (row r, dims d, d+1), d even, of a swizzled chunk tile.
__device__ __forceinline__ float2 tile_pair(const uint8_t* tile, int r, int d, float) {
    return *reinterpret_cast<const float2*>(tile + a64_off<float>(r, d));
}
__device__ __forceinline__ uint32_t tile_pair_h(const uint8_t* tile, int r, int d) {
    return *reinterpret_cast<const uint32_t*>(tile + a64_off<__half>(r, d));
}
__device__ __forceinline__ float tile_one(const uint8_t* tile, int r, int d, float) {
    return *reinterpret_cast<const float*>(tile + a64_off<float>(r, d));
}
__device__ __forceinline__ float tile_one(const uint8_t* tile, int r, int d, __half) {
    return __half2float(*reinterpret_cast<const __half*>(tile + a64_off<__half>(r, d)));
}

template <typename KV, bool FUSE>
__global__ void __launch_bounds__(A64_NT, 3)
    attention64_tc_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                          const Attn64Args a) {
    extern __shared__ uint8_t tc_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(tc_raw) + 1023) & ~uintptr_t(1023));
    constexpr bool F16 = sizeof(KV) == 2;
    constexpr int TB = a64_tile_bytes<KV>(), NS = tc_slots<KV>();
    float* S = reinterpret_cast<float*>(sm + TC_RING_F32);  // [2 halves][64][TC_SS]
    float* P = S + 2 * A64_T * TC_SS;                        // [64][TC_PS]
    float* s_alpha = P + A64_T * TC_PS;                      // [8]
    float* ow = S;  // [2 halves][64 dims][8 heads] at the end, over the score area
    __shared__ __align__(8) uint64_t full[8];
    __shared__ float s_ml[2 * A64_HP];
    __shared__ int s_abort, s_last;
    __shared__ float s_red[64];

    const int sp_i = blockIdx.x, g = blockIdx.y, s = blockIdx.z;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int gq8 = lane >> 2, t4 = lane & 3;  // MMA fragment row group, column pair
    const int length = a.pos[s] + 1;
    const int t0 = sp_i * a.split_len;
    if (t0 >= length) return;
    const int t1 = min(length, t0 + a.split_len);
    const int nch = (t1 - t0 + A64_T - 1) / A64_T;
    const int gq = a.NH / a.NKV;
    const int row0 = (((s * a.kv_seq * a.L + a.layer) * a.NKV + g) * a.capacity) + t0;

    auto issue = [&](int c) {
        const int slot = c % NS;
        uint8_t* kt = sm + slot * 2 * TB;
        uint8_t* vt = kt + TB;
        mbar_expect(&full[slot], 2 * TB);
        const int y = row0 + c * A64_T;
        if (!F16) {
            tma2d(kt, &tmK, 0, y, &full[slot]);
            tma2d(kt + TB / 2, &tmK, 32, y, &full[slot]);
            tma2d(vt, &tmV, 0, y, &full[slot]);
            tma2d(vt + TB / 2, &tmV, 32, y, &full[slot]);
        } else {
            tma2d(kt, &tmK, 0, y, &full[slot]);
            tma2d(vt, &tmV, 0, y, &full[slot]);
        }
    };
    const int pos = length - 1;
    griddep_launch_dependents();
    if (tid == 0) {
        s_abort = 0;
        for (int i = 0; i < NS; ++i) mbar_init(&full[i], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        // Chunks wholly before the new position hold earlier steps' rows and
        // load under the previous kernel's tail; when the slots are positions
        // of one sequence (kv_seq 0) the other slots' rows of this step sit
        // there too, so everything waits.
        for (int c = 0; c < NS && c < nch; ++c)
            if (a.kv_seq && t0 + (c + 1) * A64_T <= pos) issue(c);
    }
    griddep_wait();
    if (tid == 0)
        for (int c = 0; c < NS && c < nch; ++c)
            if (!a.kv_seq || t0 + (c + 1) * A64_T > pos) issue(c);

    // QK roles: positions 16*mt.., dims 32*kh..; B fragments of q (scaled by
    // log2(e)/8), head = fragment column gq8, for this warp's two k-steps.
    const int mt = warp & 3, kh = warp >> 2;
    uint32_t qb_hi[2][2], qb_lo[2][2];
    {
        const float qscale = 1.4426950408889634f / 8.0f;
        const bool hv = gq8 < gq;
        const float* qh = a.q + ((size_t)s * a.NH + (size_t)g * gq + (hv ? gq8 : 0)) * 64;
#pragma unroll
        for (int ks = 0; ks < 2; ++ks)
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                const int d = 32 * kh + 16 * ks + 2 * t4 + 8 * r;
                const float x0 = hv ? qh[d] * qscale : 0.f, x1 = hv ? qh[d + 1] * qscale : 0.f;
                split2(x0, x1, qb_hi[ks][r], qb_lo[ks][r]);
            }
    }
    float m_run = -INFINITY, l_run = 0.f;  // head `warp`'s softmax state (warps < gq)
    float o[4] = {0.f, 0.f, 0.f, 0.f};     // O^T fragment: dims 16mt + gq8 (+8) x heads 2t4, 2t4+1
    __syncthreads();

    bool ok = true;
    for (int c = 0; c < nch; ++c) {
        const int slot = c % NS;
        const uint8_t* kt = sm + slot * 2 * TB;
        const uint8_t* vt = kt + TB;
        if (tid == 0) {
            uint64_t w0 = 0;
            unsigned spins = 0;
            while (!mbar_test(&full[slot], (uint32_t)(c / NS) & 1u)) {
                if ((++spins & 63u) == 0) {
                    const uint64_t now = globaltimer();
                    if (!w0) {
                        w0 = now;
                    } else if (now - w0 > WAIT_LIMIT_NS) {
                        atomicExch(a.err, ERR_WAIT);
                        s_abort = 1;
                        break;
                    }
                }
            }
        }
        __syncthreads();
        if (s_abort) {
            ok = false;
            break;
        }
        const int cbase = t0 + c * A64_T;
        // ---- QK: S[kh][position][head] partial over this warp's 32 dims
        {
            float sc[4] = {0.f, 0.f, 0.f, 0.f};
            const int p0 = 16 * mt + gq8, p1 = p0 + 8;
#pragma unroll
            for (int ks = 0; ks < 2; ++ks) {
                const int d = 32 * kh + 16 * ks + 2 * t4;
                uint32_t ah[4], al[4];
                if (!F16) {
                    const float2 v0 = tile_pair(kt, p0, d, 0.f), v1 = tile_pair(kt, p1, d, 0.f);
                    const float2 v2 = tile_pair(kt, p0, d + 8, 0.f), v3 = tile_pair(kt, p1, d + 8, 0.f);
                    split2(v0.x, v0.y, ah[0], al[0]);
                    split2(v1.x, v1.y, ah[1], al[1]);
                    split2(v2.x, v2.y, ah[2], al[2]);
                    split2(v3.x, v3.y, ah[3], al[3]);
                    mma16816(sc, ah, qb_hi[ks]);
                    mma16816(sc, ah, qb_lo[ks]);
                    mma16816(sc, al, qb_hi[ks]);
                } else {
                    ah[0] = tile_pair_h(kt, p0, d);
                    ah[1] = tile_pair_h(kt, p1, d);
                    ah[2] = tile_pair_h(kt, p0, d + 8);
                    ah[3] = tile_pair_h(kt, p1, d + 8);
                    mma16816(sc, ah, qb_hi[ks]);
                    mma16816(sc, ah, qb_lo[ks]);
                }
            }
            float* Sh = S + kh * A64_T * TC_SS;
            Sh[p0 * TC_SS + 2 * t4] = sc[0];
            Sh[p0 * TC_SS + 2 * t4 + 1] = sc[1];
            Sh[p1 * TC_SS + 2 * t4] = sc[2];
            Sh[p1 * TC_SS + 2 * t4 + 1] = sc[3];
        }
        __syncthreads();
        // ---- softmax over the chunk: warp h owns head h
        if (warp < gq) {
            const int h = warp;
            float scv[2];
#pragma unroll
            for (int pp = 0; pp < 2; ++pp) {
                const int t = lane + 32 * pp;
                const float v = S[t * TC_SS + h] + S[(A64_T + t) * TC_SS + h];
                scv[pp] = cbase + t < t1 ? v : -INFINITY;
            }
            const float cmax = warp_max(fmaxf(scv[0], scv[1]));
            const float m_new = fmaxf(m_run, cmax);
            const float alpha = m_run > -INFINITY ? at_ex2(m_run - m_new) : 0.f;
            const float p0 = scv[0] > -INFINITY ? at_ex2(scv[0] - m_new) : 0.f;
            const float p1 = scv[1] > -INFINITY ? at_ex2(scv[1] - m_new) : 0.f;
            l_run = fmaf(l_run, alpha, warp_sum(p0 + p1));
            m_run = m_new;
            P[lane * TC_PS + h] = p0;
            P[(lane + 32) * TC_PS + h] = p1;
            if (lane == 0) s_alpha[h] = alpha;
        } else if (warp < A64_HP) {
            P[lane * TC_PS + warp] = 0.f;
            P[(lane + 32) * TC_PS + warp] = 0.f;
            if (lane == 0) s_alpha[warp] = 0.f;
        }
        __syncthreads();
        // ---- PV: O^T[dims 16mt..][heads] += V^T[dims][positions 32kh..] P[positions][heads]
        {
            const float al0 = s_alpha[2 * t4], al1 = s_alpha[2 * t4 + 1];
            o[0] *= al0;
            o[1] *= al1;
            o[2] *= al0;
            o[3] *= al1;
            const int dm0 = 16 * mt + gq8, dm1 = dm0 + 8;
#pragma unroll
            for (int ks = 0; ks < 2; ++ks) {
                const int k0 = 32 * kh + 16 * ks + 2 * t4;  // positions k0, k0+1, k0+8, k0+9
                uint32_t bh[2], bl[2];
                split2(P[k0 * TC_PS + gq8], P[(k0 + 1) * TC_PS + gq8], bh[0], bl[0]);
                split2(P[(k0 + 8) * TC_PS + gq8], P[(k0 + 9) * TC_PS + gq8], bh[1], bl[1]);
                const float v00 = tile_one(vt, k0, dm0, KV()), v01 = tile_one(vt, k0 + 1, dm0, KV());
                const float v10 = tile_one(vt, k0, dm1, KV()), v11 = tile_one(vt, k0 + 1, dm1, KV());
                const float v20 = tile_one(vt, k0 + 8, dm0, KV()), v21 = tile_one(vt, k0 + 9, dm0, KV());
                const float v30 = tile_one(vt, k0 + 8, dm1, KV()), v31 = tile_one(vt, k0 + 9, dm1, KV());
                uint32_t ah[4], al[4];
                if (!F16) {
                    split2(v00, v01, ah[0], al[0]);
                    split2(v10, v11, ah[1], al[1]);
                    split2(v20, v21, ah[2], al[2]);
                    split2(v30, v31, ah[3], al[3]);
                    mma16816(o, ah, bh);
                    mma16816(o, ah, bl);
                    mma16816(o, al, bh);
                } else {
                    ah[0] = pack2(v00, v01);
                    ah[1] = pack2(v10, v11);
                    ah[2] = pack2(v20, v21);
                    ah[3] = pack2(v30, v31);
                    mma16816(o, ah, bh);
                    mma16816(o, ah, bl);
                }
            }
        }
        __syncthreads();  // slot, S and P consumed by every warp
        if (tid == 0 && c + NS < nch) {
            fence_proxy_async();
            issue(c + NS);
        }
    }
    if (!ok) {
        if (tid == 0) {
            const uint64_t w0 = globaltimer();
            for (int c = 0; c < nch && c < NS; ++c) {
                const int last = c + ((nch - 1 - c) / NS) * NS;
                while (!mbar_test(&full[c % NS], (uint32_t)(last / NS) & 1u) && globaltimer() - w0 < WAIT_LIMIT_NS) {
                }
            }
        }
        __syncthreads();
        return;
    }
    // Sum the two position halves of O^T, then write (max, sum, output) per head.
    {
        const int dm0 = 16 * mt + gq8, dm1 = dm0 + 8;
        float* oh = ow + kh * 64 * A64_HP;
        oh[dm0 * A64_HP + 2 * t4] = o[0];
        oh[dm0 * A64_HP + 2 * t4 + 1] = o[1];
        oh[dm1 * A64_HP + 2 * t4] = o[2];
        oh[dm1 * A64_HP + 2 * t4 + 1] = o[3];
    }
    if (warp < gq && lane == 0) {
        s_ml[2 * warp] = m_run;
        s_ml[2 * warp + 1] = l_run;
    }
    __syncthreads();
    for (int e = tid; e < gq * 64; e += A64_NT) {
        const int h = e >> 6, j = e & 63;
        const float acc = ow[j * A64_HP + h] + ow[64 * A64_HP + j * A64_HP + h];
        float* pp = a.part + (((size_t)s * a.NH + (size_t)g * gq + h) * a.max_splits + sp_i) * 66;
        if (j == 0) {
            pp[0] = s_ml[2 * h];
            pp[1] = s_ml[2 * h + 1];
        }
        pp[2 + j] = acc;
    }
    if (!FUSE) return;
    __syncthreads();  // this block's partials are written
    if (tid == 0) {
        __threadfence();
        const int total = a.NKV * ((length + a.split_len - 1) / a.split_len);  // blocks of sequence s
        s_last = atomicAdd(a.seq_done + s, 1) == total - 1;
    }
    __syncthreads();
    if (s_last) {
        __threadfence();
        combine_seq(a.cb, s, reinterpret_cast<float*>(sm), s_red);  // the ring is free now
        if (tid == 0) a.seq_done[s] = 0;
    }
}

// ---- argmax over the LM-head tiles; next tokens; positions advance --------------------
struct ArgmaxArgs {
    const ArgBest* amax;  // [tiles][slots]
    int tiles, slots, nseq;
    int* argmax;  // [slots]
    int* tokens;  // [slots] next input tokens (the greedy choice)
    int* pos;     // [slots] advanced by one
};
__global__ void __launch_bounds__(ARG_NT) argmax_kernel(const ArgmaxArgs a) {
    __shared__ float sv[ARG_NT / 32];
    __shared__ int si[ARG_NT / 32];
    griddep_launch_dependents();
    griddep_wait();
    const int s = blockIdx.x;
    float v = -INFINITY;
    int vi = 0x7fffffff;
    for (int t = threadIdx.x; t < a.tiles; t += ARG_NT) {
        const ArgBest b = a.amax[(size_t)t * a.slots + s];
        if (better(b.v, b.i, v, vi)) {
            v = b.v;
            vi = b.i;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(FULL, v, o);
        const int oi = __shfl_xor_sync(FULL, vi, o);
        if (better(ov, oi, v, vi)) {
            v = ov;
            vi = oi;
        }
    }
    if ((threadIdx.x & 31) == 0) {
        sv[threadIdx.x >> 5] = v;
        si[threadIdx.x >> 5] = vi;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < ARG_NT / 32; ++w)
            if (better(sv[w], si[w], v, vi)) {
                v = sv[w];
                vi = si[w];
            }
        if (vi == 0x7fffffff) vi = 0;
        a.argmax[s] = vi;
        a.tokens[s] = vi;
        a.pos[s] += 1;
    }
}

}  // namespace batch
}  // namespace dcb
