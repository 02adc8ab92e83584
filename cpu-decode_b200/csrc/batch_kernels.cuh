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
// all four warps read TMEM in the epilogue. Every wait is bounded.
//
// Attention is split-KV over each sequence's own cache (head-major rows, one
// contiguous block per split), every staged K/V byte serving all query heads
// of its group; a combine kernel merges the splits of one sequence and stages
// the result for the O projection.
#pragma once
#include "attention.cuh"
#include "step_kernel.cuh"

#include <cuda.h>

namespace dcb {
namespace batch {

constexpr int GM = 128;        // weight rows per GEMM tile (UMMA M)
constexpr int GK = 128;        // reduction bytes per pipeline stage (one 128-byte swizzle row)
constexpr int GSTAGES = 4;     // pipeline depth
constexpr int GT = 128;        // GEMM threads (four warps: one per 32 TMEM lanes)
constexpr int MAX_SLOTS = 64;  // sequences per batch: N = 3 * slots <= 192
constexpr uint32_t TMEM_COLS = 256;
constexpr int A_BYTES = GM * GK;  // 16 KB per stage
constexpr int ST_NT = 256;        // threads of the staging kernels
constexpr int ARG_NT = 256;       // threads of the argmax kernel

enum Epi { EPI_PLAIN = 0, EPI_QKV = 1, EPI_RESID = 2, EPI_GU = 3, EPI_HEAD = 4 };

__host__ __device__ constexpr int b_bytes(int slots) { return 3 * slots * GK; }
// Dynamic shared memory of the GEMM: 1 KB alignment slack, then the A and B rings.
__host__ __device__ constexpr int gemm_smem_bytes(int slots) { return 1024 + GSTAGES * (A_BYTES + b_bytes(slots)); }

struct GemmArgs {
    int M;      // weight rows
    int nk;     // reduction stages (ceil(K / GK))
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
    const float* rope_inv;  // [D/2]
    const float* rope_den;  // [D/2]
    const int* pos;         // [slots] position of each sequence's new token
    void* kcache;           // [slots][L][NKV][capacity][D]
    void* vcache;
    ArgBest* amax;  // HEAD: [tiles][slots] best (value, row) of each tile and sequence
    int* err;       // set to ERR_WAIT when a wait runs out
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
// Instruction descriptor of kind::i8: signed A and B, S32 accumulators, both
// K-major, M = GM, N = n.
__host__ __device__ constexpr uint32_t idesc_i8(int n) {
    return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(GM >> 4) << 24);
}
__device__ __forceinline__ void umma_i8(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t accumulate) {
    const uint32_t z = 0;
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(tmem_d),
        "l"(da), "l"(db), "r"(idesc), "r"(accumulate), "r"(z), "r"(z), "r"(z), "r"(z));
}
// Arrive on m once every MMA issued so far by this thread has completed.
__device__ __forceinline__ void umma_commit(uint64_t* m) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(m))
                 : "memory");
}
__device__ __forceinline__ void tma2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* m) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
            "r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(m))
        : "memory");
}
__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t cols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)), "r"(cols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t cols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// 32 TMEM lanes (one per thread of the warp) x 16 consecutive 32-bit columns.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
          "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

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

// ---- the GEMM ----------------------------------------------------------------------
template <int EPI, typename KV>
__global__ void __launch_bounds__(GT, 1)
    gemm_i8_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, const GemmArgs a) {
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

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int m0 = blockIdx.x * GM;

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
    for (int s = tid; s < a.slots; s += GT) {
        s_xsc[s] = s < a.nseq ? a.xsc[s] : 0.f;
        s_xinv[s] = (a.xinv && s < a.nseq) ? a.xinv[s] : 1.f;
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_tmem;

    if (warp == 0) {
        if (lane == 0) {
            // Producer: weight tile rows m0.., all sequences' planes, GK bytes of K per stage.
            const uint32_t bytes = (uint32_t)(A_BYTES + BB);
            for (int kt = 0; kt < a.nk; ++kt) {
                const int s = kt % GSTAGES;
                if (kt >= GSTAGES && !wait_phase(&empty[s], (uint32_t)((kt / GSTAGES) - 1) & 1u, a.err)) break;
                mbar_expect(&full[s], bytes);
                tma2d(sA + s * A_BYTES, &tmA, kt * GK, m0, &full[s]);
                tma2d(sB + s * BB, &tmB, kt * GK, 0, &full[s]);
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0) {
            // MMA issuer: 4 MMAs of K = 32 per stage, accumulating in TMEM.
            const uint32_t idesc = idesc_i8(N);
            for (int kt = 0; kt < a.nk; ++kt) {
                const int s = kt % GSTAGES;
                if (!wait_phase(&full[s], (uint32_t)(kt / GSTAGES) & 1u, a.err)) break;
                tc_fence_after();
                const uint64_t da = sw128_desc(sA + s * A_BYTES), db = sw128_desc(sB + s * BB);
#pragma unroll
                for (int kk = 0; kk < GK / 32; ++kk)
                    umma_i8(tmem, da + 2 * kk, db + 2 * kk, idesc, (kt | kk) != 0 ? 1u : 0u);
                umma_commit(&empty[s]);
            }
            umma_commit(&done);
        }
        __syncwarp();
    }
    if (tid == 0) {
        wait_phase(&done, 0, a.err);
        // Every load issued must have landed before the block may exit (only
        // relevant after an expired wait; otherwise these phases are complete).
        for (int s = 0; s < GSTAGES && s < a.nk; ++s) {
            const int last = s + ((a.nk - 1 - s) / GSTAGES) * GSTAGES;  // last stage index kt using slot s
            wait_phase(&full[s], (uint32_t)(last / GSTAGES) & 1u, a.err);
        }
    }
    __syncthreads();
    tc_fence_after();

    // ---- epilogue: thread = weight row m0 + 32*warp + lane
    const int r = m0 + 32 * warp + lane;
    const bool rv = r < a.M;
    const float wsc = rv ? a.wscale[(size_t)r * a.wstride] : 0.f;
    const float bia = (rv && a.bias) ? a.bias[(size_t)r * a.bstride] : 0.f;
    const uint32_t trow = tmem + ((uint32_t)(32 * warp) << 16);
    for (int s0 = 0; s0 < a.nseq; s0 += 16) {
        uint32_t hi[16], md[16], lo[16];
        tmem_ld16(trow + (uint32_t)s0, hi);
        tmem_ld16(trow + (uint32_t)(a.slots + s0), md);
        tmem_ld16(trow + (uint32_t)(2 * a.slots + s0), lo);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            const int s = s0 + i;
            const bool sv = s < a.nseq;
            const float acc = planes_to_float((int)hi[i], (int)md[i], (int)lo[i]);
            float y = acc * s_xsc[s] * s_xinv[s] * wsc + bia;
            if (EPI == EPI_PLAIN) {
                if (rv && sv) a.out[(size_t)s * a.ldo + r] = y;
            } else if (EPI == EPI_RESID) {
                if (rv && sv) a.out[(size_t)s * a.ldo + r] += y;
            } else if (EPI == EPI_GU) {
                // rows (2j, 2j+1) = (gate_j, up_j) in adjacent lanes (src/model.cpp:306-308)
                const float u = __shfl_xor_sync(FULL, y, 1);
                if (rv && sv && !(lane & 1)) a.out[(size_t)s * a.ldo + (r >> 1)] = (y / (1.0f + expf(-y))) * u;
            } else if (EPI == EPI_QKV) {
                // rows (2u, 2u+1) = (j, j + D/2) of one head in adjacent lanes (src/model.cpp:277-302)
                const float other = __shfl_xor_sync(FULL, y, 1);
                if (rv && sv) {
                    const int half = a.D >> 1, u = r >> 1;
                    const int qpairs = a.NH * half, kpairs = a.NKV * half;
                    const int kind = u < qpairs ? 0 : (u < qpairs + kpairs ? 1 : 2);
                    const int pu = kind == 0 ? u : (kind == 1 ? u - qpairs : u - qpairs - kpairs);
                    const int hd = pu / half, j = pu - hd * half;
                    const bool second = lane & 1;
                    const float y0 = second ? other : y, y1 = second ? y : other;
                    float val = second ? y1 : y0;
                    const int p = a.pos[s];
                    if (kind < 2) {
                        const float angle =
                            a.cached_rope ? __fmul_rn((float)p, a.rope_inv[j]) : __fdiv_rn((float)p, a.rope_den[j]);
                        float sn, cs;
                        sincosf(angle, &sn, &cs);
                        val = second ? __fadd_rn(__fmul_rn(y1, cs), __fmul_rn(y0, sn))
                                     : __fsub_rn(__fmul_rn(y0, cs), __fmul_rn(y1, sn));
                    }
                    const int idx = j + (second ? half : 0);
                    if (kind == 0) {
                        a.out[(size_t)s * a.ldo + hd * a.D + idx] = val;
                    } else {
                        KV* cache = static_cast<KV*>(kind == 1 ? a.kcache : a.vcache) +
                                    ((((size_t)s * a.L + a.layer) * a.NKV + hd) * a.capacity + p) * a.D;
                        kv_store(cache + idx, val);
                    }
                }
            } else if (EPI == EPI_HEAD) {
                if (rv && sv && a.out) a.out[(size_t)s * a.ldo + r] = y;
                float v = (rv && sv) ? y : -INFINITY;
                int vi = r;
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    const float ov = __shfl_xor_sync(FULL, v, o);
                    const int oi = __shfl_xor_sync(FULL, vi, o);
                    if (better(ov, oi, v, vi)) {
                        v = ov;
                        vi = oi;
                    }
                }
                if (lane == 0) {
                    s_bv[warp][s] = v;
                    s_bi[warp][s] = vi;
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
    tc_fence_before();
    __syncthreads();
    if (warp == 2) {
        tc_fence_after();
        tmem_dealloc(tmem, TMEM_COLS);
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
};

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

// One block per sequence: v (embedded token row or src), sum v^2 for the
// RMSNorm factor (src/kernels.cpp:132-137), v*gain quantised into the planes.
__global__ void __launch_bounds__(ST_NT) stage_kernel(const StageArgs a) {
    extern __shared__ float st_v[];  // [n] gained values
    __shared__ float red[64];
    const int s = blockIdx.x;
    if (s >= a.nseq) return;
    const uint8_t* row = nullptr;
    float rsc = 0.f;
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
        const float4 v4 = make_float4(j < a.n ? st_v[j] : 0.f, j + 1 < a.n ? st_v[j + 1] : 0.f,
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
    const void* kcache;  // [slots][L][NKV][capacity][D]
    const void* vcache;
    float* part;  // [slots][NH][max_splits][D+2]: (max, sum, unnormalised output) of each split
    const int* pos;
    int NH, NKV, D, L, layer, capacity, split_len, max_splits;
};

// Block (split, kv head g, sequence s): positions [split*split_len, ...) up to
// pos[s] (inclusive) of sequence s, all query heads of group g.
template <typename KV, int DT>
__global__ void __launch_bounds__(AT_NT) attention_kernel(const AttnArgs a) {
    extern __shared__ __align__(16) unsigned char at_sm[];
    const int sp = blockIdx.x, g = blockIdx.y, s = blockIdx.z;
    const int D = DT ? DT : a.D;
    const int length = a.pos[s] + 1;
    const int t0 = sp * a.split_len;
    if (t0 >= length) return;
    const int t1 = min(length, t0 + a.split_len);
    const int gq = a.NH / a.NKV;
    const size_t head = (((size_t)s * a.L + a.layer) * a.NKV + g) * (size_t)a.capacity * D;
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

// One block per sequence: merge the splits of every head (in split order) and
// stage the attention output (NH*D values) as planes for the O projection.
struct CombineArgs {
    const float* part;
    const int* pos;
    int NH, D, split_len, max_splits, slots, kp;
    int8_t* planes;  // [3][slots][kp]
    float* xsc;
};
__global__ void __launch_bounds__(ST_NT) combine_stage_kernel(const CombineArgs a) {
    extern __shared__ float cb_sm[];  // [NH*D] outputs, then [NH][max_splits] weights
    __shared__ float red[64];
    const int s = blockIdx.x;
    const int n = a.NH * a.D;
    float* outv = cb_sm;
    float* wts = cb_sm + n;
    const int ns = (a.pos[s] + a.split_len) / a.split_len;  // splits covering positions 0..pos
    const float* base = a.part + (size_t)s * a.NH * a.max_splits * (a.D + 2);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = ST_NT / 32;
    // Per head: weight of split i = 2^(m_i - M) / sum_i 2^(m_i - M) l_i.
    for (int h = warp; h < a.NH; h += nw) {
        const float* hb = base + (size_t)h * a.max_splits * (a.D + 2);
        float M = -INFINITY;
        for (int i = lane; i < ns; i += 32) M = fmaxf(M, hb[(size_t)i * (a.D + 2)]);
        M = warp_max(M);
        float Ls = 0.f;
        for (int i = lane; i < ns; i += 32) {
            const float mi = hb[(size_t)i * (a.D + 2)];
            const float f = mi > -INFINITY ? at_ex2(mi - M) : 0.f;
            wts[h * a.max_splits + i] = f;
            Ls = fmaf(f, hb[(size_t)i * (a.D + 2) + 1], Ls);
        }
        Ls = warp_sum(Ls);
        __syncwarp();
        const float invL = 1.0f / Ls;
        for (int i = lane; i < ns; i += 32) wts[h * a.max_splits + i] *= invL;
    }
    __syncthreads();
    float mx = 0.f, ss = 0.f;
    for (int e = threadIdx.x; e < n; e += ST_NT) {
        const int h = e / a.D, j = e - h * a.D;
        const float* hb = base + (size_t)h * a.max_splits * (a.D + 2) + 2 + j;
        float acc = 0.f;
        for (int i = 0; i < ns; ++i) acc = fmaf(wts[h * a.max_splits + i], hb[(size_t)i * (a.D + 2)], acc);
        outv[e] = acc;
        mx = fmaxf(mx, fabsf(acc));
    }
    block_sum_max(ss, mx, red);
    const float rs = mx > 0.f ? FIX_MAX * __frcp_rn(mx) : 0.f;
    if (threadIdx.x == 0) a.xsc[s] = mx > 0.f ? __frcp_rn(rs) : 1.0f;
    int8_t* ph = a.planes + (size_t)s * a.kp;
    int8_t* pm = ph + (size_t)a.slots * a.kp;
    int8_t* pl = pm + (size_t)a.slots * a.kp;
    for (int quad = threadIdx.x; quad < a.kp / 4; quad += ST_NT) {
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
