// The decode step as one persistent kernel whose blocks take one of two roles.
//
// Same computation as step_kernel.cuh (the reference's Engine::Impl::step,
// src/model.cpp:258-329), organised so that every layer costs two grid-wide
// hand-offs and nothing else:
//
//   attention blocks (2 per query head h, "halves" s = 0, 1):
//     poll x (the down sums of the previous layer, or the embedding row) ->
//     RMSNorm + GEMV of the block's QKV rows: half of head h's q RoPE pairs
//     and a 1/(2*heads-per-group) share of its KV group's k/v pairs (bias,
//     RoPE, KV-cache row) -> swap q halves and the group's new k/v row as
//     tagged words (few writers, few readers) -> exact attention of head h
//     over every position, all of them resident in shared memory -> its half
//     of W_o's rows times the head output, added into the O sums
//     (the blocks of head 0 also add x, so the O sums are x_b itself);
//   FFN blocks (the rest):
//     poll x_b (the O sums) -> RMSNorm + gate/up GEMV of the block's rows ->
//     SiLU(gate)*up -> the block's columns of W_down times those values, added
//     into the down sums (the last FFN block also adds x_b, so the down sums
//     are the next layer's x).
//
// The sums are the self-counting fixed-point words of step_kernel.cuh
// (dacc_add): exact, order-free, complete when the count of contributions is
// reached. Each role polls exactly one of them per layer; the polls of the
// other role's all-reduce never compete with its own.
//
// Weights stream into shared-memory slots by bulk copies one layer ahead (each
// slot is refilled as soon as it is consumed), and the cached K/V rows of a
// layer are copied in while the previous layer still runs, so a phase waits
// only for its input vector. Every wait is bounded (1 s); on expiry a block
// records the error, drains its copies in flight and returns.
#pragma once
#include "step_kernel.cuh"

namespace dcb {

constexpr int RA_ROWS_MAX = 64;   // QKV rows of one attention block, at most (4 tiles of 16)
constexpr int RG_ROWS_MAX = 96;   // gate/up rows of one FFN block, at most (6 tiles of 16)
constexpr int RES_BUFS_MAX = 8;   // resident KV chunk buffers, at most
constexpr int RES_POS_MAX = RES_BUFS_MAX * ATT_CHUNK;  // positions one attention block keeps resident
// The block's last thread issues every bulk copy and never a global store or
// reduction, so its proxy fence before a refill has nothing of its own to
// wait for. Sum-word rows are spread over the other warps (SLICE_T threads).
constexpr int COPY_T = NT - 1;
constexpr int SLICE_T = NT - 32;
constexpr int SLICE_RPT = 3;  // rows per thread of a sum-word share (H <= SLICE_RPT * SLICE_T)
constexpr int ROLE_PLANE = 160;   // bytes per plane of a staged short vector (head output, SiLU*up share)
constexpr int ROLE_MISC_BYTES = 512 * 4 + 3 * ROLE_PLANE;  // q, new K/V row, head output, planes

struct RoleParams {
    int H, I, L, NH, NKV, D, V, Kh, SH;
    float eps;
    int cached_rope, capacity;
    int NA, NG;          // attention blocks (2 per query head: blocks 2h, 2h+1), FFN blocks (the rest)
    int ra_stride;       // packed QKV rows per attention block (slot stride; its own count is ra_rows())
    int q_first;         // RoPE pairs of q computed by half 0 (half 1: D/2 - q_first)
    int o_first;         // W_o rows of half 0 (a multiple of 4; half 1: H - o_first)
    int o_dw, o_slice;   // W_o column slices: bytes per row, bytes per (layer, head)
    int dw, down_slice;  // FFN blocks' W_down column slices: bytes per row, bytes per (layer, block)
    int dcontrib;        // FFN blocks with gate/up rows: the count of every down sum word
    // Coarse waits end when a sum word is this many contributions short of
    // complete (the fine poll of every word takes over from there).
    int coarse_down, coarse_o;
    int nbufs;           // resident KV chunk buffers of an attention block
    // Spread attention (positions beyond the attention blocks' buffers, head
    // dim 64): block b < NKV * sp_splits is unit (KV group b / sp_splits,
    // split b % sp_splits), which keeps chunks split, split + sp_splits, ...
    // (at most sp_bufs) resident and publishes (m, l, o) of every head of its
    // group into ll_part. FFN blocks keep them at g_ring (queries and scores
    // at g_sq), attention blocks in their chunk buffers (scratch after
    // sp_bufs of them, at a_ring + a_sq).
    int sp_splits, sp_bufs, g_ring, g_sq, a_sq;
    uint64_t* ll_part;   // [NH][sp_splits][D+2] tagged split partials
    // KV sequence split over GPUs (spread mode): this engine keeps positions
    // [kv_base, kv_end) as local cache rows; rank `rank` of `world` exchanges
    // each head's (m, l, o) through exch ([2][NH][world][D+2] tagged words,
    // its own) and peers[q] (rank q's, over NVLink).
    int kv_base, kv_end, world, rank;
    uint64_t* const* peers;
    uint64_t* exch;
    int chunk_bytes;     // one chunk buffer: [64 K rows | 64 V rows]
    int bulk_kv;         // K/V rows are a multiple of 16 bytes (bulk copies), else plain loads
    const uint8_t* qkv;     // [L][NA][ra_stride][SH] packed rows
    const uint8_t* o_cols;  // [L][NH][o_slice]: W_o's columns of head h, H rows of o_dw bytes
    const float* o_scale;   // [L][H]
    const LayerW* layers;   // gate/up rows (interleaved gate_j, up_j) per layer
    const uint8_t* down_cols;  // [L][NG][down_slice]: FFN block f's columns of W_down, H rows of dw bytes
    const float* down_scale;   // [L][H]
    const uint8_t* embed;      // V packed rows (the tied LM head)
    const float* norms;        // [L+1][2][Kh]
    const float* rope_inv;
    const float* rope_den;
    void* kcache;  // [L][NKV][capacity][D]
    void* vcache;
    uint64_t* ll_q;   // [NH][D] tagged q values (each half written by its block)
    uint64_t* ll_kv;  // [NKV][2D] tagged new k then v row of each KV group
    uint64_t* dacc;   // [2 halves][L][2: O, down][Hp] self-counting sum words
    int Hp;
    float* logits;
    ArgBest* amax;
    Sync* sync;
    uint64_t* trace;  // [2][TRACE_MAX_PHASES][grid] or null (phases as step_kernel.cuh)
    int trace_layer;
    int xq_plane;
    // shared memory layout (bytes). Attention blocks:
    int a_qkv, a_o, a_ring, a_part, a_sc;
    // FFN blocks:
    int g_gu, g_down, g_part, g_h;
    // both: staged floats, fixed-point planes, raw residual, small scratch
    int off_xf, off_xq, off_xr, off_misc;
};

// QKV rows of attention block a (its q pairs, then its k/v pairs), and where
// they go. Pair p of the block: q pair j = q0 + p for p < nq, else k/v pair
// u = kv0 + (p - nq) of its KV group (u < D/2: k pair u, else v pair u - D/2).
struct AttnRows {
    int h, s, g, q0, nq, kv0, nkv;
};
__device__ __forceinline__ AttnRows attn_rows(const RoleParams& P, int a) {
    AttnRows r;
    r.h = a >> 1;
    r.s = a & 1;
    const int hpg = P.NH / P.NKV, half = P.D / 2;
    r.g = r.h / hpg;
    r.q0 = r.s ? P.q_first : 0;
    r.nq = r.s ? half - P.q_first : P.q_first;
    const int m = 2 * (r.h % hpg) + r.s;  // this block's index among the 2*hpg blocks of the group
    r.kv0 = part_lo(m, 2 * hpg, P.D);
    r.nkv = part_lo(m + 1, 2 * hpg, P.D) - r.kv0;
    return r;
}

// Trace records exist only in the traced instantiation (TR), so the product
// kernel carries none of their code.
template <bool TR>
__device__ __forceinline__ void rtrace(const RoleParams& P, int which, int phase) {
    if (TR && P.trace && threadIdx.x == 0)
        P.trace[((size_t)which * TRACE_MAX_PHASES + phase) * gridDim.x + blockIdx.x] = globaltimer();
}

// Detailed marks m (< 8) inside phase k (< 5) of the traced layer: slot
// TRACE_DETAIL + 8k + m of the ready record (as step_kernel.cuh's trace_detail).
// The marks are SM clock counts (cheap; compare marks of one block only).
template <bool TR>
__device__ __forceinline__ void rdetail(const RoleParams& P, int layer, int k, int m) {
    if (TR && P.trace && layer == P.trace_layer && threadIdx.x == 0)
        P.trace[((size_t)TRACE_DETAIL + 8 * k + m) * gridDim.x + blockIdx.x] = clock64();
}

// Coarse part of waiting for a sum: thread 0 polls one word (w, chosen per
// block to spread the pollers over lines) until at least `first` of its
// contributions have arrived, while the block rests at a barrier. The fine
// poll of every word (all threads, all loads in flight) then covers only the
// last contributions, so the idle role does not flood the L2 lines the
// working role is adding into. Returns false when the wait ran out.
__device__ __forceinline__ bool coarse_wait(const uint64_t* w, unsigned first, const BlockState& st) {
    if (threadIdx.x == 0 && first > 0) {
        uint64_t t0 = 0;
        unsigned rounds = 0;
        while (dacc_count(ll_load(w)) < first)
            if ((++rounds & 7u) == 0 && wait_expired(st, t0)) break;
    }
    __syncthreads();
    return !should_abort(st);
}

// A block-wide mark: when tracing, every thread has reached this point.
template <bool TR>
__device__ __forceinline__ void rdetail_sync(const RoleParams& P, int layer, int k, int m) {
    if (TR && P.trace) {
        __syncthreads();
        rdetail<TR>(P, layer, k, m);
    }
}

// ---- int8 tensor-core fragments (mma.sync m16n8k16, s8 x s8 -> s32) ----
// A staged vector's three fixed-point planes are the first three columns of
// the B operand (columns 3..7 zero), so one MMA yields the hi, mid and lo
// plane sums of 16 rows over 16 columns: the same exact integer sums as three
// dp4a chains. A fragments come from row-major int8 rows in shared memory by
// ldmatrix (rows 16-byte aligned; an odd number of 16-byte units per row keeps
// each 8-row matrix in distinct banks).
__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
    const uint32_t a = (uint32_t)__cvta_generic_to_shared(p);
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(a)
                 : "memory");
}
__device__ __forceinline__ void mma_i8(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t b) {
    asm("mma.sync.aligned.m16n8k16.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%0,%1,%2,%3};"
        : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
        : "r"(a0), "r"(a1), "r"(b));
}
// B fragment of 16 staged columns starting at byte c16: lane (g, q) holds
// plane g's bytes c16 + 4q .. + 3 (zero for g >= 3).
__device__ __forceinline__ uint32_t plane_frag(const int8_t* xq, int plane, int c16) {
    const int lane = threadIdx.x & 31, g = lane >> 2, q = lane & 3;
    return g < 3 ? *reinterpret_cast<const uint32_t*>(xq + g * plane + c16 + 4 * q) : 0u;
}
// The value of one accumulator tile's row for lanes q < 2 (row g + 8q of the
// tile): lane q = 0 holds hi, mid of rows g and g + 8, lane q = 1 their lo.
// Every lane takes part in the shuffles.
__device__ __forceinline__ float tile_row_value(const int (&c)[4]) {
    const int lo_g = __shfl_xor_sync(FULL, c[0], 1);
    const int hi_g8 = __shfl_xor_sync(FULL, c[2], 1);
    const int md_g8 = __shfl_xor_sync(FULL, c[3], 1);
    return (threadIdx.x & 1) == 0 ? planes_to_float(c[0], c[1], lo_g) : planes_to_float(hi_g8, md_g8, c[2]);
}

// Rows [r0, r1) of a column slice (dw bytes per row in shared memory: an odd
// number of words, zero past the slice's columns) times v[0, dw) (floats,
// zero past the columns), scaled per row, plus fold[r] when set, added into
// the sum words acc[r]. FP32 arithmetic: each int8 widened exactly with the
// byte trick of dot4, packed f32x2 FMAs; v is read as float4 (the same
// address for every lane). Threads below SLICE_T take rows r0 + tid +
// i*SLICE_T; s0..s2 are those rows' scales, loaded by the caller well ahead.
__device__ __forceinline__ void slice_rows(const uint8_t* slice, int dw, int r0, int r1, const float* v, float s0,
                                           float s1, float s2, const float* fold, uint64_t* acc) {
    const int nw = dw / 4;
    if (threadIdx.x >= SLICE_T) return;
    const float scale[SLICE_RPT] = {s0, s1, s2};
    const float4* v4 = reinterpret_cast<const float4*>(v);
#pragma unroll
    for (int i = 0; i < SLICE_RPT; ++i) {
        const int r = r0 + (int)threadIdx.x + i * SLICE_T;
        if (r >= r1) break;
        const uint32_t* w = reinterpret_cast<const uint32_t*>(slice + (size_t)(r - r0) * dw);
        float2 a0 = make_float2(0.f, 0.f), a1 = a0, a2 = a0, a3 = a0;
        int k = 0;
#pragma unroll 2
        for (; k + 3 < nw; k += 4) {
            a0 = dot4(w[k], v4[k], a0);
            a1 = dot4(w[k + 1], v4[k + 1], a1);
            a2 = dot4(w[k + 2], v4[k + 2], a2);
            a3 = dot4(w[k + 3], v4[k + 3], a3);
        }
        for (; k < nw; ++k) a0 = dot4(w[k], v4[k], a0);
        float t = (((a0.x + a0.y) + (a1.x + a1.y)) + ((a2.x + a2.y) + (a3.x + a3.y))) * scale[i];
        if (fold) t += fold[r];
        dacc_add(acc + r, t);
    }
}

// Block GEMV of R packed rows in shared memory (stride S bytes, an odd number
// of 16-byte units; nch chunks of 16 int8) with the staged planes: warp w
// covers chunks [w*nch/NW, (w+1)*nch/NW) (at most ROLE_CPW) for every tile of
// 16 rows (MT tiles at most), one MMA per tile and chunk.
// partial[w*R + r] = the warp's share times its staging scale; the closing
// barrier publishes them. run false: only the barrier.
constexpr int ROLE_CPW = 4;  // chunks per warp, at most (hidden <= 1024)
template <int MT>
__device__ __forceinline__ void role_gemv(const uint8_t* rows, int S, int R, int nch, const int8_t* xq, int plane,
                                          float* partial, float wscale, bool run) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int c0 = warp * nch / NW, c1 = (warp + 1) * nch / NW;
    const int nt = (R + 15) >> 4;
    if (run) {
        int acc[MT][4];
#pragma unroll
        for (int t = 0; t < MT; ++t) acc[t][0] = acc[t][1] = acc[t][2] = acc[t][3] = 0;
#pragma unroll 1
        for (int c = c0; c < c1; ++c) {
            {
                const uint32_t bf = plane_frag(xq, plane, 16 * c);
#pragma unroll
                for (int t = 0; t < MT; t += 2) {
                    if (t < nt) {
                        uint32_t a[4];
                        ldsm_x4(a, rows + (size_t)min(16 * t + lane, R - 1) * S + 16 * c);
                        mma_i8(acc[t], a[0], a[1], bf);
                        if (t + 1 < MT && t + 1 < nt) mma_i8(acc[t + 1], a[2], a[3], bf);
                    }
                }
            }
        }
#pragma unroll
        for (int t = 0; t < MT; ++t) {
            if (t < nt) {
                const float v = tile_row_value(acc[t]);
                const int r = 16 * t + (lane >> 2) + 8 * (lane & 3);
                if ((lane & 3) < 2 && r < R) partial[warp * R + r] = v * wscale;
            }
        }
    }
    __syncthreads();
}

// Exact attention of one query head over positions [0, n) resident in the
// chunk ring (the new row already written into its chunk), the reference's
// src/kernels.cpp:150-179: scores q.k (q pre-scaled by log2(e)/sqrt(D)), the
// maximum, 2^(s - max), their sum, then the weighted sum of V rows. Every
// position is resident, so there is no running rescale:
//   1. scores into sc[t] (8 lanes per position), each warp keeping the
//      maximum of the scores it produced;
//   2. the block maximum from the warps' maxima; thread t turns sc[t] into
//      p_t = 2^(s_t - max) once;
//   3. P.V: warp w takes positions t = w mod 16, lane d2 dims 2*d2, 2*d2+1
//      (+64 per step); the 16 partial sums and weight sums are added in order.
// Output in out[0..D). sc: n floats; part: [16][D + 1] floats; wmax: 16 floats.
template <typename KV, int MD>
__device__ __forceinline__ void attend_resident(const uint8_t* ring, int chunk_bytes, int D, int n, const float* sq,
                                                float* sc, float* part, float* wmax, float* out) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    {
        const int grp = lane >> 3, pp = lane & 7;
        float qv[MD][4];
#pragma unroll
        for (int k = 0; k < MD; ++k)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int j = 32 * k + 4 * pp + e;
                qv[k][e] = j < D ? sq[j] : 0.f;
            }
        float m_w = -INFINITY;
        for (int t0 = 0; t0 < n; t0 += ATT_CHUNK) {
            const int t = t0 + warp * 4 + grp;
            const KV* kb = reinterpret_cast<const KV*>(ring + (size_t)(t0 / ATT_CHUNK) * chunk_bytes);
            float s = 0.f;
            if (t < n) {
                const KV* kr = kb + (size_t)(t - t0) * D;
#pragma unroll
                for (int k = 0; k < MD; ++k) {
                    const int j0 = 32 * k + 4 * pp;
                    float kk[4];
                    if (j0 + 3 < D && (D & 3) == 0) {
                        load4(kr + j0, kk);
                    } else {
#pragma unroll
                        for (int e = 0; e < 4; ++e) kk[e] = j0 + e < D ? kv_to_float(kr[j0 + e]) : 0.f;
                    }
#pragma unroll
                    for (int e = 0; e < 4; ++e) s = fmaf(qv[k][e], kk[e], s);
                }
            }
            s += __shfl_xor_sync(FULL, s, 4);
            s += __shfl_xor_sync(FULL, s, 2);
            s += __shfl_xor_sync(FULL, s, 1);
            if (t < n) {
                if (pp == 0) sc[t] = s;
                m_w = fmaxf(m_w, s);
            }
        }
        m_w = fmaxf(m_w, __shfl_xor_sync(FULL, m_w, 8));
        m_w = fmaxf(m_w, __shfl_xor_sync(FULL, m_w, 16));
        if (lane == 0) wmax[warp] = m_w;
    }
    __syncthreads();
    {
        float M = lane < NW ? wmax[lane] : -INFINITY;
        M = warp_max(M);
        for (int t = tid; t < n; t += NT) sc[t] = ex2_approx(sc[t] - M);
    }
    __syncthreads();
    constexpr int ND2 = (MD + 1) / 2;
    float2 acc[ND2];
#pragma unroll
    for (int i = 0; i < ND2; ++i) acc[i] = make_float2(0.f, 0.f);
    float lsum = 0.f;
#pragma unroll 4
    for (int t = warp; t < n; t += NW) {
        const float p = sc[t];
        lsum += p;
        const KV* vr = reinterpret_cast<const KV*>(ring + (size_t)(t / ATT_CHUNK) * chunk_bytes) +
                       (size_t)ATT_CHUNK * D + (size_t)(t % ATT_CHUNK) * D;
#pragma unroll
        for (int i = 0; i < ND2; ++i) {
            const int d = 2 * (lane + 32 * i);
            if (d + 1 < D) {
                const float2 v = kv_to_float2(vr + d);
                acc[i].x = fmaf(p, v.x, acc[i].x);
                acc[i].y = fmaf(p, v.y, acc[i].y);
            } else if (d < D) {
                acc[i].x = fmaf(p, kv_to_float(vr[d]), acc[i].x);
            }
        }
    }
#pragma unroll
    for (int i = 0; i < ND2; ++i) {
        const int d = 2 * (lane + 32 * i);
        if (d < D) part[warp * (D + 1) + d] = acc[i].x;
        if (d + 1 < D) part[warp * (D + 1) + d + 1] = acc[i].y;
    }
    if (lane == 0) part[warp * (D + 1) + D] = lsum;
    __syncthreads();
    if (tid < D) {
        float num = 0.f, den = 0.f;
#pragma unroll
        for (int w = 0; w < NW; ++w) {
            num += part[w * (D + 1) + tid];
            den += part[w * (D + 1) + D];
        }
        out[tid] = num / den;
    }
    __syncthreads();
}

// ---- per-block context and the phase functions ---------------------------------
// Each phase is a separate (non-inlined) function so that the code one block
// runs per layer stays small and is fetched from the instruction cache rather
// than from L2: the per-layer work is short, and a kernel body with every
// phase inlined is several times larger than the SM's instruction cache.

constexpr int MB_RING = 2;  // mbarriers: 0 QKV | gate/up slot, 1 O | down slot, then the chunk buffers
constexpr int ROLE_NMB = MB_RING + RES_BUFS_MAX;

// Built once per launch by thread 0, in shared memory.
struct RoleCtx {
    float* xf;       // staged floats (RMSNorm gain folded in)
    int8_t* xq;      // their fixed-point planes
    float* xr;       // the raw vector (x for attention blocks, x_b for FFN blocks)
    float* misc;     // attention: q [0,128), new K/V row [128,384), head output [384,512), planes; FFN: planes
    float* red;      // block reductions
    float* ss;       // the warps' shares of sum x^2
    float* cosv;
    float* sinv;
    uint64_t* mb;
    unsigned* fills;
    uint8_t* slot0;  // QKV rows | gate/up rows
    uint8_t* slot1;  // W_o rows | W_down columns
    uint8_t* ring;   // resident K/V chunk buffers
    float* part;     // GEMV partials, attention partials
    float* sc;       // attention scores | the block's SiLU(gate)*up values
    uint64_t* dacc;  // this step's half of the sum words
    BlockState st;
    AttnRows ar;
    int is_attn, ra, or0, or1;  // attention: QKV rows, W_o rows [or0, or1)
    int f, ga, gn;              // FFN: block index, gate/up pairs [ga, ga + gn)
    int sp_g, sp_s, sp_n;       // spread unit: KV group, split, resident chunks (0: no unit)
    int n_att, nchunks;         // positions attended (local rows), their chunks
    int lnew;                   // local row of the new token, -1 when another GPU keeps it
    float qscale;
};

__device__ __forceinline__ uint64_t* role_osum(const RoleParams& P, const RoleCtx& c, int l) {
    return c.dacc + (size_t)(2 * l) * P.Hp;
}
__device__ __forceinline__ uint64_t* role_dsum(const RoleParams& P, const RoleCtx& c, int l) {
    return c.dacc + (size_t)(2 * l + 1) * P.Hp;
}

// ---- bulk copies (the copy thread only) ----
__device__ __forceinline__ void attn_fill_qkv(const RoleParams& P, const RoleCtx& c, int l) {
    fill_slot(c.slot0, P.qkv + ((size_t)l * P.NA + blockIdx.x) * P.ra_stride * P.SH, (uint32_t)c.ra * P.SH, c.mb + 0,
              c.fills + 0);
}
__device__ __forceinline__ void attn_fill_o(const RoleParams& P, const RoleCtx& c, int l) {
    fill_slot(c.slot1, P.o_cols + ((size_t)l * P.NH + c.ar.h) * P.o_slice + (size_t)c.or0 * P.o_dw,
              (uint32_t)((c.or1 - c.or0) * P.o_dw), c.mb + 1, c.fills + 1);
}
// The cached rows (positions below pos) of layer l into the resident buffers.
__device__ __forceinline__ void attn_fill_ring(const RoleParams& P, const StepArgs& A, const RoleCtx& c, int l,
                                            int kv_bytes) {
    const size_t rb = (size_t)P.D * kv_bytes;  // bytes of one K or V row
    const size_t head = (size_t)l * P.NKV + c.ar.g;
#pragma unroll 1
    for (int ch = 0; ch < c.nchunks; ++ch) {
        const int c0 = ch * ATT_CHUNK, c1 = min(c0 + ATT_CHUNK, A.pos);
        if (c1 <= c0) continue;
        uint8_t* kd = c.ring + (size_t)ch * P.chunk_bytes;
        const uint8_t* ks = static_cast<const uint8_t*>(P.kcache) + (head * P.capacity + c0) * rb;
        const uint8_t* vs = static_cast<const uint8_t*>(P.vcache) + (head * P.capacity + c0) * rb;
        const uint32_t bytes = (uint32_t)((c1 - c0) * rb);
        ++c.fills[MB_RING + ch];
        mbar_expect(c.mb + MB_RING + ch, 2 * bytes);
        bulk_load(kd, ks, bytes, c.mb + MB_RING + ch);
        bulk_load(kd + (size_t)ATT_CHUNK * rb, vs, bytes, c.mb + MB_RING + ch);
    }
}
__device__ __forceinline__ void ffn_fill_gu(const RoleParams& P, const RoleCtx& c, int l) {
    fill_slot(c.slot0, P.layers[l].gu + (size_t)c.ga * 2 * P.SH, (uint32_t)c.gn * 2 * P.SH, c.mb + 0, c.fills + 0);
}
__device__ __forceinline__ void ffn_fill_down(const RoleParams& P, const RoleCtx& c, int l) {
    fill_slot(c.slot1, P.down_cols + ((size_t)l * P.NG + c.f) * P.down_slice, (uint32_t)P.down_slice, c.mb + 1,
              c.fills + 1);
}

// ---- staging of a GEMV input ----
// x = the sum words `sums` (complete at `expect` contributions), after a
// coarse wait until `expect - coarse` have arrived; per warp: raw values to xr,
// the gain folded in, fixed-point planes with the warp's own scale. Returns
// the warp's scale, or a negative value when a wait ran out.
__device__ __forceinline__ float role_stage(const RoleParams& P, const RoleCtx& c, const uint64_t* sums, int expect,
                                         int coarse, const float* gain) {
    const unsigned first = expect > coarse ? (unsigned)(expect - coarse) : 0u;
    if (!coarse_wait(sums + (blockIdx.x * 37) % P.H, first, c.st)) return -1.f;
    float wsc = 1.f;
    const bool ok = warp_stage_sum<false>(sums, (unsigned)expect, P.H, c.xr, c.xf, c.xq, P.xq_plane, P.Kh / 16, gain,
                                          c.ss, wsc, c.st);
    return ok ? wsc : -1.f;
}
// Layer 0 of an attention block: x is the embedding row of the token.
__device__ __forceinline__ float role_stage_embed(const RoleParams& P, const RoleCtx& c, int token, const float* gain) {
    const uint8_t* er = P.embed + (size_t)token * P.SH;
    float wsc = 1.f;
    const bool ok = warp_stage<2, true>(nullptr, er, row_scale(er, P.Kh), P.H, 0u, c.xr, c.xf, c.xq, P.xq_plane,
                                        P.Kh / 16, gain, c.ss, wsc, c.st);
    return ok ? wsc : -1.f;
}

// RoPE cos/sin of this position (src/model.cpp:269-274 cached, src/kernels.cpp:138-149 direct).
__device__ __forceinline__ void role_rope_table(const RoleParams& P, const StepArgs& A, float* cosv, float* sinv) {
    const int j = threadIdx.x;
    if (j < P.D / 2) {
        const float angle =
            P.cached_rope ? __fmul_rn((float)A.pos, P.rope_inv[j]) : __fdiv_rn((float)A.pos, P.rope_den[j]);
        sincosf(angle, &sinv[j], &cosv[j]);
    }
}

// ---- attention block phases ----
// One thread per RoPE pair of the block's QKV rows: row totals (partials of
// the GEMV) times 1/rms and the row scale, plus the bias; RoPE for q and k;
// q into misc[0, D) (scaled for the softmax in base 2) and into its tagged
// words for the other half; k/v into the group's tagged words and the cache.
template <typename KV>
__device__ __forceinline__ void attn_epilogue(const RoleParams& P, const StepArgs& A, const RoleCtx& c, int l,
                                           uint32_t tag) {
    const int p = threadIdx.x;
    if (p >= c.ra / 2) return;
    const int D = P.D, half = D / 2;
    const AttnRows& ar = c.ar;
    const float inv = rms_inv(c.ss, P.H, P.eps);
    const uint8_t* r0 = c.slot0 + (size_t)(2 * p) * P.SH;
    float y0 = gemv_row(c.part, c.ra, 2 * p) * inv * row_scale(r0, P.Kh) + row_bias(r0, P.Kh);
    float y1 = gemv_row(c.part, c.ra, 2 * p + 1) * inv * row_scale(r0 + P.SH, P.Kh) + row_bias(r0 + P.SH, P.Kh);
    const bool isq = p < ar.nq;
    const int u = isq ? ar.q0 + p : ar.kv0 + (p - ar.nq);  // q pair j, or k/v pair u
    const int kind = isq ? 0 : (u < half ? 1 : 2);
    const int j = kind == 2 ? u - half : u;
    if (kind < 2) {
        const float sn = c.sinv[j], cs = c.cosv[j];
        const float a0 = y0, a1 = y1;
        y0 = __fsub_rn(__fmul_rn(a0, cs), __fmul_rn(a1, sn));
        y1 = __fadd_rn(__fmul_rn(a1, cs), __fmul_rn(a0, sn));
    }
    if (kind == 0) {
        c.misc[j] = y0 * c.qscale;
        c.misc[j + half] = y1 * c.qscale;
        ll_store(P.ll_q + (size_t)ar.h * D + j, y0, tag);
        ll_store(P.ll_q + (size_t)ar.h * D + j + half, y1, tag);
    } else {
        if (c.lnew >= 0) {
            KV* cache = static_cast<KV*>(kind == 1 ? P.kcache : P.vcache) +
                        (((size_t)l * P.NKV + ar.g) * P.capacity + c.lnew) * D;
            kv_store(cache + j, y0);
            kv_store(cache + j + half, y1);
        }
        uint64_t* nw = P.ll_kv + (size_t)ar.g * 2 * D + (kind == 1 ? 0 : D);
        ll_store(nw + j, round_to(y0, KV()), tag);
        ll_store(nw + j + half, round_to(y1, KV()), tag);
    }
}

// The other half's q values and the group's new K/V row (one round trip,
// every load in flight), the resident cached rows of layer l, and the new row
// written into its chunk buffer. Returns false when a wait ran out (uniform).
template <typename KV>
__device__ __forceinline__ bool attn_gather(const RoleParams& P, const StepArgs& A, const RoleCtx& c, int l,
                                         uint32_t tag) {
    const int D = P.D, half = D / 2, t = threadIdx.x;
    const AttnRows& ar = c.ar;
    float* sq = c.misc;
    float* s_new = c.misc + 128;
    {
        const int pq0 = ar.s ? 0 : P.q_first, pnq = ar.s ? P.q_first : half - P.q_first;
        const int nq_words = 2 * pnq;
        if (t < nq_words + 2 * D) {
            const uint64_t* src;
            int dst_j;
            if (t < nq_words) {
                const int jj = pq0 + (t >> 1);
                dst_j = (t & 1) ? jj + half : jj;
                src = P.ll_q + (size_t)ar.h * D + dst_j;
            } else {
                dst_j = -1;
                src = P.ll_kv + (size_t)ar.g * 2 * D + (t - nq_words);
            }
            uint64_t t0 = 0;
            unsigned rounds = 0;
            uint64_t w = ll_load(src);
            while ((uint32_t)(w >> 32) != tag) {
                if ((++rounds & 7u) == 0 && wait_expired(c.st, t0)) break;
                w = ll_load(src);
            }
            const float v = __uint_as_float((uint32_t)w);
            if (dst_j >= 0) sq[dst_j] = v * c.qscale;
            else s_new[t - nq_words] = v;  // already rounded to KV by its writer
        }
    }
    if (P.bulk_kv) {
        if (t == 0) {
            uint64_t t0 = 0;
#pragma unroll 1
            for (int ch = 0; ch < c.nchunks; ++ch) {
                if (min(ch * ATT_CHUNK + ATT_CHUNK, A.pos) <= ch * ATT_CHUNK) continue;
                unsigned spins = 0;
                bool expired = false;
                while (!mbar_test(c.mb + MB_RING + ch, (uint32_t)l & 1u))
                    if ((++spins & 63u) == 0 && wait_expired(c.st, t0)) {
                        expired = true;
                        break;
                    }
                if (expired) break;
            }
        }
    } else {
#pragma unroll 1
        for (int e = t; e < A.pos * D; e += NT) {
            const int pt = e / D, j = e % D;
            KV* kd = reinterpret_cast<KV*>(c.ring + (size_t)(pt / ATT_CHUNK) * P.chunk_bytes) +
                     (size_t)(pt % ATT_CHUNK) * D + j;
            const size_t src = (((size_t)l * P.NKV + ar.g) * P.capacity + pt) * D + j;
            kd[0] = static_cast<const KV*>(P.kcache)[src];
            kd[(size_t)ATT_CHUNK * D] = static_cast<const KV*>(P.vcache)[src];
        }
    }
    __syncthreads();
    if (should_abort(c.st)) return false;
    if (t < 2 * D) {
        KV* kb = reinterpret_cast<KV*>(c.ring + (size_t)(A.pos / ATT_CHUNK) * P.chunk_bytes);
        kv_store(kb + (t < D ? 0 : (size_t)ATT_CHUNK * D) + (size_t)(A.pos % ATT_CHUNK) * D + t % D, s_new[t]);
    }
    __syncthreads();
    return true;
}

// One block's share of a sum: rows [r0, r1) of the slot behind mbarrier 1
// (dw bytes each) times the float vector v (zero past its columns), scaled
// per row (rs, as slice_rows), plus fold, added into acc. The slot wait is
// one thread's test; the closing barrier marks the slot consumed. Returns
// false when the slot wait ran out (uniform).
__device__ __forceinline__ bool sum_share(const RoleParams& P, const RoleCtx& c, const float* v, const uint8_t* slot,
                                          int dw, int r0, int r1, const float (&rs)[SLICE_RPT], const float* fold,
                                          uint64_t* acc, uint32_t parity) {
    if (threadIdx.x == 0) {
        uint64_t t0 = 0;
        unsigned spins = 0;
        while (!mbar_test(c.mb + 1, parity))
            if ((++spins & 63u) == 0 && wait_expired(c.st, t0)) break;
    }
    __syncthreads();
    if (should_abort(c.st)) return false;
    slice_rows(slot, dw, r0, r1, v, rs[0], rs[1], rs[2], fold, acc);
    __syncthreads();
    return true;
}

// ---- FFN block phase ----
// SiLU(gate) * up of the block's pairs (src/model.cpp:308) into c.sc[0, dw)
// (zero past gn); the caller's barrier publishes them.
__device__ __forceinline__ void ffn_epilogue(const RoleParams& P, const RoleCtx& c) {
    const int t = threadIdx.x;
    if (t >= P.dw) return;
    float hv = 0.f;
    if (t < c.gn) {
        const float inv = rms_inv(c.ss, P.H, P.eps);
        const uint8_t* r0 = c.slot0 + (size_t)t * 2 * P.SH;
        const float g = gemv_row(c.part, 2 * c.gn, 2 * t) * inv * row_scale(r0, P.Kh);
        const float u = gemv_row(c.part, 2 * c.gn, 2 * t + 1) * inv * row_scale(r0 + P.SH, P.Kh);
        hv = (g / (1.0f + expf(-g))) * u;
    }
    c.sc[t] = hv;
}

// ---- spread attention (positions beyond the attention blocks' buffers) ----------
// The 64-position chunks covering positions 0..pos are dealt round robin to
// the sp_splits units of each KV group: unit (g, s) keeps chunks s, s + sp,
// s + 2 sp, ... (its buffers 0, 1, 2, ...). Every position sits in exactly
// one unit, so each cached K/V byte is read from HBM once per layer for all
// the group's query heads.
__device__ __forceinline__ int sp_chunks(int nch, int split, int splits) {
    return split < nch ? (nch - split + splits - 1) / splits : 0;
}
// A unit's chunk buffers and scratch (queries, new row, maxima, sums, scores).
__device__ __forceinline__ uint8_t* sp_ring(const RoleParams& P, const RoleCtx& c) {
    return c.is_attn ? c.ring : c.slot0 + (P.g_ring - P.g_gu);
}
__device__ __forceinline__ float* sp_scratch(const RoleParams& P, const RoleCtx& c) {
    return reinterpret_cast<float*>(c.is_attn ? c.ring + P.a_sq : c.slot0 + (P.g_sq - P.g_gu));
}
// The cached rows (positions below pos) of the unit's k-th chunk of layer l
// into buffer k % sp_bufs (the copy thread only; a chunk whose rows are all
// past the cache, i.e. the one starting at pos, needs no copy).
// Local rows already in the cache: all attended ones but the new token's.
__device__ __forceinline__ int sp_cached(const RoleCtx& c) { return c.lnew >= 0 ? c.lnew : c.n_att; }
__device__ __forceinline__ bool sp_chunk_cached(const RoleParams& P, const StepArgs& A, const RoleCtx& c, int k) {
    const int t0 = (c.sp_s + k * P.sp_splits) * ATT_CHUNK;
    return min(t0 + ATT_CHUNK, sp_cached(c)) > t0;
}
__device__ __forceinline__ void sp_fill_chunk(const RoleParams& P, const StepArgs& A, const RoleCtx& c, int l, int k,
                                              int kv_bytes) {
    if (!sp_chunk_cached(P, A, c, k)) return;
    const size_t rb = (size_t)P.D * kv_bytes;
    const size_t head = (size_t)l * P.NKV + c.sp_g;
    const int b = k % P.sp_bufs;
    const int t0 = (c.sp_s + k * P.sp_splits) * ATT_CHUNK, t1 = min(t0 + ATT_CHUNK, sp_cached(c));
    uint8_t* kd = sp_ring(P, c) + (size_t)b * P.chunk_bytes;
    const uint32_t bytes = (uint32_t)((t1 - t0) * rb);
    ++c.fills[MB_RING + b];
    mbar_expect(c.mb + MB_RING + b, 2 * bytes);
    bulk_load(kd, static_cast<const uint8_t*>(P.kcache) + (head * P.capacity + t0) * rb, bytes, c.mb + MB_RING + b);
    bulk_load(kd + (size_t)ATT_CHUNK * rb, static_cast<const uint8_t*>(P.vcache) + (head * P.capacity + t0) * rb,
              bytes, c.mb + MB_RING + b);
}
// The first chunks of layer l, one per buffer (the copy thread only).
__device__ __forceinline__ void sp_fill(const RoleParams& P, const StepArgs& A, const RoleCtx& c, int l,
                                       int kv_bytes) {
#pragma unroll 1
    for (int k = 0; k < min(c.sp_n, P.sp_bufs); ++k) sp_fill_chunk(P, A, c, l, k, kv_bytes);
}

// Unit (g, s) of layer l when all its chunks are resident (at most sp_bufs):
// the group's queries and new K/V row (tagged words of the attention blocks),
// its chunks, then for every query head of the group the reference's
// attention (src/kernels.cpp:150-179) restricted to the unit's positions in one
// pass: scores q.k (q pre-scaled by log2(e)/sqrt(D)), the unit's maximum m,
// p = 2^(s - m), their sum l and sum_t p_t V_t, published as (m, l, o) tagged
// words. Scores by a reduce-scatter over 8 lanes per position, P.V by warp
// per position; head dim 64. Returns false when a wait ran out.
template <typename KV, bool TR>
__device__ __forceinline__ bool sp_partial_resident(const RoleParams& P, const StepArgs& A, const RoleCtx& c, int l,
                                          uint32_t tag) {
    constexpr int D = 64;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int hpg = P.NH / P.NKV, g = c.sp_g, SPL = P.sp_splits, np = c.sp_n * ATT_CHUNK;
    uint8_t* ring = sp_ring(P, c);
    float* sq = sp_scratch(P, c);                                                  // [GQA_MAX][D] scaled queries
    float* s_new = sq + GQA_MAX * D;                                      // [2][D] new K, V row
    float* hml = s_new + 2 * D;                                           // [GQA_MAX][2] max, sum
    float* wm = hml + 2 * GQA_MAX;                                        // [NW][GQA_MAX] warp maxima
    float* S = wm + NW * GQA_MAX;                                         // [np][GQA_MAX] scores
    {
        const int nq = hpg * D, nwords = nq + 2 * D;
        for (int i = tid; i < nwords; i += NT) {
            const uint64_t* src = i < nq ? P.ll_q + (size_t)g * nq + i : P.ll_kv + (size_t)g * 2 * D + (i - nq);
            uint64_t t0 = 0;
            unsigned rounds = 0;
            uint64_t w = ll_load(src);
            while ((uint32_t)(w >> 32) != tag) {
                if ((++rounds & 7u) == 0 && wait_expired(c.st, t0)) break;
                w = ll_load(src);
            }
            const float v = __uint_as_float((uint32_t)w);
            if (i < nq) sq[i] = v * c.qscale;
            else s_new[i - nq] = v;  // already rounded to KV by its writer
        }
    }
    if (tid == 0) {
        uint64_t t0 = 0;
#pragma unroll 1
        for (int k = 0; k < c.sp_n; ++k) {
            if (!sp_chunk_cached(P, A, c, k)) continue;
            unsigned spins = 0;
            bool expired = false;
            while (!mbar_test(c.mb + MB_RING + k, (uint32_t)l & 1u))
                if ((++spins & 63u) == 0 && wait_expired(c.st, t0)) {
                    expired = true;
                    break;
                }
            if (expired) break;
        }
    }
    __syncthreads();
    if (should_abort(c.st)) return false;
    rdetail<TR>(P, l, 3, 5);
    // The new row into its chunk buffer, when this unit keeps position pos.
    const int pch = c.lnew / ATT_CHUNK;
    if (c.lnew >= 0 && pch % SPL == c.sp_s && tid < 2 * D) {
        KV* kb = reinterpret_cast<KV*>(ring + (size_t)(pch / SPL) * P.chunk_bytes);
        kv_store(kb + (tid < D ? 0 : (size_t)ATT_CHUNK * D) + (size_t)(c.lnew % ATT_CHUNK) * D + tid % D, s_new[tid]);
    }
    __syncthreads();
    rdetail<TR>(P, l, 2, 3);
    // Scores: warp w takes local positions 4w + (lane / 8) of each 64-position
    // pass; lane q of a position's 8 lanes holds dims 4q..4q+3, 32+4q..+3 of
    // K and forms partial dots for all 8 head slots, then a reduce-scatter
    // over the 8 lanes (exchanges of 4, 2, 1 values) leaves lane q with the
    // full score of head q (head slots past hpg are never stored).
    {
        const int grp = lane >> 3, pp = lane & 7;
        float mw = -INFINITY;  // this lane's head pp
        for (int base = 0; base < np; base += 4 * NW) {
            const int li = base + warp * 4 + grp;  // local position: buffer li / 64, row li % 64
            const int t = (c.sp_s + (li >> 6) * SPL) * ATT_CHUNK + (li & 63);
            const bool valid = li < np && t < c.n_att;
            float kk[8];
            if (valid) {
                const KV* kr = reinterpret_cast<const KV*>(ring + (size_t)(li >> 6) * P.chunk_bytes) + (size_t)(li & 63) * D;
                float a4[4], b4[4];
                load4(kr + 4 * pp, a4);
                load4(kr + 32 + 4 * pp, b4);
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    kk[e] = a4[e];
                    kk[4 + e] = b4[e];
                }
            } else {
#pragma unroll
                for (int e = 0; e < 8; ++e) kk[e] = 0.f;
            }
            float sc[GQA_MAX];
#pragma unroll
            for (int h = 0; h < GQA_MAX; ++h) {
                const float4 qa = *reinterpret_cast<const float4*>(sq + h * D + 4 * pp);
                const float4 qb = *reinterpret_cast<const float4*>(sq + h * D + 32 + 4 * pp);
                float x = qa.x * kk[0];
                x = fmaf(qa.y, kk[1], x);
                x = fmaf(qa.z, kk[2], x);
                x = fmaf(qa.w, kk[3], x);
                x = fmaf(qb.x, kk[4], x);
                x = fmaf(qb.y, kk[5], x);
                x = fmaf(qb.z, kk[6], x);
                sc[h] = fmaf(qb.w, kk[7], x);
            }
            // Reduce-scatter over lanes pp ^ 4, ^ 2, ^ 1.
            const bool u4 = pp & 4, u2 = pp & 2, u1 = pp & 1;
            float r4[4], r2[2];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float send = u4 ? sc[e] : sc[e + 4];
                r4[e] = (u4 ? sc[e + 4] : sc[e]) + __shfl_xor_sync(FULL, send, 4);
            }
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const float send = u2 ? r4[e] : r4[e + 2];
                r2[e] = (u2 ? r4[e + 2] : r4[e]) + __shfl_xor_sync(FULL, send, 2);
            }
            const float total = (u1 ? r2[1] : r2[0]) + __shfl_xor_sync(FULL, u1 ? r2[0] : r2[1], 1);
            if (valid && pp < hpg) {
                S[li * GQA_MAX + pp] = total;
                mw = fmaxf(mw, total);
            }
        }
        mw = fmaxf(mw, __shfl_xor_sync(FULL, mw, 8));
        mw = fmaxf(mw, __shfl_xor_sync(FULL, mw, 16));
        if (lane < hpg) wm[warp * GQA_MAX + lane] = mw;
    }
    __syncthreads();
    rdetail<TR>(P, l, 2, 4);
    // Warp h: the unit's maximum of head h, p = 2^(s - m) in place, their sum.
    if (warp < hpg) {
        float m = lane < NW ? wm[lane * GQA_MAX + warp] : -INFINITY;
        m = warp_max(m);
        float lsum = 0.f;
        for (int li = lane; li < np; li += 32) {
            const int t = (c.sp_s + (li >> 6) * SPL) * ATT_CHUNK + (li & 63);
            float pv = 0.f;
            if (t < c.n_att) {
                pv = ex2_approx(S[li * GQA_MAX + warp] - m);
                lsum += pv;
            }
            S[li * GQA_MAX + warp] = pv;
        }
        lsum = warp_sum(lsum);
        if (lane == 0) {
            hml[2 * warp] = m;
            hml[2 * warp + 1] = lsum;
        }
    }
    __syncthreads();
    rdetail<TR>(P, l, 2, 5);
    // P.V: warp w takes local positions w, w + 16, ...; lane the dimension
    // pair (2 lane, 2 lane + 1) for every head at once (each V pair read once,
    // the position's probabilities as two broadcast float4). Positions past
    // pos have p = 0 and rows past pos are skipped.
    {
        float2 acc[GQA_MAX];
#pragma unroll
        for (int h = 0; h < GQA_MAX; ++h) acc[h] = make_float2(0.f, 0.f);
#pragma unroll 2
        for (int li = warp; li < np; li += NW) {
            const int t = (c.sp_s + (li >> 6) * SPL) * ATT_CHUNK + (li & 63);
            if (t >= c.n_att) continue;  // warp-uniform
            const KV* vr = reinterpret_cast<const KV*>(ring + (size_t)(li >> 6) * P.chunk_bytes) +
                           (size_t)ATT_CHUNK * D + (size_t)(li & 63) * D;
            const float2 v = kv_to_float2(vr + 2 * lane);
            const float4 pa = *reinterpret_cast<const float4*>(S + li * GQA_MAX);
            const float4 pb = *reinterpret_cast<const float4*>(S + li * GQA_MAX + 4);
            const float pr[GQA_MAX] = {pa.x, pa.y, pa.z, pa.w, pb.x, pb.y, pb.z, pb.w};
#pragma unroll
            for (int h = 0; h < GQA_MAX; ++h) {
                acc[h].x = fmaf(pr[h], v.x, acc[h].x);
                acc[h].y = fmaf(pr[h], v.y, acc[h].y);
            }
        }
        __syncthreads();  // every V row is read: buffer 0 takes the warps' shares
        float* shares = reinterpret_cast<float*>(ring);  // [NW][GQA_MAX][D]
#pragma unroll
        for (int h = 0; h < GQA_MAX; ++h)
            if (h < hpg) *reinterpret_cast<float2*>(shares + ((size_t)warp * GQA_MAX + h) * D + 2 * lane) = acc[h];
        __syncthreads();
        if (tid < hpg * D) {
            const int h = tid >> 6, d = tid & 63;
            float o = 0.f;
#pragma unroll
            for (int w = 0; w < NW; ++w) o += shares[((size_t)w * GQA_MAX + h) * D + d];
            uint64_t* pw = P.ll_part + ((size_t)(g * hpg + h) * SPL + c.sp_s) * (D + 2);
            ll_store(pw + 2 + d, o, tag);
            if (d == 0) {
                ll_store(pw, hml[2 * h], tag);
                ll_store(pw + 1, hml[2 * h + 1], tag);
            }
        }
    }
    rdetail<TR>(P, l, 2, 6);
    __syncthreads();  // the chunk buffers are consumed
    rdetail<TR>(P, l, 2, 7);
    return true;
}

// Unit (g, s) of layer l: the group's queries and new K/V row (tagged words of
// the attention blocks), then its chunks one at a time through its buffers
// (chunk k in buffer k % sp_bufs; the copy thread refills a buffer with chunk
// k + sp_bufs once chunk k is consumed), and for every query head of the
// group the reference's attention (src/kernels.cpp:150-179) restricted to the
// unit's positions, as an online softmax: scores q.k (q pre-scaled by
// log2(e)/sqrt(D)), the running maximum m, p = 2^(s - m), the running sum l and
// sum_t p_t V_t, rescaled by 2^(m_old - m_new) when m grows; published as
// (m, l, o) tagged words. Head dim 64. c.fills[ROLE_NMB + b]: the fills of
// buffer b thread 0 has waited for (their phase parity), kept across layers.
// Returns false when a wait ran out.
template <typename KV, bool TR>
__device__ __forceinline__ bool sp_partial(const RoleParams& P, const StepArgs& A, const RoleCtx& c, int l,
                                          uint32_t tag) {
    unsigned* waited = c.fills + ROLE_NMB;
    constexpr int D = 64;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int hpg = P.NH / P.NKV, g = c.sp_g, SPL = P.sp_splits;
    uint8_t* ring = sp_ring(P, c);
    float* sq = sp_scratch(P, c);                  // [GQA_MAX][D] scaled queries
    float* s_new = sq + GQA_MAX * D;      // [2][D] new K, V row
    float* hml = s_new + 2 * D;           // [GQA_MAX][2] running max, sum
    float* wm = hml + 2 * GQA_MAX;        // [NW][GQA_MAX] warp maxima of a chunk
    float* S = wm + NW * GQA_MAX;         // [64][GQA_MAX] a chunk's scores, then p
    float* alpha = S + ATT_CHUNK * GQA_MAX;  // [GQA_MAX] rescale of the running sums
    {
        const int nq = hpg * D, nwords = nq + 2 * D;
        for (int i = tid; i < nwords; i += NT) {
            const uint64_t* src = i < nq ? P.ll_q + (size_t)g * nq + i : P.ll_kv + (size_t)g * 2 * D + (i - nq);
            uint64_t t0 = 0;
            unsigned rounds = 0;
            uint64_t w = ll_load(src);
            while ((uint32_t)(w >> 32) != tag) {
                if ((++rounds & 7u) == 0 && wait_expired(c.st, t0)) break;
                w = ll_load(src);
            }
            const float v = __uint_as_float((uint32_t)w);
            if (i < nq) sq[i] = v * c.qscale;
            else s_new[i - nq] = v;  // already rounded to KV by its writer
        }
        if (tid < GQA_MAX) {
            hml[2 * tid] = -INFINITY;
            hml[2 * tid + 1] = 0.f;
        }
    }
    rdetail<TR>(P, l, 3, 5);
    const int grp = lane >> 3, pp = lane & 7;
    float2 acc[GQA_MAX];  // P.V: warp w's positions, lane's dimension pair, every head
#pragma unroll
    for (int h = 0; h < GQA_MAX; ++h) acc[h] = make_float2(0.f, 0.f);
#pragma unroll 1
    for (int k = 0; k < c.sp_n; ++k) {
        const int b = k % P.sp_bufs;
        const int t0 = (c.sp_s + k * SPL) * ATT_CHUNK, nr = min(ATT_CHUNK, c.n_att - t0);
        uint8_t* buf = ring + (size_t)b * P.chunk_bytes;
        if (tid == 0 && sp_chunk_cached(P, A, c, k)) {
            uint64_t w0 = 0;
            unsigned spins = 0;
            while (!mbar_test(c.mb + MB_RING + b, waited[b] & 1u))
                if ((++spins & 63u) == 0 && wait_expired(c.st, w0)) break;
            ++waited[b];
        }
        __syncthreads();  // the chunk has arrived; the queries are staged
        if (should_abort(c.st)) return false;
        if (c.lnew >= t0 && c.lnew - t0 < ATT_CHUNK) {  // block-uniform: this chunk holds the new token
            // The new row from the tagged words.
            if (tid < 2 * D) {
                KV* kb = reinterpret_cast<KV*>(buf);
                kv_store(kb + (tid < D ? 0 : (size_t)ATT_CHUNK * D) + (size_t)(c.lnew - t0) * D + tid % D, s_new[tid]);
            }
            __syncthreads();
        }
        // Scores: warp w takes rows 4w + (lane / 8); lane q of a row's 8 lanes
        // holds dims 4q..4q+3, 32+4q..+3 of K and forms partial dots for all 8
        // head slots, then a reduce-scatter over the 8 lanes (exchanges of 4,
        // 2, 1 values) leaves lane q with the full score of head q.
        {
            float mw = -INFINITY;  // this lane's head pp
            const int r = warp * 4 + grp;
            const bool valid = r < nr;
            float kk[8];
            if (valid) {
                const KV* kr = reinterpret_cast<const KV*>(buf) + (size_t)r * D;
                float a4[4], b4[4];
                load4(kr + 4 * pp, a4);
                load4(kr + 32 + 4 * pp, b4);
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    kk[e] = a4[e];
                    kk[4 + e] = b4[e];
                }
            } else {
#pragma unroll
                for (int e = 0; e < 8; ++e) kk[e] = 0.f;
            }
            float sc[GQA_MAX];
#pragma unroll
            for (int h = 0; h < GQA_MAX; ++h) {
                const float4 qa = *reinterpret_cast<const float4*>(sq + h * D + 4 * pp);
                const float4 qb = *reinterpret_cast<const float4*>(sq + h * D + 32 + 4 * pp);
                float x = qa.x * kk[0];
                x = fmaf(qa.y, kk[1], x);
                x = fmaf(qa.z, kk[2], x);
                x = fmaf(qa.w, kk[3], x);
                x = fmaf(qb.x, kk[4], x);
                x = fmaf(qb.y, kk[5], x);
                x = fmaf(qb.z, kk[6], x);
                sc[h] = fmaf(qb.w, kk[7], x);
            }
            const bool u4 = pp & 4, u2 = pp & 2, u1 = pp & 1;
            float r4[4], r2[2];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float send = u4 ? sc[e] : sc[e + 4];
                r4[e] = (u4 ? sc[e + 4] : sc[e]) + __shfl_xor_sync(FULL, send, 4);
            }
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const float send = u2 ? r4[e] : r4[e + 2];
                r2[e] = (u2 ? r4[e + 2] : r4[e]) + __shfl_xor_sync(FULL, send, 2);
            }
            const float total = (u1 ? r2[1] : r2[0]) + __shfl_xor_sync(FULL, u1 ? r2[0] : r2[1], 1);
            if (valid && pp < hpg) {
                S[r * GQA_MAX + pp] = total;
                mw = total;
            }
            mw = fmaxf(mw, __shfl_xor_sync(FULL, mw, 8));
            mw = fmaxf(mw, __shfl_xor_sync(FULL, mw, 16));
            if (lane < hpg) wm[warp * GQA_MAX + lane] = mw;
        }
        __syncthreads();
        // Warp h: the new running maximum of head h, p = 2^(s - m) in place,
        // the running sum rescaled and increased.
        if (warp < hpg) {
            float cm = lane < NW ? wm[lane * GQA_MAX + warp] : -INFINITY;
            cm = warp_max(cm);
            const float m_old = hml[2 * warp], m_new = fmaxf(m_old, cm);
            float lsum = 0.f;
            for (int r = lane; r < ATT_CHUNK; r += 32) {
                float pv = 0.f;
                if (r < nr) {
                    pv = ex2_approx(S[r * GQA_MAX + warp] - m_new);
                    lsum += pv;
                }
                S[r * GQA_MAX + warp] = pv;
            }
            lsum = warp_sum(lsum);
            if (lane == 0) {
                const float al = m_old > -INFINITY ? ex2_approx(m_old - m_new) : 0.f;
                alpha[warp] = al;
                hml[2 * warp] = m_new;
                hml[2 * warp + 1] = fmaf(hml[2 * warp + 1], al, lsum);
            }
        }
        __syncthreads();
        // P.V: warp w takes rows w, w + 16, ...; lane the dimension pair
        // (2 lane, 2 lane + 1) for every head at once.
        {
            const float4 aa = *reinterpret_cast<const float4*>(alpha);
            const float4 ab = *reinterpret_cast<const float4*>(alpha + 4);
            const float al[GQA_MAX] = {aa.x, aa.y, aa.z, aa.w, ab.x, ab.y, ab.z, ab.w};
#pragma unroll
            for (int h = 0; h < GQA_MAX; ++h) {
                acc[h].x *= al[h];
                acc[h].y *= al[h];
            }
#pragma unroll 2
            for (int r = warp; r < nr; r += NW) {
                const KV* vr = reinterpret_cast<const KV*>(buf) + (size_t)ATT_CHUNK * D + (size_t)r * D;
                const float2 v = kv_to_float2(vr + 2 * lane);
                const float4 pa = *reinterpret_cast<const float4*>(S + r * GQA_MAX);
                const float4 pb = *reinterpret_cast<const float4*>(S + r * GQA_MAX + 4);
                const float pr[GQA_MAX] = {pa.x, pa.y, pa.z, pa.w, pb.x, pb.y, pb.z, pb.w};
#pragma unroll
                for (int h = 0; h < GQA_MAX; ++h) {
                    acc[h].x = fmaf(pr[h], v.x, acc[h].x);
                    acc[h].y = fmaf(pr[h], v.y, acc[h].y);
                }
            }
        }
        __syncthreads();  // the chunk is consumed
        if (tid == COPY_T && k + P.sp_bufs < c.sp_n) {
            fence_proxy_async();
            sp_fill_chunk(P, A, c, l, k + P.sp_bufs, (int)sizeof(KV));
        }
    }
    rdetail<TR>(P, l, 2, 5);
    // The 16 warps' shares into the chunk buffers (all consumed, no refill
    // pending), then summed.
    float* shares = reinterpret_cast<float*>(ring);  // [NW][GQA_MAX][D]
#pragma unroll
    for (int h = 0; h < GQA_MAX; ++h)
        if (h < hpg) *reinterpret_cast<float2*>(shares + ((size_t)warp * GQA_MAX + h) * D + 2 * lane) = acc[h];
    __syncthreads();
    if (tid < hpg * D) {
        const int h = tid >> 6, d = tid & 63;
        float o = 0.f;
#pragma unroll
        for (int w = 0; w < NW; ++w) o += shares[((size_t)w * GQA_MAX + h) * D + d];
        uint64_t* pw = P.ll_part + ((size_t)(g * hpg + h) * SPL + c.sp_s) * (D + 2);
        ll_store(pw + 2 + d, o, tag);
        if (d == 0) {
            ll_store(pw, hml[2 * h], tag);
            ll_store(pw + 1, hml[2 * h + 1], tag);
        }
    }
    rdetail<TR>(P, l, 2, 6);
    __syncthreads();
    rdetail<TR>(P, l, 2, 7);
    return true;
}

// Attention block of head h in spread mode: the (m, l, o) of every unit of
// its group that holds positions, merged in split order into the head output
// misc[384 .. 384 + 64): weights 2^(m_s - M), sum_s w_s o_s / sum_s w_s l_s.
// The partial table and the merge scratch use the (idle) chunk buffers.
__device__ __forceinline__ bool sp_merge(const RoleParams& P, const StepArgs& A, const RoleCtx& c, int l,
                                        uint32_t tag) {
    constexpr int D = 64, W = D + 2;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int SPL = P.sp_splits, ns = min(c.nchunks, SPL);
    float* table = reinterpret_cast<float*>(c.ring);  // [ns][W]
    float* wgt = table + SPL * W;                      // [ns]
    float* share = wgt + SPL;                          // [8][D + 1]
    float* own = share + 8 * (D + 1);                  // this GPU's (m, l, o) of the head
    float* tab = own + W;                              // [world][W] every GPU's
    const uint64_t* src = P.ll_part + (size_t)c.ar.h * SPL * W;
    {
        constexpr int WT = 8;
        const int nwords = ns * W;
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
                if ((++rounds & 7u) == 0 && wait_expired(c.st, t0)) break;
#pragma unroll
                for (int k = 0; k < WT; ++k)
                    if ((pending >> k) & 1u) w[k] = ll_load(src + base + tid + k * NT);
            }
        }
    }
    __syncthreads();
    if (should_abort(c.st)) return false;
    if (warp == 0) {
        float mx = -INFINITY;
        for (int i = lane; i < ns; i += 32) mx = fmaxf(mx, table[i * W]);
        mx = warp_max(mx);
        for (int i = lane; i < ns; i += 32) wgt[i] = ex2_approx(table[i * W] - mx);
        if (lane == 0) own[0] = mx;  // -inf when this GPU keeps no attended position
    }
    __syncthreads();
    {
        const int d = tid & 63, q = tid >> 6;  // q < 8
        float num = 0.f, den = 0.f;
        for (int i = q; i < ns; i += 8) {
            num = fmaf(wgt[i], table[i * W + 2 + d], num);
            if (d == 0) den = fmaf(wgt[i], table[i * W + 1], den);
        }
        share[q * (D + 1) + d] = num;
        if (d == 0) share[q * (D + 1) + D] = den;
    }
    __syncthreads();
    if (tid < D) {
        float num = 0.f, den = 0.f;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            num += share[q * (D + 1) + tid];
            den += share[q * (D + 1) + D];
        }
        if (P.world == 1) {
            c.misc[384 + tid] = num / den;
        } else {
            own[2 + tid] = num;
            if (tid == 0) own[1] = den;
        }
    }
    __syncthreads();
    if (P.world == 1) return true;
    // KV split: this GPU's (m, l, o) into every GPU's exchange buffer (block
    // s = 0 of the head writes; system-scope tagged words over NVLink), then
    // every GPU's from the local buffer, merged in rank order so that all GPUs
    // get the same head output. Slots alternate with the global layer count, so
    // a GPU one layer ahead writes the other slot.
    const int slot = (int)((A.seq * (unsigned)P.L + (unsigned)l) & 1u), h = c.ar.h, nw = P.world * W;
    if (c.ar.s == 0)
        for (int i = tid; i < nw; i += NT) {
            const int q = i / W, k = i - q * W;
            ll_store_sys(P.peers[q] + (((size_t)slot * P.NH + h) * P.world + P.rank) * W + k, own[k], tag);
        }
    {
        const uint64_t* src = P.exch + ((size_t)slot * P.NH + h) * P.world * W;
        constexpr int WT = 2;  // world * W <= 8 * 66 < 2 * NT
        uint64_t w[WT];
        unsigned pending = 0;
#pragma unroll
        for (int k = 0; k < WT; ++k) {
            const int i = tid + k * NT;
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
                    tab[tid + k * NT] = __uint_as_float((uint32_t)w[k]);
                    pending &= ~(1u << k);
                }
            if (!pending) break;
            if ((++rounds & 7u) == 0 && wait_expired(c.st, t0)) break;
#pragma unroll
            for (int k = 0; k < WT; ++k)
                if ((pending >> k) & 1u) w[k] = ll_load_sys(src + tid + k * NT);
        }
    }
    __syncthreads();
    if (should_abort(c.st)) return false;
    if (tid < D) {
        float mx = -INFINITY;
        for (int q = 0; q < P.world; ++q) mx = fmaxf(mx, tab[q * W]);
        float num = 0.f, den = 0.f;
        for (int q = 0; q < P.world; ++q) {
            const float mq = tab[q * W];
            const float f = mq > -INFINITY ? ex2_approx(mq - mx) : 0.f;
            num = fmaf(f, tab[q * W + 2 + tid], num);
            den = fmaf(f, tab[q * W + 1], den);
        }
        c.misc[384 + tid] = num / den;
    }
    __syncthreads();
    return true;
}

// ---- one layer of each role ----
template <typename KV, int MD, bool TR, int SP>
__device__ __forceinline__ bool attn_layer(const RoleParams& P, const StepArgs& A, const RoleCtx& c, int l, int token,
                                        const float (&rs)[SLICE_RPT]) {
    const int tid = threadIdx.x, ph = 5 * l;
    const uint32_t tag = (A.seq << 8) | (uint32_t)(l + 1);
    const float* in_norm = P.norms + (size_t)l * 2 * P.Kh;
    rdetail<TR>(P, l, 0, 0);
    const float wsc = l == 0 ? role_stage_embed(P, c, token, in_norm)
                             : role_stage(P, c, role_dsum(P, c, l - 1), P.dcontrib, P.coarse_down, in_norm);
    rtrace<TR>(P, 0, ph + 1);
    rdetail_sync<TR>(P, l, 0, 1);
    const bool okg = wsc > 0.f && warp_slot_wait(c.mb + 0, (uint32_t)l & 1u, c.st);
    rdetail_sync<TR>(P, l, 0, 2);
    role_gemv<RA_ROWS_MAX / 16>(c.slot0, P.SH, c.ra, P.Kh / 16, c.xq, P.xq_plane, c.part, wsc, okg);
    rdetail<TR>(P, l, 0, 3);
    if (should_abort(c.st)) return false;
    attn_epilogue<KV>(P, A, c, l, tag);
    __syncthreads();  // the QKV slot is consumed
    rdetail<TR>(P, l, 0, 4);
    if (tid == COPY_T && l + 1 < P.L) {
        fence_proxy_async();
        attn_fill_qkv(P, c, l + 1);
    }
    rtrace<TR>(P, 1, ph + 1);
    rdetail<TR>(P, l, 1, 0);
    if (SP) {
        // Every block attends as a unit; this block then merges its head's
        // partials (its buffers are free once its unit is done) and only then
        // refills them for the next layer.
        rtrace<TR>(P, 0, ph + 2);
        if (c.sp_n && !(SP == 1 ? sp_partial_resident<KV, TR>(P, A, c, l, tag) : sp_partial<KV, TR>(P, A, c, l, tag)))
            return false;
        rdetail<TR>(P, l, 1, 1);
        if (!sp_merge(P, A, c, l, tag)) return false;
        rdetail<TR>(P, l, 1, 2);
        if (tid == COPY_T && c.sp_n && l + 1 < P.L) {
            fence_proxy_async();
            sp_fill(P, A, c, l + 1, (int)sizeof(KV));
        }
    } else {
        if (!attn_gather<KV>(P, A, c, l, tag)) return false;
        rtrace<TR>(P, 0, ph + 2);
        rdetail<TR>(P, l, 1, 1);
        attend_resident<KV, MD>(c.ring, P.chunk_bytes, P.D, c.n_att, c.misc, c.sc, c.part, c.red, c.misc + 384);
        rdetail<TR>(P, l, 1, 2);
        if (tid == COPY_T && P.bulk_kv && l + 1 < P.L) {
            fence_proxy_async();
            attn_fill_ring(P, A, c, l + 1, (int)sizeof(KV));
        }
    }
    rtrace<TR>(P, 1, ph + 2);
    rtrace<TR>(P, 0, ph + 3);
    rdetail<TR>(P, l, 2, 0);
    if (!sum_share(P, c, c.misc + 384, c.slot1, P.o_dw, c.or0, c.or1, rs, c.ar.h == 0 ? c.xr : nullptr,
                   role_osum(P, c, l), (uint32_t)l & 1u))
        return false;
    rdetail<TR>(P, l, 2, 1);
    if (tid == COPY_T && l + 1 < P.L) {
        fence_proxy_async();
        attn_fill_o(P, c, l + 1);
    }
    rtrace<TR>(P, 1, ph + 3);
    return true;
}

template <typename KV, bool TR, int SP>
__device__ __forceinline__ bool ffn_layer(const RoleParams& P, const StepArgs& A, const RoleCtx& c, int l,
                                       const float (&rs)[SLICE_RPT]) {
    const int tid = threadIdx.x, ph = 5 * l;
    const float* post_norm = P.norms + (size_t)l * 2 * P.Kh + P.Kh;
    if (SP && c.sp_n) {
        // This block's attention unit first: the attention blocks wait for it.
        rdetail<TR>(P, l, 3, 6);
        const uint32_t tag = (A.seq << 8) | (uint32_t)(l + 1);
        if (!(SP == 1 ? sp_partial_resident<KV, TR>(P, A, c, l, tag) : sp_partial<KV, TR>(P, A, c, l, tag)))
            return false;
        rdetail<TR>(P, l, 3, 7);
        if (tid == COPY_T && l + 1 < P.L) {
            fence_proxy_async();
            sp_fill(P, A, c, l + 1, (int)sizeof(KV));
        }
    }
    rtrace<TR>(P, 0, ph + 4);
    rdetail<TR>(P, l, 3, 0);
    const float wsc = role_stage(P, c, role_osum(P, c, l), P.NH, P.coarse_o, post_norm);
    rdetail_sync<TR>(P, l, 3, 1);
    const bool okg = wsc > 0.f && warp_slot_wait(c.mb + 0, (uint32_t)l & 1u, c.st);
    rdetail_sync<TR>(P, l, 3, 2);
    role_gemv<RG_ROWS_MAX / 16>(c.slot0, P.SH, 2 * c.gn, P.Kh / 16, c.xq, P.xq_plane, c.part, wsc, okg);
    rdetail<TR>(P, l, 3, 3);
    if (should_abort(c.st)) return false;
    ffn_epilogue(P, c);
    __syncthreads();  // the gate/up slot is consumed; the SiLU*up values are complete
    rdetail<TR>(P, l, 3, 4);
    if (tid == COPY_T && l + 1 < P.L) {
        fence_proxy_async();
        ffn_fill_gu(P, c, l + 1);
    }
    rtrace<TR>(P, 1, ph + 4);
    rtrace<TR>(P, 0, ph + 5);
    rdetail<TR>(P, l, 4, 0);
    // The last FFN block also adds x_b: the down sums are the next layer's x.
    if (!sum_share(P, c, c.sc, c.slot1, P.dw, 0, P.H, rs, c.f == P.NG - 1 ? c.xr : nullptr,
                   role_dsum(P, c, l), (uint32_t)l & 1u))
        return false;
    rdetail<TR>(P, l, 4, 1);
    if (tid == COPY_T && l + 1 < P.L) {
        fence_proxy_async();
        ffn_fill_down(P, c, l + 1);
    }
    rtrace<TR>(P, 1, ph + 5);
    return true;
}

// ---- final RMSNorm + tied LM head + argmax (src/model.cpp:318-326, src/main.cpp:35-37) ----
// Rows [ha, ha + hn) of this block; the block's best (value, first index) into P.amax.
template <bool TR>
__device__ __forceinline__ bool role_lm_head(const RoleParams& P, const StepArgs& A, const RoleCtx& c) {
    const int G = gridDim.x, b = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int ha = part_lo(b, G, P.V), hn = part_lo(b + 1, G, P.V) - ha;
    const int nch_h = P.Kh / 16, QP = P.xq_plane;
    float best_v = -INFINITY;
    int best_i = 0x7fffffff;
    bool ok = true;
    if (hn) {
        Staged sf{1.f, 1.f};
        const unsigned first = P.dcontrib > P.coarse_down ? (unsigned)(P.dcontrib - P.coarse_down) : 0u;
        if (!coarse_wait(role_dsum(P, c, P.L - 1) + (b * 37) % P.H, first, c.st)) ok = false;
        if (ok && !stage_sum<false>(role_dsum(P, c, P.L - 1), (unsigned)P.dcontrib, P.H, nch_h, c.xr, c.xf, c.xq, QP,
                                    P.norms + (size_t)P.L * 2 * P.Kh, c.red, P.eps, sf, c.st))
            ok = false;
        const float inv = sf.inv * sf.scale;
        if (ok) {
            int4 xv[HEAD_MAXC][3];
#pragma unroll
            for (int k = 0; k < HEAD_MAXC; ++k) {
                const int ch = lane + 32 * k;
                if (ch < nch_h) {
                    load_planes(c.xq, QP, ch, xv[k][0], xv[k][1], xv[k][2]);
                } else {
                    xv[k][0] = xv[k][1] = xv[k][2] = make_int4(0, 0, 0, 0);
                }
            }
            rtrace<TR>(P, 0, 5 * P.L + 1);
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
            const int lines = (P.SH + 127) / 128;
            for (int gi = warp; gi < ngroups; gi += NW) {
                if (gi + NW < ngroups) load_group(gi + NW, wn, sn);
                if (gi + 2 * NW < ngroups && lane < HEAD_R * lines) {
                    const int r = ha + (gi + 2 * NW) * HEAD_R + lane / lines;
                    if (r < ha + hn) prefetch_line_l2(P.embed + (size_t)r * P.SH + (size_t)(lane % lines) * 128);
                }
                float vmine = 0.f;
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
            if (should_abort(c.st)) ok = false;
        }
    }
    if (!ok) return false;
    // Each warp's best is uniform across its lanes; merge the warps, then the
    // last block to finish merges the blocks (the first index wins ties).
    if (lane == 0) {
        c.red[warp] = best_v;
        reinterpret_cast<int*>(c.red)[NW + warp] = best_i;
    }
    __syncthreads();
    __shared__ ArgBest s_best;
    __shared__ int s_last;
    if (tid == 0) {
        for (int w = 0; w < NW; ++w) {
            const float v = c.red[w];
            const int i = reinterpret_cast<const int*>(c.red)[NW + w];
            if (better(v, i, best_v, best_i)) {
                best_v = v;
                best_i = i;
            }
        }
        s_best = {best_v, best_i};
    }
    __syncthreads();
    grid_argmax<NT>(s_best, P.amax, P.sync, A.argmax_dev, reinterpret_cast<ArgBest*>(c.misc), &s_last);
    rtrace<TR>(P, 1, 5 * P.L + 1);
    return true;
}

// Warm L2 for the next token, clear the other half of the sum words, and on
// abort wait (bounded) for this block's copies in flight.
template <bool TR>
__device__ __forceinline__ void role_finish(const RoleParams& P, const StepArgs& A, const RoleCtx& c, bool ok) {
    const int G = gridDim.x, b = blockIdx.x, tid = threadIdx.x;
    if (ok && tid == 0) {
        if (c.is_attn) prefetch_l2(P.qkv + (size_t)b * P.ra_stride * P.SH, (uint32_t)c.ra * P.SH);
        else if (c.gn) prefetch_l2(P.layers[0].gu + (size_t)c.ga * 2 * P.SH, (uint32_t)c.gn * 2 * P.SH);
    }
    {
        uint64_t* z = P.dacc + (size_t)(A.par ^ 1) * P.L * 2 * P.Hp;
        const int n = P.L * 2 * P.Hp;
#pragma unroll 1
        for (int i = part_lo(b, G, n) + tid; i < part_lo(b + 1, G, n); i += NT) z[i] = 0ull;
    }
    __syncthreads();
    if (!ok && tid == 0) {
        const uint64_t t0 = globaltimer();
        for (int i = 0; i < ROLE_NMB; ++i) {
            if (!c.fills[i]) continue;
            const uint32_t parity = (c.fills[i] - 1) & 1u;
            while (!mbar_test(c.mb + i, parity) && globaltimer() - t0 < WAIT_LIMIT_NS) {
            }
        }
    }
    rtrace<TR>(P, 0, 5 * P.L + 2);
    rtrace<TR>(P, 1, 5 * P.L + 2);
}

// MD: 32-dim groups of the head dimension a lane covers in the attention
// scores (1: D <= 32, 2: D <= 64, 4: D <= 128).
// SP: 0 resident attention in the attention blocks; 1 spread units whose
// chunks are all resident; 2 spread units that stream their chunks.
template <typename KV, int MD, bool TR, int SP>
__global__ void __launch_bounds__(NT, 1)
    role_step_kernel(const __grid_constant__ RoleParams P, const __grid_constant__ StepArgs A) {
    extern __shared__ __align__(128) uint8_t sm[];
    __shared__ __align__(8) uint64_t mb[ROLE_NMB];
    __shared__ float s_cos[64], s_sin[64];
    __shared__ __align__(16) float red[2 * NW + 8];
    __shared__ float s_ss[NW];
    __shared__ int s_abort;
    __shared__ unsigned s_fills[ROLE_NMB + RES_BUFS_MAX];  // fills issued, then a unit's fills waited for
    RoleCtx c;
    const int b = blockIdx.x, tid = threadIdx.x, H = P.H;
    const bool is_attn = b < P.NA;
    // A dependent LM-head kernel may be scheduled as soon as blocks leave; it
    // waits for this grid's completion before reading anything.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    {
        c.xf = reinterpret_cast<float*>(sm + P.off_xf);
        c.xq = reinterpret_cast<int8_t*>(sm + P.off_xq);
        c.xr = reinterpret_cast<float*>(sm + P.off_xr);
        c.misc = reinterpret_cast<float*>(sm + P.off_misc);
        c.red = red;
        c.ss = s_ss;
        c.cosv = s_cos;
        c.sinv = s_sin;
        c.mb = mb;
        c.fills = s_fills;
        c.slot0 = sm + (is_attn ? P.a_qkv : P.g_gu);
        c.slot1 = sm + (is_attn ? P.a_o : P.g_down);
        c.ring = sm + P.a_ring;
        c.part = reinterpret_cast<float*>(sm + (is_attn ? P.a_part : P.g_part));
        c.sc = reinterpret_cast<float*>(sm + (is_attn ? P.a_sc : P.g_h));
        c.dacc = P.dacc + (size_t)A.par * P.L * 2 * P.Hp;
        c.st = BlockState{&s_abort, P.sync};
        c.is_attn = is_attn;
        c.n_att = A.pos < P.kv_base ? 0 : min(P.kv_end, A.pos + 1) - P.kv_base;
        c.nchunks = (c.n_att + ATT_CHUNK - 1) / ATT_CHUNK;
        c.lnew = A.pos >= P.kv_base && A.pos < P.kv_end ? A.pos - P.kv_base : -1;
        c.qscale = LOG2E / sqrtf((float)P.D);
        if (is_attn) {
            c.ar = attn_rows(P, b);
            c.ra = 2 * (c.ar.nq + c.ar.nkv);
            c.or0 = c.ar.s ? P.o_first : 0;
            c.or1 = c.ar.s ? H : P.o_first;
            c.f = c.ga = c.gn = 0;
        } else {
            c.f = b - P.NA;
            c.ga = part_lo(c.f, P.NG, P.I);
            c.gn = part_lo(c.f + 1, P.NG, P.I) - c.ga;
            c.ra = c.or0 = c.or1 = 0;
        }
        c.sp_g = c.sp_s = c.sp_n = 0;
        if (SP && b < P.NKV * P.sp_splits) {
            c.sp_g = b / P.sp_splits;
            c.sp_s = b % P.sp_splits;
            c.sp_n = sp_chunks(c.nchunks, c.sp_s, P.sp_splits);
        }
    }
    if (tid == COPY_T) {
        s_abort = 0;
        for (int i = 0; i < ROLE_NMB; ++i) mbar_init(mb + i, 1);
        for (int i = 0; i < ROLE_NMB + RES_BUFS_MAX; ++i) s_fills[i] = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    if (tid == COPY_T) {
        if (is_attn) {
            attn_fill_qkv(P, c, 0);
            attn_fill_o(P, c, 0);
            if (P.bulk_kv && !SP) attn_fill_ring(P, A, c, 0, (int)sizeof(KV));
            if (SP && c.sp_n) sp_fill(P, A, c, 0, (int)sizeof(KV));
        } else if (c.gn) {
            ffn_fill_gu(P, c, 0);
            ffn_fill_down(P, c, 0);
            if (SP && c.sp_n) sp_fill(P, A, c, 0, (int)sizeof(KV));
        }
    }
    if (is_attn) {
        role_rope_table(P, A, s_cos, s_sin);
        if (tid < 128) c.misc[384 + tid] = 0.f;  // the head output, zero past D
    }
    __syncthreads();
    rtrace<TR>(P, 0, 0);
    rtrace<TR>(P, 1, 0);

    int token = A.token_dev ? __ldcg(A.token_dev) : A.token;
    if ((unsigned)token >= (unsigned)P.V) {
        if (tid == 0) atomicCAS(&P.sync->error, 0, ERR_TOKEN);
        token = 0;
    }
    bool ok = true;
    const bool idle = !is_attn && c.gn == 0;  // FFN blocks without gate/up rows (tiny models) sit the layers out
    for (int l = 0; l < P.L && !idle; ++l) {
        if (tid == 0 && (A.head || A.head_follows) && l == P.L - 1) {
            // HBM has slack during the last layer: start this block's first LM-head rows into L2.
            const int ha = part_lo(b, gridDim.x, P.V), hn = part_lo(b + 1, gridDim.x, P.V) - ha;
            if (hn) prefetch_slice(P.embed + (size_t)ha * P.SH, (size_t)min(hn, HEAD_L2_ROWS) * P.SH, 0, 1);
        }
        // Row scales of this layer's O (attention) or down (FFN) rows this
        // thread adds: loaded now, used at the end of the layer.
        float rs[SLICE_RPT];
#pragma unroll
        for (int i = 0; i < SLICE_RPT; ++i) {
            const int r = (is_attn ? c.or0 : 0) + tid + i * SLICE_T;
            rs[i] = tid < SLICE_T && r < (is_attn ? c.or1 : H)
                        ? __ldg((is_attn ? P.o_scale : P.down_scale) + (size_t)l * H + r)
                        : 0.f;
        }
        ok = is_attn ? attn_layer<KV, MD, TR, SP>(P, A, c, l, token, rs) : ffn_layer<KV, TR, SP>(P, A, c, l, rs);
        if (!ok) break;
    }
    if (ok && A.head) ok = role_lm_head<TR>(P, A, c);
    role_finish<TR>(P, A, c, ok);
}

}  // namespace dcb
