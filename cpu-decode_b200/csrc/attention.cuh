// Split-KV GQA decode attention for one query position (the isolated
// operator): one thread block per (KV head, KV split) takes all query heads
// of its group over the split's positions, so each staged K/V byte serves every
// head of the group. Follows the reference's softmax attention
// (src/kernels.cpp:150-179): scores q.k / sqrt(d), max-subtracted exp,
// normalised, times V; here in base 2 (scores scaled by log2(e)/sqrt(d), ex2).
// K/V arrive in 64-position chunks, double-buffered with 16-byte cp.async.
// With several splits, attention_combine_kernel merges the per-split
// (max, sum, unnormalised output) in split order.
#pragma once
#include "device.cuh"

namespace dcb {

constexpr int AT_NT = 512;       // threads per block
constexpr int AT_NW = AT_NT / 32;
constexpr int AT_T = 64;         // positions per staged chunk (4 per warp, 8 lanes each)
constexpr int AT_GH = 8;         // query heads per pass over the split
constexpr int AT_MAXD = 4;       // head_dim <= 128: lane owns dims lane + 32k

struct AttnIO {
    const float* q;       // [heads*d] query
    const void* keys;     // [length][kv_heads*d] rows of KV
    const void* values;
    float* out;           // [heads*d]
    float* part;          // [heads][nsplit][d+2] (max, sum, output) per split when nsplit > 1
    float rope_theta;     // > 0: rotate q (split halves) by position length-1 while staging
    int heads, kv_heads, d, length, nsplit, split_len;
};

// Dynamic shared memory of attention_split_kernel for head_dim d, KV element
// size es and gq query heads per KV head.
__host__ __device__ constexpr size_t attention_smem_bytes(int d, int es, int gq) {
    return 2 * 2 * (size_t)AT_T * d * es                       // two chunk buffers of K and V rows
           + (size_t)gq * d * sizeof(float)                    // scaled queries
           + (size_t)AT_NW * AT_GH * (d + 2) * sizeof(float);  // warp partials of a head pass
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)),
                 "l"(src)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ float at_ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ void at_load4(const float* p, float (&o)[4]) {
    const float4 v = *reinterpret_cast<const float4*>(p);
    o[0] = v.x, o[1] = v.y, o[2] = v.z, o[3] = v.w;
}
__device__ __forceinline__ void at_load4(const __half* p, float (&o)[4]) {
    const uint2 v = *reinterpret_cast<const uint2*>(p);
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&v.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&v.y));
    o[0] = a.x, o[1] = a.y, o[2] = b.x, o[3] = b.y;
}
__device__ __forceinline__ float at_float(float v) { return v; }
__device__ __forceinline__ float at_float(__half v) { return __half2float(v); }
// Two adjacent elements (8- or 4-byte aligned) as FP32.
__device__ __forceinline__ float2 at_float2(const float* p) { return *reinterpret_cast<const float2*>(p); }
__device__ __forceinline__ float2 at_float2(const __half* p) {
    return __half22float2(*reinterpret_cast<const __half2*>(p));
}

// The pass over one split shared by the isolated operator and the batched
// engine: K/V rows t0..t1-1 of one KV head (row t at kg + t*rs and vg + t*rs),
// all gq query heads of its group, the queries already scaled by
// log2(e)/sqrt(d) in shared memory after the two chunk buffers.
// emit(head in group, j, M, L, acc) receives the split's max, sum and
// unnormalised output of dimension j.
template <typename KV, int DT, typename Emit>
__device__ __forceinline__ void attention_split_body(unsigned char* at_sm, const KV* kg, const KV* vg, int d, int rs,
                                                     int t0, int t1, int gq, Emit emit) {
    constexpr int MD = DT ? (DT + 31) / 32 : AT_MAXD;
    const int D = DT ? DT : d;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nchunks = (t1 - t0 + AT_T - 1) / AT_T;
    const size_t buf_elems = 2 * (size_t)AT_T * D;  // K rows then V rows
    KV* bufs = reinterpret_cast<KV*>(at_sm);
    float* sq = reinterpret_cast<float*>(at_sm + 2 * buf_elems * sizeof(KV));
    float* wpart = sq + gq * D;  // [AT_NW][AT_GH][D+2]
    // 16-byte copies need 16-byte rows and bases; otherwise plain loads.
    const bool async16 = (D * sizeof(KV)) % 16 == 0 && (rs * sizeof(KV)) % 16 == 0 &&
                         (reinterpret_cast<uintptr_t>(kg) & 15) == 0 && (reinterpret_cast<uintptr_t>(vg) & 15) == 0;

    auto issue = [&](int c) {
        const int c0 = t0 + c * AT_T, n = min(AT_T, t1 - c0);
        KV* kb = bufs + (size_t)(c & 1) * buf_elems;
        KV* vb = kb + (size_t)AT_T * D;
        if (async16) {
            constexpr int EP = 16 / sizeof(KV);  // elements per 16-byte piece
            const int pieces = D / EP;
            for (int e = threadIdx.x; e < n * pieces; e += AT_NT) {
                const int t = e / pieces, pc = e - t * pieces;
                const size_t src = (size_t)(c0 + t) * rs + (size_t)pc * EP;
                cp_async16(kb + (size_t)t * D + pc * EP, kg + src);
                cp_async16(vb + (size_t)t * D + pc * EP, vg + src);
            }
        } else {
            for (int e = threadIdx.x; e < n * D; e += AT_NT) {
                const int t = e / D, j = e - t * D;
                kb[(size_t)t * D + j] = kg[(size_t)(c0 + t) * rs + j];
                vb[(size_t)t * D + j] = vg[(size_t)(c0 + t) * rs + j];
            }
        }
        cp_async_commit();
    };

    const int grp = lane >> 3, part = lane & 7;
    for (int hb = 0; hb < gq; hb += AT_GH) {
        const int nh = min(AT_GH, gq - hb);
        float m_run[AT_GH], l_run[AT_GH], o[AT_GH][MD];
#pragma unroll
        for (int hh = 0; hh < AT_GH; ++hh) {
            m_run[hh] = -INFINITY;
            l_run[hh] = 0.f;
#pragma unroll
            for (int k = 0; k < MD; ++k) o[hh][k] = 0.f;
        }
        __syncthreads();  // queries staged; the previous pass is done with the buffers
        issue(0);
        for (int c = 0; c < nchunks; ++c) {
            if (c + 1 < nchunks) {
                issue(c + 1);
                cp_async_wait<1>();
            } else {
                cp_async_wait<0>();
            }
            __syncthreads();
            const int c0 = t0 + c * AT_T, n = min(AT_T, t1 - c0);
            const KV* kb = bufs + (size_t)(c & 1) * buf_elems;
            const KV* vb = kb + (size_t)AT_T * D;
            const int t = warp * 4 + grp;
            // This lane's K dims of position t: 32k + 4*part + e.
            float kk[MD][4];
#pragma unroll
            for (int k = 0; k < MD; ++k) {
                const int j0 = 32 * k + 4 * part;
                if (t < n && j0 + 3 < D && (D & 3) == 0) {
                    at_load4(kb + (size_t)t * D + j0, kk[k]);
                } else {
#pragma unroll
                    for (int e = 0; e < 4; ++e) kk[k][e] = (t < n && j0 + e < D) ? at_float(kb[(size_t)t * D + j0 + e]) : 0.f;
                }
            }
            float p[AT_GH];
#pragma unroll
            for (int hh = 0; hh < AT_GH; ++hh) {
                p[hh] = 0.f;
                if (hh < nh) {
                    const float* qh = sq + (size_t)(hb + hh) * D;
                    float sc = 0.f;
#pragma unroll
                    for (int k = 0; k < MD; ++k) {
                        const int j0 = 32 * k + 4 * part;
                        if (j0 + 3 < D && (D & 3) == 0) {
                            float qv[4];
                            at_load4(qh + j0, qv);
#pragma unroll
                            for (int e = 0; e < 4; ++e) sc = fmaf(qv[e], kk[k][e], sc);
                        } else {
#pragma unroll
                            for (int e = 0; e < 4; ++e)
                                if (j0 + e < D) sc = fmaf(qh[j0 + e], kk[k][e], sc);
                        }
                    }
                    sc += __shfl_xor_sync(FULL, sc, 4);
                    sc += __shfl_xor_sync(FULL, sc, 2);
                    sc += __shfl_xor_sync(FULL, sc, 1);
                    sc = t < n ? sc : -INFINITY;
                    float cmax = fmaxf(sc, __shfl_xor_sync(FULL, sc, 8));
                    cmax = fmaxf(cmax, __shfl_xor_sync(FULL, cmax, 16));
                    if (cmax > -INFINITY) {
                        const float m_new = fmaxf(m_run[hh], cmax);
                        const float alpha = at_ex2(m_run[hh] - m_new);
                        p[hh] = at_ex2(sc - m_new);
                        float psum = p[hh] + __shfl_xor_sync(FULL, p[hh], 8);
                        psum += __shfl_xor_sync(FULL, psum, 16);
                        l_run[hh] = fmaf(l_run[hh], alpha, psum);
#pragma unroll
                        for (int k = 0; k < MD; ++k) o[hh][k] *= alpha;
                        m_run[hh] = m_new;
                    }
                }
            }
            // V rows of this warp's 4 positions, each read once for all heads.
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int ti = warp * 4 + i;
                if (ti < n) {
                    float vr[MD];
#pragma unroll
                    for (int k = 0; k < MD; ++k)
                        vr[k] = lane + 32 * k < D ? at_float(vb[(size_t)ti * D + lane + 32 * k]) : 0.f;
#pragma unroll
                    for (int hh = 0; hh < AT_GH; ++hh) {
                        const float pi = __shfl_sync(FULL, p[hh], 8 * i);
                        if (hh < nh) {
#pragma unroll
                            for (int k = 0; k < MD; ++k) o[hh][k] = fmaf(pi, vr[k], o[hh][k]);
                        }
                    }
                }
            }
            __syncthreads();  // buffer c & 1 consumed before chunk c + 2 is issued into it
        }
        // Merge the warps: warp w's (m, l, o) per head to shared memory, then
        // thread (hh, j) weights warp w by 2^(m_w - M).
#pragma unroll
        for (int hh = 0; hh < AT_GH; ++hh) {
            if (hh < nh) {
                float* wp = wpart + ((size_t)warp * AT_GH + hh) * (D + 2);
                if (lane == 0) {
                    wp[0] = m_run[hh];
                    wp[1] = l_run[hh];
                }
#pragma unroll
                for (int k = 0; k < MD; ++k)
                    if (lane + 32 * k < D) wp[2 + lane + 32 * k] = o[hh][k];
            }
        }
        __syncthreads();
        for (int e = threadIdx.x; e < nh * D; e += AT_NT) {
            const int hh = e / D, j = e - hh * D;
            float M = -INFINITY;
#pragma unroll
            for (int w = 0; w < AT_NW; ++w) M = fmaxf(M, wpart[((size_t)w * AT_GH + hh) * (D + 2)]);
            float L = 0.f, acc = 0.f;
#pragma unroll
            for (int w = 0; w < AT_NW; ++w) {
                const float* wp = wpart + ((size_t)w * AT_GH + hh) * (D + 2);
                const float f = wp[0] > -INFINITY ? at_ex2(wp[0] - M) : 0.f;
                L = fmaf(f, wp[1], L);
                acc = fmaf(f, wp[2 + j], acc);
            }
            emit(hb + hh, j, M, L, acc);
        }
    }
}

// Queries of KV group g (gq heads of d dims) into sq, rotated at position
// length-1 when asked (cached angle formula of src/model.cpp:222-224,271) and
// scaled by log2(e)/sqrt(d).
__device__ __forceinline__ void at_stage_queries(const AttnIO& io, int g, int gq, int D, float* sq) {
    const float qscale = 1.4426950408889634f / sqrtf((float)D);
    for (int e = threadIdx.x; e < gq * D; e += AT_NT) {
        const int hl = e / D, j = e - hl * D;
        const float* qh = io.q + (size_t)(g * gq + hl) * D;
        float v = qh[j];
        if (io.rope_theta > 0.f) {
            const int half = D / 2, jj = j < half ? j : j - half;
            const float inv = 1.0f / powf(io.rope_theta, (float)(2 * jj) / (float)D);
            const float angle = __fmul_rn((float)(io.length - 1), inv);
            float sn, cs;
            sincosf(angle, &sn, &cs);
            const float a = qh[jj], b = qh[jj + half];
            v = j < half ? __fsub_rn(__fmul_rn(a, cs), __fmul_rn(b, sn)) : __fadd_rn(__fmul_rn(b, cs), __fmul_rn(a, sn));
        }
        sq[e] = v * qscale;
    }
}

// Shared memory of attention_group_kernel: two chunk buffers of K and V rows
// (head_dim 64), the group's scaled queries, the [AT_GH][AT_T] score tile and
// the per-head running max, sum and rescale.
__host__ __device__ constexpr size_t attention_group_smem_bytes(int es, int gq) {
    return 2 * 2 * (size_t)AT_T * 64 * es + (size_t)gq * 64 * sizeof(float) +
           ((size_t)AT_GH * AT_T + 3 * AT_GH) * sizeof(float);
}

// Split-KV attention for head_dim 64 and up to AT_GH query heads per KV head:
// block (KV head g, split s) reads each 64-position chunk of its split once for
// all gq heads. Per chunk, after the copy lands:
//   scores: warp w takes positions 4w..4w+3; the 8 lanes of a position own dims
//     4p..4p+3 and 32+4p..32+4p+3 (8 lanes read 128 contiguous bytes), read K
//     once and, for each head, reduce q.k over the 8 lanes into the score tile;
//   softmax: warp h turns head h's 64 scores into 2^(s - m) with its running
//     max m and adds them to its running sum;
//   P.V: thread (h, j2) rescales and accumulates o_h[2j2], o_h[2j2+1] over the
//     chunk (one 8-byte V load per two FMAs).
// Light on registers, so two blocks share an SM and their copies overlap.
template <typename KV>
__global__ void __launch_bounds__(AT_NT, 2) attention_group_kernel(AttnIO io) {
    extern __shared__ __align__(16) unsigned char at_sm[];
    constexpr int D = 64;
    const int g = blockIdx.x / io.nsplit, s = blockIdx.x % io.nsplit;
    const int gq = io.heads / io.kv_heads, kvd = io.kv_heads * D;
    const int t0 = s * io.split_len, t1 = min(io.length, t0 + io.split_len);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const size_t buf_elems = 2 * (size_t)AT_T * D;
    KV* bufs = reinterpret_cast<KV*>(at_sm);
    float* sq = reinterpret_cast<float*>(at_sm + 2 * buf_elems * sizeof(KV));
    float* tile = sq + gq * D;          // [AT_GH][AT_T]
    float* hm = tile + AT_GH * AT_T;    // [AT_GH] running max
    float* hl = hm + AT_GH;             // running sum
    float* ha = hl + AT_GH;             // rescale of the current chunk
    const KV* kg = static_cast<const KV*>(io.keys) + (size_t)g * D;
    const KV* vg = static_cast<const KV*>(io.values) + (size_t)g * D;
    at_stage_queries(io, g, gq, D, sq);
    if (tid < AT_GH) {
        hm[tid] = -INFINITY;
        hl[tid] = 0.f;
    }
    const bool async16 = (kvd * sizeof(KV)) % 16 == 0 && (reinterpret_cast<uintptr_t>(kg) & 15) == 0 &&
                         (reinterpret_cast<uintptr_t>(vg) & 15) == 0;
    const int nchunks = (t1 - t0 + AT_T - 1) / AT_T;
    auto issue = [&](int c) {
        const int c0 = t0 + c * AT_T, n = min(AT_T, t1 - c0);
        KV* kb = bufs + (size_t)(c & 1) * buf_elems;
        KV* vb = kb + (size_t)AT_T * D;
        if (async16) {
            constexpr int EP = 16 / sizeof(KV);
            constexpr int pieces = D / EP;
            for (int e = tid; e < n * pieces; e += AT_NT) {
                const int t = e / pieces, pc = e - t * pieces;
                const size_t src = (size_t)(c0 + t) * kvd + (size_t)pc * EP;
                cp_async16(kb + (size_t)t * D + pc * EP, kg + src);
                cp_async16(vb + (size_t)t * D + pc * EP, vg + src);
            }
        } else {
            for (int e = tid; e < n * D; e += AT_NT) {
                const int t = e / D, j = e - t * D;
                kb[(size_t)t * D + j] = kg[(size_t)(c0 + t) * kvd + j];
                vb[(size_t)t * D + j] = vg[(size_t)(c0 + t) * kvd + j];
            }
        }
        cp_async_commit();
    };
    const int grp = lane >> 3, part = lane & 7;
    float2 o0 = make_float2(0.f, 0.f), o1 = o0;  // thread (h, j2) = (tid / 32, tid % 32), tid < gq * 32: dims 2j2, 2j2+1
    issue(0);
    for (int c = 0; c < nchunks; ++c) {
        if (c + 1 < nchunks) {
            issue(c + 1);
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();  // chunk c landed for every thread (and the queries are staged)
        const int n = min(AT_T, t1 - (t0 + c * AT_T));
        const KV* kb = bufs + (size_t)(c & 1) * buf_elems;
        const KV* vb = kb + (size_t)AT_T * D;
        {
            const int t = warp * 4 + grp;
            float kk[8];
            if (t < n) {
                float a[4], b[4];
                at_load4(kb + (size_t)t * D + 4 * part, a);
                at_load4(kb + (size_t)t * D + 32 + 4 * part, b);
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    kk[e] = a[e];
                    kk[4 + e] = b[e];
                }
            } else {
#pragma unroll
                for (int e = 0; e < 8; ++e) kk[e] = 0.f;
            }
            for (int h = 0; h < gq; ++h) {
                const float4 q0 = *reinterpret_cast<const float4*>(sq + h * D + 4 * part);
                const float4 q1 = *reinterpret_cast<const float4*>(sq + h * D + 32 + 4 * part);
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
                if (part == 0) tile[h * AT_T + t] = t < n ? sc : -INFINITY;
            }
        }
        __syncthreads();
        if (warp < gq) {
            float* row = tile + warp * AT_T;
            const float s0 = row[lane], s1 = row[lane + 32];
            const float mx = warp_max(fmaxf(s0, s1));
            const float mo = hm[warp], mn = fmaxf(mo, mx);
            const float e0 = at_ex2(s0 - mn), e1 = at_ex2(s1 - mn);
            row[lane] = e0;
            row[lane + 32] = e1;
            const float sum = warp_sum(e0 + e1);
            if (lane == 0) {
                const float al = at_ex2(mo - mn);
                ha[warp] = al;
                hl[warp] = fmaf(hl[warp], al, sum);
                hm[warp] = mn;
            }
        }
        __syncthreads();
        if (tid < gq * 32) {
            const int h = tid >> 5, j2 = tid & 31;
            const float al = ha[h];
            o0.x *= al;
            o0.y *= al;
            o1.x *= al;
            o1.y *= al;
            const float* pr = tile + h * AT_T;
            const KV* vj = vb + 2 * j2;
            int t = 0;
#pragma unroll 2
            for (; t + 4 <= n; t += 4) {
                const float4 pv = *reinterpret_cast<const float4*>(pr + t);
                const float2 v0 = at_float2(vj + (size_t)t * D), v1 = at_float2(vj + (size_t)(t + 1) * D);
                const float2 v2 = at_float2(vj + (size_t)(t + 2) * D), v3 = at_float2(vj + (size_t)(t + 3) * D);
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
                const float2 vt = at_float2(vj + (size_t)t * D);
                o0.x = fmaf(pr[t], vt.x, o0.x);
                o0.y = fmaf(pr[t], vt.y, o0.y);
            }
        }
        __syncthreads();  // buffer c & 1 and the tile consumed before chunk c + 2 and the next scores
    }
    if (tid < gq * 32) {
        const int hh = tid >> 5, h = g * gq + hh, j = 2 * (tid & 31);
        const float a0 = o0.x + o1.x, a1 = o0.y + o1.y;
        if (io.nsplit == 1) {
            io.out[(size_t)h * D + j] = a0 / hl[hh];
            io.out[(size_t)h * D + j + 1] = a1 / hl[hh];
        } else {
            float* pp = io.part + ((size_t)h * io.nsplit + s) * (D + 2);
            if (j == 0) {
                pp[0] = hm[hh];
                pp[1] = hl[hh];
            }
            pp[2 + j] = a0;
            pp[3 + j] = a1;
        }
    }
}

// DT: head_dim known at compile time (64), or 0 for any even head_dim <= 128.
template <typename KV, int DT>
__global__ void __launch_bounds__(AT_NT) attention_split_kernel(AttnIO io) {
    extern __shared__ __align__(16) unsigned char at_sm[];
    const int D = DT ? DT : io.d;
    const int g = blockIdx.x / io.nsplit, s = blockIdx.x % io.nsplit;
    const int gq = io.heads / io.kv_heads, kvd = io.kv_heads * D;
    const int t0 = s * io.split_len, t1 = min(io.length, t0 + io.split_len);
    float* sq = reinterpret_cast<float*>(at_sm + 2 * 2 * (size_t)AT_T * D * sizeof(KV));
    const KV* kg = static_cast<const KV*>(io.keys) + (size_t)g * D;
    const KV* vg = static_cast<const KV*>(io.values) + (size_t)g * D;

    // Queries of the group, rotated at position length-1 when asked (cached
    // angle formula of src/model.cpp:222-224,271), scaled by log2(e)/sqrt(D).
    const float qscale = 1.4426950408889634f / sqrtf((float)D);
    for (int e = threadIdx.x; e < gq * D; e += AT_NT) {
        const int hl = e / D, j = e - hl * D;
        const float* qh = io.q + (size_t)(g * gq + hl) * D;
        float v = qh[j];
        if (io.rope_theta > 0.f) {
            const int half = D / 2, jj = j < half ? j : j - half;
            const float inv = 1.0f / powf(io.rope_theta, (float)(2 * jj) / (float)D);
            const float angle = __fmul_rn((float)(io.length - 1), inv);
            float sn, cs;
            sincosf(angle, &sn, &cs);
            const float a = qh[jj], b = qh[jj + half];
            v = j < half ? __fsub_rn(__fmul_rn(a, cs), __fmul_rn(b, sn)) : __fadd_rn(__fmul_rn(b, cs), __fmul_rn(a, sn));
        }
        sq[e] = v * qscale;
    }
    attention_split_body<KV, DT>(at_sm, kg, vg, D, kvd, t0, t1, gq, [&](int hl, int j, float M, float L, float acc) {
        const int h = g * gq + hl;
        if (io.nsplit == 1) {
            io.out[(size_t)h * D + j] = acc / L;
        } else {
            float* pp = io.part + ((size_t)h * io.nsplit + s) * (D + 2);
            if (j == 0) {
                pp[0] = M;
                pp[1] = L;
            }
            pp[2 + j] = acc;
        }
    });
}

// Merge the splits of head blockIdx.x: out[j] = sum_s 2^(m_s - M) o_s[j] /
// sum_s 2^(m_s - M) l_s. Every load a thread needs is issued before the
// reductions: thread i < nsplit takes split i's (m, l); thread (q, j) of group
// q (groups of d threads) takes o_s[j] of splits q, q + ngroups, ... (up to
// AT_CU of them in registers; more splits loop).
constexpr int AT_CU = 24;
static __global__ void __launch_bounds__(AT_NT) attention_combine_kernel(AttnIO io) {
    __shared__ float s_w[1024];  // 2^(m_s - M) per split (nsplit <= 1024)
    __shared__ float s_red[AT_NT];
    const int h = blockIdx.x, D = io.d, ns = io.nsplit;
    const float* base = io.part + (size_t)h * ns * (D + 2);
    const int ngroups = AT_NT / D;
    const int j = threadIdx.x % D, q = threadIdx.x / D;
    float ov[AT_CU];
#pragma unroll
    for (int u = 0; u < AT_CU; ++u) {
        const int i = q + u * ngroups;
        ov[u] = (q < ngroups && i < ns) ? base[(size_t)i * (D + 2) + 2 + j] : 0.f;
    }
    float mi = -INFINITY, li = 0.f;
    if ((int)threadIdx.x < ns) {
        mi = base[(size_t)threadIdx.x * (D + 2)];
        li = base[(size_t)threadIdx.x * (D + 2) + 1];
    }
    float m = mi;
    for (int i = threadIdx.x + AT_NT; i < ns; i += AT_NT) m = fmaxf(m, base[(size_t)i * (D + 2)]);
    m = warp_max(m);
    if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = m;
    __syncthreads();
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < AT_NW; ++w) M = fmaxf(M, s_red[w]);
    float lsum = 0.f;
    for (int i = threadIdx.x; i < ns; i += AT_NT) {
        const bool own = i == (int)threadIdx.x;
        const float f = at_ex2((own ? mi : base[(size_t)i * (D + 2)]) - M);
        s_w[i] = f;
        lsum = fmaf(f, own ? li : base[(size_t)i * (D + 2) + 1], lsum);
    }
    lsum = warp_sum(lsum);
    __syncthreads();  // s_red's maxima read by every thread before it is reused
    if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = lsum;
    __syncthreads();
    float L = 0.f;
#pragma unroll
    for (int w = 0; w < AT_NW; ++w) L += s_red[w];
    float acc = 0.f;
    if (q < ngroups) {
#pragma unroll
        for (int u = 0; u < AT_CU; ++u) {
            const int i = q + u * ngroups;
            if (i < ns) acc = fmaf(s_w[i], ov[u], acc);
        }
        for (int i = q + AT_CU * ngroups; i < ns; i += ngroups) acc = fmaf(s_w[i], base[(size_t)i * (D + 2) + 2 + j], acc);
    }
    __syncthreads();
    s_red[threadIdx.x] = acc;
    __syncthreads();
    if ((int)threadIdx.x < D) {
        float t = 0.f;
        for (int k = 0; k < ngroups; ++k) t += s_red[k * D + threadIdx.x];
        io.out[(size_t)h * D + threadIdx.x] = t / L;
    }
}

}  // namespace dcb
