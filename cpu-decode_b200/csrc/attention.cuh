// Split-KV GQA decode attention for one query position, executed by one
// thread block per (KV head, KV split). Follows the reference's softmax
// attention (src/kernels.cpp:150-179): scores q.k * (1/sqrt(d)), max-subtracted
// exp, normalised, times V. Each split keeps a running (max, sum, unnormalised
// output) over 64-position chunks staged in shared memory; splits are merged
// with a log-sum-exp combine by the last block of the KV group to finish.
#pragma once
#include "device.cuh"

namespace dcb {

constexpr int KV_CHUNK = 64;

// Shared-memory floats needed by attention_unit for head_dim d and g query
// heads per KV head.
__host__ __device__ constexpr int attention_smem_floats(int d, int g) {
    return 2 * KV_CHUNK * (d + 1) + g * d + 4;
}

struct AttnIO {
    const float* q;        // [heads*d] query, already rotated unless rope_inv != nullptr
    const float* rope_inv; // optional: rotate q by pos*rope_inv[j] while staging
    int rope_pos;
    const void* keys;      // [length][kv_heads*d] (this layer)
    const void* values;
    float* out;            // [heads*d]
    float* part;           // [heads][nsplit][d+2] partials when nsplit > 1
    unsigned* group_done;  // [kv_heads] arrival counters (zero between uses)
    int heads, kv_heads, d, length, nsplit, split_len;
};

// One (KV head g, split s) unit. Block-uniform control flow; uses all warps.
template <typename KV>
__device__ void attention_unit(const AttnIO& io, int g, int s, float* sm) {
    const int d = io.d, gq = io.heads / io.kv_heads, kvd = io.kv_heads * d;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    const int ld = d + 1;  // padded row: lane-per-position reads hit distinct banks
    float* sK = sm;
    float* sV = sK + KV_CHUNK * ld;
    float* sQ = sV + KV_CHUNK * ld;
    __shared__ int s_last;
    const KV* kb = static_cast<const KV*>(io.keys);
    const KV* vb = static_cast<const KV*>(io.values);
    const int t0 = s * io.split_len;
    const int t1 = min(io.length, t0 + io.split_len);
    const float scale = 1.0f / sqrtf((float)d);

    __syncthreads();  // the previous unit of this block is done with shared memory
    // Stage the group's queries (rotating them when asked).
    for (int e = threadIdx.x; e < gq * d; e += blockDim.x) {
        const int hl = e / d, j = e % d, h = g * gq + hl;
        float v = __ldcg(io.q + h * d + j);
        if (io.rope_inv) {
            const int half = d / 2, jj = j < half ? j : j - half;
            const float a = __ldcg(io.q + h * d + jj), b = __ldcg(io.q + h * d + jj + half);
            const float angle = __fmul_rn((float)io.rope_pos, io.rope_inv[jj]);
            float sn, cs;
            sincosf(angle, &sn, &cs);
            v = j < half ? __fsub_rn(__fmul_rn(a, cs), __fmul_rn(b, sn))
                         : __fadd_rn(__fmul_rn(b, cs), __fmul_rn(a, sn));
        }
        sQ[hl * d + j] = v;
    }

    // Per warp: one query head at a time (gq <= nwarps in practice; loop otherwise).
    constexpr int MAXD = 4;  // d <= 128: dims lane + 32*k
    for (int hb = 0; hb < gq; hb += nwarps) {
        const int hl = hb + warp;
        const bool active = hl < gq;
        float m_run = -INFINITY, l_run = 0.f;
        float o[MAXD];
#pragma unroll
        for (int k = 0; k < MAXD; ++k) o[k] = 0.f;
        for (int c0 = t0; c0 < t1; c0 += KV_CHUNK) {
            const int n = min(KV_CHUNK, t1 - c0);
            __syncthreads();  // previous chunk fully consumed (and sQ written)
            for (int e = threadIdx.x; e < n * d; e += blockDim.x) {
                const int t = e / d, j = e % d;
                const size_t off = (size_t)(c0 + t) * kvd + (size_t)g * d + j;
                sK[t * ld + j] = kv_load(kb + off);
                sV[t * ld + j] = kv_load(vb + off);
            }
            __syncthreads();
            if (active) {
                const float* qh = sQ + hl * d;
                float sc[2];
#pragma unroll
                for (int i = 0; i < 2; ++i) {
                    const int t = lane + 32 * i;
                    float dot = 0.f;
                    if (t < n) {
                        const float* kr = sK + t * ld;
                        for (int j = 0; j < d; ++j) dot = fmaf(qh[j], kr[j], dot);
                        sc[i] = dot * scale;
                    } else {
                        sc[i] = -INFINITY;
                    }
                }
                const float m_new = fmaxf(m_run, warp_max(fmaxf(sc[0], sc[1])));
                const float alpha = expf(m_run - m_new);
                float p[2];
#pragma unroll
                for (int i = 0; i < 2; ++i) p[i] = (lane + 32 * i < n) ? expf(sc[i] - m_new) : 0.f;
                l_run = l_run * alpha + warp_sum(p[0] + p[1]);
#pragma unroll
                for (int k = 0; k < MAXD; ++k) o[k] *= alpha;
                for (int t = 0; t < n; ++t) {
                    const float pt = __shfl_sync(FULL, p[t >> 5], t & 31);
                    const float* vr = sV + t * ld;
#pragma unroll
                    for (int k = 0; k < MAXD; ++k) {
                        const int j = lane + 32 * k;
                        if (j < d) o[k] = fmaf(pt, vr[j], o[k]);
                    }
                }
                m_run = m_new;
            }
        }
        if (active) {
            const int h = g * gq + hl;
            if (io.nsplit == 1) {
                const float inv = 1.0f / l_run;
#pragma unroll
                for (int k = 0; k < MAXD; ++k) {
                    const int j = lane + 32 * k;
                    if (j < d) io.out[h * d + j] = o[k] * inv;
                }
            } else {
                float* pp = io.part + ((size_t)h * io.nsplit + s) * (d + 2);
                if (lane == 0) { pp[0] = m_run; pp[1] = l_run; }
#pragma unroll
                for (int k = 0; k < MAXD; ++k) {
                    const int j = lane + 32 * k;
                    if (j < d) pp[2 + j] = o[k];
                }
            }
        }
    }
    if (io.nsplit == 1) return;

    // Last block of this KV group to finish merges all splits of its heads.
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        const unsigned prev = atomicAdd(io.group_done + g, 1u);
        s_last = (prev == (unsigned)io.nsplit - 1);
        if (s_last) __threadfence();
    }
    __syncthreads();
    if (!s_last) return;
    for (int hl = warp; hl < gq; hl += nwarps) {
        const int h = g * gq + hl;
        const float* base = io.part + (size_t)h * io.nsplit * (d + 2);
        float m = -INFINITY;
        for (int i = lane; i < io.nsplit; i += 32) m = fmaxf(m, __ldcg(base + (size_t)i * (d + 2)));
        m = warp_max(m);
        float lsum = 0.f;
        for (int i = lane; i < io.nsplit; i += 32) {
            const float* pp = base + (size_t)i * (d + 2);
            lsum += expf(__ldcg(pp) - m) * __ldcg(pp + 1);
        }
        lsum = warp_sum(lsum);
        const float inv = 1.0f / lsum;
        for (int j = lane; j < d; j += 32) {
            float acc = 0.f;
            for (int i = 0; i < io.nsplit; ++i) {
                const float* pp = base + (size_t)i * (d + 2);
                acc = fmaf(expf(__ldcg(pp) - m), __ldcg(pp + 2 + j), acc);
            }
            io.out[h * d + j] = acc * inv;
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) io.group_done[g] = 0;  // ready for the next use
}

}  // namespace dcb
