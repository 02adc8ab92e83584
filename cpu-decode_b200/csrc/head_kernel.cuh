// Final RMSNorm + tied LM head + argmax as a kernel of its own, chained to the
// step kernel by programmatic dependent launch (src/model.cpp:318-326 and the
// caller's argmax, src/main.cpp:35-37).
//
// The step kernel keeps one block per SM with most of shared memory; the LM
// head (151936 rows, 136 MB) is a pure stream and wants as many bytes in
// flight as possible: here two 512-thread blocks per SM, each warp taking
// HEADK_R rows at a time with all of a lane's 16-byte loads issued together.
// Every block stages x (the down sums of the last layer, complete once the
// step kernel has finished) as fixed-point planes, reduces its rows, keeps
// its best (value, first index), and the last block to finish merges them.
#pragma once
#include "step_kernel.cuh"

namespace dcb {

constexpr int HEADK_NT = 512, HEADK_NW = HEADK_NT / 32;
constexpr int HEADK_R = 4;  // rows a warp reduces at a time
constexpr int HEADK_C = 2;  // 16-byte chunks per lane of a row (hidden <= 1024)

struct HeadParams {
    int H, Kh, SH, V, L, Hp;
    float eps;
    unsigned expect;          // contributions of a complete down sum word
    const uint8_t* embed;     // V packed rows [int8 x Kh | scale | bias | pad]
    const float* final_norm;  // [Kh]
    const uint64_t* dacc;     // sum words [2 halves][L][2][Hp]
    float* logits;
    ArgBest* amax;            // [grid]
    Sync* sync;
};

struct HeadArgs {
    int par;              // half of the sum words the step used
    int* argmax_dev;      // or null
    float* host_logits;   // mapped pinned host memory, or null
};

__device__ __forceinline__ void griddep_wait_head() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__global__ void __launch_bounds__(HEADK_NT, 2) head_kernel(const __grid_constant__ HeadParams P,
                                                            const __grid_constant__ HeadArgs A) {
    extern __shared__ __align__(16) int8_t xq[];  // planes hi | mid | lo, Kh bytes each
    __shared__ float red[2 * HEADK_NW];
    __shared__ ArgBest wbest[HEADK_NW];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, G = gridDim.x, b = blockIdx.x;
    const int H = P.H, Kh = P.Kh, nch = Kh / 16;
    griddep_wait_head();  // the step kernel has finished: its down sums are complete and visible

    // x = the last layer's down sums; the final norm's gain folded in before quantising.
    const uint64_t* xs = P.dacc + ((size_t)A.par * P.L * 2 + 2 * (P.L - 1) + 1) * P.Hp;
    float ss = 0.f, mx = 0.f;
    float xg[2];
    bool complete = true;
#pragma unroll
    for (int k = 0; k < 2; ++k) {
        const int j = tid + k * HEADK_NT;
        xg[k] = 0.f;
        if (j < H) {
            const uint64_t w = __ldcg(xs + j);
            complete &= dacc_count(w) == P.expect;
            const float v = dacc_value(w);
            ss = fmaf(v, v, ss);
            xg[k] = v * __ldg(P.final_norm + j);
            mx = fmaxf(mx, fabsf(xg[k]));
        }
    }
    if (!complete) atomicCAS(&P.sync->error, 0, ERR_WAIT);
    ss = warp_sum(ss);
    mx = warp_max(mx);
    if (lane == 0) {
        red[warp] = ss;
        red[HEADK_NW + warp] = mx;
    }
    __syncthreads();
    float tot = 0.f, M = 0.f;
#pragma unroll
    for (int w = 0; w < HEADK_NW; ++w) {
        tot += red[w];
        M = fmaxf(M, red[HEADK_NW + w]);
    }
    const float inv = __frsqrt_rn(tot / (float)H + P.eps);  // src/kernels.cpp:132-137
    const float rs = M > 0.f ? FIX_MAX * __frcp_rn(M) : 0.f;
    const float xscale = M > 0.f ? __frcp_rn(rs) : 1.f;
    __syncthreads();
    {
        // Planes from the gain-folded values: each thread holds elements tid
        // and tid + NT, a quad needs 4 adjacent ones, so they pass through
        // shared memory once.
        __shared__ __align__(16) float xv[1024];
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const int j = tid + k * HEADK_NT;
            if (j < Kh) xv[j] = j < H ? xg[k] : 0.f;
        }
        __syncthreads();
        for (int quad = tid; quad < Kh / 4; quad += HEADK_NT) {
            const float4 v4 = reinterpret_cast<const float4*>(xv)[quad];
            uint32_t ph, pm, pl;
            fix_pack4(v4, rs, ph, pm, pl);
            reinterpret_cast<uint32_t*>(xq)[quad] = ph;
            reinterpret_cast<uint32_t*>(xq + Kh)[quad] = pm;
            reinterpret_cast<uint32_t*>(xq + 2 * Kh)[quad] = pl;
        }
        __syncthreads();
    }
    const float fin = inv * xscale;

    // Row groups of HEADK_R interleaved over every warp of the grid. Lane q
    // finishes row r0 + q of a group (scale, logit, store) and keeps the best
    // of the rows it finished; the lanes' bests are merged below.
    float best_v = -INFINITY;
    int best_i = 0x7fffffff;
    const int stride = G * HEADK_NW * HEADK_R;
    for (int r0 = (b * HEADK_NW + warp) * HEADK_R; r0 < P.V; r0 += stride) {
        // Lane q < HEADK_R: the scale of row r0 + q, in flight with the weights.
        const float my_scale =
            lane < HEADK_R && r0 + lane < P.V
                ? __ldg(reinterpret_cast<const float*>(P.embed + (size_t)(r0 + lane) * P.SH + Kh))
                : 0.f;
        int ah[HEADK_R], am[HEADK_R], al[HEADK_R];
#pragma unroll
        for (int q = 0; q < HEADK_R; ++q) ah[q] = am[q] = al[q] = 0;
        for (int c0 = lane; c0 < nch; c0 += 32 * HEADK_C) {
            int4 wv[HEADK_C][HEADK_R];
#pragma unroll
            for (int u = 0; u < HEADK_C; ++u)
#pragma unroll
                for (int q = 0; q < HEADK_R; ++q) {
                    const int c = c0 + 32 * u;
                    wv[u][q] = (c < nch && r0 + q < P.V) ? ld_stream(P.embed + (size_t)(r0 + q) * P.SH + (size_t)c * 16)
                                                         : make_int4(0, 0, 0, 0);
                }
#pragma unroll
            for (int u = 0; u < HEADK_C; ++u) {
                const int c = c0 + 32 * u;
                if (c < nch) {
                    int4 h, m, l;
                    load_planes(xq, Kh, c, h, m, l);
#pragma unroll
                    for (int q = 0; q < HEADK_R; ++q) dp4a16(wv[u][q], h, m, l, ah[q], am[q], al[q]);
                }
            }
        }
#pragma unroll
        for (int q = 0; q < HEADK_R; ++q) {
            const float d = warp_sum(planes_to_float(ah[q], am[q], al[q]));
            const int r = r0 + q;
            if (lane == q && r < P.V) {
                const float v = d * my_scale * fin;
                P.logits[r] = v;
                if (A.host_logits) A.host_logits[r] = v;
                if (better(v, r, best_v, best_i)) {
                    best_v = v;
                    best_i = r;
                }
            }
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(FULL, best_v, o);
        const int oi = __shfl_xor_sync(FULL, best_i, o);
        if (better(ov, oi, best_v, best_i)) {
            best_v = ov;
            best_i = oi;
        }
    }
    // The block's best, then the grid's (the last block merges, block-parallel).
    __shared__ ArgBest s_best;
    __shared__ int s_last;
    if (lane == 0) wbest[warp] = {best_v, best_i};
    __syncthreads();
    if (tid == 0) {
        for (int w = 0; w < HEADK_NW; ++w)
            if (better(wbest[w].v, wbest[w].i, best_v, best_i)) {
                best_v = wbest[w].v;
                best_i = wbest[w].i;
            }
        s_best = {best_v, best_i};
    }
    __syncthreads();
    grid_argmax<HEADK_NT>(s_best, P.amax, P.sync, A.argmax_dev, wbest, &s_last);
}

}  // namespace dcb
