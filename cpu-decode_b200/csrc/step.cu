// Host engine behind the C ABI in include/decode_b200.h: uploads the model in
// the step kernel's layout, owns the KV cache and the activation buffers, and
// launches one cooperative step kernel (step_kernel.cuh) per token.
#include "decode_b200.h"
#include "model_view.h"
#include "head_kernel.cuh"
#include "role_kernel.cuh"
#include "step_kernel.cuh"

#include <cuda_runtime.h>
#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <atomic>
#include <memory>
#include <string>
#include <thread>
#include <vector>

namespace dcb {
void set_last_error(const std::string& msg);
}
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
#define DCB_CUDA(call)                                                                                          \
    do {                                                                                                        \
        cudaError_t e_ = (call);                                                                                \
        if (e_ != cudaSuccess) return fail(DCB_ERR_CUDA, std::string(#call ": ") + cudaGetErrorString(e_));     \
    } while (0)

size_t round_up(size_t v, size_t m) { return (v + m - 1) / m * m; }
int ceil_div(int a, int b) { return (a + b - 1) / b; }
// Bytes per row of a column slice of n int8: a multiple of 4 with an odd
// number of 4-byte words, so a warp reading one word of 32 consecutive rows
// touches 32 different shared-memory banks.
int slice_row_bytes(int n) {
    int w = ceil_div(n, 4);
    if (w % 2 == 0) ++w;
    return 4 * w;
}
}  // namespace

struct dcb_engine {
    int device = 0;
    cudaStream_t stream = nullptr;
    bool own_stream = false;
    Params P{};
    int H, I, L, NH, NKV, D, V;
    int kv_dtype = DCB_KV_F32;
    size_t capacity = 0, pos = 0;
    // KV sequence split: this engine keeps positions [kv_base, kv_end) (local
    // rows from 0); one engine alone keeps [0, unbounded).
    size_t kv_base = 0, kv_end = SIZE_MAX;
    bool owns(size_t p) const { return p >= kv_base && p < kv_end; }
    // Positions this engine attends over at position p (its range up to p).
    size_t attended(size_t p) const { return p < kv_base ? 0 : std::min(kv_end, p + 1) - kv_base; }
    unsigned seq = 0;
    std::vector<void*> allocations;
    int grid = 0, smem = 0, sms = 0;
    void* kernel = nullptr;
    int* h_result = nullptr;  // pinned [2]: error, argmax (copied together from Sync)
    uint64_t* trace = nullptr;
    uint64_t launches = 0;
    int par = 0;  // half of the down sums the next step uses
    int split_min = 64;   // positions per attention split, at least (one chunk)
    // Group attention units (one block per KV group and split, all its query
    // heads at once): allowed for this model (gqa_ok), used from group_min
    // attended positions on, splits of at least group_split_min positions.
    bool gqa_ok = false;
    int group_min = 1024, group_split_min = 64;
    // The two-role step kernel (role_kernel.cuh): used for one GPU when every
    // attended position fits in an attention block's resident buffers.
    RoleParams R{};
    bool role_ok = false, role_on = true;
    void* role_kernel = nullptr;
    void* role_kernel_traced = nullptr;
    int role_smem = 0, role_max_pos = 0;
    // Its spread mode (the FFN blocks attend) for positions beyond the
    // attention blocks' buffers, up to role_sp_max_pos (0: not available).
    void* role_kernel_sp = nullptr;  // units with every chunk resident (up to role_sp_resident_pos)
    void* role_kernel_sp_traced = nullptr;
    void* role_kernel_sps = nullptr;  // units streaming their chunks
    void* role_kernel_sps_traced = nullptr;
    int role_sp_max_pos = 0, role_sp_resident_pos = 0;
    // The LM head as its own kernel after a two-role step (head_kernel.cuh),
    // chained by programmatic dependent launch; 2 blocks per SM.
    HeadParams HP{};
    bool head_sep = false;
    int head_grid = 0;
    // Batched prefill context over this engine's KV cache (dcb_prefill).
    dcb_batch* prefill = nullptr;

    ~dcb_engine() {
        cudaSetDevice(device);
        if (prefill) dcb_batch_destroy(prefill);
        if (stream) cudaStreamSynchronize(stream);
        for (void* p : allocations) cudaFree(p);
        if (h_result) cudaFreeHost(h_result);
        if (stream && own_stream) cudaStreamDestroy(stream);
    }
    template <class T>
    int alloc(T** out, size_t count) {
        void* p = nullptr;
        const size_t bytes = round_up(std::max<size_t>(count * sizeof(T), 16), 256);
        cudaError_t e = cudaMalloc(&p, bytes);
        if (e != cudaSuccess) return fail(DCB_ERR_CUDA, std::string("cudaMalloc: ") + cudaGetErrorString(e));
        allocations.push_back(p);
        e = cudaMemset(p, 0, bytes);
        if (e != cudaSuccess) return fail(DCB_ERR_CUDA, std::string("cudaMemset: ") + cudaGetErrorString(e));
        *out = static_cast<T*>(p);
        return 0;
    }
    size_t kv_elem() const { return kv_dtype == DCB_KV_F16 ? 2 : 4; }
};

namespace {

// Packed row: int8 weights zero-padded to K16 bytes, then FP32 scale, FP32 bias, 8 bytes pad.
void pack_row(uint8_t* dst, const int8_t* w, int K, float scale, float bias) {
    std::memcpy(dst, w, K);
    const int K16 = (int)round_up(K, 16);
    std::memset(dst + K, 0, K16 - K);
    std::memcpy(dst + K16, &scale, 4);
    std::memcpy(dst + K16 + 4, &bias, 4);
    std::memset(dst + K16 + 8, 0, 8);
}

// Runs f(i) for every i in [0, n) on up to 16 host threads. The load-time
// packing of the weight layouts uses it: task i writes only its own bytes.
template <class F>
void parallel_for(int n, const F& f) {
    const unsigned hw = std::thread::hardware_concurrency();
    const int T = std::max(1, std::min({n, 16, (int)(hw ? hw : 1)}));
    std::atomic<int> next{0};
    auto work = [&] {
        for (int i; (i = next.fetch_add(1)) < n;) f(i);
    };
    std::vector<std::thread> pool;
    for (int t = 1; t < T; ++t) pool.emplace_back(work);
    work();
    for (auto& t : pool) t.join();
}

// n bytes of host memory for a packed layout, not initialised: each packing
// task zeroes or writes every byte of its own region.
uint8_t* host_bytes(std::unique_ptr<uint8_t[]>& p, size_t n) {
    p.reset(new uint8_t[std::max<size_t>(n, 1)]);
    return p.get();
}

int upload(dcb_engine* e, uint8_t** out, const uint8_t* host, size_t n) {
    uint8_t* d = nullptr;
    if (int rc = e->alloc(&d, n)) return rc;
    DCB_CUDA(cudaMemcpy(d, host, n, cudaMemcpyHostToDevice));
    *out = d;
    return 0;
}
int upload_floats(dcb_engine* e, const float** out, const std::vector<float>& v) {
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
    if (!(m->epsilon > 0) || !std::isfinite(m->epsilon) || !(m->theta > 0) || !std::isfinite(m->theta))
        return fail(DCB_ERR_ARGUMENT, "invalid Qwen dimensions or constants");
    if (m->head_dim > 32 * MAXD) return fail(DCB_ERR_UNSUPPORTED, "head_dim above 128 is not supported");
    if (m->layers > 254) return fail(DCB_ERR_UNSUPPORTED, "more than 254 layers is not supported");
    if (m->hidden > 32 * HEAD_MAXC * 16)
        return fail(DCB_ERR_UNSUPPORTED, "hidden size above 1024 is not supported");
    if (m->hidden > 8192 || m->intermediate > 16384)
        return fail(DCB_ERR_UNSUPPORTED, "hidden size above 8192 or intermediate size above 16384 is not supported");
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

// KV split: one block per (query head, split), at most one unit per block;
// each split covers at least split_min positions (a multiple of 64). From
// group_min positions on (head_dim 64), one block per (KV group, split)
// instead, with at least one split per query head of the group (the splits'
// blocks j < heads per group merge head j). Either way each head's merged
// result is then exchanged with the other GPUs of a KV split the same way.
void choose_split(const dcb_engine* e, int length, int* nsplit, int* split_len, int* group) {
    const int chunks = ceil_div(length, ATT_CHUNK);
    *group = 0;
    if (e->gqa_ok && length >= e->group_min) {
        const int hpg = e->NH / e->NKV;
        const int table_g = std::min(GQA_MERGE_MAX, e->P.wo_off / (int)((e->D + 2) * sizeof(float)));
        const int n = std::max(1, std::min({ceil_div(length, e->group_split_min), e->grid / e->NKV, table_g}));
        const int len = ceil_div(chunks, n) * ATT_CHUNK;
        const int ns = ceil_div(length, len);
        if (ns >= hpg) {
            *group = 1;
            *nsplit = ns;
            *split_len = len;
            return;
        }
    }
    // Split 0 gathers the other splits' (D+2)-float partials into the chunk buffers.
    const int table_max = 1 + e->P.wo_off / (int)((e->D + 2) * sizeof(float));
    const int n = std::max(1, std::min({ceil_div(length, e->split_min), e->grid / e->NH, table_max}));
    *split_len = ceil_div(chunks, n) * ATT_CHUNK;
    *nsplit = ceil_div(length, *split_len);
}

// The two-role kernel takes the step when it is set up and one GPU keeps the
// whole sequence: 1 when every attended position fits in the attention
// blocks' resident buffers, 2 (spread mode) when it fits in the FFN blocks'
// units, else 0.
int use_role(const dcb_engine* e) {
    if (!e->role_ok || !e->role_on) return 0;
    const bool whole = e->P.world == 1 && e->kv_base == 0 && e->kv_end == SIZE_MAX;
    if (whole && e->pos + 1 <= (size_t)e->role_max_pos) return 1;
    // Spread mode: one GPU past the resident buffers, or a GPU of a KV split.
    if (e->role_sp_max_pos > 0 && e->attended(e->pos) <= (size_t)e->role_sp_max_pos) return 2;
    return 0;
}

int launch(dcb_engine* e, int token, const int* token_dev, int head, int* argmax_dev, float* host_logits = nullptr) {
    StepArgs A{};
    A.host_logits = host_logits;
    A.token = token;
    A.token_dev = token_dev;
    A.pos = (int)e->pos;
    A.head = head;
    A.argmax_dev = argmax_dev;
    choose_split(e, (int)e->attended(e->pos), &A.nsplit, &A.split_len, &A.group);
    if (++e->seq >= (1u << 24)) e->seq = 1;  // tags are seq << 8 | layer
    A.seq = e->seq;
    A.par = e->par;
    e->par ^= 1;
    if (const int mode = use_role(e)) {
        const bool sep = head && e->head_sep;
        A.head_follows = sep ? 1 : 0;
        if (sep) A.head = 0;
        void* args[] = {(void*)&e->R, (void*)&A};
        const bool resident_units = e->attended(e->pos) <= (size_t)e->role_sp_resident_pos;
        void* k = mode == 1 ? (e->R.trace ? e->role_kernel_traced : e->role_kernel)
                  : resident_units ? (e->R.trace ? e->role_kernel_sp_traced : e->role_kernel_sp)
                                   : (e->R.trace ? e->role_kernel_sps_traced : e->role_kernel_sps);
        DCB_CUDA(cudaLaunchCooperativeKernel(k, dim3(e->grid), dim3(NT), args, (size_t)e->role_smem,
                                             e->stream));
        ++e->launches;
        if (sep) {
            HeadArgs HA{A.par, argmax_dev, host_logits};
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = dim3(e->head_grid);
            cfg.blockDim = dim3(HEADK_NT);
            cfg.dynamicSmemBytes = 3 * (size_t)e->P.Kh;
            cfg.stream = e->stream;
            cudaLaunchAttribute at[1];
            at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
            at[0].val.programmaticStreamSerializationAllowed = 1;
            cfg.attrs = at;
            cfg.numAttrs = 1;
            DCB_CUDA(cudaLaunchKernelEx(&cfg, head_kernel, e->HP, HA));
            ++e->launches;
        }
        return 0;
    }
    void* args[] = {(void*)&e->P, (void*)&A};
    DCB_CUDA(cudaLaunchCooperativeKernel(e->kernel, dim3(e->grid), dim3(NT), args, (size_t)e->smem, e->stream));
    ++e->launches;
    return 0;
}

int device_error(dcb_engine* e, int err) {
    if (!err) return 0;
    // On the engine's stream: a legacy-stream memset is not ordered before its next launch.
    DCB_CUDA(cudaMemsetAsync(e->P.sync, 0, sizeof(Sync), e->stream));
    // An abandoned step may have left down sums behind: start both halves from zero.
    DCB_CUDA(cudaMemsetAsync(e->P.dacc, 0, (size_t)2 * e->L * 2 * e->P.Hp * sizeof(uint64_t), e->stream));
    DCB_CUDA(cudaStreamSynchronize(e->stream));
    if (err == ERR_TOKEN) return fail(DCB_ERR_TOKEN, "token ID outside vocabulary");
    return fail(DCB_ERR_DEVICE_WAIT, "a device-side wait ran out of time; the step was abandoned");
}

int check_device_error(dcb_engine* e) {
    int err = 0;
    DCB_CUDA(cudaMemcpy(&err, &e->P.sync->error, sizeof(int), cudaMemcpyDeviceToHost));
    return device_error(e, err);
}

// The two-role kernel's layout: per attention block (2 per query head) its
// QKV rows packed in the order the kernel reads them, per FFN block its
// columns of W_down; both sized from the grid. Shapes the kernel does not
// take (or that do not fit in shared memory) leave role_ok false: the step
// kernel of step_kernel.cuh then runs every step.
int setup_role(dcb_engine* e, const dcb_model_desc* m, int max_optin) {
    const Params& P = e->P;
    RoleParams& R = e->R;
    const int H = e->H, I = e->I, D = e->D, half = D / 2, G = e->grid, NH = e->NH, NKV = e->NKV;
    const int hpg = NH / NKV;
    R.NA = 2 * NH;
    R.NG = G - R.NA;
    if (R.NG < 1 || H % 4 || NH > 255 || H > SLICE_RPT * SLICE_T) return 0;
    R.H = H;
    R.I = I;
    R.L = e->L;
    R.NH = NH;
    R.NKV = NKV;
    R.D = D;
    R.V = e->V;
    R.Kh = P.Kh;
    R.SH = P.SH;
    R.eps = P.eps;
    R.cached_rope = P.cached_rope;
    R.capacity = P.capacity;
    R.q_first = (half + 1) / 2;
    R.o_first = (int)round_up((size_t)(H / 2), 4);
    R.o_dw = P.o_dw;
    R.o_slice = P.o_slice;
    R.o_cols = P.o_cols;
    R.o_scale = P.o_scale;
    R.layers = P.layers;
    R.down_scale = P.down_scale;
    R.embed = P.embed;
    R.norms = P.norms;
    R.rope_inv = P.rope_inv;
    R.rope_den = P.rope_den;
    R.kcache = P.kcache;
    R.vcache = P.vcache;
    R.ll_q = P.ll_q;
    R.ll_kv = P.ll_kv;
    R.dacc = P.dacc;
    R.Hp = P.Hp;
    R.logits = P.logits;
    R.amax = P.amax;
    R.sync = P.sync;
    R.trace = nullptr;
    R.trace_layer = P.trace_layer;
    R.xq_plane = P.xq_plane;
    auto plo = [](int b, int n, int total) { return (int)((long long)b * total / n); };
    // QKV rows per attention block a = 2h + s: q pairs [q0, q0 + nq) of head h,
    // then k/v pairs [kv0, kv0 + nkv) of its group (u < D/2: k, else v).
    struct Share { int h, g, q0, nq, kv0, nkv; };
    std::vector<Share> sh(R.NA);
    int ra_max = 0;
    for (int a = 0; a < R.NA; ++a) {
        Share& x = sh[a];
        x.h = a / 2;
        const int s = a % 2;
        x.g = x.h / hpg;
        x.q0 = s ? R.q_first : 0;
        x.nq = s ? half - R.q_first : R.q_first;
        const int mi = 2 * (x.h % hpg) + s;
        x.kv0 = plo(mi, 2 * hpg, D);
        x.nkv = plo(mi + 1, 2 * hpg, D) - x.kv0;
        ra_max = std::max(ra_max, 2 * (x.nq + x.nkv));
    }
    const int gmax = ceil_div(I, R.NG);
    // The block GEMVs give each lane at most (rows + 31) / 32 rows of these caps.
    if (ra_max > RA_ROWS_MAX || 2 * gmax > RG_ROWS_MAX) return 0;
    R.ra_stride = ra_max;
    R.dw = slice_row_bytes(gmax);
    R.down_slice = (int)round_up((size_t)H * R.dw, 16);
    R.dcontrib = 0;
    for (int f = 0; f < R.NG; ++f) R.dcontrib += plo(f + 1, R.NG, I) > plo(f, R.NG, I);
    if (R.dcontrib > 255) return 0;
    // KV rows and the resident chunk buffers.
    const size_t es = e->kv_elem();
    R.bulk_kv = ((size_t)D * es) % 16 == 0;
    R.chunk_bytes = (int)round_up(2 * (size_t)ATT_CHUNK * D * es, 128);
    // Shared memory: vectors both roles use, then either role's region.
    cudaFuncAttributes fattr;
    const bool f16 = e->kv_dtype == DCB_KV_F16;
    // Each (KV type, head size) has a plain and a traced instantiation.
    void* kt[2];
    for (int tr = 0; tr < 2; ++tr)
        kt[tr] = D <= 32 ? (f16 ? (tr ? (void*)role_step_kernel<__half, 1, true, 0> : (void*)role_step_kernel<__half, 1, false, 0>)
                                : (tr ? (void*)role_step_kernel<float, 1, true, 0> : (void*)role_step_kernel<float, 1, false, 0>))
                 : D <= 64 ? (f16 ? (tr ? (void*)role_step_kernel<__half, 2, true, 0> : (void*)role_step_kernel<__half, 2, false, 0>)
                                  : (tr ? (void*)role_step_kernel<float, 2, true, 0> : (void*)role_step_kernel<float, 2, false, 0>))
                           : (f16 ? (tr ? (void*)role_step_kernel<__half, 4, true, 0> : (void*)role_step_kernel<__half, 4, false, 0>)
                                  : (tr ? (void*)role_step_kernel<float, 4, true, 0> : (void*)role_step_kernel<float, 4, false, 0>));
    // Spread mode (the FFN blocks attend beyond the resident buffers): head
    // dim 64, at most GQA_MAX query heads per KV group, every FFN block with
    // gate/up rows, rows that bulk-copy.
    const int sp_splits = G / NKV;  // every block is a unit
    const bool sp_ok = D == 64 && hpg <= GQA_MAX && sp_splits >= 1 && I >= R.NG && R.bulk_kv;
    // ks: [resident units, streaming units] x [plain, traced].
    void* ks[4] = {nullptr, nullptr, nullptr, nullptr};
    if (sp_ok) {
        ks[0] = f16 ? (void*)role_step_kernel<__half, 2, false, 1> : (void*)role_step_kernel<float, 2, false, 1>;
        ks[1] = f16 ? (void*)role_step_kernel<__half, 2, true, 1> : (void*)role_step_kernel<float, 2, true, 1>;
        ks[2] = f16 ? (void*)role_step_kernel<__half, 2, false, 2> : (void*)role_step_kernel<float, 2, false, 2>;
        ks[3] = f16 ? (void*)role_step_kernel<__half, 2, true, 2> : (void*)role_step_kernel<float, 2, true, 2>;
    }
    void* k = kt[0];
    if (cudaFuncGetAttributes(&fattr, k) != cudaSuccess) return fail(DCB_ERR_CUDA, "role kernel attributes");
    for (void* kk : {kt[1], ks[0], ks[1], ks[2], ks[3]}) {
        if (!kk) continue;
        cudaFuncAttributes ft;
        if (cudaFuncGetAttributes(&ft, kk) != cudaSuccess) return fail(DCB_ERR_CUDA, "role kernel attributes");
        fattr.sharedSizeBytes = std::max(fattr.sharedSizeBytes, ft.sharedSizeBytes);
    }
    const size_t budget = (size_t)max_optin - fattr.sharedSizeBytes;
    size_t off = 0;
    R.off_xf = (int)off;
    off = round_up(off + (size_t)P.Kh * 4, 128);
    R.off_xq = (int)off;
    off = round_up(off + 3 * (size_t)P.xq_plane, 128);
    R.off_xr = (int)off;
    off = round_up(off + (size_t)P.Kh * 4, 128);
    R.off_misc = (int)off;
    off = round_up(off + ROLE_MISC_BYTES, 128);
    const size_t base = off;
    R.a_qkv = (int)off;
    off = round_up(off + (size_t)ra_max * P.SH, 128);
    R.a_o = (int)off;
    off = round_up(off + (size_t)std::max(R.o_first, H - R.o_first) * R.o_dw, 128);
    R.a_part = (int)off;
    off = round_up(off + (size_t)std::max(NW * ra_max, NW * (D + 1)) * 4, 128);
    R.a_sc = (int)off;
    off = round_up(off + (size_t)RES_POS_MAX * 4, 128);
    R.a_ring = (int)off;
    const size_t attn_fixed = off;
    off = base;
    R.g_gu = (int)off;
    off = round_up(off + (size_t)2 * gmax * P.SH, 128);
    R.g_down = (int)off;
    off = round_up(off + (size_t)R.down_slice, 128);
    R.g_part = (int)off;
    off = round_up(off + (size_t)NW * 2 * gmax * 4, 128);
    R.g_h = (int)off;
    off = round_up(off + (size_t)std::max(R.dw, 32) * 4, 128);
    const size_t ffn_end = off;
    if (attn_fixed >= budget || ffn_end > budget) return 0;
    R.nbufs = (int)std::min<size_t>(RES_BUFS_MAX, (budget - attn_fixed) / R.chunk_bytes);
    if (R.nbufs < 1) return 0;
    // Spread units: their chunk buffers, then queries, new row, maxima, sums
    // and the score tile ([GQA_MAX][sp_bufs * 64]), as many buffers as fit.
    R.sp_splits = sp_splits;
    R.sp_bufs = 0;
    R.g_ring = (int)ffn_end;
    size_t ffn_sp_end = ffn_end;
    if (sp_ok) {
        for (int nb = RES_BUFS_MAX; nb >= 1; --nb) {
            const size_t ring_end = ffn_end + (size_t)nb * R.chunk_bytes;
            // (scores: every resident position for the one-pass units)
            const size_t sq = ((size_t)GQA_MAX * D + 2 * D + 2 * GQA_MAX + NW * GQA_MAX +
                               (size_t)nb * ATT_CHUNK * GQA_MAX + GQA_MAX) * 4;
            // The buffers also take the P.V shares of every warp ([NW][GQA_MAX][D] floats).
            if (ring_end + sq <= budget && (size_t)nb * R.chunk_bytes >= (size_t)NW * GQA_MAX * D * 4) {
                R.sp_bufs = nb;
                R.g_sq = (int)ring_end;
                ffn_sp_end = ring_end + sq;
                break;
            }
        }
    }
    // Attention blocks keep a unit's scratch after sp_bufs of their chunk buffers.
    if (R.sp_bufs > 0) {
        const size_t sq = ((size_t)GQA_MAX * D + 2 * D + 2 * GQA_MAX + NW * GQA_MAX +
                           (size_t)R.sp_bufs * ATT_CHUNK * GQA_MAX + GQA_MAX) * 4;
        R.a_sq = R.sp_bufs * R.chunk_bytes;
        if ((size_t)R.a_sq + sq > (size_t)R.nbufs * R.chunk_bytes) R.sp_bufs = 0;
    }
    R.ll_part = P.ll_part;
    R.kv_base = P.kv_base;
    R.kv_end = P.kv_end;
    R.world = P.world;
    R.rank = P.rank;
    R.peers = P.peers;
    R.exch = P.exch;
    const size_t smem = std::max({attn_fixed + (size_t)R.nbufs * R.chunk_bytes, ffn_end, ffn_sp_end});
    for (void* kk : {kt[0], kt[1], ks[0], ks[1], ks[2], ks[3]})
        if (kk && cudaFuncSetAttribute(kk, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) {
            cudaGetLastError();
            return 0;
        }
    int per_sm = 0;
    for (void* kk : {kt[0], kt[1], ks[0], ks[1], ks[2], ks[3]})
        if (kk && (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kk, NT, smem) != cudaSuccess || per_sm < 1)) {
            cudaGetLastError();
            return 0;
        }
    // Packed QKV rows per (layer, attention block), zero rows past its count.
    std::unique_ptr<uint8_t[]> buf;
    size_t nb = (size_t)e->L * R.NA * ra_max * P.SH;
    uint8_t* b = host_bytes(buf, nb);
    parallel_for(e->L * R.NA, [&](int t) {
        const int l = t / R.NA, a = t % R.NA;
        const dcb_layer_desc& S = m->layer[l];
        {
            const Share& x = sh[a];
            uint8_t* dst = b + (size_t)t * ra_max * P.SH;
            std::memset(dst, 0, (size_t)ra_max * P.SH);
            int row = 0;
            auto put = [&](const int8_t* w, const float* sc, const float* bi, int r) {
                pack_row(dst + (size_t)(row++) * P.SH, w + (size_t)r * H, H, sc[r], bi[r]);
            };
            for (int j = x.q0; j < x.q0 + x.nq; ++j) {
                put(S.q, S.q_scales, S.q_bias, x.h * D + j);
                put(S.q, S.q_scales, S.q_bias, x.h * D + j + half);
            }
            for (int u = x.kv0; u < x.kv0 + x.nkv; ++u) {
                if (u < half) {
                    put(S.k, S.k_scales, S.k_bias, x.g * D + u);
                    put(S.k, S.k_scales, S.k_bias, x.g * D + u + half);
                } else {
                    put(S.v, S.v_scales, S.v_bias, x.g * D + u - half);
                    put(S.v, S.v_scales, S.v_bias, x.g * D + u);
                }
            }
        }
    });
    uint8_t* d8;
    if (int rc = upload(e, &d8, b, nb)) return rc;
    R.qkv = d8;
    // W_down column slices per (layer, FFN block), dw bytes per row.
    nb = (size_t)e->L * R.NG * R.down_slice;
    b = host_bytes(buf, nb);
    parallel_for(e->L * R.NG, [&](int t) {
        const int l = t / R.NG, f = t % R.NG;
        const dcb_layer_desc& S = m->layer[l];
        const int c0 = plo(f, R.NG, I), c1 = plo(f + 1, R.NG, I);
        uint8_t* dst = b + (size_t)t * R.down_slice;
        std::memset(dst, 0, R.down_slice);
        for (int r = 0; r < H; ++r) std::memcpy(dst + (size_t)r * R.dw, S.down + (size_t)r * I + c0, (size_t)(c1 - c0));
    });
    if (int rc = upload(e, &d8, b, nb)) return rc;
    R.down_cols = d8;

    // The separate LM-head kernel (argmax candidates of its own).
    {
        HeadParams& HP = e->HP;
        HP.H = H;
        HP.Kh = P.Kh;
        HP.SH = P.SH;
        HP.V = e->V;
        HP.L = e->L;
        HP.Hp = P.Hp;
        HP.eps = P.eps;
        HP.expect = (unsigned)R.dcontrib;
        HP.embed = P.embed;
        HP.final_norm = P.norms + (size_t)e->L * 2 * P.Kh;
        HP.dacc = P.dacc;
        HP.logits = P.logits;
        HP.sync = P.sync;
        e->head_grid = 2 * e->sms;
        ArgBest* amax = nullptr;
        if (int rc = e->alloc(&amax, e->head_grid)) return rc;
        HP.amax = amax;
        int per_sm = 0;
        const size_t hsmem = 3 * (size_t)P.Kh;
        e->head_sep = P.Kh <= 32 * HEADK_C * 16 &&
                      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, head_kernel, HEADK_NT, hsmem) == cudaSuccess &&
                      per_sm >= 1;
        // Measured slower in place than the step kernel's own LM head (the
        // kernel boundary and a cold start outweigh its two blocks per SM), so
        // it is opt-in.
        const char* v = std::getenv("DCB_HEAD_KERNEL");
        e->head_sep = e->head_sep && v && std::atoi(v) != 0;
        cudaGetLastError();
    }
    e->role_kernel = kt[0];
    e->role_kernel_traced = kt[1];
    if (sp_ok && R.sp_bufs > 0) {
        e->role_kernel_sp = ks[0];
        e->role_kernel_sp_traced = ks[1];
        e->role_kernel_sps = ks[2];
        e->role_kernel_sps_traced = ks[3];
        e->role_sp_resident_pos = R.sp_splits * R.sp_bufs * ATT_CHUNK;
        // Units stream their chunks through their buffers: every position the
        // engine's capacity holds.
        e->role_sp_max_pos = (int)std::min<size_t>(e->capacity, (size_t)INT32_MAX);
        if (const char* v = std::getenv("DCB_ROLE_SPREAD"))
            if (!std::atoi(v)) e->role_sp_max_pos = 0;
    }
    e->role_smem = (int)smem;
    e->role_max_pos = R.nbufs * ATT_CHUNK;
    e->role_ok = true;
    if (const char* v = std::getenv("DCB_ROLE")) e->role_on = std::atoi(v) != 0;
    // The coarse waits end at the first contribution of a sum word.
    R.coarse_down = R.dcontrib - 1;
    R.coarse_o = NH - 1;
    if (const char* v = std::getenv("DCB_COARSE_DOWN")) R.coarse_down = std::atoi(v);
    if (const char* v = std::getenv("DCB_COARSE_O")) R.coarse_o = std::atoi(v);
    return 0;
}

// Head-major cache offset (elements) of (layer, kv head, position).
size_t kv_offset(const dcb_engine* e, int layer, int g, size_t t) {
    return (((size_t)layer * e->NKV + g) * e->capacity + t) * e->D;
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
    if (!capacity || capacity > (size_t)0x7fffffff)
        return fail(DCB_ERR_ARGUMENT, "invalid thread count or context capacity");
    if (kv_dtype != DCB_KV_F32 && kv_dtype != DCB_KV_F16) return fail(DCB_ERR_ARGUMENT, "invalid KV dtype");
    DCB_CUDA(cudaSetDevice(device));
    int dev_sms = 0;
    DCB_CUDA(cudaDeviceGetAttribute(&dev_sms, cudaDevAttrMultiProcessorCount, device));
    auto* e = new dcb_engine();
    e->device = device;
    auto bail = [&](int rc) {
        delete e;
        return rc;
    };
    e->H = m->hidden;
    e->I = m->intermediate;
    e->L = m->layers;
    e->NH = m->heads;
    e->NKV = m->kv_heads;
    e->D = m->head_dim;
    e->V = m->vocab;
    e->kv_dtype = kv_dtype;
    e->capacity = capacity;
    e->sms = dev_sms;
    e->grid = dev_sms;
    const int H = e->H, I = e->I, D = e->D, half = D / 2, G = e->grid;
    Params& P = e->P;
    P.H = H;
    P.I = I;
    P.L = e->L;
    P.NH = e->NH;
    P.NKV = e->NKV;
    P.D = D;
    P.V = e->V;
    P.Kh = (int)round_up(H, 16);
    P.Ki = (int)round_up(I, 16);
    P.SH = P.Kh + 16;
    P.SI = P.Ki + 16;
    P.qkv_pairs = (e->NH + 2 * e->NKV) * half;
    P.eps = m->epsilon;
    P.cached_rope = cached_rope ? 1 : 0;
    P.capacity = (int)capacity;
    P.kv_base = 0;
    P.kv_end = 0x7fffffff;
    P.world = 1;
    P.rank = 0;

    // ---- weights in packed-row layout: every layer's four matrices packed on
    // host threads, then uploaded one by one.
    std::vector<LayerW> lw(e->L);
    {
        struct LayerPack {
            std::unique_ptr<uint8_t[]> m[4];  // QKV pairs, O, gate/up, down
            size_t n[4] = {0, 0, 0, 0};
        };
        std::vector<LayerPack> lp(e->L);
        parallel_for(4 * e->L, [&](int t) {
            const int l = t / 4, which = t % 4;
            const dcb_layer_desc& S = m->layer[l];
            LayerPack& x = lp[l];
            if (which == 0) {
                x.n[0] = (size_t)P.qkv_pairs * 2 * P.SH;
                uint8_t* b = host_bytes(x.m[0], x.n[0]);
                size_t row = 0;
                auto add_pairs = [&](const int8_t* w, const float* sc, const float* bi, int heads) {
                    for (int h = 0; h < heads; ++h)
                        for (int j = 0; j < half; ++j)
                            for (int r : {h * D + j, h * D + j + half})
                                pack_row(b + (row++) * P.SH, w + (size_t)r * H, H, sc[r], bi[r]);
                };
                add_pairs(S.q, S.q_scales, S.q_bias, e->NH);
                add_pairs(S.k, S.k_scales, S.k_bias, e->NKV);
                add_pairs(S.v, S.v_scales, S.v_bias, e->NKV);
            } else if (which == 1) {
                x.n[1] = (size_t)H * P.SH;
                uint8_t* b = host_bytes(x.m[1], x.n[1]);
                for (int r = 0; r < H; ++r) pack_row(b + (size_t)r * P.SH, S.o + (size_t)r * H, H, S.o_scales[r], 0.f);
            } else if (which == 2) {
                x.n[2] = (size_t)2 * I * P.SH;
                uint8_t* b = host_bytes(x.m[2], x.n[2]);
                for (int j = 0; j < I; ++j) {
                    pack_row(b + (size_t)(2 * j) * P.SH, S.gate + (size_t)j * H, H, S.gate_scales[j], 0.f);
                    pack_row(b + (size_t)(2 * j + 1) * P.SH, S.up + (size_t)j * H, H, S.up_scales[j], 0.f);
                }
            } else {
                x.n[3] = (size_t)H * P.SI;
                uint8_t* b = host_bytes(x.m[3], x.n[3]);
                for (int r = 0; r < H; ++r)
                    pack_row(b + (size_t)r * P.SI, S.down + (size_t)r * I, I, S.down_scales[r], 0.f);
            }
        });
        for (int l = 0; l < e->L; ++l) {
            uint8_t* d8[4];
            for (int k = 0; k < 4; ++k) {
                if (int rc = upload(e, &d8[k], lp[l].m[k].get(), lp[l].n[k])) return bail(rc);
                lp[l].m[k].reset();
            }
            lw[l].qkv = d8[0];
            lw[l].o = d8[1];
            lw[l].gu = d8[2];
            lw[l].down = d8[3];
        }
    }
    std::unique_ptr<uint8_t[]> buf;
    // Down projection for the split-K step: block b's columns [b*I/G, (b+1)*I/G)
    // of every row, DW bytes per row (zero past the block's columns), one
    // down_slice-byte region per (layer, block); per-row scales apart.
    {
        const int DW = slice_row_bytes(ceil_div(I, G));
        if (DW > NT) return bail(fail(DCB_ERR_UNSUPPORTED, "intermediate size too large for this GPU"));
        if (H > DOWN_RPT * NT) return bail(fail(DCB_ERR_UNSUPPORTED, "hidden size above 1024 is not supported"));
        // The sum words count the blocks (down) or heads (O) in 8 bits; every
        // head needs a block of its own.
        if (G > 255) return bail(fail(DCB_ERR_UNSUPPORTED, "more than 255 multiprocessors is not supported"));
        if (e->NH > G) return bail(fail(DCB_ERR_UNSUPPORTED, "more query heads than multiprocessors"));
        P.down_dw = DW;
        P.down_slice = (int)round_up((size_t)H * DW, 16);
        const size_t nb = (size_t)e->L * G * P.down_slice;
        uint8_t* b = host_bytes(buf, nb);
        parallel_for(e->L * G, [&](int t) {
            const int l = t / G, bb = t % G;
            const dcb_layer_desc& S = m->layer[l];
            const int c0 = (int)((long long)bb * I / G), c1 = (int)((long long)(bb + 1) * I / G);
            uint8_t* dst = b + (size_t)t * P.down_slice;
            std::memset(dst, 0, P.down_slice);
            for (int r = 0; r < H; ++r) std::memcpy(dst + (size_t)r * DW, S.down + (size_t)r * I + c0, (size_t)(c1 - c0));
        });
        std::vector<float> dscale((size_t)e->L * H);
        for (int l = 0; l < e->L; ++l)
            std::copy(m->layer[l].down_scales, m->layer[l].down_scales + H, dscale.begin() + (size_t)l * H);
        uint8_t* d8;
        if (int rc = upload(e, &d8, b, nb)) return bail(rc);
        P.down_cols = d8;
        if (int rc = upload_floats(e, &P.down_scale, dscale)) return bail(rc);
    }
    // O projection for the split-K-over-heads step: per (layer, head) the
    // head's D columns of every row, o_dw bytes per row (zero past D, an odd
    // number of words); per-row scales apart.
    {
        P.o_dw = slice_row_bytes(D);
        P.o_slice = (int)round_up((size_t)H * P.o_dw, 16);
        const size_t nb = (size_t)e->L * e->NH * P.o_slice;
        uint8_t* b = host_bytes(buf, nb);
        parallel_for(e->L * e->NH, [&](int t) {
            const int l = t / e->NH, h = t % e->NH;
            const dcb_layer_desc& S = m->layer[l];
            uint8_t* dst = b + (size_t)t * P.o_slice;
            std::memset(dst, 0, P.o_slice);
            for (int r = 0; r < H; ++r) std::memcpy(dst + (size_t)r * P.o_dw, S.o + (size_t)r * H + h * D, D);
        });
        std::vector<float> oscale((size_t)e->L * H);
        for (int l = 0; l < e->L; ++l)
            std::copy(m->layer[l].o_scales, m->layer[l].o_scales + H, oscale.begin() + (size_t)l * H);
        uint8_t* d8;
        if (int rc = upload(e, &d8, b, nb)) return bail(rc);
        P.o_cols = d8;
        if (int rc = upload_floats(e, &P.o_scale, oscale)) return bail(rc);
    }
    {
        LayerW* d_layers = nullptr;
        if (int rc = e->alloc(&d_layers, lw.size())) return bail(rc);
        if (cudaMemcpy(d_layers, lw.data(), lw.size() * sizeof(LayerW), cudaMemcpyHostToDevice) != cudaSuccess)
            return bail(fail(DCB_ERR_CUDA, "layer table upload failed"));
        P.layers = d_layers;
    }
    {
        const size_t nb = (size_t)e->V * P.SH;
        uint8_t* b = host_bytes(buf, nb);
        constexpr int ROWS = 1024;  // embedding rows per packing task
        parallel_for(ceil_div(e->V, ROWS), [&](int t) {
            for (int r = t * ROWS; r < std::min(e->V, (t + 1) * ROWS); ++r)
                pack_row(b + (size_t)r * P.SH, m->embed + (size_t)r * H, H, m->embed_scales[r], 0.f);
        });
        uint8_t* d8;
        if (int rc = upload(e, &d8, b, nb)) return bail(rc);
        P.embed = d8;
        buf.reset();
        // RMSNorm gains, one [input | post-attention] pair per layer, then [final | 0].
        std::vector<float> norms((size_t)(e->L + 1) * 2 * P.Kh, 0.f);
        for (int l = 0; l < e->L; ++l) {
            std::copy(m->layer[l].input_norm, m->layer[l].input_norm + H, norms.begin() + (size_t)l * 2 * P.Kh);
            std::copy(m->layer[l].post_norm, m->layer[l].post_norm + H, norms.begin() + (size_t)l * 2 * P.Kh + P.Kh);
        }
        std::copy(m->final_norm, m->final_norm + H, norms.begin() + (size_t)e->L * 2 * P.Kh);
        if (int rc = upload_floats(e, &P.norms, norms)) return bail(rc);
        // RoPE tables with the reference's float expressions (src/model.cpp:223-224, src/kernels.cpp:140).
        std::vector<float> inv(half), den(half);
        for (int j = 0; j < half; ++j) {
            den[j] = std::pow(m->theta, float(2 * j) / float(D));
            inv[j] = 1.0f / std::pow(m->theta, float(2 * j) / float(D));
        }
        if (int rc = upload_floats(e, &P.rope_inv, inv)) return bail(rc);
        if (int rc = upload_floats(e, &P.rope_den, den)) return bail(rc);
    }
    // ---- KV cache (head-major) and activation buffers
    {
        unsigned char *kc, *vc;
        const size_t n = (size_t)e->L * e->NKV * capacity * D * e->kv_elem();
        if (int rc = e->alloc(&kc, n)) return bail(rc);
        if (int rc = e->alloc(&vc, n)) return bail(rc);
        P.kcache = kc;
        P.vcache = vc;
    }
    if (int rc = e->alloc(&P.ll_q, H)) return bail(rc);
    if (int rc = e->alloc(&P.ll_kv, 2 * e->NKV * D)) return bail(rc);
    if (int rc = e->alloc(&P.ll_part, (size_t)e->NH * (G + 1) * (D + 2))) return bail(rc);
    // KV-split exchange: [2 slots][NH][MAX_WORLD][D+2] tagged words, and the
    // ranks' buffers (this engine's own until dcb_set_kv_shard).
    if (int rc = e->alloc(&P.exch, (size_t)2 * e->NH * MAX_WORLD * (D + 2))) return bail(rc);
    {
        uint64_t** peers = nullptr;
        if (int rc = e->alloc(&peers, MAX_WORLD)) return bail(rc);
        uint64_t* own[MAX_WORLD] = {P.exch};
        DCB_CUDA(cudaMemcpy(peers, own, sizeof(own), cudaMemcpyHostToDevice));
        P.peers = peers;
    }
    P.Hp = (int)round_up((size_t)H, 32);
    if (int rc = e->alloc(&P.dacc, (size_t)2 * e->L * 2 * P.Hp)) return bail(rc);
    if (int rc = e->alloc(&P.logits, e->V)) return bail(rc);
    if (int rc = e->alloc(&P.amax, G)) return bail(rc);
    if (int rc = e->alloc(&P.sync, 1)) return bail(rc);

    // ---- shared memory plan (bytes): weight slots, attention chunk ring, vectors
    e->kernel = kv_dtype == DCB_KV_F16 ? (void*)decode_step_kernel<__half> : (void*)decode_step_kernel<float>;
    int max_optin = 0;
    DCB_CUDA(cudaDeviceGetAttribute(&max_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device));
    cudaFuncAttributes fattr;
    DCB_CUDA(cudaFuncGetAttributes(&fattr, e->kernel));
    const size_t budget = (size_t)max_optin - fattr.sharedSizeBytes;  // dynamic shared memory available
    const size_t gu_slot = (size_t)ceil_div(I, G) * 2 * P.SH;
    const size_t down_slot = (size_t)P.down_slice;
    const size_t qkv_slot = (size_t)ceil_div(P.qkv_pairs, G) * 2 * P.SH;
    size_t off = 0;
    P.off_gu = (int)off;
    off = round_up(off + gu_slot, 128);
    P.off_down = (int)off;
    off = round_up(off + down_slot, 128);
    P.off_qkv = (int)off;
    off = round_up(off + qkv_slot, 128);
    P.off_att = (int)off;
    // Vectors after the attention ring: staged floats, fixed-point planes,
    // GEMV partials (two buffers), raw residual, attention scratch.
    P.xq_plane = (int)round_up((size_t)P.Kh, 128);
    {
        const int max_rows = std::max(2 * ceil_div(P.qkv_pairs, G), 2 * ceil_div(I, G));
        P.gpart_floats = NW * max_rows;
    }
    const size_t xs_bytes = round_up((size_t)P.Kh * sizeof(float), 128);
    const size_t xq_bytes = round_up(3 * (size_t)P.xq_plane, 128);
    // The GEMV partial buffers also hold a group attention unit's score tile.
    const size_t gqa_tile = D == 64 ? (size_t)GQA_MAX * GQA_PASS * ATT_CHUNK * sizeof(float) : 0;
    const size_t gpart_bytes = round_up(std::max(2 * (size_t)P.gpart_floats * sizeof(float), gqa_tile), 128);
    const size_t xr_bytes = round_up((size_t)P.Kh * sizeof(float), 128);
    const size_t misc_bytes = round_up((size_t)(384 + NW * (D + 2)) * sizeof(float), 128);
    const size_t h_bytes = round_up((size_t)P.down_dw * sizeof(float), 128);
    const size_t tail = xs_bytes + xq_bytes + gpart_bytes + xr_bytes + misc_bytes + h_bytes;
    // The attention ring takes what is left (2..ATT_MAX_BUFS chunks).
    P.att_chunk_bytes = (int)(2 * (size_t)ATT_CHUNK * D * e->kv_elem());
    const size_t room = budget > off + tail ? budget - off - tail : 0;
    P.att_bufs = (int)std::min<size_t>(ATT_MAX_BUFS, std::max<size_t>(2, room / P.att_chunk_bytes));
    // W_o's columns of a head sit at the end of the attention buffers; the
    // split-merge and KV-split tables at their start must stay below them.
    {
        const long long wo = (long long)P.att_bufs * P.att_chunk_bytes - P.o_slice;
        const long long tables = (long long)(1 + MAX_WORLD) * (D + 2) * sizeof(float);
        if (wo < tables) return bail(fail(DCB_ERR_UNSUPPORTED, "model too large for shared memory staging"));
        P.wo_off = (int)(wo / 16 * 16);
    }
    off = round_up(off + (size_t)P.att_bufs * P.att_chunk_bytes, 128);
    P.off_xs = (int)off;
    P.trace_layer = std::min(5, e->L - 1);
    if (const char* v = std::getenv("DCB_SPLIT_MIN")) e->split_min = std::max(ATT_CHUNK, std::atoi(v) / ATT_CHUNK * ATT_CHUNK);
    if (const char* v = std::getenv("DCB_GROUP_MIN")) e->group_min = std::max(1, std::atoi(v));
    if (const char* v = std::getenv("DCB_GROUP_SPLIT_MIN"))
        e->group_split_min = std::max(ATT_CHUNK, std::atoi(v) / ATT_CHUNK * ATT_CHUNK);
    // Group units stage q in the staged-vector buffer and the scores in the
    // GEMV partial buffers (both idle during attention).
    {
        const int hpg = e->NH / e->NKV;
        e->gqa_ok = D == 64 && hpg <= GQA_MAX && P.Kh >= hpg * D;
        // Chunks per pass: leave at least one buffer loading while a pass computes.
        P.gqa_pass = std::max(1, std::min(GQA_PASS, P.att_bufs - 1));
        if (const char* v = std::getenv("DCB_GQA_PASS")) P.gqa_pass = std::max(1, std::min({GQA_PASS, P.att_bufs, std::atoi(v)}));
    }
    off += xs_bytes;
    P.off_xq = (int)off;
    off += xq_bytes;
    P.off_gpart = (int)off;
    off += gpart_bytes;
    P.off_xr = (int)off;
    off += xr_bytes;
    P.off_misc = (int)off;
    off += misc_bytes;
    P.off_h = (int)off;
    off += h_bytes;
    e->smem = (int)off;
    if ((size_t)e->smem > budget) return bail(fail(DCB_ERR_UNSUPPORTED, "model too large for shared memory staging"));
    if (cudaFuncSetAttribute(e->kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, e->smem) != cudaSuccess)
        return bail(fail(DCB_ERR_UNSUPPORTED, "cannot reserve shared memory for the step kernel"));
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, e->kernel, NT, e->smem) != cudaSuccess || per_sm < 1)
        return bail(fail(DCB_ERR_UNSUPPORTED, "step kernel cannot be resident"));

    if (int rc = setup_role(e, m, max_optin)) return bail(rc);

    if (cudaMallocHost(&e->h_result, 4 * sizeof(int)) != cudaSuccess)
        return bail(fail(DCB_ERR_CUDA, "cudaMallocHost failed"));
    if (cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking) != cudaSuccess)
        return bail(fail(DCB_ERR_CUDA, "stream creation failed"));
    e->own_stream = true;
    if (cudaDeviceSynchronize() != cudaSuccess) return bail(fail(DCB_ERR_CUDA, "device synchronize failed"));
    *out = e;
    return 0;
}

void dcb_destroy(dcb_engine* e) { delete e; }

// The step at e->pos must have a row for its K/V if this engine keeps that
// position, and at least one position to attend over.
int check_position(const dcb_engine* e) {
    if (e->owns(e->pos) && e->pos - e->kv_base >= e->capacity)
        return fail(DCB_ERR_CAPACITY, "context capacity exceeded");
    if (e->pos < e->kv_base) return fail(DCB_ERR_ARGUMENT, "position before this engine's KV range");
    return 0;
}

int dcb_step(dcb_engine* e, int token, int head, float* host_logits, int* argmax_out) {
    if (!e) return fail(DCB_ERR_ARGUMENT, "null engine");
    if (token < 0 || token >= e->V) return fail(DCB_ERR_TOKEN, "token ID outside vocabulary");
    if (int rc = check_position(e)) return rc;
    DCB_CUDA(cudaSetDevice(e->device));
    // Pinned (registered or cudaHostAlloc'd) logits buffers are written by the
    // LM head itself over PCIe; any other buffer gets a copy after the kernel.
    float* mapped = nullptr;
    if (head && host_logits) {
        cudaPointerAttributes at{};
        if (cudaPointerGetAttributes(&at, host_logits) == cudaSuccess && at.type == cudaMemoryTypeHost &&
            at.devicePointer)
            mapped = static_cast<float*>(at.devicePointer);
        else
            cudaGetLastError();  // a pageable pointer is not an error here
    }
    if (int rc = launch(e, token, nullptr, head, nullptr, mapped)) return rc;
    if (head && host_logits && !mapped)
        DCB_CUDA(cudaMemcpyAsync(host_logits, e->P.logits, (size_t)e->V * sizeof(float), cudaMemcpyDeviceToHost,
                                 e->stream));
    // error and argmax in one copy (adjacent in Sync)
    DCB_CUDA(cudaMemcpyAsync(e->h_result, &e->P.sync->error, 2 * sizeof(int), cudaMemcpyDeviceToHost, e->stream));
    DCB_CUDA(cudaStreamSynchronize(e->stream));
    if (int rc = device_error(e, e->h_result[0])) return rc;
    if (head && argmax_out) *argmax_out = e->h_result[1];
    ++e->pos;
    return 0;
}

int dcb_step_async(dcb_engine* e, int token, const int* token_dev, int head, int* argmax_dev) {
    if (!e) return fail(DCB_ERR_ARGUMENT, "null engine");
    if (!token_dev && (token < 0 || token >= e->V)) return fail(DCB_ERR_TOKEN, "token ID outside vocabulary");
    if (int rc = check_position(e)) return rc;
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
    if (position > e->kv_base && std::min(position, e->kv_end) - e->kv_base > e->capacity)
        return fail(DCB_ERR_CAPACITY, "context capacity exceeded");
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

// Host rows are [count][kv_heads*head_dim] (the reference's layout); the device
// cache is head-major, so each head is one strided 2-D copy.
int dcb_kv_write(dcb_engine* e, int layer, size_t start, size_t count, const float* keys, const float* values) {
    if (!e || !keys || !values) return fail(DCB_ERR_ARGUMENT, "null argument");
    if (layer < 0 || layer >= e->L || start < e->kv_base || start + count > e->kv_end ||
        start - e->kv_base + count > e->capacity)
        return fail(DCB_ERR_ARGUMENT, "KV rows out of range");
    start -= e->kv_base;  // local rows
    if (!count) return 0;
    DCB_CUDA(cudaSetDevice(e->device));
    DCB_CUDA(cudaStreamSynchronize(e->stream));
    const size_t kvd = (size_t)e->NKV * e->D, es = e->kv_elem();
    for (int which = 0; which < 2; ++which) {
        const float* src = which ? values : keys;
        char* base = static_cast<char*>(which ? e->P.vcache : e->P.kcache);
        if (es == 4) {
            for (int g = 0; g < e->NKV; ++g)
                DCB_CUDA(cudaMemcpy2DAsync(base + kv_offset(e, layer, g, start) * es, e->D * es, src + (size_t)g * e->D,
                                           kvd * sizeof(float), e->D * es, count, cudaMemcpyHostToDevice, e->stream));
        } else {
            std::vector<__half> h(count * kvd);
            for (size_t i = 0; i < h.size(); ++i) h[i] = __float2half_rn(src[i]);
            for (int g = 0; g < e->NKV; ++g)
                DCB_CUDA(cudaMemcpy2DAsync(base + kv_offset(e, layer, g, start) * es, e->D * es,
                                           h.data() + (size_t)g * e->D, kvd * es, e->D * es, count,
                                           cudaMemcpyHostToDevice, e->stream));
            DCB_CUDA(cudaStreamSynchronize(e->stream));  // h is released at the end of this block
        }
    }
    DCB_CUDA(cudaStreamSynchronize(e->stream));  // the caller may reuse keys/values on return
    return 0;
}

int dcb_kv_read(const dcb_engine* e, int layer, size_t start, size_t count, float* keys, float* values) {
    if (!e || !keys || !values) return fail(DCB_ERR_ARGUMENT, "null argument");
    if (layer < 0 || layer >= e->L || start < e->kv_base || start + count > e->kv_end ||
        start - e->kv_base + count > e->capacity)
        return fail(DCB_ERR_ARGUMENT, "KV rows out of range");
    start -= e->kv_base;  // local rows
    if (!count) return 0;
    DCB_CUDA(cudaSetDevice(e->device));
    DCB_CUDA(cudaStreamSynchronize(e->stream));
    const size_t kvd = (size_t)e->NKV * e->D, es = e->kv_elem();
    for (int which = 0; which < 2; ++which) {
        float* dst = which ? values : keys;
        const char* base = static_cast<const char*>(which ? e->P.vcache : e->P.kcache);
        if (es == 4) {
            for (int g = 0; g < e->NKV; ++g)
                DCB_CUDA(cudaMemcpy2D(dst + (size_t)g * e->D, kvd * sizeof(float),
                                      base + kv_offset(e, layer, g, start) * es, e->D * es, e->D * es, count,
                                      cudaMemcpyDeviceToHost));
        } else {
            std::vector<__half> h(count * kvd);
            for (int g = 0; g < e->NKV; ++g)
                DCB_CUDA(cudaMemcpy2D(h.data() + (size_t)g * e->D, kvd * es, base + kv_offset(e, layer, g, start) * es,
                                      e->D * es, e->D * es, count, cudaMemcpyDeviceToHost));
            for (size_t i = 0; i < h.size(); ++i) dst[i] = __half2float(h[i]);
        }
    }
    return 0;
}

int dcb_exchange_buffer(dcb_engine* e, void** exchange, size_t* bytes) {
    if (!e || !exchange) return fail(DCB_ERR_ARGUMENT, "null argument");
    *exchange = e->P.exch;
    if (bytes) *bytes = (size_t)2 * e->NH * MAX_WORLD * (e->D + 2) * sizeof(uint64_t);
    return 0;
}

int dcb_ipc_handle(const void* device_ptr, void* handle) {
    if (!device_ptr || !handle) return fail(DCB_ERR_ARGUMENT, "null argument");
    static_assert(sizeof(cudaIpcMemHandle_t) <= DCB_IPC_HANDLE_BYTES, "IPC handle size");
    cudaIpcMemHandle_t h;
    DCB_CUDA(cudaIpcGetMemHandle(&h, const_cast<void*>(device_ptr)));
    std::memcpy(handle, &h, sizeof(h));
    return 0;
}

int dcb_ipc_open(const void* handle, void** device_ptr) {
    if (!handle || !device_ptr) return fail(DCB_ERR_ARGUMENT, "null argument");
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    DCB_CUDA(cudaIpcOpenMemHandle(device_ptr, h, cudaIpcMemLazyEnablePeerAccess));
    return 0;
}

int dcb_ipc_close(void* device_ptr) {
    if (!device_ptr) return fail(DCB_ERR_ARGUMENT, "null argument");
    DCB_CUDA(cudaIpcCloseMemHandle(device_ptr));
    return 0;
}

int dcb_set_kv_shard(dcb_engine* e, int rank, int world, size_t kv_begin, size_t kv_end, void* const* peer_exchange) {
    if (!e) return fail(DCB_ERR_ARGUMENT, "null engine");
    if (world < 1 || world > MAX_WORLD || rank < 0 || rank >= world)
        return fail(DCB_ERR_ARGUMENT, "invalid rank or world size (at most 8 GPUs)");
    if (kv_begin >= kv_end || kv_begin > 0x7ffffffe || (kv_end != SIZE_MAX && kv_end > 0x7fffffff))
        return fail(DCB_ERR_ARGUMENT, "invalid KV range");
    if (kv_end != SIZE_MAX && kv_end - kv_begin > e->capacity)
        return fail(DCB_ERR_CAPACITY, "KV range larger than the context capacity");
    if (world > 1 && !peer_exchange) return fail(DCB_ERR_ARGUMENT, "null peer exchange buffers");
    uint64_t* ptrs[MAX_WORLD] = {};
    for (int q = 0; q < world; ++q) {
        ptrs[q] = world == 1 || q == rank ? e->P.exch : static_cast<uint64_t*>(peer_exchange[q]);
        if (!ptrs[q]) return fail(DCB_ERR_ARGUMENT, "null peer exchange buffer");
    }
    DCB_CUDA(cudaSetDevice(e->device));
    DCB_CUDA(cudaStreamSynchronize(e->stream));
    DCB_CUDA(cudaMemcpyAsync(const_cast<uint64_t**>(e->P.peers), ptrs, sizeof(ptrs), cudaMemcpyHostToDevice, e->stream));
    DCB_CUDA(cudaStreamSynchronize(e->stream));
    e->kv_base = kv_begin;
    e->kv_end = kv_end;
    e->P.kv_base = (int)kv_begin;
    e->P.kv_end = kv_end == SIZE_MAX ? 0x7fffffff : (int)kv_end;
    e->P.world = world;
    e->P.rank = rank;
    e->R.kv_base = e->P.kv_base;
    e->R.kv_end = e->P.kv_end;
    e->R.world = world;
    e->R.rank = rank;
    return 0;
}

int dcb_launch_info(const dcb_engine* e, int* blocks, int* threads, int* smem_bytes, int* sms) {
    if (!e) return fail(DCB_ERR_ARGUMENT, "null engine");
    if (blocks) *blocks = e->grid;
    if (threads) *threads = NT;
    if (smem_bytes) *smem_bytes = e->role_ok && e->role_on ? e->role_smem : e->smem;
    if (sms) *sms = e->sms;
    return 0;
}

uint64_t dcb_launch_count(const dcb_engine* e) { return e ? e->launches : 0; }

int dcb_trace_enable(dcb_engine* e, int on) {
    if (!e) return fail(DCB_ERR_ARGUMENT, "null engine");
    if (on && 5 * e->L + 3 > TRACE_MAX_PHASES) return fail(DCB_ERR_UNSUPPORTED, "too many layers to trace");
    DCB_CUDA(cudaSetDevice(e->device));
    DCB_CUDA(cudaStreamSynchronize(e->stream));
    if (on && !e->trace) {
        if (int rc = e->alloc(&e->trace, (size_t)2 * TRACE_MAX_PHASES * e->grid)) return rc;
    }
    e->P.trace = on ? e->trace : nullptr;
    e->R.trace = e->P.trace;
    return 0;
}

int dcb_trace_read(dcb_engine* e, uint64_t* ready, uint64_t* done, int* phases) {
    if (!e || !e->trace) return fail(DCB_ERR_ARGUMENT, "tracing is not enabled");
    DCB_CUDA(cudaSetDevice(e->device));
    DCB_CUDA(cudaStreamSynchronize(e->stream));
    const int n = 5 * e->L + 3;
    if (phases) *phases = n;
    const size_t per = (size_t)TRACE_MAX_PHASES * e->grid * sizeof(uint64_t);
    if (ready) DCB_CUDA(cudaMemcpy(ready, e->trace, per, cudaMemcpyDeviceToHost));
    if (done) DCB_CUDA(cudaMemcpy(done, e->trace + (size_t)TRACE_MAX_PHASES * e->grid, per, cudaMemcpyDeviceToHost));
    if (ready || done) {
        DCB_CUDA(cudaMemsetAsync(e->trace, 0, (size_t)2 * TRACE_MAX_PHASES * e->grid * sizeof(uint64_t), e->stream));
        DCB_CUDA(cudaStreamSynchronize(e->stream));
    }
    return 0;
}

}  // extern "C"

int dcb::engine_kv(const dcb_engine* e, EngineKV* out) {
    if (!e || !out) return fail(DCB_ERR_ARGUMENT, "null engine");
    out->kcache = e->P.kcache;
    out->vcache = e->P.vcache;
    out->capacity = e->capacity;
    out->pos = e->pos;
    out->kv_dtype = e->kv_dtype;
    out->whole_sequence = e->P.world == 1 && e->kv_base == 0 && e->kv_end == SIZE_MAX;
    out->stream = e->stream;
    return 0;
}
void dcb::engine_advance(dcb_engine* e, size_t n) { e->pos += n; }
dcb_batch*& dcb::engine_prefill_batch(dcb_engine* e) { return e->prefill; }

int dcb::model_view(const dcb_engine* e, ModelView* out) {
    if (!e || !out) return fail(DCB_ERR_ARGUMENT, "null engine");
    DCB_CUDA(cudaSetDevice(e->device));
    out->device = e->device;
    out->P = e->P;
    out->layers.resize(e->L);
    DCB_CUDA(cudaMemcpy(out->layers.data(), e->P.layers, (size_t)e->L * sizeof(LayerW), cudaMemcpyDeviceToHost));
    return 0;
}
