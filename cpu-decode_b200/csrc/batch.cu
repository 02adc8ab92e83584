// Batched decode engine behind the dcb_batch_* C ABI: up to 64 independent
// sequences on one GPU, sharing the weights a dcb_engine uploaded, each with
// its own KV cache and position. One step is one CUDA graph of
//   stage(embed, input norm)
//   per layer: QKV GEMM (+bias, RoPE, KV write) -> split-KV attention ->
//              combine + stage -> O GEMM (+residual) -> stage(post norm) ->
//              gate/up GEMM (SiLU*up) -> stage -> down GEMM (+residual) ->
//              stage(next norm)
//   LM-head GEMM (+argmax per tile) -> argmax (next tokens, positions + 1)
// with every projection on tcgen05 (batch_kernels.cuh). Positions and tokens
// live on the device, so graph replays chain greedy steps without the host.
#include "batch_kernels.cuh"
#include "decode_b200.h"
#include "model_view.h"

#include <cuda.h>
#include <cuda_runtime.h>
#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <utility>
#include <string>
#include <vector>

using namespace dcb;
using namespace dcb::batch;

namespace {
int bfail(int code, const std::string& msg) {
    set_last_error(msg);
    return code;
}
#define BT_CUDA(call)                                                                                          \
    do {                                                                                                       \
        cudaError_t e_ = (call);                                                                               \
        if (e_ != cudaSuccess) return bfail(DCB_ERR_CUDA, std::string(#call ": ") + cudaGetErrorString(e_));   \
    } while (0)

size_t rup(size_t v, size_t m) { return (v + m - 1) / m * m; }
int cdiv(int a, int b) { return (a + b - 1) / b; }

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    return fn;
}

// 2D tensor map: `inner` elements of each row (the rest of its `stride`
// bytes is not read), `rows` rows; boxes of box_inner elements (128 bytes) x
// box_rows rows with the 128-byte swizzle; out-of-range elements read as zero.
int make_map(CUtensorMap* m, const void* base, CUtensorMapDataType type, uint64_t inner, uint64_t rows,
             uint64_t stride, uint32_t box_inner, uint32_t box_rows) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return bfail(DCB_ERR_CUDA, "cuTensorMapEncodeTiled is not available");
    if ((reinterpret_cast<uintptr_t>(base) & 15) || (stride & 15) || box_rows < 1 || box_rows > 256)
        return bfail(DCB_ERR_ARGUMENT, "tensor map: misaligned base or stride");
    const cuuint64_t dims[2] = {inner, rows};
    const cuuint64_t strides[1] = {stride};
    const cuuint32_t box[2] = {box_inner, box_rows};
    const cuuint32_t es[2] = {1, 1};
    const CUresult r = fn(m, type, 2, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                          CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return bfail(DCB_ERR_CUDA, "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
    return 0;
}
// Int8 rows in GK-byte boxes.
int make_map(CUtensorMap* m, const void* base, uint64_t inner, uint64_t rows, uint64_t stride, uint32_t box_rows) {
    return make_map(m, base, CU_TENSOR_MAP_DATA_TYPE_UINT8, inner, rows, stride, GK, box_rows);
}

// FP32 rows -> the cache's element type, on the device.
template <typename KV>
__global__ void to_kv_kernel(const float* src, KV* dst, size_t n) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        kv_store(dst + i, src[i]);
}
}  // namespace

struct dcb_batch {
    int device = 0;
    cudaStream_t stream = nullptr;
    ModelView M;
    int slots = 0, kv_dtype = DCB_KV_F32;
    size_t capacity = 0;
    int split_len = 256, max_splits = 0;
    int sms = 148;
    std::vector<void*> allocations;
    float *x = nullptr, *h = nullptr, *q = nullptr, *xsc = nullptr, *xinv = nullptr, *part = nullptr,
          *logits = nullptr;
    int8_t *ph = nullptr, *pi = nullptr;
    ArgBest* amax = nullptr;
    int *tokens = nullptr, *pos = nullptr, *argmax = nullptr, *err = nullptr;
    void *kc = nullptr, *vc = nullptr;
    float* stage_f = nullptr;  // FP32 rows waiting for conversion to F16 (kv_write from device memory)
    float2* rope = nullptr;    // [slots][D/2] (cos, sin) of each sequence's position, per step
    int* seq_done = nullptr;   // [slots] attention blocks finished per sequence (fused split merge)
    int* gbar = nullptr;       // [3][2] grid barriers of the O, gate/up and down projections
    int* kpart = nullptr;      // [sms][3 * slots][GM] int32 split-K partials of one projection
    bool fuse_combine = false; // split merge inside the attention kernel
    bool fuse_stage = false;   // staging of the next input inside the O, gate/up and down projections
    bool head_persistent = false;  // LM head on head_gemm_kernel (B resident in shared memory)
    size_t stage_f_elems = 0;
    int* h_io = nullptr;  // pinned: [slots] tokens in, then [slots] argmax + error word out
    int* h_pos = nullptr;  // pinned: [slots] positions in (prefill)
    // 1: every slot has its own cache; 0 (prefill): the slots are consecutive
    // positions of one sequence whose cache (borrowed from a step engine) they share.
    int kv_seq = 1;
    std::vector<CUtensorMap> map_qkv, map_o, map_gu, map_down;
    CUtensorMap map_head{}, map_ph{}, map_pi{}, map_k{}, map_v{};
    bool attn64 = false;  // head_dim 64, at most 8 query heads per KV head: attention64_tc_kernel
    std::vector<size_t> pos_host;
    // Instantiated step graphs by (sequences, logits copied, LM head); exec is
    // the one the last build_graph chose.
    struct GraphEntry {
        int n;
        bool logits, head;
        cudaGraphExec_t exec;
    };
    std::vector<GraphEntry> graphs;
    cudaGraphExec_t exec = nullptr;
    uint64_t steps = 0;

    ~dcb_batch() {
        cudaSetDevice(device);
        if (stream) cudaStreamSynchronize(stream);
        for (const GraphEntry& g : graphs) cudaGraphExecDestroy(g.exec);
        for (void* p : allocations) cudaFree(p);
        if (h_io) cudaFreeHost(h_io);
        if (h_pos) cudaFreeHost(h_pos);
        if (stream) cudaStreamDestroy(stream);
    }
    template <class T>
    int alloc(T** out, size_t count) {
        void* p = nullptr;
        const size_t bytes = rup(std::max<size_t>(count * sizeof(T), 16), 256);
        cudaError_t e = cudaMalloc(&p, bytes);
        if (e != cudaSuccess) return bfail(DCB_ERR_CUDA, std::string("cudaMalloc: ") + cudaGetErrorString(e));
        allocations.push_back(p);
        e = cudaMemset(p, 0, bytes);
        if (e != cudaSuccess) return bfail(DCB_ERR_CUDA, std::string("cudaMemset: ") + cudaGetErrorString(e));
        *out = static_cast<T*>(p);
        return 0;
    }
    size_t kv_elem() const { return kv_dtype == DCB_KV_F16 ? 2 : 4; }
    // Element offset of (sequence, layer, kv head, position) in the caches.
    size_t kv_offset(int s, int l, int g, size_t t) const {
        return ((((size_t)s * M.P.L + l) * M.P.NKV + g) * capacity + t) * M.P.D;
    }
};

namespace {

// Every kernel of a step is launched with programmatic stream serialization:
// it may start (and run the part before its griddepcontrol.wait) while the
// previous kernel finishes. `cluster` > 1 groups that many CTAs along x.
template <typename... KArgs, typename... Args>
int launch(void (*kernel)(KArgs...), dim3 grid, int threads, size_t smem, cudaStream_t stream, int cluster,
           Args&&... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(threads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    int na = 0;
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
    if (cluster > 1) {
        attr[na].id = cudaLaunchAttributeClusterDimension;
        attr[na].val.clusterDim.x = (unsigned)cluster;
        attr[na].val.clusterDim.y = 1;
        attr[na].val.clusterDim.z = 1;
        ++na;
    }
    cfg.attrs = attr;
    cfg.numAttrs = na;
    BT_CUDA(cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...));
    return 0;
}

// Row tiles of 128 x all sequences; with fewer tiles than SMs the reduction
// is split over a cluster of up to 4 CTAs per tile (one stage at least each;
// 8 measured 4.6 % slower at 64 sequences: more partials to merge through
// distributed shared memory). DCB_BATCH_KSPLIT sets another cap (1..8).
int gemm_split(const dcb_batch* b, int epi, int rows, int K) {
    const int tiles = cdiv(rows, GM), nk = cdiv(K, GK);
    static const int cap = [] {
        const char* v = std::getenv("DCB_BATCH_KSPLIT");
        return v ? std::max(1, std::min(8, std::atoi(v))) : 4;
    }();
    return epi == EPI_HEAD ? 1 : std::max(1, std::min({cap, nk, b->sms / tiles}));
}

template <int EPI>
constexpr int stages_of() {
    return EPI == EPI_HEAD ? HEAD_STAGES : GSTAGES;
}

template <int EPI, typename KV>
int launch_gemm(dcb_batch* b, const CUtensorMap& ma, const CUtensorMap& mb, int rows, int K, const GemmArgs& a0) {
    GemmArgs a = a0;
    a.M = rows;
    a.nk = cdiv(K, GK);
    const int tiles = cdiv(rows, GM);
    a.ksplit = gemm_split(b, EPI, rows, K);
    constexpr int ST = stages_of<EPI>();
    const int smem = gemm_smem_bytes(b->slots, ST);
    // One [3 * slots][GM] block of split-K partials per CTA.
    if (a.ksplit > 1 && tiles * a.ksplit > b->sms) return bfail(DCB_ERR_UNSUPPORTED, "split-K grid above the SM count");
    if (a.st_planes)
        return launch(gemm_i8_kernel<EPI, KV, ST, true>, dim3(tiles * a.ksplit), gemm_threads<EPI>(), smem, b->stream, a.ksplit, ma, mb,
                      a);
    return launch(gemm_i8_kernel<EPI, KV, ST>, dim3(tiles * a.ksplit), gemm_threads<EPI>(), smem, b->stream, a.ksplit, ma, mb, a);
}

// Can every CTA of this projection's grid be resident at once (needed by its
// grid barrier)?
template <int EPI, typename KV>
bool co_resident(const dcb_batch* b, int rows, int K) {
    const int S = gemm_split(b, EPI, rows, K), grid = cdiv(rows, GM) * S;
    constexpr int ST = stages_of<EPI>();
    const int smem = gemm_smem_bytes(b->slots, ST);
    if (S == 1) {
        int per_sm = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, gemm_i8_kernel<EPI, KV, ST, true>, gemm_threads<EPI>(), smem) !=
            cudaSuccess)
            return false;
        return per_sm * b->sms >= grid;
    }
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(gemm_threads<EPI>());
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = (unsigned)S;
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, gemm_i8_kernel<EPI, KV, ST, true>, &cfg) != cudaSuccess) return false;
    return clusters * S >= grid;
}

template <int EPI, typename KV>
int allow_smem(int slots) {
    constexpr int ST = stages_of<EPI>();
    BT_CUDA(cudaFuncSetAttribute(gemm_i8_kernel<EPI, KV, ST>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 gemm_smem_bytes(slots, ST)));
    if (EPI == EPI_RESID || EPI == EPI_GU)
        BT_CUDA(cudaFuncSetAttribute(gemm_i8_kernel<EPI, KV, ST, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     gemm_smem_bytes(slots, ST)));
    return 0;
}

// One step of n slots; head false: no LM head and no argmax (the slots'
// positions and tokens are then not advanced on the device).
template <typename KV>
int enqueue_step(dcb_batch* b, int n, bool want_logits, bool head) {
    const Params& P = b->M.P;
    const int H = P.H, I = P.I, D = P.D;
    const int st_smem_h = P.Kh * (int)sizeof(float), st_smem_i = P.Ki * (int)sizeof(float);

    StageArgs sa{};
    sa.slots = b->slots;
    sa.nseq = n;
    sa.eps = P.eps;
    sa.err = b->err;
    sa.vocab = P.V;

    GemmArgs g{};
    g.nseq = n;
    g.slots = b->slots;
    g.xsc = b->xsc;
    g.NH = P.NH;
    g.NKV = P.NKV;
    g.D = D;
    g.L = P.L;
    g.capacity = (int)b->capacity;
    g.cached_rope = P.cached_rope;
    g.rope_inv = P.rope_inv;
    g.rope_den = P.rope_den;
    g.pos = b->pos;
    g.rope = b->rope;
    g.kcache = b->kc;
    g.vcache = b->vc;
    g.kv_seq = b->kv_seq;
    g.amax = b->amax;
    g.kpart = b->kpart;
    g.err = b->err;

    // Layer 0 input: the tokens' embedding rows, RMSNorm-staged.
    {
        StageArgs s = sa;
        s.n = H;
        s.kp = P.Kh;
        s.lds = P.Kh;
        s.embed = P.embed;
        s.SE = P.SH;
        s.eoff = P.Kh;
        s.tokens = b->tokens;
        s.x_out = b->x;
        s.gain = P.norms;
        s.planes = b->ph;
        s.xsc = b->xsc;
        s.xinv = b->xinv;
        s.pos = b->pos;
        s.rope_inv = P.rope_inv;
        s.rope_den = P.rope_den;
        s.cached_rope = P.cached_rope;
        s.half = D / 2;
        s.rope = b->rope;
        if (int rc = launch(stage_kernel, dim3(n), ST_NT, st_smem_h, b->stream, 1, s)) return rc;
    }
    AttnArgs aa{};
    aa.q = b->q;
    aa.kcache = b->kc;
    aa.vcache = b->vc;
    aa.part = b->part;
    aa.pos = b->pos;
    aa.NH = P.NH;
    aa.NKV = P.NKV;
    aa.D = D;
    aa.L = P.L;
    aa.capacity = (int)b->capacity;
    aa.split_len = b->split_len;
    aa.max_splits = b->max_splits;
    aa.kv_seq = b->kv_seq;
    const size_t at_smem = attention_smem_bytes(D, (int)sizeof(KV), P.NH / P.NKV);
    CombineArgs ca{};
    ca.part = b->part;
    ca.pos = b->pos;
    ca.NH = P.NH;
    ca.D = D;
    ca.split_len = b->split_len;
    ca.max_splits = b->max_splits;
    ca.slots = b->slots;
    ca.kp = P.Kh;
    ca.planes = b->ph;
    ca.xsc = b->xsc;
    const int cb_smem = (P.NH * D + 2 * P.NH * b->max_splits) * (int)sizeof(float);

    for (int l = 0; l < P.L; ++l) {
        const float* in_norm = P.norms + (size_t)l * 2 * P.Kh;
        const float* post_norm = in_norm + P.Kh;
        const LayerW& W = b->M.layers[l];
        // QKV + bias + RoPE; K/V rows of the new tokens into the caches.
        {
            GemmArgs a = g;
            a.wscale = reinterpret_cast<const float*>(W.qkv + P.Kh);
            a.wstride = P.SH / 4;
            a.bias = a.wscale + 1;
            a.bstride = P.SH / 4;
            a.xinv = b->xinv;
            a.out = b->q;
            a.ldo = P.NH * D;
            a.layer = l;
            if (int rc = launch_gemm<EPI_QKV, KV>(b, b->map_qkv[l], b->map_ph, 2 * P.qkv_pairs, P.Kh, a)) return rc;
        }
        aa.layer = l;
        if (b->attn64) {
            Attn64Args a6{};
            a6.q = b->q;
            a6.part = b->part;
            a6.pos = b->pos;
            a6.NH = P.NH;
            a6.NKV = P.NKV;
            a6.L = P.L;
            a6.layer = l;
            a6.capacity = (int)b->capacity;
            a6.split_len = b->split_len;
            a6.max_splits = b->max_splits;
            a6.kv_seq = b->kv_seq;
            a6.err = b->err;
            a6.seq_done = b->seq_done;
            a6.cb = ca;
            const dim3 grid(b->max_splits, P.NKV, n);
            const int rc = b->fuse_combine ? launch(attention64_tc_kernel<KV, true>, grid, A64_NT, tc_smem_bytes(),
                                                    b->stream, 1, b->map_k, b->map_v, a6)
                                           : launch(attention64_tc_kernel<KV, false>, grid, A64_NT, tc_smem_bytes(),
                                                    b->stream, 1, b->map_k, b->map_v, a6);
            if (rc) return rc;
        } else if (D == 64) {
            if (int rc = launch(attention_kernel<KV, 64>, dim3(b->max_splits, P.NKV, n), AT_NT, at_smem, b->stream, 1, aa))
                return rc;
        } else {
            if (int rc = launch(attention_kernel<KV, 0>, dim3(b->max_splits, P.NKV, n), AT_NT, at_smem, b->stream, 1, aa))
                return rc;
        }
        if (!(b->attn64 && b->fuse_combine))
            if (int rc = launch(combine_stage_kernel, dim3(n), CB_NT, cb_smem, b->stream, 1, ca)) return rc;
        // O + residual.
        {
            GemmArgs a = g;
            a.wscale = reinterpret_cast<const float*>(W.o + P.Kh);
            a.wstride = P.SH / 4;
            a.out = b->x;
            a.ldo = P.Kh;
            if (b->fuse_stage) {  // then the post-attention RMSNorm input of gate/up
                a.gbar = b->gbar;
                a.st_src = b->x;
                a.st_lds = P.Kh;
                a.st_n = H;
                a.st_kp = P.Kh;
                a.st_gain = post_norm;
                a.st_planes = b->ph;
                a.st_xsc = b->xsc;
                a.st_xinv = b->xinv;
                a.st_eps = P.eps;
            }
            if (int rc = launch_gemm<EPI_RESID, KV>(b, b->map_o[l], b->map_ph, H, P.Kh, a)) return rc;
        }
        if (!b->fuse_stage) {
            StageArgs s = sa;
            s.n = H;
            s.kp = P.Kh;
            s.src = b->x;
            s.lds = P.Kh;
            s.gain = post_norm;
            s.planes = b->ph;
            s.xsc = b->xsc;
            s.xinv = b->xinv;
            if (int rc = launch(stage_kernel, dim3(n), ST_NT, st_smem_h, b->stream, 1, s)) return rc;
        }
        // gate/up + SiLU.
        {
            GemmArgs a = g;
            a.wscale = reinterpret_cast<const float*>(W.gu + P.Kh);
            a.wstride = P.SH / 4;
            a.xinv = b->xinv;
            a.out = b->h;
            a.ldo = P.Ki;
            if (b->fuse_stage) {  // then the down projection's input
                a.gbar = b->gbar + 2;
                a.st_src = b->h;
                a.st_lds = P.Ki;
                a.st_n = I;
                a.st_kp = P.Ki;
                a.st_planes = b->pi;
                a.st_xsc = b->xsc;
            }
            if (int rc = launch_gemm<EPI_GU, KV>(b, b->map_gu[l], b->map_ph, 2 * I, P.Kh, a)) return rc;
        }
        if (!b->fuse_stage) {
            StageArgs s = sa;
            s.n = I;
            s.kp = P.Ki;
            s.src = b->h;
            s.lds = P.Ki;
            s.planes = b->pi;
            s.xsc = b->xsc;
            if (int rc = launch(stage_kernel, dim3(n), ST_NT, st_smem_i, b->stream, 1, s)) return rc;
        }
        // down + residual.
        {
            GemmArgs a = g;
            a.wscale = reinterpret_cast<const float*>(W.down + P.Ki);
            a.wstride = P.SI / 4;
            a.out = b->x;
            a.ldo = P.Kh;
            if (b->fuse_stage) {  // then the next layer's input norm, or the final norm before the head
                a.gbar = b->gbar + 4;
                a.st_src = b->x;
                a.st_lds = P.Kh;
                a.st_n = H;
                a.st_kp = P.Kh;
                a.st_gain = l + 1 < P.L ? P.norms + (size_t)(l + 1) * 2 * P.Kh : P.norms + (size_t)P.L * 2 * P.Kh;
                a.st_planes = b->ph;
                a.st_xsc = b->xsc;
                a.st_xinv = b->xinv;
                a.st_eps = P.eps;
            }
            if (int rc = launch_gemm<EPI_RESID, KV>(b, b->map_down[l], b->map_pi, H, P.Ki, a)) return rc;
        }
        // Next layer's input norm, or the final norm before the head.
        if (!b->fuse_stage) {
            StageArgs s = sa;
            s.n = H;
            s.kp = P.Kh;
            s.src = b->x;
            s.lds = P.Kh;
            s.gain = l + 1 < P.L ? P.norms + (size_t)(l + 1) * 2 * P.Kh : P.norms + (size_t)P.L * 2 * P.Kh;
            s.planes = b->ph;
            s.xsc = b->xsc;
            s.xinv = b->xinv;
            if (int rc = launch(stage_kernel, dim3(n), ST_NT, st_smem_h, b->stream, 1, s)) return rc;
        }
    }
    if (!head) return 0;
    // Tied LM head + per-tile argmax, then the argmax per sequence.
    {
        GemmArgs a = g;
        a.wscale = reinterpret_cast<const float*>(P.embed + P.Kh);
        a.wstride = P.SH / 4;
        a.xinv = b->xinv;
        a.out = want_logits ? b->logits : nullptr;
        a.ldo = P.V;
        if (b->head_persistent) {
            a.M = P.V;
            a.nk = cdiv(P.Kh, GK);
            a.ksplit = 1;
            const int grid = std::min(cdiv(P.V, GM), b->sms);
            if (int rc = launch(head_gemm_kernel, dim3(grid), HB_NT, head_smem_bytes(b->slots), b->stream, 1,
                                b->map_head, b->map_ph, a))
                return rc;
        } else if (int rc = launch_gemm<EPI_HEAD, KV>(b, b->map_head, b->map_ph, P.V, P.Kh, a)) {
            return rc;
        }
    }
    ArgmaxArgs ga{};
    ga.amax = b->amax;
    ga.tiles = cdiv(P.V, GM);
    ga.slots = b->slots;
    ga.nseq = n;
    ga.argmax = b->argmax;
    ga.tokens = b->tokens;
    ga.pos = b->pos;
    return launch(argmax_kernel, dim3(n), ARG_NT, 0, b->stream, 1, ga);
}

constexpr size_t MAX_GRAPHS = 6;

int build_graph(dcb_batch* b, int n, bool want_logits, bool head = true) {
    for (const auto& g : b->graphs)
        if (g.n == n && g.logits == want_logits && g.head == head) {
            b->exec = g.exec;
            return 0;
        }
    b->exec = nullptr;
    if (b->graphs.size() >= MAX_GRAPHS) {
        cudaGraphExecDestroy(b->graphs.front().exec);
        b->graphs.erase(b->graphs.begin());
    }
    BT_CUDA(cudaStreamBeginCapture(b->stream, cudaStreamCaptureModeThreadLocal));
    const int rc = b->kv_dtype == DCB_KV_F16 ? enqueue_step<__half>(b, n, want_logits, head)
                                             : enqueue_step<float>(b, n, want_logits, head);
    cudaGraph_t graph = nullptr;
    const cudaError_t ce = cudaStreamEndCapture(b->stream, &graph);
    if (rc) {
        if (graph) cudaGraphDestroy(graph);
        return rc;
    }
    if (ce != cudaSuccess) return bfail(DCB_ERR_CUDA, std::string("graph capture: ") + cudaGetErrorString(ce));
    cudaGraphExec_t exec = nullptr;
    const cudaError_t ie = cudaGraphInstantiate(&exec, graph, 0);
    cudaGraphDestroy(graph);
    if (ie != cudaSuccess) return bfail(DCB_ERR_CUDA, std::string("graph instantiate: ") + cudaGetErrorString(ie));
    b->graphs.push_back({n, want_logits, head, exec});
    b->exec = exec;
    return 0;
}

int check_seq(const dcb_batch* b, int s) {
    if (s < 0 || s >= b->slots) return bfail(DCB_ERR_ARGUMENT, "sequence index out of range");
    return 0;
}

// After a step: read the error word; on error reset it and report.
int device_status(dcb_batch* b, int err) {
    if (!err) return 0;
    BT_CUDA(cudaMemsetAsync(b->err, 0, sizeof(int), b->stream));
    // An abandoned step may leave counters part-way: start them from zero.
    BT_CUDA(cudaMemsetAsync(b->seq_done, 0, (size_t)b->slots * sizeof(int), b->stream));
    BT_CUDA(cudaMemsetAsync(b->gbar, 0, 6 * sizeof(int), b->stream));
    BT_CUDA(cudaStreamSynchronize(b->stream));
    if (err == ERR_TOKEN) return bfail(DCB_ERR_TOKEN, "token ID outside vocabulary");
    return bfail(DCB_ERR_DEVICE_WAIT, "a device-side wait ran out of time; the step was abandoned");
}

}  // namespace

// A batched context over engine `model`'s weights. kc/vc null: every slot
// gets a cache of `capacity` positions; else the slots share that one cache
// (the engine's own, for its prefill).
static int create_batch(const dcb_engine* model, int max_seqs, size_t capacity, int kv_dtype, void* shared_kc,
                        void* shared_vc, dcb_batch** out) {
    if (!model || !out) return bfail(DCB_ERR_ARGUMENT, "null argument");
    *out = nullptr;
    if (max_seqs < 1 || max_seqs > MAX_SLOTS) return bfail(DCB_ERR_ARGUMENT, "max_seqs must be 1..64");
    if (capacity < 1 || capacity > (size_t)1 << 24) return bfail(DCB_ERR_ARGUMENT, "invalid context capacity");
    if (kv_dtype != DCB_KV_F32 && kv_dtype != DCB_KV_F16) return bfail(DCB_ERR_ARGUMENT, "invalid KV dtype");
    dcb_batch* b = new dcb_batch();
    auto bail = [&](int rc) {
        delete b;
        return rc;
    };
    if (int rc = model_view(model, &b->M)) return bail(rc);
    const Params& P = b->M.P;
    b->device = b->M.device;
    BT_CUDA(cudaSetDevice(b->device));
    BT_CUDA(cudaDeviceGetAttribute(&b->sms, cudaDevAttrMultiProcessorCount, b->device));
    int major = 0, minor = 0;
    BT_CUDA(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, b->device));
    BT_CUDA(cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, b->device));
    if (major != 10 || minor != 0) return bail(bfail(DCB_ERR_UNSUPPORTED, "the batched engine needs an sm_100 GPU"));
    if (P.D % 2 || P.D > 128 || P.NH % P.NKV) return bail(bfail(DCB_ERR_UNSUPPORTED, "unsupported head shape"));
    b->slots = (int)rup((size_t)max_seqs, 16);
    b->capacity = capacity;
    b->kv_dtype = kv_dtype;
    b->attn64 = P.D == 64 && P.NH / P.NKV <= A64_HP;
    b->split_len = b->attn64 ? 768 : 256;
    // DCB_BATCH_SPLIT: positions per attention split (a multiple of 64), for tuning.
    if (const char* sv = std::getenv("DCB_BATCH_SPLIT"))
        b->split_len = std::max(64, std::min(1 << 16, std::atoi(sv) / 64 * 64));
    b->max_splits = cdiv((int)capacity, b->split_len);
    const int S = b->slots;
    if (int rc = b->alloc(&b->x, (size_t)S * P.Kh)) return bail(rc);
    if (int rc = b->alloc(&b->h, (size_t)S * P.Ki)) return bail(rc);
    if (int rc = b->alloc(&b->q, (size_t)S * P.NH * P.D)) return bail(rc);
    if (int rc = b->alloc(&b->rope, (size_t)S * (P.D / 2))) return bail(rc);
    if (int rc = b->alloc(&b->seq_done, S)) return bail(rc);
    if (int rc = b->alloc(&b->gbar, 6)) return bail(rc);
    if (int rc = b->alloc(&b->kpart, (size_t)b->sms * 3 * S * GM)) return bail(rc);
    if (int rc = b->alloc(&b->xsc, S)) return bail(rc);
    if (int rc = b->alloc(&b->xinv, S)) return bail(rc);
    if (int rc = b->alloc(&b->part, (size_t)S * P.NH * b->max_splits * (P.D + 2))) return bail(rc);
    if (int rc = b->alloc(&b->logits, (size_t)S * P.V)) return bail(rc);
    if (int rc = b->alloc(&b->ph, (size_t)3 * S * P.Kh)) return bail(rc);
    if (int rc = b->alloc(&b->pi, (size_t)3 * S * P.Ki)) return bail(rc);
    if (int rc = b->alloc(&b->amax, (size_t)cdiv(P.V, GM) * S)) return bail(rc);
    if (int rc = b->alloc(&b->tokens, S)) return bail(rc);
    if (int rc = b->alloc(&b->pos, S)) return bail(rc);
    if (int rc = b->alloc(&b->argmax, S + 1)) return bail(rc);
    b->err = b->argmax + S;  // read with the argmax in one copy
    if (shared_kc) {
        b->kc = shared_kc;
        b->vc = shared_vc;
        b->kv_seq = 0;
    } else {
        unsigned char *kc, *vc;
        const size_t n = (size_t)S * P.L * P.NKV * capacity * P.D * b->kv_elem();
        if (int rc = b->alloc(&kc, n)) return bail(rc);
        if (int rc = b->alloc(&vc, n)) return bail(rc);
        b->kc = kc;
        b->vc = vc;
    }
    const size_t caches = shared_kc ? 1 : (size_t)S;
    b->pos_host.assign(S, 0);
    // Tensor maps: weights in their packed rows (int8 part only), and the planes.
    b->map_qkv.resize(P.L);
    b->map_o.resize(P.L);
    b->map_gu.resize(P.L);
    b->map_down.resize(P.L);
    for (int l = 0; l < P.L; ++l) {
        const LayerW& W = b->M.layers[l];
        if (int rc = make_map(&b->map_qkv[l], W.qkv, P.Kh, 2 * (uint64_t)P.qkv_pairs, P.SH, GM)) return bail(rc);
        if (int rc = make_map(&b->map_o[l], W.o, P.Kh, P.H, P.SH, GM)) return bail(rc);
        if (int rc = make_map(&b->map_gu[l], W.gu, P.Kh, 2 * (uint64_t)P.I, P.SH, GM)) return bail(rc);
        if (int rc = make_map(&b->map_down[l], W.down, P.Ki, P.H, P.SI, GM)) return bail(rc);
    }
    if (int rc = make_map(&b->map_head, P.embed, P.Kh, P.V, P.SH, GM)) return bail(rc);
    if (int rc = make_map(&b->map_ph, b->ph, P.Kh, 3 * (uint64_t)S, P.Kh, 3 * S)) return bail(rc);
    if (int rc = make_map(&b->map_pi, b->pi, P.Ki, 3 * (uint64_t)S, P.Ki, 3 * S)) return bail(rc);
    if (b->attn64) {
        // KV rows of every sequence, layer and head as one 2D array of 64-element rows.
        const uint64_t rows = (uint64_t)caches * P.L * P.NKV * capacity;
        const bool f16 = kv_dtype == DCB_KV_F16;
        const CUtensorMapDataType t = f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
        const uint32_t inner = f16 ? 64 : 32;  // 128-byte boxes
        if (rows > 0x7fffffffull) return bail(bfail(DCB_ERR_UNSUPPORTED, "KV cache too large for one tensor map"));
        if (int rc = make_map(&b->map_k, b->kc, t, 64, rows, 64 * b->kv_elem(), inner, A64_T)) return bail(rc);
        if (int rc = make_map(&b->map_v, b->vc, t, 64, rows, 64 * b->kv_elem(), inner, A64_T)) return bail(rc);
        for (const void* f : {(const void*)attention64_tc_kernel<float, false>,
                              (const void*)attention64_tc_kernel<float, true>,
                              (const void*)attention64_tc_kernel<__half, false>,
                              (const void*)attention64_tc_kernel<__half, true>})
            BT_CUDA(cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, tc_smem_bytes()));
    }
    if (int rc = allow_smem<EPI_QKV, float>(S)) return bail(rc);
    if (int rc = allow_smem<EPI_QKV, __half>(S)) return bail(rc);
    if (int rc = allow_smem<EPI_RESID, float>(S)) return bail(rc);
    if (int rc = allow_smem<EPI_RESID, __half>(S)) return bail(rc);
    if (int rc = allow_smem<EPI_GU, float>(S)) return bail(rc);
    if (int rc = allow_smem<EPI_GU, __half>(S)) return bail(rc);
    if (int rc = allow_smem<EPI_HEAD, float>(S)) return bail(rc);
    if (int rc = allow_smem<EPI_HEAD, __half>(S)) return bail(rc);
    {
        // The persistent LM head's 5-stage ring; when it does not fit (or
        // DCB_BATCH_HEAD=0), the tiled head runs.
        int optin = 0;
        BT_CUDA(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, b->device));
        const int hs = head_smem_bytes(S);
        const char* hv = std::getenv("DCB_BATCH_HEAD");
        if (hs + 4096 <= optin && !(hv && !std::atoi(hv))) {
            if (cudaFuncSetAttribute(head_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, hs) != cudaSuccess)
                return bail(bfail(DCB_ERR_CUDA, "LM-head kernel shared memory"));
            b->head_persistent = true;
        }
    }
    {
        // The split merge's shared memory: outputs, then a weight and a sum per (head, split).
        const size_t cb = (size_t)(P.NH * P.D + 2 * P.NH * b->max_splits) * sizeof(float);
        if (cb > 227 * 1024) return bail(bfail(DCB_ERR_UNSUPPORTED, "context capacity too large for the split merge"));
        if (cudaFuncSetAttribute(combine_stage_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)cb) !=
            cudaSuccess)
            return bail(bfail(DCB_ERR_CUDA, "combine kernel shared memory"));
    }
    // Optional fusions (DCB_BATCH_FUSE=1): the split merge by the last
    // attention block of each sequence, and the staging of the next input by
    // the O, gate/up and down projections after a grid barrier. Measured on a
    // B200 with 64 sequences they are slower than the separate kernels (the
    // merge and the staging of a sequence then run on one block at the end of
    // the kernel instead of in parallel), so they are off by default. The
    // merge needs its scratch to fit the attention kernel's score area; the
    // staging needs every CTA of a projection resident at once.
    const char* fv = std::getenv("DCB_BATCH_FUSE");
    if (fv && std::atoi(fv)) {
        b->fuse_combine = b->attn64 && (size_t)(P.NH * 64 + 2 * P.NH * b->max_splits) * 4 <= (size_t)TC_RING_F32;
        if (kv_dtype == DCB_KV_F16)
            b->fuse_stage = co_resident<EPI_RESID, __half>(b, P.H, P.Kh) &&
                            co_resident<EPI_GU, __half>(b, 2 * P.I, P.Kh) && co_resident<EPI_RESID, __half>(b, P.H, P.Ki);
        else
            b->fuse_stage = co_resident<EPI_RESID, float>(b, P.H, P.Kh) &&
                            co_resident<EPI_GU, float>(b, 2 * P.I, P.Kh) && co_resident<EPI_RESID, float>(b, P.H, P.Ki);
    }
    {
        const int at = (int)attention_smem_bytes(P.D, (int)b->kv_elem(), P.NH / P.NKV);
        auto set = [&](const void* f) {
            return cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, at);
        };
        if (kv_dtype == DCB_KV_F16) {
            BT_CUDA(set((const void*)attention_kernel<__half, 64>));
            BT_CUDA(set((const void*)attention_kernel<__half, 0>));
        } else {
            BT_CUDA(set((const void*)attention_kernel<float, 64>));
            BT_CUDA(set((const void*)attention_kernel<float, 0>));
        }
    }
    if (cudaMallocHost(&b->h_io, (size_t)2 * (S + 1) * sizeof(int)) != cudaSuccess ||
        cudaMallocHost(&b->h_pos, (size_t)S * sizeof(int)) != cudaSuccess)
        return bail(bfail(DCB_ERR_CUDA, "cudaMallocHost failed"));
    BT_CUDA(cudaStreamCreateWithFlags(&b->stream, cudaStreamNonBlocking));
    BT_CUDA(cudaDeviceSynchronize());
    *out = b;
    return 0;
}

extern "C" {

int dcb_batch_create(const dcb_engine* model, int max_seqs, size_t capacity, int kv_dtype, dcb_batch** out) {
    return create_batch(model, max_seqs, capacity, kv_dtype, nullptr, nullptr, out);
}

void dcb_batch_destroy(dcb_batch* b) { delete b; }

int dcb_batch_info(const dcb_batch* b, int* slots, size_t* capacity, int* split_len) {
    if (!b) return bfail(DCB_ERR_ARGUMENT, "null batch");
    if (slots) *slots = b->slots;
    if (capacity) *capacity = b->capacity;
    if (split_len) *split_len = b->split_len;
    return 0;
}

int dcb_batch_set_position(dcb_batch* b, int seq, size_t position) {
    if (!b) return bfail(DCB_ERR_ARGUMENT, "null batch");
    if (int rc = check_seq(b, seq)) return rc;
    if (position >= b->capacity) return bfail(DCB_ERR_CAPACITY, "context capacity exceeded");
    BT_CUDA(cudaSetDevice(b->device));
    BT_CUDA(cudaStreamSynchronize(b->stream));
    const int p = (int)position;
    BT_CUDA(cudaMemcpyAsync(b->pos + seq, &p, sizeof(int), cudaMemcpyHostToDevice, b->stream));
    BT_CUDA(cudaStreamSynchronize(b->stream));
    b->pos_host[seq] = position;
    return 0;
}

size_t dcb_batch_position(const dcb_batch* b, int seq) {
    if (!b || seq < 0 || seq >= b->slots) return 0;
    return b->pos_host[seq];
}

int dcb_batch_kv_write(dcb_batch* b, int seq, int layer, size_t start, size_t count, const float* keys,
                       const float* values) {
    if (!b || !keys || !values) return bfail(DCB_ERR_ARGUMENT, "null argument");
    if (int rc = check_seq(b, seq)) return rc;
    const Params& P = b->M.P;
    if (layer < 0 || layer >= P.L || start + count > b->capacity) return bfail(DCB_ERR_ARGUMENT, "KV rows out of range");
    if (!count) return 0;
    BT_CUDA(cudaSetDevice(b->device));
    BT_CUDA(cudaStreamSynchronize(b->stream));
    const size_t kvd = (size_t)P.NKV * P.D, es = b->kv_elem();
    for (int which = 0; which < 2; ++which) {
        const float* src = which ? values : keys;
        char* base = static_cast<char*>(which ? b->vc : b->kc);
        if (es == 4) {
            // Host or device rows (cudaMemcpyDefault: unified addressing).
            for (int g = 0; g < P.NKV; ++g)
                BT_CUDA(cudaMemcpy2DAsync(base + b->kv_offset(seq, layer, g, start) * es, P.D * es,
                                          src + (size_t)g * P.D, kvd * sizeof(float), P.D * es, count,
                                          cudaMemcpyDefault, b->stream));
        } else {
            // FP32 rows gathered per head into device scratch, rounded to F16 on the device.
            if (b->stage_f_elems < count * P.D) {
                if (int rc = b->alloc(&b->stage_f, count * P.D)) return rc;
                b->stage_f_elems = count * P.D;
            }
            for (int g = 0; g < P.NKV; ++g) {
                BT_CUDA(cudaMemcpy2DAsync(b->stage_f, P.D * sizeof(float), src + (size_t)g * P.D,
                                          kvd * sizeof(float), P.D * sizeof(float), count, cudaMemcpyDefault,
                                          b->stream));
                to_kv_kernel<__half><<<256, 256, 0, b->stream>>>(
                    b->stage_f, reinterpret_cast<__half*>(base) + b->kv_offset(seq, layer, g, start), count * P.D);
                BT_CUDA(cudaGetLastError());
                BT_CUDA(cudaStreamSynchronize(b->stream));  // stage_f is reused by the next head
            }
        }
    }
    BT_CUDA(cudaStreamSynchronize(b->stream));  // the caller may reuse keys/values on return
    return 0;
}

int dcb_batch_kv_read(const dcb_batch* b, int seq, int layer, size_t start, size_t count, float* keys, float* values) {
    if (!b || !keys || !values) return bfail(DCB_ERR_ARGUMENT, "null argument");
    if (int rc = check_seq(b, seq)) return rc;
    const Params& P = b->M.P;
    if (layer < 0 || layer >= P.L || start + count > b->capacity) return bfail(DCB_ERR_ARGUMENT, "KV rows out of range");
    if (!count) return 0;
    BT_CUDA(cudaSetDevice(b->device));
    BT_CUDA(cudaStreamSynchronize(b->stream));
    const size_t kvd = (size_t)P.NKV * P.D, es = b->kv_elem();
    for (int which = 0; which < 2; ++which) {
        float* dst = which ? values : keys;
        const char* base = static_cast<const char*>(which ? b->vc : b->kc);
        if (es == 4) {
            for (int g = 0; g < P.NKV; ++g)
                BT_CUDA(cudaMemcpy2D(dst + (size_t)g * P.D, kvd * sizeof(float),
                                     base + b->kv_offset(seq, layer, g, start) * es, P.D * es, P.D * es, count,
                                     cudaMemcpyDefault));
        } else {
            std::vector<__half> hbuf(count * P.D);
            for (int g = 0; g < P.NKV; ++g) {
                BT_CUDA(cudaMemcpy(hbuf.data(), base + b->kv_offset(seq, layer, g, start) * es, count * P.D * es,
                                   cudaMemcpyDeviceToHost));
                for (size_t t = 0; t < count; ++t)
                    for (int j = 0; j < P.D; ++j) dst[t * kvd + (size_t)g * P.D + j] = __half2float(hbuf[t * P.D + j]);
            }
        }
    }
    return 0;
}

int dcb_batch_step(dcb_batch* b, int n, const int* tokens, float* logits, int* argmax_out) {
    if (!b) return bfail(DCB_ERR_ARGUMENT, "null batch");
    if (n < 1 || n > b->slots) return bfail(DCB_ERR_ARGUMENT, "sequence count out of range");
    const Params& P = b->M.P;
    for (int s = 0; s < n; ++s)
        if (b->pos_host[s] >= b->capacity) return bfail(DCB_ERR_CAPACITY, "context capacity exceeded");
    if (tokens)
        for (int s = 0; s < n; ++s)
            if (tokens[s] < 0 || tokens[s] >= P.V) return bfail(DCB_ERR_TOKEN, "token ID outside vocabulary");
    BT_CUDA(cudaSetDevice(b->device));
    if (int rc = build_graph(b, n, logits != nullptr)) return rc;
    if (tokens) {
        std::memcpy(b->h_io, tokens, (size_t)n * sizeof(int));
        BT_CUDA(cudaMemcpyAsync(b->tokens, b->h_io, (size_t)n * sizeof(int), cudaMemcpyHostToDevice, b->stream));
    }
    BT_CUDA(cudaGraphLaunch(b->exec, b->stream));
    ++b->steps;
    if (logits)
        BT_CUDA(cudaMemcpyAsync(logits, b->logits, (size_t)n * P.V * sizeof(float), cudaMemcpyDeviceToHost, b->stream));
    int* hout = b->h_io + b->slots + 1;
    BT_CUDA(cudaMemcpyAsync(hout, b->argmax, (size_t)(b->slots + 1) * sizeof(int), cudaMemcpyDeviceToHost, b->stream));
    BT_CUDA(cudaStreamSynchronize(b->stream));
    if (int rc = device_status(b, hout[b->slots])) {
        // Positions advanced on the device with the abandoned step: put them back.
        std::vector<int> p(b->slots);
        for (int s = 0; s < b->slots; ++s) p[s] = (int)b->pos_host[s];
        BT_CUDA(cudaMemcpyAsync(b->pos, p.data(), p.size() * sizeof(int), cudaMemcpyHostToDevice, b->stream));
        BT_CUDA(cudaStreamSynchronize(b->stream));
        return rc;
    }
    if (argmax_out) std::memcpy(argmax_out, hout, (size_t)n * sizeof(int));
    for (int s = 0; s < n; ++s) ++b->pos_host[s];
    return 0;
}

int dcb_batch_step_greedy(dcb_batch* b, int n, int steps) {
    if (!b) return bfail(DCB_ERR_ARGUMENT, "null batch");
    if (n < 1 || n > b->slots || steps < 0) return bfail(DCB_ERR_ARGUMENT, "sequence or step count out of range");
    for (int s = 0; s < n; ++s)
        if (b->pos_host[s] + (size_t)steps > b->capacity) return bfail(DCB_ERR_CAPACITY, "context capacity exceeded");
    BT_CUDA(cudaSetDevice(b->device));
    if (int rc = build_graph(b, n, false)) return rc;
    for (int i = 0; i < steps; ++i) BT_CUDA(cudaGraphLaunch(b->exec, b->stream));
    b->steps += (uint64_t)steps;
    for (int s = 0; s < n; ++s) b->pos_host[s] += (size_t)steps;
    return 0;
}

int dcb_batch_read(dcb_batch* b, int n, int* tokens_out, float* logits) {
    if (!b) return bfail(DCB_ERR_ARGUMENT, "null batch");
    if (n < 0 || n > b->slots) return bfail(DCB_ERR_ARGUMENT, "sequence count out of range");
    BT_CUDA(cudaSetDevice(b->device));
    int* hout = b->h_io + b->slots + 1;
    BT_CUDA(cudaMemcpyAsync(hout, b->argmax, (size_t)(b->slots + 1) * sizeof(int), cudaMemcpyDeviceToHost, b->stream));
    BT_CUDA(cudaStreamSynchronize(b->stream));
    if (int rc = device_status(b, hout[b->slots])) return rc;
    if (tokens_out) std::memcpy(tokens_out, hout, (size_t)n * sizeof(int));
    if (logits)
        BT_CUDA(cudaMemcpyAsync(logits, b->logits, (size_t)n * b->M.P.V * sizeof(float), cudaMemcpyDeviceToHost,
                                b->stream));
    BT_CUDA(cudaStreamSynchronize(b->stream));
    return 0;
}

void* dcb_batch_stream(const dcb_batch* b) { return b ? b->stream : nullptr; }

uint64_t dcb_batch_kernels_per_step(const dcb_batch* b, int n) {
    (void)n;
    if (!b) return 0;
    const uint64_t per_layer = 5 + (b->attn64 && b->fuse_combine ? 0 : 1) + (b->fuse_stage ? 0 : 3);
    return 1 + (uint64_t)b->M.P.L * per_layer + 2;
}

// Prefill of an engine's prompt in batched form. The reference prefills one
// token at a time (src/main.cpp:134-137: Engine::step with the head only on
// the last token); here up to 64 consecutive positions form one batched step
// whose slots share the engine's cache: the QKV projection writes every
// slot's K/V row at its position, then each slot attends over positions 0 ..
// its own (causal), so the rows and the last token's logits are those of the
// token-by-token steps (up to the rounding of the batched staging, which
// scales each token's activations as a whole vector).
// all_logits: every position's logits ([n][V], host) and argmax ([n], host,
// or null), the LM head on every chunk; else only the last token's.
static int prefill_impl(dcb_engine* e, const int* tokens, int n, float* logits, int* argmax_out, bool all_logits) {
    if (!e || !tokens) return bfail(DCB_ERR_ARGUMENT, "null argument");
    if (all_logits && !logits) return bfail(DCB_ERR_ARGUMENT, "null logits buffer");
    if (n < 1) return bfail(DCB_ERR_ARGUMENT, "prefill needs at least one token");
    EngineKV kv;
    if (int rc = engine_kv(e, &kv)) return rc;
    if (!kv.whole_sequence)
        return bfail(DCB_ERR_UNSUPPORTED, "prefill needs an engine that keeps the whole sequence (no KV split)");
    if (kv.pos + (size_t)n > kv.capacity) return bfail(DCB_ERR_CAPACITY, "context capacity exceeded");
    dcb_batch*& b = engine_prefill_batch(e);
    if (b && b->capacity != kv.capacity) {
        dcb_batch_destroy(b);
        b = nullptr;
    }
    if (!b)
        if (int rc = create_batch(e, MAX_SLOTS, kv.capacity, kv.kv_dtype, kv.kcache, kv.vcache, &b)) return rc;
    const int V = b->M.P.V;
    for (int i = 0; i < n; ++i)
        if (tokens[i] < 0 || tokens[i] >= V) return bfail(DCB_ERR_TOKEN, "token ID outside vocabulary");
    BT_CUDA(cudaSetDevice(b->device));
    // The engine's earlier steps have written their rows.
    BT_CUDA(cudaStreamSynchronize(static_cast<cudaStream_t>(kv.stream)));
    int* hout = b->h_io + b->slots + 1;
    for (int c = 0; c < n; c += b->slots) {
        const int m = std::min(b->slots, n - c);
        const bool last = c + m == n, head = all_logits || last;
        BT_CUDA(cudaStreamSynchronize(b->stream));  // h_io and h_pos are reused
        for (int i = 0; i < m; ++i) {
            b->h_io[i] = tokens[c + i];
            b->h_pos[i] = (int)(kv.pos + (size_t)(c + i));
        }
        BT_CUDA(cudaMemcpyAsync(b->tokens, b->h_io, (size_t)m * sizeof(int), cudaMemcpyHostToDevice, b->stream));
        BT_CUDA(cudaMemcpyAsync(b->pos, b->h_pos, (size_t)m * sizeof(int), cudaMemcpyHostToDevice, b->stream));
        if (int rc = build_graph(b, m, head && logits != nullptr, head)) return rc;
        BT_CUDA(cudaGraphLaunch(b->exec, b->stream));
        if (!head) continue;
        if (all_logits)
            BT_CUDA(cudaMemcpyAsync(logits + (size_t)c * V, b->logits, (size_t)m * V * sizeof(float),
                                    cudaMemcpyDeviceToHost, b->stream));
        else if (logits)
            BT_CUDA(cudaMemcpyAsync(logits, b->logits + (size_t)(m - 1) * V, (size_t)V * sizeof(float),
                                    cudaMemcpyDeviceToHost, b->stream));
        BT_CUDA(cudaMemcpyAsync(hout, b->argmax, (size_t)(b->slots + 1) * sizeof(int), cudaMemcpyDeviceToHost,
                                b->stream));
        BT_CUDA(cudaStreamSynchronize(b->stream));
        if (int rc = device_status(b, hout[b->slots])) return rc;
        if (all_logits && argmax_out) std::memcpy(argmax_out + c, hout, (size_t)m * sizeof(int));
        if (!all_logits && argmax_out) *argmax_out = hout[m - 1];
    }
    engine_advance(e, (size_t)n);
    return 0;
}

int dcb_prefill(dcb_engine* e, const int* tokens, int n, float* logits, int* argmax_out) {
    return prefill_impl(e, tokens, n, logits, argmax_out, false);
}

// The reference's `logits` command (src/main.cpp:93-114) steps every prompt
// token with the head on and writes each position's logits to PREFIX.bin;
// this is that stream from batched steps.
int dcb_prefill_logits(dcb_engine* e, const int* tokens, int n, float* logits, int* argmax_out) {
    return prefill_impl(e, tokens, n, logits, argmax_out, true);
}

}  // extern "C"
