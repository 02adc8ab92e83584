/* decode_b200.h — C ABI of the B200 (sm_100a) int8 decode engine.
 *
 * Plain C types only; no exceptions cross this boundary. Every call returns 0
 * (DCB_OK) or an error code; dcb_last_error() gives the message of the last
 * failure on the calling thread. Messages of argument errors are the
 * reference engine's own strings, so a C++ wrapper can rethrow them unchanged.
 *
 * Each entry point names the interface of mottopanikeiku/cpu-decode it
 * replaces (file:line in that project).
 */
#ifndef DECODE_B200_H
#define DECODE_B200_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
    DCB_OK = 0,
    DCB_ERR_ARGUMENT = 1,   /* invalid argument; message says which */
    DCB_ERR_TOKEN = 2,      /* "token ID outside vocabulary" */
    DCB_ERR_CAPACITY = 3,   /* "context capacity exceeded" */
    DCB_ERR_REWIND = 4,     /* "cannot rewind forward" */
    DCB_ERR_CUDA = 5,       /* a CUDA runtime call failed */
    DCB_ERR_DEVICE_WAIT = 6,/* a device-side wait ran out of time; state was reset */
    DCB_ERR_UNSUPPORTED = 7
};

enum { DCB_KV_F32 = 0, DCB_KV_F16 = 1 };

/* One decoder layer, host pointers, reference layout: row-major [rows][cols]
 * int8 matrices with FP32 per-row scales, FP32 vectors
 * (src/model.cpp:159-163, 196-215). */
typedef struct {
    const int8_t *q, *k, *v, *o, *gate, *up, *down;
    const float *q_scales, *k_scales, *v_scales, *o_scales, *gate_scales, *up_scales, *down_scales;
    const float *input_norm, *post_norm, *q_bias, *k_bias, *v_bias;
} dcb_layer_desc;

/* A tied-head Qwen2 model (src/model.cpp:134-158 Config, :192 embedding). The
 * embedding matrix is also the LM head. */
typedef struct {
    int32_t hidden, intermediate, layers, heads, kv_heads, head_dim, vocab;
    float epsilon, theta;
    const int8_t* embed;
    const float* embed_scales;
    const float* final_norm;
    const dcb_layer_desc* layer; /* [layers] */
} dcb_model_desc;

typedef struct dcb_engine dcb_engine;

/* Message of the last failed call on this thread ("" if none). */
const char* dcb_last_error(void);

/* Replaces Engine::Impl::Impl (src/model.cpp:185-229): uploads the weights to
 * the device once, in the engine's own layout, and allocates a device KV cache
 * of `capacity` positions (kv_dtype DCB_KV_F32 or DCB_KV_F16). cached_rope
 * selects the cached (model.cpp:269-274) or direct (kernels.cpp:138-149)
 * angle formula. The host weights may be freed after the call returns. */
int dcb_create(const dcb_model_desc* model, size_t capacity, int kv_dtype, int cached_rope,
               int device, dcb_engine** out);
void dcb_destroy(dcb_engine* e);

/* Same, from a model directory in the reference's format (config.json +
 * model.safetensors[.index.json]), validated like the reference's loader
 * (src/model.cpp:63-158, 185-250) with its messages. `capacity` is checked
 * against max_position_embeddings, as Engine::Engine does (src/model.cpp:187). */
int dcb_create_from_dir(const char* directory, size_t capacity, int kv_dtype, int cached_rope, int device,
                        dcb_engine** out);

/* Set the message returned by dcb_last_error() on this thread. */
void dcb_set_error(const char* message);

/* Replaces Engine::step (src/model.cpp:258-329) plus the caller's argmax
 * (src/main.cpp:35-37). Runs one token at the current position and advances
 * it. With head != 0 the LM head runs: the logits are copied to host_logits
 * (vocab floats) when it is not NULL, and the first index of the maximum to
 * *argmax_out when it is not NULL. With head == 0 neither output is written.
 * Synchronous: returns when the outputs are in host memory. */
int dcb_step(dcb_engine* e, int token, int head, float* host_logits, int* argmax_out);

/* Device-resident variant for callers that chain steps on the GPU: the token
 * is read from device memory `token_dev` when it is not NULL (else `token` is
 * used) and the argmax is written to device memory `argmax_dev` when it is not
 * NULL; both may be the same address, so greedy decoding needs no host round
 * trip. Asynchronous on the engine's stream; errors of the device side are
 * reported by the next dcb_synchronize(). No counterpart in the reference. */
int dcb_step_async(dcb_engine* e, int token, const int* token_dev, int head, int* argmax_dev);
int dcb_synchronize(dcb_engine* e);

/* Engine::rewind / reset / position (src/model.cpp:335-342). */
int dcb_rewind(dcb_engine* e, size_t position);
int dcb_reset(dcb_engine* e);
size_t dcb_position(const dcb_engine* e);

/* The stream the engine launches on (a cudaStream_t; NULL = its own stream). */
int dcb_set_stream(dcb_engine* e, void* stream);
void* dcb_stream(const dcb_engine* e);

/* Device pointer of the last logits (vocab floats) and of the argmax int. */
const float* dcb_logits_device(const dcb_engine* e);

/* KV cache access, for a cache pre-filled from elsewhere (e.g. a long prompt
 * computed by another engine). Rows [start, start+count) of `layer`, each
 * kv_heads*head_dim FP32 values, host memory. Writing rows does not move the
 * position; dcb_set_position() does (it may move forward, unlike rewind).
 * No counterpart in the reference, whose KV cache is private. */
int dcb_kv_write(dcb_engine* e, int layer, size_t start, size_t count, const float* keys, const float* values);
int dcb_kv_read(const dcb_engine* e, int layer, size_t start, size_t count, float* keys, float* values);
int dcb_set_position(dcb_engine* e, size_t position);

/* Launch configuration actually used (for reports): grid blocks, threads per
 * block, shared bytes per block, SM count. */
int dcb_launch_info(const dcb_engine* e, int* blocks, int* threads, int* smem_bytes, int* sms);

/* Number of device kernel launches issued by the engine since creation. */
uint64_t dcb_launch_count(const dcb_engine* e);

/* Phase tracing (diagnostics; no counterpart in the reference, whose Profile
 * times operations on the host). When enabled, every step records per block b
 * and phase k (k = 0 kernel start; 5*l+1..5*l+5 the QKV, ATTN, O, GU, DOWN
 * phases of layer l; 5*L+1 the LM head; 5*L+2 the kernel end) the globaltimer
 * ns at which the block's inputs were ready (ready[k*blocks + b]; 0 when the
 * block had no work in that phase) and at which it finished it (done[...]).
 * Both records hold 512 phase rows of `blocks` entries; rows 400+8k+m of
 * `ready` hold detailed marks m inside phase k (0..4) of one traced layer.
 * dcb_trace_read clears the record after reading it. */
int dcb_trace_enable(dcb_engine* e, int on);
int dcb_trace_read(dcb_engine* e, uint64_t* ready, uint64_t* done, int* phases);

/* ---- one decode stream over several GPUs (KV sequence split) -------------- */

/* No counterpart in the reference (it runs one sequence on one CPU): for very
 * long contexts the KV cache of one stream can be split over up to 8 GPUs of a
 * node, one engine (and one process) per GPU, all on the same model. Every
 * engine runs the whole step; each attends only over the KV positions it
 * keeps, and per layer the engines exchange each head's partial softmax state
 * (max, sum, output) through NVLink peer memory and merge them in rank order,
 * so all of them produce the same logits and tokens. Steps must be issued on
 * all engines alike (same tokens, same order).
 *
 * Setup: each engine exports its exchange buffer (dcb_exchange_buffer,
 * dcb_ipc_handle); the handles are shared between the processes (any
 * transport); each process opens its peers' handles (dcb_ipc_open) and calls
 * dcb_set_kv_shard with the opened pointers, indexed by rank. */
enum { DCB_IPC_HANDLE_BYTES = 64 };

/* The engine's exchange buffer (device memory) and its size in bytes. */
int dcb_exchange_buffer(dcb_engine* e, void** exchange, size_t* bytes);

/* cudaIpcGetMemHandle / cudaIpcOpenMemHandle / cudaIpcCloseMemHandle on a
 * device pointer; handle points to DCB_IPC_HANDLE_BYTES bytes. */
int dcb_ipc_handle(const void* device_ptr, void* handle);
int dcb_ipc_open(const void* handle, void** device_ptr);
int dcb_ipc_close(void* device_ptr);

/* Make e rank `rank` of `world` engines sharing one stream: it keeps the KV
 * rows of absolute positions [kv_begin, kv_end) (kv_end = SIZE_MAX: open, for
 * the last rank, which then keeps the new tokens' rows too), as local rows
 * 0.., and exchanges partials through peer_exchange[q] (rank q's exchange
 * buffer as opened in this process; entry `rank` is ignored). dcb_kv_write,
 * dcb_kv_read and dcb_set_position then take absolute positions. */
int dcb_set_kv_shard(dcb_engine* e, int rank, int world, size_t kv_begin, size_t kv_end,
                     void* const* peer_exchange);

/* ---- isolated operators (device pointers, on `stream`) -------------------- */

/* Replaces decode::matvec for int8 matrices (src/kernels.cpp:107-120):
 * y[r] = scales[r] * sum_j float(w[r][j]) * x[j]  (+ bias[r] when bias != NULL).
 * w is row-major [rows][cols]; cols % 4 == 0. All pointers are device memory. */
int dcb_gemv_i8(const int8_t* w, const float* scales, const float* bias, const float* x, float* y,
                int rows, int cols, void* stream);

/* Replaces decode::attention (src/kernels.cpp:150-179) for one query at
 * position length-1 with the split-half RoPE of that position applied to q
 * first when rope_theta > 0 (cached angle formula, src/model.cpp:222-224,271).
 * keys/values: [length][kv_heads*dim] rows of kv_dtype; q_in, out: heads*dim
 * FP32. Split-KV flash decoding with a log-sum-exp combine. Device pointers. */
int dcb_attention(const float* q_in, const void* keys, const void* values, int kv_dtype, float* out,
                  int length, int heads, int kv_heads, int dim, float rope_theta, void* stream);

/* No counterpart in the reference: its attention (src/kernels.cpp:150-179)
 * works in host memory and needs no scratch. dcb_attention_noalloc is
 * dcb_attention with the same arguments, results and errors, but its scratch
 * (the per-split partial results) lives in one fixed array of
 * DCB_ATTENTION_NOALLOC_SCRATCH_BYTES compiled into this library, one per
 * device, instead of a cudaMallocAsync per call. It is for callers that must
 * not allocate device memory once serving starts: a server that reserved all
 * of HBM up front for weights and KV cache (a per-call allocation can fail
 * there), or a decode loop that keeps the allocator off its latency-critical
 * path (a stream-ordered allocation may grow its pool through the driver).
 * Limit: heads * splits * (dim + 2) * 4 <= DCB_ATTENTION_NOALLOC_SCRATCH_BYTES,
 * with splits chosen as dcb_attention chooses them (about two blocks per SM
 * across the KV heads, 64-position chunks); larger calls return
 * DCB_ERR_ARGUMENT and a message giving the bytes needed. Nothing in the
 * scratch has to start at zero: a call writes every word before it reads it.
 * The scratch is shared: calls on the same device that overlap in time
 * (streams without ordering between them, or concurrent host threads) race on
 * it; issue them on one stream or order them with events. The first call on
 * each device does setup (it looks up the scratch's address with that device
 * current and raises the attention kernels' shared-memory caps, once per
 * device and never lowered) and should come before any stream capture. */
enum { DCB_ATTENTION_NOALLOC_SCRATCH_BYTES = 1 << 20 };
int dcb_attention_noalloc(const float* q_in, const void* keys, const void* values, int kv_dtype, float* out,
                          int length, int heads, int kv_heads, int dim, float rope_theta, void* stream);

/* Replaces decode::rmsnorm (src/kernels.cpp:132-137) on device memory. */
int dcb_rmsnorm(const float* x, const float* weight, float* out, int n, float epsilon, void* stream);

/* Replaces decode::rope (src/kernels.cpp:138-149, direct != 0) and the cached
 * rotation (src/model.cpp:269-297, direct == 0) in place on device memory. */
int dcb_rope(float* x, int heads, int dim, int position, float theta, int direct, void* stream);

/* Index of the first maximum of x[0..n) written to *out (device pointers),
 * std::max_element semantics (src/main.cpp:35-37). */
int dcb_argmax(const float* x, int n, int* out, void* stream);

/* Read-only STREAM-style sweep of HBM on `device`, replacing the reference's
 * host read-bandwidth probe (tools/bandwidth.cpp:58-109, read512 :37-56) as the
 * roofline denominator. An array of mib MiB (32..65536; above the 126 MB L2
 * for an honest number) is filled with word i = i*6364136223846793005 + 1, as
 * the reference does; after a 3-pass warm-up, each of `repeats` samples times
 * `passes` full sweeps of 16-byte streaming loads with CUDA events and stores
 * bytes*passes/seconds/1e9 in gb_per_s[r]. *checksum receives the XOR of all
 * words from one extra sweep; the reference instead prints the XOR of its last
 * timed repeat of `passes` sweeps, which is 0 for an even count, so only the
 * one-sweep value checks the data. The size range is wider than the
 * reference's (its limit is 1024 MiB, under which the B200's 126 MB L2 still
 * holds much of a small array; figures reported here use 2 GiB). Allocates
 * and frees its array (a measurement tool, not a serving path); runs on its
 * own stream, synchronises, and leaves the calling thread's current device as
 * it was. Invalid sizes give DCB_ERR_ARGUMENT ("invalid sweep parameters"). */
int dcb_read_bandwidth(int device, size_t mib, int passes, int repeats, double* gb_per_s, uint64_t* checksum);

/* ---- the quantiser on the GPU ------------------------------------------------
 * decode::quantize_row (src/kernels.cpp:121-131) for a whole BF16 matrix
 * (host, row-major rows x cols): per row the largest magnitude, scale =
 * max/127 (1 for an all-zero row), weight/scale rounded half away from zero
 * and clamped to [-127, 127], in IEEE FP32 as the reference computes it, so
 * out [rows][cols] (host) and scales [rows] (host) are bit-identical to the
 * CPU rule. Non-finite weights: DCB_ERR_ARGUMENT "nonfinite model weight";
 * cols 0: "empty quantization row". Uses `device`, synchronises, restores the
 * calling thread's device. */
int dcb_quantize_rows_bf16(const uint16_t* weights, size_t rows, size_t cols, int8_t* out, float* scales, int device);
/* decode::quantize_model (src/model.cpp:354-417) with every matrix quantised
 * by dcb_quantize_rows_bf16: BF16 checkpoint directory `source` -> per-row
 * int8 checkpoint `output`, the same file byte for byte and the same checks
 * and messages. */
int dcb_quantize_model(const char* source, const char* output, int device);

/* ---- batched decode of independent sequences (one GPU) --------------------
 * No counterpart in the reference, which decodes one sequence per Engine
 * (src/model.cpp:258-329); a caller with many sequences would run one Engine
 * each. Here up to 64 sequences (slots 0..max_seqs-1) step together: every
 * projection is one int8 GEMM on the tensor cores over all sequences, each
 * sequence attends over its own KV cache (capacity positions, kv_dtype), and
 * the argmax of step t becomes sequence s's token of step t+1 on the device.
 * The batch shares the weights of `model` (same device; keep `model` alive
 * while the batch exists; its own KV capacity may be 1). Per sequence the
 * results are those of dcb_step on an engine at the same position with the
 * same KV rows (logits within the FP32 tolerance, not bit-identical). */
typedef struct dcb_batch dcb_batch;
int dcb_batch_create(const dcb_engine* model, int max_seqs, size_t capacity, int kv_dtype, dcb_batch** out);
void dcb_batch_destroy(dcb_batch* b);
/* Sequence slots (max_seqs rounded up to 16), capacity, attention split length. */
int dcb_batch_info(const dcb_batch* b, int* slots, size_t* capacity, int* split_len);
/* Position (rows 0..position-1 of the sequence's cache are its context). */
int dcb_batch_set_position(dcb_batch* b, int seq, size_t position);
size_t dcb_batch_position(const dcb_batch* b, int seq);
/* KV rows [start, start+count) of `layer` of sequence seq: count rows of
 * kv_heads*head_dim FP32 values, in host or device memory. */
int dcb_batch_kv_write(dcb_batch* b, int seq, int layer, size_t start, size_t count, const float* keys,
                       const float* values);
int dcb_batch_kv_read(const dcb_batch* b, int seq, int layer, size_t start, size_t count, float* keys,
                      float* values);
/* One step of sequences 0..n-1: tokens[s] (host; NULL: each sequence's
 * previous argmax), logits [n][vocab] (host, or NULL), argmax_out [n] (host,
 * or NULL). Positions advance by one. Errors as dcb_step. */
int dcb_batch_step(dcb_batch* b, int n, const int* tokens, float* logits, int* argmax_out);
/* `steps` greedy steps of sequences 0..n-1 queued on the batch's stream
 * without host round trips (each step's argmax is the next token); read the
 * last tokens with dcb_batch_read, which also reports a device error. */
int dcb_batch_step_greedy(dcb_batch* b, int n, int steps);
int dcb_batch_read(dcb_batch* b, int n, int* tokens_out, float* logits);
/* The batch's CUDA stream, and the kernels one step launches. */
void* dcb_batch_stream(const dcb_batch* b);
uint64_t dcb_batch_kernels_per_step(const dcb_batch* b, int n);

/* Prefill: tokens[0..n) enter the engine at positions pos .. pos+n-1 in
 * batched form instead of n calls of dcb_step (the reference's prefill loop,
 * src/main.cpp:134-137: Engine::step per prompt token, the LM head on the last
 * only). Up to 64 positions form one batched step on the tensor cores whose
 * slots share the engine's KV cache; each attends causally over positions 0
 * .. its own. The engine's K/V rows and position afterwards are those of the
 * token-by-token steps (rows within the FP32 tolerance, not bit-identical);
 * logits (host, V floats, or NULL) and argmax_out (or NULL) are the last
 * token's. For an engine that keeps the whole sequence (no KV split); runs
 * after the engine's queued steps and returns when the rows are written.
 * Errors: DCB_ERR_CAPACITY (pos + n > capacity), DCB_ERR_TOKEN, as dcb_step. */
int dcb_prefill(dcb_engine* e, const int* tokens, int n, float* logits, int* argmax_out);
/* The same prefill with the LM head on every position: logits [n][vocab]
 * (host, required) and argmax_out [n] (host, or NULL) of every prompt
 * position, as the reference's `logits` command writes them
 * (src/main.cpp:93-114: one step with the head per token, PREFIX.bin rows).
 * Each chunk of up to 64 positions is copied back as it completes. */
int dcb_prefill_logits(dcb_engine* e, const int* tokens, int n, float* logits, int* argmax_out);

#ifdef __cplusplus
}
#endif
#endif
