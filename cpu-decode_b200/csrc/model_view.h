// What another engine on the same device may read of a dcb_engine's uploaded
// model: the device pointers and shapes of the packed weights (step_kernel.cuh
// layout), so a batched engine shares one copy of the weights in HBM.
#pragma once
#include "step_kernel.cuh"

#include <string>
#include <vector>

struct dcb_engine;
struct dcb_batch;

namespace dcb {

struct ModelView {
    int device;
    Params P;                   // shapes, packed-row strides, embed/norm/RoPE device pointers
    std::vector<LayerW> layers;  // host copy of the per-layer weight pointers (device memory)
};

// Fills `out` for engine e. Returns DCB_OK or an error code (message set).
int model_view(const dcb_engine* e, ModelView* out);

// The KV cache and position of an engine, for the batched prefill that writes
// into it (whole_sequence: one GPU holding every position, no KV shard).
struct EngineKV {
    void* kcache;  // [L][NKV][capacity][D]
    void* vcache;
    size_t capacity, pos;
    int kv_dtype;
    bool whole_sequence;
    void* stream;  // the engine's cudaStream_t
};
int engine_kv(const dcb_engine* e, EngineKV* out);
// Moves the engine's position forward by n after a prefill wrote rows pos .. pos+n-1.
void engine_advance(dcb_engine* e, size_t n);
// The batched context the engine's prefills run in (created on first use,
// destroyed with the engine).
struct dcb_batch*& engine_prefill_batch(dcb_engine* e);
void set_last_error(const std::string& msg);

}  // namespace dcb
