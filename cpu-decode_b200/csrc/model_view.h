// What another engine on the same device may read of a dcb_engine's uploaded
// model: the device pointers and shapes of the packed weights (step_kernel.cuh
// layout), so a batched engine shares one copy of the weights in HBM.
#pragma once
#include "step_kernel.cuh"

#include <string>
#include <vector>

struct dcb_engine;

namespace dcb {

struct ModelView {
    int device;
    Params P;                   // shapes, packed-row strides, embed/norm/RoPE device pointers
    std::vector<LayerW> layers;  // host copy of the per-layer weight pointers (device memory)
};

// Fills `out` for engine e. Returns DCB_OK or an error code (message set).
int model_view(const dcb_engine* e, ModelView* out);
void set_last_error(const std::string& msg);

}  // namespace dcb
