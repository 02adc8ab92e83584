// decode::Engine and the free functions of include/decode.hpp, implemented
// over the C ABI of the B200 engine (include/decode_b200.h).
//
// The loader keeps the reference's on-disk contract and its rejections
// (safetensors Store, src/model.cpp:34-133; Config, :134-158; tensor checks,
// :185-250) with the same messages, then hands host pointers into the mapping
// to dcb_create(), which uploads them to HBM once. Each step() is one device
// launch; the logits land in a pinned vector that the caller reads.
#include "decode.hpp"
#include "decode_b200.h"

#include <cuda_runtime.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <chrono>
#include <functional>
#include <cmath>
#include <cstring>
#include <filesystem>
#include <fstream>
#include <limits>
#include <map>
#include <memory>
#include <numeric>
#include <set>
#include <stdexcept>

namespace decode {
namespace {
namespace fs = std::filesystem;

void check(int rc) {
    if (rc != DCB_OK) throw std::runtime_error(dcb_last_error());
}

size_t mul_checked(size_t a, size_t b) {
    if (a && b > std::numeric_limits<size_t>::max() / a) throw std::runtime_error("tensor size overflow");
    return a * b;
}

Json load_json(const fs::path& path) {
    std::ifstream in(path);
    if (!in) throw std::runtime_error("cannot open " + path.string());
    Json j;
    in >> j;
    return j;
}

// ---- checkpoint files ----------------------------------------------------------
// A checkpoint is read in two passes per file. The JSON header first becomes a
// table of validated entries (element type, shape, byte range); then the byte
// ranges are checked to tile the payload exactly. Tensors point into a
// read-only mapping of the file until dcb_create() has copied them to HBM.
// The rejections and their messages are the reference loader's
// (src/model.cpp:34-133), which callers and tests match.

// A whole file mapped read-only; unmapped when the last owner lets go.
using FileBytes = std::shared_ptr<const char>;
FileBytes map_whole_file(const fs::path& path, size_t* size) {
    const int fd = ::open(path.c_str(), O_RDONLY);
    if (fd < 0) throw std::runtime_error("cannot open " + path.string());
    struct stat info{};
    const bool sized = ::fstat(fd, &info) == 0 && info.st_size >= 8;
    void* addr = sized ? ::mmap(nullptr, size_t(info.st_size), PROT_READ, MAP_PRIVATE, fd, 0) : MAP_FAILED;
    ::close(fd);
    if (!sized) throw std::runtime_error("invalid safetensors file");
    if (addr == MAP_FAILED) throw std::runtime_error("mmap failed: " + path.string());
    const size_t n = size_t(info.st_size);
    *size = n;
    return FileBytes(static_cast<const char*>(addr), [n](const char* q) { ::munmap(const_cast<char*>(q), n); });
}

struct ElementType {
    const char* tag;
    DType type;
    size_t width;
};
constexpr ElementType kElementTypes[] = {{"BF16", DType::bf16, 2}, {"F32", DType::f32, 4}, {"I8", DType::i8, 1}};

struct TensorView {
    const void* data = nullptr;
    std::vector<size_t> shape;
    DType type = DType::f32;
    size_t bytes = 0;
    size_t count() const {
        return std::accumulate(shape.begin(), shape.end(), size_t(1), [](size_t a, size_t b) { return mul_checked(a, b); });
    }
    float value(size_t i) const {
        switch (type) {
            case DType::bf16: return bf16_float(static_cast<const uint16_t*>(data)[i]);
            case DType::i8: return float(static_cast<const int8_t*>(data)[i]);
            default: {
                float v;
                std::memcpy(&v, static_cast<const char*>(data) + 4 * i, 4);
                return v;
            }
        }
    }
};

// One header entry, validated against the payload it indexes (origin: the
// payload's offset in the file, for the alignment rule).
struct HeaderEntry {
    TensorView view;
    size_t begin = 0, end = 0;
};
HeaderEntry read_entry(const std::string& name, const Json& e, size_t origin, size_t payload) {
    HeaderEntry out;
    const std::string tag = e.at("dtype").get<std::string>();
    const auto* et = std::find_if(std::begin(kElementTypes), std::end(kElementTypes),
                                  [&](const ElementType& x) { return tag == x.tag; });
    if (et == std::end(kElementTypes)) throw std::runtime_error("unsupported tensor dtype: " + tag);
    out.view.type = et->type;
    for (const Json& d : e.at("shape")) {
        if (!d.is_number_integer() || d.get<int64_t>() <= 0) throw std::runtime_error("invalid tensor shape");
        out.view.shape.push_back(d.get<size_t>());
    }
    if (out.view.shape.empty() || out.view.shape.size() > 2) throw std::runtime_error("expected vector or matrix tensor");
    const Json& range = e.at("data_offsets");
    if (range.size() != 2 || !range[0].is_number_unsigned() || !range[1].is_number_unsigned())
        throw std::runtime_error("invalid tensor offsets");
    out.begin = range[0].get<size_t>();
    out.end = range[1].get<size_t>();
    out.view.bytes = mul_checked(out.view.count(), et->width);
    const bool inside = out.begin <= out.end && out.end <= payload;
    if (!inside || out.end - out.begin != out.view.bytes || (origin + out.begin) % et->width)
        throw std::runtime_error("tensor bounds/alignment mismatch: " + name);
    return out;
}

// The entries' byte ranges must cover [0, payload) once each, in any order.
void check_tiling(std::vector<std::pair<size_t, size_t>> ranges, size_t payload) {
    std::sort(ranges.begin(), ranges.end());
    const auto seam = std::adjacent_find(ranges.begin(), ranges.end(),
                                         [](const auto& a, const auto& b) { return a.second != b.first; });
    if ((!ranges.empty() && ranges.front().first != 0) || seam != ranges.end())
        throw std::runtime_error("gapped or overlapping safetensors payload");
    if ((ranges.empty() ? 0 : ranges.back().second) != payload) throw std::runtime_error("unindexed safetensors payload");
}

// Shard file names of a checkpoint directory: the index's weight map, or the
// single model.safetensors.
std::set<std::string> shard_names(const fs::path& dir) {
    std::set<std::string> names;
    if (!fs::exists(dir / "model.safetensors.index.json")) return {"model.safetensors"};
    for (const auto& kv : load_json(dir / "model.safetensors.index.json").at("weight_map").items()) {
        const std::string shard = kv.value().get<std::string>();
        if (fs::path(shard).filename() != shard) throw std::runtime_error("unsafe shard filename");
        names.insert(shard);
    }
    return names;
}

// All tensors of a (possibly sharded) checkpoint, validated.
class TensorStore {
public:
    explicit TensorStore(const fs::path& dir) {
        const uint32_t probe = 0x01020304u;
        if (reinterpret_cast<const unsigned char*>(&probe)[0] != 0x04) throw std::runtime_error("little-endian host required");
        for (const std::string& shard : shard_names(dir)) index_file(dir / shard);
    }
    const TensorView& get(const std::string& name, const std::vector<size_t>& shape) const {
        const auto it = tensors.find(name);
        if (it == tensors.end()) throw std::runtime_error("missing tensor: " + name);
        if (it->second.shape != shape) throw std::runtime_error("wrong shape: " + name);
        return it->second;
    }
    std::map<std::string, TensorView> tensors;

private:
    void index_file(const fs::path& path) {
        size_t size = 0;
        FileBytes bytes = map_whole_file(path, &size);
        uint64_t header_len = 0;
        std::memcpy(&header_len, bytes.get(), 8);
        if (header_len > 64ull * 1024 * 1024 || header_len > size - 8)
            throw std::runtime_error("invalid safetensors header length");
        const size_t origin = 8 + size_t(header_len), payload = size - origin;
        const Json header = Json::parse(bytes.get() + 8, bytes.get() + origin);
        // Pass 1: the entry table.
        std::vector<std::pair<std::string, HeaderEntry>> table;
        for (const auto& item : header.items())
            if (item.key() != "__metadata__") table.emplace_back(item.key(), read_entry(item.key(), item.value(), origin, payload));
        // Pass 2: the byte ranges tile the payload.
        std::vector<std::pair<size_t, size_t>> ranges;
        ranges.reserve(table.size());
        for (auto& [name, entry] : table) {
            entry.view.data = bytes.get() + origin + entry.begin;
            if (!tensors.emplace(name, entry.view).second) throw std::runtime_error("duplicate tensor: " + name);
            ranges.emplace_back(entry.begin, entry.end);
        }
        check_tiling(std::move(ranges), payload);
        files.push_back(std::move(bytes));
    }
    std::vector<FileBytes> files;
};

// config.json of a tied-head Qwen2 checkpoint (the reference's accepted set
// and messages, src/model.cpp:134-158).
struct ModelConfig {
    size_t hidden = 0, intermediate = 0, layers = 0, heads = 0, kv_heads = 0, vocab = 0, max_positions = 0, dim = 0;
    float epsilon = 0, theta = 0;
    explicit ModelConfig(const Json& j) {
        if (j.at("model_type") != "qwen2" || !j.value("tie_word_embeddings", false))
            throw std::runtime_error("requires tied-head Qwen2 architecture");
        if (j.contains("rope_scaling") && !j["rope_scaling"].is_null())
            throw std::runtime_error("scaled RoPE is not supported");
        if (j.value("hidden_act", std::string("silu")) != "silu") throw std::runtime_error("requires SiLU");
        static const std::pair<const char*, size_t ModelConfig::*> kDims[] = {
            {"hidden_size", &ModelConfig::hidden},          {"intermediate_size", &ModelConfig::intermediate},
            {"num_hidden_layers", &ModelConfig::layers},    {"num_attention_heads", &ModelConfig::heads},
            {"num_key_value_heads", &ModelConfig::kv_heads}, {"vocab_size", &ModelConfig::vocab},
            {"max_position_embeddings", &ModelConfig::max_positions}};
        for (const auto& [key, member] : kDims) {
            const int64_t n = j.at(key).get<int64_t>();
            if (n <= 0 || n > 1000000) throw std::runtime_error(std::string("invalid config: ") + key);
            this->*member = size_t(n);
        }
        epsilon = j.at("rms_norm_eps").get<float>();
        theta = j.at("rope_theta").get<float>();
        const bool shapes_ok = hidden % heads == 0 && heads % kv_heads == 0 && (hidden / heads) % 2 == 0;
        const bool constants_ok = std::isfinite(epsilon) && epsilon > 0 && std::isfinite(theta) && theta > 0;
        if (!shapes_ok || !constants_ok) throw std::runtime_error("invalid Qwen dimensions or constants");
        dim = hidden / heads;
        if (j.contains("head_dim") && j["head_dim"].get<size_t>() != dim) throw std::runtime_error("incompatible head_dim");
    }
};

// The reference's operation buckets (src/kernels.cpp:181-182), plus
// device_step: the GPU runs the whole step as one kernel, so its wall time
// (launch, kernel, logits copy) is attributed there as one bucket.
const char* const kOperations[] = {"embedding", "rmsnorm", "qkv", "rope", "kv_write", "attention",
                                   "attention_output", "residual", "mlp_gate_up", "silu", "mlp_down",
                                   "lm_head", "argmax", "device_step", "timing_overhead_and_loop"};

}  // namespace

// A validated model directory and the C description of its tensors, which
// point into the file mapping (src/model.cpp:185-250).
struct LoadedModel {
    ModelConfig config;
    TensorStore store;
    dcb_model_desc desc{};
    std::vector<dcb_layer_desc> layers;
    uint64_t stored_bytes = 0, stored_scales = 0;

    explicit LoadedModel(const std::string& dir)
        : config(load_json(fs::path(dir) / "config.json")), store(dir) {}

    // Tensor checks of the reference engine; call after the capacity checks so
    // errors surface in the reference's order.
    void describe() {
        const TensorView& emb = store.get("model.embed_tokens.weight", {config.vocab, config.hidden});
        if (emb.type == DType::f32) throw std::runtime_error("full FP32 model is not supported");
        if (emb.type != DType::i8)
            throw std::runtime_error("the B200 engine runs per-row int8 models; quantize the BF16 checkpoint first");
        if (store.tensors.count("lm_head.weight")) throw std::runtime_error("tied model must not store duplicate lm_head.weight");
        desc.hidden = int32_t(config.hidden);
        desc.intermediate = int32_t(config.intermediate);
        desc.layers = int32_t(config.layers);
        desc.heads = int32_t(config.heads);
        desc.kv_heads = int32_t(config.kv_heads);
        desc.head_dim = int32_t(config.dim);
        desc.vocab = int32_t(config.vocab);
        desc.epsilon = config.epsilon;
        desc.theta = config.theta;
        desc.embed = static_cast<const int8_t*>(emb.data);
        desc.embed_scales = scales("model.embed_tokens.weight", config.vocab);
        layers.assign(config.layers, dcb_layer_desc{});
        const size_t H = config.hidden, I = config.intermediate, KVD = config.kv_heads * config.dim;
        for (size_t l = 0; l < config.layers; ++l) {
            const std::string b = "model.layers." + std::to_string(l) + ".";
            dcb_layer_desc& L = layers[l];
            L.q = int8_matrix(b + "self_attn.q_proj.weight", H, H, &L.q_scales);
            L.k = int8_matrix(b + "self_attn.k_proj.weight", KVD, H, &L.k_scales);
            L.v = int8_matrix(b + "self_attn.v_proj.weight", KVD, H, &L.v_scales);
            L.o = int8_matrix(b + "self_attn.o_proj.weight", H, H, &L.o_scales);
            L.gate = int8_matrix(b + "mlp.gate_proj.weight", I, H, &L.gate_scales);
            L.up = int8_matrix(b + "mlp.up_proj.weight", I, H, &L.up_scales);
            L.down = int8_matrix(b + "mlp.down_proj.weight", H, I, &L.down_scales);
            L.input_norm = vector(b + "input_layernorm.weight", H);
            L.post_norm = vector(b + "post_attention_layernorm.weight", H);
            L.q_bias = vector(b + "self_attn.q_proj.bias", H);
            L.k_bias = vector(b + "self_attn.k_proj.bias", KVD);
            L.v_bias = vector(b + "self_attn.v_proj.bias", KVD);
        }
        desc.final_norm = vector("model.norm.weight", H);
        desc.layer = layers.data();
        for (const auto& item : store.tensors) {
            const std::string& n = item.first;
            if (n.size() >= 7 && n.compare(n.size() - 7, 7, ".scales") == 0) stored_scales += item.second.bytes;
            else stored_bytes += item.second.bytes;
        }
    }
    const float* scales(const std::string& name, size_t rows) {
        const TensorView& s = store.get(name + ".scales", {rows});
        if (s.type != DType::f32) throw std::runtime_error("scales must be FP32");
        const float* p = static_cast<const float*>(s.data);
        for (size_t j = 0; j < rows; ++j)
            if (!std::isfinite(p[j]) || p[j] <= 0) throw std::runtime_error("invalid quantization scale");
        return p;
    }
    const int8_t* int8_matrix(const std::string& name, size_t rows, size_t cols, const float** out_scales) {
        const TensorView& t = store.get(name, {rows, cols});
        if (t.type != DType::i8) throw std::runtime_error("mixed matrix dtypes are not supported");
        *out_scales = scales(name, rows);
        return static_cast<const int8_t*>(t.data);
    }
    const float* vector(const std::string& name, size_t n) {
        const TensorView& t = store.get(name, {n});
        if (t.type != DType::f32) throw std::runtime_error("norms/biases must be floating point (FP32 in quantized model)");
        const float* p = static_cast<const float*>(t.data);
        for (size_t j = 0; j < n; ++j)
            if (!std::isfinite(p[j])) throw std::runtime_error("nonfinite norm or bias");
        return p;
    }
};

// ---------------------------------------------------------------------------
struct Engine::Impl {
    LoadedModel model;
    const ModelConfig& config;
    Kernel kernel;
    int threads;
    bool cached_rope;
    size_t capacity;
    std::string weight_dtype = "int8";
    std::vector<float> logits;
    bool logits_registered = false;
    dcb_engine* engine = nullptr;
    std::string device_name;

    Impl(const std::string& dir, Kernel k, int nthreads, size_t cap, bool cached)
        : model(dir), config(model.config), kernel(k), threads(nthreads), cached_rope(cached), capacity(cap) {
        if (threads < 1 || threads > 1024 || !capacity || capacity > config.max_positions)
            throw std::runtime_error("invalid thread count or context capacity");
        parse_kernel(kernel_name(kernel));
        const size_t kv_bytes =
            mul_checked(mul_checked(mul_checked(capacity, config.kv_heads * config.dim), config.layers), 2 * sizeof(float));
        if (kv_bytes > 768ull * 1024 * 1024) throw std::runtime_error("KV cache exceeds 768MiB safety limit");
        model.describe();
        int device = 0;
        cudaGetDevice(&device);
        check(dcb_create(&model.desc, capacity, DCB_KV_F32, cached_rope ? 1 : 0, device, &engine));
        cudaDeviceProp prop{};
        if (cudaGetDeviceProperties(&prop, device) == cudaSuccess) device_name = prop.name;
        logits.assign(config.vocab, 0.0f);
        logits_registered =
            cudaHostRegister(logits.data(), logits.size() * sizeof(float), cudaHostRegisterDefault) == cudaSuccess;
        if (!logits_registered) cudaGetLastError();
    }
    ~Impl() {
        if (logits_registered) cudaHostUnregister(logits.data());
        dcb_destroy(engine);
    }

    // Algorithmic byte model of the reference (src/model.cpp:251-257, 268, 311-316, 321-325).
    void account(Profile* p, size_t pos, bool head) const {
        if (!p) return;
        const uint64_t H = config.hidden, I = config.intermediate, KVD = config.kv_heads * config.dim, V = config.vocab;
        p->embedding_bytes += H + 4;
        ++p->steps;
        for (size_t l = 0; l < config.layers; ++l) {
            p->matrix_weight_bytes += H * H + 2 * KVD * H + H * H + 2 * I * H + H * I;
            p->scale_bytes += (H + 2 * KVD + H + 2 * I + H) * 4;
            p->norm_bias_bytes += (2 * H + H + 2 * KVD) * 4;
            p->kv_write_bytes += 2 * KVD * 4;
            p->kv_read_min_bytes += 2 * (pos + 1) * KVD * 4;
            p->kv_read_logical_bytes += 2 * (pos + 1) * H * 4;
        }
        if (head) {
            p->matrix_weight_bytes += V * H;
            p->scale_bytes += V * 4;
            p->norm_bias_bytes += H * 4;
            ++p->head_steps;
            p->lm_head_weight_bytes += V * H;
            p->lm_head_scale_bytes += V * 4;
        }
    }

    const std::vector<float>& step(int token, bool head, Profile* p) {
        const size_t pos = dcb_position(engine);
        const auto start = std::chrono::steady_clock::now();
        check(dcb_step(engine, token, head ? 1 : 0, head ? logits.data() : nullptr, nullptr));
        if (p) p->seconds["device_step"] += std::chrono::duration<double>(std::chrono::steady_clock::now() - start).count();
        account(p, pos, head);
        return logits;
    }
};

Engine::Engine(const std::string& dir, Kernel kernel, int threads, size_t capacity, bool cached_rope)
    : impl(std::make_unique<Impl>(dir, kernel, threads, capacity, cached_rope)) {}
Engine::~Engine() = default;
Engine::Engine(Engine&&) noexcept = default;
Engine& Engine::operator=(Engine&&) noexcept = default;
void Engine::reset() { check(dcb_reset(impl->engine)); }
void Engine::rewind(size_t position) { check(dcb_rewind(impl->engine, position)); }
const std::vector<float>& Engine::step(int token, bool head, Profile* profile) { return impl->step(token, head, profile); }
size_t Engine::vocab_size() const { return impl->config.vocab; }
size_t Engine::position() const { return dcb_position(impl->engine); }
Json Engine::metadata() const {
    const auto& c = impl->config;
    int blocks = 0, nthreads = 0, smem = 0, sms = 0;
    dcb_launch_info(impl->engine, &blocks, &nthreads, &smem, &sms);
    return {{"weight_dtype", impl->weight_dtype},
            {"quantization", "symmetric per-row int8, float32 scales, float32 activations"},
            {"kernel", kernel_name(impl->kernel)},
            {"kernel_scope", "whole decode step in one persistent sm_100a kernel; per-operation timers are not separable, "
                             "the step's wall time is the device_step bucket"},
            {"threads", impl->threads},
            {"stored_weight_bytes", impl->model.stored_bytes},
            {"rope", impl->cached_rope ? "cached" : "direct"},
            {"thread_scheduling", "cooperative launch, one " + std::to_string(nthreads) + "-thread block per SM (" +
                                      std::to_string(blocks) + " blocks); blocks hand activations to each other through "
                                      "L2 (tagged words and self-counting sums), no grid barriers"},
            {"stored_scale_bytes", impl->model.stored_scales},
            {"kv_capacity", impl->capacity},
            {"auxiliary_fp32_weight_bytes", (c.layers * (3 * c.hidden + 2 * c.kv_heads * c.dim) + c.hidden) * 4},
            {"kv_cache_bytes", impl->capacity * c.kv_heads * c.dim * c.layers * 2 * 4},
            {"tied_head", true},
            {"vocab_size", c.vocab},
            {"device", impl->device_name}};
}

// ---------------------------------------------------------------------------
// Profile (include/decode.hpp:31-40; src/kernels.cpp:180-193)
Profile::Profile() {
    for (const char* name : kOperations) seconds.emplace(name, 0.0);
}
Json Profile::json() const {
    const uint64_t minimum =
        matrix_weight_bytes + scale_bytes + norm_bias_bytes + embedding_bytes + kv_write_bytes + kv_read_min_bytes;
    return {{"operation_seconds", seconds}, {"steps", steps}, {"head_steps", head_steps},
            {"matrix_weight_bytes", matrix_weight_bytes}, {"scale_bytes", scale_bytes},
            {"lm_head_weight_bytes", lm_head_weight_bytes}, {"lm_head_scale_bytes", lm_head_scale_bytes},
            {"norm_bias_bytes", norm_bias_bytes}, {"embedding_bytes", embedding_bytes},
            {"kv_write_bytes", kv_write_bytes}, {"kv_read_min_bytes", kv_read_min_bytes},
            {"kv_read_logical_bytes", kv_read_logical_bytes}, {"minimum_bytes", minimum},
            {"byte_model", "algorithmic weight/scale reads plus embedding row, FP32 KV writes and minimum GQA KV reads; "
                           "excludes activation/cache-line/allocator traffic"}};
}

// ---------------------------------------------------------------------------
// Free functions
Kernel parse_kernel(const std::string& name) {
    // The names select CPU instruction sets in the reference; the B200 engine
    // accepts all four and records the choice.
    if (name == "scalar") return Kernel::scalar;
    if (name == "simd256") return Kernel::simd256;
    if (name == "simd512") return Kernel::simd512;
    if (name == "simd512x4") return Kernel::simd512x4;
    throw std::runtime_error("unknown or unsupported kernel: " + name);
}
std::string kernel_name(Kernel k) {
    if (k == Kernel::scalar) return "scalar";
    if (k == Kernel::simd256) return "simd256";
    if (k == Kernel::simd512) return "simd512";
    return "simd512x4";
}
float bf16_float(uint16_t value) {
    const uint32_t bits = uint32_t(value) << 16;
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}

namespace {
// Device scratch for the free functions, freed on scope exit.
struct DeviceBuffer {
    void* p = nullptr;
    explicit DeviceBuffer(size_t bytes) {
        if (cudaMalloc(&p, std::max<size_t>(bytes, 16)) != cudaSuccess) throw std::runtime_error("cudaMalloc failed");
    }
    ~DeviceBuffer() { cudaFree(p); }
    template <class T> T* as() const { return static_cast<T*>(p); }
};
void to_device(void* dst, const void* src, size_t bytes) {
    if (cudaMemcpy(dst, src, bytes, cudaMemcpyHostToDevice) != cudaSuccess) throw std::runtime_error("cudaMemcpy failed");
}
void to_host(void* dst, const void* src, size_t bytes) {
    if (cudaMemcpy(dst, src, bytes, cudaMemcpyDeviceToHost) != cudaSuccess) throw std::runtime_error("cudaMemcpy failed");
}
}  // namespace

void matvec(const Matrix& m, const float* x, float* y, Kernel, int threads) {
    if (!m.data || !m.rows || !m.cols || (m.dtype == DType::i8 && !m.scales) || threads < 1)
        throw std::runtime_error("invalid matvec arguments");
    if (m.dtype != DType::i8) throw std::runtime_error("the B200 matvec runs per-row int8 matrices");
    DeviceBuffer w(m.rows * m.cols), s(m.rows * 4), dx(m.cols * 4), dy(m.rows * 4);
    to_device(w.p, m.data, m.rows * m.cols);
    to_device(s.p, m.scales, m.rows * 4);
    to_device(dx.p, x, m.cols * 4);
    check(dcb_gemv_i8(w.as<int8_t>(), s.as<float>(), nullptr, dx.as<float>(), dy.as<float>(), int(m.rows),
                      int(m.cols), nullptr));
    to_host(y, dy.p, m.rows * 4);
}

void rmsnorm(const float* x, const float* weight, float* out, size_t n, float epsilon) {
    DeviceBuffer dx(n * 4), dw(n * 4), dout(n * 4);
    to_device(dx.p, x, n * 4);
    to_device(dw.p, weight, n * 4);
    check(dcb_rmsnorm(dx.as<float>(), dw.as<float>(), dout.as<float>(), int(n), epsilon, nullptr));
    to_host(out, dout.p, n * 4);
}

void rope(float* x, size_t heads, size_t dim, size_t position, float theta) {
    DeviceBuffer dx(heads * dim * 4);
    to_device(dx.p, x, heads * dim * 4);
    check(dcb_rope(dx.as<float>(), int(heads), int(dim), int(position), theta, 1, nullptr));
    to_host(x, dx.p, heads * dim * 4);
}

void attention(const float* q, const float* keys, const float* values, float* out, float*, size_t length,
               size_t heads, size_t kv_heads, size_t dim, int threads) {
    if (!length || !kv_heads || heads % kv_heads || !dim || threads < 1)
        throw std::runtime_error("invalid attention dimensions");
    const size_t kv = length * kv_heads * dim * 4;
    DeviceBuffer dq(heads * dim * 4), dk(kv), dv(kv), dout(heads * dim * 4);
    to_device(dq.p, q, heads * dim * 4);
    to_device(dk.p, keys, kv);
    to_device(dv.p, values, kv);
    check(dcb_attention(dq.as<float>(), dk.p, dv.p, DCB_KV_F32, dout.as<float>(), int(length), int(heads),
                        int(kv_heads), int(dim), 0.0f, nullptr));
    if (cudaDeviceSynchronize() != cudaSuccess) throw std::runtime_error("attention failed");
    to_host(out, dout.p, heads * dim * 4);
}

// Offline per-row quantiser (the format tool; src/kernels.cpp:121-131). The
// rule: the row's scale is its largest magnitude over 127 (1 for an all-zero
// row); each weight becomes weight / scale rounded half away from zero and
// clamped to [-127, 127]. Non-finite weights and empty rows are rejected.
void quantize_row(const float* source, size_t n, int8_t* out, float& scale) {
    if (!n) throw std::runtime_error("empty quantization row");
    const float* const last = source + n;
    if (std::find_if(source, last, [](float v) { return !std::isfinite(v); }) != last)
        throw std::runtime_error("nonfinite model weight");
    const float peak = std::accumulate(source, last, 0.0f, [](float m, float v) { return std::max(m, std::fabs(v)); });
    scale = peak > 0.0f ? peak / 127.0f : 1.0f;
    const float s = scale;
    std::transform(source, last, out, [s](float v) {
        const float q = std::round(v / s);  // halves away from zero
        return static_cast<int8_t>(q > 127.0f ? 127.0f : (q < -127.0f ? -127.0f : q));
    });
}

namespace {
// Quantises one BF16 matrix (rows x cols, a view into the mapped file) into
// q [rows][cols] and per-row scales.
using MatrixQuantizer = std::function<void(const TensorView&, size_t rows, size_t cols, int8_t* q, float* scales)>;

// BF16 checkpoint -> per-row int8 checkpoint in the reference's file layout
// (src/model.cpp:354-417): name-ordered tensors, matrices as I8 followed by
// "<name>.scales" F32, vectors as F32, header padded to 8 bytes.
void write_quantized(const std::string& source, const std::string& output, const MatrixQuantizer& quantize_matrix) {
    const fs::path src(source), dst(output);
    if (fs::weakly_canonical(src) == fs::weakly_canonical(dst)) throw std::runtime_error("quantization output must differ from input");
    const ModelConfig config(load_json(src / "config.json"));
    TensorStore store(src);
    if (fs::exists(dst / "model.safetensors") || fs::exists(dst / "config.json"))
        throw std::runtime_error("quantization output already contains a model");
    for (const auto& item : store.tensors) {
        if (item.second.type != DType::bf16) throw std::runtime_error("quantization input must be BF16");
        if (item.second.shape.size() == 2 && item.second.count() % 4)
            throw std::runtime_error("int8 matrices must contain a multiple of four elements");
    }
    if (store.tensors.count("lm_head.weight")) throw std::runtime_error("duplicate tied head in input");
    (void)config;
    Json header;
    uint64_t offset = 0;
    auto entry = [&](const std::string& name, const char* dtype, const std::vector<size_t>& shape, uint64_t bytes) {
        header[name] = {{"dtype", dtype}, {"shape", shape}, {"data_offsets", {offset, offset + bytes}}};
        offset += bytes;
    };
    for (const auto& item : store.tensors) {
        const TensorView& t = item.second;
        if (t.shape.size() == 2) {
            entry(item.first, "I8", t.shape, t.count());
            entry(item.first + ".scales", "F32", {t.shape[0]}, t.shape[0] * 4);
        } else {
            entry(item.first, "F32", t.shape, t.count() * 4);
        }
    }
    header["__metadata__"] = {{"format", "pt"}, {"quantization", "symmetric-per-row-int8"}};
    std::string text = header.dump();
    while (text.size() % 8) text.push_back(' ');
    fs::create_directories(dst);
    const fs::path partial = dst / "model.safetensors.partial";
    try {
        std::ofstream out(partial, std::ios::binary | std::ios::trunc);
        if (!out) throw std::runtime_error("cannot create quantized model");
        const uint64_t n = text.size();
        out.write(reinterpret_cast<const char*>(&n), 8);
        out.write(text.data(), text.size());
        for (const auto& item : store.tensors) {
            const TensorView& t = item.second;
            if (t.shape.size() == 2) {
                const size_t rows = t.shape[0], cols = t.shape[1];
                std::vector<float> sc(rows);
                std::vector<int8_t> q(rows * cols);
                quantize_matrix(t, rows, cols, q.data(), sc.data());
                out.write(reinterpret_cast<const char*>(q.data()), (std::streamsize)q.size());
                out.write(reinterpret_cast<const char*>(sc.data()), rows * 4);
            } else {
                for (size_t j = 0; j < t.count(); ++j) {
                    const float v = t.value(j);
                    if (!std::isfinite(v)) throw std::runtime_error("nonfinite model vector");
                    out.write(reinterpret_cast<const char*>(&v), 4);
                }
            }
            if (!out) throw std::runtime_error("quantization write failed");
        }
        out.close();
        if (!out) throw std::runtime_error("quantization flush failed");
        fs::copy_file(src / "config.json", dst / "config.json");
        fs::rename(partial, dst / "model.safetensors");
    } catch (...) {
        fs::remove(partial);
        throw;
    }
}
}  // namespace

void quantize_model(const std::string& source, const std::string& output) {
    write_quantized(source, output, [](const TensorView& t, size_t rows, size_t cols, int8_t* q, float* sc) {
        std::vector<float> row(cols);
        for (size_t r = 0; r < rows; ++r) {
            for (size_t j = 0; j < cols; ++j) row[j] = t.value(r * cols + j);
            quantize_row(row.data(), cols, q + r * cols, sc[r]);
        }
    });
}

}  // namespace decode

// The same checkpoint with the per-row rule on a GPU (dcb_quantize_rows_bf16):
// the output file is byte for byte the CPU quantiser's.
extern "C" int dcb_quantize_model(const char* source, const char* output, int device) {
    try {
        if (!source || !output) throw std::runtime_error("null argument");
        decode::write_quantized(source, output, [device](const decode::TensorView& t, size_t rows, size_t cols, int8_t* q,
                                                          float* sc) {
            if (dcb_quantize_rows_bf16(static_cast<const uint16_t*>(t.data), rows, cols, q, sc, device) != DCB_OK)
                throw std::runtime_error(dcb_last_error());
        });
        return DCB_OK;
    } catch (const std::exception& e) {
        dcb_set_error(e.what());
        return DCB_ERR_ARGUMENT;
    }
}

// ---------------------------------------------------------------------------
// C entry over the loader, so callers without C++ (ctypes, cgo) open a model
// directory with the same validation and messages as decode::Engine.
extern "C" int dcb_create_from_dir(const char* directory, size_t capacity, int kv_dtype, int cached_rope, int device,
                                   dcb_engine** out) {
    try {
        if (!directory || !out) throw std::runtime_error("null argument");
        decode::LoadedModel model(directory);
        if (!capacity || capacity > model.config.max_positions)
            throw std::runtime_error("invalid thread count or context capacity");
        model.describe();
        return dcb_create(&model.desc, capacity, kv_dtype, cached_rope, device, out);
    } catch (const std::exception& e) {
        dcb_set_error(e.what());
        return DCB_ERR_ARGUMENT;
    }
}
