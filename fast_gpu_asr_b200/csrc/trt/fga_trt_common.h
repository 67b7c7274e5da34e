// Shared pieces of the TensorRT plugin shims: each shim is an IPluginV3 whose enqueue
// converts TensorRT's tensor descriptors to fga_tensor_desc and forwards to the C ABI of
// libfga_attention.so. Plugin names, version, namespace and fields are those of the
// reference plugins (src/fast_gpu_asr/tensorrt_plugins/*_plugin.cu), so engines and ONNX
// graphs that name them resolve to these shims.
#pragma once

#include <NvInfer.h>

#include <cstdint>
#include <cstdio>
#include <limits>

#include "../../../include/fga_attention.h"

#define FGA_TRT_EXPORT extern "C" __attribute__((visibility("default")))

namespace fga_trt {

using namespace nvinfer1;

// The reference's plugin namespace (plugin_namespace.h:12); engines store it.
constexpr char kPluginNamespace[] = "fast_gpu_asr";
constexpr char kVersion[] = "1";
// Part of every timing-cache ID: a new implementation identity invalidates timings that
// TensorRT recorded for another one (the reference's cuBLAS tactics among them).
constexpr char kImplementation[] = "impl=fga-sm100a-tcgen05";

inline bool is_float(DataType t) noexcept {
    return t == DataType::kFLOAT || t == DataType::kHALF || t == DataType::kBF16;
}

inline int64_t element_bytes(DataType t) noexcept {
    switch (t) {
        case DataType::kFLOAT: return 4;
        case DataType::kHALF: return 2;
        case DataType::kBF16: return 2;
        case DataType::kINT32: return 4;
        case DataType::kBOOL: return 1;
        default: return 0;
    }
}

// Every dimension known and positive, and the byte size representable in int64 (the
// reference's hasAddressableBytes on profile bounds).
inline bool addressable(Dims const& d, int64_t bytes) noexcept {
    if (d.nbDims < 1 || d.nbDims > Dims::MAX_DIMS || bytes < 1) return false;
    int64_t total = bytes;
    for (int32_t i = 0; i < d.nbDims; ++i) {
        if (d.d[i] < 1 || d.d[i] > std::numeric_limits<int64_t>::max() / total) return false;
        total *= d.d[i];
    }
    return true;
}

inline bool to_desc(Dims const& dims, DataType type, fga_tensor_desc& out) noexcept {
    if (dims.nbDims < 1 || dims.nbDims > FGA_MAX_DIMS) return false;
    out.type = static_cast<int32_t>(type);  // fga_data_type uses TensorRT's numbering
    out.nb_dims = dims.nbDims;
    for (int32_t i = 0; i < FGA_MAX_DIMS; ++i) out.dims[i] = i < dims.nbDims ? dims.d[i] : 0;
    return true;
}

template <int32_t N>
bool to_descs(PluginTensorDesc const* in, fga_tensor_desc (&out)[N]) noexcept {
    for (int32_t i = 0; i < N; ++i)
        if (!to_desc(in[i].dims, in[i].type, out[i])) return false;
    return true;
}

template <int32_t N>
bool to_descs_max(DynamicPluginTensorDesc const* in, fga_tensor_desc (&out)[N]) noexcept {
    for (int32_t i = 0; i < N; ++i)
        if (!to_desc(in[i].max, in[i].desc.type, out[i])) return false;
    return true;
}

inline bool all_linear(PluginTensorDesc const* d, int32_t n) noexcept {
    for (int32_t i = 0; i < n; ++i)
        if (d[i].format != TensorFormat::kLINEAR) return false;
    return true;
}

// enqueue's convention: 0 on success, 1 on failure; a CUDA error already pending is a
// failure reported without launching (the C ABI checks cudaPeekAtLastError itself).
inline int32_t enqueue_status(int32_t fga_status) noexcept {
    return fga_status == FGA_SUCCESS ? 0 : 1;
}

// IPluginV3 boilerplate shared by the three shims: capability interfaces, identity, one
// output, no tactics to time (one implementation; TensorRT's tactic 0 is the default),
// the timing-cache ID, and attachToContext returning a clone so that each execution
// context owns its instance (the reference's concurrency contract).
template <class Derived>
class ShimBase : public IPluginV3,
                 public IPluginV3OneCore,
                 public IPluginV3OneBuild,
                 public IPluginV3OneRuntime {
  public:
    IPluginCapability* getCapabilityInterface(PluginCapabilityType type) noexcept override {
        switch (type) {
            case PluginCapabilityType::kBUILD: return static_cast<IPluginV3OneBuild*>(this);
            case PluginCapabilityType::kRUNTIME: return static_cast<IPluginV3OneRuntime*>(this);
            case PluginCapabilityType::kCORE: return static_cast<IPluginV3OneCore*>(this);
            default: return nullptr;
        }
    }
    char const* getPluginName() const noexcept override { return Derived::kName; }
    char const* getPluginVersion() const noexcept override { return kVersion; }
    char const* getPluginNamespace() const noexcept override { return kPluginNamespace; }
    int32_t getNbOutputs() const noexcept override { return 1; }
    int32_t getNbTactics() noexcept override { return 0; }
    int32_t getValidTactics(int32_t* tactics, int32_t nbTactics) noexcept override {
        static_cast<void>(tactics);
        static_cast<void>(nbTactics);
        return 0;
    }
    int32_t setTactic(int32_t tactic) noexcept override { return tactic == 0 ? 0 : 1; }
    char const* getTimingCacheID() noexcept override { return timing_id_; }
    IPluginV3* attachToContext(IPluginResourceContext* context) noexcept override {
        static_cast<void>(context);
        return this->clone();
    }

  protected:
    // "<implementation>;abi=<n>;<plugin-specific>": false if it does not fit.
    bool set_timing_id(char const* specific) noexcept {
        const int n = std::snprintf(timing_id_, sizeof(timing_id_), "%s;abi=%d;%s",
                                    kImplementation, FGA_ABI_VERSION, specific);
        return n > 0 && static_cast<size_t>(n) < sizeof(timing_id_);
    }

  private:
    char timing_id_[192] = {};
};

// Registers `runtime` in the runtime registry and `builder` in the builder registry,
// unless a creator of the same name, version and namespace is there already (repeated
// initialisation is a success). True when both registries hold the plugin.
template <class Creator>
bool register_in_both_registries(Creator& runtime, Creator& builder) noexcept {
    auto ensure = [](IPluginRegistry* registry, Creator& creator) noexcept {
        if (registry == nullptr) return false;
        if (registry->getCreator(Creator::kName, kVersion, kPluginNamespace) != nullptr) return true;
        return registry->registerCreator(creator, kPluginNamespace) ||
               registry->getCreator(Creator::kName, kVersion, kPluginNamespace) != nullptr;
    };
    const bool rt = ensure(getPluginRegistry(), runtime);
    const bool bd = ensure(getBuilderPluginRegistry(EngineCapability::kSTANDARD), builder);
    return rt && bd;
}

}  // namespace fga_trt
