// TensorRT plugin `parakeet_relative_attention` v1 (namespace fast_gpu_asr) over the C ABI.
//
// Drop-in for the reference's ParakeetRelativeAttentionPlugin and its creator
// (src/fast_gpu_asr/tensorrt_plugins/parakeet_relative_attention_plugin.cu:701-1256):
// same name, version, namespace, `scale` field and its validation, bindings, output
// rules and error convention. The computation is fga_parakeet_relative_attention_enqueue
// (the sm_100a tcgen05 kernel); it needs no workspace where the reference needed its
// score buffers.
#include <cmath>
#include <cstring>
#include <new>

#include "fga_trt_common.h"

namespace fga_trt {
namespace {

constexpr char kScaleField[] = "scale";
constexpr float kLog2e = 1.4426950408889634F;

bool scale_ok(float scale) noexcept {
    return std::isfinite(scale) && scale > 0.0F && std::isfinite(scale * kLog2e);
}

class ParakeetPlugin final : public ShimBase<ParakeetPlugin> {
  public:
    static constexpr char kName[] = "parakeet_relative_attention";

    explicit ParakeetPlugin(float scale) noexcept : scale_(scale) {
        char id[96];
        const int n = std::snprintf(id, sizeof(id), "layout=nt3c-ntc;relative=2t-1;scale=%a",
                                    static_cast<double>(scale));
        ok_ = n > 0 && static_cast<size_t>(n) < sizeof(id) && set_timing_id(id);
        field_ = {kScaleField, &scale_, PluginFieldType::kFLOAT32, 1};
        fields_ = {1, &field_};
    }
    bool ok() const noexcept { return ok_; }

    IPluginV3* clone() noexcept override {
        auto* p = new (std::nothrow) ParakeetPlugin(scale_);
        if (p == nullptr || !p->ok()) {
            delete p;
            return nullptr;
        }
        return p;
    }

    // Profile-invariant metadata only (ranks, dtypes, formats, addressable bounds); exact
    // cross-input relations are checked per shape in onShapeChange.
    int32_t configurePlugin(DynamicPluginTensorDesc const* in, int32_t nbInputs,
                            DynamicPluginTensorDesc const* out, int32_t nbOutputs) noexcept override {
        if (in == nullptr || out == nullptr || nbInputs != 5 || nbOutputs != 1 || !ok_) return 1;
        static constexpr int32_t kRanks[5] = {3, 3, 2, 2, 1};
        const DataType t = in[0].desc.type;
        if (!is_float(t) || out[0].desc.type != t || out[0].desc.dims.nbDims != 3 ||
            out[0].desc.format != TensorFormat::kLINEAR ||
            !addressable(out[0].max, element_bytes(t)))
            return 1;
        for (int32_t i = 0; i < 5; ++i) {
            const DataType want = i == 4 ? DataType::kINT32 : t;
            if (in[i].desc.type != want || in[i].desc.dims.nbDims != kRanks[i] ||
                in[i].desc.format != TensorFormat::kLINEAR ||
                !addressable(in[i].max, element_bytes(want)))
                return 1;
        }
        if (in[0].max.d[1] > std::numeric_limits<int32_t>::max() / 2 + 1) return 1;
        return 0;
    }

    int32_t getOutputDataTypes(DataType* outTypes, int32_t nbOutputs, DataType const* inTypes,
                               int32_t nbInputs) const noexcept override {
        if (outTypes == nullptr || inTypes == nullptr || nbInputs != 5 || nbOutputs != 1 ||
            !is_float(inTypes[0]) || inTypes[4] != DataType::kINT32)
            return 1;
        for (int32_t i = 1; i < 4; ++i)
            if (inTypes[i] != inTypes[0]) return 1;
        outTypes[0] = inTypes[0];
        return 0;
    }

    // output [N, T, C]: N and T of qkv, C of the positional table.
    int32_t getOutputShapes(DimsExprs const* in, int32_t nbInputs, DimsExprs const* shapeIn,
                            int32_t nbShapeInputs, DimsExprs* out, int32_t nbOutputs,
                            IExprBuilder& builder) noexcept override {
        static_cast<void>(shapeIn);
        static_cast<void>(builder);
        if (in == nullptr || out == nullptr || nbInputs != 5 || nbOutputs != 1 ||
            nbShapeInputs != 0 || in[0].nbDims != 3 || in[1].nbDims != 3 || in[2].nbDims != 2 ||
            in[3].nbDims != 2 || in[4].nbDims != 1 || in[0].d[0] == nullptr ||
            in[0].d[1] == nullptr || in[1].d[2] == nullptr)
            return 1;
        out[0].nbDims = 3;
        out[0].d[0] = in[0].d[0];
        out[0].d[1] = in[0].d[1];
        out[0].d[2] = in[1].d[2];
        return 0;
    }

    bool supportsFormatCombination(int32_t pos, DynamicPluginTensorDesc const* io,
                                   int32_t nbInputs, int32_t nbOutputs) noexcept override {
        if (io == nullptr || nbInputs != 5 || nbOutputs != 1 || pos < 0 || pos > 5) return false;
        const PluginTensorDesc& d = io[pos].desc;
        if (d.format != TensorFormat::kLINEAR) return false;
        if (pos == 4) return d.type == DataType::kINT32;
        return is_float(d.type) && (pos == 0 || d.type == io[0].desc.type);
    }

    size_t getWorkspaceSize(DynamicPluginTensorDesc const* in, int32_t nbInputs,
                            DynamicPluginTensorDesc const* out,
                            int32_t nbOutputs) const noexcept override {
        fga_tensor_desc d[5];
        if (in == nullptr || out == nullptr || nbInputs != 5 || nbOutputs != 1 ||
            !to_descs_max(in, d))
            return 0;
        return fga_parakeet_relative_attention_workspace_size(d, 5);
    }

    int32_t onShapeChange(PluginTensorDesc const* in, int32_t nbInputs, PluginTensorDesc const* out,
                          int32_t nbOutputs) noexcept override {
        fga_tensor_desc di[5], dout[1];
        if (in == nullptr || out == nullptr || nbInputs != 5 || nbOutputs != 1 || !ok_ ||
            !all_linear(in, 5) || !all_linear(out, 1) || !to_descs(in, di) || !to_descs(out, dout))
            return 1;
        return fga_parakeet_relative_attention_check(di, 5, dout, 1, scale_) == FGA_SUCCESS ? 0 : 1;
    }

    int32_t enqueue(PluginTensorDesc const* inDesc, PluginTensorDesc const* outDesc,
                    void const* const* inputs, void* const* outputs, void* workspace,
                    cudaStream_t stream) noexcept override {
        fga_tensor_desc di[5], dout[1];
        if (inDesc == nullptr || outDesc == nullptr || inputs == nullptr || outputs == nullptr ||
            !to_descs(inDesc, di) || !to_descs(outDesc, dout))
            return 1;
        const size_t ws = fga_parakeet_relative_attention_workspace_size(di, 5);
        return enqueue_status(fga_parakeet_relative_attention_enqueue(
            di, dout, inputs, outputs, scale_, workspace, ws, stream));
    }

    PluginFieldCollection const* getFieldsToSerialize() noexcept override { return &fields_; }

  private:
    float scale_;
    bool ok_ = false;
    PluginField field_{};
    PluginFieldCollection fields_{};
};

class ParakeetCreator final : public IPluginCreatorV3One {
  public:
    static constexpr char const* kName = ParakeetPlugin::kName;

    ParakeetCreator() noexcept {
        attribute_ = {kScaleField, nullptr, PluginFieldType::kFLOAT32, 1};
        names_ = {1, &attribute_};
    }
    char const* getPluginName() const noexcept override { return kName; }
    char const* getPluginVersion() const noexcept override { return kVersion; }
    char const* getPluginNamespace() const noexcept override { return kPluginNamespace; }
    PluginFieldCollection const* getFieldNames() noexcept override { return &names_; }

    // Exactly one field, `scale`, kFLOAT32 of length 1, finite, > 0 and with a finite
    // scale * log2(e) (the reference creator's rules); anything else gives nullptr.
    IPluginV3* createPlugin(char const* name, PluginFieldCollection const* fc,
                            TensorRTPhase phase) noexcept override {
        static_cast<void>(name);
        static_cast<void>(phase);
        if (fc == nullptr || fc->fields == nullptr || fc->nbFields != 1) return nullptr;
        const PluginField& f = fc->fields[0];
        if (f.name == nullptr || std::strcmp(f.name, kScaleField) != 0 ||
            f.type != PluginFieldType::kFLOAT32 || f.length != 1 || f.data == nullptr)
            return nullptr;
        const float scale = *static_cast<float const*>(f.data);
        if (!scale_ok(scale)) return nullptr;
        auto* p = new (std::nothrow) ParakeetPlugin(scale);
        if (p == nullptr || !p->ok()) {
            delete p;
            return nullptr;
        }
        return p;
    }

  private:
    PluginField attribute_{};
    PluginFieldCollection names_{};
};

}  // namespace
}  // namespace fga_trt

FGA_TRT_EXPORT bool initFastGpuAsrParakeetRelativeAttentionPlugin() noexcept {
    static fga_trt::ParakeetCreator runtime_creator;
    static fga_trt::ParakeetCreator builder_creator;
    return fga_trt::register_in_both_registries(runtime_creator, builder_creator);
}
