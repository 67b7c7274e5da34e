// TensorRT plugin `zipformer_attention_value` v1 (namespace fast_gpu_asr) over the C ABI.
//
// Drop-in for the reference's AttentionValuePlugin and its creator
// (src/fast_gpu_asr/tensorrt_plugins/zipformer_attention_value_plugin.cu:217-692): same
// name, version, namespace, `num_heads` field and its validation (kINT32, length 1, >= 1,
// no duplicates, other fields ignored), bindings, output rules and error convention. The
// computation is fga_zipformer_attention_value_enqueue; it needs no workspace.
#include <cstring>
#include <new>

#include "fga_trt_common.h"

namespace fga_trt {
namespace {

constexpr char kNumHeadsField[] = "num_heads";

class AttentionValuePlugin final : public ShimBase<AttentionValuePlugin> {
  public:
    static constexpr char kName[] = "zipformer_attention_value";

    explicit AttentionValuePlugin(int32_t heads) noexcept : heads_(heads) {
        char id[32];
        const int n = std::snprintf(id, sizeof(id), "num_heads=%d", heads);
        ok_ = heads >= 1 && n > 0 && static_cast<size_t>(n) < sizeof(id) && set_timing_id(id);
        field_ = {kNumHeadsField, &heads_, PluginFieldType::kINT32, 1};
        fields_ = {1, &field_};
    }
    bool ok() const noexcept { return ok_; }

    IPluginV3* clone() noexcept override {
        auto* p = new (std::nothrow) AttentionValuePlugin(heads_);
        if (p == nullptr || !p->ok()) {
            delete p;
            return nullptr;
        }
        return p;
    }

    // The shape relations hold on every profile bound (min, opt and max), as the
    // reference requires.
    int32_t configurePlugin(DynamicPluginTensorDesc const* in, int32_t nbInputs,
                            DynamicPluginTensorDesc const* out, int32_t nbOutputs) noexcept override {
        if (in == nullptr || out == nullptr || nbInputs != 2 || nbOutputs != 1 || !ok_) return 1;
        const DataType t = in[1].desc.type;
        if (!is_float(t) || in[0].desc.type != t || out[0].desc.type != t ||
            in[0].desc.format != TensorFormat::kLINEAR || in[1].desc.format != TensorFormat::kLINEAR ||
            out[0].desc.format != TensorFormat::kLINEAR)
            return 1;
        for (int bound = 0; bound < 3; ++bound) {
            auto pick = [bound](DynamicPluginTensorDesc const& d) -> Dims const& {
                return bound == 0 ? d.min : bound == 1 ? d.opt : d.max;
            };
            fga_tensor_desc di[2], dout[1];
            if (!to_desc(pick(in[0]), t, di[0]) || !to_desc(pick(in[1]), t, di[1]) ||
                !to_desc(pick(out[0]), t, dout[0]) ||
                fga_zipformer_attention_value_check(di, 2, dout, 1, heads_) != FGA_SUCCESS)
                return 1;
        }
        return 0;
    }

    int32_t getOutputDataTypes(DataType* outTypes, int32_t nbOutputs, DataType const* inTypes,
                               int32_t nbInputs) const noexcept override {
        if (outTypes == nullptr || inTypes == nullptr || nbInputs != 2 || nbOutputs != 1) return 1;
        outTypes[0] = inTypes[1];
        return 0;
    }

    // The output has the value tensor's shape.
    int32_t getOutputShapes(DimsExprs const* in, int32_t nbInputs, DimsExprs const* shapeIn,
                            int32_t nbShapeInputs, DimsExprs* out, int32_t nbOutputs,
                            IExprBuilder& builder) noexcept override {
        static_cast<void>(shapeIn);
        static_cast<void>(builder);
        if (in == nullptr || out == nullptr || nbInputs != 2 || nbOutputs != 1 || nbShapeInputs != 0)
            return 1;
        out[0] = in[1];
        return 0;
    }

    bool supportsFormatCombination(int32_t pos, DynamicPluginTensorDesc const* io,
                                   int32_t nbInputs, int32_t nbOutputs) noexcept override {
        if (io == nullptr || nbInputs != 2 || nbOutputs != 1 || pos < 0 || pos > 2) return false;
        const PluginTensorDesc& d = io[pos].desc;
        return d.format == TensorFormat::kLINEAR && is_float(d.type) &&
               (pos == 0 || d.type == io[0].desc.type);
    }

    size_t getWorkspaceSize(DynamicPluginTensorDesc const* in, int32_t nbInputs,
                            DynamicPluginTensorDesc const* out,
                            int32_t nbOutputs) const noexcept override {
        fga_tensor_desc d[2];
        if (in == nullptr || out == nullptr || nbInputs != 2 || nbOutputs != 1 ||
            !to_descs_max(in, d))
            return 0;
        return fga_zipformer_attention_value_workspace_size(d, 2, heads_);
    }

    int32_t onShapeChange(PluginTensorDesc const* in, int32_t nbInputs, PluginTensorDesc const* out,
                          int32_t nbOutputs) noexcept override {
        fga_tensor_desc di[2], dout[1];
        if (in == nullptr || out == nullptr || nbInputs != 2 || nbOutputs != 1 || !ok_ ||
            !all_linear(in, 2) || !all_linear(out, 1) || !to_descs(in, di) || !to_descs(out, dout))
            return 1;
        return fga_zipformer_attention_value_check(di, 2, dout, 1, heads_) == FGA_SUCCESS ? 0 : 1;
    }

    int32_t enqueue(PluginTensorDesc const* inDesc, PluginTensorDesc const* outDesc,
                    void const* const* inputs, void* const* outputs, void* workspace,
                    cudaStream_t stream) noexcept override {
        fga_tensor_desc di[2], dout[1];
        if (inDesc == nullptr || outDesc == nullptr || inputs == nullptr || outputs == nullptr ||
            !to_descs(inDesc, di) || !to_descs(outDesc, dout))
            return 1;
        const size_t ws = fga_zipformer_attention_value_workspace_size(di, 2, heads_);
        return enqueue_status(fga_zipformer_attention_value_enqueue(
            di, dout, inputs, outputs, heads_, workspace, ws, stream));
    }

    PluginFieldCollection const* getFieldsToSerialize() noexcept override { return &fields_; }

  private:
    int32_t heads_;
    bool ok_ = false;
    PluginField field_{};
    PluginFieldCollection fields_{};
};

class AttentionValueCreator final : public IPluginCreatorV3One {
  public:
    static constexpr char const* kName = AttentionValuePlugin::kName;

    AttentionValueCreator() noexcept {
        attribute_ = {kNumHeadsField, nullptr, PluginFieldType::kINT32, 1};
        names_ = {1, &attribute_};
    }
    char const* getPluginName() const noexcept override { return kName; }
    char const* getPluginVersion() const noexcept override { return kVersion; }
    char const* getPluginNamespace() const noexcept override { return kPluginNamespace; }
    PluginFieldCollection const* getFieldNames() noexcept override { return &names_; }

    IPluginV3* createPlugin(char const* name, PluginFieldCollection const* fc,
                            TensorRTPhase phase) noexcept override {
        static_cast<void>(name);
        static_cast<void>(phase);
        if (fc == nullptr || fc->nbFields < 0 || (fc->nbFields > 0 && fc->fields == nullptr))
            return nullptr;
        int32_t heads = 0;
        bool found = false;
        for (int32_t i = 0; i < fc->nbFields; ++i) {
            const PluginField& f = fc->fields[i];
            if (f.name == nullptr || std::strcmp(f.name, kNumHeadsField) != 0) continue;
            if (found || f.type != PluginFieldType::kINT32 || f.length != 1 || f.data == nullptr)
                return nullptr;  // malformed or duplicate
            heads = *static_cast<int32_t const*>(f.data);
            found = true;
        }
        if (!found || heads < 1) return nullptr;
        auto* p = new (std::nothrow) AttentionValuePlugin(heads);
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

FGA_TRT_EXPORT bool initFastGpuAsrZipformerAttentionValuePlugin() noexcept {
    static fga_trt::AttentionValueCreator runtime_creator;
    static fga_trt::AttentionValueCreator builder_creator;
    return fga_trt::register_in_both_registries(runtime_creator, builder_creator);
}
