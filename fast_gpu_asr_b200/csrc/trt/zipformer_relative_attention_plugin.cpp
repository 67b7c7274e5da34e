// TensorRT plugin `zipformer_relative_attention` v1 (namespace fast_gpu_asr) over the C ABI.
//
// Drop-in for the reference's RelativeAttentionPlugin and its creator
// (src/fast_gpu_asr/tensorrt_plugins/zipformer_relative_attention_plugin.cu:573-901): same
// name, version, namespace, no fields, bindings, output rules and error convention. The
// computation is fga_zipformer_relative_attention_enqueue; its workspace
// (FGA_SCHED_WORKSPACE_BYTES, the kernel's work counter) replaces the reference's 16 MB
// cuBLAS workspace, and TensorRT gives each execution context its own.
#include <new>

#include "fga_trt_common.h"

namespace fga_trt {
namespace {

class ZipformerWeightsPlugin final : public ShimBase<ZipformerWeightsPlugin> {
  public:
    static constexpr char kName[] = "zipformer_relative_attention";

    ZipformerWeightsPlugin() noexcept {
        ok_ = set_timing_id("layout=ntc;position_head_dim=4;padded_query_halo=7");
    }
    bool ok() const noexcept { return ok_; }

    IPluginV3* clone() noexcept override {
        auto* p = new (std::nothrow) ZipformerWeightsPlugin();
        if (p == nullptr || !p->ok()) {
            delete p;
            return nullptr;
        }
        return p;
    }

    int32_t configurePlugin(DynamicPluginTensorDesc const* in, int32_t nbInputs,
                            DynamicPluginTensorDesc const* out, int32_t nbOutputs) noexcept override {
        if (in == nullptr || out == nullptr || nbInputs != 3 || nbOutputs != 1 || !ok_) return 1;
        const DataType t = in[0].desc.type;
        if (!is_float(t) || in[1].desc.type != t || in[2].desc.type != DataType::kBOOL ||
            out[0].desc.type != t || in[0].desc.dims.nbDims != 3 || in[1].desc.dims.nbDims != 4 ||
            in[2].desc.dims.nbDims != 2 || out[0].desc.dims.nbDims != 4)
            return 1;
        for (int32_t i = 0; i < 3; ++i)
            if (in[i].desc.format != TensorFormat::kLINEAR ||
                !addressable(in[i].max, element_bytes(in[i].desc.type)))
                return 1;
        if (out[0].desc.format != TensorFormat::kLINEAR || !addressable(out[0].max, element_bytes(t)))
            return 1;
        return 0;
    }

    int32_t getOutputDataTypes(DataType* outTypes, int32_t nbOutputs, DataType const* inTypes,
                               int32_t nbInputs) const noexcept override {
        if (outTypes == nullptr || inTypes == nullptr || nbInputs != 3 || nbOutputs != 1 ||
            !is_float(inTypes[0]) || inTypes[1] != inTypes[0] || inTypes[2] != DataType::kBOOL)
            return 1;
        outTypes[0] = inTypes[0];
        return 0;
    }

    // weights [N, H, T, T]: N and T of the projection, H of the positional table.
    int32_t getOutputShapes(DimsExprs const* in, int32_t nbInputs, DimsExprs const* shapeIn,
                            int32_t nbShapeInputs, DimsExprs* out, int32_t nbOutputs,
                            IExprBuilder& builder) noexcept override {
        static_cast<void>(shapeIn);
        static_cast<void>(builder);
        if (in == nullptr || out == nullptr || nbInputs != 3 || nbOutputs != 1 ||
            nbShapeInputs != 0 || in[0].nbDims != 3 || in[1].nbDims != 4 || in[2].nbDims != 2 ||
            in[0].d[0] == nullptr || in[0].d[1] == nullptr || in[1].d[2] == nullptr)
            return 1;
        out[0].nbDims = 4;
        out[0].d[0] = in[0].d[0];
        out[0].d[1] = in[1].d[2];
        out[0].d[2] = in[0].d[1];
        out[0].d[3] = in[0].d[1];
        return 0;
    }

    bool supportsFormatCombination(int32_t pos, DynamicPluginTensorDesc const* io,
                                   int32_t nbInputs, int32_t nbOutputs) noexcept override {
        if (io == nullptr || nbInputs != 3 || nbOutputs != 1 || pos < 0 || pos > 3) return false;
        const PluginTensorDesc& d = io[pos].desc;
        if (d.format != TensorFormat::kLINEAR) return false;
        if (pos == 2) return d.type == DataType::kBOOL;
        return is_float(d.type) && (pos == 0 || d.type == io[0].desc.type);
    }

    size_t getWorkspaceSize(DynamicPluginTensorDesc const* in, int32_t nbInputs,
                            DynamicPluginTensorDesc const* out,
                            int32_t nbOutputs) const noexcept override {
        fga_tensor_desc d[3];
        if (in == nullptr || out == nullptr || nbInputs != 3 || nbOutputs != 1 ||
            !to_descs_max(in, d))
            return 0;
        return fga_zipformer_relative_attention_workspace_size(d, 3);
    }

    int32_t onShapeChange(PluginTensorDesc const* in, int32_t nbInputs, PluginTensorDesc const* out,
                          int32_t nbOutputs) noexcept override {
        fga_tensor_desc di[3], dout[1];
        if (in == nullptr || out == nullptr || nbInputs != 3 || nbOutputs != 1 || !ok_ ||
            !all_linear(in, 3) || !all_linear(out, 1) || !to_descs(in, di) || !to_descs(out, dout))
            return 1;
        return fga_zipformer_relative_attention_check(di, 3, dout, 1) == FGA_SUCCESS ? 0 : 1;
    }

    int32_t enqueue(PluginTensorDesc const* inDesc, PluginTensorDesc const* outDesc,
                    void const* const* inputs, void* const* outputs, void* workspace,
                    cudaStream_t stream) noexcept override {
        fga_tensor_desc di[3], dout[1];
        if (inDesc == nullptr || outDesc == nullptr || inputs == nullptr || outputs == nullptr ||
            !to_descs(inDesc, di) || !to_descs(outDesc, dout))
            return 1;
        const size_t ws = fga_zipformer_relative_attention_workspace_size(di, 3);
        return enqueue_status(fga_zipformer_relative_attention_enqueue(
            di, dout, inputs, outputs, workspace, ws, stream));
    }

    PluginFieldCollection const* getFieldsToSerialize() noexcept override { return &fields_; }

  private:
    bool ok_ = false;
    PluginFieldCollection fields_{0, nullptr};
};

class ZipformerWeightsCreator final : public IPluginCreatorV3One {
  public:
    static constexpr char const* kName = ZipformerWeightsPlugin::kName;

    char const* getPluginName() const noexcept override { return kName; }
    char const* getPluginVersion() const noexcept override { return kVersion; }
    char const* getPluginNamespace() const noexcept override { return kPluginNamespace; }
    PluginFieldCollection const* getFieldNames() noexcept override { return &names_; }

    // The plugin has no fields: a collection with any field is rejected (the reference
    // creator's rule, zipformer_relative_attention_plugin.cu:855).
    IPluginV3* createPlugin(char const* name, PluginFieldCollection const* fc,
                            TensorRTPhase phase) noexcept override {
        static_cast<void>(name);
        static_cast<void>(phase);
        if (fc == nullptr || fc->nbFields != 0) return nullptr;
        auto* p = new (std::nothrow) ZipformerWeightsPlugin();
        if (p == nullptr || !p->ok()) {
            delete p;
            return nullptr;
        }
        return p;
    }

  private:
    PluginFieldCollection names_{0, nullptr};
};

}  // namespace
}  // namespace fga_trt

FGA_TRT_EXPORT bool initFastGpuAsrZipformerRelativeAttentionPlugin() noexcept {
    static fga_trt::ZipformerWeightsCreator runtime_creator;
    static fga_trt::ZipformerWeightsCreator builder_creator;
    return fga_trt::register_in_both_registries(runtime_creator, builder_creator);
}
