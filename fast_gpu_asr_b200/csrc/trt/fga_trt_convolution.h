// The two depthwise-convolution plugin shims share everything but their identity and C ABI
// functions: bindings x [N, T, C], valid_lengths [N] int32, weight [K, C], bias [C] ->
// output [N, T, C] of x's type; no fields; no workspace (the reference plugins'
// parakeet_convolution_plugin.cu:364-694 and zipformer_convolution_plugin.cu:513-917).
#pragma once

#include <new>

#include "../../../include/fga_convolution.h"
#include "fga_trt_common.h"

namespace fga_trt {

// Traits: kName, check / enqueue (the C ABI functions), the tactic IDs the reference
// advertised (accepted by setTactic so engines that recorded one still deserialize; the
// shim has one implementation) and the timing-cache tag.
template <class Traits>
class ConvolutionShim final : public ShimBase<ConvolutionShim<Traits>> {
  public:
    static constexpr char const* kName = Traits::kName;

    ConvolutionShim() noexcept { ok_ = this->set_timing_id(Traits::kTimingTag); }
    bool ok() const noexcept { return ok_; }

    IPluginV3* clone() noexcept override {
        auto* p = new (std::nothrow) ConvolutionShim();
        if (p == nullptr || !p->ok()) {
            delete p;
            return nullptr;
        }
        return p;
    }

    int32_t setTactic(int32_t tactic) noexcept override {
        if (tactic == 0) return 0;
        for (int32_t t : Traits::kReferenceTactics)
            if (t == tactic) return 0;
        return 1;
    }

    int32_t configurePlugin(DynamicPluginTensorDesc const* in, int32_t nbInputs,
                            DynamicPluginTensorDesc const* out, int32_t nbOutputs) noexcept override {
        if (in == nullptr || out == nullptr || nbInputs != 4 || nbOutputs != 1 || !ok_) return 1;
        const DataType t = in[0].desc.type;
        if (!is_float(t) || in[1].desc.type != DataType::kINT32 || in[2].desc.type != t ||
            in[3].desc.type != t || out[0].desc.type != t || in[0].desc.dims.nbDims != 3 ||
            in[1].desc.dims.nbDims != 1 || in[2].desc.dims.nbDims != 2 ||
            in[3].desc.dims.nbDims != 1 || out[0].desc.dims.nbDims != 3)
            return 1;
        for (int32_t i = 0; i < 4; ++i)
            if (in[i].desc.format != TensorFormat::kLINEAR) return 1;
        if (out[0].desc.format != TensorFormat::kLINEAR) return 1;
        // The contract holds at the profile's min, opt and max shapes.
        for (int which = 0; which < 3; ++which) {
            fga_tensor_desc di[4], dout[1];
            for (int32_t i = 0; i < 4; ++i)
                if (!to_desc(pick(in[i], which), in[i].desc.type, di[i])) return 1;
            if (!to_desc(pick(out[0], which), t, dout[0])) return 1;
            if (Traits::check(di, 4, dout, 1) != FGA_SUCCESS) return 1;
        }
        return 0;
    }

    int32_t getOutputDataTypes(DataType* outTypes, int32_t nbOutputs, DataType const* inTypes,
                               int32_t nbInputs) const noexcept override {
        if (outTypes == nullptr || inTypes == nullptr || nbInputs != 4 || nbOutputs != 1 ||
            !is_float(inTypes[0]) || inTypes[1] != DataType::kINT32 || inTypes[2] != inTypes[0] ||
            inTypes[3] != inTypes[0])
            return 1;
        outTypes[0] = inTypes[0];
        return 0;
    }

    // output: the shape of x.
    int32_t getOutputShapes(DimsExprs const* in, int32_t nbInputs, DimsExprs const* shapeIn,
                            int32_t nbShapeInputs, DimsExprs* out, int32_t nbOutputs,
                            IExprBuilder& builder) noexcept override {
        static_cast<void>(shapeIn);
        static_cast<void>(builder);
        if (in == nullptr || out == nullptr || nbInputs != 4 || nbOutputs != 1 ||
            nbShapeInputs != 0 || in[0].nbDims != 3 || in[0].d[0] == nullptr ||
            in[0].d[1] == nullptr || in[0].d[2] == nullptr || in[1].nbDims != 1 ||
            in[2].nbDims != 2 || in[3].nbDims != 1)
            return 1;
        out[0] = in[0];
        return 0;
    }

    bool supportsFormatCombination(int32_t pos, DynamicPluginTensorDesc const* io,
                                   int32_t nbInputs, int32_t nbOutputs) noexcept override {
        if (io == nullptr || nbInputs != 4 || nbOutputs != 1 || pos < 0 || pos > 4) return false;
        const PluginTensorDesc& d = io[pos].desc;
        if (d.format != TensorFormat::kLINEAR) return false;
        if (pos == 1) return d.type == DataType::kINT32;
        return is_float(d.type) && (pos == 0 || d.type == io[0].desc.type);
    }

    int32_t onShapeChange(PluginTensorDesc const* in, int32_t nbInputs, PluginTensorDesc const* out,
                          int32_t nbOutputs) noexcept override {
        fga_tensor_desc di[4], dout[1];
        if (in == nullptr || out == nullptr || nbInputs != 4 || nbOutputs != 1 || !ok_ ||
            !all_linear(in, 4) || !all_linear(out, 1) || !to_descs(in, di) || !to_descs(out, dout))
            return 1;
        return Traits::check(di, 4, dout, 1) == FGA_SUCCESS ? 0 : 1;
    }

    int32_t enqueue(PluginTensorDesc const* inDesc, PluginTensorDesc const* outDesc,
                    void const* const* inputs, void* const* outputs, void* workspace,
                    cudaStream_t stream) noexcept override {
        fga_tensor_desc di[4], dout[1];
        if (inDesc == nullptr || outDesc == nullptr || inputs == nullptr || outputs == nullptr ||
            !to_descs(inDesc, di) || !to_descs(outDesc, dout))
            return 1;
        return enqueue_status(Traits::enqueue(di, dout, inputs, outputs, workspace, 0, stream));
    }

    PluginFieldCollection const* getFieldsToSerialize() noexcept override { return &fields_; }

  private:
    static Dims const& pick(DynamicPluginTensorDesc const& d, int which) noexcept {
        return which == 0 ? d.min : (which == 1 ? d.opt : d.max);
    }
    bool ok_ = false;
    PluginFieldCollection fields_{0, nullptr};
};

template <class Traits>
class ConvolutionCreator final : public IPluginCreatorV3One {
  public:
    static constexpr char const* kName = Traits::kName;

    char const* getPluginName() const noexcept override { return kName; }
    char const* getPluginVersion() const noexcept override { return kVersion; }
    char const* getPluginNamespace() const noexcept override { return kPluginNamespace; }
    PluginFieldCollection const* getFieldNames() noexcept override { return &names_; }

    // No fields: a collection with any field is rejected (the reference creators' rule).
    IPluginV3* createPlugin(char const* name, PluginFieldCollection const* fc,
                            TensorRTPhase phase) noexcept override {
        static_cast<void>(name);
        static_cast<void>(phase);
        if (fc == nullptr || fc->nbFields != 0) return nullptr;
        auto* p = new (std::nothrow) ConvolutionShim<Traits>();
        if (p == nullptr || !p->ok()) {
            delete p;
            return nullptr;
        }
        return p;
    }

  private:
    PluginFieldCollection names_{0, nullptr};
};

}  // namespace fga_trt
