// Minimal stand-in for TensorRT's NvInfer.h: only the declarations the plugin shims in
// fast_gpu_asr_b200/csrc/trt/ use (IPluginV3 with its OneCore/OneBuild/OneRuntime
// capabilities, IPluginCreatorV3One, the plugin registries), with TensorRT's names and
// signatures, so the shims compile and their contracts can be exercised on a machine
// without TensorRT. TEST INFRASTRUCTURE ONLY: never used to build the product.
//
// The registries are declared here and defined by the test harness.
#pragma once

#include <cuda_runtime_api.h>

#include <cstddef>
#include <cstdint>

#define FGA_TENSORRT_STUB 1

namespace nvinfer1 {

using AsciiChar = char;

enum class DataType : int32_t {
    kFLOAT = 0, kHALF = 1, kINT8 = 2, kINT32 = 3, kBOOL = 4, kUINT8 = 5, kFP8 = 6,
    kBF16 = 7, kINT64 = 8, kINT4 = 9, kFP4 = 10, kE8M0 = 11,
};

enum class TensorFormat : int32_t { kLINEAR = 0, kCHW2 = 1, kHWC8 = 2, kCHW4 = 3 };

class Dims64 {
  public:
    static constexpr int32_t MAX_DIMS{8};
    int32_t nbDims{0};
    int64_t d[MAX_DIMS]{};
};
using Dims = Dims64;

struct PluginTensorDesc {
    Dims dims;
    DataType type{DataType::kFLOAT};
    TensorFormat format{TensorFormat::kLINEAR};
    float scale{1.0F};
};

struct DynamicPluginTensorDesc {
    PluginTensorDesc desc;
    Dims min;
    Dims max;
    Dims opt;
};

class IDimensionExpr {
  public:
    virtual ~IDimensionExpr() = default;
};

class IExprBuilder {
  public:
    virtual ~IExprBuilder() = default;
};

class DimsExprs {
  public:
    int32_t nbDims{0};
    IDimensionExpr const* d[Dims::MAX_DIMS]{};
};

enum class PluginFieldType : int32_t {
    kFLOAT16 = 0, kFLOAT32 = 1, kFLOAT64 = 2, kINT8 = 3, kINT16 = 4, kINT32 = 5, kCHAR = 6,
    kDIMS = 7, kUNKNOWN = 8, kBF16 = 9, kINT64 = 10, kFP8 = 11, kINT4 = 12, kFP4 = 13,
};

class PluginField {
  public:
    AsciiChar const* name{nullptr};
    void const* data{nullptr};
    PluginFieldType type{PluginFieldType::kUNKNOWN};
    int32_t length{0};
};

struct PluginFieldCollection {
    int32_t nbFields{0};
    PluginField const* fields{nullptr};
};

enum class PluginCapabilityType : int32_t { kCORE = 0, kBUILD = 1, kRUNTIME = 2 };
enum class TensorRTPhase : int32_t { kBUILD = 0, kRUNTIME = 1 };
enum class EngineCapability : int32_t { kSTANDARD = 0, kSAFETY = 1, kDLA_STANDALONE = 2 };

class IPluginResourceContext {
  public:
    virtual ~IPluginResourceContext() = default;
};

class IPluginCapability {
  public:
    virtual ~IPluginCapability() = default;
};

class IPluginV3 {
  public:
    virtual ~IPluginV3() = default;
    virtual IPluginCapability* getCapabilityInterface(PluginCapabilityType type) noexcept = 0;
    virtual IPluginV3* clone() noexcept = 0;
};

class IPluginV3OneCore : public IPluginCapability {
  public:
    virtual AsciiChar const* getPluginName() const noexcept = 0;
    virtual AsciiChar const* getPluginVersion() const noexcept = 0;
    virtual AsciiChar const* getPluginNamespace() const noexcept = 0;
};

class IPluginV3OneBuild : public IPluginCapability {
  public:
    virtual int32_t configurePlugin(DynamicPluginTensorDesc const* in, int32_t nbInputs,
                                    DynamicPluginTensorDesc const* out, int32_t nbOutputs) noexcept = 0;
    virtual int32_t getOutputDataTypes(DataType* outputTypes, int32_t nbOutputs,
                                       DataType const* inputTypes, int32_t nbInputs) const noexcept = 0;
    virtual int32_t getOutputShapes(DimsExprs const* inputs, int32_t nbInputs,
                                    DimsExprs const* shapeInputs, int32_t nbShapeInputs,
                                    DimsExprs* outputs, int32_t nbOutputs,
                                    IExprBuilder& exprBuilder) noexcept = 0;
    virtual bool supportsFormatCombination(int32_t pos, DynamicPluginTensorDesc const* inOut,
                                           int32_t nbInputs, int32_t nbOutputs) noexcept = 0;
    virtual int32_t getNbOutputs() const noexcept = 0;
    virtual size_t getWorkspaceSize(DynamicPluginTensorDesc const* /*inputs*/, int32_t /*nbInputs*/,
                                    DynamicPluginTensorDesc const* /*outputs*/,
                                    int32_t /*nbOutputs*/) const noexcept { return 0; }
    virtual int32_t getValidTactics(int32_t* /*tactics*/, int32_t /*nbTactics*/) noexcept { return 0; }
    virtual int32_t getNbTactics() noexcept { return 0; }
    virtual char const* getTimingCacheID() noexcept { return nullptr; }
    virtual int32_t getFormatCombinationLimit() noexcept { return 100; }
    virtual char const* getMetadataString() noexcept { return nullptr; }
};

class IPluginV3OneRuntime : public IPluginCapability {
  public:
    virtual int32_t setTactic(int32_t /*tactic*/) noexcept { return 0; }
    virtual int32_t onShapeChange(PluginTensorDesc const* in, int32_t nbInputs,
                                  PluginTensorDesc const* out, int32_t nbOutputs) noexcept = 0;
    virtual int32_t enqueue(PluginTensorDesc const* inputDesc, PluginTensorDesc const* outputDesc,
                            void const* const* inputs, void* const* outputs, void* workspace,
                            cudaStream_t stream) noexcept = 0;
    virtual IPluginV3* attachToContext(IPluginResourceContext* context) noexcept = 0;
    virtual PluginFieldCollection const* getFieldsToSerialize() noexcept = 0;
};

class IPluginCreatorInterface {
  public:
    virtual ~IPluginCreatorInterface() = default;
};

class IPluginCreatorV3One : public IPluginCreatorInterface {
  public:
    virtual IPluginV3* createPlugin(AsciiChar const* name, PluginFieldCollection const* fc,
                                    TensorRTPhase phase) noexcept = 0;
    virtual PluginFieldCollection const* getFieldNames() noexcept = 0;
    virtual AsciiChar const* getPluginName() const noexcept = 0;
    virtual AsciiChar const* getPluginVersion() const noexcept = 0;
    virtual AsciiChar const* getPluginNamespace() const noexcept = 0;
};

class IPluginRegistry {
  public:
    virtual ~IPluginRegistry() = default;
    virtual bool registerCreator(IPluginCreatorInterface& creator,
                                 AsciiChar const* pluginNamespace) noexcept = 0;
    virtual IPluginCreatorInterface* getCreator(AsciiChar const* pluginName,
                                                AsciiChar const* pluginVersion,
                                                AsciiChar const* pluginNamespace = "") noexcept = 0;
};

extern "C" IPluginRegistry* getBuilderPluginRegistry(EngineCapability capability) noexcept;

}  // namespace nvinfer1

extern "C" nvinfer1::IPluginRegistry* getPluginRegistry() noexcept;
