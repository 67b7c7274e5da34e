// Contract tests of the TensorRT plugin shims, compiled on a machine without TensorRT or a
// GPU: the shims are built against the stub NvInfer.h beside this file, the plugin
// registries are in-memory fakes, and the C ABI is a fake that records what each shim
// forwards. TEST INFRASTRUCTURE ONLY.
//
// Checked for each of the five plugins: registration in both registries and idempotent
// re-initialisation; the creator's field validation; identity (name, version "1",
// namespace "fast_gpu_asr"), capabilities, output types, shapes and formats; that
// onShapeChange and enqueue hand TensorRT's descriptors, pointers, field values,
// workspace and stream to the C ABI unchanged and map its status to 0/1; clone,
// attachToContext and the serialised fields.
#include <NvInfer.h>

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <limits>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "../../include/fga_attention.h"
#include "../../include/fga_convolution.h"

using namespace nvinfer1;

extern "C" bool initFastGpuAsrParakeetRelativeAttentionPlugin() noexcept;
extern "C" bool initFastGpuAsrZipformerRelativeAttentionPlugin() noexcept;
extern "C" bool initFastGpuAsrZipformerAttentionValuePlugin() noexcept;
extern "C" bool initFastGpuAsrParakeetConvolutionPlugin() noexcept;
extern "C" bool initFastGpuAsrZipformerConvolutionPlugin() noexcept;

static int g_failures = 0;
#define CHECK(cond)                                                                   \
    do {                                                                              \
        if (!(cond)) {                                                                \
            std::fprintf(stderr, "%s:%d: CHECK failed: %s\n", __FILE__, __LINE__, #cond); \
            ++g_failures;                                                             \
        }                                                                             \
    } while (0)

// ---- in-memory plugin registries -------------------------------------------------------
class FakeRegistry final : public IPluginRegistry {
  public:
    bool registerCreator(IPluginCreatorInterface& creator, char const* ns) noexcept override {
        auto* c = dynamic_cast<IPluginCreatorV3One*>(&creator);
        if (c == nullptr || ns == nullptr) return false;
        const std::string key = std::string(c->getPluginName()) + "/" + c->getPluginVersion() + "/" + ns;
        ++registrations;
        if (creators.count(key) != 0) return false;
        creators[key] = c;
        return true;
    }
    IPluginCreatorInterface* getCreator(char const* name, char const* version,
                                        char const* ns) noexcept override {
        auto it = creators.find(std::string(name) + "/" + version + "/" + ns);
        return it == creators.end() ? nullptr : it->second;
    }
    std::map<std::string, IPluginCreatorV3One*> creators;
    int registrations = 0;
};

static FakeRegistry g_runtime, g_builder;
extern "C" IPluginRegistry* getPluginRegistry() noexcept { return &g_runtime; }
namespace nvinfer1 {
extern "C" IPluginRegistry* getBuilderPluginRegistry(EngineCapability c) noexcept {
    return c == EngineCapability::kSTANDARD ? &g_builder : nullptr;
}
}  // namespace nvinfer1

// ---- fake C ABI: records the last call ------------------------------------------------
struct Call {
    std::string fn;
    fga_tensor_desc in[8];
    fga_tensor_desc out[4];
    int32_t nin = 0, nout = 0;
    const void* const* inputs = nullptr;
    void* const* outputs = nullptr;
    float scale = 0;
    int32_t heads = 0;
    void* workspace = nullptr;
    size_t workspace_bytes = 0;
    void* stream = nullptr;
};
static Call g_last;
static int32_t g_status = FGA_SUCCESS;  // what the fake returns
static size_t g_workspace = 0;          // what the fake's *_workspace_size returns

static void record(const char* fn, const fga_tensor_desc* in, int32_t nin, const fga_tensor_desc* out,
                   int32_t nout) {
    g_last = Call{};
    g_last.fn = fn;
    g_last.nin = nin;
    g_last.nout = nout;
    for (int i = 0; i < nin && i < 8; ++i) g_last.in[i] = in[i];
    for (int i = 0; i < nout && i < 4; ++i) g_last.out[i] = out[i];
}

extern "C" {
int32_t fga_parakeet_relative_attention_check(const fga_tensor_desc* in, int32_t nin,
                                              const fga_tensor_desc* out, int32_t nout, float scale) {
    record("parakeet_check", in, nin, out, nout);
    g_last.scale = scale;
    return g_status;
}
size_t fga_parakeet_relative_attention_workspace_size(const fga_tensor_desc* in, int32_t nin) {
    record("parakeet_workspace", in, nin, nullptr, 0);
    return g_workspace;
}
int32_t fga_parakeet_relative_attention_enqueue(const fga_tensor_desc* in, const fga_tensor_desc* out,
                                                const void* const* inputs, void* const* outputs,
                                                float scale, void* ws, size_t wsb, void* stream) {
    record("parakeet_enqueue", in, 5, out, 1);
    g_last.inputs = inputs;
    g_last.outputs = outputs;
    g_last.scale = scale;
    g_last.workspace = ws;
    g_last.workspace_bytes = wsb;
    g_last.stream = stream;
    return g_status;
}
int32_t fga_zipformer_relative_attention_check(const fga_tensor_desc* in, int32_t nin,
                                               const fga_tensor_desc* out, int32_t nout) {
    record("weights_check", in, nin, out, nout);
    return g_status;
}
size_t fga_zipformer_relative_attention_workspace_size(const fga_tensor_desc* in, int32_t nin) {
    record("weights_workspace", in, nin, nullptr, 0);
    return g_workspace;
}
int32_t fga_zipformer_relative_attention_enqueue(const fga_tensor_desc* in, const fga_tensor_desc* out,
                                                 const void* const* inputs, void* const* outputs,
                                                 void* ws, size_t wsb, void* stream) {
    record("weights_enqueue", in, 3, out, 1);
    g_last.inputs = inputs;
    g_last.outputs = outputs;
    g_last.workspace = ws;
    g_last.workspace_bytes = wsb;
    g_last.stream = stream;
    return g_status;
}
int32_t fga_zipformer_attention_value_check(const fga_tensor_desc* in, int32_t nin,
                                            const fga_tensor_desc* out, int32_t nout, int32_t heads) {
    record("value_check", in, nin, out, nout);
    g_last.heads = heads;
    return g_status;
}
size_t fga_zipformer_attention_value_workspace_size(const fga_tensor_desc* in, int32_t nin,
                                                    int32_t heads) {
    record("value_workspace", in, nin, nullptr, 0);
    g_last.heads = heads;
    return g_workspace;
}
int32_t fga_zipformer_attention_value_enqueue(const fga_tensor_desc* in, const fga_tensor_desc* out,
                                              const void* const* inputs, void* const* outputs,
                                              int32_t heads, void* ws, size_t wsb, void* stream) {
    record("value_enqueue", in, 2, out, 1);
    g_last.inputs = inputs;
    g_last.outputs = outputs;
    g_last.heads = heads;
    g_last.workspace = ws;
    g_last.workspace_bytes = wsb;
    g_last.stream = stream;
    return g_status;
}
int32_t fga_parakeet_conformer_convolution_check(const fga_tensor_desc* in, int32_t nin,
                                                 const fga_tensor_desc* out, int32_t nout) {
    record("pconv_check", in, nin, out, nout);
    return g_status;
}
size_t fga_parakeet_conformer_convolution_workspace_size(const fga_tensor_desc* in, int32_t nin) {
    record("pconv_workspace", in, nin, nullptr, 0);
    return 0;
}
int32_t fga_parakeet_conformer_convolution_enqueue(const fga_tensor_desc* in,
                                                   const fga_tensor_desc* out,
                                                   const void* const* inputs, void* const* outputs,
                                                   void* ws, size_t wsb, void* stream) {
    record("pconv_enqueue", in, 4, out, 1);
    g_last.inputs = inputs;
    g_last.outputs = outputs;
    g_last.workspace = ws;
    g_last.workspace_bytes = wsb;
    g_last.stream = stream;
    return g_status;
}
int32_t fga_zipformer_convolution_check(const fga_tensor_desc* in, int32_t nin,
                                        const fga_tensor_desc* out, int32_t nout) {
    record("zconv_check", in, nin, out, nout);
    return g_status;
}
size_t fga_zipformer_convolution_workspace_size(const fga_tensor_desc* in, int32_t nin) {
    record("zconv_workspace", in, nin, nullptr, 0);
    return 0;
}
int32_t fga_zipformer_convolution_enqueue(const fga_tensor_desc* in, const fga_tensor_desc* out,
                                          const void* const* inputs, void* const* outputs,
                                          void* ws, size_t wsb, void* stream) {
    record("zconv_enqueue", in, 4, out, 1);
    g_last.inputs = inputs;
    g_last.outputs = outputs;
    g_last.workspace = ws;
    g_last.workspace_bytes = wsb;
    g_last.stream = stream;
    return g_status;
}
}  // extern "C"

// ---- helpers ----------------------------------------------------------------------------
static Dims dims(std::initializer_list<int64_t> d) {
    Dims r;
    r.nbDims = static_cast<int32_t>(d.size());
    int i = 0;
    for (int64_t v : d) r.d[i++] = v;
    return r;
}
static PluginTensorDesc desc(DataType t, std::initializer_list<int64_t> d) {
    PluginTensorDesc p;
    p.dims = dims(d);
    p.type = t;
    p.format = TensorFormat::kLINEAR;
    return p;
}
static DynamicPluginTensorDesc dyn(PluginTensorDesc p) {
    DynamicPluginTensorDesc d;
    d.desc = p;
    d.min = d.opt = d.max = p.dims;
    return d;
}
static bool same(const fga_tensor_desc& f, const PluginTensorDesc& p) {
    if (f.type != static_cast<int32_t>(p.type) || f.nb_dims != p.dims.nbDims) return false;
    for (int i = 0; i < p.dims.nbDims; ++i)
        if (f.dims[i] != p.dims.d[i]) return false;
    return true;
}
static IPluginCreatorV3One* creator(FakeRegistry& r, const char* name) {
    return static_cast<IPluginCreatorV3One*>(r.getCreator(name, "1", "fast_gpu_asr"));
}
template <class I>
static I* cap(IPluginV3* p, PluginCapabilityType t) {
    return dynamic_cast<I*>(p->getCapabilityInterface(t));
}
static PluginFieldCollection fields(const PluginField* f, int32_t n) { return {n, f}; }

// ---- tests --------------------------------------------------------------------------------
static void test_registration() {
    CHECK(initFastGpuAsrParakeetRelativeAttentionPlugin());
    CHECK(initFastGpuAsrZipformerRelativeAttentionPlugin());
    CHECK(initFastGpuAsrZipformerAttentionValuePlugin());
    CHECK(initFastGpuAsrParakeetConvolutionPlugin());
    CHECK(initFastGpuAsrZipformerConvolutionPlugin());
    for (FakeRegistry* r : {&g_runtime, &g_builder}) {
        CHECK(r->creators.size() == 5);
        CHECK(creator(*r, "parakeet_conformer_convolution") != nullptr);
        CHECK(creator(*r, "zipformer_convolution") != nullptr);
        CHECK(creator(*r, "parakeet_relative_attention") != nullptr);
        CHECK(creator(*r, "zipformer_relative_attention") != nullptr);
        CHECK(creator(*r, "zipformer_attention_value") != nullptr);
        CHECK(r->getCreator("parakeet_relative_attention", "2", "fast_gpu_asr") == nullptr);
        CHECK(r->getCreator("parakeet_relative_attention", "1", "") == nullptr);
    }
    // The runtime and builder registries hold distinct creator objects.
    CHECK(creator(g_runtime, "parakeet_relative_attention") !=
          creator(g_builder, "parakeet_relative_attention"));
    const int before = g_runtime.registrations + g_builder.registrations;
    CHECK(initFastGpuAsrParakeetRelativeAttentionPlugin());  // idempotent: no re-registration
    CHECK(initFastGpuAsrZipformerRelativeAttentionPlugin());
    CHECK(initFastGpuAsrZipformerAttentionValuePlugin());
    CHECK(initFastGpuAsrParakeetConvolutionPlugin());
    CHECK(initFastGpuAsrZipformerConvolutionPlugin());
    CHECK(g_runtime.registrations + g_builder.registrations == before);
    for (auto* r : {&g_runtime, &g_builder})
        for (auto& kv : r->creators) {
            CHECK(std::strcmp(kv.second->getPluginVersion(), "1") == 0);
            CHECK(std::strcmp(kv.second->getPluginNamespace(), "fast_gpu_asr") == 0);
        }
}

static std::unique_ptr<IPluginV3> make_parakeet(float scale) {
    PluginField f{"scale", &scale, PluginFieldType::kFLOAT32, 1};
    auto fc = fields(&f, 1);
    return std::unique_ptr<IPluginV3>(
        creator(g_runtime, "parakeet_relative_attention")->createPlugin("p", &fc, TensorRTPhase::kBUILD));
}

static void test_parakeet_fields() {
    auto* c = creator(g_runtime, "parakeet_relative_attention");
    const PluginFieldCollection* names = c->getFieldNames();
    CHECK(names->nbFields == 1 && std::strcmp(names->fields[0].name, "scale") == 0 &&
          names->fields[0].type == PluginFieldType::kFLOAT32);
    CHECK(make_parakeet(0.125F) != nullptr);
    for (float bad : {0.0F, -0.5F, std::numeric_limits<float>::infinity(),
                      std::numeric_limits<float>::quiet_NaN(), 3.0e38F})
        CHECK(make_parakeet(bad) == nullptr);
    float s = 0.125F;
    int32_t i = 1;
    PluginField wrong_type{"scale", &i, PluginFieldType::kINT32, 1};
    PluginField wrong_len{"scale", &s, PluginFieldType::kFLOAT32, 2};
    PluginField wrong_name{"scal", &s, PluginFieldType::kFLOAT32, 1};
    PluginField null_data{"scale", nullptr, PluginFieldType::kFLOAT32, 1};
    for (PluginField* f : {&wrong_type, &wrong_len, &wrong_name, &null_data}) {
        auto fc = fields(f, 1);
        CHECK(c->createPlugin("p", &fc, TensorRTPhase::kBUILD) == nullptr);
    }
    PluginField two[2] = {{"scale", &s, PluginFieldType::kFLOAT32, 1},
                          {"extra", &s, PluginFieldType::kFLOAT32, 1}};
    auto fc2 = fields(two, 2);
    CHECK(c->createPlugin("p", &fc2, TensorRTPhase::kBUILD) == nullptr);
    auto fc0 = fields(nullptr, 0);
    CHECK(c->createPlugin("p", &fc0, TensorRTPhase::kBUILD) == nullptr);
    CHECK(c->createPlugin("p", nullptr, TensorRTPhase::kBUILD) == nullptr);
}

static void test_parakeet_plugin() {
    auto p = make_parakeet(0.088388F);
    CHECK(p != nullptr);
    auto* core = cap<IPluginV3OneCore>(p.get(), PluginCapabilityType::kCORE);
    auto* build = cap<IPluginV3OneBuild>(p.get(), PluginCapabilityType::kBUILD);
    auto* rt = cap<IPluginV3OneRuntime>(p.get(), PluginCapabilityType::kRUNTIME);
    CHECK(core && build && rt);
    CHECK(std::strcmp(core->getPluginName(), "parakeet_relative_attention") == 0);
    CHECK(std::strcmp(core->getPluginVersion(), "1") == 0);
    CHECK(std::strcmp(core->getPluginNamespace(), "fast_gpu_asr") == 0);
    CHECK(build->getNbOutputs() == 1);
    const std::string id = build->getTimingCacheID();
    CHECK(id.find("impl=fga-sm100a") != std::string::npos);
    CHECK(id.find("scale=0x1.") != std::string::npos);
    CHECK(std::string(cap<IPluginV3OneBuild>(make_parakeet(0.25F).get(),
                                             PluginCapabilityType::kBUILD)->getTimingCacheID()) != id);
    CHECK(build->getNbTactics() == 0 && rt->setTactic(0) == 0 && rt->setTactic(1) != 0);

    DataType ins[5] = {DataType::kHALF, DataType::kHALF, DataType::kHALF, DataType::kHALF,
                       DataType::kINT32};
    DataType out;
    CHECK(build->getOutputDataTypes(&out, 1, ins, 5) == 0 && out == DataType::kHALF);
    ins[2] = DataType::kBF16;
    CHECK(build->getOutputDataTypes(&out, 1, ins, 5) != 0);

    // N, T from qkv, C from the positional table.
    IDimensionExpr n, t, c3, one, rel, c, h, d, len;
    DimsExprs ein[5];
    ein[0].nbDims = 3; ein[0].d[0] = &n; ein[0].d[1] = &t; ein[0].d[2] = &c3;
    ein[1].nbDims = 3; ein[1].d[0] = &one; ein[1].d[1] = &rel; ein[1].d[2] = &c;
    ein[2].nbDims = 2; ein[2].d[0] = &h; ein[2].d[1] = &d;
    ein[3] = ein[2];
    ein[4].nbDims = 1; ein[4].d[0] = &len;
    DimsExprs eout[1];
    IExprBuilder eb;
    CHECK(build->getOutputShapes(ein, 5, nullptr, 0, eout, 1, eb) == 0);
    CHECK(eout[0].nbDims == 3 && eout[0].d[0] == &n && eout[0].d[1] == &t && eout[0].d[2] == &c);

    PluginTensorDesc pin[5] = {desc(DataType::kHALF, {2, 375, 3072}), desc(DataType::kHALF, {1, 749, 1024}),
                               desc(DataType::kHALF, {8, 128}), desc(DataType::kHALF, {8, 128}),
                               desc(DataType::kINT32, {2})};
    PluginTensorDesc pout[1] = {desc(DataType::kHALF, {2, 375, 1024})};
    DynamicPluginTensorDesc din[5], dout[1];
    for (int i = 0; i < 5; ++i) din[i] = dyn(pin[i]);
    dout[0] = dyn(pout[0]);
    CHECK(build->configurePlugin(din, 5, dout, 1) == 0);
    din[4].desc.type = DataType::kFLOAT;
    CHECK(build->configurePlugin(din, 5, dout, 1) != 0);
    din[4].desc.type = DataType::kINT32;
    din[1].desc.format = TensorFormat::kCHW2;
    CHECK(build->configurePlugin(din, 5, dout, 1) != 0);
    din[1].desc.format = TensorFormat::kLINEAR;

    DynamicPluginTensorDesc io[6];
    for (int i = 0; i < 5; ++i) io[i] = din[i];
    io[5] = dout[0];
    CHECK(build->supportsFormatCombination(0, io, 5, 1));
    CHECK(build->supportsFormatCombination(4, io, 5, 1));
    io[5].desc.type = DataType::kBF16;
    CHECK(!build->supportsFormatCombination(5, io, 5, 1));
    io[5].desc.type = DataType::kHALF;
    io[3].desc.format = TensorFormat::kHWC8;
    CHECK(!build->supportsFormatCombination(3, io, 5, 1));

    g_workspace = 0;
    CHECK(build->getWorkspaceSize(din, 5, dout, 1) == 0);
    CHECK(g_last.fn == "parakeet_workspace" && same(g_last.in[0], pin[0]));

    g_status = FGA_SUCCESS;
    CHECK(rt->onShapeChange(pin, 5, pout, 1) == 0);
    CHECK(g_last.fn == "parakeet_check" && g_last.nin == 5 && g_last.nout == 1);
    for (int i = 0; i < 5; ++i) CHECK(same(g_last.in[i], pin[i]));
    CHECK(same(g_last.out[0], pout[0]) && g_last.scale == 0.088388F);
    g_status = FGA_ERROR_BAD_SHAPE;
    CHECK(rt->onShapeChange(pin, 5, pout, 1) == 1);

    const void* inputs[5] = {reinterpret_cast<void*>(0x100), reinterpret_cast<void*>(0x200),
                             reinterpret_cast<void*>(0x300), reinterpret_cast<void*>(0x400),
                             reinterpret_cast<void*>(0x500)};
    void* outputs[1] = {reinterpret_cast<void*>(0x600)};
    void* ws = reinterpret_cast<void*>(0x700);
    cudaStream_t stream = reinterpret_cast<cudaStream_t>(0x800);
    g_status = FGA_SUCCESS;
    CHECK(rt->enqueue(pin, pout, inputs, outputs, ws, stream) == 0);
    CHECK(g_last.fn == "parakeet_enqueue" && g_last.inputs == inputs && g_last.outputs == outputs);
    CHECK(g_last.workspace == ws && g_last.stream == stream && g_last.scale == 0.088388F);
    for (int i = 0; i < 5; ++i) CHECK(same(g_last.in[i], pin[i]));
    g_status = FGA_ERROR_LAUNCH;
    CHECK(rt->enqueue(pin, pout, inputs, outputs, ws, stream) == 1);
    g_status = FGA_SUCCESS;

    std::unique_ptr<IPluginV3> copy(rt->attachToContext(nullptr));
    CHECK(copy != nullptr && copy.get() != p.get());
    auto* rt2 = cap<IPluginV3OneRuntime>(copy.get(), PluginCapabilityType::kRUNTIME);
    const PluginFieldCollection* ser = rt2->getFieldsToSerialize();
    CHECK(ser->nbFields == 1 && std::strcmp(ser->fields[0].name, "scale") == 0 &&
          ser->fields[0].type == PluginFieldType::kFLOAT32 && ser->fields[0].length == 1 &&
          *static_cast<const float*>(ser->fields[0].data) == 0.088388F);
    std::unique_ptr<IPluginV3> c2(p->clone());
    CHECK(c2 != nullptr);
}

static void test_weights_plugin() {
    auto* c = creator(g_runtime, "zipformer_relative_attention");
    CHECK(c->getFieldNames()->nbFields == 0);
    auto fc0 = fields(nullptr, 0);
    std::unique_ptr<IPluginV3> p(c->createPlugin("w", &fc0, TensorRTPhase::kRUNTIME));
    CHECK(p != nullptr);
    float s = 1;
    PluginField extra{"scale", &s, PluginFieldType::kFLOAT32, 1};
    auto fc1 = fields(&extra, 1);
    CHECK(c->createPlugin("w", &fc1, TensorRTPhase::kRUNTIME) == nullptr);
    CHECK(c->createPlugin("w", nullptr, TensorRTPhase::kRUNTIME) == nullptr);

    auto* build = cap<IPluginV3OneBuild>(p.get(), PluginCapabilityType::kBUILD);
    auto* rt = cap<IPluginV3OneRuntime>(p.get(), PluginCapabilityType::kRUNTIME);
    CHECK(std::string(build->getTimingCacheID()).find("impl=fga-sm100a") != std::string::npos);
    IDimensionExpr n, t, pd, one, rel, h, four, mn, mt;
    DimsExprs ein[3];
    ein[0].nbDims = 3; ein[0].d[0] = &n; ein[0].d[1] = &t; ein[0].d[2] = &pd;
    ein[1].nbDims = 4; ein[1].d[0] = &one; ein[1].d[1] = &rel; ein[1].d[2] = &h; ein[1].d[3] = &four;
    ein[2].nbDims = 2; ein[2].d[0] = &mn; ein[2].d[1] = &mt;
    DimsExprs eout[1];
    IExprBuilder eb;
    CHECK(build->getOutputShapes(ein, 3, nullptr, 0, eout, 1, eb) == 0);
    CHECK(eout[0].nbDims == 4 && eout[0].d[0] == &n && eout[0].d[1] == &h && eout[0].d[2] == &t &&
          eout[0].d[3] == &t);
    DataType ins[3] = {DataType::kBF16, DataType::kBF16, DataType::kBOOL}, out;
    CHECK(build->getOutputDataTypes(&out, 1, ins, 3) == 0 && out == DataType::kBF16);

    PluginTensorDesc pin[3] = {desc(DataType::kBF16, {4, 100, 272}), desc(DataType::kBF16, {1, 199, 4, 4}),
                               desc(DataType::kBOOL, {4, 100})};
    PluginTensorDesc pout[1] = {desc(DataType::kBF16, {4, 4, 100, 100})};
    DynamicPluginTensorDesc din[3] = {dyn(pin[0]), dyn(pin[1]), dyn(pin[2])}, dout[1] = {dyn(pout[0])};
    CHECK(build->configurePlugin(din, 3, dout, 1) == 0);
    din[2].desc.type = DataType::kINT32;
    CHECK(build->configurePlugin(din, 3, dout, 1) != 0);
    din[2].desc.type = DataType::kBOOL;
    g_workspace = FGA_SCHED_WORKSPACE_BYTES;
    CHECK(build->getWorkspaceSize(din, 3, dout, 1) == FGA_SCHED_WORKSPACE_BYTES);
    CHECK(rt->onShapeChange(pin, 3, pout, 1) == 0 && g_last.fn == "weights_check");
    const void* inputs[3] = {reinterpret_cast<void*>(0x10), reinterpret_cast<void*>(0x20),
                             reinterpret_cast<void*>(0x30)};
    void* outputs[1] = {reinterpret_cast<void*>(0x40)};
    void* ws = reinterpret_cast<void*>(0x1000);
    cudaStream_t stream = reinterpret_cast<cudaStream_t>(0x50);
    CHECK(rt->enqueue(pin, pout, inputs, outputs, ws, stream) == 0);
    CHECK(g_last.fn == "weights_enqueue" && g_last.workspace == ws &&
          g_last.workspace_bytes == FGA_SCHED_WORKSPACE_BYTES && g_last.stream == stream &&
          g_last.inputs == inputs && g_last.outputs == outputs);
    for (int i = 0; i < 3; ++i) CHECK(same(g_last.in[i], pin[i]));
    CHECK(same(g_last.out[0], pout[0]));
    g_status = FGA_ERROR_WORKSPACE;
    CHECK(rt->enqueue(pin, pout, inputs, outputs, nullptr, stream) == 1);
    g_status = FGA_SUCCESS;
    CHECK(rt->getFieldsToSerialize()->nbFields == 0);
    std::unique_ptr<IPluginV3> copy(rt->attachToContext(nullptr));
    CHECK(copy != nullptr);
}

static std::unique_ptr<IPluginV3> make_value(std::initializer_list<PluginField> fl) {
    std::vector<PluginField> v(fl);
    auto fc = fields(v.data(), static_cast<int32_t>(v.size()));
    return std::unique_ptr<IPluginV3>(
        creator(g_runtime, "zipformer_attention_value")->createPlugin("v", &fc, TensorRTPhase::kBUILD));
}

static void test_value_plugin() {
    int32_t four = 4, zero = 0, one = 1;
    float f = 4;
    CHECK(make_value({{"num_heads", &four, PluginFieldType::kINT32, 1}}) != nullptr);
    CHECK(make_value({{"other", &f, PluginFieldType::kFLOAT32, 1},
                      {"num_heads", &one, PluginFieldType::kINT32, 1}}) != nullptr);  // unknown ignored
    CHECK(make_value({}) == nullptr);
    CHECK(make_value({{"num_heads", &zero, PluginFieldType::kINT32, 1}}) == nullptr);
    CHECK(make_value({{"num_heads", &f, PluginFieldType::kFLOAT32, 1}}) == nullptr);
    CHECK(make_value({{"num_heads", &four, PluginFieldType::kINT32, 2}}) == nullptr);
    CHECK(make_value({{"num_heads", &four, PluginFieldType::kINT32, 1},
                      {"num_heads", &four, PluginFieldType::kINT32, 1}}) == nullptr);  // duplicate

    auto p = make_value({{"num_heads", &four, PluginFieldType::kINT32, 1}});
    auto* build = cap<IPluginV3OneBuild>(p.get(), PluginCapabilityType::kBUILD);
    auto* rt = cap<IPluginV3OneRuntime>(p.get(), PluginCapabilityType::kRUNTIME);
    CHECK(std::string(build->getTimingCacheID()).find("num_heads=4") != std::string::npos);
    PluginTensorDesc pin[2] = {desc(DataType::kHALF, {2, 4, 65, 65}), desc(DataType::kHALF, {2, 65, 48})};
    PluginTensorDesc pout[1] = {desc(DataType::kHALF, {2, 65, 48})};
    DynamicPluginTensorDesc din[2] = {dyn(pin[0]), dyn(pin[1])}, dout[1] = {dyn(pout[0])};
    g_status = FGA_SUCCESS;
    CHECK(build->configurePlugin(din, 2, dout, 1) == 0 && g_last.fn == "value_check" && g_last.heads == 4);
    g_status = FGA_ERROR_BAD_SHAPE;
    CHECK(build->configurePlugin(din, 2, dout, 1) != 0);
    g_status = FGA_SUCCESS;
    DataType ins[2] = {DataType::kHALF, DataType::kHALF}, out;
    CHECK(build->getOutputDataTypes(&out, 1, ins, 2) == 0 && out == DataType::kHALF);
    IDimensionExpr a, b, cc;
    DimsExprs ein[2];
    ein[1].nbDims = 3; ein[1].d[0] = &a; ein[1].d[1] = &b; ein[1].d[2] = &cc;
    DimsExprs eout[1];
    IExprBuilder eb;
    CHECK(build->getOutputShapes(ein, 2, nullptr, 0, eout, 1, eb) == 0 && eout[0].nbDims == 3 &&
          eout[0].d[2] == &cc);
    const void* inputs[2] = {reinterpret_cast<void*>(0x10), reinterpret_cast<void*>(0x20)};
    void* outputs[1] = {reinterpret_cast<void*>(0x40)};
    cudaStream_t stream = reinterpret_cast<cudaStream_t>(0x50);
    g_workspace = 0;
    CHECK(rt->enqueue(pin, pout, inputs, outputs, nullptr, stream) == 0);
    CHECK(g_last.fn == "value_enqueue" && g_last.heads == 4 && g_last.stream == stream &&
          g_last.inputs == inputs && g_last.outputs == outputs);
    const PluginFieldCollection* ser = rt->getFieldsToSerialize();
    CHECK(ser->nbFields == 1 && std::strcmp(ser->fields[0].name, "num_heads") == 0 &&
          *static_cast<const int32_t*>(ser->fields[0].data) == 4);
    std::unique_ptr<IPluginV3> copy(rt->attachToContext(nullptr));
    CHECK(copy != nullptr);
}

// Both convolution plugins: no fields, x-shaped output of x's type, int32 lengths, the
// profile's min/opt/max checked through the C ABI, the reference's tactic IDs accepted,
// exact forwarding with no workspace.
static void test_convolution_plugin(const char* name, const char* prefix, int32_t tactic) {
    auto* c = creator(g_runtime, name);
    CHECK(c->getFieldNames()->nbFields == 0);
    auto fc0 = fields(nullptr, 0);
    std::unique_ptr<IPluginV3> p(c->createPlugin("c", &fc0, TensorRTPhase::kBUILD));
    CHECK(p != nullptr);
    int32_t k = 9;
    PluginField extra{"kernel_size", &k, PluginFieldType::kINT32, 1};
    auto fc1 = fields(&extra, 1);
    CHECK(c->createPlugin("c", &fc1, TensorRTPhase::kBUILD) == nullptr);
    CHECK(c->createPlugin("c", nullptr, TensorRTPhase::kBUILD) == nullptr);
    auto* core = cap<IPluginV3OneCore>(p.get(), PluginCapabilityType::kCORE);
    auto* build = cap<IPluginV3OneBuild>(p.get(), PluginCapabilityType::kBUILD);
    auto* rt = cap<IPluginV3OneRuntime>(p.get(), PluginCapabilityType::kRUNTIME);
    CHECK(std::strcmp(core->getPluginName(), name) == 0);
    CHECK(std::strcmp(core->getPluginVersion(), "1") == 0);
    CHECK(std::strcmp(core->getPluginNamespace(), "fast_gpu_asr") == 0);
    CHECK(std::string(build->getTimingCacheID()).find("impl=fga-sm100a") != std::string::npos);
    CHECK(rt->setTactic(0) == 0 && rt->setTactic(tactic) == 0 && rt->setTactic(7) != 0);

    DataType ins[4] = {DataType::kHALF, DataType::kINT32, DataType::kHALF, DataType::kHALF}, out;
    CHECK(build->getOutputDataTypes(&out, 1, ins, 4) == 0 && out == DataType::kHALF);
    ins[1] = DataType::kHALF;
    CHECK(build->getOutputDataTypes(&out, 1, ins, 4) != 0);
    IDimensionExpr n, t, ch, nl, kk, wc, bc;
    DimsExprs ein[4];
    ein[0].nbDims = 3; ein[0].d[0] = &n; ein[0].d[1] = &t; ein[0].d[2] = &ch;
    ein[1].nbDims = 1; ein[1].d[0] = &nl;
    ein[2].nbDims = 2; ein[2].d[0] = &kk; ein[2].d[1] = &wc;
    ein[3].nbDims = 1; ein[3].d[0] = &bc;
    DimsExprs eout[1];
    IExprBuilder eb;
    CHECK(build->getOutputShapes(ein, 4, nullptr, 0, eout, 1, eb) == 0);
    CHECK(eout[0].nbDims == 3 && eout[0].d[0] == &n && eout[0].d[1] == &t && eout[0].d[2] == &ch);

    PluginTensorDesc pin[4] = {desc(DataType::kHALF, {2, 17, 16}), desc(DataType::kINT32, {2}),
                               desc(DataType::kHALF, {9, 16}), desc(DataType::kHALF, {16})};
    PluginTensorDesc pout[1] = {desc(DataType::kHALF, {2, 17, 16})};
    DynamicPluginTensorDesc din[4] = {dyn(pin[0]), dyn(pin[1]), dyn(pin[2]), dyn(pin[3])};
    DynamicPluginTensorDesc dout[1] = {dyn(pout[0])};
    DynamicPluginTensorDesc io[5] = {din[0], din[1], din[2], din[3], dout[0]};
    CHECK(build->supportsFormatCombination(1, io, 4, 1));
    CHECK(build->supportsFormatCombination(4, io, 4, 1));
    io[4].desc.type = DataType::kBF16;
    CHECK(!build->supportsFormatCombination(4, io, 4, 1));
    g_status = FGA_SUCCESS;
    CHECK(build->configurePlugin(din, 4, dout, 1) == 0 &&
          g_last.fn == std::string(prefix) + "_check");
    g_status = FGA_ERROR_BAD_SHAPE;
    CHECK(build->configurePlugin(din, 4, dout, 1) != 0);
    CHECK(rt->onShapeChange(pin, 4, pout, 1) != 0);
    g_status = FGA_SUCCESS;
    din[1].desc.type = DataType::kHALF;
    CHECK(build->configurePlugin(din, 4, dout, 1) != 0);
    din[1].desc.type = DataType::kINT32;
    CHECK(build->getWorkspaceSize(din, 4, dout, 1) == 0);
    CHECK(rt->onShapeChange(pin, 4, pout, 1) == 0);
    const void* inputs[4] = {reinterpret_cast<void*>(0x10), reinterpret_cast<void*>(0x20),
                             reinterpret_cast<void*>(0x30), reinterpret_cast<void*>(0x38)};
    void* outputs[1] = {reinterpret_cast<void*>(0x40)};
    cudaStream_t stream = reinterpret_cast<cudaStream_t>(0x50);
    CHECK(rt->enqueue(pin, pout, inputs, outputs, nullptr, stream) == 0);
    CHECK(g_last.fn == std::string(prefix) + "_enqueue" && g_last.stream == stream &&
          g_last.inputs == inputs && g_last.outputs == outputs && g_last.workspace_bytes == 0);
    for (int i = 0; i < 4; ++i) CHECK(same(g_last.in[i], pin[i]));
    CHECK(same(g_last.out[0], pout[0]));
    g_status = FGA_ERROR_PRIOR_CUDA_ERROR;
    CHECK(rt->enqueue(pin, pout, inputs, outputs, nullptr, stream) == 1);
    g_status = FGA_SUCCESS;
    CHECK(rt->getFieldsToSerialize()->nbFields == 0);
    std::unique_ptr<IPluginV3> copy(rt->attachToContext(nullptr));
    CHECK(copy != nullptr);
}

int main() {
    test_registration();
    test_parakeet_fields();
    test_parakeet_plugin();
    test_weights_plugin();
    test_value_plugin();
    test_convolution_plugin("parakeet_conformer_convolution", "pconv", 2304);
    test_convolution_plugin("zipformer_convolution", "zconv", 4096 + 256);
    if (g_failures != 0) {
        std::fprintf(stderr, "%d check(s) failed\n", g_failures);
        return 1;
    }
    std::printf("trt shim contracts: ok\n");
    return 0;
}
