// In-memory TensorRT plugin registries for the plugin-loader test: a stand-in for the two
// registry entry points of libnvinfer, loaded with global visibility before the shim
// libraries. FGA_STUB_REGISTRY_REFUSE=1 makes every registration fail. TEST INFRASTRUCTURE.
#include <NvInfer.h>

#include <cstdlib>
#include <cstring>
#include <map>
#include <string>

using namespace nvinfer1;

namespace {
class Registry final : public IPluginRegistry {
  public:
    bool registerCreator(IPluginCreatorInterface& creator, char const* ns) noexcept override {
        const char* refuse = std::getenv("FGA_STUB_REGISTRY_REFUSE");
        if (refuse != nullptr && std::strcmp(refuse, "1") == 0) return false;
        auto* c = dynamic_cast<IPluginCreatorV3One*>(&creator);
        if (c == nullptr || ns == nullptr) return false;
        const std::string key = std::string(c->getPluginName()) + "/" + c->getPluginVersion() + "/" + ns;
        if (creators_.count(key) != 0) return false;
        creators_[key] = c;
        ++registered;
        return true;
    }
    IPluginCreatorInterface* getCreator(char const* name, char const* version,
                                        char const* ns) noexcept override {
        auto it = creators_.find(std::string(name) + "/" + version + "/" + ns);
        return it == creators_.end() ? nullptr : it->second;
    }
    int registered = 0;

  private:
    std::map<std::string, IPluginCreatorV3One*> creators_;
};
Registry g_runtime, g_builder;
}  // namespace

extern "C" __attribute__((visibility("default"))) IPluginRegistry* getPluginRegistry() noexcept {
    return &g_runtime;
}
namespace nvinfer1 {
extern "C" __attribute__((visibility("default"))) IPluginRegistry* getBuilderPluginRegistry(
    EngineCapability capability) noexcept {
    return capability == EngineCapability::kSTANDARD ? &g_builder : nullptr;
}
}  // namespace nvinfer1

// Creators registered so far in the runtime and builder registries.
extern "C" __attribute__((visibility("default"))) int fga_stub_registered(int builder) {
    return builder ? g_builder.registered : g_runtime.registered;
}
