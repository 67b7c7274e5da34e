// TensorRT plugin `parakeet_conformer_convolution` v1 (namespace fast_gpu_asr) over the C ABI.
//
// Drop-in for the reference's ParakeetConvolutionPlugin and its creator
// (src/fast_gpu_asr/tensorrt_plugins/parakeet_convolution_plugin.cu:364-694): same name,
// version, namespace, no fields, bindings, output rules and error convention; the
// computation is fga_parakeet_conformer_convolution_enqueue.
#include "fga_trt_convolution.h"

namespace fga_trt {
namespace {

struct ParakeetConvolutionTraits {
    static constexpr char const* kName = "parakeet_conformer_convolution";
    static constexpr char const* kTimingTag = "layout=ntc;activation=silu;bn=folded";
    // The reference's single tactic ID (parakeet_convolution_plugin.cu:41).
    static constexpr int32_t kReferenceTactics[1] = {2304};
    static int32_t check(const fga_tensor_desc* in, int32_t nin, const fga_tensor_desc* out,
                         int32_t nout) noexcept {
        return fga_parakeet_conformer_convolution_check(in, nin, out, nout);
    }
    static int32_t enqueue(const fga_tensor_desc* in, const fga_tensor_desc* out,
                           const void* const* inputs, void* const* outputs, void* ws,
                           size_t ws_bytes, void* stream) noexcept {
        return fga_parakeet_conformer_convolution_enqueue(in, out, inputs, outputs, ws, ws_bytes,
                                                          stream);
    }
};

}  // namespace
}  // namespace fga_trt

FGA_TRT_EXPORT bool initFastGpuAsrParakeetConvolutionPlugin() noexcept {
    static fga_trt::ConvolutionCreator<fga_trt::ParakeetConvolutionTraits> runtime_creator;
    static fga_trt::ConvolutionCreator<fga_trt::ParakeetConvolutionTraits> builder_creator;
    return fga_trt::register_in_both_registries(runtime_creator, builder_creator);
}
