// TensorRT plugin `zipformer_convolution` v1 (namespace fast_gpu_asr) over the C ABI.
//
// Drop-in for the reference's ZipformerConvolutionPlugin and its creator
// (src/fast_gpu_asr/tensorrt_plugins/zipformer_convolution_plugin.cu:513-917): same name,
// version, namespace, no fields, bindings, output rules and error convention; the
// computation is fga_zipformer_convolution_enqueue.
#include "fga_trt_convolution.h"

namespace fga_trt {
namespace {

struct ZipformerConvolutionTraits {
    static constexpr char const* kName = "zipformer_convolution";
    static constexpr char const* kTimingTag = "layout=ntc;activation=swoosh_r;zero_padding";
    // The reference's tactic IDs (block size 128/256/512, two or four frames per thread,
    // zipformer_convolution_plugin.cu:36-53): all compute the same values.
    static constexpr int32_t kReferenceTactics[6] = {2048 + 128, 2048 + 256, 2048 + 512,
                                                     4096 + 128, 4096 + 256, 4096 + 512};
    static int32_t check(const fga_tensor_desc* in, int32_t nin, const fga_tensor_desc* out,
                         int32_t nout) noexcept {
        return fga_zipformer_convolution_check(in, nin, out, nout);
    }
    static int32_t enqueue(const fga_tensor_desc* in, const fga_tensor_desc* out,
                           const void* const* inputs, void* const* outputs, void* ws,
                           size_t ws_bytes, void* stream) noexcept {
        return fga_zipformer_convolution_enqueue(in, out, inputs, outputs, ws, ws_bytes, stream);
    }
};

}  // namespace
}  // namespace fga_trt

FGA_TRT_EXPORT bool initFastGpuAsrZipformerConvolutionPlugin() noexcept {
    static fga_trt::ConvolutionCreator<fga_trt::ZipformerConvolutionTraits> runtime_creator;
    static fga_trt::ConvolutionCreator<fga_trt::ZipformerConvolutionTraits> builder_creator;
    return fga_trt::register_in_both_registries(runtime_creator, builder_creator);
}
