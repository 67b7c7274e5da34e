/*
 * fga_convolution.h - C ABI of the encoder convolution-module entry points of
 * libfga_attention.so (B200, sm_100a).
 *
 * Each entry point replaces the body of the `enqueue` method of one of the reference's
 * two depthwise-convolution TensorRT plugins, with the same tensor descriptors, binding
 * order, raw device pointers and stream, and the conventions of fga_attention.h (types,
 * status codes, no allocation, one stream, re-validation on every call, a pending CUDA
 * error reported without launching).
 *
 * inputs[0] x             [N, T, C] f32|f16|bf16   (NTC activations after the GLU)
 * inputs[1] valid_lengths [N]       int32          (clamped to [0, T])
 * inputs[2] weight        [K, C]    same type      (depthwise taps, K odd)
 * inputs[3] bias          [C]       same type
 * outputs[0] output       [N, T, C] same type
 *
 * output[n,t,c] = act(bias[c] + sum_k weight[k,c] * x[n, t+k-K/2, c]), where frames at or
 * past the valid length and outside [0, T) contribute zero. Output frames past the valid
 * length are written, not re-masked. f16/bf16 accumulate in the storage type (one fused
 * multiply-add per tap, in tap order, each rounded) and apply the activation in fp32 to the
 * rounded sum; fp32 accumulates in fp32. C must be a multiple of 4 (fp32) or 2 (f16/bf16),
 * and every buffer aligned to two elements (fp32: 8 bytes) - allocations are - else
 * FGA_ERROR_UNSUPPORTED. No workspace (the queries return 0).
 */
#ifndef FGA_CONVOLUTION_H
#define FGA_CONVOLUTION_H

#include "fga_attention.h"

#ifdef __cplusplus
extern "C" {
#endif

/* --------------------------------------------------------------------------------
 * parakeet_conformer_convolution: masked depthwise convolution, BatchNorm folded into
 * weight and bias by the exporter, then SiLU: act(v) = v / (1 + exp(-v)).
 *
 * Replaces ParakeetConvolutionPlugin::enqueue,
 *   src/fast_gpu_asr/tensorrt_plugins/parakeet_convolution_plugin.cu:552-625,
 * with the shape contract of haveValidShapes (same file :85-103) and the type checks of
 * configurePlugin (:403-441). The plugin has no fields.
 * -------------------------------------------------------------------------------- */
FGA_API int32_t fga_parakeet_conformer_convolution_check(const fga_tensor_desc* input_descs,
    int32_t nb_inputs, const fga_tensor_desc* output_descs, int32_t nb_outputs);
FGA_API size_t fga_parakeet_conformer_convolution_workspace_size(
    const fga_tensor_desc* input_descs, int32_t nb_inputs);
FGA_API int32_t fga_parakeet_conformer_convolution_enqueue(const fga_tensor_desc* input_descs,
    const fga_tensor_desc* output_descs, const void* const* inputs, void* const* outputs,
    void* workspace, size_t workspace_bytes, void* stream);

/* --------------------------------------------------------------------------------
 * zipformer_convolution: masked depthwise convolution, then Swoosh-R:
 * act(v) = softplus(v - 1) - 0.08 v - 0.313261687.
 *
 * Replaces ZipformerConvolutionPlugin::enqueue,
 *   src/fast_gpu_asr/tensorrt_plugins/zipformer_convolution_plugin.cu:757-846,
 * with the shape contract of haveValidShapes (same file :130-150). The reference's tactic
 * (block size and frames per thread) does not change results; this entry point takes none.
 * -------------------------------------------------------------------------------- */
FGA_API int32_t fga_zipformer_convolution_check(const fga_tensor_desc* input_descs,
    int32_t nb_inputs, const fga_tensor_desc* output_descs, int32_t nb_outputs);
FGA_API size_t fga_zipformer_convolution_workspace_size(const fga_tensor_desc* input_descs,
    int32_t nb_inputs);
FGA_API int32_t fga_zipformer_convolution_enqueue(const fga_tensor_desc* input_descs,
    const fga_tensor_desc* output_descs, const void* const* inputs, void* const* outputs,
    void* workspace, size_t workspace_bytes, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* FGA_CONVOLUTION_H */
