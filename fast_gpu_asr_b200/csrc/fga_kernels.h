// Internal launch interface between the C ABI (fga_capi.cu) and the kernels.
// Every problem struct holds already-validated shapes; launchers only choose a
// kernel variant and launch it on the given stream.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace fga {

struct ParakeetProblem {
    const void* qkv;       // [N, T, 3C]
    const void* position;  // [1, 2T-1, C]
    const void* content_bias;   // [H, D]
    const void* position_bias;  // [H, D]
    const int32_t* valid_lengths;  // [N]
    void* output;          // [N, T, C]
    int32_t batch, length, heads, head_dim;
    float scale;
    int32_t dtype;  // fga_data_type
};

struct ZipformerWeightsProblem {
    const void* projection;  // [N, T, H*(2qd+4)]
    const void* position;    // [1, 2T-1, H, 4]
    const uint8_t* mask;     // [N, T] bool
    void* weights;           // [N, H, T, T]
    unsigned int* sched;     // tensor-core path: the launch's work counter (workspace)
    int32_t batch, length, heads, query_dim;
    int32_t dtype;
};

// Zipformer weights applied in the same kernel to the two SelfAttention value tensors
// (no [N, H, T, T] tensor is written), plus head 0's weights for NonlinAttention, all
// in one kernel.
struct ZipformerFusedProblem {
    const void* projection;  // [N, T, H*(2qd+4)]
    const void* position;    // [1, 2T-1, H, 4]
    const uint8_t* mask;     // [N, T] bool
    const void* value1;      // [N, T, H*vd]
    const void* value2;      // [N, T, H*vd]
    void* output1;           // [N, T, H*vd]
    void* output2;           // [N, T, H*vd]
    void* weights0;          // [N, 1, T, T]: head 0's weights
    unsigned int* sched;     // the launch's work counter (workspace)
    int32_t batch, length, heads, query_dim, value_dim;
    int32_t dtype;
};

struct ZipformerValueProblem {
    const void* attention;  // [N, Ha, T, T]
    const void* value;      // [N, T, C]
    void* output;           // [N, T, C]
    int32_t batch, attention_heads, length, channels, value_heads;
    int32_t dtype;
};

// Depthwise temporal convolution of an encoder convolution module (Parakeet Conformer:
// SiLU; Zipformer: Swoosh-R).
struct ConvolutionProblem {
    enum Kind : int32_t { kParakeet = 0, kZipformer = 1 };
    const void* x;                 // [N, T, C]
    const int32_t* valid_lengths;  // [N]
    const void* weight;            // [K, C]
    const void* bias;              // [C]
    void* output;                  // [N, T, C]
    int32_t batch, length, channels, taps;
    int32_t dtype;
    int32_t kind;
};

// Each launcher returns cudaSuccess or the launch error, and records the variant.
cudaError_t launch_parakeet(const ParakeetProblem& p, cudaStream_t stream, const char** variant);
cudaError_t launch_zipformer_weights(const ZipformerWeightsProblem& p, cudaStream_t stream,
                                     const char** variant);
cudaError_t launch_zipformer_value(const ZipformerValueProblem& p, cudaStream_t stream,
                                   const char** variant);
cudaError_t launch_convolution(const ConvolutionProblem& p, cudaStream_t stream,
                               const char** variant);
// Tensor cores only: cudaErrorNotSupported outside the envelope (f16/bf16, qd = 32,
// T <= 768, vd a multiple of 4 up to 16, H*vd a multiple of 8, aligned buffers).
cudaError_t launch_zipformer_fused(const ZipformerFusedProblem& p, cudaStream_t stream);

// Device address (current device) of the scratch that the weights entry point without a
// workspace uses for its work counter (FGA_NO_WORKSPACE_SCRATCH_BYTES bytes).
cudaError_t no_workspace_scratch(void** ptr);

// SIMT (CUDA-core) kernels: every dtype and shape the contract accepts.
cudaError_t launch_parakeet_simt(const ParakeetProblem& p, cudaStream_t stream);
cudaError_t launch_zipformer_weights_simt(const ZipformerWeightsProblem& p, cudaStream_t stream);
cudaError_t launch_zipformer_value_simt(const ZipformerValueProblem& p, cudaStream_t stream);

// Tensor-core (tcgen05/TMEM) kernels for f16/bf16. Each returns cudaErrorNotSupported
// without launching when the problem is outside the kernel's envelope.
cudaError_t launch_parakeet_tc(const ParakeetProblem& p, cudaStream_t stream);
cudaError_t launch_zipformer_weights_tc(const ZipformerWeightsProblem& p, cudaStream_t stream);
cudaError_t launch_zipformer_value_tc(const ZipformerValueProblem& p, cudaStream_t stream);

// True when the current device is sm_100 (the only target of this library).
bool device_is_sm100();

// Per-device error words of the tensor-core kernels (nonzero: a bounded wait gave up, or
// a launch found its shared memory misaligned), read after the work queued on `stream`
// and optionally cleared. CUDA errors of the reads go to *err.
uint32_t take_parakeet_tc_error(cudaStream_t stream, bool clear, cudaError_t* err);
uint32_t take_zipformer_tc_error(cudaStream_t stream, bool clear, cudaError_t* err);
uint32_t take_value_tc_error(cudaStream_t stream, bool clear, cudaError_t* err);

}  // namespace fga
