/*
 * fga_attention.h - C ABI of the B200 (sm_100a) encoder self-attention library
 * (libfga_attention.so).
 *
 * The first three entry points below replace the bodies of the `enqueue` methods of
 * the reference's three attention TensorRT plugins. Each takes the same tensor
 * descriptors (type, rank, dims), the same raw device pointers in the same binding
 * order and the same stream, and returns 0 on success and nonzero on failure, so a
 * TensorRT shim converts `PluginTensorDesc` to `fga_tensor_desc` one field at a time
 * and forwards. No torch, TensorRT or CUDA type appears in any signature: a stream is
 * passed as `void*` (a `cudaStream_t`), device buffers as `void*`. A fourth entry
 * point, fga_zipformer_attention_fused_enqueue, has no reference plugin (it replaces
 * three plugin calls of one Zipformer layer at once) and follows the same conventions.
 *
 * Memory: the caller owns every input, output and workspace buffer; no entry point
 * allocates device memory. The Zipformer weights and fused entry points need a small
 * workspace (FGA_SCHED_WORKSPACE_BYTES, reported by their `*_workspace_size` queries):
 * it holds the launch's work counter, which the entry point zeroes on the given stream
 * before the kernel, so it needs no initialisation. The other entry points need none
 * (their queries return 0). All launches go on the given stream only, so an entry point
 * is safe to capture in a CUDA graph. Calls from several host threads on different
 * streams may run at once as long as each call has its own workspace (TensorRT gives each
 * execution context its own); two launches that share a workspace must not overlap.
 *
 * Error behaviour mirrors the reference plugins: descriptors are re-validated on every
 * call (rank, dtype, cross-input shape relations, 64-bit size arithmetic), a CUDA
 * error left over from earlier asynchronous work is reported without launching, and
 * the launch status is returned.
 */
#ifndef FGA_ATTENTION_H
#define FGA_ATTENTION_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define FGA_API __attribute__((visibility("default")))
#else
#define FGA_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define FGA_ABI_VERSION 2
/* Workspace of the Zipformer weights and fused entry points (at least 4-byte aligned). */
#define FGA_SCHED_WORKSPACE_BYTES 256
#define FGA_MAX_DIMS 8

/* Element types. The values equal TensorRT's nvinfer1::DataType numbering, so a
 * plugin shim passes `PluginTensorDesc::type` through unchanged. */
enum fga_data_type {
    FGA_FLOAT = 0, /* float32 */
    FGA_HALF = 1,  /* float16 */
    FGA_INT32 = 3,
    FGA_BOOL = 4,  /* one byte per element, 0 or 1 */
    FGA_BF16 = 7,
};

/* Status codes. Every nonzero value means that nothing was launched, except
 * FGA_ERROR_LAUNCH, which reports a failed kernel launch. */
enum fga_status {
    FGA_SUCCESS = 0,
    FGA_ERROR_NULL_POINTER = 1,
    FGA_ERROR_BAD_DESCRIPTOR = 2, /* rank, dtype or format not accepted */
    FGA_ERROR_BAD_SHAPE = 3,      /* cross-tensor shape relation violated */
    FGA_ERROR_OVERFLOW = 4,       /* a size product leaves the int32/int64 range */
    FGA_ERROR_BAD_FIELD = 5,      /* plugin field (scale, num_heads) rejected */
    FGA_ERROR_PRIOR_CUDA_ERROR = 6,
    FGA_ERROR_LAUNCH = 7,
    FGA_ERROR_NO_DEVICE = 8,      /* current device is not sm_100 */
    FGA_ERROR_UNSUPPORTED = 9,    /* valid, but outside an entry point's stated envelope */
    FGA_ERROR_WORKSPACE = 10,     /* workspace missing, too small or misaligned */
    FGA_ERROR_DEVICE_ABORT = 11,  /* fga_device_status: a kernel gave up a bounded wait */
};

/* Mirrors nvinfer1::PluginTensorDesc minus format (row-major linear is implied). */
typedef struct fga_tensor_desc {
    int32_t type;     /* enum fga_data_type */
    int32_t nb_dims;  /* 1..FGA_MAX_DIMS */
    int64_t dims[FGA_MAX_DIMS];
} fga_tensor_desc;

/* --------------------------------------------------------------------------------
 * parakeet_relative_attention (Transformer-XL relative-position MHSA, FastConformer)
 *
 * Replaces ParakeetRelativeAttentionPlugin::enqueue,
 *   src/fast_gpu_asr/tensorrt_plugins/parakeet_relative_attention_plugin.cu:923-1139,
 * with the shape contract of haveValidShapes (same file :237-290) and the field
 * contract of the creator (:1189-1220).
 *
 * inputs[0] qkv            [N, T, 3C]  f32|f16|bf16   (Q heads, K heads, V heads)
 * inputs[1] position       [1, 2T-1, C] same type     (linear_pos(pos_emb))
 * inputs[2] content_bias   [H, D]       same type     (pos_bias_u)
 * inputs[3] position_bias  [H, D]       same type     (pos_bias_v)
 * inputs[4] valid_lengths  [N]          int32
 * outputs[0] output        [N, T, C]    same type, C = H*D
 *
 * out[n,q,h,:] = sum_k softmax_k(scale*((q+u).k_k + (q+v).p[T-1-q+k])) v_k over keys
 * k < valid_lengths[n]; rows of an utterance with valid_lengths[n] <= 0 are zero.
 * scale must be finite, > 0, and scale*log2(e) finite.
 * -------------------------------------------------------------------------------- */
FGA_API int32_t fga_parakeet_relative_attention_check(const fga_tensor_desc* input_descs,
    int32_t nb_inputs, const fga_tensor_desc* output_descs, int32_t nb_outputs, float scale);
FGA_API size_t fga_parakeet_relative_attention_workspace_size(const fga_tensor_desc* input_descs,
    int32_t nb_inputs);
FGA_API int32_t fga_parakeet_relative_attention_enqueue(const fga_tensor_desc* input_descs,
    const fga_tensor_desc* output_descs, const void* const* inputs, void* const* outputs,
    float scale, void* workspace, size_t workspace_bytes, void* stream);

/* --------------------------------------------------------------------------------
 * zipformer_relative_attention (relative-position attention weights)
 *
 * Replaces RelativeAttentionPlugin::enqueue and enqueueRelativeAttention,
 *   src/fast_gpu_asr/tensorrt_plugins/zipformer_relative_attention_plugin.cu:761-815
 *   and :490-566, with the shape contract of haveValidShapes (:96-133).
 *
 * inputs[0] projection [N, T, H*(2*qd+4)] f32|f16|bf16 (Q heads, K heads, 4-dim pos queries)
 * inputs[1] position   [1, 2T-1, H, 4]     same type
 * inputs[2] mask       [N, T]              bool, True = padded key (contiguous suffix)
 * outputs[0] weights   [N, H, T, T]        same type
 *
 * No scale is applied. Masked keys get weight 0, a row whose keys are all masked is
 * zero, and query rows q >= 7 with mask[q-7] set (the 7-frame padded-query halo) are
 * zero. workspace: FGA_SCHED_WORKSPACE_BYTES (the reference reported 16 MB for cuBLAS,
 * zipformer_relative_attention_plugin.cu:705-716); FGA_ERROR_WORKSPACE without it.
 * -------------------------------------------------------------------------------- */
FGA_API int32_t fga_zipformer_relative_attention_check(const fga_tensor_desc* input_descs,
    int32_t nb_inputs, const fga_tensor_desc* output_descs, int32_t nb_outputs);
FGA_API size_t fga_zipformer_relative_attention_workspace_size(const fga_tensor_desc* input_descs,
    int32_t nb_inputs);
FGA_API int32_t fga_zipformer_relative_attention_enqueue(const fga_tensor_desc* input_descs,
    const fga_tensor_desc* output_descs, const void* const* inputs, void* const* outputs,
    void* workspace, size_t workspace_bytes, void* stream);

/* No counterpart in the reference: a variant of fga_zipformer_relative_attention_enqueue
 * for callers that cannot allocate device memory - code running where cudaMalloc is not
 * permitted or not wanted (a fixed memory budget decided up front, an embedding host that
 * hands out only input and output buffers, a binding with no device allocator) - and so
 * cannot provide the FGA_SCHED_WORKSPACE_BYTES workspace. It takes no workspace and
 * allocates nothing (no cudaMalloc, cudaFree or allocating library call): the kernel's
 * work counter lives in a fixed device array of FGA_NO_WORKSPACE_SCRATCH_BYTES inside the
 * library, which every GPU that loads the library holds until the process exits. A
 * problem whose scratch needs exceed that array is rejected with FGA_ERROR_WORKSPACE.
 * The first call on a device looks up the array's device address (cudaGetSymbolAddress,
 * with that device current); make that first call before any stream capture. Every call
 * on a device shares the array: the counter is zeroed on the stream before each kernel,
 * but calls that overlap on the GPU (different streams, concurrent graph replays) race
 * on it and may produce wrong weights - order them, or use the workspace entry point.
 * Same inputs, outputs, results and status codes as fga_zipformer_relative_attention_enqueue. */
#define FGA_NO_WORKSPACE_SCRATCH_BYTES 256
FGA_API int32_t fga_zipformer_relative_attention_enqueue_no_workspace(
    const fga_tensor_desc* input_descs, const fga_tensor_desc* output_descs,
    const void* const* inputs, void* const* outputs, void* stream);

/* --------------------------------------------------------------------------------
 * zipformer_attention_value (apply shared attention weights to NTC values)
 *
 * Replaces AttentionValuePlugin::enqueue,
 *   src/fast_gpu_asr/tensorrt_plugins/zipformer_attention_value_plugin.cu:438-572,
 * with the shape contract of haveValidShapes (:79-94) and field `num_heads` (:616-655).
 *
 * inputs[0] attention [N, Ha, T, T] f32|f16|bf16
 * inputs[1] value     [N, T, C]     same type, C % num_heads == 0
 * outputs[0] output   [N, T, C]     same type
 *
 * out[n,q,h,d] = sum_k attention[n,h,q,k] * value[n,k,h,d], fp32 accumulation.
 * num_heads == 1 (NonlinAttention) uses attention head 0 of any Ha >= 1;
 * num_heads > 1 requires Ha == num_heads.
 * -------------------------------------------------------------------------------- */
FGA_API int32_t fga_zipformer_attention_value_check(const fga_tensor_desc* input_descs,
    int32_t nb_inputs, const fga_tensor_desc* output_descs, int32_t nb_outputs,
    int32_t num_heads);
FGA_API size_t fga_zipformer_attention_value_workspace_size(const fga_tensor_desc* input_descs,
    int32_t nb_inputs, int32_t num_heads);
FGA_API int32_t fga_zipformer_attention_value_enqueue(const fga_tensor_desc* input_descs,
    const fga_tensor_desc* output_descs, const void* const* inputs, void* const* outputs,
    int32_t num_heads, void* workspace, size_t workspace_bytes, void* stream);

/* --------------------------------------------------------------------------------
 * zipformer_attention_fused (weights applied to both SelfAttention values in one pass)
 *
 * No reference plugin corresponds to this entry point: it goes beyond the drop-in
 * surface. It computes what zipformer_relative_attention followed by two
 * zipformer_attention_value calls (num_heads = H) compute, for the two SelfAttention
 * modules of a Zipformer layer that share one set of weights
 * (src/fast_gpu_asr/export/model/zipformer/attention.py:62-73), without writing the
 * [N, H, T, T] weights: each 64-key piece of rounded weights goes from the softmax
 * straight into the value MMAs on chip. Head 0's weights, which NonlinAttention reads
 * (attention.py:130-138), are written as [N, 1, T, T] for a following
 * fga_zipformer_attention_value_enqueue call with num_heads = 1.
 *
 * inputs[0] projection [N, T, H*(2*qd+4)] f16|bf16 (as zipformer_relative_attention)
 * inputs[1] position   [1, 2T-1, H, 4]     same type
 * inputs[2] mask       [N, T]              bool, True = padded key
 * inputs[3] value1     [N, T, H*vd]        same type
 * inputs[4] value2     [N, T, H*vd]        same type
 * outputs[0] out1      [N, T, H*vd]        same type
 * outputs[1] out2      [N, T, H*vd]        same type
 * outputs[2] weights0  [N, 1, T, T]        same type
 *
 * The weights are rounded to the I/O type before they are applied, as the two-plugin
 * path does; the products are accumulated in fp32. Envelope: f16/bf16, qd = 32, H even,
 * T <= 768, vd a multiple of 4 in [4, 16], H*vd*2 bytes a multiple of 16, value tensors
 * and weights0 16-byte aligned, outputs 4-byte aligned. Outside it the entry point
 * returns FGA_ERROR_UNSUPPORTED and launches nothing. workspace: FGA_SCHED_WORKSPACE_BYTES.
 * -------------------------------------------------------------------------------- */
FGA_API int32_t fga_zipformer_attention_fused_check(const fga_tensor_desc* input_descs,
    int32_t nb_inputs, const fga_tensor_desc* output_descs, int32_t nb_outputs);
FGA_API size_t fga_zipformer_attention_fused_workspace_size(const fga_tensor_desc* input_descs,
    int32_t nb_inputs);
FGA_API int32_t fga_zipformer_attention_fused_enqueue(const fga_tensor_desc* input_descs,
    const fga_tensor_desc* output_descs, const void* const* inputs, void* const* outputs,
    void* workspace, size_t workspace_bytes, void* stream);

/* --------------------------------------------------------------------------------
 * Library identity and diagnostics (no counterpart needed in the reference; the
 * reference reports failures only through enqueue's return value).
 * -------------------------------------------------------------------------------- */
FGA_API int32_t fga_abi_version(void);
FGA_API const char* fga_status_string(int32_t status);
/* Name of the kernel variant the last successful enqueue on this host thread chose
 * ("tcgen05", "simt", ...); for tests and benchmarks. */
FGA_API const char* fga_last_kernel_variant(void);

/* Device-side status of the tensor-core kernels on the current device. Every wait inside
 * them is bounded (2 s); a kernel that gives up records it in a per-device error word and
 * tears down, leaving its outputs incomplete, while enqueue has already returned success.
 * This call waits for the work queued on `stream`, reads the words and, if `clear` is
 * nonzero, resets them. Returns FGA_SUCCESS when no kernel gave up since the last clear,
 * FGA_ERROR_DEVICE_ABORT when one did, FGA_ERROR_PRIOR_CUDA_ERROR when the read failed.
 * `detail` (optional) receives the words: bits 0-7 Parakeet, 8-15 Zipformer weights and
 * fused, 16-23 attention-value (1 = a wait gave up, 2 = misaligned shared memory). */
FGA_API int32_t fga_device_status(void* stream, int32_t clear, uint32_t* detail);

/* Test hook: the time limit (ns) of the bounded waits in the main loops of the Zipformer
 * weights and fused kernels, for launches made later by this host thread; 0 restores the
 * default (2 s). Waits that drain a CTA's own copies and MMAs keep the default, so a short
 * limit makes the kernel give up cleanly, never fault. */
FGA_API void fga_debug_set_wait_limit_ns(uint64_t limit_ns);

#ifdef __cplusplus
}
#endif

#endif /* FGA_ATTENTION_H */
