// C ABI of libfga_attention.so: descriptor validation and dispatch.
//
// Validation restates the reference plugins' shape contracts in this library's own
// code (the relations must be identical for the entry points to be drop-in):
//   parakeet:  parakeet_relative_attention_plugin.cu:237-290 (haveValidShapes)
//   zipformer: zipformer_relative_attention_plugin.cu:96-133 (haveValidShapes)
//   value:     zipformer_attention_value_plugin.cu:79-94 (haveValidShapes)
//   convolutions: parakeet_convolution_plugin.cu:85-103, zipformer_convolution_plugin.cu:130-150
//              (haveValidShapes, the same relations in both)
// and the field checks of their creators (parakeet…cu:1206-1211,
// zipformer_attention_value…cu:639-650).
#include <cmath>
#include <cstdint>
#include <limits>

#include "../../include/fga_attention.h"
#include "../../include/fga_convolution.h"
#include "fga_kernels.h"
#include "host_util.h"

namespace {

constexpr int64_t kInt32Max = std::numeric_limits<int32_t>::max();
constexpr int64_t kInt64Max = std::numeric_limits<int64_t>::max();
constexpr float kLog2e = 1.4426950408889634f;

thread_local const char* t_last_variant = "none";
thread_local uint64_t t_wait_limit_ns = 0;  // 0: the kernels' default
constexpr uint64_t kDefaultWaitLimitNs = 2000000000ull;  // 2 s, as sm100::kWaitLimitNs

bool is_float_type(int32_t t) { return t == FGA_FLOAT || t == FGA_HALF || t == FGA_BF16; }

int64_t type_bytes(int32_t t) {
    switch (t) {
        case FGA_FLOAT: return 4;
        case FGA_HALF: return 2;
        case FGA_BF16: return 2;
        case FGA_INT32: return 4;
        case FGA_BOOL: return 1;
        default: return 0;
    }
}

bool checked_mul(int64_t a, int64_t b, int64_t& out) {
    if (a < 0 || b < 0) return false;
    if (a != 0 && b > kInt64Max / a) return false;
    out = a * b;
    return true;
}

// Every dimension >= 1 and the byte size fits in int64 (hasAddressableBytes in all
// three reference plugins; the zipformer plugins also cap each dim at INT32_MAX).
bool addressable(const fga_tensor_desc& d, bool cap_dims_int32) {
    int64_t bytes = type_bytes(d.type);
    if (d.nb_dims < 1 || d.nb_dims > FGA_MAX_DIMS || bytes < 1) return false;
    int64_t elems = 1;
    for (int i = 0; i < d.nb_dims; ++i) {
        if (d.dims[i] < 1) return false;
        if (cap_dims_int32 && d.dims[i] > kInt32Max) return false;
        if (!checked_mul(elems, d.dims[i], elems)) return false;
    }
    int64_t total;
    return checked_mul(elems, bytes, total);
}

bool scale_ok(float scale) {
    return std::isfinite(scale) && scale > 0.0f && std::isfinite(scale * kLog2e);
}

int32_t check_parakeet(const fga_tensor_desc* in, int32_t nin, const fga_tensor_desc* out,
                       int32_t nout, float scale, fga::ParakeetProblem* prob) {
    if (in == nullptr || out == nullptr) return FGA_ERROR_NULL_POINTER;
    if (nin != 5 || nout != 1) return FGA_ERROR_BAD_DESCRIPTOR;
    if (!scale_ok(scale)) return FGA_ERROR_BAD_FIELD;
    const fga_tensor_desc &qkv = in[0], &pos = in[1], &u = in[2], &v = in[3], &len = in[4],
                          &o = out[0];
    if (qkv.nb_dims != 3 || pos.nb_dims != 3 || u.nb_dims != 2 || v.nb_dims != 2 ||
        len.nb_dims != 1 || o.nb_dims != 3)
        return FGA_ERROR_BAD_DESCRIPTOR;
    const int32_t t = qkv.type;
    if (!is_float_type(t) || pos.type != t || u.type != t || v.type != t || o.type != t ||
        len.type != FGA_INT32)
        return FGA_ERROR_BAD_DESCRIPTOR;
    for (int i = 0; i < 5; ++i)
        if (!addressable(in[i], false)) return FGA_ERROR_OVERFLOW;
    if (!addressable(o, false)) return FGA_ERROR_OVERFLOW;

    const int64_t batch = qkv.dims[0], length = qkv.dims[1], channels = pos.dims[2];
    const int64_t heads = u.dims[0], head_dim = u.dims[1];
    if (length > kInt32Max / 2 + 1 || channels > kInt32Max / 3) return FGA_ERROR_OVERFLOW;
    const int64_t rel = 2 * length - 1;
    if (qkv.dims[2] != 3 * channels || heads * head_dim != channels || pos.dims[0] != 1 ||
        pos.dims[1] != rel || v.dims[0] != heads || v.dims[1] != head_dim ||
        len.dims[0] != batch || o.dims[0] != batch || o.dims[1] != length ||
        o.dims[2] != channels)
        return FGA_ERROR_BAD_SHAPE;
    if (batch > kInt32Max / heads) return FGA_ERROR_OVERFLOW;
    if (batch * heads > kInt32Max / length) return FGA_ERROR_OVERFLOW;
    // This library's SIMT kernel keeps a query row of up to 512 channels per warp.
    if (head_dim > 512) return FGA_ERROR_BAD_SHAPE;
    if (prob != nullptr) {
        prob->batch = static_cast<int32_t>(batch);
        prob->length = static_cast<int32_t>(length);
        prob->heads = static_cast<int32_t>(heads);
        prob->head_dim = static_cast<int32_t>(head_dim);
        prob->scale = scale;
        prob->dtype = t;
    }
    return FGA_SUCCESS;
}

int32_t check_zipformer(const fga_tensor_desc* in, int32_t nin, const fga_tensor_desc* out,
                        int32_t nout, fga::ZipformerWeightsProblem* prob) {
    if (in == nullptr || out == nullptr) return FGA_ERROR_NULL_POINTER;
    if (nin != 3 || nout != 1) return FGA_ERROR_BAD_DESCRIPTOR;
    const fga_tensor_desc &proj = in[0], &pos = in[1], &mask = in[2], &sc = out[0];
    if (proj.nb_dims != 3 || pos.nb_dims != 4 || mask.nb_dims != 2 || sc.nb_dims != 4)
        return FGA_ERROR_BAD_DESCRIPTOR;
    const int32_t t = proj.type;
    if (!is_float_type(t) || pos.type != t || sc.type != t || mask.type != FGA_BOOL)
        return FGA_ERROR_BAD_DESCRIPTOR;
    if (!addressable(proj, true) || !addressable(pos, true) || !addressable(mask, true) ||
        !addressable(sc, true))
        return FGA_ERROR_OVERFLOW;
    if (pos.dims[0] != 1 || pos.dims[3] != 4 || mask.dims[0] != proj.dims[0] ||
        mask.dims[1] != proj.dims[1] || sc.dims[0] != proj.dims[0] ||
        sc.dims[1] != pos.dims[2] || sc.dims[2] != proj.dims[1] || sc.dims[3] != proj.dims[1])
        return FGA_ERROR_BAD_SHAPE;
    const int64_t batch = proj.dims[0], length = proj.dims[1], pdim = proj.dims[2];
    const int64_t heads = pos.dims[2];
    if (pos.dims[1] != 2 * length - 1 || pdim % heads != 0) return FGA_ERROR_BAD_SHAPE;
    int64_t bh, rows;
    if (!checked_mul(batch, heads, bh) || !checked_mul(bh, length, rows) || rows > kInt32Max)
        return FGA_ERROR_OVERFLOW;
    const int64_t per_head = pdim / heads;
    if (per_head <= 4 || (per_head - 4) % 2 != 0) return FGA_ERROR_BAD_SHAPE;
    const int64_t qd = (per_head - 4) / 2;
    // This library's SIMT kernel stages one query row of up to 256 channels per warp.
    if (qd > 256) return FGA_ERROR_BAD_SHAPE;
    if (prob != nullptr) {
        prob->batch = static_cast<int32_t>(batch);
        prob->length = static_cast<int32_t>(length);
        prob->heads = static_cast<int32_t>(heads);
        prob->query_dim = static_cast<int32_t>(qd);
        prob->dtype = t;
    }
    return FGA_SUCCESS;
}

int32_t check_value(const fga_tensor_desc* in, int32_t nin, const fga_tensor_desc* out,
                    int32_t nout, int32_t value_heads, fga::ZipformerValueProblem* prob) {
    if (in == nullptr || out == nullptr) return FGA_ERROR_NULL_POINTER;
    if (nin != 2 || nout != 1) return FGA_ERROR_BAD_DESCRIPTOR;
    if (value_heads < 1) return FGA_ERROR_BAD_FIELD;
    const fga_tensor_desc &a = in[0], &v = in[1], &o = out[0];
    if (a.nb_dims != 4 || v.nb_dims != 3 || o.nb_dims != 3) return FGA_ERROR_BAD_DESCRIPTOR;
    const int32_t t = v.type;
    if (!is_float_type(t) || a.type != t || o.type != t) return FGA_ERROR_BAD_DESCRIPTOR;
    if (!addressable(a, true) || !addressable(v, true) || !addressable(o, true))
        return FGA_ERROR_OVERFLOW;
    if (a.dims[1] < value_heads || (value_heads > 1 && a.dims[1] != value_heads) ||
        a.dims[0] != v.dims[0] || a.dims[2] != a.dims[3] || a.dims[2] != v.dims[1] ||
        v.dims[2] % value_heads != 0 || o.dims[0] != v.dims[0] || o.dims[1] != v.dims[1] ||
        o.dims[2] != v.dims[2])
        return FGA_ERROR_BAD_SHAPE;
    if (a.dims[0] > kInt32Max / value_heads) return FGA_ERROR_OVERFLOW;
    // Rows (batch * value_heads * T) index a 32-bit grid in this library.
    int64_t rows;
    if (!checked_mul(a.dims[0] * value_heads, a.dims[2], rows) || rows > kInt32Max)
        return FGA_ERROR_OVERFLOW;
    if (prob != nullptr) {
        prob->batch = static_cast<int32_t>(a.dims[0]);
        prob->attention_heads = static_cast<int32_t>(a.dims[1]);
        prob->length = static_cast<int32_t>(a.dims[2]);
        prob->channels = static_cast<int32_t>(v.dims[2]);
        prob->value_heads = value_heads;
        prob->dtype = t;
    }
    return FGA_SUCCESS;
}

// The fused Zipformer entry point: the weights contract of check_zipformer on inputs
// 0..2, two value tensors and two outputs [N, T, H*vd], head 0's weights [N, 1, T, T],
// then the tensor-core envelope (FGA_ERROR_UNSUPPORTED outside it).
int32_t check_fused(const fga_tensor_desc* in, int32_t nin, const fga_tensor_desc* out,
                    int32_t nout, fga::ZipformerFusedProblem* prob) {
    if (in == nullptr || out == nullptr) return FGA_ERROR_NULL_POINTER;
    if (nin != 5 || nout != 3) return FGA_ERROR_BAD_DESCRIPTOR;
    const fga_tensor_desc &proj = in[0], &pos = in[1], &v1 = in[3], &v2 = in[4];
    if (proj.nb_dims != 3 || pos.nb_dims != 4) return FGA_ERROR_BAD_DESCRIPTOR;
    // The weights contract, checked against the [N, H, T, T] tensor it would produce.
    fga_tensor_desc weights{};
    weights.type = proj.type;
    weights.nb_dims = 4;
    weights.dims[0] = proj.dims[0];
    weights.dims[1] = pos.dims[2];
    weights.dims[2] = proj.dims[1];
    weights.dims[3] = proj.dims[1];
    fga::ZipformerWeightsProblem w{};
    int32_t st = check_zipformer(in, 3, &weights, 1, &w);
    if (st != FGA_SUCCESS) return st;
    const int32_t t = proj.type;
    for (const fga_tensor_desc* d : {&v1, &v2, &out[0], &out[1]})
        if (d->nb_dims != 3 || d->type != t) return FGA_ERROR_BAD_DESCRIPTOR;
    if (out[2].nb_dims != 4 || out[2].type != t) return FGA_ERROR_BAD_DESCRIPTOR;
    for (const fga_tensor_desc* d : {&v1, &v2, &out[0], &out[1], &out[2]})
        if (!addressable(*d, true)) return FGA_ERROR_OVERFLOW;
    const int64_t n = proj.dims[0], len = proj.dims[1], heads = w.heads;
    for (const fga_tensor_desc* d : {&v2, &out[0], &out[1]})
        if (d->dims[0] != v1.dims[0] || d->dims[1] != v1.dims[1] || d->dims[2] != v1.dims[2])
            return FGA_ERROR_BAD_SHAPE;
    if (v1.dims[0] != n || v1.dims[1] != len || v1.dims[2] % heads != 0 ||
        out[2].dims[0] != n || out[2].dims[1] != 1 || out[2].dims[2] != len ||
        out[2].dims[3] != len)
        return FGA_ERROR_BAD_SHAPE;
    const int64_t vd = v1.dims[2] / heads;
    // Projection and value rows are read by TMA: 16-byte multiples (an even H for qd = 32).
    if ((t != FGA_HALF && t != FGA_BF16) || w.query_dim != 32 || len > 768 || vd < 4 ||
        vd > 16 || vd % 4 != 0 || (heads * vd * 2) % 16 != 0 || (heads * 68 * 2) % 16 != 0)
        return FGA_ERROR_UNSUPPORTED;
    if (prob != nullptr) {
        prob->batch = w.batch;
        prob->length = w.length;
        prob->heads = w.heads;
        prob->query_dim = w.query_dim;
        prob->value_dim = static_cast<int32_t>(vd);
        prob->dtype = t;
    }
    return FGA_SUCCESS;
}

// The work-counter workspace of the Zipformer weights and fused entry points: present,
// large enough and aligned for 32-bit atomics.
// Depthwise-convolution plugins: x [N, T, C], valid_lengths [N] int32, weight [K, C],
// bias [C], output [N, T, C]; K odd; C a multiple of the reference's vector width (4 for
// fp32, 2 for f16/bf16); every dim in [1, INT32_MAX] and the byte sizes in int64.
int32_t check_convolution(const fga_tensor_desc* in, int32_t nin, const fga_tensor_desc* out,
                          int32_t nout, int32_t kind, fga::ConvolutionProblem* prob) {
    if (in == nullptr || out == nullptr) return FGA_ERROR_NULL_POINTER;
    if (nin != 4 || nout != 1) return FGA_ERROR_BAD_DESCRIPTOR;
    const fga_tensor_desc &x = in[0], &len = in[1], &w = in[2], &b = in[3], &o = out[0];
    if (x.nb_dims != 3 || len.nb_dims != 1 || w.nb_dims != 2 || b.nb_dims != 1 || o.nb_dims != 3)
        return FGA_ERROR_BAD_DESCRIPTOR;
    const int32_t t = x.type;
    if (!is_float_type(t) || len.type != FGA_INT32 || w.type != t || b.type != t || o.type != t)
        return FGA_ERROR_BAD_DESCRIPTOR;
    for (int i = 0; i < 4; ++i)
        if (!addressable(in[i], true)) return FGA_ERROR_OVERFLOW;
    if (!addressable(o, true)) return FGA_ERROR_OVERFLOW;
    const int64_t batch = x.dims[0], length = x.dims[1], channels = x.dims[2], taps = w.dims[0];
    const int64_t width = t == FGA_FLOAT ? 4 : 2;
    if (len.dims[0] != batch || taps % 2 != 1 || w.dims[1] != channels || b.dims[0] != channels ||
        channels % width != 0 || o.dims[0] != batch || o.dims[1] != length ||
        o.dims[2] != channels)
        return FGA_ERROR_BAD_SHAPE;
    if (prob != nullptr) {
        prob->batch = static_cast<int32_t>(batch);
        prob->length = static_cast<int32_t>(length);
        prob->channels = static_cast<int32_t>(channels);
        prob->taps = static_cast<int32_t>(taps);
        prob->dtype = t;
        prob->kind = kind;
    }
    return FGA_SUCCESS;
}

int32_t check_sched_workspace(void* workspace, size_t bytes) {
    if (workspace == nullptr || bytes < FGA_SCHED_WORKSPACE_BYTES ||
        (reinterpret_cast<uintptr_t>(workspace) & 3u) != 0)
        return FGA_ERROR_WORKSPACE;
    return FGA_SUCCESS;
}

// Common epilogue of every enqueue: report an earlier asynchronous error without
// launching (parakeet…cu:948-952), launch, report the launch status.
int32_t prior_error_status() {
    return cudaPeekAtLastError() == cudaSuccess ? FGA_SUCCESS : FGA_ERROR_PRIOR_CUDA_ERROR;
}

int32_t convolution_enqueue(const fga_tensor_desc* in, const fga_tensor_desc* out,
                            const void* const* inputs, void* const* outputs, int32_t kind,
                            void* stream) {
    fga::ConvolutionProblem p{};
    int32_t st = check_convolution(in, 4, out, 1, kind, &p);
    if (st != FGA_SUCCESS) return st;
    if (inputs == nullptr || outputs == nullptr || outputs[0] == nullptr)
        return FGA_ERROR_NULL_POINTER;
    for (int i = 0; i < 4; ++i)
        if (inputs[i] == nullptr) return FGA_ERROR_NULL_POINTER;
    // The kernels move channel pairs: every buffer aligned to two elements.
    const uintptr_t align = p.dtype == FGA_FLOAT ? 8u : 4u;
    for (const void* q : {inputs[0], inputs[2], inputs[3], static_cast<const void*>(outputs[0])})
        if ((reinterpret_cast<uintptr_t>(q) & (align - 1)) != 0) return FGA_ERROR_UNSUPPORTED;
    if ((reinterpret_cast<uintptr_t>(inputs[1]) & 3u) != 0) return FGA_ERROR_UNSUPPORTED;
    if ((st = prior_error_status()) != FGA_SUCCESS) return st;
    if (!fga::device_is_sm100()) return FGA_ERROR_NO_DEVICE;
    p.x = inputs[0];
    p.valid_lengths = static_cast<const int32_t*>(inputs[1]);
    p.weight = inputs[2];
    p.bias = inputs[3];
    p.output = outputs[0];
    const char* variant = "none";
    if (fga::launch_convolution(p, static_cast<cudaStream_t>(stream), &variant) != cudaSuccess)
        return FGA_ERROR_LAUNCH;
    t_last_variant = variant;
    return FGA_SUCCESS;
}

}  // namespace

namespace fga {
uint64_t wait_limit_ns() { return t_wait_limit_ns != 0 ? t_wait_limit_ns : kDefaultWaitLimitNs; }
}  // namespace fga

extern "C" {

int32_t fga_abi_version(void) { return FGA_ABI_VERSION; }

const char* fga_status_string(int32_t status) {
    switch (status) {
        case FGA_SUCCESS: return "success";
        case FGA_ERROR_NULL_POINTER: return "null pointer";
        case FGA_ERROR_BAD_DESCRIPTOR: return "unsupported tensor rank or type";
        case FGA_ERROR_BAD_SHAPE: return "tensor shapes do not satisfy the plugin contract";
        case FGA_ERROR_OVERFLOW: return "tensor size exceeds the addressable range";
        case FGA_ERROR_BAD_FIELD: return "invalid plugin field";
        case FGA_ERROR_PRIOR_CUDA_ERROR: return "an earlier CUDA error is pending";
        case FGA_ERROR_LAUNCH: return "kernel launch failed";
        case FGA_ERROR_NO_DEVICE: return "current CUDA device is not sm_100";
        case FGA_ERROR_UNSUPPORTED: return "outside this entry point's supported envelope";
        case FGA_ERROR_WORKSPACE: return "workspace missing, smaller than required or misaligned";
        case FGA_ERROR_DEVICE_ABORT:
            return "a kernel on this device gave up a bounded wait; its outputs are incomplete";
        default: return "unknown status";
    }
}

const char* fga_last_kernel_variant(void) { return t_last_variant; }

int32_t fga_device_status(void* stream, int32_t clear, uint32_t* detail) {
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t err = cudaSuccess;
    const uint32_t p = fga::take_parakeet_tc_error(s, clear != 0, &err);
    const uint32_t z = fga::take_zipformer_tc_error(s, clear != 0, &err);
    const uint32_t v = fga::take_value_tc_error(s, clear != 0, &err);
    if (detail != nullptr) *detail = (p & 0xFFu) | ((z & 0xFFu) << 8) | ((v & 0xFFu) << 16);
    if (err != cudaSuccess) return FGA_ERROR_PRIOR_CUDA_ERROR;
    return (p | z | v) != 0u ? FGA_ERROR_DEVICE_ABORT : FGA_SUCCESS;
}

void fga_debug_set_wait_limit_ns(uint64_t limit_ns) { t_wait_limit_ns = limit_ns; }

// ---- parakeet -----------------------------------------------------------------------
int32_t fga_parakeet_relative_attention_check(const fga_tensor_desc* in, int32_t nin,
                                              const fga_tensor_desc* out, int32_t nout,
                                              float scale) {
    return check_parakeet(in, nin, out, nout, scale, nullptr);
}

size_t fga_parakeet_relative_attention_workspace_size(const fga_tensor_desc*, int32_t) {
    return 0;  // the fused kernel keeps scores on chip
}

int32_t fga_parakeet_relative_attention_enqueue(const fga_tensor_desc* in,
                                                const fga_tensor_desc* out,
                                                const void* const* inputs,
                                                void* const* outputs, float scale,
                                                void* /*workspace*/, size_t /*bytes*/,
                                                void* stream) {
    fga::ParakeetProblem p{};
    int32_t st = check_parakeet(in, 5, out, 1, scale, &p);
    if (st != FGA_SUCCESS) return st;
    if (inputs == nullptr || outputs == nullptr || outputs[0] == nullptr)
        return FGA_ERROR_NULL_POINTER;
    for (int i = 0; i < 5; ++i)
        if (inputs[i] == nullptr) return FGA_ERROR_NULL_POINTER;
    if ((st = prior_error_status()) != FGA_SUCCESS) return st;
    if (!fga::device_is_sm100()) return FGA_ERROR_NO_DEVICE;
    p.qkv = inputs[0];
    p.position = inputs[1];
    p.content_bias = inputs[2];
    p.position_bias = inputs[3];
    p.valid_lengths = static_cast<const int32_t*>(inputs[4]);
    p.output = outputs[0];
    const char* variant = "none";
    cudaError_t e = fga::launch_parakeet(p, static_cast<cudaStream_t>(stream), &variant);
    if (e != cudaSuccess) return FGA_ERROR_LAUNCH;
    t_last_variant = variant;
    return FGA_SUCCESS;
}

// ---- zipformer weights ----------------------------------------------------------------
int32_t fga_zipformer_relative_attention_check(const fga_tensor_desc* in, int32_t nin,
                                               const fga_tensor_desc* out, int32_t nout) {
    return check_zipformer(in, nin, out, nout, nullptr);
}

size_t fga_zipformer_relative_attention_workspace_size(const fga_tensor_desc*, int32_t) {
    return FGA_SCHED_WORKSPACE_BYTES;  // the tensor-core kernel's work counter
}

int32_t fga_zipformer_relative_attention_enqueue(const fga_tensor_desc* in,
                                                 const fga_tensor_desc* out,
                                                 const void* const* inputs,
                                                 void* const* outputs, void* workspace,
                                                 size_t workspace_bytes, void* stream) {
    fga::ZipformerWeightsProblem p{};
    int32_t st = check_zipformer(in, 3, out, 1, &p);
    if (st != FGA_SUCCESS) return st;
    if (inputs == nullptr || outputs == nullptr || outputs[0] == nullptr ||
        inputs[0] == nullptr || inputs[1] == nullptr || inputs[2] == nullptr)
        return FGA_ERROR_NULL_POINTER;
    if ((st = check_sched_workspace(workspace, workspace_bytes)) != FGA_SUCCESS) return st;
    if ((st = prior_error_status()) != FGA_SUCCESS) return st;
    if (!fga::device_is_sm100()) return FGA_ERROR_NO_DEVICE;
    p.projection = inputs[0];
    p.position = inputs[1];
    p.mask = static_cast<const uint8_t*>(inputs[2]);
    p.weights = outputs[0];
    p.sched = static_cast<unsigned int*>(workspace);
    const char* variant = "none";
    cudaError_t e =
        fga::launch_zipformer_weights(p, static_cast<cudaStream_t>(stream), &variant);
    if (e != cudaSuccess) return FGA_ERROR_LAUNCH;
    t_last_variant = variant;
    return FGA_SUCCESS;
}

// Same computation without a workspace: the work counter comes from a file-scope device
// array (FGA_NO_WORKSPACE_SCRATCH_BYTES) in the kernel's file, so nothing is allocated.
int32_t fga_zipformer_relative_attention_enqueue_no_workspace(const fga_tensor_desc* in,
                                                              const fga_tensor_desc* out,
                                                              const void* const* inputs,
                                                              void* const* outputs, void* stream) {
    fga::ZipformerWeightsProblem p{};
    int32_t st = check_zipformer(in, 3, out, 1, &p);
    if (st != FGA_SUCCESS) return st;
    if (inputs == nullptr || outputs == nullptr || outputs[0] == nullptr ||
        inputs[0] == nullptr || inputs[1] == nullptr || inputs[2] == nullptr)
        return FGA_ERROR_NULL_POINTER;
    // The scratch this problem needs must fit the fixed array.
    if (fga_zipformer_relative_attention_workspace_size(in, 3) > FGA_NO_WORKSPACE_SCRATCH_BYTES)
        return FGA_ERROR_WORKSPACE;
    if ((st = prior_error_status()) != FGA_SUCCESS) return st;
    if (!fga::device_is_sm100()) return FGA_ERROR_NO_DEVICE;
    void* scratch = nullptr;
    if (fga::no_workspace_scratch(&scratch) != cudaSuccess) return FGA_ERROR_LAUNCH;
    p.projection = inputs[0];
    p.position = inputs[1];
    p.mask = static_cast<const uint8_t*>(inputs[2]);
    p.weights = outputs[0];
    p.sched = static_cast<unsigned int*>(scratch);
    const char* variant = "none";
    cudaError_t e =
        fga::launch_zipformer_weights(p, static_cast<cudaStream_t>(stream), &variant);
    if (e != cudaSuccess) return FGA_ERROR_LAUNCH;
    t_last_variant = variant;
    return FGA_SUCCESS;
}

// ---- zipformer attention-value ----------------------------------------------------------
int32_t fga_zipformer_attention_value_check(const fga_tensor_desc* in, int32_t nin,
                                            const fga_tensor_desc* out, int32_t nout,
                                            int32_t num_heads) {
    return check_value(in, nin, out, nout, num_heads, nullptr);
}

size_t fga_zipformer_attention_value_workspace_size(const fga_tensor_desc*, int32_t, int32_t) {
    return 0;
}

int32_t fga_zipformer_attention_value_enqueue(const fga_tensor_desc* in,
                                              const fga_tensor_desc* out,
                                              const void* const* inputs, void* const* outputs,
                                              int32_t num_heads, void*, size_t, void* stream) {
    fga::ZipformerValueProblem p{};
    int32_t st = check_value(in, 2, out, 1, num_heads, &p);
    if (st != FGA_SUCCESS) return st;
    if (inputs == nullptr || outputs == nullptr || outputs[0] == nullptr ||
        inputs[0] == nullptr || inputs[1] == nullptr)
        return FGA_ERROR_NULL_POINTER;
    if ((st = prior_error_status()) != FGA_SUCCESS) return st;
    if (!fga::device_is_sm100()) return FGA_ERROR_NO_DEVICE;
    p.attention = inputs[0];
    p.value = inputs[1];
    p.output = outputs[0];
    const char* variant = "none";
    cudaError_t e = fga::launch_zipformer_value(p, static_cast<cudaStream_t>(stream), &variant);
    if (e != cudaSuccess) return FGA_ERROR_LAUNCH;
    t_last_variant = variant;
    return FGA_SUCCESS;
}

// ---- zipformer fused weights + attention-value -------------------------------------------
int32_t fga_zipformer_attention_fused_check(const fga_tensor_desc* in, int32_t nin,
                                            const fga_tensor_desc* out, int32_t nout) {
    return check_fused(in, nin, out, nout, nullptr);
}

size_t fga_zipformer_attention_fused_workspace_size(const fga_tensor_desc*, int32_t) {
    return FGA_SCHED_WORKSPACE_BYTES;  // the kernel's work counter
}

int32_t fga_zipformer_attention_fused_enqueue(const fga_tensor_desc* in,
                                              const fga_tensor_desc* out,
                                              const void* const* inputs, void* const* outputs,
                                              void* workspace, size_t workspace_bytes,
                                              void* stream) {
    fga::ZipformerFusedProblem p{};
    int32_t st = check_fused(in, 5, out, 3, &p);
    if (st != FGA_SUCCESS) return st;
    if (inputs == nullptr || outputs == nullptr) return FGA_ERROR_NULL_POINTER;
    for (int i = 0; i < 5; ++i)
        if (inputs[i] == nullptr) return FGA_ERROR_NULL_POINTER;
    for (int i = 0; i < 3; ++i)
        if (outputs[i] == nullptr) return FGA_ERROR_NULL_POINTER;
    if ((st = check_sched_workspace(workspace, workspace_bytes)) != FGA_SUCCESS) return st;
    if ((st = prior_error_status()) != FGA_SUCCESS) return st;
    if (!fga::device_is_sm100()) return FGA_ERROR_NO_DEVICE;
    p.projection = inputs[0];
    p.position = inputs[1];
    p.mask = static_cast<const uint8_t*>(inputs[2]);
    p.value1 = inputs[3];
    p.value2 = inputs[4];
    p.output1 = outputs[0];
    p.output2 = outputs[1];
    p.weights0 = outputs[2];
    p.sched = static_cast<unsigned int*>(workspace);
    const cudaError_t e = fga::launch_zipformer_fused(p, static_cast<cudaStream_t>(stream));
    if (e == cudaErrorNotSupported) return FGA_ERROR_UNSUPPORTED;  // buffer alignment
    if (e != cudaSuccess) return FGA_ERROR_LAUNCH;
    t_last_variant = "tcgen05";
    return FGA_SUCCESS;
}

// ---- depthwise convolutions ---------------------------------------------------------------

int32_t fga_parakeet_conformer_convolution_check(const fga_tensor_desc* in, int32_t nin,
                                                 const fga_tensor_desc* out, int32_t nout) {
    return check_convolution(in, nin, out, nout, fga::ConvolutionProblem::kParakeet, nullptr);
}

size_t fga_parakeet_conformer_convolution_workspace_size(const fga_tensor_desc*, int32_t) {
    return 0;
}

int32_t fga_parakeet_conformer_convolution_enqueue(const fga_tensor_desc* in,
                                                   const fga_tensor_desc* out,
                                                   const void* const* inputs,
                                                   void* const* outputs, void*, size_t,
                                                   void* stream) {
    return convolution_enqueue(in, out, inputs, outputs, fga::ConvolutionProblem::kParakeet,
                               stream);
}

int32_t fga_zipformer_convolution_check(const fga_tensor_desc* in, int32_t nin,
                                        const fga_tensor_desc* out, int32_t nout) {
    return check_convolution(in, nin, out, nout, fga::ConvolutionProblem::kZipformer, nullptr);
}

size_t fga_zipformer_convolution_workspace_size(const fga_tensor_desc*, int32_t) { return 0; }

int32_t fga_zipformer_convolution_enqueue(const fga_tensor_desc* in, const fga_tensor_desc* out,
                                          const void* const* inputs, void* const* outputs,
                                          void*, size_t, void* stream) {
    return convolution_enqueue(in, out, inputs, outputs, fga::ConvolutionProblem::kZipformer,
                               stream);
}

}  // extern "C"
