// Host-side helpers shared by the tensor-core launchers: the driver's tensor-map encoder,
// per-device caches (SM count, the dynamic shared-memory attribute of each kernel), and the
// per-thread wait limit that the kernels' bounded waits receive as a parameter.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>

namespace fga {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// cuTensorMapEncodeTiled through the runtime's driver entry point (no -lcuda needed).
inline EncodeTiledFn encode_fn() {
    static const EncodeTiledFn fn = [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) !=
                cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return static_cast<EncodeTiledFn>(nullptr);
        return reinterpret_cast<EncodeTiledFn>(p);
    }();
    return fn;
}

// Devices with an ordinal below this get cached attributes; others query every call.
constexpr int kMaxCachedDevices = 64;

inline int current_device() {
    int dev = -1;
    return cudaGetDevice(&dev) == cudaSuccess ? dev : -1;
}

// Multiprocessor count of the current device (0 if it cannot be queried). Cached per
// device: a process may drive several GPUs, from several threads.
inline int sm_count() {
    static std::atomic<int> cache[kMaxCachedDevices];  // 0 = not yet known
    const int dev = current_device();
    if (dev < 0) return 0;
    if (dev < kMaxCachedDevices) {
        const int c = cache[dev].load(std::memory_order_relaxed);
        if (c > 0) return c;
    }
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
    if (dev < kMaxCachedDevices && n > 0) cache[dev].store(n, std::memory_order_relaxed);
    return n;
}

// cudaFuncSetAttribute(MaxDynamicSharedMemorySize) takes effect per device, so it is
// made once per (kernel, device). Two threads may both set it the first time; the call is
// idempotent, so that race is harmless.
class SmemAttr {
  public:
    cudaError_t ensure(const void* kernel, int bytes) {
        const int dev = current_device();
        if (dev < 0) return cudaErrorNoDevice;
        if (dev < kMaxCachedDevices && done_[dev].load(std::memory_order_acquire)) return cudaSuccess;
        const cudaError_t e =
            cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
        if (e == cudaSuccess && dev < kMaxCachedDevices)
            done_[dev].store(true, std::memory_order_release);
        return e;
    }

  private:
    std::atomic<bool> done_[kMaxCachedDevices] = {};
};

// Time limit of the Zipformer weights and fused kernels' bounded waits, in nanoseconds,
// for launches made by this host thread (fga_debug_set_wait_limit_ns; default 2 s).
uint64_t wait_limit_ns();

// Reads a kernel file's per-device `__device__ unsigned int` error word on `stream` (after
// the work already queued there) and, when `clear` is set and it is nonzero, zeroes it.
// The first CUDA error met is stored in *err (left unchanged on success).
template <typename Word>
uint32_t take_error_word(Word& word, cudaStream_t stream, bool clear, cudaError_t* err) {
    unsigned int v = 0;
    cudaError_t e =
        cudaMemcpyFromSymbolAsync(&v, word, sizeof(v), 0, cudaMemcpyDeviceToHost, stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
    if (e == cudaSuccess && clear && v != 0) {
        const unsigned int zero = 0;
        e = cudaMemcpyToSymbolAsync(word, &zero, sizeof(zero), 0, cudaMemcpyHostToDevice, stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
    }
    if (e != cudaSuccess && *err == cudaSuccess) *err = e;
    return e == cudaSuccess ? v : 0u;
}

}  // namespace fga
