// Kernel-variant selection. The tensor-core (tcgen05) kernels serve f16/bf16 inside
// their envelope; everything else runs on the SIMT kernels. There is no host path.
#include <cstdlib>
#include <cstring>

#include "fga_kernels.h"

namespace fga {

namespace {
// FGA_FORCE_SIMT=1 pins the SIMT kernels (used by tests that compare the two variants).
bool force_simt() {
    const char* v = std::getenv("FGA_FORCE_SIMT");
    return v != nullptr && std::strcmp(v, "1") == 0;
}
}  // namespace

bool device_is_sm100() {
    int dev = 0, major = 0, minor = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return false;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess)
        return false;
    return major == 10 && minor == 0;
}

cudaError_t launch_parakeet(const ParakeetProblem& p, cudaStream_t s, const char** variant) {
    if (!force_simt()) {
        cudaError_t e = launch_parakeet_tc(p, s);
        if (e != cudaErrorNotSupported) {
            *variant = "tcgen05";
            return e;
        }
    }
    *variant = "simt";
    return launch_parakeet_simt(p, s);
}

cudaError_t launch_zipformer_weights(const ZipformerWeightsProblem& p, cudaStream_t s,
                                     const char** variant) {
    if (!force_simt()) {
        cudaError_t e = launch_zipformer_weights_tc(p, s);
        if (e != cudaErrorNotSupported) {
            *variant = "tcgen05";
            return e;
        }
    }
    *variant = "simt";
    return launch_zipformer_weights_simt(p, s);
}

cudaError_t launch_zipformer_value(const ZipformerValueProblem& p, cudaStream_t s,
                                   const char** variant) {
    if (!force_simt()) {
        cudaError_t e = launch_zipformer_value_tc(p, s);
        if (e != cudaErrorNotSupported) {
            *variant = "tcgen05";
            return e;
        }
    }
    *variant = "simt";
    return launch_zipformer_value_simt(p, s);
}

}  // namespace fga
