// Placeholder tensor-core launchers: report "not supported" so dispatch uses SIMT.
#include "fga_kernels.h"

namespace fga {
cudaError_t launch_zipformer_weights_tc(const ZipformerWeightsProblem&, cudaStream_t) {
    return cudaErrorNotSupported;
}
cudaError_t launch_zipformer_value_tc(const ZipformerValueProblem&, cudaStream_t) {
    return cudaErrorNotSupported;
}
}  // namespace fga
