// gdn_prefill.cu -- placeholder until the chunked Gated DeltaNet prefill lands.
#include "dz_internal.h"
namespace dz {
cudaError_t launch_gdn_prefill(dz_ctx*, int, int, int64_t, const float*, const float*, const float*, const float*,
                               float*, cudaStream_t, int*) {
    return cudaErrorNotSupported;
}
}  // namespace dz
