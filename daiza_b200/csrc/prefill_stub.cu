// prefill_stub.cu -- placeholder launchers until the prefill kernels land.
#include "dz_internal.h"
namespace dz {
cudaError_t launch_gqa_prefill(dz_ctx*, int, int, int64_t, const uint16_t*, const uint16_t*, const uint16_t*,
                               const float*, const float*, const float*, float*, cudaStream_t, int*) {
    return cudaErrorNotSupported;
}
cudaError_t launch_gdn_prefill(dz_ctx*, int, int, int64_t, const float*, const float*, const float*, const float*,
                               float*, cudaStream_t, int*) {
    return cudaErrorNotSupported;
}
}  // namespace dz
