// dcn_fwd_tc.cu -- tcgen05 forward (work in progress: not yet enabled).
#include "dcn_tc.h"

namespace dcn {

bool tc_fwd_supported(const Geom&) { return false; }
size_t tc_fwd_weight_bytes(const Geom&) { return 0; }
cudaError_t launch_tc_pack_weight(const float*, float*, const Geom&, cudaStream_t) {
  return cudaErrorNotSupported;
}
cudaError_t launch_fwd_tc(const Geom&, const float*, const float*, const float*, const float*,
                          const float*, float*, int, cudaStream_t) {
  return cudaErrorNotSupported;
}

}  // namespace dcn
