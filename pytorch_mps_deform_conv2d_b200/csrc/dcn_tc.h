// dcn_tc.h -- tcgen05 (5th-generation tensor core) kernels of libdcn_b200:
// TF32 operands staged in shared memory, fp32 accumulators in tensor memory.
#pragma once

#include <cuda_runtime.h>

#include "dcn_common.cuh"

namespace dcn {

// Whether the tensor-core forward covers this geometry.
bool tc_fwd_supported(const Geom& g);
// Bytes of the packed weight operand of the tensor-core forward.
size_t tc_fwd_weight_bytes(const Geom& g);
// weight (outC, Cg, kh, kw) -> packed tensor-core B operand.
cudaError_t launch_tc_pack_weight(const float* w, float* wt, const Geom& g,
                                  cudaStream_t stream);
// Forward on tcgen05: implicit GEMM whose A tiles are gathered (bilinear
// deformable sampling) by producer warps straight into swizzled shared memory.
cudaError_t launch_fwd_tc(const Geom& g, const float* xt, const float* wt,
                          const float* off, const float* mask, const float* bias,
                          float* out, int num_sms, cudaStream_t stream);

}  // namespace dcn
