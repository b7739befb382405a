// dcn_launch.h -- host-side launch helpers shared by the kernel files.
#pragma once

#include <cuda_runtime.h>

namespace dcn {

// cudaFuncSetAttribute(MaxDynamicSharedMemorySize) once per (kernel, device)
// and size: later calls with the same or a smaller size return at once.
cudaError_t ensure_dynamic_smem(const void* func, int bytes);

// Multiprocessor count of the current device (queried once per device).
int device_sm_count();

}  // namespace dcn
