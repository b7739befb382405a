// dcn_noalloc.cu -- a forward entry point that allocates nothing.
//
// dcn_forward needs scratch memory (the NHWC copy of the input and the packed
// weight) and takes it from the caller.  Some callers cannot produce that
// buffer: code that runs inside a memory pool's or allocator's own hooks (a
// cudaMalloc there would re-enter the allocator), plugins of host frameworks
// that only ever hand out input and output buffers, and deployments whose
// device memory is fixed at start-up so that no allocation may happen on the
// serving path.  dcn_forward_noalloc serves them from a fixed scratch array
// that is part of the library image itself.
//
// The array is a file-scope __device__ variable, so it is created together
// with this module's code on every GPU that loads the library and stays there
// until the process exits.  In host code its name is only a stand-in for the
// symbol, not a device address: its address on the current device is looked
// up with cudaGetSymbolAddress (once per device, on the first call there) and
// that address is what the kernels get.
#include <cuda_runtime.h>

#include <cstdio>
#include <mutex>

#include "dcn_b200.h"

namespace dcn {
void set_last_error(int code, const char* msg);                    // dcn_capi.cu
size_t forward_min_workspace(const dcn_shape* s, uint32_t flags);  // dcn_capi.cu
}

namespace {

// Upper bound of the scratch one call may use (the least workspace
// dcn_forward accepts for the call's shape must not exceed it): 16 MiB, e.g. a
// 2x64x128x128 input.  Whatever is left over serves as the optional scratch of
// the tensor-core forward's split last round where it fits.
constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_setup_mu;
void* g_scratch_addr[kMaxDevices] = {};

// Device address of the scratch array on the current device; the first call
// per device resolves it (with that device current, which it is here).
int scratch_address(void** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    char msg[160];
    std::snprintf(msg, sizeof(msg), "dcn_forward_noalloc: cudaGetDevice failed: %s",
                  cudaGetErrorString(e));
    dcn::set_last_error(DCN_ERR_CUDA, msg);
    return DCN_ERR_CUDA;
  }
  if (dev < 0 || dev >= kMaxDevices) {
    dcn::set_last_error(DCN_ERR_UNSUPPORTED, "dcn_forward_noalloc: device index beyond 63");
    return DCN_ERR_UNSUPPORTED;
  }
  std::lock_guard<std::mutex> lk(g_setup_mu);
  if (g_scratch_addr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      char msg[200];
      std::snprintf(msg, sizeof(msg),
                    "dcn_forward_noalloc: cudaGetSymbolAddress of the scratch array failed on "
                    "device %d: %s",
                    dev, cudaGetErrorString(e));
      dcn::set_last_error(DCN_ERR_CUDA, msg);
      return DCN_ERR_CUDA;
    }
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return DCN_OK;
}

}  // namespace

extern "C" DCN_API int dcn_forward_noalloc(const dcn_shape* shape, const float* input,
                                           const float* weight, const float* offset,
                                           const float* mask, const float* bias, float* output,
                                           uint32_t flags, void* stream) {
  int64_t ho = 0, wo = 0;
  int rc = dcn_output_size(shape, &ho, &wo);  // validates the geometry, sets the message
  if (rc != DCN_OK) return rc;
  const size_t need = dcn::forward_min_workspace(shape, flags);
  if (need > kNoAllocScratchBytes) {
    char msg[256];
    std::snprintf(msg, sizeof(msg),
                  "dcn_forward_noalloc: this shape needs %zu bytes of scratch, more than the "
                  "%zu bytes built into the library; call dcn_forward with a workspace instead",
                  need, kNoAllocScratchBytes);
    dcn::set_last_error(DCN_ERR_WORKSPACE, msg);
    return DCN_ERR_WORKSPACE;
  }
  void* scratch = nullptr;
  rc = scratch_address(&scratch);
  if (rc != DCN_OK) return rc;
  return dcn_forward(shape, input, weight, offset, mask, bias, output, flags, scratch,
                     kNoAllocScratchBytes, stream);
}
