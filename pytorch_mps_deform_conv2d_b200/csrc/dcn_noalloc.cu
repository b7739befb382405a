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
// up with cudaGetSymbolAddress (once per device and CUDA context, on the first
// call there) and that address is what the kernels get.
#include <cuda_runtime.h>

#include <cuda.h>
#include <cudaTypedefs.h>

#include <atomic>
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

// The array's address belongs to the CUDA context it was resolved in: the
// device's primary context normally, but a caller may run in a context of its
// own, and cudaDeviceReset replaces the primary context.  So each device's
// cached address is tagged with the unique ID of the context it was resolved
// in (cuCtxGetId, never reused within a process), and a call from any other
// context resolves it again.  Reading a cached address takes no lock.
struct ScratchSlot {
  std::atomic<unsigned long long> ctx_id{0};  // 0: nothing resolved yet
  std::atomic<void*> addr{nullptr};
};
ScratchSlot g_slots[kMaxDevices];
std::mutex g_setup_mu;

PFN_cuCtxGetCurrent_v4000 g_ctx_current = nullptr;
PFN_cuCtxGetId_v12000 g_ctx_id = nullptr;
std::once_flag g_ctx_once;

void resolve_ctx_queries() {
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
  if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn, cudaEnableDefault, &q) == cudaSuccess &&
      q == cudaDriverEntryPointSuccess)
    g_ctx_current = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(fn);
  fn = nullptr;
  if (cudaGetDriverEntryPoint("cuCtxGetId", &fn, cudaEnableDefault, &q) == cudaSuccess &&
      q == cudaDriverEntryPointSuccess)
    g_ctx_id = reinterpret_cast<PFN_cuCtxGetId_v12000>(fn);
  cudaGetLastError();
}

// Unique ID of the context current on this thread (0: none yet, or the
// driver cannot say -- then every call takes the resolving path).
unsigned long long current_ctx_id() {
  std::call_once(g_ctx_once, resolve_ctx_queries);
  if (g_ctx_current == nullptr || g_ctx_id == nullptr) return 0;
  CUcontext ctx = nullptr;
  if (g_ctx_current(&ctx) != CUDA_SUCCESS || ctx == nullptr) return 0;
  unsigned long long id = 0;
  if (g_ctx_id(ctx, &id) != CUDA_SUCCESS) return 0;
  return id;
}

int cuda_error(const char* what, int dev, cudaError_t e) {
  char msg[200];
  std::snprintf(msg, sizeof(msg), "dcn_forward_noalloc: %s failed on device %d: %s", what, dev,
                cudaGetErrorString(e));
  dcn::set_last_error(DCN_ERR_CUDA, msg);
  return DCN_ERR_CUDA;
}

// Device address of the scratch array in the current device's current
// context.  The first call per device (and per context) resolves it with
// cudaGetSymbolAddress, with that device current, which it is here.
int scratch_address(void** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_error("cudaGetDevice", dev, e);
  if (dev < 0 || dev >= kMaxDevices) {
    dcn::set_last_error(DCN_ERR_UNSUPPORTED, "dcn_forward_noalloc: device index beyond 63");
    return DCN_ERR_UNSUPPORTED;
  }
  ScratchSlot& slot = g_slots[dev];
  unsigned long long id = current_ctx_id();
  if (id != 0 && slot.ctx_id.load(std::memory_order_acquire) == id) {
    *out = slot.addr.load(std::memory_order_relaxed);
    return DCN_OK;
  }
  std::lock_guard<std::mutex> lk(g_setup_mu);
  void* p = nullptr;
  e = cudaGetSymbolAddress(&p, g_noalloc_scratch);  // makes a context current if none was
  if (e != cudaSuccess || p == nullptr)
    return cuda_error("cudaGetSymbolAddress of the scratch array", dev, e);
  if (id == 0) id = current_ctx_id();
  slot.addr.store(p, std::memory_order_relaxed);
  slot.ctx_id.store(id, std::memory_order_release);
  *out = p;
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
