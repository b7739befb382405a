// dcn_launch.cu -- host-side launch helpers (see dcn_launch.h).
#include "dcn_launch.h"

#include <atomic>
#include <map>
#include <mutex>
#include <utility>

namespace dcn {

namespace {
std::mutex g_attr_mu;
std::map<std::pair<const void*, int>, int> g_smem_set;  // (kernel, device) -> bytes
constexpr int kMaxDevices = 64;
std::atomic<int> g_sms[kMaxDevices] = {};
}  // namespace

cudaError_t ensure_dynamic_smem(const void* func, int bytes) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lk(g_attr_mu);
  int& cur = g_smem_set[{func, dev}];
  if (bytes <= cur) return cudaSuccess;
  e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) cur = bytes;
  return e;
}

int device_sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0) return 148;
  if (dev < kMaxDevices) {
    const int known = g_sms[dev].load(std::memory_order_relaxed);
    if (known > 0) return known;
  }
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0)
    sms = 148;
  if (dev < kMaxDevices) g_sms[dev].store(sms, std::memory_order_relaxed);
  return sms;
}

}  // namespace dcn
