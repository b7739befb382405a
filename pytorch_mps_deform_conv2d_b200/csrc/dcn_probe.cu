// L2 <-> SM bandwidth probes: the denominators of the roofline that binds the
// gather / scatter kernels.  Both deformable-convolution passes move most of
// their bytes between L2 and the SMs, not between HBM and L2: every sample
// reads four 16-byte corner vectors per 4 channels (the forward's columns, the
// backward's coordinate gradient) and the backward adds four 16-byte
// reductions per sample into grad_input.  The probes run the same access
// kinds over an L2-resident buffer from every SM, so that the bytes a kernel
// moves (counted by ncu) divided by its time can be set against what this
// GPU sustains:
//   kind 0: 16-byte loads cached in L2 only (ld.global.cg), the corner gather;
//   kind 1: 16-byte fp32 reductions (red.global.add.v4.f32), the col2im scatter;
//   kind 2: both at once, 5 loads to 2 reductions in every thread's loop (the
//           fused backward moves 2.4 bytes in per byte reduced): whether the
//           two directions overlap or share one budget;
//   kind 3: 16-byte loads cached in L2 only from random 128-byte lines, 8
//           lanes to a line (4 lines a warp instruction): the access pattern
//           of the corner gathers, whose lines follow the sampling offsets;
//   kind 4: 16-byte fp32 reductions into random 128-byte lines, 8 lanes to a
//           line: the col2im scatter's pattern.
// No reference counterpart: the reference has no device kernels of this kind.
#include <cuda_runtime.h>

#include <cstdint>

#include "dcn_b200.h"

namespace {

constexpr int kProbeThreads = 512;
constexpr int kUnroll = 4;

// `passes` sweeps over buf (n16 16-byte vectors), four independent loads in
// flight per thread per step; the XOR of everything read decides one store,
// so the loads stay.
__global__ void __launch_bounds__(kProbeThreads)
    l2_read_probe_kernel(const int4* __restrict__ buf, long long n16, int passes, int* sink) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  const long long t0 = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  int acc = 0;
  for (int it = 0; it < passes; ++it) {
    long long i = t0;
    for (; i + (kUnroll - 1) * stride < n16; i += kUnroll * stride) {
      int4 v[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) v[u] = __ldcg(buf + i + u * stride);
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) acc ^= v[u].x ^ v[u].y ^ v[u].z ^ v[u].w;
    }
    for (; i < n16; i += stride) {
      const int4 v = __ldcg(buf + i);
      acc ^= v.x ^ v.y ^ v.z ^ v.w;
    }
  }
  if (acc == 0x13579bdf) sink[0] = acc;
}

// `passes` sweeps of 16-byte reductions over buf (n4 float4 slots); a warp
// covers 512 consecutive bytes per instruction (four 128-byte lines), as the
// col2im scatter of one corner and 32 channels does.
__global__ void __launch_bounds__(kProbeThreads)
    l2_red_probe_kernel(float* __restrict__ buf, long long n4, int passes) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  const long long t0 = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  for (int it = 0; it < passes; ++it)
    for (long long i = t0; i < n4; i += stride)
      asm volatile("red.global.add.v4.f32 [%0], {%1, %1, %1, %1};" ::"l"(buf + 4 * i),
                   "f"(1.0f)
                   : "memory");
}

// Kind 2: block b of a pass (one warp) loads vectors 160b .. 160b + 159 of
// the first 5/7 of buf and adds 1.0f to vectors 64b .. 64b + 63 of the last
// 2/7, 512 contiguous bytes an instruction.
__global__ void __launch_bounds__(kProbeThreads)
    l2_mixed_probe_kernel(int4* __restrict__ buf, long long blocks, int passes) {
  const long long wstride = (long long)gridDim.x * (blockDim.x >> 5);
  const long long w0 = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const int4* rd = buf;
  float* wr = reinterpret_cast<float*>(buf + 160 * blocks);
  int acc = 0;
  for (int it = 0; it < passes; ++it)
    for (long long b = w0; b < blocks; b += wstride) {
      int4 v[5];
#pragma unroll
      for (int u = 0; u < 5; ++u) v[u] = __ldcg(rd + 160 * b + 32 * u + lane);
#pragma unroll
      for (int u = 0; u < 2; ++u)
        asm volatile("red.global.add.v4.f32 [%0], {%1, %1, %1, %1};" ::"l"(
                         wr + 4 * (64 * b + 32 * u + lane)),
                     "f"(1.0f)
                     : "memory");
#pragma unroll
      for (int u = 0; u < 5; ++u) acc ^= v[u].x ^ v[u].y ^ v[u].z ^ v[u].w;
    }
  if (acc == 0x13579bdf) reinterpret_cast<int*>(buf)[0] = acc;
}

// Kind 3: `passes` x n16 16-byte loads; load j of a warp reads line
// mix(warp, j, lane / 8) % nlines, lanes 8i .. 8i + 7 its 16-byte pieces.
__device__ __forceinline__ uint32_t mix32(uint32_t x) {
  x ^= x >> 16;
  x *= 0x7feb352du;
  x ^= x >> 15;
  x *= 0x846ca68bu;
  x ^= x >> 16;
  return x;
}
// Line of load / reduction j of warp w in pass `it` (lanes 8i .. 8i + 7
// share line i of the four).
__device__ __forceinline__ long long probe_line(long long w, long long j, int lane, int it,
                                                long long nlines) {
  const uint32_t h = mix32((uint32_t)(w * 0x9e3779b1u) ^
                           mix32((uint32_t)j * 4u + (uint32_t)(lane >> 3) +
                                 (uint32_t)it * 0x85ebca6bu));
  return (long long)(h % (uint32_t)nlines);
}
__global__ void __launch_bounds__(kProbeThreads)
    l2_gather_probe_kernel(const int4* __restrict__ buf, long long n16, int passes, int* sink) {
  const long long nlines = n16 / 8;
  const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
  const long long w = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  // loads of one warp per pass: 4 lines (512 bytes) an instruction
  const long long per_warp = n16 / 32 / warps;
  int acc = 0;
  for (int it = 0; it < passes; ++it) {
    for (long long j = 0; j + kUnroll <= per_warp; j += kUnroll) {
      int4 v[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u)
        v[u] = __ldcg(buf + probe_line(w, j + u, lane, it, nlines) * 8 + (lane & 7));
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) acc ^= v[u].x ^ v[u].y ^ v[u].z ^ v[u].w;
    }
  }
  if (acc == 0x13579bdf) sink[0] = acc;
}

// Kind 4: as kind 3 with 16-byte reductions (adding 1.0f) instead of loads.
__global__ void __launch_bounds__(kProbeThreads)
    l2_scatter_probe_kernel(float* __restrict__ buf, long long n16, int passes) {
  const long long nlines = n16 / 8;
  const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
  const long long w = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const long long per_warp = n16 / 32 / warps;
  for (int it = 0; it < passes; ++it)
    for (long long j = 0; j + kUnroll <= per_warp; j += kUnroll)
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        float* dst = buf + (probe_line(w, j + u, lane, it, nlines) * 8 + (lane & 7)) * 4;
        asm volatile("red.global.add.v4.f32 [%0], {%1, %1, %1, %1};" ::"l"(dst), "f"(1.0f)
                     : "memory");
      }
}

}  // namespace

extern "C" DCN_API int dcn_l2_probe(int kind, void* buf, size_t bytes, int passes,
                                    void* stream) {
  if (kind < 0 || kind > 4 || buf == nullptr || passes < 1 || bytes < 16 ||
      (reinterpret_cast<uintptr_t>(buf) & 15) != 0)
    return DCN_ERR_INVALID_ARGUMENT;
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return DCN_ERR_CUDA;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const long long n16 = (long long)(bytes / 16);
  const int grid = sms * 4;  // 2048 threads an SM
  if (kind == 0) {
    // the sink is the buffer's first word: written only when the XOR of all
    // values read equals an arbitrary constant
    l2_read_probe_kernel<<<grid, kProbeThreads, 0, s>>>(static_cast<const int4*>(buf), n16,
                                                       passes, static_cast<int*>(buf));
  } else if (kind == 1) {
    l2_red_probe_kernel<<<grid, kProbeThreads, 0, s>>>(static_cast<float*>(buf), n16, passes);
  } else if (kind >= 3) {
    if (n16 / 8 > 0xffffffffLL || n16 / 32 < (long long)grid * (kProbeThreads / 32) * kUnroll)
      return DCN_ERR_INVALID_ARGUMENT;
    if (kind == 3)
      l2_gather_probe_kernel<<<grid, kProbeThreads, 0, s>>>(static_cast<const int4*>(buf), n16,
                                                           passes, static_cast<int*>(buf));
    else
      l2_scatter_probe_kernel<<<grid, kProbeThreads, 0, s>>>(static_cast<float*>(buf), n16,
                                                            passes);
  } else {
    if (n16 < 224) return DCN_ERR_INVALID_ARGUMENT;
    l2_mixed_probe_kernel<<<grid, kProbeThreads, 0, s>>>(static_cast<int4*>(buf), n16 / 224,
                                                        passes);
  }
  return cudaGetLastError() == cudaSuccess ? DCN_OK : DCN_ERR_CUDA;
}
