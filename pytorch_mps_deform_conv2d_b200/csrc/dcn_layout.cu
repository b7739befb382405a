// dcn_layout.cu -- layout kernels around the deformable-convolution hot path:
// NCHW <-> NHWC transposes (the gathers and the scatter work on a
// channel-contiguous copy so one sample's channel vector is one run of
// 16-byte loads / vector reductions), weight repacking and the bias gradient.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "dcn_kernels.h"
#include "dcn_transpose.cuh"

namespace dcn {

namespace {

constexpr int TT = 32;  // transpose tile

// Extras of a transpose launch: `zout` (same shape as the output, or NULL)
// is zeroed tile by tile alongside; `tail` (NULL or `tail_n` floats) is
// zeroed by the first block.
struct TransposeExtras {
  float* zout;
  float* tail;
  int tail_n;
};

__device__ __forceinline__ void zero_tail(const TransposeExtras& ex) {
  if (ex.tail != nullptr && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0) {
    const int tid = threadIdx.y * blockDim.x + threadIdx.x;
    for (int i = tid; i < ex.tail_n; i += blockDim.x * blockDim.y) ex.tail[i] = 0.f;
  }
}

// in (N, R, S) -> out (N, S, R); one 32x32 tile per block, 32x8 threads.
__global__ void __launch_bounds__(256) transpose_kernel(const float* __restrict__ in,
                                                        float* __restrict__ out,
                                                        int R, int S, TransposeExtras ex) {
  __shared__ float tile[TT][TT + 1];
  zero_tail(ex);
  const int n = blockIdx.z;
  const int r0 = blockIdx.y * TT, s0 = blockIdx.x * TT;
  const float* src = in + (long long)n * R * S;
  float* dst = out + (long long)n * R * S;
  const int tx = threadIdx.x, ty = threadIdx.y;
#pragma unroll
  for (int i = 0; i < TT; i += 8) {
    const int r = r0 + ty + i, s = s0 + tx;
    if (r < R && s < S) tile[ty + i][tx] = src[(long long)r * S + s];
  }
  __syncthreads();
#pragma unroll
  for (int i = 0; i < TT; i += 8) {
    const int s = s0 + ty + i, r = r0 + tx;
    if (r < R && s < S) {
      dst[(long long)s * R + r] = tile[tx][ty + i];
      if (ex.zout) ex.zout[(long long)n * R * S + (long long)s * R + r] = 0.f;
    }
  }
}

// Same transpose with 64 x 64 tiles and 16-byte loads and stores; needs R and
// S multiples of 4 and 16-byte aligned buffers.
__global__ void __launch_bounds__(256) transpose4_kernel(const float* __restrict__ in,
                                                         float* __restrict__ out, int R, int S,
                                                         TransposeExtras ex) {
  __shared__ float tile[64][65];
  zero_tail(ex);
  transpose4_tile(in, out, R, S, blockIdx.z, blockIdx.x, blockIdx.y, tile, ex.zout);
}

cudaError_t launch_transpose(const float* in, float* out, int N, int R, int S,
                             const TransposeExtras& ex, cudaStream_t stream) {
  if ((long long)N * R * S == 0) {
    if (ex.tail != nullptr && ex.tail_n > 0)
      return cudaMemsetAsync(ex.tail, 0, (size_t)ex.tail_n * sizeof(float), stream);
    return cudaSuccess;
  }
  const bool vec = R % 4 == 0 && S % 4 == 0 && (reinterpret_cast<uintptr_t>(in) & 15u) == 0 &&
                   (reinterpret_cast<uintptr_t>(out) & 15u) == 0 &&
                   (reinterpret_cast<uintptr_t>(ex.zout) & 15u) == 0 && ceil_div(R, 64) <= 65535;
  if (vec) {
    dim3 grid(ceil_div(S, 64), ceil_div(R, 64), N);
    transpose4_kernel<<<grid, 256, 0, stream>>>(in, out, R, S, ex);
  } else {
    dim3 grid(ceil_div(S, TT), ceil_div(R, TT), N);
    transpose_kernel<<<grid, dim3(TT, 8), 0, stream>>>(in, out, R, S, ex);
  }
  return cudaGetLastError();
}

__global__ void pack_weight_fwd_kernel(const float* __restrict__ w,
                                       float* __restrict__ wf, Geom g, int cpad) {
  // wf[gi][k][c][o], c < cpad (zero beyond Cg)
  const long long total = (long long)g.G * g.kk * cpad * g.Og;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int o = (int)(i % g.Og);
    long long t = i / g.Og;
    const int c = (int)(t % cpad);
    t /= cpad;
    const int k = (int)(t % g.kk);
    const int gi = (int)(t / g.kk);
    float v = 0.f;
    if (c < g.Cg) v = w[((long long)(gi * g.Og + o) * g.Cg + c) * g.kk + k];
    wf[i] = v;
  }
}

__global__ void pack_weight_bwd_kernel(const float* __restrict__ w,
                                       float* __restrict__ wb, Geom g) {
  // wb[gi][k][o][c]
  const long long total = (long long)g.G * g.kk * g.Og * g.Cg;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int c = (int)(i % g.Cg);
    long long t = i / g.Cg;
    const int o = (int)(t % g.Og);
    t /= g.Og;
    const int k = (int)(t % g.kk);
    const int gi = (int)(t / g.kk);
    wb[i] = w[((long long)(gi * g.Og + o) * g.Cg + c) * g.kk + k];
  }
}

// grad_bias: block o sums grad_out[:, o, :] (16-byte loads when the rows
// allow it) and writes grad_bias[o]; no atomics, no pre-zeroing.
template <bool VEC>
__global__ void __launch_bounds__(256) grad_bias_kernel(const float* __restrict__ go,
                                                        float* __restrict__ gb, Geom g) {
  const int o = blockIdx.x;
  float s = 0.f;
  for (int n = 0; n < g.N; ++n) {
    const float* row = go + ((long long)n * g.outC + o) * g.P;
    if (VEC) {
      const float4* r4 = reinterpret_cast<const float4*>(row);
      for (int i = threadIdx.x; i < (g.P >> 2); i += blockDim.x) {
        const float4 v = __ldg(r4 + i);
        s += (v.x + v.y) + (v.z + v.w);
      }
    } else {
      for (int i = threadIdx.x; i < g.P; i += blockDim.x) s += __ldg(row + i);
    }
  }
  __shared__ float red[32];
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) s += __shfl_xor_sync(0xffffffffu, s, d);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    s = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) s += __shfl_xor_sync(0xffffffffu, s, d);
    if (threadIdx.x == 0) gb[o] = s;
  }
}

// Zeroes up to four buffers in one launch (16-byte stores where aligned).
__global__ void __launch_bounds__(256) zero_kernel(ZeroList z) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  const long long t0 = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  for (int b = 0; b < z.count; ++b) {
    float* p = z.ptr[b];
    const long long n = z.n[b];
    const long long n4 = (reinterpret_cast<uintptr_t>(p) & 15u) == 0 ? n >> 2 : 0;
    float4* p4 = reinterpret_cast<float4*>(p);
    for (long long i = t0; i < n4; i += stride) p4[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    for (long long i = (n4 << 2) + t0; i < n; i += stride) p[i] = 0.f;
  }
}

__global__ void fill_bias_kernel(float* __restrict__ out, const float* __restrict__ bias,
                                 Geom g) {
  const long long total = (long long)g.N * g.outC * g.P;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int o = (int)((i / g.P) % g.outC);
    out[i] = bias ? bias[o] : 0.f;
  }
}

int grid_for(long long total) {
  long long b = (total + 255) / 256;
  if (b > 148LL * 32) b = 148LL * 32;
  if (b < 1) b = 1;
  return (int)b;
}

}  // namespace

namespace {
// bf16 (as 16-bit words) in (N, R, S) -> out (N, S, R), 32 x 32 tiles; the
// first block also zeroes `tail_n` words at `tail`.
__global__ void __launch_bounds__(256) transpose16_kernel(const unsigned short* __restrict__ in,
                                                          unsigned short* __restrict__ out, int R,
                                                          int S, unsigned short* tail,
                                                          int tail_n) {
  __shared__ unsigned short tile[32][34];
  if (tail != nullptr && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0)
    for (int i = threadIdx.y * 32 + threadIdx.x; i < tail_n; i += 256) tail[i] = 0;
  const int n = blockIdx.z;
  const int r0 = blockIdx.y * 32, s0 = blockIdx.x * 32;
  const unsigned short* src = in + (long long)n * R * S;
  unsigned short* dst = out + (long long)n * R * S;
  const int tx = threadIdx.x, ty = threadIdx.y;
#pragma unroll
  for (int i = 0; i < 32; i += 8) {
    const int r = r0 + ty + i, s = s0 + tx;
    if (r < R && s < S) tile[ty + i][tx] = src[(long long)r * S + s];
  }
  __syncthreads();
#pragma unroll
  for (int i = 0; i < 32; i += 8) {
    const int s = s0 + ty + i, r = r0 + tx;
    if (r < R && s < S) dst[(long long)s * R + r] = tile[tx][ty + i];
  }
}

// 16-bit (bf16, or fp16 with `f16`) <-> fp32, element-wise; fp32 -> 16-bit
// rounds to nearest even.
__global__ void h16_to_f32_kernel(const unsigned short* __restrict__ in, float* __restrict__ out,
                                  long long n, int f16) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x)
    out[i] = f16 ? __half2float(__ushort_as_half(in[i])) : __uint_as_float((uint32_t)in[i] << 16);
}

__global__ void f32_to_h16_kernel(const float* __restrict__ in, unsigned short* __restrict__ out,
                                  long long n, int f16) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x)
    out[i] = f16 ? __half_as_ushort(__float2half_rn(in[i]))
                 : __bfloat16_as_ushort(__float2bfloat16_rn(in[i]));
}
}  // namespace

cudaError_t launch_nchw_to_nhwc_bf16(const void* x, void* xt, int N, int C, int HW, bool zero_row,
                                     cudaStream_t stream) {
  unsigned short* out = static_cast<unsigned short*>(xt);
  unsigned short* tail = zero_row ? out + (long long)N * HW * C : nullptr;
  if ((long long)N * C * HW == 0) {
    if (tail != nullptr && C > 0) return cudaMemsetAsync(tail, 0, (size_t)C * 2, stream);
    return cudaSuccess;
  }
  if (ceil_div(C, 32) > 65535 || N > 65535) return cudaErrorInvalidValue;
  dim3 grid(ceil_div(HW, 32), ceil_div(C, 32), N);
  transpose16_kernel<<<grid, dim3(32, 8), 0, stream>>>(static_cast<const unsigned short*>(x), out,
                                                       C, HW, tail, C);
  return cudaGetLastError();
}

cudaError_t launch_h16_to_f32(const void* in, float* out, long long n, bool f16,
                              cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  h16_to_f32_kernel<<<grid_for(n), 256, 0, stream>>>(static_cast<const unsigned short*>(in), out,
                                                     n, f16 ? 1 : 0);
  return cudaGetLastError();
}

cudaError_t launch_f32_to_h16(const float* in, void* out, long long n, bool f16,
                              cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  f32_to_h16_kernel<<<grid_for(n), 256, 0, stream>>>(in, static_cast<unsigned short*>(out), n,
                                                     f16 ? 1 : 0);
  return cudaGetLastError();
}

cudaError_t launch_nchw_to_nhwc(const float* x, float* xt, int N, int C, int HW,
                                bool zero_row, float* zero_like, cudaStream_t stream) {
  TransposeExtras ex{zero_like, zero_row ? xt + (long long)N * HW * C : nullptr, C};
  return launch_transpose(x, xt, N, C, HW, ex, stream);
}

namespace {
// Channels-last input: a straight copy into the workspace copy (16-byte
// accesses when aligned), the C floats after it zeroed, and `zero_like` (the
// grad-input accumulator, or NULL) zeroed in the same pass.
__global__ void __launch_bounds__(256) copy_nhwc_kernel(const float* __restrict__ x,
                                                        float* __restrict__ xt, long long n,
                                                        int C, int zero_row,
                                                        float* __restrict__ zero_like, int vec) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  const long long t0 = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  if (vec) {
    const float4* s4 = reinterpret_cast<const float4*>(x);
    float4* d4 = reinterpret_cast<float4*>(xt);
    float4* z4 = reinterpret_cast<float4*>(zero_like);
    for (long long i = t0; i < n / 4; i += stride) {
      d4[i] = __ldg(s4 + i);
      if (zero_like) z4[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  } else {
    for (long long i = t0; i < n; i += stride) {
      xt[i] = __ldg(x + i);
      if (zero_like) zero_like[i] = 0.f;
    }
  }
  if (zero_row && blockIdx.x == 0)
    for (int c = threadIdx.x; c < C; c += blockDim.x) xt[n + c] = 0.f;
}
}  // namespace

cudaError_t launch_copy_nhwc(const float* x, float* xt, int N, int C, int HW, bool zero_row,
                             float* zero_like, cudaStream_t stream) {
  const long long n = (long long)N * HW * C;
  if (n == 0 && !(zero_row && C > 0)) return cudaSuccess;
  const int vec = n % 4 == 0 && (reinterpret_cast<uintptr_t>(x) & 15u) == 0 &&
                  (reinterpret_cast<uintptr_t>(xt) & 15u) == 0 &&
                  (reinterpret_cast<uintptr_t>(zero_like) & 15u) == 0;
  long long blocks = ((vec ? n / 4 : n) + 255) / 256;
  if (blocks > 148LL * 16) blocks = 148LL * 16;
  if (blocks < 1) blocks = 1;
  copy_nhwc_kernel<<<(int)blocks, 256, 0, stream>>>(x, xt, n, C, zero_row ? 1 : 0, zero_like, vec);
  return cudaGetLastError();
}

cudaError_t launch_nhwc_to_nchw(const float* gxt, float* gx, int N, int C, int HW,
                                cudaStream_t stream) {
  return launch_transpose(gxt, gx, N, HW, C, TransposeExtras{nullptr, nullptr, 0}, stream);
}

cudaError_t launch_zero(const ZeroList& z, cudaStream_t stream) {
  long long most = 0;
  for (int b = 0; b < z.count; ++b) most = z.n[b] > most ? z.n[b] : most;
  if (most == 0) return cudaSuccess;
  long long blocks = (most / 4 + 255) / 256;
  if (blocks > 148LL * 8) blocks = 148LL * 8;
  if (blocks < 1) blocks = 1;
  zero_kernel<<<(int)blocks, 256, 0, stream>>>(z);
  return cudaGetLastError();
}

cudaError_t launch_pack_weight_fwd(const float* w, float* wf, const Geom& g, int cpad,
                                   cudaStream_t stream) {
  const long long total = (long long)g.G * g.kk * cpad * g.Og;
  if (total == 0) return cudaSuccess;
  pack_weight_fwd_kernel<<<grid_for(total), 256, 0, stream>>>(w, wf, g, cpad);
  return cudaGetLastError();
}

cudaError_t launch_pack_weight_bwd(const float* w, float* wb, const Geom& g,
                                   cudaStream_t stream) {
  const long long total = (long long)g.G * g.kk * g.Og * g.Cg;
  if (total == 0) return cudaSuccess;
  pack_weight_bwd_kernel<<<grid_for(total), 256, 0, stream>>>(w, wb, g);
  return cudaGetLastError();
}

cudaError_t launch_fill_bias(float* out, const float* bias, const Geom& g,
                             cudaStream_t stream) {
  const long long total = (long long)g.N * g.outC * g.P;
  if (total == 0) return cudaSuccess;
  fill_bias_kernel<<<grid_for(total), 256, 0, stream>>>(out, bias, g);
  return cudaGetLastError();
}

cudaError_t launch_grad_bias(const float* go, float* gb, const Geom& g,
                             cudaStream_t stream) {
  if (g.outC == 0) return cudaSuccess;
  if ((long long)g.N * g.P == 0)
    return cudaMemsetAsync(gb, 0, (size_t)g.outC * sizeof(float), stream);
  const bool vec = (g.P % 4 == 0) && ((reinterpret_cast<uintptr_t>(go) & 15u) == 0);
  dim3 grid(g.outC);
  if (vec)
    grad_bias_kernel<true><<<grid, 256, 0, stream>>>(go, gb, g);
  else
    grad_bias_kernel<false><<<grid, 256, 0, stream>>>(go, gb, g);
  return cudaGetLastError();
}
}  // namespace dcn
