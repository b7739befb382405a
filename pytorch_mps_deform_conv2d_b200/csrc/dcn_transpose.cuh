// dcn_transpose.cuh -- one 64 x 64 tile of the 16-byte NCHW <-> NHWC
// transpose as a device function.  The transpose kernel runs one tile per
// block; the kernels that merge a transpose with other small jobs into one
// launch (the tensor-core forward's input staging + weight pack, the fused
// backward's grad-input transpose + grad_weight layout) run it for their
// transpose blocks.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace dcn {

// in (N, R, S) -> out (N, S, R): the tile of rows [64 by, 64 by + 64) and
// columns [64 bx, 64 bx + 64) of image n.  256 threads; R and S multiples of
// 4 and both buffers 16-byte aligned (transpose4_fits).  `tile` is 64 x 65
// floats of shared memory.  `zout` (NULL, or a buffer of the output's shape)
// is zeroed over the tile's output elements.
__device__ __forceinline__ void transpose4_tile(const float* __restrict__ in,
                                                float* __restrict__ out, int R, int S, int n,
                                                int bx, int by, float (*tile)[65],
                                                float* __restrict__ zout) {
  const int r0 = by * 64, s0 = bx * 64;
  const float* src = in + (long long)n * R * S;
  float* dst = out + (long long)n * R * S;
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = r0 + ty + 16 * i, s = s0 + tx * 4;
    if (r < R && s < S) {
      const float4 v = *reinterpret_cast<const float4*>(src + (long long)r * S + s);
      tile[ty + 16 * i][tx * 4 + 0] = v.x;
      tile[ty + 16 * i][tx * 4 + 1] = v.y;
      tile[ty + 16 * i][tx * 4 + 2] = v.z;
      tile[ty + 16 * i][tx * 4 + 3] = v.w;
    }
  }
  __syncthreads();
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int s = s0 + ty + 16 * i, r = r0 + tx * 4;
    if (s < S && r < R) {
      float4 v;
      v.x = tile[tx * 4 + 0][ty + 16 * i];
      v.y = tile[tx * 4 + 1][ty + 16 * i];
      v.z = tile[tx * 4 + 2][ty + 16 * i];
      v.w = tile[tx * 4 + 3][ty + 16 * i];
      *reinterpret_cast<float4*>(dst + (long long)s * R + r) = v;
      if (zout)
        *reinterpret_cast<float4*>(zout + (long long)n * R * S + (long long)s * R + r) =
            make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
}

// Whether transpose4_tile applies to an (N, R, S) transpose of these buffers.
inline bool transpose4_fits(const void* in, const void* out, int R, int S) {
  return R % 4 == 0 && S % 4 == 0 && (reinterpret_cast<uintptr_t>(in) & 15u) == 0 &&
         (reinterpret_cast<uintptr_t>(out) & 15u) == 0;
}

// 64 x 64 tiles of an (N, R, S) transpose: along S, per image, in all.
inline int transpose4_tiles_x(int S) { return (S + 63) / 64; }
inline long long transpose4_tiles(int N, int R, int S) {
  return (long long)N * ((S + 63) / 64) * ((R + 63) / 64);
}

}  // namespace dcn
