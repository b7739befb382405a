// dcn_common.cuh -- geometry, sampling descriptors and small device helpers
// shared by every deformable-convolution kernel of libdcn_b200.
//
// Sampling semantics follow the reference's bilinear helpers exactly
// (src/deform_conv2d_mps/_C/bilinear.metalh:13-99): a sample is dropped
// entirely when h <= -1 || h >= H || w <= -1 || w >= W; otherwise each of the
// four corners (floor/floor+1) contributes only when it lies inside the image.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace dcn {

// Kernel parameter block (the reference passes DeformConvParams,
// deform_conv2d.metal:53-65).  Per-image element counts are checked on the
// host to fit in int32; cross-image offsets are formed in int64.
struct Geom {
  int N, C, H, W;      // input (N, C, H, W)
  int outC, kh, kw;    // weight (outC, C/G, kh, kw)
  int sh, sw, ph, pw, dh, dw;
  int G, dg;           // groups, deformable groups
  int Ho, Wo;
  int use_mask, use_bias;
  int mask_logits;     // the mask tensor holds logits: mask = sigmoid(stored)
  int oy0;             // full-output row of local output row 0 (row windows)
  // derived
  int Cg, Og;          // channels per group (in / out)
  int cpg;             // channels per deformable group
  int kk;              // kh * kw
  int P;               // Ho * Wo
  int HW;              // H * W
  long long NP;        // N * P
  // tensor-core kernels: SM clock cycles one mbarrier wait may take before
  // the CTA gives up (raises its error word and leaves), and a test switch
  // under which their TMA producers issue nothing, so that the waits run out
  long long wait_limit;
  int no_async;
};

// Bilinear sampling plan of one (pixel, tap, deformable group): the four
// corner positions (spatial index y*W+x, 0 when the corner is dropped), their
// bilinear weights (0 when dropped) and a bit per live corner (bit j-1 for
// corner j; a live corner can still have weight 0 when the sample sits on the
// grid, and the coordinate gradient needs its value).  `lh`/`lw` are the
// fractional parts.  `valid` is false when the whole sample is out of range.
struct Sample {
  int i1, i2, i3, i4;
  float w1, w2, w3, w4;
  float lh, lw;
  unsigned live;
  bool valid;
};

__device__ __forceinline__ Sample make_sample(float h, float w, int H, int W) {
  Sample s;
  if (h <= -1.f || (float)H <= h || w <= -1.f || (float)W <= w) {
    s.i1 = s.i2 = s.i3 = s.i4 = 0;
    s.w1 = s.w2 = s.w3 = s.w4 = 0.f;
    s.lh = s.lw = 0.f;
    s.live = 0u;
    s.valid = false;
    return s;
  }
  const int hl = (int)floorf(h), wl = (int)floorf(w);
  const int hh_i = hl + 1, wh_i = wl + 1;
  const float lh = h - (float)hl, lw = w - (float)wl;
  const float hh = 1.f - lh, hw = 1.f - lw;
  const bool y0 = hl >= 0, y1 = hh_i <= H - 1, x0 = wl >= 0, x1 = wh_i <= W - 1;
  s.i1 = (y0 && x0) ? hl * W + wl : 0;
  s.i2 = (y0 && x1) ? hl * W + wh_i : 0;
  s.i3 = (y1 && x0) ? hh_i * W + wl : 0;
  s.i4 = (y1 && x1) ? hh_i * W + wh_i : 0;
  s.w1 = (y0 && x0) ? hh * hw : 0.f;
  s.w2 = (y0 && x1) ? hh * lw : 0.f;
  s.w3 = (y1 && x0) ? lh * hw : 0.f;
  s.w4 = (y1 && x1) ? lh * lw : 0.f;
  s.lh = lh;
  s.lw = lw;
  s.live = (y0 && x0 ? 1u : 0u) | (y0 && x1 ? 2u : 0u) | (y1 && x0 ? 4u : 0u) |
           (y1 && x1 ? 8u : 0u);
  s.valid = true;
  return s;
}

// Sampling position of tap (ki, kj) for output pixel (oy, ox) and its
// offset pair; index math of deform_conv2d.metal:100-113.
__device__ __forceinline__ void sample_pos(const Geom& g, int oy, int ox,
                                           int ki, int kj, float off_h,
                                           float off_w, float& h, float& w) {
  h = (float)((oy + g.oy0) * g.sh - g.ph + ki * g.dh) + off_h;
  w = (float)(ox * g.sw - g.pw + kj * g.dw) + off_w;
}

// Offset / mask element addresses for image n, deformable group dgi, tap k,
// output pixel p (offset channels interleave (h, w) per tap:
// deform_conv2d.metal:107-108, mask :118).
__device__ __forceinline__ long long off_h_index(const Geom& g, int n, int dgi, int k, int p) {
  return ((long long)n * 2 * g.dg * g.kk + 2 * (dgi * g.kk + k)) * g.P + p;
}
__device__ __forceinline__ long long mask_index(const Geom& g, int n, int dgi, int k, int p) {
  return ((long long)n * g.dg * g.kk + (dgi * g.kk + k)) * g.P + p;
}

// Mask value of one (image, deformable group, tap, pixel): the stored value,
// or sigmoid(stored) when the mask tensor holds logits (a DCNv2 block feeding
// the raw output of its mask convolution); 1 without a mask (DCNv1).
__device__ __forceinline__ float mask_of(const Geom& g, const float* __restrict__ mask,
                                         long long i) {
  if (!g.use_mask) return 1.f;
  const float v = __ldg(mask + i);
  return g.mask_logits ? 1.f / (1.f + expf(-v)) : v;
}
// d(mask) / d(stored value): 1, or sigmoid'(x) = m (1 - m) for logits.
__device__ __forceinline__ float mask_grad_scale(const Geom& g, float m) {
  return g.mask_logits ? m * (1.f - m) : 1.f;
}

// Vector reduction into global memory (sm_90+): four consecutive fp32
// values in one L2 atomic transaction.  `addr` must be 16-byte aligned.
__device__ __forceinline__ void red_add_v4(float* addr, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};"
               :: "l"(addr), "f"(a), "f"(b), "f"(c), "f"(d) : "memory");
}
__device__ __forceinline__ void red_add_f32(float* addr, float a) {
  asm volatile("red.global.add.f32 [%0], %1;" :: "l"(addr), "f"(a) : "memory");
}

__device__ __forceinline__ float4 ldg4(const float* p) {
  return __ldg(reinterpret_cast<const float4*>(p));
}

// Forward bilinear value from the four corner values (dead corners carry 0):
// bilinear.metalh:36-37.
__device__ __forceinline__ float bilerp(const Sample& s, float v1, float v2,
                                        float v3, float v4) {
  return s.w1 * v1 + s.w2 * v2 + s.w3 * v3 + s.w4 * v4;
}
// d(bilinear)/dh and d(bilinear)/dw: bilinear.metalh:94-98.
__device__ __forceinline__ float coord_dh(const Sample& s, float v1, float v2,
                                          float v3, float v4) {
  return (1.f - s.lw) * (v3 - v1) + s.lw * (v4 - v2);
}
__device__ __forceinline__ float coord_dw(const Sample& s, float v1, float v2,
                                          float v3, float v4) {
  return (1.f - s.lh) * (v2 - v1) + s.lh * (v4 - v3);
}

__host__ __device__ __forceinline__ int ceil_div(int a, int b) { return (a + b - 1) / b; }

}  // namespace dcn
