// dcn_debug_ops.cu -- single-image backward building blocks with the
// contracts of the reference's debug ops: deformable_col2im
// (deform_conv2d_mps.mm:388-504) and deformable_col2im_coord (:516-651).
// They take an explicit column-gradient buffer (C*kh*kw, Ho*Wo), row
// c*kh*kw + k, and exist to isolate the scatter and the coordinate reduction
// in tests.  The fused backward of dcn_simt.cu does not use them.
#include "dcn_kernels.h"

namespace dcn {

namespace {

// One thread per column element (c, k, p); scatter into grad_im (C, H, W),
// pre-zeroed.  Visits the live corners of the sample, which is the set the
// reference's +-2 window with the |delta| < 1 guard selects.
__global__ void col2im_single_kernel(Geom g, const float* __restrict__ col,
                                     const float* __restrict__ off,
                                     const float* __restrict__ mask,
                                     float* __restrict__ grad_im) {
  const long long total = (long long)g.C * g.kk * g.P;
  for (long long gid = blockIdx.x * (long long)blockDim.x + threadIdx.x; gid < total;
       gid += (long long)gridDim.x * blockDim.x) {
    const int p = (int)(gid % g.P);
    const int k = (int)((gid / g.P) % g.kk);
    const int c = (int)(gid / ((long long)g.P * g.kk));
    const int oy = p / g.Wo, ox = p - oy * g.Wo;
    const int ki = k / g.kw, kj = k - ki * g.kw;
    const int dgi = c / g.cpg;
    const long long oi = off_h_index(g, 0, dgi, k, p);
    float h, w;
    sample_pos(g, oy, ox, ki, kj, off[oi], off[oi + g.P], h, w);
    const Sample s = make_sample(h, w, g.H, g.W);
    if (!s.valid) continue;
    float top = col[gid];
    if (g.use_mask) top *= mask[mask_index(g, 0, dgi, k, p)];
    float* plane = grad_im + (long long)c * g.HW;
    if (s.live & 1u) atomicAdd(plane + s.i1, s.w1 * top);
    if (s.live & 2u) atomicAdd(plane + s.i2, s.w2 * top);
    if (s.live & 4u) atomicAdd(plane + s.i3, s.w3 * top);
    if (s.live & 8u) atomicAdd(plane + s.i4, s.w4 * top);
  }
}

// One thread per offset element (dgi, k, dir, p), looping over the channels
// of its deformable group; the mask gradient comes from the dir == 0 thread.
__global__ void col2im_coord_single_kernel(Geom g, const float* __restrict__ col,
                                           const float* __restrict__ im,
                                           const float* __restrict__ off,
                                           const float* __restrict__ mask,
                                           float* __restrict__ grad_off,
                                           float* __restrict__ grad_mask) {
  const long long total = 2LL * g.dg * g.kk * g.P;
  for (long long gid = blockIdx.x * (long long)blockDim.x + threadIdx.x; gid < total;
       gid += (long long)gridDim.x * blockDim.x) {
    const int p = (int)(gid % g.P);
    const int oc = (int)(gid / g.P);
    const int dgi = oc / (2 * g.kk);
    const int rem = oc - dgi * 2 * g.kk;
    const int dir = rem & 1, k = rem >> 1;
    const int oy = p / g.Wo, ox = p - oy * g.Wo;
    const int ki = k / g.kw, kj = k - ki * g.kw;
    const long long oi = off_h_index(g, 0, dgi, k, p);
    float h, w;
    sample_pos(g, oy, ox, ki, kj, off[oi], off[oi + g.P], h, w);
    const float m = g.use_mask ? mask[mask_index(g, 0, dgi, k, p)] : 1.f;
    const Sample s = make_sample(h, w, g.H, g.W);  // invalid == the -2 sentinel
    float val = 0.f, mval = 0.f;
    if (s.valid) {
      for (int ch = 0; ch < g.cpg; ++ch) {
        const int c = dgi * g.cpg + ch;
        const float* plane = im + (long long)c * g.HW;
        const float v1 = (s.live & 1u) ? plane[s.i1] : 0.f;
        const float v2 = (s.live & 2u) ? plane[s.i2] : 0.f;
        const float v3 = (s.live & 4u) ? plane[s.i3] : 0.f;
        const float v4 = (s.live & 8u) ? plane[s.i4] : 0.f;
        const float cv = col[((long long)c * g.kk + k) * g.P + p];
        const float cw = dir == 0 ? coord_dh(s, v1, v2, v3, v4) : coord_dw(s, v1, v2, v3, v4);
        val += m * cw * cv;
        if (g.use_mask && dir == 0) mval += cv * bilerp(s, v1, v2, v3, v4);
      }
    }
    grad_off[gid] = val;
    if (g.use_mask && dir == 0) grad_mask[mask_index(g, 0, dgi, k, p)] = mval;
  }
}

int grid_1d(long long total) {
  long long b = (total + 255) / 256;
  if (b > 148LL * 16) b = 148LL * 16;
  return (int)(b < 1 ? 1 : b);
}

}  // namespace

cudaError_t launch_col2im_single(const Geom& g, const float* col, const float* off,
                                 const float* mask, float* grad_im, cudaStream_t stream) {
  const long long total = (long long)g.C * g.kk * g.P;
  if (total == 0) return cudaSuccess;
  col2im_single_kernel<<<grid_1d(total), 256, 0, stream>>>(g, col, off, mask, grad_im);
  return cudaGetLastError();
}

cudaError_t launch_col2im_coord_single(const Geom& g, const float* col, const float* im,
                                       const float* off, const float* mask, float* grad_off,
                                       float* grad_mask, cudaStream_t stream) {
  const long long total = 2LL * g.dg * g.kk * g.P;
  if (total == 0) return cudaSuccess;
  col2im_coord_single_kernel<<<grid_1d(total), 256, 0, stream>>>(g, col, im, off, mask,
                                                                 grad_off, grad_mask);
  return cudaGetLastError();
}

}  // namespace dcn
