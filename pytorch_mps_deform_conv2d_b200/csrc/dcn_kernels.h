// dcn_kernels.h -- host-side launchers of the libdcn_b200 kernels.  Every
// launcher enqueues on `stream` and returns cudaGetLastError() of its launch;
// none allocates or synchronises.
#pragma once

#include <cuda_runtime.h>

#include "dcn_common.cuh"

namespace dcn {

// ---- layout kernels (dcn_layout.cu) --------------------------------------
// x (N, C, H, W) -> xt (N, H, W, C).  `zero_row`: also zeroes the C floats
// after xt (the zero pixel row the gathers read for dropped corners);
// `zero_like` (NULL or an (N, H, W, C) buffer) is zeroed in the same pass.
cudaError_t launch_nchw_to_nhwc(const float* x, float* xt, int N, int C, int HW,
                                bool zero_row, float* zero_like, cudaStream_t stream);
// 16-bit x (N, C, H, W) -> xt (N, H, W, C) (+ zero row when `zero_row`).
cudaError_t launch_nchw_to_nhwc_bf16(const void* x, void* xt, int N, int C, int HW, bool zero_row,
                                     cudaStream_t stream);
// Element-wise 16-bit (bf16, or fp16 with `f16`) <-> fp32 copies (round to
// nearest even on the way down).
cudaError_t launch_h16_to_f32(const void* in, float* out, long long n, bool f16,
                              cudaStream_t stream);
cudaError_t launch_f32_to_h16(const float* in, void* out, long long n, bool f16,
                              cudaStream_t stream);
// Channels-last x (N, H, W, C) copied to xt (+ zero row, + zeroed
// `zero_like` of the same size when not NULL).
cudaError_t launch_copy_nhwc(const float* x, float* xt, int N, int C, int HW, bool zero_row,
                             float* zero_like, cudaStream_t stream);
// gxt (N, H, W, C) -> gx (N, C, H, W)
cudaError_t launch_nhwc_to_nchw(const float* gxt, float* gx, int N, int C, int HW,
                                cudaStream_t stream);
// weight (outC, Cg, kk) -> wf[G][kk][cpad][Og] (forward SIMT operand,
// channels zero-padded to cpad)
cudaError_t launch_pack_weight_fwd(const float* w, float* wf, const Geom& g,
                                   int cpad, cudaStream_t stream);
// weight (outC, Cg, kk) -> wb[G][kk][Og][Cg] (grad-column operand)
cudaError_t launch_pack_weight_bwd(const float* w, float* wb, const Geom& g,
                                   cudaStream_t stream);
// out[n, o, p] = bias[o] (0 when bias is NULL); the C == 0 forward
cudaError_t launch_fill_bias(float* out, const float* bias, const Geom& g,
                             cudaStream_t stream);
// grad_bias[o] = sum_{n,p} grad_out[n, o, p] (written, not accumulated)
cudaError_t launch_grad_bias(const float* go, float* gb, const Geom& g,
                             cudaStream_t stream);
// Zeroes up to four fp32 buffers with one launch.
struct ZeroList {
  float* ptr[4];
  long long n[4];
  int count;
  void add(float* p, long long count_) {
    if (p != nullptr && count_ > 0) {
      ptr[count] = p;
      n[count] = count_;
      ++count;
    }
  }
};
cudaError_t launch_zero(const ZeroList& z, cudaStream_t stream);

// ---- fp32 SIMT kernels (dcn_simt.cu) --------------------------------------
// Forward, fp32 FFMA.  `xt` is the NHWC copy of the input.
cudaError_t launch_fwd_simt_gemm(const Geom& g, const float* xt, const float* wf,
                                 int cpad, const float* off, const float* mask,
                                 const float* bias, float* out, cudaStream_t stream);
cudaError_t launch_fwd_simt_direct(const Geom& g, const float* xt, const float* w,
                                   const float* off, const float* mask,
                                   const float* bias, float* out, cudaStream_t stream);
bool fwd_direct_supported(const Geom& g);
// Backward data path: grad_col = W^T go per tap, fused with the col2im
// scatter (into gxt, NHWC, pre-zeroed) and the coordinate / mask gradient
// reduction (into goff / gmask, pre-zeroed).
cudaError_t launch_bwd_data_simt(const Geom& g, const float* go, const float* wb,
                                 const float* xt, const float* off, const float* mask,
                                 float* gxt, float* goff, float* gmask,
                                 cudaStream_t stream);
// grad_weight (outC, Cg, kh, kw) += go . col^T, col gathered on the fly;
// `gw` pre-zeroed.
cudaError_t launch_bwd_weight_simt(const Geom& g, const float* go, const float* xt,
                                   const float* off, const float* mask, float* gw,
                                   int num_sms, cudaStream_t stream);

// Whole backward for small groups (out channels per group <= 8, in channels
// per group <= 16): grad-input scatter into gxt (NHWC), coordinate / mask
// gradients and grad_weight, all pre-zeroed accumulators.
bool bwd_small_supported(const Geom& g);
cudaError_t launch_bwd_small(const Geom& g, const float* go, const float* w, const float* xt,
                             const float* off, const float* mask, float* gxt, float* goff,
                             float* gmask, float* gw, cudaStream_t stream);

// Small convolution groups tiling a deformable group (dcn_dgroup.cu): one
// thread per (pixel, deformable group), 16-byte corner loads.  Covered:
// (Cg, Og) in {(1,1), (2,2), (4,4), (1,2), (2,4)} with 4, 8 or 16 channels
// per deformable group.  Forward writes `out`; backward accumulates into gxt
// (NHWC) and gw (pre-zeroed) and writes goff / gmask.
bool dgroup_supported(const Geom& g);
cudaError_t launch_fwd_dgroup(const Geom& g, const float* xt, const float* w, const float* off,
                              const float* mask, const float* bias, float* out,
                              cudaStream_t stream);
cudaError_t launch_bwd_dgroup(const Geom& g, const float* go, const float* w, const float* xt,
                              const float* off, const float* mask, float* gxt, float* goff,
                              float* gmask, float* gw, cudaStream_t stream);

// ---- single-image building blocks (dcn_debug_ops.cu) ----------------------
cudaError_t launch_col2im_single(const Geom& g, const float* col, const float* off,
                                 const float* mask, float* grad_im,
                                 cudaStream_t stream);
cudaError_t launch_col2im_coord_single(const Geom& g, const float* col,
                                       const float* im, const float* off,
                                       const float* mask, float* grad_off,
                                       float* grad_mask, cudaStream_t stream);

}  // namespace dcn
