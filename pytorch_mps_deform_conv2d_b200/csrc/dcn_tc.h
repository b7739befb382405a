// dcn_tc.h -- tcgen05 (5th-generation tensor core) kernels of libdcn_b200:
// TF32 operands staged in shared memory, fp32 accumulators in tensor memory.
#pragma once

#include <cuda_runtime.h>

#include "dcn_common.cuh"

namespace dcn {
struct ZeroList;  // dcn_kernels.h

// Error words of the tensor-core kernels (a bit per kernel family whose
// bounded mbarrier wait ran out: kStatusFwd, kStatusBwdData,
// kStatusBwdWeight), read after the work already on `stream` (the host
// waits for it) and cleared when `clear` is set.
constexpr int kStatusFwd = 0x1, kStatusBwdData = 0x2, kStatusBwdWeight = 0x4;
cudaError_t read_fwd_status(int* status, bool clear, cudaStream_t stream);
cudaError_t read_bwd_status(int* status, bool clear, cudaStream_t stream);
// Cycles a wait of the tensor-core kernels may take before it gives up
// (~2 s at 1.9 GHz), and the short budget of the timeout test switch.
constexpr long long kWaitLimit = 4000000000LL;
constexpr long long kTestWaitLimit = 2000000LL;

// Whether the tensor-core forward covers this geometry.
bool tc_fwd_supported(const Geom& g);
// Bytes of the packed weight operand of the tensor-core forward (`split`:
// high and low TF32 parts, for 3xTF32).
size_t tc_fwd_weight_bytes(const Geom& g, bool split);
// Scratch ("tail") with which the tensor-core forward splits a short last
// round of tiles over all SMs (0 when this shape has none on `num_sms` SMs;
// `h16`: the 16-bit forward): the pieces' partial sums, which a second
// launch adds.  Without the scratch the forward runs whole tiles only.
size_t tc_fwd_tail_bytes(const Geom& g, bool split, bool h16, int num_sms);
// weight (outC, Cg, kh, kw) -> packed tensor-core B operand.
cudaError_t launch_tc_pack_weight(const float* w, float* wt, const Geom& g, bool split,
                                  cudaStream_t stream);
// The NCHW input's NHWC staging copy (with its zero pixel row) and the
// packed weight of launch_tc_pack_weight in one launch.  Needs C and HW
// multiples of 4 and 16-byte aligned x / xt (fwd_prologue_fits); else
// cudaErrorInvalidValue, and the two separate launches apply.
bool fwd_prologue_fits(const float* x, const float* xt, const Geom& g);
cudaError_t launch_fwd_prologue(const float* x, float* xt, const float* w, float* wt,
                                const Geom& g, bool split, cudaStream_t stream);
// Forward on tcgen05: implicit GEMM whose A tiles are gathered (bilinear
// deformable sampling) by producer warps straight into swizzled shared memory.
// `split`: 3xTF32 (fp32-level accuracy).  `tail` / `tail_bytes`: the scratch
// of tc_fwd_tail_bytes (NULL: whole tiles only).
cudaError_t launch_fwd_tc(const Geom& g, const float* xt, const float* wt,
                          const float* off, const float* mask, const float* bias,
                          float* out, bool split, void* tail, size_t tail_bytes, int num_sms,
                          cudaStream_t stream);

// 16-bit forward (all tensors bf16, or all fp16 with `f16`; kind::f16 UMMAs,
// fp32 accumulation): 64 channels of a tap per K step, so channels per group
// and per deformable group must be multiples of 64.  `xt` is the 16-bit NHWC
// copy with its zero row, `wt` the packed 16-bit weight
// (tc_fwd_weight_bf16_bytes).
bool tc_fwd_bf16_supported(const Geom& g);
size_t tc_fwd_weight_bf16_bytes(const Geom& g);
cudaError_t launch_tc_pack_weight_bf16(const void* w, void* wt, const Geom& g,
                                       cudaStream_t stream);
cudaError_t launch_fwd_tc_bf16(const Geom& g, const void* xt, const void* wt, const void* off,
                               const void* mask, const void* bias, void* out, bool f16,
                               void* tail, size_t tail_bytes, int num_sms,
                               cudaStream_t stream);

// Whether the tensor-core backward covers this geometry (grad-column kernel
// and the column-buffer weight gradient), and whether the gather-based
// weight-gradient kernel does too (128-channel multiples only).
bool tc_bwd_supported(const Geom& g);
bool tc_wgather_supported(const Geom& g);
// go -> go_r (NCHW, rows padded to Ppad = P rounded up to 4, tf32-rounded);
// with `split` (3xTF32) the low TF32 parts follow in rows N*outC ...  `gb`
// (NULL or grad_bias, zeroed by the caller) also receives the bias gradient.
cudaError_t launch_tc_prep_go(const Geom& g, const float* go, float* go_r, float* gb,
                              bool split, cudaStream_t stream);
cudaError_t launch_tc_pack_weight_bwd(const float* w, float* wbt, const Geom& g, bool split,
                                      cudaStream_t stream);
// grad_col = W^T go on the tensor core per (pixel tile, tap), fused with the
// col2im scatter into gxt (NHWC, pre-zeroed) and the coordinate / mask
// reductions into goff / gmask (pre-zeroed).  `go_r` as written by
// launch_tc_prep_go; `split` selects 3xTF32 (wbt then holds high and low
// parts).  `col` non-NULL: also writes the column buffer (tc_col_bytes) that
// launch_bwd_weight_col reads.
cudaError_t launch_bwd_data_tc(const Geom& g, const float* go_r, bool split, const float* wbt,
                               const float* xt, const float* off, const float* mask, float* gxt,
                               float* goff, float* gmask, float* col, cudaStream_t stream);
// The fused TF32 backward (out channels per group <= 256): the grad-column
// GEMM with the col2im scatter into gxt and the coordinate / mask reductions
// into goff / gmask (as launch_bwd_data_tc), and the weight gradient from the
// column tiles it samples on chip, summed into `gwt`, the tap-major
// [outC][kh*kw][Cg] copy of grad_weight (pre-zeroed).  No column buffer.
bool tc_fused_supported(const Geom& g);
cudaError_t launch_bwd_fused_tc(const Geom& g, const float* go_r, const float* wbt,
                                const float* xt, const float* off, const float* mask, float* gxt,
                                float* goff, float* gmask, float* gwt, int num_sms,
                                cudaStream_t stream);
// The fused backward for bf16 / fp16 tensors (`f16`): kind::f16 UMMAs with
// the tensors' 16-bit type, 16-bit gathers and column values, fp32
// accumulation and fp32 reductions into gxt, goff, gmask, gwt (pre-zeroed,
// fp32).  `xt`: the 16-bit NHWC copy with its zero row; `go_r`: the 16-bit
// grad_out rows padded to a multiple of 8 pixels (launch_prep_go16); `wbt`:
// the 16-bit packed weight (launch_pack_weight_bwd16).  Needs C % 8 == 0.
bool tc_fused16_supported(const Geom& g);
cudaError_t launch_bwd_fused_tc_h16(const Geom& g, const void* go_r, const void* wbt,
                                    const void* xt, const void* off, const void* mask,
                                    float* gxt, float* goff, float* gmask, float* gwt, bool f16,
                                    int num_sms, cudaStream_t stream);
cudaError_t launch_prep_go16(const Geom& g, const void* go, void* go_r, float* gb, bool f16,
                             cudaStream_t stream);
cudaError_t launch_pack_weight_bwd16(const void* w, void* wbt, const Geom& g,
                                     cudaStream_t stream);
// fp32 NHWC grad-input accumulator -> 16-bit NCHW grad_input.
cudaError_t launch_nhwc_to_nchw16(const float* gxt, void* gx, int N, int C, int HW, bool f16,
                                  cudaStream_t stream);
// fp32 gradients to their 16-bit outputs in one launch: the tap-major weight
// gradient `gwt` ([outC][kk][Cg]) to `gw` ([outC][Cg][kk]) and the `count`
// arrays of `H16List` element-wise (rounded to nearest even).
struct H16List {
  const float* src[3];
  unsigned short* dst[3];
  long long n[3];
  int count;
  void add(const float* s, void* d, long long count_) {
    if (s != nullptr && d != nullptr && count_ > 0) {
      src[count] = s;
      dst[count] = static_cast<unsigned short*>(d);
      n[count] = count_;
      ++count;
    }
  }
};
// With `gpart` and `gb`: also the 16-bit grad_bias from launch_bwd_prologue16's
// partial sums.
cudaError_t launch_grads_to_h16(const float* gwt, void* gw, const Geom& g, const H16List& rest,
                                bool f16, cudaStream_t stream, const float* gpart = nullptr,
                                void* gb = nullptr);
// The 16-bit fused backward's helpers in one launch (as launch_bwd_prologue):
// 16-bit grad_out rows with fp32 grad_bias partial sums into `gpart`
// (tc_bias_part_floats16 of them; NULL: no bias), the 16-bit packed weight,
// the zeroing of `z`.
size_t tc_bias_part_floats16(const Geom& g);
cudaError_t launch_bwd_prologue16(const Geom& g, const void* go, void* go_r, float* gpart,
                                  const void* w, void* wbt, const ZeroList& z, bool f16,
                                  cudaStream_t stream);
// Weight gradient as a dense TMA-fed GEMM over the column buffer, summed into
// `gw` (pre-zeroed): grad_weight itself ([outC][Cg][kh*kw]), or with
// `tap_major` a [outC][kh*kw][Cg] copy, whose reductions coalesce, for the
// caller to transpose into place.
bool tc_wcol_supported(const Geom& g, bool split);
size_t tc_col_bytes(const Geom& g, bool split);
cudaError_t launch_bwd_weight_col(const Geom& g, const float* col, const float* go_r, float* gw,
                                  bool tap_major, bool split, int num_sms, cudaStream_t stream);
// [outC][kh*kw][Cg] -> grad_weight's [outC][Cg][kh*kw]; with `gpart` and
// `gb`, grad_bias from launch_bwd_prologue's partial sums as well.
cudaError_t launch_weight_from_tap_major(const float* gwt, float* gw, const Geom& g,
                                         cudaStream_t stream, const float* gpart = nullptr,
                                         float* gb = nullptr);
// launch_nhwc_to_nchw(gxt -> gx) and launch_weight_from_tap_major in one
// launch.  Needs C and HW multiples of 4 and 16-byte aligned gxt / gx
// (bwd_finish_fits); else cudaErrorInvalidValue, and the two separate
// launches apply.
bool bwd_finish_fits(const float* gxt, const float* gx, const Geom& g);
cudaError_t launch_bwd_finish(const float* gxt, float* gx, const float* gwt, float* gw,
                              const Geom& g, const float* gpart, float* gb, cudaStream_t stream);
// The fused TF32 backward's helpers for a staged input, in one launch:
// launch_tc_prep_go's work with grad_bias as per-block partial sums into
// `gpart` (tc_bias_part_floats of them; NULL: no bias), the packed weight of
// launch_tc_pack_weight_bwd (TF32, no split), and the zeroing of the
// accumulators in `z`.  No block depends on another.
size_t tc_bias_part_floats(const Geom& g);
cudaError_t launch_bwd_prologue(const Geom& g, const float* go, float* go_r, float* gpart,
                                const float* w, float* wbt, const ZeroList& z,
                                cudaStream_t stream);
// Sampling plans of every (n, deformable group, tap, pixel): 32 bytes each
// (corner element offsets into the NHWC copy, weights times mask).
inline size_t tc_plan_bytes(const Geom& g) { return (size_t)g.N * g.dg * g.kk * g.P * 32; }
cudaError_t launch_tc_plans(const Geom& g, const float* off, const float* mask, void* plans,
                            cudaStream_t stream);
// grad_weight (pre-zeroed) += col^T go on the tensor core, split over pixels;
// `tap_major`: into a [outC][kh*kw][Cg] copy as launch_bwd_weight_col.
cudaError_t launch_bwd_weight_tc(const Geom& g, const float* go_r, const float* xt,
                                 const void* plans, float* gw, bool tap_major, bool split,
                                 int num_sms, cudaStream_t stream);

}  // namespace dcn
