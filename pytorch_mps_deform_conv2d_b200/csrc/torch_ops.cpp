// torch_ops.cpp -- PyTorch operator registration for libdcn_b200.
//
// Registers the reference's operator schemas
// (src/deform_conv2d_mps/_C/deform_conv2d_mps.mm:892-916) under the namespace
// `deform_conv2d_b200` with a CUDA dispatch implementation.  Each
// implementation validates with the reference's messages, makes inputs
// contiguous, allocates outputs and scratch through PyTorch's caching
// allocator, and calls the C ABI (include/dcn_b200.h) on the current CUDA
// stream.  Every schema has one extra trailing argument, `int math=-1`: -1
// follows torch.backends.cuda.matmul.allow_tf32, otherwise it is the
// DCN_MATH_* / DCN_ALGO_* flag word of the C ABI.  The forward and backward
// operators take one more, `Tensor? staged=None`: the input's NHWC staging
// copy (deform_conv2d_stage_input), which the differentiable operator makes
// once per step for both passes.
#include <ATen/ATen.h>
#include <ATen/Context.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/csrc/autograd/custom_function.h>
#include <torch/library.h>

#include "dcn_b200.h"

namespace {

uint32_t resolve_flags(int64_t math) {
  if (math >= 0) return static_cast<uint32_t>(math);
  return at::globalContext().allowTF32CuBLAS() ? DCN_MATH_TF32 : DCN_MATH_FP32;
}

void check_rc(int rc) {
  TORCH_CHECK(rc == DCN_OK, dcn_last_error());
}

void check_cuda_f32(const at::Tensor& t, const char* what) {
  TORCH_CHECK(t.device().is_cuda() && t.scalar_type() == at::kFloat, what);
}

dcn_shape make_shape(const at::Tensor& x, const at::Tensor& w, int64_t stride_h,
                     int64_t stride_w, int64_t pad_h, int64_t pad_w, int64_t dilation_h,
                     int64_t dilation_w, int64_t groups, int64_t dg) {
  dcn_shape s;
  s.batch = x.size(0);
  s.in_channels = x.size(1);
  s.height = x.size(2);
  s.width = x.size(3);
  s.out_channels = w.size(0);
  s.kernel_h = w.size(2);
  s.kernel_w = w.size(3);
  s.stride_h = stride_h;
  s.stride_w = stride_w;
  s.pad_h = pad_h;
  s.pad_w = pad_w;
  s.dilation_h = dilation_h;
  s.dilation_w = dilation_w;
  s.groups = groups;
  s.deformable_groups = dg;
  return s;
}

// Shape checks of .mm:202-267 (forward) / :693-760 (backward).
void check_shapes(const at::Tensor& x, const at::Tensor& w, const at::Tensor& off,
                  const at::Tensor& msk, bool use_mask, int64_t stride_h, int64_t stride_w,
                  int64_t pad_h, int64_t pad_w, int64_t dilation_h, int64_t dilation_w,
                  int64_t groups, int64_t dg, int64_t& out_h, int64_t& out_w,
                  int64_t row_begin = -1) {
  TORCH_CHECK(x.dim() == 4, "input must be 4-D (N, C, H, W), got ", x.dim());
  TORCH_CHECK(w.dim() == 4, "weight must be 4-D (outC, C/groups, kh, kw), got ", w.dim());
  TORCH_CHECK(off.dim() == 4, "offset must be 4-D (N, 2*dg*kh*kw, oh, ow), got ", off.dim());
  TORCH_CHECK(groups > 0, "groups must be positive, got ", groups);
  TORCH_CHECK(stride_h > 0 && stride_w > 0, "stride must be positive");
  TORCH_CHECK(dilation_h > 0 && dilation_w > 0, "dilation must be positive");
  const int64_t N = x.size(0), C = x.size(1), H = x.size(2), W = x.size(3);
  const int64_t outC = w.size(0), kh = w.size(2), kw = w.size(3);
  TORCH_CHECK(w.size(1) * groups == C, "weight shape mismatch: expected in-channels ", C,
              ", got ", w.size(1) * groups);
  TORCH_CHECK(C % groups == 0, "channels (", C, ") not divisible by groups (", groups, ")");
  TORCH_CHECK(outC % groups == 0, "out_channels (", outC, ") not divisible by groups (", groups,
              ")");
  out_h = (H + 2 * pad_h - dilation_h * (kh - 1) - 1) / stride_h + 1;
  out_w = (W + 2 * pad_w - dilation_w * (kw - 1) - 1) / stride_w + 1;
  TORCH_CHECK(out_h > 0 && out_w > 0, "calculated output size (", out_h, "x", out_w,
              ") is non-positive");
  if (row_begin >= 0) {  // row window: offset / mask hold output rows [row_begin, +rows)
    const int64_t rows = off.size(2);
    TORCH_CHECK(rows > 0 && row_begin + rows <= out_h, "output rows [", row_begin, ", ",
                row_begin + rows, ") outside the ", out_h, " output rows");
    out_h = rows;
  }
  TORCH_CHECK(dg > 0, "deformable_groups must be positive, got ", dg);
  TORCH_CHECK(C % dg == 0, "channels (", C, ") not divisible by deformable_groups (", dg, ")");
  TORCH_CHECK(off.size(0) == N && off.size(1) == 2 * dg * kh * kw && off.size(2) == out_h &&
                  off.size(3) == out_w,
              "offset shape mismatch: expected (", N, ", ", 2 * dg * kh * kw, ", ", out_h, ", ",
              out_w, "), got ", off.sizes());
  if (use_mask) {
    if (x.scalar_type() == at::kBFloat16 || x.scalar_type() == at::kHalf) {
      TORCH_CHECK(msk.device().is_cuda() && msk.scalar_type() == x.scalar_type(),
                  "mask must be a ", x.scalar_type() == at::kHalf ? "float16" : "bfloat16",
                  " CUDA tensor");
    } else {
      check_cuda_f32(msk, "mask must be a float32 CUDA tensor");
    }
    TORCH_CHECK(msk.dim() == 4 && msk.size(0) == N && msk.size(1) == dg * kh * kw &&
                    msk.size(2) == out_h && msk.size(3) == out_w,
                "mask shape mismatch: expected (", N, ", ", dg * kh * kw, ", ", out_h, ", ",
                out_w, "), got ", msk.sizes());
  }
}

// A dense channels-last input (torch's NHWC strides, e.g. from
// .to(memory_format=torch.channels_last)) goes to the library as it lies,
// with DCN_INPUT_NHWC; anything else is made contiguous NCHW.
bool channels_last(const at::Tensor& t) {
  return t.dim() == 4 && !t.is_contiguous() &&
         t.is_contiguous(at::MemoryFormat::ChannelsLast);
}

// The staging copy of `x` for DCN_INPUT_STAGED, when the caller passed one
// (a float32 tensor of dcn_staged_input_size bytes on x's device); NULL
// otherwise.
const float* staged_ptr(const c10::optional<at::Tensor>& staged, const at::Tensor& x,
                        const dcn_shape& s) {
  if (!staged.has_value() || !staged->defined() || staged->numel() == 0) return nullptr;
  TORCH_CHECK(staged->device() == x.device() && staged->scalar_type() == at::kFloat &&
                  staged->is_contiguous() &&
                  (size_t)staged->numel() * sizeof(float) == dcn_staged_input_size(&s),
              "staged must be the float32 staging copy of the input "
              "(deform_conv2d_stage_input)");
  return staged->data_ptr<float>();
}

// The 16-bit staging copy of `x` (a tensor of x's dtype, dcn_staged_input_size_h16
// bytes) when the caller passed one; NULL otherwise.
const void* staged_ptr16(const c10::optional<at::Tensor>& staged, const at::Tensor& x,
                         const dcn_shape& s) {
  if (!staged.has_value() || !staged->defined() || staged->numel() == 0) return nullptr;
  TORCH_CHECK(staged->device() == x.device() && staged->scalar_type() == x.scalar_type() &&
                  staged->is_contiguous() &&
                  (size_t)staged->numel() * 2 == dcn_staged_input_size_h16(&s),
              "staged must be the 16-bit staging copy of the input "
              "(deform_conv2d_stage_input)");
  return staged->data_ptr();
}

// Whether the 16-bit forward and backward of this call take a staging copy
// (dcn_h16_staging: both on their tensor-core routes).
bool h16_staging(const at::Tensor& input, const at::Tensor& weight, int64_t stride_h,
                 int64_t stride_w, int64_t pad_h, int64_t pad_w, int64_t dilation_h,
                 int64_t dilation_w, int64_t groups, int64_t deformable_groups, int64_t math) {
  if (input.dim() != 4 || weight.dim() != 4) return false;
  const dcn_shape s = make_shape(input, weight, stride_h, stride_w, pad_h, pad_w, dilation_h,
                                 dilation_w, groups, deformable_groups);
  const uint32_t flags = resolve_flags(math) | (channels_last(input) ? DCN_INPUT_NHWC : 0u);
  return dcn_h16_staging(&s, flags) == 1;
}

at::Tensor deform_conv2d_stage_input(const at::Tensor& input);

// Whether a forward whose workspace is `ws_bytes` should keep its staging
// copy (`staged_bytes`) in that workspace: the kept copy pins the whole
// workspace until the backward, so not when the rest of it (packed weight,
// a split round's partial sums) would hold much more than the copy itself.
bool keep_in_workspace(size_t ws_bytes, size_t staged_bytes) {
  return ws_bytes <= staged_bytes + staged_bytes / 8 + (size_t(1) << 20);
}

// The staging copy a forward with DCN_KEEP_STAGED left at the 256-byte
// aligned start of its workspace `ws`: `bytes` bytes viewed as `dt`.
at::Tensor kept_staging(const at::Tensor& ws, size_t bytes, at::ScalarType dt) {
  const uintptr_t base = reinterpret_cast<uintptr_t>(ws.data_ptr());
  const int64_t lead = (int64_t)(((base + 255) & ~(uintptr_t)255) - base);
  TORCH_CHECK(bytes > 0 && lead + (int64_t)bytes <= ws.numel(),
              "deform_conv2d_forward: no staging copy");
  return ws.narrow(0, lead, (int64_t)bytes).view(dt);
}

at::Tensor forward_impl(const at::Tensor& input, const at::Tensor& weight,
                        const at::Tensor& offset, const at::Tensor& mask,
                        const c10::optional<at::Tensor>& bias, int64_t stride_h,
                        int64_t stride_w, int64_t pad_h, int64_t pad_w, int64_t dilation_h,
                        int64_t dilation_w, int64_t groups, int64_t deformable_groups,
                        int64_t row_begin, int64_t math,
                        const c10::optional<at::Tensor>& staged = c10::nullopt,
                        at::Tensor* keep_staged = nullptr) {
  TORCH_CHECK(input.device().is_cuda() && weight.device().is_cuda() && offset.device().is_cuda(),
              "deform_conv2d_forward: input, weight and offset must be CUDA tensors");
  // float32 (the reference's only dtype, .mm:206-209) or, as an addition,
  // bfloat16 for every tensor
  // (as another addition) float16 for every tensor
  const auto dt = input.scalar_type();
  const bool h16 = dt == at::kBFloat16 || dt == at::kHalf;  // 16-bit tensors
  const bool f16 = dt == at::kHalf;
  if (h16) {
    TORCH_CHECK(weight.scalar_type() == dt && offset.scalar_type() == dt,
                "deform_conv2d_forward: input, weight and offset must all be float32, all "
                "bfloat16 or all float16");
  } else {
    TORCH_CHECK(input.scalar_type() == at::kFloat && weight.scalar_type() == at::kFloat &&
                    offset.scalar_type() == at::kFloat,
                "deform_conv2d_forward: only float32 is supported");
  }
  const bool use_mask = mask.defined() && mask.numel() > 0;
  int64_t out_h = 0, out_w = 0;
  check_shapes(input, weight, offset, mask, use_mask, stride_h, stride_w, pad_h, pad_w,
               dilation_h, dilation_w, groups, deformable_groups, out_h, out_w, row_begin);
  TORCH_CHECK(row_begin < 0 || !h16, "deform_conv2d_forward_rows: float32 tensors only");
  at::Tensor b;
  if (bias.has_value() && bias->defined() && bias->numel() > 0) {
    if (h16) {
      TORCH_CHECK(bias->device().is_cuda() && bias->scalar_type() == dt, "bias must be a ",
                  f16 ? "float16" : "bfloat16", " CUDA tensor");
    } else {
      check_cuda_f32(*bias, "bias must be a float32 CUDA tensor");
    }
    TORCH_CHECK(bias->numel() == weight.size(0), "bias must have ", weight.size(0),
                " elements, got ", bias->numel());
    b = bias->contiguous();
  }
  c10::cuda::CUDAGuard guard(input.device());
  const bool nhwc = channels_last(input);
  auto x = nhwc ? input : input.contiguous();
  auto w = weight.contiguous();
  auto off = offset.contiguous();
  auto msk = use_mask ? mask.contiguous() : at::Tensor();
  auto out = at::empty({x.size(0), w.size(0), out_h, out_w}, x.options());
  if (out.numel() == 0) return out;
  const dcn_shape s = make_shape(x, w, stride_h, stride_w, pad_h, pad_w, dilation_h, dilation_w,
                                 groups, deformable_groups);
  const uint32_t flags = resolve_flags(math) | (nhwc ? DCN_INPUT_NHWC : 0u);
  auto stream = at::cuda::getCurrentCUDAStream();
  if (h16) {
    const void* xs = staged_ptr16(staged, x, s);
    if (keep_staged != nullptr) {
      const size_t wsk = f16 ? dcn_forward_f16_workspace_size(&s, flags | DCN_KEEP_STAGED)
                             : dcn_forward_bf16_workspace_size(&s, flags | DCN_KEEP_STAGED);
      if (!keep_in_workspace(wsk, dcn_staged_input_size_h16(&s))) {
        *keep_staged = deform_conv2d_stage_input(x);
        xs = keep_staged->data_ptr();
        keep_staged = nullptr;
      }
    }
    const uint32_t flags16 =
        flags | (xs ? DCN_INPUT_STAGED : 0u) | (keep_staged != nullptr ? DCN_KEEP_STAGED : 0u);
    const size_t ws16 = f16 ? dcn_forward_f16_workspace_size(&s, flags16)
                            : dcn_forward_bf16_workspace_size(&s, flags16);
    auto ws = at::empty({(int64_t)std::max<size_t>(ws16, 1)}, x.options().dtype(at::kByte));
    auto fwd16 = f16 ? dcn_forward_f16 : dcn_forward_bf16;
    check_rc(fwd16(&s, xs ? xs : x.data_ptr(), w.data_ptr(), off.data_ptr(),
                   use_mask ? msk.data_ptr() : nullptr, b.defined() ? b.data_ptr() : nullptr,
                   out.data_ptr(), flags16, ws.data_ptr(), ws16, stream.stream()));
    if (keep_staged != nullptr)
      *keep_staged = kept_staging(ws, dcn_staged_input_size_h16(&s), x.scalar_type());
    return out;
  }
  const float* mp = use_mask ? msk.data_ptr<float>() : nullptr;
  const float* bp = b.defined() ? b.data_ptr<float>() : nullptr;
  const float* xs = staged_ptr(staged, x, s);
  if (keep_staged != nullptr) {
    // stage on its own (then run staged) when the workspace would pin more
    // than the copy
    const size_t wsk = row_begin >= 0
                           ? dcn_forward_rows_workspace_size(&s, out_h, flags | DCN_KEEP_STAGED)
                           : dcn_forward_workspace_size(&s, flags | DCN_KEEP_STAGED);
    if (!keep_in_workspace(wsk, dcn_staged_input_size(&s))) {
      *keep_staged = deform_conv2d_stage_input(x);
      xs = keep_staged->data_ptr<float>();
      keep_staged = nullptr;
    }
  }
  if (row_begin >= 0) {
    const uint32_t rflags =
        flags | (xs ? DCN_INPUT_STAGED : 0u) | (keep_staged != nullptr ? DCN_KEEP_STAGED : 0u);
    const size_t wsr = dcn_forward_rows_workspace_size(&s, out_h, rflags);
    auto ws = at::empty({(int64_t)std::max<size_t>(wsr, 1)}, x.options().dtype(at::kByte));
    check_rc(dcn_forward_rows(&s, row_begin, out_h, xs ? xs : x.data_ptr<float>(),
                              w.data_ptr<float>(), off.data_ptr<float>(), mp, bp,
                              out.data_ptr<float>(), rflags, ws.data_ptr(), wsr, stream.stream()));
    if (keep_staged != nullptr)
      *keep_staged = kept_staging(ws, dcn_staged_input_size(&s), at::kFloat);
    return out;
  }
  const uint32_t fflags =
      flags | (xs ? DCN_INPUT_STAGED : 0u) | (keep_staged != nullptr ? DCN_KEEP_STAGED : 0u);
  const size_t ws_bytes = dcn_forward_workspace_size(&s, fflags);
  auto ws = at::empty({(int64_t)std::max<size_t>(ws_bytes, 1)}, x.options().dtype(at::kByte));
  check_rc(dcn_forward(&s, xs ? xs : x.data_ptr<float>(), w.data_ptr<float>(),
                       off.data_ptr<float>(), mp, bp, out.data_ptr<float>(), fflags,
                       ws.data_ptr(), ws_bytes, stream.stream()));
  if (keep_staged != nullptr)
    *keep_staged = kept_staging(ws, dcn_staged_input_size(&s), at::kFloat);
  return out;
}

at::Tensor deform_conv2d_forward(const at::Tensor& input, const at::Tensor& weight,
                                 const at::Tensor& offset, const at::Tensor& mask,
                                 const c10::optional<at::Tensor>& bias, int64_t stride_h,
                                 int64_t stride_w, int64_t pad_h, int64_t pad_w,
                                 int64_t dilation_h, int64_t dilation_w, int64_t groups,
                                 int64_t deformable_groups, int64_t math,
                                 const c10::optional<at::Tensor>& staged) {
  return forward_impl(input, weight, offset, mask, bias, stride_h, stride_w, pad_h, pad_w,
                      dilation_h, dilation_w, groups, deformable_groups, -1, math, staged);
}

// The differentiable operator's kernel below autograd: the forward without a
// staging copy (its schema has none).
at::Tensor deform_conv2d_plain(const at::Tensor& input, const at::Tensor& weight,
                               const at::Tensor& offset, const at::Tensor& mask,
                               const c10::optional<at::Tensor>& bias, int64_t stride_h,
                               int64_t stride_w, int64_t pad_h, int64_t pad_w,
                               int64_t dilation_h, int64_t dilation_w, int64_t groups,
                               int64_t deformable_groups, int64_t math) {
  return forward_impl(input, weight, offset, mask, bias, stride_h, stride_w, pad_h, pad_w,
                      dilation_h, dilation_w, groups, deformable_groups, -1, math);
}

// NHWC staging copy of a float32 input (its zero pixel row included), for
// the `staged` argument of the forward and backward operators: a training
// step stages its input once for both.
at::Tensor deform_conv2d_stage_input(const at::Tensor& input) {
  const auto dt = input.scalar_type();
  const bool h16 = dt == at::kBFloat16 || dt == at::kHalf;
  TORCH_CHECK(input.device().is_cuda() && (dt == at::kFloat || h16) && input.dim() == 4,
              "deform_conv2d_stage_input: input must be a 4-D float32, bfloat16 or float16 "
              "CUDA tensor");
  c10::cuda::CUDAGuard guard(input.device());
  const bool nhwc = channels_last(input);
  auto x = nhwc ? input : input.contiguous();
  dcn_shape s{};
  s.batch = x.size(0);
  s.in_channels = x.size(1);
  s.height = x.size(2);
  s.width = x.size(3);
  s.out_channels = 1;
  s.kernel_h = s.kernel_w = 1;
  s.stride_h = s.stride_w = 1;
  s.dilation_h = s.dilation_w = 1;
  s.groups = 1;
  s.deformable_groups = 1;
  if (h16) {  // the same layout in the input's 16-bit type
    const size_t bytes = dcn_staged_input_size_h16(&s);
    TORCH_CHECK(bytes > 0, dcn_last_error());
    auto staged = at::empty({(int64_t)(bytes / 2)}, x.options());
    check_rc(dcn_stage_input_h16(&s, x.data_ptr(), staged.data_ptr(), nhwc ? DCN_INPUT_NHWC : 0u,
                                 at::cuda::getCurrentCUDAStream().stream()));
    return staged;
  }
  const size_t bytes = dcn_staged_input_size(&s);
  TORCH_CHECK(bytes > 0, dcn_last_error());
  auto staged = at::empty({(int64_t)(bytes / sizeof(float))}, x.options());
  check_rc(dcn_stage_input(&s, x.data_ptr<float>(), staged.data_ptr<float>(),
                           nhwc ? DCN_INPUT_NHWC : 0u,
                           at::cuda::getCurrentCUDAStream().stream()));
  return staged;
}

// The forward that also returns its NHWC staging copy of the (float32)
// input, for the `staged` argument of the backward: a training step stages
// inside the forward, where the weight pack runs beside the staging.
std::tuple<at::Tensor, at::Tensor> deform_conv2d_forward_staging(
    const at::Tensor& input, const at::Tensor& weight, const at::Tensor& offset,
    const at::Tensor& mask, const c10::optional<at::Tensor>& bias, int64_t stride_h,
    int64_t stride_w, int64_t pad_h, int64_t pad_w, int64_t dilation_h, int64_t dilation_w,
    int64_t groups, int64_t deformable_groups, int64_t math, int64_t row_begin) {
  TORCH_CHECK(input.dim() == 4 && input.numel() > 0,
              "deform_conv2d_forward_staging: input must be a non-empty 4-D tensor");
  const auto dt = input.scalar_type();
  if (dt == at::kBFloat16 || dt == at::kHalf) {
    TORCH_CHECK(row_begin < 0, "deform_conv2d_forward_staging: row windows take float32 tensors");
    // the 16-bit forward keeps its staging copy on its tensor-core route;
    // elsewhere the copy is made on its own (and the backward's upcast route
    // does not take it)
    at::Tensor staged;
    const bool keep = h16_staging(input, weight, stride_h, stride_w, pad_h, pad_w, dilation_h,
                                  dilation_w, groups, deformable_groups, math);
    auto out = forward_impl(input, weight, offset, mask, bias, stride_h, stride_w, pad_h, pad_w,
                            dilation_h, dilation_w, groups, deformable_groups, -1, math,
                            c10::nullopt, keep ? &staged : nullptr);
    if (!staged.defined()) staged = deform_conv2d_stage_input(input);
    return std::make_tuple(out, staged);
  }
  at::Tensor staged;
  auto out = forward_impl(input, weight, offset, mask, bias, stride_h, stride_w, pad_h, pad_w,
                          dilation_h, dilation_w, groups, deformable_groups,
                          row_begin >= 0 ? row_begin : -1, math, c10::nullopt, &staged);
  if (!staged.defined()) staged = deform_conv2d_stage_input(input);  // no output pixels
  return std::make_tuple(out, staged);
}

at::Tensor deform_conv2d_forward_rows(const at::Tensor& input, const at::Tensor& weight,
                                      const at::Tensor& offset, const at::Tensor& mask,
                                      const c10::optional<at::Tensor>& bias, int64_t stride_h,
                                      int64_t stride_w, int64_t pad_h, int64_t pad_w,
                                      int64_t dilation_h, int64_t dilation_w, int64_t groups,
                                      int64_t deformable_groups, int64_t row_begin,
                                      int64_t math) {
  TORCH_CHECK(row_begin >= 0, "deform_conv2d_forward_rows: row_begin must be >= 0");
  return forward_impl(input, weight, offset, mask, bias, stride_h, stride_w, pad_h, pad_w,
                      dilation_h, dilation_w, groups, deformable_groups, row_begin, math);
}

using Grads = std::tuple<at::Tensor, at::Tensor, at::Tensor, at::Tensor, at::Tensor>;

// grad_weight and grad_bias.  `adjacent` (with a bias): two views of one
// buffer, the bias right after the weight, so that a data-parallel step sums
// both with a single all-reduce of that buffer (distributed.allreduce_grads
// and GradAllReduce find them adjacent); autograd hands such views on as the
// parameters' .grad when nothing else holds them.  Only the autograd nodes
// ask for it: a registered operator's outputs must not alias one another.
std::pair<at::Tensor, at::Tensor> param_grads(const at::Tensor& w, bool use_bias,
                                              bool adjacent) {
  if (adjacent && use_bias) {
    auto flat = at::empty({w.numel() + w.size(0)}, w.options());
    return {flat.narrow(0, 0, w.numel()).view(w.sizes()), flat.narrow(0, w.numel(), w.size(0))};
  }
  return {at::empty_like(w), use_bias ? at::empty({w.size(0)}, w.options())
                                      : at::empty({0}, w.options())};
}

Grads backward_impl(const at::Tensor& grad_output, const at::Tensor& input,
                    const at::Tensor& weight, const at::Tensor& offset, const at::Tensor& mask,
                    const c10::optional<at::Tensor>& bias, int64_t stride_h, int64_t stride_w,
                    int64_t pad_h, int64_t pad_w, int64_t dilation_h, int64_t dilation_w,
                    int64_t groups, int64_t deformable_groups, int64_t row_begin, int64_t math,
                    const c10::optional<at::Tensor>& staged = c10::nullopt,
                    bool adjacent_param_grads = false) {
  TORCH_CHECK(grad_output.device().is_cuda() && input.device().is_cuda() &&
                  weight.device().is_cuda() && offset.device().is_cuda(),
              "deform_conv2d_backward: grad_output, input, weight and offset must be CUDA tensors");
  const auto dt = input.scalar_type();
  if (dt == at::kBFloat16 || dt == at::kHalf) {
    // 16-bit tensors: the library's 16-bit backward (the fused tensor-core
    // kernel with 16-bit operands where it covers the shape, else the fp32
    // route on upcast copies); gradients in the input's dtype
    const bool f16 = dt == at::kHalf;
    TORCH_CHECK(grad_output.scalar_type() == dt && weight.scalar_type() == dt &&
                    offset.scalar_type() == dt,
                "deform_conv2d_backward: grad_output, input, weight and offset must all be "
                "float32, all bfloat16 or all float16");
    TORCH_CHECK(row_begin < 0, "deform_conv2d_backward_rows: float32 tensors only");
    TORCH_CHECK(grad_output.dim() == 4, "grad_output must be 4-D, got ", grad_output.dim());
    const bool use_mask = mask.defined() && mask.numel() > 0;
    int64_t out_h = 0, out_w = 0;
    check_shapes(input, weight, offset, mask, use_mask, stride_h, stride_w, pad_h, pad_w,
                 dilation_h, dilation_w, groups, deformable_groups, out_h, out_w);
    TORCH_CHECK(grad_output.size(0) == input.size(0) && grad_output.size(1) == weight.size(0) &&
                    grad_output.size(2) == out_h && grad_output.size(3) == out_w,
                "grad_output shape mismatch: expected (", input.size(0), ", ", weight.size(0),
                ", ", out_h, ", ", out_w, "), got ", grad_output.sizes());
    const bool use_bias = bias.has_value() && bias->defined() && bias->numel() > 0;
    c10::cuda::CUDAGuard guard(input.device());
    auto go = grad_output.contiguous();
    const bool nhwc = channels_last(input);
    auto x = nhwc ? input : input.contiguous();
    auto w = weight.contiguous();
    auto off = offset.contiguous();
    auto msk = use_mask ? mask.contiguous() : at::Tensor();
    auto grad_input = at::empty_like(x);
    auto grad_offset = at::empty_like(off);
    auto grad_mask = use_mask ? at::empty_like(msk) : at::empty({0}, x.options());
    auto [grad_weight, grad_bias] = param_grads(w, use_bias, adjacent_param_grads);
    if (x.numel() == 0 && off.numel() == 0) {
      grad_weight.zero_();
      if (use_bias) grad_bias.zero_();
      return std::make_tuple(grad_input, grad_offset, grad_mask, grad_weight, grad_bias);
    }
    const dcn_shape s = make_shape(x, w, stride_h, stride_w, pad_h, pad_w, dilation_h,
                                   dilation_w, groups, deformable_groups);
    const void* xs = staged_ptr16(staged, x, s);
    const uint32_t flags =
        resolve_flags(math) | (nhwc ? DCN_INPUT_NHWC : 0u) | (xs ? DCN_INPUT_STAGED : 0u);
    const size_t ws_bytes = f16 ? dcn_backward_f16_workspace_size(&s, flags)
                                : dcn_backward_bf16_workspace_size(&s, flags);
    auto ws = at::empty({(int64_t)std::max<size_t>(ws_bytes, 1)}, x.options().dtype(at::kByte));
    auto vp = [](const at::Tensor& t) -> void* { return t.numel() ? t.data_ptr() : nullptr; };
    auto bwd16 = f16 ? dcn_backward_f16 : dcn_backward_bf16;
    check_rc(bwd16(&s, vp(go), xs ? const_cast<void*>(xs) : vp(x), vp(w), vp(off),
                   use_mask ? vp(msk) : nullptr,
                   vp(grad_input), vp(grad_offset), use_mask ? vp(grad_mask) : nullptr,
                   vp(grad_weight), use_bias ? vp(grad_bias) : nullptr, flags, ws.data_ptr(),
                   ws_bytes, at::cuda::getCurrentCUDAStream().stream()));
    return std::make_tuple(grad_input, grad_offset, grad_mask, grad_weight, grad_bias);
  }
  TORCH_CHECK(grad_output.scalar_type() == at::kFloat && input.scalar_type() == at::kFloat &&
                  weight.scalar_type() == at::kFloat && offset.scalar_type() == at::kFloat,
              "deform_conv2d_backward: only float32 is supported");
  TORCH_CHECK(grad_output.dim() == 4, "grad_output must be 4-D, got ", grad_output.dim());
  const bool use_mask = mask.defined() && mask.numel() > 0;
  int64_t out_h = 0, out_w = 0;
  check_shapes(input, weight, offset, mask, use_mask, stride_h, stride_w, pad_h, pad_w,
               dilation_h, dilation_w, groups, deformable_groups, out_h, out_w, row_begin);
  TORCH_CHECK(grad_output.size(0) == input.size(0) && grad_output.size(1) == weight.size(0) &&
                  grad_output.size(2) == out_h && grad_output.size(3) == out_w,
              "grad_output shape mismatch: expected (", input.size(0), ", ", weight.size(0), ", ",
              out_h, ", ", out_w, "), got ", grad_output.sizes());
  const bool use_bias = bias.has_value() && bias->defined() && bias->numel() > 0;
  c10::cuda::CUDAGuard guard(input.device());
  auto go = grad_output.contiguous();
  const bool nhwc = channels_last(input);
  auto x = nhwc ? input : input.contiguous();  // grad_input below takes x's layout
  auto w = weight.contiguous();
  auto off = offset.contiguous();
  auto msk = use_mask ? mask.contiguous() : at::Tensor();
  auto grad_input = at::empty_like(x);
  auto grad_offset = at::empty_like(off);
  auto grad_mask = use_mask ? at::empty_like(msk) : at::empty({0}, x.options());
  auto [grad_weight, grad_bias] = param_grads(w, use_bias, adjacent_param_grads);
  const dcn_shape s = make_shape(x, w, stride_h, stride_w, pad_h, pad_w, dilation_h, dilation_w,
                                 groups, deformable_groups);
  const float* xs = staged_ptr(staged, x, s);
  const uint32_t flags = resolve_flags(math) | (nhwc ? DCN_INPUT_NHWC : 0u) |
                         (xs ? DCN_INPUT_STAGED : 0u);
  const size_t ws_bytes = row_begin >= 0 ? dcn_backward_rows_workspace_size(&s, out_h, flags)
                                         : dcn_backward_workspace_size(&s, flags);
  auto ws = at::empty({(int64_t)std::max<size_t>(ws_bytes, 1)}, x.options().dtype(at::kByte));
  auto stream = at::cuda::getCurrentCUDAStream();
  auto ptr = [](at::Tensor& t) { return t.numel() ? t.data_ptr<float>() : nullptr; };
  auto cptr = [](const at::Tensor& t) -> const float* {
    return t.defined() && t.numel() ? t.data_ptr<float>() : nullptr;
  };
  float* gm = use_mask ? ptr(grad_mask) : nullptr;
  float* gb = use_bias ? ptr(grad_bias) : nullptr;
  const float* mp = use_mask ? cptr(msk) : nullptr;
  if (row_begin >= 0)
    check_rc(dcn_backward_rows(&s, row_begin, out_h, cptr(go), xs ? xs : cptr(x), cptr(w),
                               cptr(off), mp,
                               ptr(grad_input), ptr(grad_offset), gm, ptr(grad_weight), gb, flags,
                               ws.data_ptr(), ws_bytes, stream.stream()));
  else
    check_rc(dcn_backward(&s, cptr(go), xs ? xs : cptr(x), cptr(w), cptr(off), mp, ptr(grad_input),
                          ptr(grad_offset), gm, ptr(grad_weight), gb, flags, ws.data_ptr(),
                          ws_bytes, stream.stream()));
  return std::make_tuple(grad_input, grad_offset, grad_mask, grad_weight, grad_bias);
}

Grads deform_conv2d_backward(const at::Tensor& grad_output, const at::Tensor& input,
                             const at::Tensor& weight, const at::Tensor& offset,
                             const at::Tensor& mask, const c10::optional<at::Tensor>& bias,
                             int64_t stride_h, int64_t stride_w, int64_t pad_h, int64_t pad_w,
                             int64_t dilation_h, int64_t dilation_w, int64_t groups,
                             int64_t deformable_groups, int64_t math,
                             const c10::optional<at::Tensor>& staged) {
  return backward_impl(grad_output, input, weight, offset, mask, bias, stride_h, stride_w, pad_h,
                       pad_w, dilation_h, dilation_w, groups, deformable_groups, -1, math, staged);
}

Grads deform_conv2d_backward_rows(const at::Tensor& grad_output, const at::Tensor& input,
                                  const at::Tensor& weight, const at::Tensor& offset,
                                  const at::Tensor& mask, const c10::optional<at::Tensor>& bias,
                                  int64_t stride_h, int64_t stride_w, int64_t pad_h,
                                  int64_t pad_w, int64_t dilation_h, int64_t dilation_w,
                                  int64_t groups, int64_t deformable_groups, int64_t row_begin,
                                  int64_t math, const c10::optional<at::Tensor>& staged) {
  TORCH_CHECK(row_begin >= 0, "deform_conv2d_backward_rows: row_begin must be >= 0");
  return backward_impl(grad_output, input, weight, offset, mask, bias, stride_h, stride_w, pad_h,
                       pad_w, dilation_h, dilation_w, groups, deformable_groups, row_begin, math,
                       staged);
}

at::Tensor deformable_col2im(const at::Tensor& columns, const at::Tensor& offset,
                             const at::Tensor& mask, int64_t height, int64_t width,
                             int64_t kernel_h, int64_t kernel_w, int64_t stride_h,
                             int64_t stride_w, int64_t pad_h, int64_t pad_w, int64_t dilation_h,
                             int64_t dilation_w, int64_t deformable_groups, int64_t math) {
  (void)math;
  TORCH_CHECK(columns.device().is_cuda() && offset.device().is_cuda(),
              "deformable_col2im: columns and offset must be CUDA tensors");
  TORCH_CHECK(columns.scalar_type() == at::kFloat && offset.scalar_type() == at::kFloat,
              "deformable_col2im: only float32 is supported");
  TORCH_CHECK(columns.dim() == 2, "columns must be 2-D (C*kh*kw, oh*ow)");
  TORCH_CHECK(offset.dim() == 3, "offset must be 3-D (2*dg*kh*kw, oh, ow)");
  TORCH_CHECK(kernel_h > 0 && kernel_w > 0, "kernel dims must be positive");
  TORCH_CHECK(stride_h > 0 && stride_w > 0, "stride must be positive");
  TORCH_CHECK(dilation_h > 0 && dilation_w > 0, "dilation must be positive");
  const int64_t kk = kernel_h * kernel_w;
  TORCH_CHECK(columns.size(0) % kk == 0, "columns rows (", columns.size(0),
              ") not divisible by kh*kw (", kk, ")");
  const int64_t C = columns.size(0) / kk;
  const int64_t out_h = (height + 2 * pad_h - dilation_h * (kernel_h - 1) - 1) / stride_h + 1;
  const int64_t out_w = (width + 2 * pad_w - dilation_w * (kernel_w - 1) - 1) / stride_w + 1;
  TORCH_CHECK(columns.size(1) == out_h * out_w, "columns cols (", columns.size(1),
              ") != out_h*out_w (", out_h * out_w, ")");
  const int64_t dg = deformable_groups;
  TORCH_CHECK(dg > 0, "deformable_groups must be positive, got ", dg);
  TORCH_CHECK(C % dg == 0, "channels (", C, ") not divisible by deformable_groups (", dg, ")");
  TORCH_CHECK(offset.size(0) == 2 * dg * kk && offset.size(1) == out_h && offset.size(2) == out_w,
              "offset shape mismatch: expected (", 2 * dg * kk, ", ", out_h, ", ", out_w,
              "), got ", offset.sizes());
  const bool use_mask = mask.defined() && mask.numel() > 0;
  if (use_mask) {
    check_cuda_f32(mask, "mask must be a float32 CUDA tensor");
    TORCH_CHECK(mask.dim() == 3 && mask.size(0) == dg * kk && mask.size(1) == out_h &&
                    mask.size(2) == out_w,
                "mask shape mismatch: expected (", dg * kk, ", ", out_h, ", ", out_w, "), got ",
                mask.sizes());
  }
  c10::cuda::CUDAGuard guard(columns.device());
  auto col = columns.contiguous();
  auto off = offset.contiguous();
  auto msk = use_mask ? mask.contiguous() : at::Tensor();
  auto grad_im = at::empty({C, height, width}, col.options());
  if (grad_im.numel() == 0) return grad_im;
  auto stream = at::cuda::getCurrentCUDAStream();
  check_rc(dcn_col2im(col.data_ptr<float>(), off.data_ptr<float>(),
                      use_mask ? msk.data_ptr<float>() : nullptr, grad_im.data_ptr<float>(), C,
                      height, width, kernel_h, kernel_w, stride_h, stride_w, pad_h, pad_w,
                      dilation_h, dilation_w, dg, stream.stream()));
  return grad_im;
}

std::tuple<at::Tensor, at::Tensor> deformable_col2im_coord(
    const at::Tensor& columns, const at::Tensor& input, const at::Tensor& offset,
    const at::Tensor& mask, int64_t kernel_h, int64_t kernel_w, int64_t stride_h,
    int64_t stride_w, int64_t pad_h, int64_t pad_w, int64_t dilation_h, int64_t dilation_w,
    int64_t deformable_groups, int64_t math) {
  (void)math;
  TORCH_CHECK(columns.device().is_cuda() && input.device().is_cuda() && offset.device().is_cuda(),
              "deformable_col2im_coord: columns, input and offset must be CUDA tensors");
  TORCH_CHECK(columns.scalar_type() == at::kFloat && input.scalar_type() == at::kFloat &&
                  offset.scalar_type() == at::kFloat,
              "deformable_col2im_coord: only float32 is supported");
  TORCH_CHECK(columns.dim() == 2, "columns must be 2-D (C*kh*kw, oh*ow)");
  TORCH_CHECK(input.dim() == 3, "input must be 3-D (C, H, W)");
  TORCH_CHECK(offset.dim() == 3, "offset must be 3-D (2*dg*kh*kw, oh, ow)");
  TORCH_CHECK(kernel_h > 0 && kernel_w > 0, "kernel dims must be positive");
  TORCH_CHECK(stride_h > 0 && stride_w > 0, "stride must be positive");
  TORCH_CHECK(dilation_h > 0 && dilation_w > 0, "dilation must be positive");
  const int64_t C = input.size(0), H = input.size(1), W = input.size(2);
  const int64_t kk = kernel_h * kernel_w;
  TORCH_CHECK(columns.size(0) == C * kk, "columns rows (", columns.size(0), ") != C*kh*kw (",
              C * kk, ")");
  const int64_t out_h = (H + 2 * pad_h - dilation_h * (kernel_h - 1) - 1) / stride_h + 1;
  const int64_t out_w = (W + 2 * pad_w - dilation_w * (kernel_w - 1) - 1) / stride_w + 1;
  TORCH_CHECK(columns.size(1) == out_h * out_w, "columns cols (", columns.size(1),
              ") != out_h*out_w (", out_h * out_w, ")");
  const int64_t dg = deformable_groups;
  TORCH_CHECK(dg > 0, "deformable_groups must be positive, got ", dg);
  TORCH_CHECK(C % dg == 0, "channels (", C, ") not divisible by deformable_groups (", dg, ")");
  TORCH_CHECK(offset.size(0) == 2 * dg * kk && offset.size(1) == out_h && offset.size(2) == out_w,
              "offset shape mismatch: expected (", 2 * dg * kk, ", ", out_h, ", ", out_w,
              "), got ", offset.sizes());
  const bool use_mask = mask.defined() && mask.numel() > 0;
  if (use_mask) {
    check_cuda_f32(mask, "mask must be a float32 CUDA tensor");
    TORCH_CHECK(mask.dim() == 3 && mask.size(0) == dg * kk && mask.size(1) == out_h &&
                    mask.size(2) == out_w,
                "mask shape mismatch: expected (", dg * kk, ", ", out_h, ", ", out_w, "), got ",
                mask.sizes());
  }
  c10::cuda::CUDAGuard guard(columns.device());
  auto col = columns.contiguous();
  auto x = input.contiguous();
  auto off = offset.contiguous();
  auto msk = use_mask ? mask.contiguous() : at::Tensor();
  auto grad_offset = at::empty({2 * dg * kk, out_h, out_w}, off.options());
  auto grad_mask = use_mask ? at::empty({dg * kk, out_h, out_w}, off.options())
                            : at::empty({0}, off.options());
  if (grad_offset.numel() == 0) return std::make_tuple(grad_offset, grad_mask);
  auto stream = at::cuda::getCurrentCUDAStream();
  check_rc(dcn_col2im_coord(col.numel() ? col.data_ptr<float>() : nullptr,
                            x.numel() ? x.data_ptr<float>() : nullptr, off.data_ptr<float>(),
                            use_mask ? msk.data_ptr<float>() : nullptr,
                            grad_offset.data_ptr<float>(),
                            use_mask ? grad_mask.data_ptr<float>() : nullptr, C, H, W, kernel_h,
                            kernel_w, stride_h, stride_w, pad_h, pad_w, dilation_h, dilation_w,
                            dg, stream.stream()));
  return std::make_tuple(grad_offset, grad_mask);
}

// Differentiable deform_conv2d as one operator, its autograd node in C++: the
// eager path of the public Python API, with no Python frame in the forward or
// the backward.  The same computation as ops._DeformConv2dFunction
// (src/deform_conv2d_mps/ops.py:68-115 in the reference): the forward and
// backward operators above, gradients for input, weight, offset, mask (none
// for an empty mask) and bias (none when absent).  Both operators are reached
// through the dispatcher, so fake tensors take their fake kernels.
class DeformConv2dFn : public torch::autograd::Function<DeformConv2dFn> {
 public:
  static at::Tensor forward(torch::autograd::AutogradContext* ctx, const at::Tensor& input,
                            const at::Tensor& weight, const at::Tensor& offset,
                            const at::Tensor& mask, const at::Tensor& bias, int64_t stride_h,
                            int64_t stride_w, int64_t pad_h, int64_t pad_w, int64_t dilation_h,
                            int64_t dilation_w, int64_t groups, int64_t deformable_groups,
                            int64_t math) {
    static auto op = c10::Dispatcher::singleton()
                         .findSchemaOrThrow("deform_conv2d_b200::deform_conv2d_forward", "")
                         .typed<at::Tensor(const at::Tensor&, const at::Tensor&,
                                           const at::Tensor&, const at::Tensor&,
                                           const c10::optional<at::Tensor>&, int64_t, int64_t,
                                           int64_t, int64_t, int64_t, int64_t, int64_t, int64_t,
                                           int64_t, const c10::optional<at::Tensor>&)>();
    static auto fwd_staging =
        c10::Dispatcher::singleton()
            .findSchemaOrThrow("deform_conv2d_b200::deform_conv2d_forward_staging", "")
            .typed<std::tuple<at::Tensor, at::Tensor>(
                const at::Tensor&, const at::Tensor&, const at::Tensor&, const at::Tensor&,
                const c10::optional<at::Tensor>&, int64_t, int64_t, int64_t, int64_t, int64_t,
                int64_t, int64_t, int64_t, int64_t, int64_t)>();
    const bool has_bias = bias.defined() && bias.numel() > 0;
    c10::optional<at::Tensor> b;
    if (has_bias) b = bias;
    at::Tensor out, staged;
    {
      at::AutoDispatchBelowADInplaceOrView below;
      // a float32 input, or a 16-bit one whose passes both run on the tensor
      // cores, is staged (NHWC) once, inside the forward, and the staging
      // copy kept for the backward
      const auto dt = input.scalar_type();
      const bool stage_once =
          input.dim() == 4 && input.numel() > 0 &&
          (dt == at::kFloat ||
           ((dt == at::kBFloat16 || dt == at::kHalf) &&
            h16_staging(input, weight, stride_h, stride_w, pad_h, pad_w, dilation_h, dilation_w,
                        groups, deformable_groups, math)));
      if (stage_once) {
        std::tie(out, staged) =
            fwd_staging.call(input, weight, offset, mask, b, stride_h, stride_w, pad_h, pad_w,
                             dilation_h, dilation_w, groups, deformable_groups, math, -1);
      } else {
        out = op.call(input, weight, offset, mask, b, stride_h, stride_w, pad_h, pad_w,
                      dilation_h, dilation_w, groups, deformable_groups, math, c10::nullopt);
      }
    }
    ctx->save_for_backward({input, weight, offset, mask, bias});
    if (staged.defined()) ctx->saved_data["staged"] = staged;
    ctx->saved_data["ints"] = std::vector<int64_t>{stride_h,   stride_w, pad_h,
                                                   pad_w,      dilation_h, dilation_w,
                                                   groups,     deformable_groups, math};
    ctx->saved_data["has_bias"] = has_bias;
    return out;
  }

  static torch::autograd::variable_list backward(torch::autograd::AutogradContext* ctx,
                                                 torch::autograd::variable_list grads) {
    const auto saved = ctx->get_saved_variables();
    const auto v = ctx->saved_data["ints"].toIntVector();
    const bool has_bias = ctx->saved_data["has_bias"].toBool();
    const at::Tensor& mask = saved[3];
    c10::optional<at::Tensor> b;
    if (has_bias) b = saved[4];
    c10::optional<at::Tensor> st;
    if (ctx->saved_data.count("staged")) st = ctx->saved_data["staged"].toTensor();
    // the backward operator's work, with grad_weight / grad_bias side by side
    auto r = backward_impl(grads[0].contiguous(), saved[0], saved[1], saved[2], mask, b, v[0],
                           v[1], v[2], v[3], v[4], v[5], v[6], v[7], -1, v[8], st, true);
    const bool has_mask = mask.numel() > 0;
    return {std::get<0>(r),
            std::get<3>(r),
            std::get<1>(r),
            has_mask ? std::get<2>(r) : at::Tensor(),
            has_bias ? std::get<4>(r) : at::Tensor(),
            at::Tensor(), at::Tensor(), at::Tensor(), at::Tensor(), at::Tensor(),
            at::Tensor(), at::Tensor(), at::Tensor(), at::Tensor()};
  }
};

// The row-window operator's C++ autograd node: output rows [row_begin,
// row_begin + offset.size(2)) of a replicated input, their gradients by the
// row-window backward (no Python frame in either pass).
class DeformConv2dRowsFn : public torch::autograd::Function<DeformConv2dRowsFn> {
 public:
  static at::Tensor forward(torch::autograd::AutogradContext* ctx, const at::Tensor& input,
                            const at::Tensor& weight, const at::Tensor& offset,
                            const at::Tensor& mask, const at::Tensor& bias, int64_t stride_h,
                            int64_t stride_w, int64_t pad_h, int64_t pad_w, int64_t dilation_h,
                            int64_t dilation_w, int64_t groups, int64_t deformable_groups,
                            int64_t row_begin, int64_t math) {
    static auto op =
        c10::Dispatcher::singleton()
            .findSchemaOrThrow("deform_conv2d_b200::deform_conv2d_forward_rows", "")
            .typed<at::Tensor(const at::Tensor&, const at::Tensor&, const at::Tensor&,
                              const at::Tensor&, const c10::optional<at::Tensor>&, int64_t,
                              int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, int64_t,
                              int64_t, int64_t)>();
    static auto fwd_staging =
        c10::Dispatcher::singleton()
            .findSchemaOrThrow("deform_conv2d_b200::deform_conv2d_forward_staging", "")
            .typed<std::tuple<at::Tensor, at::Tensor>(
                const at::Tensor&, const at::Tensor&, const at::Tensor&, const at::Tensor&,
                const c10::optional<at::Tensor>&, int64_t, int64_t, int64_t, int64_t, int64_t,
                int64_t, int64_t, int64_t, int64_t, int64_t)>();
    const bool has_bias = bias.defined() && bias.numel() > 0;
    c10::optional<at::Tensor> b;
    if (has_bias) b = bias;
    at::Tensor out, staged;
    {
      at::AutoDispatchBelowADInplaceOrView below;
      // a float32 input is staged inside the forward and kept for the backward
      if (input.scalar_type() == at::kFloat && input.dim() == 4 && input.numel() > 0)
        std::tie(out, staged) =
            fwd_staging.call(input, weight, offset, mask, b, stride_h, stride_w, pad_h, pad_w,
                             dilation_h, dilation_w, groups, deformable_groups, math, row_begin);
      else
        out = op.call(input, weight, offset, mask, b, stride_h, stride_w, pad_h, pad_w,
                      dilation_h, dilation_w, groups, deformable_groups, row_begin, math);
    }
    if (staged.defined()) ctx->saved_data["staged"] = staged;
    ctx->save_for_backward({input, weight, offset, mask, bias});
    ctx->saved_data["ints"] = std::vector<int64_t>{stride_h,   stride_w,   pad_h,
                                                   pad_w,      dilation_h, dilation_w,
                                                   groups,     deformable_groups, row_begin,
                                                   math};
    ctx->saved_data["has_bias"] = has_bias;
    return out;
  }

  static torch::autograd::variable_list backward(torch::autograd::AutogradContext* ctx,
                                                 torch::autograd::variable_list grads) {
    const auto saved = ctx->get_saved_variables();
    const auto v = ctx->saved_data["ints"].toIntVector();
    const bool has_bias = ctx->saved_data["has_bias"].toBool();
    const at::Tensor& mask = saved[3];
    c10::optional<at::Tensor> b;
    if (has_bias) b = saved[4];
    c10::optional<at::Tensor> st;
    if (ctx->saved_data.count("staged")) st = ctx->saved_data["staged"].toTensor();
    TORCH_CHECK(v[8] >= 0, "deform_conv2d_backward_rows: row_begin must be >= 0");
    auto r = backward_impl(grads[0].contiguous(), saved[0], saved[1], saved[2], mask, b, v[0],
                           v[1], v[2], v[3], v[4], v[5], v[6], v[7], v[8], v[9], st, true);
    const bool has_mask = mask.numel() > 0;
    return {std::get<0>(r),
            std::get<3>(r),
            std::get<1>(r),
            has_mask ? std::get<2>(r) : at::Tensor(),
            has_bias ? std::get<4>(r) : at::Tensor(),
            at::Tensor(), at::Tensor(), at::Tensor(), at::Tensor(), at::Tensor(),
            at::Tensor(), at::Tensor(), at::Tensor(), at::Tensor(), at::Tensor()};
  }
};

at::Tensor deform_conv2d_rows_autograd(const at::Tensor& input, const at::Tensor& weight,
                                       const at::Tensor& offset, const at::Tensor& mask,
                                       const c10::optional<at::Tensor>& bias, int64_t stride_h,
                                       int64_t stride_w, int64_t pad_h, int64_t pad_w,
                                       int64_t dilation_h, int64_t dilation_w, int64_t groups,
                                       int64_t deformable_groups, int64_t row_begin,
                                       int64_t math) {
  return DeformConv2dRowsFn::apply(
      input, weight, offset, mask,
      bias.has_value() && bias->defined() ? *bias : input.new_empty({0}), stride_h, stride_w,
      pad_h, pad_w, dilation_h, dilation_w, groups, deformable_groups, row_begin, math);
}

// The row-window operator below autograd.
at::Tensor deform_conv2d_rows_plain(const at::Tensor& input, const at::Tensor& weight,
                                    const at::Tensor& offset, const at::Tensor& mask,
                                    const c10::optional<at::Tensor>& bias, int64_t stride_h,
                                    int64_t stride_w, int64_t pad_h, int64_t pad_w,
                                    int64_t dilation_h, int64_t dilation_w, int64_t groups,
                                    int64_t deformable_groups, int64_t row_begin, int64_t math) {
  return deform_conv2d_forward_rows(input, weight, offset, mask, bias, stride_h, stride_w, pad_h,
                                    pad_w, dilation_h, dilation_w, groups, deformable_groups,
                                    row_begin, math);
}

at::Tensor deform_conv2d_autograd(const at::Tensor& input, const at::Tensor& weight,
                                  const at::Tensor& offset, const at::Tensor& mask,
                                  const c10::optional<at::Tensor>& bias, int64_t stride_h,
                                  int64_t stride_w, int64_t pad_h, int64_t pad_w,
                                  int64_t dilation_h, int64_t dilation_w, int64_t groups,
                                  int64_t deformable_groups, int64_t math) {
  // an absent bias travels as an empty tensor (the autograd node takes
  // defined tensors only)
  return DeformConv2dFn::apply(input, weight, offset, mask,
                               bias.has_value() && bias->defined() ? *bias : input.new_empty({0}),
                               stride_h, stride_w,
                               pad_h, pad_w, dilation_h, dilation_w, groups, deformable_groups,
                               math);
}

}  // namespace

TORCH_LIBRARY(deform_conv2d_b200, m) {
  m.def(
      "deformable_col2im(Tensor columns, Tensor offset, Tensor mask, int height, int width, "
      "int kernel_h, int kernel_w, int stride_h, int stride_w, int pad_h, int pad_w, "
      "int dilation_h, int dilation_w, int deformable_groups, int math=-1) -> Tensor");
  m.def(
      "deformable_col2im_coord(Tensor columns, Tensor input, Tensor offset, Tensor mask, "
      "int kernel_h, int kernel_w, int stride_h, int stride_w, int pad_h, int pad_w, "
      "int dilation_h, int dilation_w, int deformable_groups, int math=-1) -> (Tensor, Tensor)");
  m.def(
      "deform_conv2d_forward(Tensor input, Tensor weight, Tensor offset, Tensor mask, "
      "Tensor? bias, int stride_h, int stride_w, int pad_h, int pad_w, int dilation_h, "
      "int dilation_w, int groups, int deformable_groups, int math=-1, Tensor? staged=None) "
      "-> Tensor");
  m.def(
      "deform_conv2d_backward(Tensor grad_output, Tensor input, Tensor weight, Tensor offset, "
      "Tensor mask, Tensor? bias, int stride_h, int stride_w, int pad_h, int pad_w, "
      "int dilation_h, int dilation_w, int groups, int deformable_groups, int math=-1, "
      "Tensor? staged=None) -> (Tensor, Tensor, Tensor, Tensor, Tensor)");
  // NHWC staging copy of a float32 input for the `staged` argument above (no
  // reference counterpart): a training step stages its input once.
  m.def("deform_conv2d_stage_input(Tensor input) -> Tensor");
  // The forward that also returns its staging copy of a float32 input (no
  // reference counterpart): what the differentiable operator runs.
  m.def(
      "deform_conv2d_forward_staging(Tensor input, Tensor weight, Tensor offset, Tensor mask, "
      "Tensor? bias, int stride_h, int stride_w, int pad_h, int pad_w, int dilation_h, "
      "int dilation_w, int groups, int deformable_groups, int math=-1, int row_begin=-1) "
      "-> (Tensor, Tensor)");
  // Row windows (no reference counterpart): offset / mask / output /
  // grad_output hold output rows [row_begin, row_begin + offset.size(2)).
  m.def(
      "deform_conv2d_forward_rows(Tensor input, Tensor weight, Tensor offset, Tensor mask, "
      "Tensor? bias, int stride_h, int stride_w, int pad_h, int pad_w, int dilation_h, "
      "int dilation_w, int groups, int deformable_groups, int row_begin, int math=-1) -> Tensor");
  m.def(
      "deform_conv2d_backward_rows(Tensor grad_output, Tensor input, Tensor weight, "
      "Tensor offset, Tensor mask, Tensor? bias, int stride_h, int stride_w, int pad_h, "
      "int pad_w, int dilation_h, int dilation_w, int groups, int deformable_groups, "
      "int row_begin, int math=-1, Tensor? staged=None) "
      "-> (Tensor, Tensor, Tensor, Tensor, Tensor)");
  // The differentiable operator (forward + the C++ autograd node above).
  m.def(
      "deform_conv2d(Tensor input, Tensor weight, Tensor offset, Tensor mask, Tensor? bias, "
      "int stride_h, int stride_w, int pad_h, int pad_w, int dilation_h, int dilation_w, "
      "int groups, int deformable_groups, int math=-1) -> Tensor");
  // Its row-window form (no reference counterpart).
  m.def(
      "deform_conv2d_rows(Tensor input, Tensor weight, Tensor offset, Tensor mask, "
      "Tensor? bias, int stride_h, int stride_w, int pad_h, int pad_w, int dilation_h, "
      "int dilation_w, int groups, int deformable_groups, int row_begin, int math=-1) -> Tensor");
}

TORCH_LIBRARY_IMPL(deform_conv2d_b200, Autograd, m) {
  m.impl("deform_conv2d", TORCH_FN(deform_conv2d_autograd));
  m.impl("deform_conv2d_rows", TORCH_FN(deform_conv2d_rows_autograd));
}

TORCH_LIBRARY_IMPL(deform_conv2d_b200, CUDA, m) {
  m.impl("deformable_col2im", TORCH_FN(deformable_col2im));
  m.impl("deformable_col2im_coord", TORCH_FN(deformable_col2im_coord));
  m.impl("deform_conv2d_forward", TORCH_FN(deform_conv2d_forward));
  m.impl("deform_conv2d_backward", TORCH_FN(deform_conv2d_backward));
  m.impl("deform_conv2d_forward_rows", TORCH_FN(deform_conv2d_forward_rows));
  m.impl("deform_conv2d_backward_rows", TORCH_FN(deform_conv2d_backward_rows));
  m.impl("deform_conv2d_stage_input", TORCH_FN(deform_conv2d_stage_input));
  m.impl("deform_conv2d_forward_staging", TORCH_FN(deform_conv2d_forward_staging));
  m.impl("deform_conv2d", TORCH_FN(deform_conv2d_plain));  // below autograd
  m.impl("deform_conv2d_rows", TORCH_FN(deform_conv2d_rows_plain));
}
