"""Python-side registrations of the ``torch.ops.deform_conv2d_b200`` operators.

* Fake (meta) kernels: output shapes and dtypes from the input shapes, no
  data, so FakeTensor tracing, ``torch.compile`` and
  ``torch.library.opcheck`` can reason about the CUDA operators.  They follow
  the allocation rules of the CUDA implementations (csrc/torch_ops.cpp): an
  empty mask (DCNv1) gives an empty grad_mask, an absent or empty bias an
  empty grad_bias.
* Autograd formulas for ``deform_conv2d_forward`` and
  ``deform_conv2d_forward_rows``, so the operators are differentiable when
  called directly.  The public ``deform_conv2d`` runs the ``deform_conv2d``
  operator in eager mode (its autograd node is registered in C++,
  csrc/torch_ops.cpp) and, while torch.compile traces, goes through
  ``ops._DeformConv2dFunction``, which mirrors the reference's
  ``_DeformConv2dFunction`` (src/deform_conv2d_mps/ops.py:68-115).

The reference registers only a real-device implementation
(src/deform_conv2d_mps/_C/deform_conv2d_mps.mm:918-925); these are additions.
"""
from __future__ import annotations

import torch

NS = "deform_conv2d_b200"


def _out_size(size, k, s, p, d):
    return (size + 2 * p - d * (k - 1) - 1) // s + 1


def _forward_fake(input, weight, offset, mask, bias, stride_h, stride_w, pad_h, pad_w,
                  dilation_h, dilation_w, groups, deformable_groups, math=-1, staged=None):
    ho = _out_size(input.shape[2], weight.shape[2], stride_h, pad_h, dilation_h)
    wo = _out_size(input.shape[3], weight.shape[3], stride_w, pad_w, dilation_w)
    return input.new_empty((input.shape[0], weight.shape[0], ho, wo))


def _input_format(input):
    """Layout of grad_input: channels-last for a dense channels-last input
    (the CUDA operators keep it), contiguous NCHW otherwise."""
    if (input.dim() == 4 and not input.is_contiguous()
            and input.is_contiguous(memory_format=torch.channels_last)):
        return torch.channels_last
    return torch.contiguous_format


def _backward_fake(grad_output, input, weight, offset, mask, bias, stride_h, stride_w, pad_h,
                   pad_w, dilation_h, dilation_w, groups, deformable_groups, math=-1,
                   staged=None):
    grad_mask = mask.new_empty(mask.shape) if mask.numel() > 0 else input.new_empty((0,))
    use_bias = bias is not None and bias.numel() > 0
    grad_bias = input.new_empty((weight.shape[0],)) if use_bias else input.new_empty((0,))
    grad_input = torch.empty(input.shape, dtype=input.dtype, device=input.device,
                             memory_format=_input_format(input))
    return (grad_input, offset.new_empty(offset.shape), grad_mask,
            weight.new_empty(weight.shape), grad_bias)


def _stage_input_fake(input):
    n, c, h, w = input.shape
    return input.new_empty((n * h * w * c + c,))


def _forward_staging_fake(input, weight, offset, mask, bias, stride_h, stride_w, pad_h, pad_w,
                          dilation_h, dilation_w, groups, deformable_groups, math=-1,
                          row_begin=-1):
    if row_begin >= 0:  # a row window: offset holds its rows
        out = _forward_rows_fake(input, weight, offset, mask, bias, stride_h, stride_w, pad_h,
                                 pad_w, dilation_h, dilation_w, groups, deformable_groups,
                                 row_begin, math)
    else:
        out = _forward_fake(input, weight, offset, mask, bias, stride_h, stride_w, pad_h, pad_w,
                            dilation_h, dilation_w, groups, deformable_groups, math)
    return out, _stage_input_fake(input)


def _forward_rows_fake(input, weight, offset, mask, bias, stride_h, stride_w, pad_h, pad_w,
                       dilation_h, dilation_w, groups, deformable_groups, row_begin, math=-1):
    wo = _out_size(input.shape[3], weight.shape[3], stride_w, pad_w, dilation_w)
    return input.new_empty((input.shape[0], weight.shape[0], offset.shape[2], wo))


def _backward_rows_fake(grad_output, input, weight, offset, mask, bias, stride_h, stride_w,
                        pad_h, pad_w, dilation_h, dilation_w, groups, deformable_groups,
                        row_begin, math=-1, staged=None):
    return _backward_fake(grad_output, input, weight, offset, mask, bias, stride_h, stride_w,
                          pad_h, pad_w, dilation_h, dilation_w, groups, deformable_groups, math)


def _col2im_fake(columns, offset, mask, height, width, kernel_h, kernel_w, stride_h, stride_w,
                 pad_h, pad_w, dilation_h, dilation_w, deformable_groups, math=-1):
    channels = columns.shape[0] // (kernel_h * kernel_w)
    return columns.new_empty((channels, height, width))


def _col2im_coord_fake(columns, input, offset, mask, kernel_h, kernel_w, stride_h, stride_w,
                       pad_h, pad_w, dilation_h, dilation_w, deformable_groups, math=-1):
    grad_mask = (offset.new_empty((offset.shape[0] // 2, offset.shape[1], offset.shape[2]))
                 if mask.numel() > 0 else offset.new_empty((0,)))
    return offset.new_empty(offset.shape), grad_mask


_INT_ARGS = ("stride_h", "stride_w", "pad_h", "pad_w", "dilation_h", "dilation_w", "groups",
             "deformable_groups", "math")


def _setup(ctx, inputs, nints):
    input, weight, offset, mask, bias = inputs[:5]
    ctx.ints = tuple(inputs[5:5 + nints])   # the integer arguments
    ctx.n_rest = len(inputs) - 5           # + the staging copy, if the schema has one
    ctx.has_mask = mask.numel() > 0
    ctx.has_bias = bias is not None and bias.numel() > 0
    ctx.save_for_backward(input, weight, offset, mask, bias if ctx.has_bias else None)


def _setup_context(ctx, inputs, output):
    _setup(ctx, inputs, len(_INT_ARGS))  # deform_conv2d_forward: ints, then `staged`


def _setup_rows_context(ctx, inputs, output):
    _setup(ctx, inputs, len(_INT_ARGS) + 1)  # deform_conv2d_forward_rows: + row_begin


def _forward_backward(ctx, grad_output):
    input, weight, offset, mask, bias = ctx.saved_tensors
    grads = getattr(torch.ops, NS).deform_conv2d_backward(
        grad_output.contiguous(), input, weight, offset, mask, bias, *ctx.ints)
    grad_input, grad_offset, grad_mask, grad_weight, grad_bias = grads
    return ((grad_input, grad_weight, grad_offset,
             grad_mask if ctx.has_mask else None,
             grad_bias if ctx.has_bias else None) + (None,) * ctx.n_rest)


def _forward_rows_backward(ctx, grad_output):
    input, weight, offset, mask, bias = ctx.saved_tensors
    grads = getattr(torch.ops, NS).deform_conv2d_backward_rows(
        grad_output.contiguous(), input, weight, offset, mask, bias, *ctx.ints)
    grad_input, grad_offset, grad_mask, grad_weight, grad_bias = grads
    return ((grad_input, grad_weight, grad_offset,
             grad_mask if ctx.has_mask else None,
             grad_bias if ctx.has_bias else None) + (None,) * ctx.n_rest)


def register() -> None:
    """Attach the fake kernels and the autograd formula (once, after the
    operator library has been loaded)."""
    q = NS + "::"
    torch.library.register_fake(q + "deform_conv2d_forward")(_forward_fake)
    torch.library.register_fake(q + "deform_conv2d")(_forward_fake)
    torch.library.register_fake(q + "deform_conv2d_backward")(_backward_fake)
    torch.library.register_fake(q + "deform_conv2d_stage_input")(_stage_input_fake)
    torch.library.register_fake(q + "deform_conv2d_forward_staging")(_forward_staging_fake)
    torch.library.register_fake(q + "deformable_col2im")(_col2im_fake)
    torch.library.register_fake(q + "deformable_col2im_coord")(_col2im_coord_fake)
    torch.library.register_autograd(q + "deform_conv2d_forward", _forward_backward,
                                    setup_context=_setup_context)
    torch.library.register_fake(q + "deform_conv2d_forward_rows")(_forward_rows_fake)
    torch.library.register_fake(q + "deform_conv2d_rows")(_forward_rows_fake)
    torch.library.register_fake(q + "deform_conv2d_backward_rows")(_backward_rows_fake)
    torch.library.register_autograd(q + "deform_conv2d_forward_rows", _forward_rows_backward,
                                    setup_context=_setup_rows_context)
