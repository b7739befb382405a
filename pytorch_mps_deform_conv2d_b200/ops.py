"""Functional deformable convolution, API-compatible with torchvision.

Mirrors the reference's functional layer
(src/deform_conv2d_mps/ops.py:62-169): same signature, same inference of
``groups`` and ``deformable_groups`` from the tensor shapes, same autograd
conventions (an empty mask means DCNv1, an empty bias means no bias; absent
inputs get ``None`` gradients).  CUDA tensors run the sm_100a kernels of
``libdcn_b200`` through the ``torch.ops.deform_conv2d_b200`` operators.
There is no fallback to another backend: tensors on any other device raise.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch
from torch import Tensor

from . import _native

# Flag words of the C ABI (include/dcn_b200.h).
MATH_FP32 = 0x0
MATH_TF32 = 0x1
MATH_3XTF32 = 0x2
ALGO_SIMT_GEMM = 0x100
ALGO_SIMT_DIRECT = 0x200
ALGO_TC_GATHER_WEIGHT = 0x400
ALGO_TC_COLUMN_BUFFER = 0x800
MASK_LOGITS = 0x10000
# test switch: the tensor-core kernels' waits run out (checks the error word)
TEST_WAIT_TIMEOUT = 0x1000000
# bits of the device error word (dcn_device_status)
STATUS_FWD_WAIT_TIMEOUT = 0x1
STATUS_BWD_DATA_TIMEOUT = 0x2
STATUS_BWD_WEIGHT_TIMEOUT = 0x4
_STATUS_NAMES = {STATUS_FWD_WAIT_TIMEOUT: "forward (fwd_tc)",
                 STATUS_BWD_DATA_TIMEOUT: "grad-column kernel (bwd_data_tc)",
                 STATUS_BWD_WEIGHT_TIMEOUT: "weight-gradient kernel"}


def device_status(clear: bool = True) -> int:
    """Error word of the tensor-core kernels on the current CUDA device:
    a bit per kernel family one of whose bounded waits ran out since the last
    clearing read (0: none).  Waits for the work already on the current
    stream; ``clear`` resets the word."""
    import ctypes
    stream = torch.cuda.current_stream()
    status = ctypes.c_int(0)
    lib = _native.load_capi()
    rc = lib.dcn_device_status(ctypes.c_void_p(stream.cuda_stream), 1 if clear else 0,
                               ctypes.byref(status))
    if rc != 0:
        raise RuntimeError(_native.capi_error())
    return int(status.value)


def check_device_status() -> None:
    """Raises RuntimeError when a wait of a tensor-core kernel gave up since
    the last check (the results of that call are incomplete); clears the
    error word."""
    word = device_status(clear=True)
    if word:
        names = [n for bit, n in _STATUS_NAMES.items() if word & bit]
        raise RuntimeError("deform_conv2d: a device wait ran out in the " + ", ".join(names) +
                           "; the results of that call are incomplete")

_MODES = {"fp32": MATH_FP32, "tf32": MATH_TF32, "3xtf32": MATH_3XTF32}
_NAMES = {v: k for k, v in _MODES.items()}
_math_override: Optional[int] = None


def set_math_mode(mode: Optional[str]) -> None:
    """Select the arithmetic of the CUDA kernels.

    ``"fp32"``: fp32 FFMA on the CUDA cores (tolerance of the reference's own
    tests, 1e-4).  ``"tf32"``: tcgen05 tensor cores with TF32 operands and
    fp32 accumulation.  ``"3xtf32"``: the same tensor-core kernels with each
    operand split into high and low TF32 parts (three products per
    multiply-add), close to fp32 accuracy.  ``None`` (default): follow
    ``torch.backends.cuda.matmul.allow_tf32``, as PyTorch's own convolutions
    and matmuls do.
    """
    global _math_override
    if mode is None:
        _math_override = None
        return
    if mode not in _MODES:
        raise ValueError(f"math mode must be one of {sorted(_MODES)} or None, got {mode!r}")
    _math_override = _MODES[mode]


def get_math_mode() -> str:
    """The math mode the next call will use ("fp32", "tf32" or "3xtf32")."""
    if _math_override is not None:
        return _NAMES.get(_math_override & 0xff, "fp32")
    return "tf32" if torch.backends.cuda.matmul.allow_tf32 else "fp32"


def _flags(flags: Optional[int]) -> int:
    if flags is not None:
        return int(flags)
    return -1 if _math_override is None else _math_override


def _ops():
    """``torch.ops.deform_conv2d_b200``; loads the library on first use.  The
    loaded case reads one flag and takes no lock, so torch.compile traces
    through it without a graph break."""
    if _native._ops_loaded:
        return torch.ops.deform_conv2d_b200
    return _native.load_ops()


def _pair(x) -> Tuple[int, int]:
    if isinstance(x, (tuple, list)):
        return int(x[0]), int(x[1])
    return int(x), int(x)


class _DeformConv2dFunction(torch.autograd.Function):
    """Autograd node over the native forward / backward operators.

    Same saved tensors and gradient layout as the reference's
    ``_DeformConv2dFunction`` (src/deform_conv2d_mps/ops.py:68-115).
    """

    @staticmethod
    def forward(ctx, input, weight, offset, mask, bias, stride, padding,
                dilation, groups, deformable_groups, flags):
        ops = _ops()
        empty = input.new_empty(0)
        out = ops.deform_conv2d_forward(
            input, weight, offset, mask if mask is not None else empty, bias,
            stride[0], stride[1], padding[0], padding[1], dilation[0],
            dilation[1], groups, deformable_groups, math=flags)
        ctx.save_for_backward(input, weight, offset,
                              mask if mask is not None else empty,
                              bias if bias is not None else empty)
        ctx.params = (stride, padding, dilation, groups, deformable_groups, flags)
        return out

    @staticmethod
    def backward(ctx, grad_output):
        input, weight, offset, mask, bias = ctx.saved_tensors
        stride, padding, dilation, groups, deformable_groups, flags = ctx.params
        has_mask = mask.numel() > 0
        has_bias = bias.numel() > 0
        ops = _ops()
        grad_input, grad_offset, grad_mask, grad_weight, grad_bias = \
            ops.deform_conv2d_backward(
                grad_output.contiguous(), input, weight, offset, mask,
                bias if has_bias else None, stride[0], stride[1], padding[0],
                padding[1], dilation[0], dilation[1], groups,
                deformable_groups, math=flags)
        return (grad_input, grad_weight, grad_offset,
                grad_mask if has_mask else None,
                grad_bias if has_bias else None,
                None, None, None, None, None, None)


def deform_conv2d(
    input: Tensor,
    offset: Tensor,
    weight: Tensor,
    bias: Optional[Tensor] = None,
    stride=(1, 1),
    padding=(0, 0),
    dilation=(1, 1),
    mask: Optional[Tensor] = None,
) -> Tensor:
    """Deformable Conv2d (DCNv2; DCNv1 when ``mask is None``).

    Signature of ``torchvision.ops.deform_conv2d``; ``groups`` and
    ``deformable_groups`` are inferred from ``weight`` and ``offset`` like the
    reference does (src/deform_conv2d_mps/ops.py:151-153).
    """
    return deform_conv2d_ex(input, offset, weight, bias, stride, padding,
                            dilation, mask)


def _resolved_math() -> int:
    if _math_override is not None:
        return _math_override
    return MATH_TF32 if torch.backends.cuda.matmul.allow_tf32 else MATH_FP32


def deform_conv2d_ex(input, offset, weight, bias=None, stride=(1, 1),
                     padding=(0, 0), dilation=(1, 1), mask=None,
                     flags: Optional[int] = None, mask_logits: bool = False) -> Tensor:
    """:func:`deform_conv2d` with an explicit C-ABI flag word (``MATH_*`` |
    ``ALGO_*``); ``flags=None`` uses the current math mode.

    ``mask_logits=True``: ``mask`` holds logits and the kernels apply the
    sigmoid themselves (forward) and return the gradient with respect to the
    logits -- the DCNv2 block's ``sigmoid(mask)`` fused into the op."""
    if mask_logits and mask is not None:
        flags = (_resolved_math() if flags is None or int(flags) < 0 else int(flags)) | MASK_LOGITS
    stride, padding, dilation = _pair(stride), _pair(padding), _pair(dilation)
    for name, t in (("input", input), ("offset", offset), ("weight", weight),
                    ("bias", bias), ("mask", mask)):
        if t is not None and t.device.type != "cuda":
            raise NotImplementedError(
                f"pytorch_mps_deform_conv2d_b200.deform_conv2d runs on CUDA "
                f"(sm_100a) tensors only; {name} is on {t.device}")
    kh, kw = weight.shape[-2], weight.shape[-1]
    if weight.dim() != 4 or weight.shape[1] == 0:
        raise RuntimeError("weight must be 4-D (outC, C/groups, kh, kw) with C/groups > 0")
    groups = input.shape[1] // weight.shape[1]
    deformable_groups = offset.shape[1] // (2 * kh * kw)
    if not torch.compiler.is_compiling():
        # eager: the differentiable operator, whose autograd node is C++ (no
        # Python frame in the forward or the backward)
        return _ops().deform_conv2d(
            input, weight, offset, mask if mask is not None else input.new_empty(0), bias,
            stride[0], stride[1], padding[0], padding[1], dilation[0], dilation[1], groups,
            deformable_groups, math=_flags(flags))
    return _DeformConv2dFunction.apply(
        input, weight, offset, mask, bias, stride, padding, dilation, groups,
        deformable_groups, _flags(flags))


def deform_conv2d_rows(input, offset, weight, bias=None, stride=(1, 1), padding=(0, 0),
                       dilation=(1, 1), mask=None, row_begin: int = 0,
                       flags: Optional[int] = None) -> Tensor:
    """Output rows ``[row_begin, row_begin + offset.shape[2])`` of
    :func:`deform_conv2d` (a row window; no reference counterpart).

    ``input`` is the whole input; ``offset`` / ``mask`` hold the window's
    rows only, and so does the result.  Differentiable: the input's, the
    weight's and the bias' gradients are this window's contributions, so
    summing them over a partition of the rows gives the full gradients (see
    :func:`pytorch_mps_deform_conv2d_b200.distributed.deform_conv2d_row_sharded`).
    """
    stride, padding, dilation = _pair(stride), _pair(padding), _pair(dilation)
    for name, t in (("input", input), ("offset", offset), ("weight", weight),
                    ("bias", bias), ("mask", mask)):
        if t is not None and t.device.type != "cuda":
            raise NotImplementedError(
                f"pytorch_mps_deform_conv2d_b200.deform_conv2d_rows runs on CUDA tensors "
                f"only; {name} is on {t.device}")
    kh, kw = weight.shape[-2], weight.shape[-1]
    groups = input.shape[1] // weight.shape[1]
    deformable_groups = offset.shape[1] // (2 * kh * kw)
    m = mask if mask is not None else input.new_empty(0)
    # eager: the row operator whose autograd node is C++; traced: the
    # operator with the registered autograd formula
    op = (_ops().deform_conv2d_rows if not torch.compiler.is_compiling()
          else _ops().deform_conv2d_forward_rows)
    return op(input, weight, offset, m, bias, stride[0], stride[1], padding[0], padding[1],
              dilation[0], dilation[1], groups, deformable_groups, int(row_begin), _flags(flags))
