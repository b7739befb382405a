"""``DeformConv2d`` module, interchangeable with torchvision's.

Same constructor, parameters (``weight`` (outC, C/groups, kh, kw), optional
``bias`` (outC)), initialisation and ``forward(input, offset, mask=None)`` as
the reference's module (src/deform_conv2d_mps/module.py:19-57), so state dicts
load in either direction.
"""
from __future__ import annotations

import math
from typing import Optional

import torch
from torch import Tensor, nn

from . import _native
from .ops import _pair, deform_conv2d, deform_conv2d_ex


class DeformConv2d(nn.Module):
    def __init__(self, in_channels: int, out_channels: int, kernel_size,
                 stride=1, padding=0, dilation=1, groups: int = 1,
                 bias: bool = True):
        super().__init__()
        if in_channels % groups != 0:
            raise ValueError("in_channels must be divisible by groups")
        if out_channels % groups != 0:
            raise ValueError("out_channels must be divisible by groups")
        self.in_channels = in_channels
        self.out_channels = out_channels
        self.kernel_size = _pair(kernel_size)
        self.stride = _pair(stride)
        self.padding = _pair(padding)
        self.dilation = _pair(dilation)
        self.groups = groups
        kh, kw = self.kernel_size
        self.weight = nn.Parameter(torch.empty(out_channels, in_channels // groups, kh, kw))
        if bias:
            self.bias = nn.Parameter(torch.empty(out_channels))
        else:
            self.register_parameter("bias", None)
        self.reset_parameters()
        # Load the operator library now, outside any torch.compile trace; a
        # missing library raises at the first forward instead.
        try:
            _native.load_ops()
        except _native.NativeLibraryError:
            pass

    def reset_parameters(self) -> None:
        # kaiming_uniform_(a=sqrt(5)) and a uniform bias in +-1/sqrt(fan_in),
        # the initialisation of module.py:37-44 (and of torch's Conv2d).
        nn.init.kaiming_uniform_(self.weight, a=math.sqrt(5))
        if self.bias is not None:
            fan_in = (self.in_channels // self.groups) * self.kernel_size[0] * self.kernel_size[1]
            bound = 1.0 / math.sqrt(fan_in) if fan_in > 0 else 0.0
            nn.init.uniform_(self.bias, -bound, bound)

    def forward(self, input: Tensor, offset: Tensor, mask: Optional[Tensor] = None) -> Tensor:
        return deform_conv2d(input, offset, self.weight, bias=self.bias,
                             stride=self.stride, padding=self.padding,
                             dilation=self.dilation, mask=mask)

    def extra_repr(self) -> str:
        return (f"{self.in_channels}, {self.out_channels}, "
                f"kernel_size={self.kernel_size}, stride={self.stride}, "
                f"padding={self.padding}, dilation={self.dilation}, "
                f"groups={self.groups}, bias={self.bias is not None}")


class DeformConv2dPack(DeformConv2d):
    """A DCNv2 block: a regular convolution predicts the offsets and the
    modulation mask from the input, and the deformable convolution consumes
    them -- the caller pattern of the reference's tests and examples
    (tests/test_training.py:32-47, example/example01_deform_conv2d_cpu_mps.py:80-84).

    ``conv_offset`` (same kernel, stride, padding, dilation) outputs
    ``3 * deformable_groups * kh * kw`` channels: the first
    ``2 * deformable_groups * kh * kw`` are the offsets (the op's layout), the
    rest the mask logits.  The mask's sigmoid is applied inside the CUDA
    kernels (``mask_logits=True``) rather than as a separate pass, and the
    backward returns the logits' gradient directly.  ``modulated=False``
    gives the DCNv1 block (offsets only).  ``conv_offset`` starts at zero:
    a regular convolution at initialisation (mask 0.5 for DCNv2).
    """

    def __init__(self, in_channels: int, out_channels: int, kernel_size, stride=1, padding=0,
                 dilation=1, groups: int = 1, deformable_groups: int = 1, bias: bool = True,
                 modulated: bool = True):
        super().__init__(in_channels, out_channels, kernel_size, stride=stride, padding=padding,
                         dilation=dilation, groups=groups, bias=bias)
        self.deformable_groups = deformable_groups
        self.modulated = modulated
        kh, kw = self.kernel_size
        per_tap = 3 if modulated else 2
        self.conv_offset = nn.Conv2d(in_channels, per_tap * deformable_groups * kh * kw,
                                     self.kernel_size, stride=self.stride, padding=self.padding,
                                     dilation=self.dilation, bias=True)
        nn.init.zeros_(self.conv_offset.weight)
        nn.init.zeros_(self.conv_offset.bias)

    def forward(self, input: Tensor) -> Tensor:  # type: ignore[override]
        kh, kw = self.kernel_size
        n_off = 2 * self.deformable_groups * kh * kw
        om = self.conv_offset(input)
        offset = om[:, :n_off]
        mask = om[:, n_off:] if self.modulated else None
        return deform_conv2d_ex(input, offset, self.weight, self.bias, self.stride,
                                self.padding, self.dilation, mask, mask_logits=self.modulated)
