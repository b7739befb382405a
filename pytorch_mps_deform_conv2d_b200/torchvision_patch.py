"""Route ``torchvision.ops.deform_conv2d`` / ``torchvision.ops.DeformConv2d``
to this package for CUDA tensors.

The reference's goal is drop-in torchvision compatibility (its
``deform_conv2d`` has torchvision's signature, src/deform_conv2d_mps/ops.py:
126-135).  ``patch_torchvision()`` goes one step further for code that calls
torchvision directly: it replaces ``torchvision.ops.deform_conv2d`` (and the
name ``torchvision.ops.deform_conv.deform_conv2d`` that
``torchvision.ops.DeformConv2d.forward`` calls) with a router that sends
calls whose tensors are on a CUDA device to :func:`deform_conv2d` of this
package and everything else to torchvision's original function, unchanged.
``unpatch_torchvision()`` restores the original.
"""
from __future__ import annotations

import functools
import threading

from .ops import deform_conv2d as _ours

_lock = threading.Lock()
_original = None


def _route(original):
    @functools.wraps(original)
    def deform_conv2d(input, offset, weight, bias=None, stride=(1, 1), padding=(0, 0),
                      dilation=(1, 1), mask=None):
        if input.is_cuda:
            return _ours(input, offset, weight, bias=bias, stride=stride, padding=padding,
                         dilation=dilation, mask=mask)
        return original(input, offset, weight, bias=bias, stride=stride, padding=padding,
                        dilation=dilation, mask=mask)

    deform_conv2d.__wrapped_torchvision__ = original
    return deform_conv2d


def patch_torchvision() -> None:
    """Install the router (idempotent)."""
    global _original
    import torchvision.ops as tv_ops
    import torchvision.ops.deform_conv as tv_dc
    with _lock:
        if _original is not None:
            return
        _original = tv_dc.deform_conv2d
        routed = _route(_original)
        tv_dc.deform_conv2d = routed
        tv_ops.deform_conv2d = routed


def unpatch_torchvision() -> None:
    """Restore torchvision's own function (idempotent)."""
    global _original
    import torchvision.ops as tv_ops
    import torchvision.ops.deform_conv as tv_dc
    with _lock:
        if _original is None:
            return
        tv_dc.deform_conv2d = _original
        tv_ops.deform_conv2d = _original
        _original = None


def is_patched() -> bool:
    return _original is not None
