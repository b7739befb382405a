"""ctypes/numpy front end of the CPU oracle (``dcn_oracle.c``).

TEST INFRASTRUCTURE ONLY.  The oracle restates the reference algorithm of
ilirium/pytorch_mps_deform_conv2d on the CPU (``dcn_oracle.c`` names the
reference file:line of every function).  Results are checked against it:
``tests/``, the smoke entry and the bench's CPU-baseline leg may call it; the product
package never imports it.

All arrays are float32 numpy arrays in the reference's layouts.  ``mask`` and
``bias`` may be ``None`` (DCNv1 / no bias), as in the reference's op
(``src/deform_conv2d_mps/ops.py:118-123``).
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from typing import Optional, Tuple

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "libdcn_oracle.so")
_lib = None

_F = ctypes.POINTER(ctypes.c_float)
_I = ctypes.c_int64


def build() -> str:
    """Compile the oracle with its Makefile (idempotent)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def _load():
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(_LIB_PATH):
        build()
    lib = ctypes.CDLL(_LIB_PATH)
    ints15 = [_I] * 15
    lib.oracle_forward.argtypes = [_F] * 6 + ints15
    lib.oracle_backward.argtypes = [_F] * 10 + ints15
    lib.oracle_col2im.argtypes = [_F] * 4 + [_I] * 12
    lib.oracle_col2im_coord.argtypes = [_F] * 6 + [_I] * 12
    lib.oracle_im2col.argtypes = [_F] * 4 + [_I] * 12
    for f in (lib.oracle_forward, lib.oracle_backward, lib.oracle_col2im,
              lib.oracle_col2im_coord, lib.oracle_im2col):
        f.restype = ctypes.c_int
    _lib = lib
    return lib


def _ptr(a: Optional[np.ndarray]):
    if a is None:
        return ctypes.cast(None, _F)
    assert a.dtype == np.float32 and a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(_F)


def _f32(a):
    if a is None:
        return None
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32))


def _pair(v) -> Tuple[int, int]:
    if isinstance(v, (tuple, list)):
        return int(v[0]), int(v[1])
    return int(v), int(v)


def out_size(H, W, kh, kw, stride, padding, dilation):
    sh, sw = _pair(stride)
    ph, pw = _pair(padding)
    dh, dw = _pair(dilation)
    return ((H + 2 * ph - dh * (kh - 1) - 1) // sh + 1,
            (W + 2 * pw - dw * (kw - 1) - 1) // sw + 1)


def _geometry(x, weight, offset, stride, padding, dilation):
    N, C, H, W = x.shape
    outC, cg, kh, kw = weight.shape
    groups = C // cg
    if cg * groups != C:
        raise ValueError(f"weight shape mismatch: expected in-channels {C}, got {cg * groups}")
    dg = offset.shape[1] // (2 * kh * kw)
    sh, sw = _pair(stride)
    ph, pw = _pair(padding)
    dh, dw = _pair(dilation)
    return (N, C, H, W, outC, kh, kw, sh, sw, ph, pw, dh, dw, groups, dg)


def forward(x, offset, weight, bias=None, stride=1, padding=0, dilation=1,
            mask=None) -> np.ndarray:
    """Reference forward (``deform_conv2d_mps.mm:192-374``)."""
    x, offset, weight, bias, mask = map(_f32, (x, offset, weight, bias, mask))
    geo = _geometry(x, weight, offset, stride, padding, dilation)
    N, C, H, W, outC, kh, kw, sh, sw, ph, pw, dh, dw, groups, dg = geo
    Ho, Wo = out_size(H, W, kh, kw, (sh, sw), (ph, pw), (dh, dw))
    out = np.zeros((N, outC, Ho, Wo), np.float32)
    rc = _load().oracle_forward(_ptr(x), _ptr(weight), _ptr(offset),
                                _ptr(mask), _ptr(bias), _ptr(out), *geo)
    if rc != 0:
        raise ValueError(f"oracle_forward rejected the geometry (rc={rc})")
    return out


def backward(grad_out, x, offset, weight, bias=None, stride=1, padding=0,
             dilation=1, mask=None):
    """Reference backward (``deform_conv2d_mps.mm:682-890``).

    Returns ``(grad_input, grad_offset, grad_mask, grad_weight, grad_bias)``
    with ``None`` for an absent mask / bias.
    """
    grad_out, x, offset, weight, bias, mask = map(
        _f32, (grad_out, x, offset, weight, bias, mask))
    geo = _geometry(x, weight, offset, stride, padding, dilation)
    gx = np.zeros_like(x)
    goff = np.zeros_like(offset)
    gmsk = np.zeros_like(mask) if mask is not None else None
    gw = np.zeros_like(weight)
    gb = np.zeros_like(bias) if bias is not None else None
    rc = _load().oracle_backward(_ptr(grad_out), _ptr(x), _ptr(weight),
                                 _ptr(offset), _ptr(mask), _ptr(gx),
                                 _ptr(goff), _ptr(gmsk), _ptr(gw), _ptr(gb),
                                 *geo)
    if rc != 0:
        raise ValueError(f"oracle_backward rejected the geometry (rc={rc})")
    return gx, goff, gmsk, gw, gb


def _single_geo(kh, kw, stride, padding, dilation):
    sh, sw = _pair(stride)
    ph, pw = _pair(padding)
    dh, dw = _pair(dilation)
    return (kh, kw, sh, sw, ph, pw, dh, dw)


def im2col(im, offset, mask, kh, kw, stride=1, padding=0, dilation=1):
    """Column buffer (C*kh*kw, Ho*Wo) of one image (``deform_conv2d.metal:74-125``)."""
    im, offset, mask = map(_f32, (im, offset, mask))
    C, H, W = im.shape
    dg = offset.shape[0] // (2 * kh * kw)
    Ho, Wo = out_size(H, W, kh, kw, stride, padding, dilation)
    col = np.zeros((C * kh * kw, Ho * Wo), np.float32)
    rc = _load().oracle_im2col(_ptr(im), _ptr(offset), _ptr(mask), _ptr(col),
                               C, H, W, *_single_geo(kh, kw, stride, padding,
                                                     dilation), dg)
    if rc != 0:
        raise ValueError("oracle_im2col rejected the geometry")
    return col


def col2im(columns, offset, mask, H, W, kh, kw, stride=1, padding=0,
           dilation=1):
    """grad_input (C, H, W) of one image (``deform_conv2d.metal:141-204``)."""
    columns, offset, mask = map(_f32, (columns, offset, mask))
    C = columns.shape[0] // (kh * kw)
    dg = offset.shape[0] // (2 * kh * kw)
    gim = np.zeros((C, H, W), np.float32)
    rc = _load().oracle_col2im(_ptr(columns), _ptr(offset), _ptr(mask),
                               _ptr(gim), C, H, W,
                               *_single_geo(kh, kw, stride, padding, dilation),
                               dg)
    if rc != 0:
        raise ValueError("oracle_col2im rejected the geometry")
    return gim


def col2im_coord(columns, im, offset, mask, kh, kw, stride=1, padding=0,
                 dilation=1):
    """(grad_offset, grad_mask) of one image (``deform_conv2d.metal:225-295``)."""
    columns, im, offset, mask = map(_f32, (columns, im, offset, mask))
    C, H, W = im.shape
    dg = offset.shape[0] // (2 * kh * kw)
    goff = np.zeros_like(offset)
    gmsk = np.zeros_like(mask) if mask is not None else None
    rc = _load().oracle_col2im_coord(_ptr(columns), _ptr(im), _ptr(offset),
                                     _ptr(mask), _ptr(goff), _ptr(gmsk),
                                     C, H, W,
                                     *_single_geo(kh, kw, stride, padding,
                                                  dilation), dg)
    if rc != 0:
        raise ValueError("oracle_col2im_coord rejected the geometry")
    return goff, gmsk
