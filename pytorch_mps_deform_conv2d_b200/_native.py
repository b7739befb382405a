"""Loading of the in-tree native libraries.

``lib/libdcn_b200.so`` holds every CUDA kernel and the C ABI of
``include/dcn_b200.h``; ``lib/libdcn_b200_torch.so`` registers the
``torch.ops.deform_conv2d_b200`` operators on top of it.  Both are built by
``pytorch_mps_deform_conv2d_b200._build``.  There is no fallback: when a
library is missing or fails to load, every entry point raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "lib", "libdcn_b200.so")
TORCH_LIB_PATH = os.path.join(_PKG, "lib", "libdcn_b200_torch.so")

_lock = threading.Lock()
_ops_loaded = False
_capi = None


class NativeLibraryError(RuntimeError):
    """The CUDA extension of pytorch_mps_deform_conv2d_b200 is unavailable."""


def _missing(path: str) -> NativeLibraryError:
    return NativeLibraryError(
        f"{path} is missing: build the CUDA extension first with "
        "`python -m pytorch_mps_deform_conv2d_b200._build` (nvcc, sm_100a)")


def load_ops():
    """Load the operator library once; returns ``torch.ops.deform_conv2d_b200``."""
    global _ops_loaded
    import torch
    with _lock:
        if not _ops_loaded:
            if not os.path.exists(TORCH_LIB_PATH):
                raise _missing(TORCH_LIB_PATH)
            torch.ops.load_library(TORCH_LIB_PATH)
            from . import _registrations
            _registrations.register()
            _ops_loaded = True
    return torch.ops.deform_conv2d_b200


class DcnShape(ctypes.Structure):
    """``dcn_shape`` of include/dcn_b200.h."""
    _fields_ = [(name, ctypes.c_int64) for name in (
        "batch", "in_channels", "height", "width", "out_channels", "kernel_h",
        "kernel_w", "stride_h", "stride_w", "pad_h", "pad_w", "dilation_h",
        "dilation_w", "groups", "deformable_groups")]


class KernelStat(ctypes.Structure):
    """``dcn_kernel_stat`` of include/dcn_b200.h."""
    _fields_ = [("name", ctypes.c_char * 48), ("launches", ctypes.c_int64),
                ("total_ms", ctypes.c_double)]


def load_capi():
    """ctypes handle of libdcn_b200.so with the C ABI prototypes set."""
    global _capi
    with _lock:
        if _capi is not None:
            return _capi
        if not os.path.exists(LIB_PATH):
            raise _missing(LIB_PATH)
        lib = ctypes.CDLL(LIB_PATH)
        vp, sz, u32, i64 = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_uint32, ctypes.c_int64
        shp = ctypes.POINTER(DcnShape)
        lib.dcn_abi_version.restype = ctypes.c_int
        lib.dcn_last_error.restype = ctypes.c_char_p
        lib.dcn_output_size.argtypes = [shp, ctypes.POINTER(i64), ctypes.POINTER(i64)]
        lib.dcn_output_size.restype = ctypes.c_int
        lib.dcn_forward_workspace_size.argtypes = [shp, u32]
        lib.dcn_forward_workspace_size.restype = sz
        lib.dcn_backward_workspace_size.argtypes = [shp, u32]
        lib.dcn_backward_workspace_size.restype = sz
        lib.dcn_forward.argtypes = [shp] + [vp] * 6 + [u32, vp, sz, vp]
        lib.dcn_forward.restype = ctypes.c_int
        lib.dcn_backward.argtypes = [shp] + [vp] * 10 + [u32, vp, sz, vp]
        lib.dcn_backward.restype = ctypes.c_int
        lib.dcn_forward_bf16_workspace_size.argtypes = [shp, u32]
        lib.dcn_forward_bf16_workspace_size.restype = sz
        lib.dcn_forward_bf16.argtypes = [shp] + [vp] * 6 + [u32, vp, sz, vp]
        lib.dcn_forward_bf16.restype = ctypes.c_int
        lib.dcn_backward_bf16_workspace_size.argtypes = [shp, u32]
        lib.dcn_backward_bf16_workspace_size.restype = sz
        lib.dcn_backward_bf16.argtypes = [shp] + [vp] * 10 + [u32, vp, sz, vp]
        lib.dcn_backward_bf16.restype = ctypes.c_int
        lib.dcn_forward_f16_workspace_size.argtypes = [shp, u32]
        lib.dcn_forward_f16_workspace_size.restype = sz
        lib.dcn_forward_f16.argtypes = [shp] + [vp] * 6 + [u32, vp, sz, vp]
        lib.dcn_forward_f16.restype = ctypes.c_int
        lib.dcn_backward_f16_workspace_size.argtypes = [shp, u32]
        lib.dcn_backward_f16_workspace_size.restype = sz
        lib.dcn_backward_f16.argtypes = [shp] + [vp] * 10 + [u32, vp, sz, vp]
        lib.dcn_backward_f16.restype = ctypes.c_int
        lib.dcn_col2im.argtypes = [vp] * 4 + [i64] * 12 + [vp]
        lib.dcn_col2im.restype = ctypes.c_int
        lib.dcn_col2im_coord.argtypes = [vp] * 6 + [i64] * 12 + [vp]
        lib.dcn_col2im_coord.restype = ctypes.c_int
        lib.dcn_device_status.argtypes = [vp, ctypes.c_int, ctypes.POINTER(ctypes.c_int)]
        lib.dcn_device_status.restype = ctypes.c_int
        lib.dcn_l2_probe.argtypes = [ctypes.c_int, vp, ctypes.c_size_t, ctypes.c_int, vp]
        lib.dcn_l2_probe.restype = ctypes.c_int
        lib.dcn_profiler_enable.argtypes = [ctypes.c_int]
        lib.dcn_profiler_enable.restype = ctypes.c_int
        lib.dcn_profiler_read.argtypes = [ctypes.POINTER(KernelStat), ctypes.c_int,
                                          ctypes.POINTER(ctypes.c_int)]
        lib.dcn_profiler_read.restype = ctypes.c_int
        _capi = lib
        return lib


def capi_error() -> str:
    return load_capi().dcn_last_error().decode()


def profiler_enable(on: bool = True) -> None:
    """Bracket every kernel launch of the library with CUDA events."""
    load_capi().dcn_profiler_enable(1 if on else 0)


def profiler_read(max_kernels: int = 64):
    """Per-kernel ``{name: (launches, total_ms)}`` since the last read
    (waits for the recorded events)."""
    lib = load_capi()
    stats = (KernelStat * max_kernels)()
    count = ctypes.c_int(0)
    rc = lib.dcn_profiler_read(stats, max_kernels, ctypes.byref(count))
    if rc != 0:
        raise RuntimeError(capi_error())
    return {stats[i].name.decode(): (int(stats[i].launches), float(stats[i].total_ms))
            for i in range(min(count.value, max_kernels))}
