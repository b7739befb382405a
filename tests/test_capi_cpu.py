"""The C-ABI library loads, exports every entry point include/dcn_b200.h
declares, and validates its arguments on the host (no kernel is launched in
this file; it runs without a GPU)."""
import ctypes
import os
import re

import pytest

from pytorch_mps_deform_conv2d_b200 import _native

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "dcn_b200.h")


def _declared():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"DCN_API\s+[\w\s\*]+?\b(dcn_\w+)\s*\(", text)))


def _shape(**kw):
    base = dict(batch=2, in_channels=4, height=9, width=9, out_channels=6,
                kernel_h=3, kernel_w=3, stride_h=1, stride_w=1, pad_h=1, pad_w=1,
                dilation_h=1, dilation_w=1, groups=1, deformable_groups=1)
    base.update(kw)
    return _native.DcnShape(**base)


def test_header_declares_the_reference_ops():
    names = _declared()
    for name in ("dcn_forward", "dcn_backward", "dcn_col2im", "dcn_col2im_coord",
                 "dcn_forward_workspace_size", "dcn_backward_workspace_size",
                 "dcn_output_size", "dcn_last_error", "dcn_abi_version"):
        assert name in names


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(_native.LIB_PATH)
    for name in _declared():
        assert hasattr(lib, name), f"{name} declared in dcn_b200.h but not exported"


def test_library_exports_nothing_else():
    # -fvisibility=hidden: only the C ABI is visible
    out = os.popen(f"nm -D --defined-only {_native.LIB_PATH}").read()
    exported = {l.split()[-1] for l in out.splitlines() if " T " in l}
    assert exported == set(_declared())


def test_abi_version_and_output_size():
    lib = _native.load_capi()
    assert lib.dcn_abi_version() == 1
    ho, wo = ctypes.c_int64(), ctypes.c_int64()
    s = _shape(height=8, width=11, kernel_h=1, kernel_w=3, stride_h=2, stride_w=1,
               pad_h=0, pad_w=2, dilation_h=2, dilation_w=1)
    assert lib.dcn_output_size(ctypes.byref(s), ctypes.byref(ho), ctypes.byref(wo)) == 0
    assert (ho.value, wo.value) == ((8 - 1) // 2 + 1, (11 + 4 - 2 - 1) // 1 + 1)


def test_workspace_sizes_cover_scratch():
    lib = _native.load_capi()
    s = _shape(batch=2, in_channels=256, height=100, width=152, out_channels=256)
    nhwc = 2 * 256 * 100 * 152 * 4
    assert lib.dcn_forward_workspace_size(ctypes.byref(s), 0) >= nhwc
    assert lib.dcn_backward_workspace_size(ctypes.byref(s), 0) >= 2 * nhwc


@pytest.mark.parametrize("bad,msg", [
    (dict(groups=0), "groups must be positive"),
    (dict(stride_h=0), "stride must be positive"),
    (dict(dilation_w=0), "dilation must be positive"),
    (dict(in_channels=5, groups=2), "not divisible by groups"),
    (dict(out_channels=5, groups=2), "out_channels (5) not divisible by groups"),
    (dict(deformable_groups=3), "not divisible by deformable_groups"),
    (dict(deformable_groups=0), "deformable_groups must be positive"),
    (dict(height=1, width=1, pad_h=0, pad_w=0), "is non-positive"),
])
def test_invalid_geometry_rejected(bad, msg):
    lib = _native.load_capi()
    s = _shape(**bad)
    rc = lib.dcn_forward(ctypes.byref(s), None, None, None, None, None, None, 0, None, 0, None)
    assert rc == 1  # DCN_ERR_INVALID_ARGUMENT
    assert msg in _native.capi_error()


def test_host_pointers_rejected():
    lib = _native.load_capi()
    s = _shape()
    buf = (ctypes.c_float * 4096)()
    p = ctypes.cast(buf, ctypes.c_void_p)
    rc = lib.dcn_forward(ctypes.byref(s), p, p, p, None, None, p, 0, p, 4096 * 4, None)
    assert rc == 1
    assert "CUDA" in _native.capi_error()
