"""dcn_forward_noalloc: the forward for callers that cannot allocate device
memory (allocator / memory-pool hooks, plugins that only receive input and
output buffers, deployments with device memory fixed at start-up).  It takes
no workspace; its scratch is a 16 MiB array built into libdcn_b200.so.

Checked through the C ABI against dcn_forward (caller-provided workspace) on
two calls in a row, with the tolerance the forward tests use (1e-4), and the
rejection of a shape whose scratch would exceed the built-in array.  This file
is collected last so that a stop-at-first-failure run has run every other
test before it."""
import ctypes

import numpy as np
import pytest
import torch

from _util import make_case
from pytorch_mps_deform_conv2d_b200 import _native

pytestmark = pytest.mark.gpu

DCN_ERR_WORKSPACE = 2


def _lib():
    lib = _native.load_capi()
    lib.dcn_forward_noalloc.argtypes = [ctypes.POINTER(_native.DcnShape)] + \
        [ctypes.c_void_p] * 6 + [ctypes.c_uint32, ctypes.c_void_p]
    lib.dcn_forward_noalloc.restype = ctypes.c_int
    return lib


def _p(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _shape(case):
    x, w = case["x"], case["w"]
    k = w.shape[2] * w.shape[3]
    return _native.DcnShape(
        batch=x.shape[0], in_channels=x.shape[1], height=x.shape[2], width=x.shape[3],
        out_channels=w.shape[0], kernel_h=w.shape[2], kernel_w=w.shape[3],
        stride_h=case["stride"][0], stride_w=case["stride"][1], pad_h=case["padding"][0],
        pad_w=case["padding"][1], dilation_h=case["dilation"][0], dilation_w=case["dilation"][1],
        groups=x.shape[1] // w.shape[1], deformable_groups=case["off"].shape[1] // (2 * k))


def _both(lib, case, dev, flags=0, calls=1):
    d = {k: (v.to(dev) if isinstance(v, torch.Tensor) else v) for k, v in case.items()}
    s = _shape(case)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    want = torch.empty(case["go"].shape, device=dev)
    nbytes = lib.dcn_forward_workspace_size(ctypes.byref(s), flags)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    rc = lib.dcn_forward(ctypes.byref(s), _p(d["x"]), _p(d["w"]), _p(d["off"]), _p(d["m"]),
                         _p(d["b"]), _p(want), flags, _p(ws), nbytes, stream)
    assert rc == 0, _native.capi_error()
    gots = []
    for _ in range(calls):
        got = torch.full(case["go"].shape, float("nan"), device=dev)
        rc = lib.dcn_forward_noalloc(ctypes.byref(s), _p(d["x"]), _p(d["w"]), _p(d["off"]),
                                     _p(d["m"]), _p(d["b"]), _p(got), flags, stream)
        assert rc == 0, _native.capi_error()
        gots.append(got)
    torch.cuda.synchronize()
    if calls == 1:
        return gots[0].cpu().numpy(), want.cpu().numpy()
    return [g.cpu().numpy() for g in gots], want.cpu().numpy()


def test_noalloc_matches_forward_two_calls_in_a_row(cuda_device):
    lib = _lib()
    cases = [make_case(N=2, inC=32, outC=48, H=17, W=19, dg=2, offset_scale=3.0, seed=1),
             make_case(N=1, inC=16, outC=24, H=12, W=10, kh=3, kw=1, stride=(2, 1),
                       pad=(1, 0), use_mask=False, use_bias=False, seed=2)]
    for case in cases:
        got, want = _both(lib, case, cuda_device)
        scale = max(1.0, float(np.abs(want).max()))
        np.testing.assert_allclose(got, want, rtol=1e-4, atol=1e-4 * scale)


# Tensor-core forward through the built-in array: its TMA tensor map is built
# over the array (the packed weight lives there, high and low TF32 parts in
# 3xTF32), and 168 tiles of 128 pixels on 148 SMs leave a last round of 20
# tiles, which the forward splits over the SMs with partial sums kept in the
# rest of the array (a second launch adds them).  Two calls in a row: the
# second one reuses the array's slots and gives the same bits.
@pytest.mark.parametrize("mode", ["tf32", "3xtf32"])
def test_noalloc_tensor_core_split_round_two_calls(cuda_device, mode):
    from pytorch_mps_deform_conv2d_b200.ops import MATH_3XTF32, MATH_TF32
    flags = MATH_TF32 if mode == "tf32" else MATH_3XTF32
    lib = _lib()
    case = make_case(N=1, inC=32, outC=32, H=128, W=168, offset_scale=2.0,
                     mask_kind="sigmoid", seed=4)
    _native.profiler_read()
    _native.profiler_enable(True)
    try:
        gots, want = _both(lib, case, cuda_device, flags=flags, calls=2)
    finally:
        _native.profiler_enable(False)
    stats = _native.profiler_read()
    assert stats.get("fwd_tc", (0, 0.0))[0] == 3, sorted(stats)  # dcn_forward + two calls
    scale = max(1.0, float(np.abs(want).max()))
    for got in gots:
        np.testing.assert_allclose(got, want, rtol=1e-4, atol=1e-4 * scale)


def test_noalloc_rejects_shapes_beyond_its_scratch(cuda_device):
    lib = _lib()
    # NHWC copy alone: 1 x 256 x 128 x 160 x 4 B = 21 MB > 16 MiB
    case = make_case(N=1, inC=256, outC=8, H=128, W=160, seed=3)
    d = {k: (v.to(cuda_device) if isinstance(v, torch.Tensor) else v) for k, v in case.items()}
    out = torch.full(case["go"].shape, 7.0, device=cuda_device)
    rc = lib.dcn_forward_noalloc(ctypes.byref(_shape(case)), _p(d["x"]), _p(d["w"]), _p(d["off"]),
                                 _p(d["m"]), _p(d["b"]), _p(out), 0, None)
    assert rc == DCN_ERR_WORKSPACE
    msg = _native.capi_error()
    assert "16777216" in msg and "scratch" in msg
    torch.cuda.synchronize()
    assert bool((out == 7.0).all())  # nothing was launched
