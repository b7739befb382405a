"""Parity through the C ABI itself (ctypes on libdcn_b200.so, torch only for
device memory and the stream): dcn_forward, dcn_backward, dcn_col2im and
dcn_col2im_coord against the oracle."""
import ctypes

import numpy as np
import pytest
import torch

from _util import assert_close, make_case, np_, run_oracle
from oracle import oracle
from pytorch_mps_deform_conv2d_b200 import _native

pytestmark = pytest.mark.gpu


def _p(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _shape(case):
    x, w = case["x"], case["w"]
    return _native.DcnShape(
        batch=x.shape[0], in_channels=x.shape[1], height=x.shape[2], width=x.shape[3],
        out_channels=w.shape[0], kernel_h=w.shape[2], kernel_w=w.shape[3],
        stride_h=case["stride"][0], stride_w=case["stride"][1], pad_h=case["padding"][0],
        pad_w=case["padding"][1], dilation_h=case["dilation"][0], dilation_w=case["dilation"][1],
        groups=x.shape[1] // w.shape[1], deformable_groups=case["off"].shape[1] // (2 * w.shape[2] * w.shape[3]))


@pytest.mark.parametrize("kw", [dict(), dict(inC=32, outC=40, dg=2, offset_scale=3.0),
                                dict(use_mask=False, use_bias=False, groups=2, inC=8, outC=8)])
def test_capi_forward_backward(cuda_device, kw):
    lib = _native.load_capi()
    case = make_case(**kw)
    d = {k: (v.to(cuda_device) if isinstance(v, torch.Tensor) else v) for k, v in case.items()}
    s = _shape(case)
    ho, wo = ctypes.c_int64(), ctypes.c_int64()
    assert lib.dcn_output_size(ctypes.byref(s), ctypes.byref(ho), ctypes.byref(wo)) == 0
    out = torch.empty(case["go"].shape, device=cuda_device)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    nbytes = lib.dcn_forward_workspace_size(ctypes.byref(s), 0)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=cuda_device)
    rc = lib.dcn_forward(ctypes.byref(s), _p(d["x"]), _p(d["w"]), _p(d["off"]), _p(d["m"]),
                         _p(d["b"]), _p(out), 0, _p(ws), nbytes, stream)
    assert rc == 0, _native.capi_error()
    ref, rg = run_oracle(case)
    assert_close(np_(out), ref, rtol=1e-4, atol=1e-4 * max(1, np.abs(ref).max()))

    gx = torch.empty_like(d["x"])
    goff = torch.empty_like(d["off"])
    gm = torch.empty_like(d["m"]) if d["m"] is not None else None
    gw = torch.empty_like(d["w"])
    gb = torch.empty_like(d["b"]) if d["b"] is not None else None
    nbytes = lib.dcn_backward_workspace_size(ctypes.byref(s), 0)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=cuda_device)
    rc = lib.dcn_backward(ctypes.byref(s), _p(d["go"]), _p(d["x"]), _p(d["w"]), _p(d["off"]),
                          _p(d["m"]), _p(gx), _p(goff), _p(gm), _p(gw), _p(gb), 0, _p(ws), nbytes,
                          stream)
    assert rc == 0, _native.capi_error()
    torch.cuda.synchronize()
    got = dict(x=gx, off=goff, w=gw, m=gm, b=gb)
    for k, want in rg.items():
        tol = 2e-3 if k == "x" else 1e-4
        assert_close(np_(got[k]), want, rtol=tol, atol=tol * max(1, np.abs(want).max()), name=k)


def test_capi_workspace_too_small(cuda_device):
    lib = _native.load_capi()
    case = make_case(inC=16, outC=16)
    d = {k: (v.to(cuda_device) if isinstance(v, torch.Tensor) else v) for k, v in case.items()}
    s = _shape(case)
    out = torch.empty(case["go"].shape, device=cuda_device)
    ws = torch.empty(64, dtype=torch.uint8, device=cuda_device)
    rc = lib.dcn_forward(ctypes.byref(s), _p(d["x"]), _p(d["w"]), _p(d["off"]), _p(d["m"]),
                         _p(d["b"]), _p(out), 0, _p(ws), 64, None)
    assert rc == 2 and "workspace" in _native.capi_error()


@pytest.mark.parametrize("use_mask,dg", [(True, 1), (False, 2), (True, 2)])
def test_capi_col2im_and_coord(cuda_device, use_mask, dg):
    """The single-image ops (reference debug ops .mm:388-651) against the
    oracle's col2im / col2im_coord."""
    lib = _native.load_capi()
    torch.manual_seed(3)
    C, H, W, k = 4, 9, 10, 3
    Ho, Wo = oracle.out_size(H, W, k, k, 1, 1, 1)
    col = torch.randn(C * k * k, Ho * Wo)
    im = torch.randn(C, H, W)
    off = 2.0 * torch.randn(2 * dg * k * k, Ho, Wo)
    m = torch.rand(dg * k * k, Ho, Wo) if use_mask else None
    dev = lambda t: t.to(cuda_device) if t is not None else None
    colg, img, offg, mg = map(dev, (col, im, off, m))
    gim = torch.full((C, H, W), float("nan"), device=cuda_device)
    rc = lib.dcn_col2im(_p(colg), _p(offg), _p(mg), _p(gim), C, H, W, k, k, 1, 1, 1, 1, 1, 1,
                        dg, None)
    assert rc == 0, _native.capi_error()
    goff = torch.empty_like(offg)
    gm = torch.empty_like(mg) if use_mask else None
    rc = lib.dcn_col2im_coord(_p(colg), _p(img), _p(offg), _p(mg), _p(goff), _p(gm), C, H, W,
                              k, k, 1, 1, 1, 1, 1, 1, dg, None)
    assert rc == 0, _native.capi_error()
    torch.cuda.synchronize()
    ref_im = oracle.col2im(col.numpy(), off.numpy(), np_(m), H, W, k, k, 1, 1, 1)
    ref_off, ref_m = oracle.col2im_coord(col.numpy(), im.numpy(), off.numpy(), np_(m), k, k, 1, 1, 1)
    assert_close(np_(gim), ref_im, rtol=1e-4, atol=1e-4)
    assert_close(np_(goff), ref_off, rtol=1e-4, atol=1e-4)
    if use_mask:
        assert_close(np_(gm), ref_m, rtol=1e-4, atol=1e-4)


def test_torch_debug_ops_match_oracle(cuda_device):
    ops = _native.load_ops()
    torch.manual_seed(4)
    C, H, W, k = 6, 8, 11, 3
    Ho, Wo = oracle.out_size(H, W, k, k, (2, 1), (0, 2), (2, 1))
    col = torch.randn(C * k * k, Ho * Wo)
    im = torch.randn(C, H, W)
    off = torch.randn(2 * 3 * k * k, Ho, Wo)
    m = torch.rand(3 * k * k, Ho, Wo)
    g = lambda t: t.to(cuda_device)
    gim = ops.deformable_col2im(g(col), g(off), g(m), H, W, k, k, 2, 1, 0, 2, 2, 1, 3)
    goff, gm = ops.deformable_col2im_coord(g(col), g(im), g(off), g(m), k, k, 2, 1, 0, 2, 2, 1, 3)
    assert_close(np_(gim), oracle.col2im(col.numpy(), off.numpy(), m.numpy(), H, W, k, k, (2, 1),
                                         (0, 2), (2, 1)), rtol=1e-4, atol=1e-4)
    ro, rm = oracle.col2im_coord(col.numpy(), im.numpy(), off.numpy(), m.numpy(), k, k, (2, 1),
                                 (0, 2), (2, 1))
    assert_close(np_(goff), ro, rtol=1e-4, atol=1e-4)
    assert_close(np_(gm), rm, rtol=1e-4, atol=1e-4)
