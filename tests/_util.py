"""Shared helpers of the test suite: seeded input factories in the style of
the reference's tests (tests/test_forward.py:102-132,
tests/test_backward.py:50-106) and comparison helpers."""
from __future__ import annotations

import numpy as np
import torch


def pair(v):
    return (v, v) if isinstance(v, int) else tuple(v)


def make_case(N=2, inC=4, outC=6, H=9, W=9, kh=3, kw=3, stride=1, pad=1, dil=1,
              use_mask=True, use_bias=True, dg=1, groups=1, offset_scale=1.0,
              upstream="randn", seed=0, mask_kind="rand", weight_kind="randn"):
    """Seeded CPU tensors x, w, b, offset, mask, grad_out and the conv args."""
    torch.manual_seed(seed)
    sh, sw = pair(stride)
    ph, pw = pair(pad)
    dh, dw = pair(dil)
    Ho = (H + 2 * ph - dh * (kh - 1) - 1) // sh + 1
    Wo = (W + 2 * pw - dw * (kw - 1) - 1) // sw + 1
    x = torch.randn(N, inC, H, W)
    if weight_kind == "kaiming":
        w = torch.empty(outC, inC // groups, kh, kw)
        torch.nn.init.kaiming_uniform_(w, a=5 ** 0.5)
    else:
        w = torch.randn(outC, inC // groups, kh, kw)
    b = torch.randn(outC) if use_bias else None
    off = offset_scale * torch.randn(N, 2 * dg * kh * kw, Ho, Wo)
    m = None
    if use_mask:
        m = (torch.rand(N, dg * kh * kw, Ho, Wo) if mask_kind == "rand"
             else torch.sigmoid(torch.randn(N, dg * kh * kw, Ho, Wo)))
    if upstream == "sum":
        go = torch.ones(N, outC, Ho, Wo)
    else:
        go = torch.randn(N, outC, Ho, Wo)
    return dict(x=x, w=w, b=b, off=off, m=m, go=go, stride=(sh, sw),
                padding=(ph, pw), dilation=(dh, dw))


def np_(t):
    return None if t is None else t.detach().cpu().numpy()


def scaled_err(got, want):
    """max |got - want| / max(1, max |want|)."""
    got, want = np.asarray(got, np.float64), np.asarray(want, np.float64)
    if want.size == 0:
        return 0.0
    return float(np.abs(got - want).max() / max(1.0, np.abs(want).max()))


def rel_norm_err(got, want):
    """||got - want|| / ||want|| (norm-wise relative error)."""
    got, want = np.asarray(got, np.float64), np.asarray(want, np.float64)
    den = np.linalg.norm(want)
    return float(np.linalg.norm(got - want) / (den if den > 0 else 1.0))


def assert_close(got, want, rtol, atol, name=""):
    got, want = np.asarray(got), np.asarray(want)
    assert got.shape == want.shape, f"{name}: shape {got.shape} vs {want.shape}"
    np.testing.assert_allclose(got, want, rtol=rtol, atol=atol, err_msg=name)


def run_ours(case, flags=None, device="cuda", backward=True):
    """Forward (+ backward with the case's grad_out) through the public
    functional API on `device`; returns numpy out and grads dict."""
    from pytorch_mps_deform_conv2d_b200.ops import deform_conv2d_ex
    leaves = {}
    for k in ("x", "w", "b", "off", "m"):
        t = case[k]
        leaves[k] = None if t is None else t.to(device).requires_grad_(backward)
    out = deform_conv2d_ex(leaves["x"], leaves["off"], leaves["w"], leaves["b"],
                           case["stride"], case["padding"], case["dilation"], leaves["m"],
                           flags=flags)
    grads = {}
    if backward:
        out.backward(case["go"].to(device))
        grads = {k: np_(v.grad) for k, v in leaves.items() if v is not None}
    torch.cuda.synchronize()
    return np_(out), grads


def run_oracle(case, backward=True):
    from oracle import oracle
    args = dict(stride=case["stride"], padding=case["padding"], dilation=case["dilation"])
    out = oracle.forward(np_(case["x"]), np_(case["off"]), np_(case["w"]), np_(case["b"]),
                         mask=np_(case["m"]), **args)
    grads = {}
    if backward:
        gx, goff, gm, gw, gb = oracle.backward(np_(case["go"]), np_(case["x"]), np_(case["off"]),
                                               np_(case["w"]), np_(case["b"]), mask=np_(case["m"]),
                                               **args)
        grads = dict(x=gx, off=goff, w=gw)
        if gm is not None:
            grads["m"] = gm
        if gb is not None:
            grads["b"] = gb
    return out, grads


def staging_launches(stats):
    """Launches that staged an input as its NHWC copy, by the library's
    profiler: the plain transpose / copy, or the tensor-core forward's
    prologue that stages and packs the weight in one launch."""
    return sum(stats[k][0] for k in ("nchw_to_nhwc", "copy_nhwc", "fwd_prologue") if k in stats)
