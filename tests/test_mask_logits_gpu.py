"""DCNv2 block fusion: the mask's sigmoid inside the kernels (DCN_MASK_LOGITS).
Fused (mask logits given to the op) against unfused (torch.sigmoid, then the
op) on every kernel family and math mode -- forward and all five gradients,
the logits' gradient through torch's sigmoid backward in the unfused run --
plus oracle parity of the fused path and the DeformConv2dPack module."""
import numpy as np
import pytest
import torch

import pytorch_mps_deform_conv2d_b200 as dcn
from _util import assert_close, make_case, run_oracle
from pytorch_mps_deform_conv2d_b200 import _native
from pytorch_mps_deform_conv2d_b200.ops import (ALGO_SIMT_DIRECT, ALGO_SIMT_GEMM,
                                                ALGO_TC_COLUMN_BUFFER, ALGO_TC_GATHER_WEIGHT, MATH_3XTF32, MATH_FP32,
                                                MATH_TF32, deform_conv2d_ex)

pytestmark = pytest.mark.gpu

# name -> (case, flags, kernels that must run)
CASES = {
    "tc-tf32": (dict(inC=128, outC=64, H=10, W=9, offset_scale=2.0), MATH_TF32,
                ("fwd_tc", "bwd_fused_tc")),
    "tc-tf32-column-buffer": (dict(inC=128, outC=64, H=10, W=9, offset_scale=2.0),
                              MATH_TF32 | ALGO_TC_COLUMN_BUFFER,
                              ("fwd_tc", "bwd_data_tc", "bwd_weight_col")),
    "tc-tf32-gather-weight": (dict(inC=128, outC=64, H=10, W=9, offset_scale=2.0),
                              MATH_TF32 | ALGO_TC_GATHER_WEIGHT, ("bwd_weight_tc",)),
    "tc-3xtf32-cg64": (dict(inC=64, outC=64, H=9, W=11, offset_scale=2.0), MATH_3XTF32,
                       ("fwd_tc", "bwd_data_tc")),
    "simt-fp32": (dict(inC=8, outC=12, H=9, W=10, dg=2, offset_scale=2.0), MATH_FP32,
                  ("bwd_data_simt", "bwd_weight_simt")),
    "simt-gemm-fp32": (dict(inC=6, outC=6, H=8, W=9, offset_scale=2.0),
                       MATH_FP32 | ALGO_SIMT_GEMM, ("fwd_simt_gemm", "bwd_data_simt")),
    "dgroup": (dict(inC=32, outC=32, groups=16, dg=2, H=9, W=10, offset_scale=2.0), MATH_FP32,
               ("fwd_dgroup", "bwd_dgroup")),
    "small-direct": (dict(inC=6, outC=6, groups=3, H=8, W=9, offset_scale=2.0),
                     MATH_FP32 | ALGO_SIMT_DIRECT, ("fwd_simt_direct", "bwd_small")),
}


def _leaves(case, logits):
    d = lambda t: None if t is None else t.cuda().requires_grad_(True)
    return d(case["x"]), d(case["off"]), d(case["w"]), d(case["b"]), d(logits)


def _run(case, flags, logits, fused):
    x, off, w, b, lg = _leaves(case, logits)
    mask = lg if fused else torch.sigmoid(lg)
    out = deform_conv2d_ex(x, off, w, b, case["stride"], case["padding"], case["dilation"],
                           mask, flags=flags, mask_logits=fused)
    out.backward(case["go"].cuda())
    torch.cuda.synchronize()
    return out.detach().cpu(), {k: t.grad.cpu() for k, t in
                                (("x", x), ("off", off), ("w", w), ("b", b), ("m", lg))}


@pytest.mark.parametrize("name", sorted(CASES))
def test_fused_sigmoid_matches_unfused(cuda_device, name):
    spec, flags, kernels = CASES[name]
    case = make_case(upstream="randn", **spec)
    logits = 2.0 * torch.randn(case["m"].shape, generator=torch.Generator().manual_seed(7))
    _native.profiler_read()
    _native.profiler_enable(True)
    try:
        out_f, g_f = _run(case, flags, logits, fused=True)
    finally:
        _native.profiler_enable(False)
    stats = _native.profiler_read()
    for k in kernels:
        assert k in stats, (k, sorted(stats))
    out_u, g_u = _run(case, flags, logits, fused=False)
    torch.testing.assert_close(out_f, out_u, rtol=1e-4, atol=1e-5 * max(1.0, out_u.abs().max()))
    for k in g_u:
        s = max(1.0, float(g_u[k].abs().max()))
        torch.testing.assert_close(g_f[k], g_u[k], rtol=1e-3, atol=1e-4 * s, msg=f"grad_{k}")


def test_fused_sigmoid_oracle_parity(cuda_device):
    case = make_case(inC=8, outC=6, H=9, W=10, upstream="randn", offset_scale=2.0)
    logits = 2.0 * torch.randn(case["m"].shape, generator=torch.Generator().manual_seed(3))
    out, grads = _run(case, MATH_FP32, logits, fused=True)
    sig = torch.sigmoid(logits)
    ocase = dict(case, m=sig)
    ref, rg = run_oracle(ocase)
    scale = max(1.0, float(np.abs(ref).max()))
    assert_close(out.numpy(), ref, rtol=1e-4, atol=1e-4 * scale, name="out")
    # chain rule through the sigmoid for the mask's gradient
    want_m = rg["m"] * (sig * (1 - sig)).numpy()
    assert_close(grads["m"].numpy(), want_m, rtol=1e-4, atol=1e-4 * max(1.0, np.abs(want_m).max()),
                 name="grad_logits")
    for k, tol in (("x", 2e-3), ("off", 1e-4), ("w", 1e-4), ("b", 1e-4)):
        s = max(1.0, float(np.abs(rg[k]).max()))
        assert_close(grads[k].numpy(), rg[k], rtol=tol, atol=tol * s, name=f"grad_{k}")


@pytest.mark.parametrize("modulated", [True, False])
def test_pack_module_matches_composition(cuda_device, modulated):
    torch.manual_seed(0)
    mod = dcn.DeformConv2dPack(16, 8, 3, padding=1, deformable_groups=2,
                               modulated=modulated).cuda()
    with torch.no_grad():  # non-trivial offsets and masks
        mod.conv_offset.weight.normal_(0, 0.05)
        mod.conv_offset.bias.normal_(0, 0.5)
    x = torch.randn(2, 16, 9, 10, device="cuda", requires_grad=True)
    dcn.set_math_mode("fp32")
    try:
        out = mod(x)
        go = torch.randn_like(out)
        out.backward(go)
        got = [out.detach(), x.grad.clone()] + [p.grad.clone() for p in mod.parameters()]
        x.grad = None
        mod.zero_grad()
        om = mod.conv_offset(x)
        n_off = 2 * 2 * 9
        mask = torch.sigmoid(om[:, n_off:]) if modulated else None
        ref = dcn.deform_conv2d(x, om[:, :n_off], mod.weight, mod.bias, padding=1, mask=mask)
        ref.backward(go)
        want = [ref.detach(), x.grad.clone()] + [p.grad.clone() for p in mod.parameters()]
    finally:
        dcn.set_math_mode(None)
    for a, b in zip(got, want):
        torch.testing.assert_close(a, b, rtol=1e-4, atol=1e-4 * max(1.0, float(b.abs().max())))
