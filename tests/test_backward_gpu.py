"""Backward parity on the GPU against the CPU oracle, per gradient, with the
reference's per-gradient tolerances (tests/test_backward.py:41-47):
grad_input 2e-3 (atomic scatter order), offset / mask / weight / bias 1e-4.
Matrix of tests/test_backward.py:115-130, the non-scalar upstream gradient
(:137-140), the extras (:148-196), the routing asserts (:210-242) and an fp32
gradcheck with its CPU calibration twin (:256-344)."""
import numpy as np
import pytest
import torch

from _util import assert_close, make_case, run_oracle, run_ours
from pytorch_mps_deform_conv2d_b200.ops import ALGO_SIMT_GEMM, MATH_FP32

pytestmark = pytest.mark.gpu

# "auto" takes the small-group kernel for the narrow cases of the reference's
# matrix; "gemm" pins the tiled fp32 kernels on the same cases.
ALGOS = {"auto": MATH_FP32, "gemm": MATH_FP32 | ALGO_SIMT_GEMM}

TOL = {"x": 2e-3, "off": 1e-4, "m": 1e-4, "w": 1e-4, "b": 1e-4}


def check_grads(case, flags=MATH_FP32):
    out, grads = run_ours(case, flags=flags)
    ref, rgrads = run_oracle(case)
    scale = max(1.0, float(np.abs(ref).max()))
    assert_close(out, ref, rtol=1e-4, atol=1e-4 * scale, name="out")
    assert set(grads) == set(rgrads)
    for k, want in rgrads.items():
        s = max(1.0, float(np.abs(want).max()))
        assert_close(grads[k], want, rtol=TOL[k], atol=TOL[k] * s, name=f"grad_{k}")


KERNELS = [(3, 3), (1, 1), (1, 3)]
_CASES = [(*k, s, p, d, m) for k in KERNELS for s in (1, 2) for p in (0, 1)
          for d in (1, 2) for m in (False, True)]


@pytest.mark.parametrize("algo", sorted(ALGOS))
@pytest.mark.parametrize("kh,kw,stride,pad,dil,use_mask", _CASES)
def test_backward_matrix(cuda_device, kh, kw, stride, pad, dil, use_mask, algo):
    check_grads(make_case(kh=kh, kw=kw, stride=stride, pad=pad, dil=dil,
                          use_mask=use_mask, upstream="sum"), flags=ALGOS[algo])


@pytest.mark.parametrize("use_mask", [False, True])
def test_backward_nonscalar_upstream(cuda_device, use_mask):
    check_grads(make_case(use_mask=use_mask, upstream="randn"))


EXTRA = {
    "asym-everything": dict(H=8, W=11, kh=1, kw=3, stride=(2, 1), pad=(0, 2), dil=(2, 1)),
    "no-bias": dict(use_bias=False),
    "no-bias-v1": dict(use_bias=False, use_mask=False),
    "n1-odd-channels": dict(N=1, inC=3, outC=5),
    "boundary-stress": dict(offset_scale=8.0),
    "boundary-stress-v1": dict(offset_scale=8.0, use_mask=False),
    "large-spatial": dict(N=2, inC=8, H=33, W=35, stride=2, pad=1),
    "dg2": dict(dg=2),
    "dg2-v1": dict(dg=2, use_mask=False),
    "dg2-cpg3": dict(dg=2, inC=6),
    "dg-eq-C": dict(dg=4),
    "dg2-asym": dict(dg=2, H=8, W=11, stride=(2, 1), pad=(0, 2), dil=(2, 1)),
    "dg2-nonscalar-grad": dict(dg=2, upstream="randn"),
    "g2": dict(groups=2),
    "g2-v1": dict(groups=2, use_mask=False),
    "g2-c6": dict(groups=2, inC=6),
    "g2-asym": dict(groups=2, H=8, W=11, stride=(2, 1), pad=(0, 2), dil=(2, 1)),
    "g2-dg2": dict(groups=2, dg=2),
    "g-eq-outC-depthwise": dict(inC=6, outC=6, groups=6),
    "g2-nonscalar-grad": dict(groups=2, upstream="randn"),
    "g2-dg2-nonscalar-grad": dict(groups=2, dg=2, upstream="randn"),
    # wider channel counts: vector paths, tile edges, cross-tile reductions
    "c32-o40-dg2": dict(inC=32, outC=40, H=13, W=17, dg=2, offset_scale=2.0),
    "c64-o136-tiles": dict(N=3, inC=64, outC=136, H=15, W=19, offset_scale=3.0),
    "c128-dg1-two-ctiles": dict(N=1, inC=128, outC=24, H=12, W=12, offset_scale=2.0),
    "c48-g3-dg4": dict(inC=48, outC=48, groups=3, dg=4, H=11, W=12),
    "c24-dg3-cpg8": dict(inC=24, outC=16, dg=3, H=10, W=10),
    "c20-dg10-cpg2": dict(inC=20, outC=12, dg=10, H=10, W=10),
    "c64-g32-dg4": dict(inC=64, outC=64, groups=32, dg=4, H=12, W=12, offset_scale=2.0),
}


@pytest.mark.parametrize("algo", sorted(ALGOS))
@pytest.mark.parametrize("name", sorted(EXTRA))
def test_backward_extra(cuda_device, name, algo):
    kw = dict(upstream="sum")
    kw.update(EXTRA[name])
    check_grads(make_case(**kw), flags=ALGOS[algo])


def test_grad_call_routes_native(cuda_device):
    import pytorch_mps_deform_conv2d_b200 as dcn
    x = torch.randn(1, 4, 5, 5, device=cuda_device, requires_grad=True)
    w = torch.randn(4, 2, 3, 3, device=cuda_device)  # groups = 2
    o = torch.randn(1, 2 * 2 * 9, 3, 3, device=cuda_device)  # dg = 2
    out = dcn.deform_conv2d(x, o, w)
    # eager calls run the library's differentiable operator, whose autograd
    # node is the C++ DeformConv2dFn
    assert "DeformConv2dFn" in out.grad_fn.name(), out.grad_fn.name()


def test_no_bias_grad_is_none(cuda_device):
    import pytorch_mps_deform_conv2d_b200 as dcn
    x = torch.randn(1, 4, 5, 5, device=cuda_device, requires_grad=True)
    w = torch.randn(4, 4, 3, 3, device=cuda_device, requires_grad=True)
    o = torch.randn(1, 18, 3, 3, device=cuda_device, requires_grad=True)
    dcn.deform_conv2d(x, o, w).sum().backward()
    assert x.grad is not None and w.grad is not None and o.grad is not None


_FP32_GRADCHECK_KW = dict(eps=1e-3, atol=1e-2, rtol=1e-2, nondet_tol=1e-3)


def _gradcheck_inputs(device, use_mask, groups=1, dg=1):
    torch.manual_seed(0)
    N, inC, outC, k, H, W = 1, 2, 2, 2, 5, 5
    out = H - k + 1
    mk = lambda *s: torch.randn(*s, device=device, requires_grad=True)
    x = mk(N, inC, H, W)
    w = mk(outC, inC // groups, k, k)
    b = mk(outC)
    o = torch.randn(N, 2 * dg * k * k, out, out, device=device) * 0.5
    o = (o.floor() + (o - o.floor()).clamp(0.1, 0.9)).requires_grad_(True)
    m = None
    if use_mask:
        m = (torch.rand(N, dg * k * k, out, out, device=device) * 0.8 + 0.1).requires_grad_(True)
    return x, o, w, b, m


def _gradcheck(op, device, use_mask, groups=1, dg=1):
    x, o, w, b, m = _gradcheck_inputs(device, use_mask, groups, dg)
    if use_mask:
        fn = lambda xx, oo, ww, bb, mm: op(xx, oo, ww, bias=bb, mask=mm)
        inputs = (x, o, w, b, m)
    else:
        fn = lambda xx, oo, ww, bb: op(xx, oo, ww, bias=bb)
        inputs = (x, o, w, b)
    assert torch.autograd.gradcheck(fn, inputs, **_FP32_GRADCHECK_KW)


@pytest.mark.filterwarnings("ignore:Input #.*double precision:UserWarning")
@pytest.mark.parametrize("use_mask,groups,dg", [(False, 1, 1), (True, 1, 1), (True, 2, 1), (True, 1, 2)])
def test_gradcheck_fp32(cuda_device, use_mask, groups, dg):
    import pytorch_mps_deform_conv2d_b200 as dcn
    dcn.set_math_mode("fp32")
    try:
        _gradcheck(dcn.deform_conv2d, cuda_device, use_mask, groups, dg)
    finally:
        dcn.set_math_mode(None)
