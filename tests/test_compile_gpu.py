"""torch.library consistency checks and torch.compile on the GPU: opcheck of
the operators (schema, fake kernel, autograd registration against the CUDA
kernels) and a compiled DeformConv2d training step against eager."""
import pytest
import torch

import pytorch_mps_deform_conv2d_b200 as dcn
from pytorch_mps_deform_conv2d_b200 import _native
from pytorch_mps_deform_conv2d_b200.ops import MATH_FP32

pytestmark = pytest.mark.gpu


def _inputs(use_mask=True, use_bias=True, requires_grad=True):
    g = torch.Generator().manual_seed(0)
    mk = lambda *s: torch.randn(*s, generator=g).cuda().requires_grad_(requires_grad)
    x, w = mk(2, 8, 9, 10), mk(6, 8, 3, 3)
    off = (torch.randn(2, 18, 9, 10, generator=g) * 2).cuda().requires_grad_(requires_grad)
    m = (torch.rand(2, 9, 9, 10, generator=g).cuda().requires_grad_(requires_grad)
         if use_mask else torch.empty(0, device="cuda"))
    b = mk(6) if use_bias else None
    return x, w, off, m, b


@pytest.mark.parametrize("use_mask,use_bias", [(True, True), (False, False)])
def test_opcheck_forward(cuda_device, use_mask, use_bias):
    ops = _native.load_ops()
    x, w, off, m, b = _inputs(use_mask, use_bias)
    torch.library.opcheck(ops.deform_conv2d_forward,
                          (x, w, off, m, b, 1, 1, 1, 1, 1, 1, 1, 1, MATH_FP32))


def test_opcheck_forward_staging(cuda_device):
    ops = _native.load_ops()
    x, w, off, m, b = _inputs(requires_grad=False)
    torch.library.opcheck(ops.deform_conv2d_forward_staging,
                          (x, w, off, m, b, 1, 1, 1, 1, 1, 1, 1, 1, MATH_FP32))


def test_opcheck_backward(cuda_device):
    ops = _native.load_ops()
    x, w, off, m, b = _inputs(requires_grad=False)
    go = torch.randn(2, 6, 9, 10, device="cuda")
    torch.library.opcheck(ops.deform_conv2d_backward,
                          (go, x, w, off, m, b, 1, 1, 1, 1, 1, 1, 1, 1, MATH_FP32))


def test_operator_is_differentiable(cuda_device):
    ops = _native.load_ops()
    x, w, off, m, b = _inputs()
    out = ops.deform_conv2d_forward(x, w, off, m, b, 1, 1, 1, 1, 1, 1, 1, 1, MATH_FP32)
    go = torch.randn_like(out)
    out.backward(go)
    got = [t.grad.clone() for t in (x, w, off, m, b)]
    for t in (x, w, off, m, b):
        t.grad = None
    ref = dcn.ops.deform_conv2d_ex(x, off, w, b, 1, 1, 1, m, flags=MATH_FP32)
    ref.backward(go)
    for a, t in zip(got, (x, w, off, m, b)):
        torch.testing.assert_close(a, t.grad, rtol=1e-5, atol=1e-5)


def test_compiled_module_matches_eager(cuda_device):
    torch.manual_seed(0)
    mod = dcn.DeformConv2d(8, 6, 3, padding=1).cuda()
    x = torch.randn(2, 8, 9, 10, device="cuda", requires_grad=True)
    off = (2 * torch.randn(2, 18, 9, 10, device="cuda")).requires_grad_()
    m = torch.rand(2, 9, 9, 10, device="cuda", requires_grad=True)
    dcn.set_math_mode("fp32")
    try:
        def step(fn):
            for t in (x, off, m, mod.weight, mod.bias):
                t.grad = None
            out = fn(x, off, m)
            out.square().sum().backward()
            return [out.detach()] + [t.grad.clone() for t in (x, off, m, mod.weight, mod.bias)]

        eager = step(mod)
        compiled = step(torch.compile(mod, fullgraph=True, backend="aot_eager"))
    finally:
        dcn.set_math_mode(None)
    for a, b in zip(eager, compiled):
        torch.testing.assert_close(a, b, rtol=1e-5, atol=1e-5)
