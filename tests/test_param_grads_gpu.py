"""The operator's autograd node returns grad_weight and grad_bias as
neighbouring views of one buffer, so that a data-parallel step sums both
with one all-reduce (`distributed.allreduce_grads` / `GradAllReduce` find
them adjacent): after a backward through the module the parameters' .grad
tensors are adjacent, carry the values of the backward operator (whose own
outputs stay separate tensors), and stay adjacent when a second backward
accumulates into them; float32 (TF32 route, whole image and row window) and
bfloat16."""
import pytest
import torch

import pytorch_mps_deform_conv2d_b200 as dcn
from pytorch_mps_deform_conv2d_b200 import _native
from pytorch_mps_deform_conv2d_b200.distributed import _adjacent_view
from pytorch_mps_deform_conv2d_b200.ops import MATH_TF32, deform_conv2d_rows

pytestmark = pytest.mark.gpu


def _inputs(dtype, C=64, H=12, W=14):
    g = torch.Generator().manual_seed(5)
    x = torch.randn(2, C, H, W, generator=g)
    off = 2 * torch.randn(2, 18, H, W, generator=g)
    m = torch.sigmoid(torch.randn(2, 9, H, W, generator=g))
    go = torch.randn(2, C, H, W, generator=g)
    return [t.to("cuda", dtype) for t in (x, off, m, go)]


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_module_grads_are_adjacent_and_match_the_operator(cuda_device, dtype):
    x, off, m, go = _inputs(dtype)
    torch.manual_seed(0)
    layer = dcn.DeformConv2d(64, 64, 3, padding=1).to("cuda", dtype)
    dcn.set_math_mode("tf32")
    try:
        layer(x, off, m).backward(go)
        gw, gb = layer.weight.grad, layer.bias.grad
        assert _adjacent_view([layer.weight.grad, layer.bias.grad]) is not None
        assert gb.data_ptr() == gw.data_ptr() + gw.numel() * gw.element_size()
        ops = _native.load_ops()
        ref = ops.deform_conv2d_backward(go, x, layer.weight.detach(), off, m,
                                         layer.bias.detach(), 1, 1, 1, 1, 1, 1, 1, 1, MATH_TF32)
        assert ref[3].untyped_storage().data_ptr() != ref[4].untyped_storage().data_ptr()
        tol = 1e-5 if dtype == torch.float32 else 1e-2
        for got, want in ((gw, ref[3]), (gb, ref[4])):
            torch.testing.assert_close(got.float(), want.float(), rtol=tol,
                                       atol=tol * max(1.0, float(want.abs().max())))
        first = [gw.clone(), gb.clone()]
        layer(x, off, m).backward(go)  # accumulates in place: same buffer, doubled values
        assert layer.weight.grad.data_ptr() == gw.data_ptr()
        assert _adjacent_view([layer.weight.grad, layer.bias.grad]) is not None
        for got, once in zip((layer.weight.grad, layer.bias.grad), first):
            torch.testing.assert_close(got.float(), 2 * once.float(), rtol=2 * tol,
                                       atol=2 * tol * max(1.0, float(once.abs().max())))
    finally:
        dcn.set_math_mode(None)


def test_row_window_grads_are_adjacent(cuda_device):
    x, off, m, go = _inputs(torch.float32)
    rows = slice(4, 10)
    w = (torch.randn(64, 64, 3, 3, device="cuda") / 24).requires_grad_()
    b = torch.randn(64, device="cuda", requires_grad=True)
    out = deform_conv2d_rows(x, off[:, :, rows].contiguous(), w, b, (1, 1), (1, 1), (1, 1),
                             m[:, :, rows].contiguous(), row_begin=rows.start, flags=MATH_TF32)
    out.backward(go[:, :, rows].contiguous())
    assert _adjacent_view([w.grad, b.grad]) is not None
    assert torch.isfinite(w.grad).all() and torch.isfinite(b.grad).all()
    torch.testing.assert_close(b.grad, go[:, :, rows].sum(dim=(0, 2, 3)), rtol=1e-5, atol=1e-4)
