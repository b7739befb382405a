"""CPU calibration twins of the fp32 gradcheck (tests/test_backward.py:301-344)
and the fp64 gradcheck of the math the kernels implement
(tests/test_backward.py:347-362): if the knobs are too tight for fp32, these
fail first, on the CPU reference path."""
import pytest
import torch

torchvision = pytest.importorskip("torchvision")
from torchvision.ops import deform_conv2d as tv_deform_conv2d  # noqa: E402

from test_backward_gpu import _gradcheck  # noqa: E402


@pytest.mark.filterwarnings("ignore:Input #.*double precision:UserWarning")
@pytest.mark.parametrize("use_mask,groups,dg", [(False, 1, 1), (True, 1, 1), (True, 2, 1), (True, 1, 2)])
def test_gradcheck_cpu_fp32_calibration(use_mask, groups, dg):
    _gradcheck(tv_deform_conv2d, "cpu", use_mask, groups, dg)


def test_gradcheck_cpu_fp64_reference():
    torch.manual_seed(0)
    N, inC, outC, H, W, k = 2, 4, 6, 7, 7, 3
    out = H - k + 1
    mk = lambda *s: torch.randn(*s, dtype=torch.float64, requires_grad=True)
    x, w, b = mk(N, inC, H, W), mk(outC, inC, k, k), mk(outC)
    offset = mk(N, 2 * k * k, out, out)
    mask = torch.rand(N, k * k, out, out, dtype=torch.float64).requires_grad_(True)
    assert torch.autograd.gradcheck(
        lambda xx, oo, ww, bb: tv_deform_conv2d(xx, oo, ww, bias=bb, mask=mask),
        (x, offset, w, b), eps=1e-6, atol=1e-4)
