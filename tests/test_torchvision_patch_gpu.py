"""patch_torchvision() on the GPU: torchvision.ops.deform_conv2d and
torchvision.ops.DeformConv2d on CUDA tensors run this package's kernels (the
library profiler sees them) and agree with torchvision's CPU kernel, forward
and gradients, at the fp32 tolerances."""
import pytest
import torch
import torchvision

import pytorch_mps_deform_conv2d_b200 as dcn
from pytorch_mps_deform_conv2d_b200 import _native

pytestmark = pytest.mark.gpu


def test_patched_torchvision_runs_our_kernels(cuda_device):
    g = torch.Generator().manual_seed(0)
    x = torch.randn(2, 8, 9, 11, generator=g)
    off = 2 * torch.randn(2, 18, 9, 11, generator=g)
    m = torch.rand(2, 9, 9, 11, generator=g)
    cpu_mod = torchvision.ops.DeformConv2d(8, 6, 3, padding=1)
    leaves_cpu = [t.clone().requires_grad_() for t in (x, off, m)]
    want = cpu_mod(*leaves_cpu)
    go = torch.randn(want.shape, generator=g)
    want.backward(go)

    dcn.patch_torchvision()
    dcn.set_math_mode("fp32")
    try:
        gpu_mod = torchvision.ops.DeformConv2d(8, 6, 3, padding=1).cuda()
        gpu_mod.load_state_dict(cpu_mod.state_dict())
        leaves = [t.cuda().requires_grad_() for t in (x, off, m)]
        _native.profiler_read()
        _native.profiler_enable(True)
        try:
            out = gpu_mod(*leaves)
            out.backward(go.cuda())
            torch.cuda.synchronize()
        finally:
            _native.profiler_enable(False)
        stats = _native.profiler_read()
    finally:
        dcn.set_math_mode(None)
        dcn.unpatch_torchvision()
    assert any(k.startswith("fwd_") for k in stats) and any(k.startswith("bwd_") for k in stats)
    torch.testing.assert_close(out.cpu(), want.detach(), rtol=1e-4, atol=1e-4)
    for a, b in zip(leaves, leaves_cpu):
        torch.testing.assert_close(a.grad.cpu(), b.grad, rtol=2e-3, atol=2e-3)
    torch.testing.assert_close(gpu_mod.weight.grad.cpu(), cpu_mod.weight.grad, rtol=1e-4,
                               atol=1e-4)
