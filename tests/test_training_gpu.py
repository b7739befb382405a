"""Training through the operator: a small teacher-student regression (an
offset conv and, for DCNv2, a mask conv feeding DeformConv2d, then a 1x1
head; the target comes from a frozen net of the same architecture, so the
loss can fall far) trained with Adam on the GPU through this library.
Per-call parity tests cannot see an error that only shows over optimizer
steps (a gradient accumulated into the wrong buffer, a stale workspace,
state carried between calls); this does, in two ways:

* the loss falls below a tenth of its start in 150 steps;
* the first steps follow a CPU twin of the same net (same weights, same
  data, torchvision's `deform_conv2d`, the reference's CPU route) within a
  bound set by how much the trajectory itself moves under gradient noise
  of the kernels' size: 1e-3 of the loss for the fp32 kernels, 5e-2 for
  TF32, where every gradient carries ~3e-4 of rounding and Adam's first,
  sign-like updates of the 64-channel net amplify it.

The reference's own training test (`tests/test_training.py:64-86`) runs the
same teacher-student scheme against its CPU route.
"""
import copy

import pytest
import torch
from torch import nn

import pytorch_mps_deform_conv2d_b200 as dcn
from pytorch_mps_deform_conv2d_b200 import _native

pytestmark = pytest.mark.gpu

torchvision = pytest.importorskip("torchvision")


class _Net(nn.Module):
    def __init__(self, ch, use_mask, dcn_cls):
        super().__init__()
        self.offset_conv = nn.Conv2d(ch, 18, 3, padding=1)
        self.mask_conv = nn.Conv2d(ch, 9, 3, padding=1) if use_mask else None
        self.dcn = dcn_cls(ch, ch, 3, padding=1)
        self.head = nn.Conv2d(ch, 1, 1)

    def forward(self, x):
        mask = torch.sigmoid(self.mask_conv(x)) if self.mask_conv is not None else None
        return self.head(torch.relu(self.dcn(x, self.offset_conv(x), mask)))


def _train(net, x, y, steps, lr=1e-2):
    opt = torch.optim.Adam(net.parameters(), lr=lr)
    losses = []
    for _ in range(steps):
        opt.zero_grad(set_to_none=True)
        loss = nn.functional.mse_loss(net(x), y)
        loss.backward()
        opt.step()
        losses.append(loss.item())
    return losses


@pytest.mark.parametrize("ch,use_mask,mode,rel", [(6, True, "fp32", 1e-3),
                                                  (6, False, "fp32", 1e-3),
                                                  (64, True, "tf32", 5e-2)])
def test_training_converges_and_tracks_cpu(cuda_device, ch, use_mask, mode, rel):
    torch.manual_seed(0)
    x = torch.randn(8, ch, 16, 16)
    teacher = _Net(ch, use_mask, torchvision.ops.DeformConv2d)
    with torch.no_grad():
        y = teacher(x)
    torch.manual_seed(1)
    cpu_net = _Net(ch, use_mask, torchvision.ops.DeformConv2d)
    gpu_net = _Net(ch, use_mask, dcn.DeformConv2d)
    gpu_net.load_state_dict(copy.deepcopy(cpu_net.state_dict()))  # same keys, same layout
    gpu_net = gpu_net.cuda()

    cudnn_tf32 = torch.backends.cudnn.allow_tf32
    torch.backends.cudnn.allow_tf32 = mode == "tf32"  # the helper convs at the same precision
    dcn.set_math_mode(mode)
    try:
        _native.profiler_read()
        _native.profiler_enable(True)
        try:
            losses = _train(gpu_net, x.cuda(), y.cuda(), steps=150)
        finally:
            _native.profiler_enable(False)
        kernels = _native.profiler_read()
    finally:
        dcn.set_math_mode(None)
        torch.backends.cudnn.allow_tf32 = cudnn_tf32
    if mode == "tf32":  # the tensor-core forward and the fused backward did the work
        assert "fwd_tc" in kernels and "bwd_fused_tc" in kernels, sorted(kernels)
        assert kernels["bwd_fused_tc"][0] == 150, kernels["bwd_fused_tc"]
    assert losses[-1] < 0.1 * losses[0], f"no convergence: {losses[0]:.5f} -> {losses[-1]:.5f}"

    cpu_losses = _train(cpu_net, x, y, steps=5)
    for i, (lc, lg) in enumerate(zip(cpu_losses, losses)):
        assert abs(lg - lc) <= rel * abs(lc) + 1e-7, (
            f"step {i}: CPU loss {lc:.6f}, GPU loss {lg:.6f} ({mode})")
