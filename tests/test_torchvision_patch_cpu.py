"""patch_torchvision(): CPU tensors keep torchvision's own kernel (bit-identical
results), calls on CUDA tensors reach this package (checked on fake CUDA
tensors), and unpatching restores torchvision."""
import pytest
import torch
import torchvision
from torch._subclasses.fake_tensor import FakeTensorMode

import pytorch_mps_deform_conv2d_b200 as dcn
from pytorch_mps_deform_conv2d_b200 import torchvision_patch


@pytest.fixture
def patched():
    dcn.patch_torchvision()
    try:
        yield
    finally:
        dcn.unpatch_torchvision()


def _case():
    g = torch.Generator().manual_seed(0)
    x = torch.randn(1, 4, 7, 8, generator=g)
    w = torch.randn(6, 4, 3, 3, generator=g)
    off = torch.randn(1, 18, 7, 8, generator=g)
    m = torch.rand(1, 9, 7, 8, generator=g)
    b = torch.randn(6, generator=g)
    return x, off, w, b, m


def test_cpu_calls_keep_torchvision(patched):
    original = torchvision.ops.deform_conv2d.__wrapped_torchvision__
    x, off, w, b, m = _case()
    got = torchvision.ops.deform_conv2d(x, off, w, b, padding=(1, 1), mask=m)
    want = original(x, off, w, b, padding=(1, 1), mask=m)
    assert torch.equal(got, want)
    mod = torchvision.ops.DeformConv2d(4, 6, 3, padding=1)
    assert mod(x, off, m).shape == (1, 6, 7, 8)


def test_cuda_calls_reach_this_package(patched, monkeypatch):
    seen = []

    def spy(*args, **kwargs):
        seen.append(args[0].device.type)
        return dcn.ops.deform_conv2d(*args, **kwargs)

    monkeypatch.setattr(torchvision_patch, "_ours", spy)
    with FakeTensorMode():
        x = torch.empty(1, 4, 7, 8, device="cuda")
        off = torch.empty(1, 18, 7, 8, device="cuda")
        w = torch.empty(6, 4, 3, 3, device="cuda")
        out = torchvision.ops.deform_conv2d(x, off, w, padding=(1, 1))
        with torch.device("cuda"):
            mod = torchvision.ops.DeformConv2d(4, 6, 3, padding=1)
        mod_out = mod(x, off)
    assert out.shape == (1, 6, 7, 8) and mod_out.shape == (1, 6, 7, 8)
    assert seen == ["cuda", "cuda"]


def test_unpatch_restores_and_is_idempotent():
    original = torchvision.ops.deform_conv2d
    dcn.patch_torchvision()
    dcn.patch_torchvision()
    assert torchvision.ops.deform_conv2d is not original
    assert torchvision.ops.deform_conv.deform_conv2d is torchvision.ops.deform_conv2d
    dcn.unpatch_torchvision()
    dcn.unpatch_torchvision()
    assert torchvision.ops.deform_conv2d is original
    assert torchvision.ops.deform_conv.deform_conv2d is original
