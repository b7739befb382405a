"""Host-side behaviour of the Python layer and the operator registration."""
import pytest
import torch

import pytorch_mps_deform_conv2d_b200 as dcn
from pytorch_mps_deform_conv2d_b200 import _native

torchvision = pytest.importorskip("torchvision")
from torchvision.ops import DeformConv2d as TVDeformConv2d  # noqa: E402


def test_operator_schemas_mirror_the_reference():
    ops = _native.load_ops()
    fwd = str(ops.deform_conv2d_forward.default._schema)
    assert ("deform_conv2d_forward(Tensor input, Tensor weight, Tensor offset, Tensor mask, "
            "Tensor? bias, int stride_h, int stride_w, int pad_h, int pad_w, int dilation_h, "
            "int dilation_w, int groups, int deformable_groups") in fwd
    bwd = str(ops.deform_conv2d_backward.default._schema)
    assert bwd.endswith("-> (Tensor, Tensor, Tensor, Tensor, Tensor)")
    assert "deformable_col2im_coord(Tensor columns, Tensor input" in str(
        ops.deformable_col2im_coord.default._schema)
    assert "deformable_col2im(Tensor columns, Tensor offset, Tensor mask, int height" in str(
        ops.deformable_col2im.default._schema)


def test_cpu_tensors_are_refused_no_fallback():
    x = torch.randn(1, 2, 5, 5)
    w = torch.randn(2, 2, 3, 3)
    o = torch.randn(1, 18, 3, 3)
    with pytest.raises(NotImplementedError, match="CUDA"):
        dcn.deform_conv2d(x, o, w)


def test_math_mode_switch():
    dcn.set_math_mode("fp32")
    assert dcn.get_math_mode() == "fp32"
    dcn.set_math_mode("tf32")
    assert dcn.get_math_mode() == "tf32"
    dcn.set_math_mode("3xtf32")
    assert dcn.get_math_mode() == "3xtf32"
    dcn.set_math_mode(None)
    with pytest.raises(ValueError):
        dcn.set_math_mode("bf16")


def test_state_dict_layout_matches_torchvision():
    ours = dcn.DeformConv2d(4, 6, kernel_size=3, padding=1)
    tv = TVDeformConv2d(4, 6, kernel_size=3, padding=1)
    assert list(ours.state_dict()) == ["weight", "bias"]
    assert {k: v.shape for k, v in ours.state_dict().items()} == \
        {k: v.shape for k, v in tv.state_dict().items()}
    tv.load_state_dict(ours.state_dict())
    ours.load_state_dict(tv.state_dict())
    nb = dcn.DeformConv2d(4, 6, kernel_size=(3, 1), groups=2, bias=False)
    assert list(nb.state_dict()) == ["weight"] and nb.weight.shape == (6, 2, 3, 1)


def test_module_init_statistics():
    torch.manual_seed(0)
    m = dcn.DeformConv2d(64, 64, 3, padding=1)
    bound = 1.0 / (64 * 9) ** 0.5
    assert m.bias.abs().max() <= bound
    # kaiming_uniform_(a=sqrt(5)) on fan_in 576 -> bound 1/sqrt(576)
    assert m.weight.abs().max() <= bound + 1e-7
    assert "kernel_size=(3, 3)" in repr(m)
