"""DeformConv2dPack without a GPU: parameters, state_dict keys, the zero
initialisation of the offset/mask convolution, and the CUDA-only error."""
import pytest
import torch

import pytorch_mps_deform_conv2d_b200 as dcn


@pytest.mark.parametrize("modulated,per_tap", [(True, 3), (False, 2)])
def test_pack_module_layout(modulated, per_tap):
    m = dcn.DeformConv2dPack(8, 6, (3, 2), padding=1, deformable_groups=2, modulated=modulated)
    assert list(m.state_dict()) == ["weight", "bias", "conv_offset.weight", "conv_offset.bias"]
    assert m.conv_offset.out_channels == per_tap * 2 * 3 * 2
    assert m.conv_offset.kernel_size == (3, 2) and m.conv_offset.padding == (1, 1)
    assert torch.count_nonzero(m.conv_offset.weight) == 0
    assert torch.count_nonzero(m.conv_offset.bias) == 0


def test_pack_module_rejects_cpu_tensors():
    m = dcn.DeformConv2dPack(4, 4, 3, padding=1)
    with pytest.raises(NotImplementedError, match="CUDA"):
        m(torch.randn(1, 4, 5, 5))
