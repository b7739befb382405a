"""B200 (sm_100a) deformable convolution, DCNv1 / DCNv2.

Drop-in for the public API of ilirium/pytorch_mps_deform_conv2d
(``deform_conv2d``, ``DeformConv2d``), itself the API of torchvision.ops:

    from pytorch_mps_deform_conv2d_b200 import deform_conv2d, DeformConv2d

or, for code that calls torchvision directly, ``patch_torchvision()`` routes
``torchvision.ops.deform_conv2d`` / ``DeformConv2d`` on CUDA tensors here.
"""
from .ops import check_device_status, deform_conv2d, device_status, get_math_mode, set_math_mode
from .module import DeformConv2d, DeformConv2dPack
from .torchvision_patch import patch_torchvision, unpatch_torchvision

__all__ = ["deform_conv2d", "DeformConv2d", "DeformConv2dPack", "set_math_mode", "get_math_mode",
           "patch_torchvision", "unpatch_torchvision", "device_status", "check_device_status"]
__version__ = "0.1.0"
