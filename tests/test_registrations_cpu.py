"""Fake (meta) kernels and the operator-level autograd formula, without a GPU:
shape inference of the four operators on meta tensors, the public API's
forward traced on fake CUDA tensors, and the operator's autograd formula run
on meta tensors."""
import pytest
import torch
from torch._subclasses.fake_tensor import FakeTensorMode

import pytorch_mps_deform_conv2d_b200 as dcn
from pytorch_mps_deform_conv2d_b200 import _native


@pytest.fixture(scope="module")
def ops():
    return _native.load_ops()


def meta(*shape):
    return torch.empty(*shape, device="meta")


@pytest.mark.parametrize("stride,pad,dil", [((1, 1), (1, 1), (1, 1)), ((2, 1), (2, 1), (2, 1)),
                                            ((1, 2), (0, 0), (1, 1))])
def test_forward_fake_shape(ops, stride, pad, dil):
    x, w = meta(2, 8, 11, 13), meta(6, 4, 3, 3)
    ho = (11 + 2 * pad[0] - dil[0] * 2 - 1) // stride[0] + 1
    wo = (13 + 2 * pad[1] - dil[1] * 2 - 1) // stride[1] + 1
    off, m = meta(2, 18 * 2, ho, wo), meta(2, 9 * 2, ho, wo)
    out = ops.deform_conv2d_forward(x, w, off, m, meta(6), stride[0], stride[1], pad[0], pad[1],
                                    dil[0], dil[1], 2, 2)
    assert out.shape == (2, 6, ho, wo) and out.dtype == torch.float32


def test_backward_fake_shapes(ops):
    x, w, off, m = meta(2, 4, 10, 12), meta(6, 4, 3, 3), meta(2, 18, 10, 12), meta(2, 9, 10, 12)
    go = meta(2, 6, 10, 12)
    gi, goff, gm, gw, gb = ops.deform_conv2d_backward(go, x, w, off, m, meta(6), 1, 1, 1, 1, 1,
                                                      1, 1, 1)
    assert (gi.shape, goff.shape, gm.shape, gw.shape, gb.shape) == (
        x.shape, off.shape, m.shape, w.shape, (6,))
    # DCNv1 (empty mask) and no bias: empty grad_mask / grad_bias, as the CUDA op
    _, _, gm, _, gb = ops.deform_conv2d_backward(go, x, w, off, meta(0), None, 1, 1, 1, 1, 1, 1,
                                                 1, 1)
    assert gm.shape == (0,) and gb.shape == (0,)


def test_debug_ops_fake_shapes(ops):
    cols, off, m = meta(4 * 9, 10 * 12), meta(18, 10, 12), meta(9, 10, 12)
    assert ops.deformable_col2im(cols, off, m, 10, 12, 3, 3, 1, 1, 1, 1, 1, 1, 1).shape == (
        4, 10, 12)
    goff, gm = ops.deformable_col2im_coord(cols, meta(4, 10, 12), off, m, 3, 3, 1, 1, 1, 1, 1,
                                           1, 1)
    assert goff.shape == off.shape and gm.shape == m.shape
    _, gm = ops.deformable_col2im_coord(cols, meta(4, 10, 12), off, meta(0), 3, 3, 1, 1, 1, 1,
                                        1, 1, 1)
    assert gm.shape == (0,)


@pytest.mark.parametrize("use_mask,use_bias", [(True, True), (False, False)])
def test_public_api_traces_on_fake_cuda_tensors(ops, use_mask, use_bias):
    # forward only: the autograd engine needs a CUDA context for CUDA tensors,
    # even fake ones (the backward is traced on meta tensors below)
    with FakeTensorMode():
        x = torch.empty(2, 8, 9, 9, device="cuda")
        w = torch.empty(4, 4, 3, 3, device="cuda")
        b = torch.empty(4, device="cuda") if use_bias else None
        off = torch.empty(2, 36, 9, 9, device="cuda")
        m = torch.empty(2, 18, 9, 9, device="cuda") if use_mask else None
        out = dcn.deform_conv2d(x, off, w, b, padding=1, mask=m)
        assert out.shape == (2, 4, 9, 9) and out.device.type == "cuda"


@pytest.mark.parametrize("use_mask,use_bias", [(True, True), (False, False)])
def test_operator_autograd_formula_on_meta_tensors(ops, use_mask, use_bias):
    # the operator called directly is differentiable (register_autograd)
    x = meta(1, 4, 6, 6).requires_grad_()
    w = meta(4, 4, 3, 3).requires_grad_()
    off = meta(1, 18, 6, 6).requires_grad_()
    m = meta(1, 9, 6, 6).requires_grad_() if use_mask else meta(0)
    b = meta(4).requires_grad_() if use_bias else None
    out = ops.deform_conv2d_forward(x, w, off, m, b, 1, 1, 1, 1, 1, 1, 1, 1)
    out.sum().backward()
    assert x.grad.shape == x.shape and w.grad.shape == w.shape and off.grad.shape == off.shape
    assert (m.grad.shape == m.shape) if use_mask else (m.grad is None)
    if use_bias:
        assert b.grad.shape == b.shape


def test_backward_fake_keeps_channels_last_input_layout(ops):
    # the CUDA operator accumulates grad_input in the layout of a dense
    # channels-last input; any other input gets a contiguous grad_input
    x = meta(2, 4, 10, 12).to(memory_format=torch.channels_last)
    w, off, go = meta(6, 4, 3, 3), meta(2, 18, 10, 12), meta(2, 6, 10, 12)
    gi = ops.deform_conv2d_backward(go, x, w, off, meta(0), None, 1, 1, 1, 1, 1, 1, 1, 1)[0]
    assert gi.is_contiguous(memory_format=torch.channels_last) and not gi.is_contiguous()
    strided = meta(2, 4, 10, 24)[:, :, :, ::2]
    gi = ops.deform_conv2d_backward(go, strided, w, off, meta(0), None, 1, 1, 1, 1, 1, 1, 1,
                                    1)[0]
    assert gi.is_contiguous()
