"""Staged input (DCN_INPUT_STAGED): the NHWC staging copy that
deform_conv2d_stage_input makes once per step feeds both the forward and the
backward operator.  Results equal those of the unstaged calls (the forward
bitwise, the gradients within the grad_input reductions' run-to-run noise),
in every math mode and for NCHW and channels-last input, and the
differentiable operator stages its input once per training step."""
import numpy as np
import pytest
import torch

from _util import make_case, staging_launches
from pytorch_mps_deform_conv2d_b200 import _native
from pytorch_mps_deform_conv2d_b200.ops import MATH_3XTF32, MATH_FP32, MATH_TF32, deform_conv2d_ex

pytestmark = pytest.mark.gpu

MODES = {"fp32": MATH_FP32, "tf32": MATH_TF32, "3xtf32": MATH_3XTF32}


def _ops():
    _native.load_ops()
    return torch.ops.deform_conv2d_b200


@pytest.mark.parametrize("layout", ["nchw", "channels_last"])
@pytest.mark.parametrize("mode", sorted(MODES))
def test_staged_equals_unstaged(cuda_device, mode, layout):
    flags = MODES[mode]
    case = make_case(N=2, inC=64, outC=64, H=12, W=14, offset_scale=2.0, mask_kind="sigmoid")
    d = {k: (v.cuda() if isinstance(v, torch.Tensor) else v) for k, v in case.items()}
    x = d["x"]
    if layout == "channels_last":
        x = x.contiguous(memory_format=torch.channels_last)
    ops = _ops()
    args = (1, 1, 1, 1, 1, 1, 1, 1)  # stride, pad, dilation, groups, deformable groups
    staged = ops.deform_conv2d_stage_input(x)
    assert staged.numel() == 2 * 12 * 14 * 64 + 64
    out_a = ops.deform_conv2d_forward(x, d["w"], d["off"], d["m"], d["b"], *args, flags)
    out_b = ops.deform_conv2d_forward(x, d["w"], d["off"], d["m"], d["b"], *args, flags, staged)
    assert torch.equal(out_a, out_b)
    ga = ops.deform_conv2d_backward(d["go"], x, d["w"], d["off"], d["m"], d["b"], *args, flags)
    gb = ops.deform_conv2d_backward(d["go"], x, d["w"], d["off"], d["m"], d["b"], *args, flags,
                                    staged)
    torch.cuda.synchronize()
    assert gb[0].is_contiguous(memory_format=torch.channels_last) == (layout == "channels_last")
    for a, b in zip(ga, gb):
        a, b = a.cpu().numpy(), b.cpu().numpy()
        scale = max(1.0, float(np.abs(a).max()))
        np.testing.assert_allclose(b, a, rtol=1e-5, atol=1e-5 * scale)


@pytest.mark.parametrize("layout", ["nchw", "channels_last"])
@pytest.mark.parametrize("mode", sorted(MODES))
def test_forward_staging_keeps_the_staging_copy(cuda_device, mode, layout):
    """deform_conv2d_forward_staging (DCN_KEEP_STAGED): the output of the
    plain forward and the copy deform_conv2d_stage_input makes, bit for bit."""
    flags = MODES[mode]
    case = make_case(N=2, inC=64, outC=64, H=12, W=14, offset_scale=2.0, mask_kind="sigmoid")
    d = {k: (v.cuda() if isinstance(v, torch.Tensor) else v) for k, v in case.items()}
    x = d["x"]
    if layout == "channels_last":
        x = x.contiguous(memory_format=torch.channels_last)
    ops = _ops()
    args = (1, 1, 1, 1, 1, 1, 1, 1)
    out, staged = ops.deform_conv2d_forward_staging(x, d["w"], d["off"], d["m"], d["b"], *args,
                                                    flags)
    ref = ops.deform_conv2d_forward(x, d["w"], d["off"], d["m"], d["b"], *args, flags)
    assert torch.equal(out, ref)
    assert staged.dtype == torch.float32 and staged.numel() == 2 * 12 * 14 * 64 + 64
    assert torch.equal(staged, ops.deform_conv2d_stage_input(x))


def test_keep_staged_refuses_a_staged_input(cuda_device):
    import ctypes
    lib = _native.load_capi()
    case = make_case(N=1, inC=32, outC=32, H=8, W=9)
    d = {k: (v.cuda() if isinstance(v, torch.Tensor) else v) for k, v in case.items()}
    shape = _native.DcnShape(batch=1, in_channels=32, height=8, width=9, out_channels=32,
                             kernel_h=3, kernel_w=3, stride_h=1, stride_w=1, pad_h=1, pad_w=1,
                             dilation_h=1, dilation_w=1, groups=1, deformable_groups=1)
    out = torch.empty(1, 32, 8, 9, device="cuda")
    ws = torch.empty(1 << 24, dtype=torch.uint8, device="cuda")
    vp = ctypes.c_void_p
    rc = lib.dcn_forward(ctypes.byref(shape), vp(d["x"].data_ptr()), vp(d["w"].data_ptr()),
                         vp(d["off"].data_ptr()), vp(d["m"].data_ptr()), vp(d["b"].data_ptr()),
                         vp(out.data_ptr()), 0x40000 | 0x80000, vp(ws.data_ptr()), ws.numel(),
                         vp(torch.cuda.current_stream().cuda_stream))
    assert rc == 1 and b"KEEP_STAGED" in lib.dcn_last_error()


def test_staged_size_is_checked(cuda_device):
    case = make_case(N=1, inC=32, outC=32, H=8, W=9)
    d = {k: (v.cuda() if isinstance(v, torch.Tensor) else v) for k, v in case.items()}
    bad = torch.zeros(17, device="cuda")
    with pytest.raises(RuntimeError, match="staging copy"):
        _ops().deform_conv2d_forward(d["x"], d["w"], d["off"], d["m"], d["b"],
                                     1, 1, 1, 1, 1, 1, 1, 1, MATH_TF32, bad)


@pytest.mark.parametrize("mode", ["fp32", "tf32"])
def test_training_step_stages_its_input_once(cuda_device, mode):
    case = make_case(N=2, inC=64, outC=64, H=12, W=14, offset_scale=2.0)
    leaves = {k: case[k].cuda().requires_grad_(True) for k in ("x", "w", "b", "off", "m")}
    _native.profiler_read()
    _native.profiler_enable(True)
    try:
        out = deform_conv2d_ex(leaves["x"], leaves["off"], leaves["w"], leaves["b"],
                               case["stride"], case["padding"], case["dilation"], leaves["m"],
                               flags=MODES[mode])
        out.backward(case["go"].cuda())
        torch.cuda.synchronize()
    finally:
        _native.profiler_enable(False)
    stats = _native.profiler_read()
    assert staging_launches(stats) == 1, stats  # staged once, for both passes


H16 = {"bf16": torch.bfloat16, "fp16": torch.float16}


@pytest.mark.parametrize("layout", ["nchw", "channels_last"])
@pytest.mark.parametrize("dt", sorted(H16))
def test_forward_staging_h16_keeps_the_staging_copy(cuda_device, dt, layout):
    """16-bit tensors on the tensor-core route: the forward keeps its 16-bit
    staging copy (DCN_KEEP_STAGED), the same bits deform_conv2d_stage_input
    makes, and its output equals the plain forward's."""
    case = make_case(N=2, inC=64, outC=64, H=12, W=14, offset_scale=2.0, mask_kind="sigmoid")
    d = {k: (v.cuda().to(H16[dt]) if isinstance(v, torch.Tensor) else v)
         for k, v in case.items()}
    x = d["x"]
    if layout == "channels_last":
        x = x.contiguous(memory_format=torch.channels_last)
    ops = _ops()
    args = (1, 1, 1, 1, 1, 1, 1, 1)
    out, staged = ops.deform_conv2d_forward_staging(x, d["w"], d["off"], d["m"], d["b"], *args,
                                                    MATH_TF32)
    ref = ops.deform_conv2d_forward(x, d["w"], d["off"], d["m"], d["b"], *args, MATH_TF32)
    assert torch.equal(out, ref)
    assert staged.dtype == H16[dt] and staged.numel() == 2 * 12 * 14 * 64 + 64
    assert torch.equal(staged, ops.deform_conv2d_stage_input(x))
    # the backward on the staging copy gives the unstaged gradients (up to
    # the order of the fp32 reductions, then one 16-bit rounding)
    ga = ops.deform_conv2d_backward(d["go"], x, d["w"], d["off"], d["m"], d["b"], *args,
                                    MATH_TF32)
    gb = ops.deform_conv2d_backward(d["go"], x, d["w"], d["off"], d["m"], d["b"], *args,
                                    MATH_TF32, staged)
    torch.cuda.synchronize()
    for a, b in zip(ga, gb):
        a, b = a.float().cpu().numpy(), b.float().cpu().numpy()
        scale = max(1.0, float(np.abs(a).max()))
        np.testing.assert_allclose(b, a, rtol=2e-2, atol=1e-2 * scale)


@pytest.mark.parametrize("dt", sorted(H16))
def test_h16_training_step_stages_its_input_once(cuda_device, dt):
    case = make_case(N=2, inC=64, outC=64, H=12, W=14, offset_scale=2.0)
    leaves = {k: case[k].cuda().to(H16[dt]).requires_grad_(True)
              for k in ("x", "w", "b", "off", "m")}
    _native.profiler_read()
    _native.profiler_enable(True)
    try:
        out = deform_conv2d_ex(leaves["x"], leaves["off"], leaves["w"], leaves["b"],
                               case["stride"], case["padding"], case["dilation"], leaves["m"],
                               flags=MATH_TF32)
        out.backward(case["go"].cuda().to(H16[dt]))
        torch.cuda.synchronize()
    finally:
        _native.profiler_enable(False)
    stats = _native.profiler_read()
    tag = "bf16" if dt == "bf16" else "f16"
    assert f"fwd_tc_{tag}" in stats and f"bwd_fused_tc_{tag}" in stats, sorted(stats)
    assert staging_launches(stats) == 1, stats  # staged once, for both passes
    assert all(leaves[k].grad is not None and leaves[k].grad.dtype == H16[dt] for k in leaves)


def test_h16_uncovered_shape_is_not_staged(cuda_device):
    # 48 channels: not a multiple of 64, so the 16-bit calls take the upcast
    # route, which takes no staging copy; the training step still runs
    case = make_case(N=1, inC=48, outC=32, H=8, W=9, offset_scale=2.0)
    leaves = {k: case[k].cuda().to(torch.bfloat16).requires_grad_(True)
              for k in ("x", "w", "b", "off", "m")}
    out = deform_conv2d_ex(leaves["x"], leaves["off"], leaves["w"], leaves["b"],
                           case["stride"], case["padding"], case["dilation"], leaves["m"],
                           flags=MATH_TF32)
    out.backward(case["go"].cuda().to(torch.bfloat16))
    torch.cuda.synchronize()
    assert all(leaves[k].grad is not None for k in leaves)
    ops = _ops()
    args = (1, 1, 1, 1, 1, 1, 1, 1)
    d = {k: leaves[k].detach() for k in leaves}
    staged = ops.deform_conv2d_stage_input(d["x"])
    with pytest.raises(RuntimeError, match="staging copy"):
        ops.deform_conv2d_forward(d["x"], d["w"], d["off"], d["m"], d["b"], *args, MATH_TF32,
                                  staged)


@pytest.mark.parametrize("H,W,kept", [(119, 256, True), (60, 128, False)])
def test_staging_copy_does_not_pin_a_large_workspace(cuda_device, H, W, kept):
    """The forward keeps its staging copy in its workspace only when the rest
    of that workspace is small: 238 tiles of 128 pixels (no split round) keep
    it there; 60 tiles (a split round whose partial sums would be pinned with
    it) stage into a buffer of their own.  Either way the copy is the one
    deform_conv2d_stage_input makes."""
    case = make_case(N=1, inC=32, outC=32, H=H, W=W, offset_scale=2.0, mask_kind="sigmoid")
    d = {k: (v.cuda() if isinstance(v, torch.Tensor) else v) for k, v in case.items()}
    ops = _ops()
    args = (1, 1, 1, 1, 1, 1, 1, 1)
    out, staged = ops.deform_conv2d_forward_staging(d["x"], d["w"], d["off"], d["m"], d["b"],
                                                    *args, MATH_TF32)
    nbytes = staged.numel() * 4
    pinned = staged.untyped_storage().nbytes()
    assert (pinned > nbytes) == kept, (pinned, nbytes)
    assert pinned <= nbytes + nbytes // 8 + (1 << 20) + 512
    assert torch.equal(staged, ops.deform_conv2d_stage_input(d["x"]))
    ref = ops.deform_conv2d_forward(d["x"], d["w"], d["off"], d["m"], d["b"], *args, MATH_TF32)
    assert torch.equal(out, ref)
