"""Row windows (deform_conv2d_rows / dcn_forward_rows / dcn_backward_rows):
over an uneven partition of the output rows, the slabs' outputs and their
offset / mask gradients concatenate to the full op's, and their input,
weight and bias gradients sum to the full op's -- for every kernel family."""
import pytest
import torch

from _util import make_case, staging_launches
from pytorch_mps_deform_conv2d_b200 import _native
from pytorch_mps_deform_conv2d_b200.ops import (ALGO_SIMT_DIRECT, ALGO_SIMT_GEMM, MATH_3XTF32,
                                                MATH_FP32, MATH_TF32, deform_conv2d_ex,
                                                deform_conv2d_rows)

pytestmark = pytest.mark.gpu

CASES = {  # name -> (case, flags, kernel that must run)
    "tc-tf32": (dict(inC=128, outC=64, H=11, W=9, offset_scale=3.0), MATH_TF32, "fwd_tc"),
    "tc-3xtf32-cg64-stride2": (dict(inC=64, outC=64, H=13, W=10, stride=(2, 1), pad=(1, 1),
                                    offset_scale=2.0), MATH_3XTF32, "bwd_data_tc"),
    "simt-fp32-dg2": (dict(inC=8, outC=12, H=10, W=9, dg=2, offset_scale=2.0), MATH_FP32,
                      "bwd_data_simt"),
    "simt-gemm-v1": (dict(inC=6, outC=6, H=9, W=8, use_mask=False, use_bias=False),
                     MATH_FP32 | ALGO_SIMT_GEMM, "fwd_simt_gemm"),
    "dgroup": (dict(inC=32, outC=32, groups=16, dg=2, H=10, W=9, offset_scale=2.0), MATH_FP32,
               "bwd_dgroup"),
    "small-direct-asym": (dict(inC=6, outC=6, groups=3, H=9, W=11, kh=3, kw=2, dil=(2, 1),
                               pad=(2, 1)), MATH_FP32 | ALGO_SIMT_DIRECT, "bwd_small"),
}


def _leaf(t):
    return None if t is None else t.detach().clone().cuda().requires_grad_()


@pytest.mark.parametrize("name", sorted(CASES))
def test_row_slabs_reassemble_the_full_op(cuda_device, name):
    spec, flags, kernel = CASES[name]
    case = make_case(upstream="randn", **spec)
    args = (case["stride"], case["padding"], case["dilation"])
    x, w, b, off, m = (_leaf(case[k]) for k in ("x", "w", "b", "off", "m"))
    go = case["go"].cuda()
    full = deform_conv2d_ex(x, off, w, b, *args, m, flags=flags)
    full.backward(go)
    ho = full.shape[2]
    cuts = sorted({0, 1, max(1, ho // 2), ho})  # uneven: a one-row slab first
    outs, goffs, gms = [], [], []
    gx = torch.zeros_like(x)
    gw = torch.zeros_like(w)
    gb = torch.zeros_like(b) if b is not None else None
    _native.profiler_read()
    _native.profiler_enable(True)
    try:
        for r0, r1 in zip(cuts, cuts[1:]):
            xs, ws, bs = _leaf(case["x"]), _leaf(case["w"]), _leaf(case["b"])
            offs = off.detach()[:, :, r0:r1].contiguous().requires_grad_()
            ms = m.detach()[:, :, r0:r1].contiguous().requires_grad_() if m is not None else None
            out = deform_conv2d_rows(xs, offs, ws, bs, *args, ms, row_begin=r0, flags=flags)
            out.backward(go[:, :, r0:r1].contiguous())
            outs.append(out.detach())
            goffs.append(offs.grad)
            if ms is not None:
                gms.append(ms.grad)
            gx += xs.grad
            gw += ws.grad
            if gb is not None:
                gb += bs.grad
    finally:
        _native.profiler_enable(False)
    assert kernel in _native.profiler_read()
    close = lambda a, b_: torch.testing.assert_close(a, b_, rtol=1e-4,
                                                     atol=1e-4 * max(1.0, float(b_.abs().max())))
    close(torch.cat(outs, 2), full.detach())
    close(torch.cat(goffs, 2), off.grad)
    if m is not None:
        close(torch.cat(gms, 2), m.grad)
    close(gx, x.grad)
    close(gw, w.grad)
    if gb is not None:
        close(gb, b.grad)


def test_row_window_out_of_range_raises(cuda_device):
    case = make_case(inC=4, outC=4, H=6, W=6)
    x, w = case["x"].cuda(), case["w"].cuda()
    off = case["off"].cuda()[:, :, 2:].contiguous()  # rows 2..5 of 6
    with pytest.raises(RuntimeError, match="outside the 6 output rows"):
        deform_conv2d_rows(x, off, w, None, 1, 1, 1, None, row_begin=3)


def test_row_window_step_stages_its_input_once(cuda_device):
    """The row operator's C++ autograd node stages the replicated input once,
    inside its forward, and hands the copy to the row backward (the fused
    tensor-core backward with its one-launch prologue), with the gradients
    of the unstaged row operators."""
    case = make_case(N=1, inC=64, outC=64, H=14, W=12, offset_scale=2.0, upstream="randn")
    args = (case["stride"], case["padding"], case["dilation"])
    rows = slice(4, 11)
    off_r = case["off"][:, :, rows].contiguous()
    m_r = case["m"][:, :, rows].contiguous()
    go_r = case["go"][:, :, rows].contiguous().cuda()
    x, w, b, off, m = (_leaf(t) for t in (case["x"], case["w"], case["b"], off_r, m_r))
    _native.profiler_read()
    _native.profiler_enable(True)
    try:
        out = deform_conv2d_rows(x, off, w, b, *args, m, row_begin=rows.start, flags=MATH_TF32)
        out.backward(go_r)
        torch.cuda.synchronize()
    finally:
        _native.profiler_enable(False)
    stats = _native.profiler_read()
    assert staging_launches(stats) == 1, stats
    assert "bwd_prologue" in stats and "bwd_fused_tc" in stats, sorted(stats)
    ops = _native.load_ops()
    ints = (1, 1, 1, 1, 1, 1, 1, 1, rows.start, MATH_TF32)
    ref = ops.deform_conv2d_backward_rows(go_r, x.detach(), w.detach(), off.detach(),
                                          m.detach(), b.detach(), *ints)
    got = (x.grad, off.grad, m.grad, w.grad, b.grad)
    for a, r in zip(got, ref):
        scale = max(1.0, float(r.abs().max()))
        torch.testing.assert_close(a, r, rtol=1e-4, atol=1e-4 * scale)
