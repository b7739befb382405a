"""Channels-last input (DCN_INPUT_NHWC): an input in torch's channels_last
memory format goes to the library as it lies.  Its results equal the
contiguous input's on every kernel family and math mode, grad_input comes back
channels-last, and neither layout transpose runs (the input is staged by a
plain copy, the input gradient accumulated in place)."""
import pytest
import torch

from _util import make_case
from pytorch_mps_deform_conv2d_b200 import _native
from pytorch_mps_deform_conv2d_b200.ops import (ALGO_SIMT_DIRECT, ALGO_SIMT_GEMM,
                                                ALGO_TC_COLUMN_BUFFER, ALGO_TC_GATHER_WEIGHT, MATH_3XTF32, MATH_FP32,
                                                MATH_TF32, deform_conv2d_ex, deform_conv2d_rows)

pytestmark = pytest.mark.gpu

CL = torch.channels_last

# name -> (case, flags, kernels that must run)
CASES = {
    "tc-tf32": (dict(inC=128, outC=64, H=10, W=9, offset_scale=2.0), MATH_TF32,
                ("fwd_tc", "bwd_fused_tc")),
    "tc-tf32-column-buffer": (dict(inC=128, outC=64, H=10, W=9, offset_scale=2.0),
                              MATH_TF32 | ALGO_TC_COLUMN_BUFFER,
                              ("fwd_tc", "bwd_data_tc", "bwd_weight_col")),
    "tc-tf32-gather-weight": (dict(inC=128, outC=64, H=10, W=9, offset_scale=2.0),
                              MATH_TF32 | ALGO_TC_GATHER_WEIGHT, ("bwd_weight_tc",)),
    "tc-3xtf32-cg32-dg2": (dict(inC=64, outC=32, H=9, W=11, dg=2, offset_scale=2.0),
                           MATH_3XTF32, ("fwd_tc", "bwd_data_tc")),
    "simt-fp32": (dict(inC=8, outC=12, H=9, W=10, dg=2, offset_scale=2.0), MATH_FP32,
                  ("bwd_data_simt", "bwd_weight_simt")),
    "simt-gemm-fp32-v1": (dict(inC=6, outC=6, H=8, W=9, use_mask=False, use_bias=False),
                          MATH_FP32 | ALGO_SIMT_GEMM, ("fwd_simt_gemm", "bwd_data_simt")),
    "dgroup": (dict(inC=32, outC=32, groups=16, dg=2, H=9, W=10, offset_scale=2.0), MATH_FP32,
               ("fwd_dgroup", "bwd_dgroup")),
    "small-direct-stride2": (dict(inC=6, outC=6, groups=3, H=11, W=9, stride=2, offset_scale=2.0),
                             MATH_FP32 | ALGO_SIMT_DIRECT, ("fwd_simt_direct", "bwd_small")),
}


def _run(case, flags, fmt, rows=None):
    x = case["x"].cuda().to(memory_format=fmt).requires_grad_(True)
    d = lambda t: None if t is None else t.cuda().requires_grad_(True)
    off, w, b, m = d(case["off"]), d(case["w"]), d(case["b"]), d(case["m"])
    args = (case["stride"], case["padding"], case["dilation"])
    if rows is None:
        out = deform_conv2d_ex(x, off, w, b, *args, m, flags=flags)
        out.backward(case["go"].cuda())
    else:
        r0, r1 = rows
        offs = off.detach()[:, :, r0:r1].contiguous().requires_grad_()
        ms = m.detach()[:, :, r0:r1].contiguous().requires_grad_() if m is not None else None
        out = deform_conv2d_rows(x, offs, w, b, *args, ms, row_begin=r0, flags=flags)
        out.backward(case["go"].cuda()[:, :, r0:r1].contiguous())
        off, m = offs, ms
    torch.cuda.synchronize()
    grads = {k: t.grad for k, t in (("x", x), ("off", off), ("w", w), ("b", b), ("m", m))
             if t is not None}
    return out.detach(), grads


def _same(a, b, name):
    # the kernels compute from the same NHWC staging copy; the grad_input,
    # grad_weight and grad_offset reductions use atomics, whose order differs
    s = max(1.0, float(b.abs().max()))
    torch.testing.assert_close(a, b, rtol=1e-5, atol=1e-5 * s, msg=name)


@pytest.mark.parametrize("name", sorted(CASES))
def test_channels_last_matches_contiguous(cuda_device, name):
    spec, flags, kernels = CASES[name]
    case = make_case(upstream="randn", **spec)
    _native.profiler_read()
    _native.profiler_enable(True)
    try:
        out_cl, g_cl = _run(case, flags, CL)
    finally:
        _native.profiler_enable(False)
    stats = _native.profiler_read()
    for k in kernels + ("copy_nhwc",):
        assert k in stats, (k, sorted(stats))
    assert not {"nchw_to_nhwc", "nhwc_to_nchw", "fwd_prologue", "bwd_finish"} & set(stats), \
        sorted(stats)
    assert g_cl["x"].is_contiguous(memory_format=CL) and not g_cl["x"].is_contiguous()
    out, g = _run(case, flags, torch.contiguous_format)
    assert out.is_contiguous() and out_cl.is_contiguous()
    _same(out_cl, out, "out")
    for k in g:
        _same(g_cl[k], g[k], f"grad_{k}")


def test_channels_last_row_window(cuda_device):
    case = make_case(inC=128, outC=64, H=12, W=9, offset_scale=2.0, upstream="randn")
    out_cl, g_cl = _run(case, MATH_TF32, CL, rows=(3, 8))
    out, g = _run(case, MATH_TF32, torch.contiguous_format, rows=(3, 8))
    assert g_cl["x"].is_contiguous(memory_format=CL)
    _same(out_cl, out, "out")
    for k in g:
        _same(g_cl[k], g[k], f"grad_{k}")


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("inC", [64, 24])  # 16-bit tensor-core forward / upcast forward
def test_channels_last_half(cuda_device, inC, dt):
    case = make_case(inC=inC, outC=64, H=9, W=10, offset_scale=2.0, upstream="randn")
    bf = {k: (v.to(dt) if isinstance(v, torch.Tensor) else v) for k, v in case.items()}
    out_cl, g_cl = _run(bf, MATH_TF32, CL)
    out, g = _run(bf, MATH_TF32, torch.contiguous_format)
    assert out_cl.dtype == dt
    assert g_cl["x"].dtype == dt and g_cl["x"].is_contiguous(memory_format=CL)
    torch.testing.assert_close(out_cl.float(), out.float(), rtol=0, atol=0)
    for k in g:
        s = max(1.0, float(g[k].float().abs().max()))
        torch.testing.assert_close(g_cl[k].float(), g[k].float(), rtol=1e-2, atol=1e-2 * s,
                                   msg=f"grad_{k}")


def test_non_dense_input_is_made_contiguous(cuda_device):
    # a strided view (every other column) is neither layout: copied to NCHW
    case = make_case(inC=8, outC=6, H=9, W=9, upstream="randn")
    wide = torch.randn(2, 8, 9, 18, device="cuda")
    x = wide[:, :, :, ::2]
    args = (case["stride"], case["padding"], case["dilation"])
    d = lambda t: t.cuda()
    got = deform_conv2d_ex(x, d(case["off"]), d(case["w"]), d(case["b"]), *args, d(case["m"]),
                           flags=MATH_FP32)
    want = deform_conv2d_ex(x.contiguous(), d(case["off"]), d(case["w"]), d(case["b"]), *args,
                            d(case["m"]), flags=MATH_FP32)
    torch.testing.assert_close(got, want, rtol=0, atol=0)
