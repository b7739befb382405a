"""16-bit I/O: every tensor bf16, or every tensor fp16.  Forward on tcgen05
with 16-bit operands of the same type when channels per group and per
deformable group are multiples of 64, else the fp32 kernels on upcast copies.
Backward on the fused tensor-core kernel with 16-bit operands of the same type
(kind::f16: 16-bit corner gathers and column values, fp32 accumulation and
fp32 reductions) when channels per group and per deformable group are
multiples of 32 and a group has at most 256 out channels, else the fp32 route
on upcast copies; gradients returned in the input's dtype.  Parity against the oracle run on the same rounded inputs:
norm-wise relative error <= 1e-2 for outputs and gradients (bf16 keeps 8
mantissa bits, fp16 11: one rounding of the column values and one of the
result are ~2e-3 each in bf16)."""
import numpy as np
import pytest
import torch

import pytorch_mps_deform_conv2d_b200 as dcn
from _util import make_case, rel_norm_err, run_oracle
from pytorch_mps_deform_conv2d_b200 import _native

pytestmark = pytest.mark.gpu

TOL = 1e-2

CASES = {  # name -> (case, bf16 tensor-core forward expected)
    "c64-o64": (dict(inC=64, outC=64, H=10, W=11, offset_scale=2.0), True),
    "c128-o128-dg2": (dict(inC=128, outC=128, dg=2, H=9, W=10, offset_scale=3.0), True),
    "c256-o256-neck-like": (dict(N=1, inC=256, outC=256, H=16, W=19, offset_scale=4.0,
                                 mask_kind="sigmoid", weight_kind="kaiming"), True),
    "c128-o64-g2-v1-nobias": (dict(inC=128, outC=64, groups=2, H=9, W=9, use_mask=False,
                                   use_bias=False, offset_scale=2.0), True),
    "c64-o48-asym-boundary": (dict(inC=64, outC=48, H=9, W=13, kh=3, kw=2, stride=(2, 1),
                                   pad=(1, 2), dil=(2, 1), offset_scale=8.0), True),
    "c64-o512-wide": (dict(N=1, inC=64, outC=512, H=7, W=8, offset_scale=2.0), True),
    "c32-o32-upcast": (dict(inC=32, outC=32, H=9, W=10, offset_scale=2.0), False),
    "c6-o6-g3-upcast": (dict(inC=6, outC=6, groups=3, H=8, W=9), False),
}


DTYPES = {"bf16": (torch.bfloat16, "bf16"), "fp16": (torch.float16, "f16")}


def _bf16_case(spec, dt=torch.bfloat16):
    case = make_case(upstream="randn", **spec)
    r = lambda t: None if t is None else t.to(dt)
    c16 = {k: r(case[k]) for k in ("x", "w", "b", "off", "m", "go")}
    # the oracle sees exactly the bf16 values, upcast
    c32 = dict(case, **{k: (None if v is None else v.float()) for k, v in c16.items()})
    return case, c16, c32


def _run(case, c16, backward):
    leaves = {k: (None if c16[k] is None else c16[k].cuda().requires_grad_(backward))
              for k in ("x", "w", "b", "off", "m")}
    out = dcn.deform_conv2d(leaves["x"], leaves["off"], leaves["w"], leaves["b"],
                            case["stride"], case["padding"], case["dilation"], leaves["m"])
    grads = {}
    if backward:
        out.backward(c16["go"].cuda())
        grads = {k: v.grad for k, v in leaves.items() if v is not None}
    torch.cuda.synchronize()
    return out, grads


@pytest.mark.parametrize("dtype", sorted(DTYPES))
@pytest.mark.parametrize("name", sorted(CASES))
def test_half_forward(cuda_device, name, dtype):
    dt, tag = DTYPES[dtype]
    spec, tc = CASES[name]
    case, c16, c32 = _bf16_case(spec, dt)
    _native.profiler_read()
    _native.profiler_enable(True)
    try:
        out, _ = _run(case, c16, backward=False)
    finally:
        _native.profiler_enable(False)
    stats = _native.profiler_read()
    assert out.dtype == dt
    assert (f"fwd_tc_{tag}" in stats) == tc, sorted(stats)
    if not tc:
        assert f"{tag}_to_f32" in stats and f"f32_to_{tag}" in stats, sorted(stats)
    ref, _ = run_oracle(c32, backward=False)
    got = out.float().cpu().numpy()
    assert rel_norm_err(got, ref) <= TOL
    np.testing.assert_allclose(got, ref, rtol=0, atol=2 * TOL * float(np.abs(ref).max()))


def _fused16(spec):
    """Whether the fused 16-bit tensor-core backward covers the case."""
    g = spec.get("groups", 1)
    cg, og = spec["inC"] // g, spec["outC"] // g
    cpg = spec["inC"] // spec.get("dg", 1)
    return cg % 32 == 0 and cpg % 32 == 0 and og % 16 == 0 and og <= 256 and spec["inC"] % 8 == 0


@pytest.mark.parametrize("dtype", sorted(DTYPES))
@pytest.mark.parametrize("name", sorted(CASES))
def test_half_backward(cuda_device, name, dtype):
    dt, tag = DTYPES[dtype]
    spec, _ = CASES[name]
    case, c16, c32 = _bf16_case(spec, dt)
    _native.profiler_read()
    _native.profiler_enable(True)
    try:
        out, grads = _run(case, c16, backward=True)
    finally:
        _native.profiler_enable(False)
    stats = _native.profiler_read()
    fused = f"bwd_fused_tc_{tag}"
    assert (fused in stats) == _fused16(spec), sorted(stats)
    ref, rgrads = run_oracle(c32)
    assert rel_norm_err(out.detach().float().cpu().numpy(), ref) <= TOL
    assert set(grads) == set(rgrads)
    for k, want in rgrads.items():
        assert grads[k].dtype == dt, k
        err = rel_norm_err(grads[k].float().cpu().numpy(), want)
        assert err <= TOL, f"grad_{k}: {err:.2e}"


@pytest.mark.parametrize("dtype", sorted(DTYPES))
def test_half_pack_module(cuda_device, dtype):
    dt, _ = DTYPES[dtype]
    torch.manual_seed(0)
    mod = dcn.DeformConv2dPack(64, 64, 3, padding=1).cuda()
    with torch.no_grad():
        mod.conv_offset.weight.normal_(0, 0.02)
    x = torch.randn(2, 64, 10, 12, device="cuda")
    ref = mod(x)
    mod16 = mod.to(dt)
    x16 = x.to(dt).requires_grad_()
    out = mod16(x16)
    assert out.dtype == dt
    assert rel_norm_err(out.float().detach().cpu().numpy(), ref.detach().cpu().numpy()) <= 3 * TOL
    out.float().square().sum().backward()
    assert x16.grad.dtype == dt and torch.isfinite(x16.grad.float()).all()
    assert mod16.weight.grad.dtype == dt


@pytest.mark.parametrize("dtype", sorted(DTYPES))
def test_capi_half_backward_matches_operator(cuda_device, dtype):
    """dcn_backward_bf16 / dcn_backward_f16 through ctypes give the operator's
    16-bit gradients."""
    from pytorch_mps_deform_conv2d_b200.ops import MATH_FP32
    dt, tag = DTYPES[dtype]
    spec, _ = CASES["c64-o64"]
    case, c16, _ = _bf16_case(spec, dt)
    ops = _native.load_ops()
    d = {k: (None if v is None else v.cuda().contiguous()) for k, v in c16.items()}
    want = ops.deform_conv2d_backward(d["go"], d["x"], d["w"], d["off"], d["m"], d["b"],
                                      1, 1, 1, 1, 1, 1, 1, 1, MATH_FP32)
    lib = _native.load_capi()
    N, C, H, W = d["x"].shape
    s = _native.DcnShape(N, C, H, W, d["w"].shape[0], 3, 3, 1, 1, 1, 1, 1, 1, 1, 1)
    nbytes = getattr(lib, f"dcn_backward_{tag}_workspace_size")(s, MATH_FP32)
    assert nbytes > 0
    ws = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    outs = [torch.empty_like(t) for t in (d["x"], d["off"], d["m"], d["w"], d["b"])]
    ptr = lambda t: t.data_ptr()
    rc = getattr(lib, f"dcn_backward_{tag}")(s, ptr(d["go"]), ptr(d["x"]), ptr(d["w"]), ptr(d["off"]),
                               ptr(d["m"]), *[ptr(t) for t in outs], MATH_FP32, ptr(ws), nbytes,
                               torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib.dcn_last_error()
    torch.cuda.synchronize()
    for got, ref in zip(outs, want):
        assert got.dtype == dt
        torch.testing.assert_close(got.float(), ref.float(), rtol=1e-2, atol=1e-2)
