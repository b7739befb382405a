"""Forward parity on the GPU against the CPU oracle: the reference's forward
matrix (tests/test_forward.py:47-89) and its hand-picked extras
(tests/test_forward.py:135-181), in fp32 mode with the reference's tolerance
(1e-4), through every fp32 kernel family; plus the golden vectors."""
import glob
import os

import numpy as np
import pytest
import torch

from _util import assert_close, make_case, np_, run_oracle, run_ours
from pytorch_mps_deform_conv2d_b200.ops import ALGO_SIMT_DIRECT, ALGO_SIMT_GEMM, MATH_FP32

pytestmark = pytest.mark.gpu

KERNELS = [(3, 3), (1, 1), (3, 1)]
_CASES = [(*k, s, p, d, m) for k in KERNELS for s in (1, 2) for p in (0, 1)
          for d in (1, 2) for m in (False, True)]
ALGOS = {"auto": MATH_FP32, "gemm": MATH_FP32 | ALGO_SIMT_GEMM,
         "direct": MATH_FP32 | ALGO_SIMT_DIRECT}


@pytest.mark.parametrize("algo", sorted(ALGOS))
@pytest.mark.parametrize("kh,kw,stride,pad,dil,use_mask", _CASES)
def test_forward_matrix(cuda_device, kh, kw, stride, pad, dil, use_mask, algo):
    case = make_case(kh=kh, kw=kw, stride=stride, pad=pad, dil=dil, use_mask=use_mask,
                     offset_scale=1.0)
    out, _ = run_ours(case, flags=ALGOS[algo], backward=False)
    ref, _ = run_oracle(case, backward=False)
    assert_close(out, ref, rtol=1e-4, atol=1e-4, name="out")


EXTRA = {
    "rect-input": dict(H=8, W=11),
    "asym-stride": dict(H=8, W=11, stride=(2, 1)),
    "asym-pad": dict(H=8, W=11, pad=(0, 2)),
    "asym-dilation": dict(H=8, W=11, dil=(2, 1)),
    "rect-kernel-1x3": dict(H=8, W=11, kh=1, kw=3, pad=(0, 1)),
    "asym-everything": dict(H=8, W=11, kh=1, kw=3, stride=(2, 1), pad=(0, 2), dil=(2, 1)),
    "no-bias": dict(use_bias=False),
    "no-bias-v1": dict(use_bias=False, use_mask=False),
    "n1-odd-channels": dict(N=1, inC=3, outC=5),
    "boundary-stress": dict(offset_scale=8.0),
    "boundary-stress-v1": dict(offset_scale=8.0, use_mask=False),
    "large-spatial": dict(N=2, inC=8, H=33, W=35, stride=2, pad=1),
    "dg2": dict(dg=2),
    "dg2-v1": dict(dg=2, use_mask=False),
    "dg2-cpg3": dict(dg=2, inC=6),
    "dg-eq-C": dict(dg=4),
    "dg2-asym": dict(dg=2, H=8, W=11, stride=(2, 1), pad=(0, 2), dil=(2, 1)),
    "g2": dict(groups=2),
    "g2-v1": dict(groups=2, use_mask=False),
    "g2-c6": dict(groups=2, inC=6),
    "g2-asym": dict(groups=2, H=8, W=11, stride=(2, 1), pad=(0, 2), dil=(2, 1)),
    "g2-dg2": dict(groups=2, dg=2),
    "g-eq-outC-depthwise": dict(inC=6, outC=6, groups=6),
    # wider channel counts: the tiled kernels' vector paths and tile edges
    "c32-o40-dg2": dict(inC=32, outC=40, H=13, W=17, dg=2, offset_scale=2.0),
    "c64-o136-tiles": dict(N=3, inC=64, outC=136, H=15, W=19, offset_scale=3.0),
    "c48-g3-dg4": dict(inC=48, outC=48, groups=3, dg=4, H=11, W=12),
    "c24-dg3-cpg8": dict(inC=24, outC=16, dg=3, H=10, W=10),
    "c20-dg10-cpg2": dict(inC=20, outC=12, dg=10, H=10, W=10),
}


@pytest.mark.parametrize("algo", sorted(ALGOS))
@pytest.mark.parametrize("name", sorted(EXTRA))
def test_forward_extra(cuda_device, name, algo):
    case = make_case(**EXTRA[name])
    out, _ = run_ours(case, flags=ALGOS[algo], backward=False)
    ref, _ = run_oracle(case, backward=False)
    scale = max(1.0, float(np.abs(ref).max()))
    assert_close(out, ref, rtol=1e-4, atol=1e-4 * scale, name=name)


GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.mark.parametrize("name", sorted(os.path.splitext(os.path.basename(p))[0]
                                        for p in glob.glob(os.path.join(GOLDEN, "*.npz"))))
def test_forward_golden(cuda_device, name):
    import pytorch_mps_deform_conv2d_b200 as dcn
    z = np.load(os.path.join(GOLDEN, name + ".npz"))
    t = lambda k: torch.from_numpy(z[k]).to(cuda_device) if k in z.files else None
    dcn.set_math_mode("fp32")
    try:
        out = dcn.deform_conv2d(t("x"), t("offset"), t("weight"), bias=t("bias"),
                                stride=tuple(z["stride"]), padding=tuple(z["padding"]),
                                dilation=tuple(z["dilation"]), mask=t("mask"))
    finally:
        dcn.set_math_mode(None)
    scale = max(1.0, float(np.abs(z["out"]).max()))
    assert_close(np_(out), z["out"], rtol=1e-4, atol=1e-4 * scale, name=name)
    if name == "example01":
        assert round(float(out.mean()), 5) == -0.70549


def test_output_is_not_aliased_and_inputs_untouched(cuda_device):
    case = make_case(inC=16, outC=16)
    before = {k: v.clone() for k, v in case.items() if isinstance(v, torch.Tensor)}
    run_ours(case, flags=MATH_FP32)
    for k, v in before.items():
        assert torch.equal(case[k], v)


def test_noncontiguous_inputs(cuda_device):
    case = make_case(inC=8, outC=8, H=10, W=10)
    x = case["x"].to(cuda_device).permute(0, 1, 3, 2).contiguous().permute(0, 1, 3, 2)
    assert not x.is_contiguous()
    from pytorch_mps_deform_conv2d_b200.ops import deform_conv2d_ex
    out = deform_conv2d_ex(x, case["off"].to(cuda_device), case["w"].to(cuda_device),
                           case["b"].to(cuda_device), case["stride"], case["padding"],
                           case["dilation"], case["m"].to(cuda_device), flags=MATH_FP32)
    ref, _ = run_oracle(case, backward=False)
    assert_close(np_(out), ref, rtol=1e-4, atol=1e-4)


def test_empty_batch(cuda_device):
    import pytorch_mps_deform_conv2d_b200 as dcn
    x = torch.randn(0, 4, 9, 9, device=cuda_device)
    w = torch.randn(6, 4, 3, 3, device=cuda_device)
    o = torch.randn(0, 18, 9, 9, device=cuda_device)
    out = dcn.deform_conv2d(x, o, w, padding=1)
    assert out.shape == (0, 6, 9, 9)
