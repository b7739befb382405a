"""Small convolution groups that tile a deformable group (one thread per
pixel and deformable group, dcn_dgroup.cu): forward and all gradients against
the CPU oracle at the fp32 tolerances of the reference's tests (forward 1e-4;
grad_input 2e-3, offset / mask / weight / bias 1e-4, tests/test_backward.py:
41-47), every (channels, out channels, groups per deformable group) the
library instantiates, plus DCNv1, asymmetric geometry and boundary-heavy
offsets; the profiler confirms these kernels ran."""
import numpy as np
import pytest

from _util import assert_close, make_case, run_oracle, run_ours
from pytorch_mps_deform_conv2d_b200 import _native
from pytorch_mps_deform_conv2d_b200.ops import MATH_FP32, MATH_TF32

pytestmark = pytest.mark.gpu

TOL = {"x": 2e-3, "off": 1e-4, "m": 1e-4, "w": 1e-4, "b": 1e-4}

CASES = {
    # (Cg, Og, groups per deformable group)
    "cg2-og2-gpd8-grouped-like": dict(inC=64, outC=64, groups=32, dg=4, H=12, W=13,
                                      offset_scale=2.0, mask_kind="sigmoid"),
    "cg1-og1-gpd16-depthwise": dict(inC=16, outC=16, groups=16, dg=1, H=10, W=11),
    "cg1-og1-gpd4": dict(inC=8, outC=8, groups=8, dg=2, H=9, W=10),
    "cg1-og1-gpd8": dict(inC=16, outC=16, groups=16, dg=2, H=9, W=9),
    "cg2-og2-gpd2": dict(inC=8, outC=8, groups=4, dg=2, H=9, W=10),
    "cg2-og2-gpd4": dict(inC=16, outC=16, groups=8, dg=2, H=9, W=10),
    "cg4-og4-gpd1": dict(inC=8, outC=8, groups=2, dg=2, H=9, W=10),
    "cg4-og4-gpd2": dict(inC=16, outC=16, groups=4, dg=2, H=9, W=10),
    "cg1-og2-gpd4": dict(inC=8, outC=16, groups=8, dg=2, H=9, W=10),
    "cg1-og2-gpd8": dict(inC=16, outC=32, groups=16, dg=2, H=9, W=10),
    "cg2-og4-gpd2": dict(inC=8, outC=16, groups=4, dg=2, H=9, W=10),
    "cg2-og4-gpd4": dict(inC=16, outC=32, groups=8, dg=2, H=9, W=10),
    "cg2-og2-gpd8-v1-nobias": dict(inC=64, outC=64, groups=32, dg=4, H=10, W=9,
                                   use_mask=False, use_bias=False, offset_scale=2.0),
    "cg2-og2-gpd8-asym": dict(inC=32, outC=32, groups=16, dg=2, H=9, W=12, kh=3, kw=2,
                              stride=(2, 1), pad=(1, 2), dil=(2, 1), offset_scale=2.0),
    "cg2-og2-gpd8-boundary": dict(N=3, inC=32, outC=32, groups=16, dg=2, H=7, W=8,
                                  offset_scale=8.0),
}


def _profiled(case, flags, backward):
    _native.profiler_read()
    _native.profiler_enable(True)
    try:
        out, grads = run_ours(case, flags=flags, backward=backward)
    finally:
        _native.profiler_enable(False)
    return out, grads, _native.profiler_read()


@pytest.mark.parametrize("flags", [MATH_FP32, MATH_TF32], ids=["fp32", "tf32"])
@pytest.mark.parametrize("name", sorted(CASES))
def test_dgroup_forward_backward(cuda_device, name, flags):
    # tiny groups have no tensor-core tiling: TF32 mode runs these fp32 kernels too
    case = make_case(upstream="randn", **CASES[name])
    out, grads, stats = _profiled(case, flags, backward=True)
    assert "fwd_dgroup" in stats and "bwd_dgroup" in stats, sorted(stats)
    ref, rgrads = run_oracle(case)
    scale = max(1.0, float(np.abs(ref).max()))
    assert_close(out, ref, rtol=1e-4, atol=1e-4 * scale, name="out")
    assert set(grads) == set(rgrads)
    for k, want in rgrads.items():
        s = max(1.0, float(np.abs(want).max()))
        assert_close(grads[k], want, rtol=TOL[k], atol=TOL[k] * s, name=f"grad_{k}")
