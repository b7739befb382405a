"""TF32 tensor-core mode (tcgen05): parity against the CPU oracle within the
stated TF32 tolerance -- outputs <= 5e-3 relative (norm-wise, and element-wise
against 5e-3 x max|ref|) -- and checks that the tensor-core kernels are the
ones that ran."""
import numpy as np
import pytest
import torch

from _util import make_case, rel_norm_err, run_oracle, run_ours
from pytorch_mps_deform_conv2d_b200 import _native
from pytorch_mps_deform_conv2d_b200.ops import ALGO_TC_COLUMN_BUFFER, ALGO_TC_GATHER_WEIGHT, MATH_TF32

pytestmark = pytest.mark.gpu

OUT_TOL = 5e-3

TC_CASES = {
    "c32-o32": dict(inC=32, outC=32, H=12, W=14, offset_scale=2.0),
    "c64-o48-v1-nobias": dict(inC=64, outC=48, H=11, W=9, use_mask=False, use_bias=False),
    "c64-o64-dg2": dict(inC=64, outC=64, dg=2, H=10, W=13, offset_scale=3.0),
    "c64-o32-g2": dict(inC=64, outC=32, groups=2, H=9, W=9),
    "c128-o16-asym": dict(inC=128, outC=16, H=8, W=11, kh=1, kw=3, stride=(2, 1),
                          pad=(0, 2), dil=(2, 1)),
    "c32-o512-ntiles": dict(N=1, inC=32, outC=512, H=7, W=9),
    # 512 out channels a tile (two 256-column accumulators), two tiles per
    # group, and two groups of 512
    "c64-o1024-wide-ntiles": dict(N=1, inC=64, outC=1024, H=6, W=9),
    "c128-o1024-g2-wide": dict(N=1, inC=128, outC=1024, groups=2, H=7, W=6, offset_scale=2.0),
    "c64-o256-boundary": dict(N=3, inC=64, outC=256, H=13, W=17, offset_scale=8.0),
    "c256-o256-neck-like": dict(N=1, inC=256, outC=256, H=20, W=30, offset_scale=4.0,
                                mask_kind="sigmoid", weight_kind="kaiming"),
    "c512-o512-dcnv1-like": dict(N=2, inC=512, outC=512, H=10, W=10, stride=(2, 1),
                                 pad=(2, 1), dil=(2, 1), dg=8, use_mask=False,
                                 use_bias=False, offset_scale=3.0, weight_kind="kaiming"),
}


@pytest.mark.parametrize("name", sorted(TC_CASES))
def test_forward_tf32(cuda_device, name):
    case = make_case(**TC_CASES[name])
    _native.profiler_read()
    _native.profiler_enable(True)
    try:
        out, _ = run_ours(case, flags=MATH_TF32, backward=False)
    finally:
        _native.profiler_enable(False)
    stats = _native.profiler_read()
    assert "fwd_tc" in stats, f"tensor-core forward did not run: {sorted(stats)}"
    ref, _ = run_oracle(case, backward=False)
    assert rel_norm_err(out, ref) <= OUT_TOL
    np.testing.assert_allclose(out, ref, rtol=0, atol=OUT_TOL * float(np.abs(ref).max()))


def test_tf32_falls_back_to_fp32_kernels_when_shape_not_covered(cuda_device):
    case = make_case(inC=6, outC=6)  # 6 channels per group: no tensor-core tiling
    _native.profiler_read()
    _native.profiler_enable(True)
    try:
        out, _ = run_ours(case, flags=MATH_TF32, backward=False)
    finally:
        _native.profiler_enable(False)
    stats = _native.profiler_read()
    assert "fwd_tc" not in stats
    ref, _ = run_oracle(case, backward=False)
    np.testing.assert_allclose(out, ref, rtol=1e-4, atol=1e-4 * max(1, np.abs(ref).max()))


def test_tf32_repeatable(cuda_device):
    case = make_case(inC=64, outC=64, H=16, W=16, offset_scale=2.0)
    a, _ = run_ours(case, flags=MATH_TF32, backward=False)
    b, _ = run_ours(case, flags=MATH_TF32, backward=False)
    assert np.array_equal(a, b)  # split tiles are summed in a fixed order: bitwise repeatable


GRAD_TOL = 1e-3  # norm-wise relative error of every gradient in TF32 mode

TC_BWD_CASES = {
    "c128-o64": dict(inC=128, outC=64, H=12, W=10, offset_scale=2.0),
    "c128-o32-dg4-v1": dict(inC=128, outC=32, H=8, W=12, dg=4, use_mask=False,
                            use_bias=False, offset_scale=3.0),
    "c256-o64-g2": dict(inC=256, outC=64, groups=2, H=10, W=8),
    "c256-o256-neck-like": dict(N=2, inC=256, outC=256, H=16, W=20, offset_scale=4.0,
                                mask_kind="sigmoid", weight_kind="kaiming"),
    "c512-o512-dcnv1-like": dict(N=2, inC=512, outC=512, H=10, W=8, stride=(2, 1),
                                 pad=(2, 1), dil=(2, 1), dg=8, use_mask=False,
                                 use_bias=False, offset_scale=3.0, weight_kind="kaiming"),
    "c128-o128-asym-boundary-p70": dict(inC=128, outC=128, H=9, W=14, kh=3, kw=1,
                                    stride=(2, 1), pad=(1, 0), offset_scale=8.0),
    # 64 / 32 channels per group: 128-row slots of 2 / 4 taps, the last one partial
    "c64-o64-training-like": dict(N=2, inC=64, outC=64, H=12, W=10, offset_scale=2.0,
                                  mask_kind="sigmoid", weight_kind="kaiming"),
    "c128-o64-g2-cg64": dict(inC=128, outC=64, groups=2, H=9, W=11, offset_scale=2.0),
    "c64-o64-g2-dg2-cg32": dict(inC=64, outC=64, groups=2, dg=2, H=10, W=9, offset_scale=3.0),
    "c32-o32-k1x3-v1": dict(inC=32, outC=32, kh=1, kw=3, H=8, W=13, pad=(0, 1),
                            use_mask=False, use_bias=False, offset_scale=2.0),
    # channels per group a multiple of 32 but neither of nor a divisor of 128:
    # slots straddle taps
    "c96-o64-cg96": dict(inC=96, outC=64, H=9, W=11, offset_scale=2.0),
    "c192-o128-g2-dg3-cg96": dict(inC=192, outC=128, groups=2, dg=3, H=8, W=10,
                                 offset_scale=2.0),
    "c160-o32-cg160-v1": dict(inC=160, outC=32, H=9, W=9, use_mask=False, use_bias=False,
                              offset_scale=3.0),
    # out channels per group a multiple of 16 but not of 32: a partial last K step
    "c64-o48-og48": dict(inC=64, outC=48, H=9, W=10, offset_scale=2.0),
    "c128-o96-g2-og48-cg64": dict(inC=128, outC=96, groups=2, H=8, W=9, offset_scale=2.0),
    "c128-o16-og16": dict(inC=128, outC=16, H=10, W=9, offset_scale=2.0),
}


def _kernels(case, path):
    """(flags, kernels that must run) of a backward route: the fused kernel
    covers up to 256 out channels per group (others keep the column buffer);
    the gather kernel covers only 128-channel multiples per group (others
    keep the column buffer)."""
    algo, kernels = WEIGHT_PATHS[path]
    g = case.get("groups", 1)
    cg, og = case["inC"] // g, case["outC"] // g
    col = ("bwd_data_tc", "bwd_weight_col")
    if path == "fused" and og > 256:
        return algo, col
    if path == "gather" and cg % 128 != 0:
        return algo, col
    return algo, kernels


# The tensor-core backward routes: the fused kernel (default in TF32: the
# columns stay on chip), the grad-column kernel with the dense weight GEMM
# over the column buffer, and the grad-column kernel with the weight kernel
# that gathers its own columns (no column buffer).
WEIGHT_PATHS = {"fused": (0, ("bwd_fused_tc",)),
                "col": (ALGO_TC_COLUMN_BUFFER, ("bwd_data_tc", "bwd_weight_col")),
                "gather": (ALGO_TC_GATHER_WEIGHT, ("bwd_data_tc", "bwd_weight_tc"))}


def _grad_errors(case, flags=MATH_TF32):
    _native.profiler_read()
    _native.profiler_enable(True)
    try:
        out, grads = run_ours(case, flags=flags)
    finally:
        _native.profiler_enable(False)
    stats = _native.profiler_read()
    ref, rgrads = run_oracle(case)
    errs = {k: rel_norm_err(grads[k], v) for k, v in rgrads.items()}
    elem = {k: float(np.abs(grads[k] - v).max() / max(1e-30, np.abs(v).max()))
            for k, v in rgrads.items()}
    return stats, rel_norm_err(out, ref), errs, elem


@pytest.mark.parametrize("path", sorted(WEIGHT_PATHS))
@pytest.mark.parametrize("name", sorted(TC_BWD_CASES))
def test_backward_tf32(cuda_device, name, path):
    algo, kernels = _kernels(TC_BWD_CASES[name], path)
    stats, out_err, errs, elem = _grad_errors(make_case(upstream="randn", **TC_BWD_CASES[name]),
                                              flags=MATH_TF32 | algo)
    assert all(k in stats for k in kernels), (kernels, sorted(stats))
    assert out_err <= OUT_TOL
    for k, e in errs.items():
        assert e <= GRAD_TOL, f"grad_{k}: norm-wise rel err {e:.2e} (all: {errs}, elem: {elem})"
        assert elem[k] <= 10 * GRAD_TOL, f"grad_{k}: max elem err {elem[k]:.2e} of max|ref|"


def test_backward_tf32_uncovered_shape_uses_fp32_kernels(cuda_device):
    # 48 input channels per group: not a multiple of 32, so the fp32 backward
    # kernels run and meet the fp32 tolerances.
    case = make_case(inC=48, outC=64, H=9, W=9, upstream="randn")
    stats, out_err, errs, elem = _grad_errors(case)
    assert "bwd_data_tc" not in stats and "bwd_fused_tc" not in stats
    assert "bwd_data_simt" in stats
    for k, e in errs.items():
        assert e <= 1e-4, f"grad_{k}: {e:.2e}"
