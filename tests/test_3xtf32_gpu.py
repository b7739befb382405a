"""3xTF32 tensor-core mode: the tcgen05 kernels with every operand split into
high and low TF32 parts must meet the fp32 tolerances of the reference's own
tests (forward 1e-4; grad_input 2e-3, offset / mask / weight / bias 1e-4,
tests/test_backward.py:41-47) on the shapes the tensor-core kernels cover,
and the tensor-core kernels must be the ones that ran."""
import numpy as np
import pytest

from _util import assert_close, make_case, run_oracle, run_ours
from pytorch_mps_deform_conv2d_b200 import _native
from pytorch_mps_deform_conv2d_b200.ops import MATH_3XTF32
from test_tf32_gpu import TC_BWD_CASES, TC_CASES, _kernels

pytestmark = pytest.mark.gpu

TOL = {"x": 2e-3, "off": 1e-4, "m": 1e-4, "w": 1e-4, "b": 1e-4}


def _run_profiled(case, backward, algo=0):
    _native.profiler_read()
    _native.profiler_enable(True)
    try:
        out, grads = run_ours(case, flags=MATH_3XTF32 | algo, backward=backward)
    finally:
        _native.profiler_enable(False)
    return out, grads, _native.profiler_read()


@pytest.mark.parametrize("name", sorted(TC_CASES))
def test_forward_3xtf32(cuda_device, name):
    case = make_case(**TC_CASES[name])
    out, _, stats = _run_profiled(case, backward=False)
    assert "fwd_tc" in stats, f"tensor-core forward did not run: {sorted(stats)}"
    ref, _ = run_oracle(case, backward=False)
    scale = max(1.0, float(np.abs(ref).max()))
    assert_close(out, ref, rtol=1e-4, atol=1e-4 * scale, name="out")


@pytest.mark.parametrize("path", ["col", "gather"])
@pytest.mark.parametrize("name", sorted(TC_BWD_CASES))
def test_backward_3xtf32(cuda_device, name, path):
    # the fused backward is TF32 only: 3xTF32 keeps the grad-column kernel
    algo, kernels = _kernels(TC_BWD_CASES[name], path)
    case = make_case(upstream="randn", **TC_BWD_CASES[name])
    out, grads, stats = _run_profiled(case, backward=True, algo=algo)
    assert all(k in stats for k in kernels), (kernels, sorted(stats))
    ref, rgrads = run_oracle(case)
    scale = max(1.0, float(np.abs(ref).max()))
    assert_close(out, ref, rtol=1e-4, atol=1e-4 * scale, name="out")
    assert set(grads) == set(rgrads)
    for k, want in rgrads.items():
        s = max(1.0, float(np.abs(want).max()))
        assert_close(grads[k], want, rtol=TOL[k], atol=TOL[k] * s, name=f"grad_{k}")


def test_3xtf32_is_closer_than_tf32(cuda_device):
    # The low parts must actually contribute: on a deep reduction the 3xTF32
    # forward error is far below the single-TF32 one.
    from pytorch_mps_deform_conv2d_b200.ops import MATH_TF32
    case = make_case(N=1, inC=256, outC=64, H=12, W=12, offset_scale=2.0)
    ref, _ = run_oracle(case, backward=False)
    one, _ = run_ours(case, flags=MATH_TF32, backward=False)
    three, _ = run_ours(case, flags=MATH_3XTF32, backward=False)
    e1 = float(np.abs(one - ref).max())
    e3 = float(np.abs(three - ref).max())
    assert e3 * 20 < e1, (e1, e3)
