"""Bounded device waits of the tensor-core kernels surface as an error.

Every mbarrier wait of the warp-specialised kernels has a cycle budget.  The
test switch DCN_TEST_WAIT_TIMEOUT makes the kernels' TMA producers issue
nothing and shortens the budget to about a millisecond, so the consumers'
waits run out: each CTA then raises its kernel family's bit of the device
error word, drains what it issued, frees its tensor memory and returns
(nothing traps, nothing spins without a bound).  The tests check that the
word reports it, that check_device_status() raises, that reading clears it,
and that the device stays usable: the next normal call matches the oracle.
"""
import time

import numpy as np
import pytest

from _util import make_case, rel_norm_err, run_oracle, run_ours
from pytorch_mps_deform_conv2d_b200 import check_device_status, device_status
from pytorch_mps_deform_conv2d_b200.ops import (MATH_TF32, STATUS_BWD_DATA_TIMEOUT,
                                                STATUS_BWD_WEIGHT_TIMEOUT,
                                                STATUS_FWD_WAIT_TIMEOUT, TEST_WAIT_TIMEOUT)

pytestmark = pytest.mark.gpu

# 64 channels in and out: the tensor-core forward, grad-column and
# weight-gradient kernels all take this shape
CASE = dict(N=2, inC=64, outC=64, H=16, W=16, offset_scale=2.0, mask_kind="sigmoid")


def _normal_call_matches_oracle():
    case = make_case(**CASE, seed=1)
    out, grads = run_ours(case, flags=MATH_TF32)
    ref, rgrads = run_oracle(case)
    assert rel_norm_err(out, ref) <= 5e-3
    for k, v in rgrads.items():
        assert rel_norm_err(grads[k], v) <= 1e-3, k
    assert device_status() == 0


def test_status_word_starts_clear(cuda_device):
    device_status(clear=True)
    assert device_status(clear=False) == 0
    check_device_status()  # no error: does not raise


def test_forward_wait_timeout_is_reported(cuda_device):
    device_status(clear=True)
    case = make_case(**CASE)
    t0 = time.perf_counter()
    run_ours(case, flags=MATH_TF32 | TEST_WAIT_TIMEOUT, backward=False)
    word = device_status(clear=False)
    assert time.perf_counter() - t0 < 30.0
    assert word & STATUS_FWD_WAIT_TIMEOUT, word
    with pytest.raises(RuntimeError, match="forward"):
        check_device_status()
    assert device_status(clear=False) == 0  # the check cleared it
    _normal_call_matches_oracle()


def test_backward_wait_timeouts_are_reported(cuda_device):
    device_status(clear=True)
    case = make_case(**CASE)
    run_ours(case, flags=MATH_TF32 | TEST_WAIT_TIMEOUT, backward=True)
    word = device_status(clear=True)
    assert word & STATUS_BWD_DATA_TIMEOUT, word
    assert word & STATUS_BWD_WEIGHT_TIMEOUT, word
    assert device_status(clear=False) == 0
    _normal_call_matches_oracle()


def test_repeated_timeouts_leave_the_device_usable(cuda_device):
    case = make_case(**CASE)
    for _ in range(3):
        run_ours(case, flags=MATH_TF32 | TEST_WAIT_TIMEOUT, backward=True)
    assert device_status(clear=True) != 0
    _normal_call_matches_oracle()
    out, _ = run_ours(case, flags=MATH_TF32, backward=False)
    assert np.isfinite(out).all()
