"""Pins the CPU oracle (oracle/dcn_oracle.c) before anything is checked
against it.

* golden vectors: tests/golden/*.npz were produced by the reference package
  itself (its CPU route, src/deform_conv2d_mps/ops.py:165-169) by
  tests/golden/make_golden.py; the oracle must reproduce every forward output
  and all five gradients;
* known answer: example/example01_deform_conv2d_cpu_mps.py prints an output
  mean of -0.70549 on every platform the reference recorded;
* the unfold / fold ladder of the reference (tests/diag_im2col.py:127-145,
  tests/diag_col2im.py:83-100): with zero offsets and no mask the column
  buffer is F.unfold and the col2im scatter is F.fold.
"""
import glob
import json
import os

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import oracle
from _util import assert_close

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
CASES = sorted(os.path.splitext(os.path.basename(p))[0]
               for p in glob.glob(os.path.join(GOLDEN, "*.npz")))


def _load(name):
    z = np.load(os.path.join(GOLDEN, name + ".npz"))
    return {k: z[k] for k in z.files}


def test_golden_set_present():
    assert len(CASES) >= 14
    with open(os.path.join(GOLDEN, "index.json")) as f:
        idx = json.load(f)
    assert set(idx["cases"]) == set(CASES)


@pytest.mark.parametrize("name", CASES)
def test_oracle_matches_golden(name):
    z = _load(name)
    args = dict(stride=tuple(z["stride"]), padding=tuple(z["padding"]),
                dilation=tuple(z["dilation"]))
    out = oracle.forward(z["x"], z["offset"], z["weight"], z.get("bias"), mask=z.get("mask"), **args)
    scale = max(1.0, float(np.abs(z["out"]).max()))
    assert_close(out, z["out"], rtol=1e-5, atol=1e-5 * scale, name=f"{name}: out")
    gx, goff, gm, gw, gb = oracle.backward(z["grad_out"], z["x"], z["offset"], z["weight"],
                                           z.get("bias"), mask=z.get("mask"), **args)
    for key, got in (("grad_x", gx), ("grad_offset", goff), ("grad_weight", gw),
                     ("grad_mask", gm), ("grad_bias", gb)):
        if key not in z:
            assert got is None
            continue
        scale = max(1.0, float(np.abs(z[key]).max()))
        assert_close(got, z[key], rtol=1e-4, atol=1e-5 * scale, name=f"{name}: {key}")


def test_known_answer_example01():
    z = _load("example01")
    out = oracle.forward(z["x"], z["offset"], z["weight"], z["bias"], 1, 1, 1, z["mask"])
    assert out.shape == (2, 6, 10, 12)
    assert round(float(out.mean()), 5) == -0.70549


@pytest.mark.parametrize("k,stride,pad,dil", [((3, 3), 1, 1, 1), ((3, 1), 2, 0, 2),
                                              ((1, 3), (2, 1), (0, 2), (2, 1))])
def test_im2col_zero_offset_is_unfold(k, stride, pad, dil):
    torch.manual_seed(0)
    C, H, W = 3, 8, 11
    x = torch.randn(C, H, W)
    Ho, Wo = oracle.out_size(H, W, k[0], k[1], stride, pad, dil)
    off = torch.zeros(2 * k[0] * k[1], Ho, Wo)
    col = oracle.im2col(x.numpy(), off.numpy(), None, k[0], k[1], stride, pad, dil)
    ref = F.unfold(x[None], k, dilation=dil, padding=pad, stride=stride)[0]
    assert_close(col, ref.numpy(), rtol=1e-6, atol=1e-6)


@pytest.mark.parametrize("k,stride,pad,dil", [((3, 3), 1, 1, 1), ((3, 1), 2, 0, 2)])
def test_col2im_zero_offset_is_fold(k, stride, pad, dil):
    torch.manual_seed(1)
    C, H, W = 3, 8, 11
    Ho, Wo = oracle.out_size(H, W, k[0], k[1], stride, pad, dil)
    col = torch.randn(C * k[0] * k[1], Ho * Wo)
    off = torch.zeros(2 * k[0] * k[1], Ho, Wo)
    gim = oracle.col2im(col.numpy(), off.numpy(), None, H, W, k[0], k[1], stride, pad, dil)
    ref = F.fold(col[None], (H, W), k, dilation=dil, padding=pad, stride=stride)[0]
    assert_close(gim, ref.numpy(), rtol=1e-5, atol=1e-5)


def test_oracle_rejects_bad_geometry():
    x = np.zeros((1, 4, 5, 5), np.float32)
    w = np.zeros((6, 3, 3, 3), np.float32)  # 4 channels not divisible into groups of 3
    off = np.zeros((1, 18, 3, 3), np.float32)
    with pytest.raises(ValueError):
        oracle.forward(x, off, w)
