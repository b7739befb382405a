"""The tensor-core forward's split last round.  When the tile count leaves the
last round of the persistent grid short, the remaining tiles are cut by K
over all SMs and each tile's pieces are summed, in CTA order, by the piece that
finishes last.  Checked through the C ABI: against the oracle; bitwise
repeatable; equal (up to the order of fp32 additions) to the whole-tile
schedule that a workspace without the split scratch -- one byte short of the
size query -- selects; and for every operand mode (TF32, 3xTF32, bf16 with
512-column tiles)."""
import ctypes

import numpy as np
import pytest
import torch

from _util import make_case, rel_norm_err, run_oracle
from pytorch_mps_deform_conv2d_b200 import _native
from pytorch_mps_deform_conv2d_b200.ops import MATH_3XTF32, MATH_TF32

pytestmark = pytest.mark.gpu


def _p(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _shape(case):
    x, w = case["x"], case["w"]
    k = w.shape[2] * w.shape[3]
    return _native.DcnShape(
        batch=x.shape[0], in_channels=x.shape[1], height=x.shape[2], width=x.shape[3],
        out_channels=w.shape[0], kernel_h=w.shape[2], kernel_w=w.shape[3],
        stride_h=case["stride"][0], stride_w=case["stride"][1], pad_h=case["padding"][0],
        pad_w=case["padding"][1], dilation_h=case["dilation"][0], dilation_w=case["dilation"][1],
        groups=x.shape[1] // w.shape[1], deformable_groups=case["off"].shape[1] // (2 * k))


def _forward(case, dev, flags, short=False, dtype=torch.float32):
    """dcn_forward (or dcn_forward_bf16) with the queried workspace, or one
    byte less (`short`)."""
    lib = _native.load_capi()
    tag = "" if dtype == torch.float32 else "_bf16"
    d = {k: (v.to(dev, dtype) if isinstance(v, torch.Tensor) else v) for k, v in case.items()}
    s = _shape(case)
    size_fn = getattr(lib, f"dcn_forward{tag}_workspace_size")
    size_fn.restype = ctypes.c_size_t
    size_fn.argtypes = [ctypes.POINTER(_native.DcnShape), ctypes.c_uint32]
    nbytes = size_fn(ctypes.byref(s), flags) - (1 if short else 0)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    out = torch.full(case["go"].shape, float("nan"), device=dev, dtype=dtype)
    fn = getattr(lib, f"dcn_forward{tag}")
    fn.argtypes = [ctypes.POINTER(_native.DcnShape)] + [ctypes.c_void_p] * 6 + \
        [ctypes.c_uint32, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]
    fn.restype = ctypes.c_int
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    _native.profiler_read()
    _native.profiler_enable(True)
    try:
        rc = fn(ctypes.byref(s), _p(d["x"]), _p(d["w"]), _p(d["off"]), _p(d["m"]), _p(d["b"]),
                _p(out), flags, _p(ws), nbytes, stream)
        torch.cuda.synchronize()
    finally:
        _native.profiler_enable(False)
    assert rc == 0, _native.capi_error()
    stats = _native.profiler_read()
    assert any(k.startswith("fwd_tc") for k in stats), sorted(stats)
    return out.float().cpu().numpy()


# name -> (case, flags, dtype).  188 tiles of 128 pixels on 148 SMs: one whole
# round, then 40 tiles of 9 K steps cut over 148 CTAs (3-4 pieces a tile); the
# small cases have fewer tiles than SMs, so every tile is cut.
CASES = {
    "tf32-whole-round-plus-split": (dict(N=1, inC=32, outC=32, H=155, W=155, offset_scale=3.0),
                                    MATH_TF32, torch.float32),
    "tf32-dg2-bias": (dict(N=2, inC=64, outC=64, dg=2, H=13, W=17, offset_scale=3.0),
                      MATH_TF32, torch.float32),
    "3xtf32-two-groups": (dict(N=1, inC=64, outC=64, groups=2, H=12, W=15, offset_scale=2.0),
                          MATH_3XTF32, torch.float32),
    "bf16-wide-512": (dict(N=1, inC=64, outC=512, H=11, W=13, offset_scale=2.0),
                      MATH_TF32, torch.bfloat16),
}


@pytest.mark.parametrize("name", sorted(CASES))
def test_split_round_repeatable_and_equal_to_whole_tiles(cuda_device, name):
    spec, flags, dt = CASES[name]
    case = make_case(**spec)
    a = _forward(case, cuda_device, flags, dtype=dt)
    b = _forward(case, cuda_device, flags, dtype=dt)
    assert np.array_equal(a, b)  # pieces are summed in a fixed order
    whole = _forward(case, cuda_device, flags, short=True, dtype=dt)
    scale = max(1.0, float(np.abs(whole).max()))
    tol = 1e-2 if dt == torch.bfloat16 else 1e-5
    np.testing.assert_allclose(a, whole, rtol=0, atol=tol * scale)


def test_split_round_matches_oracle(cuda_device):
    spec, flags, _ = CASES["tf32-whole-round-plus-split"]
    case = make_case(**spec)
    out = _forward(case, cuda_device, flags)
    ref, _ = run_oracle(case, backward=False)
    assert rel_norm_err(out, ref) <= 5e-3
    np.testing.assert_allclose(out, ref, rtol=0, atol=5e-3 * float(np.abs(ref).max()))
