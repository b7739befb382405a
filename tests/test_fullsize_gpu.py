"""Full benchmark sizes, checked through properties that do not need the CPU
oracle (too slow at these sizes):
  * zero offsets and a mask of ones make the op a regular convolution: the
    forward, grad_input and grad_weight equal cuDNN's conv2d (fp32, TF32
    off) on the same tensors -- every tap's sampling then sits exactly on the
    grid, so this covers the whole gather / scatter / GEMM machinery;
  * batch independence: image n alone gives slice n of the batched result,
    gradients included;
  * grad_bias is the sum of grad_out;
  * the math modes agree on the real (random-offset) workload: 3xTF32 with
    fp32 FFMA to 1e-4, TF32 with fp32 to the TF32 tolerance (5e-3 outputs,
    1e-3 gradients, norm-wise)."""
import pytest
import torch
import torch.nn.functional as F

from _util import rel_norm_err
from pytorch_mps_deform_conv2d_b200.ops import MATH_3XTF32, MATH_FP32, MATH_TF32, deform_conv2d_ex

pytestmark = pytest.mark.gpu

# the benchmark configurations (N, C, outC, H, W, stride, pad, dil, groups, dg, mask, bias)
CONFIGS = {
    "training-8x64x64x64": dict(N=8, C=64, O=64, H=64, W=64, s=(1, 1), p=(1, 1), d=(1, 1), g=1,
                                dg=1, mask=True, bias=True, osc=2.0),
    "grouped-g32-dg4": dict(N=8, C=64, O=64, H=64, W=64, s=(1, 1), p=(1, 1), d=(1, 1), g=32,
                            dg=4, mask=True, bias=True, osc=2.0),
    "neck-2x256x100x152": dict(N=2, C=256, O=256, H=100, W=152, s=(1, 1), p=(1, 1), d=(1, 1),
                               g=1, dg=1, mask=True, bias=True, osc=4.0),
    "dcnv1-64x512x28x28": dict(N=64, C=512, O=512, H=28, W=28, s=(2, 1), p=(2, 1), d=(2, 1), g=1,
                               dg=8, mask=False, bias=False, osc=3.0),
}


def _out_hw(c):
    ho = (c["H"] + 2 * c["p"][0] - c["d"][0] * 2 - 1) // c["s"][0] + 1
    wo = (c["W"] + 2 * c["p"][1] - c["d"][1] * 2 - 1) // c["s"][1] + 1
    return ho, wo


def _tensors(c, zero_offsets, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    ho, wo = _out_hw(c)
    x = torch.randn(c["N"], c["C"], c["H"], c["W"], device="cuda", generator=g)
    w = torch.randn(c["O"], c["C"] // c["g"], 3, 3, device="cuda", generator=g) * (
        1.0 / (c["C"] // c["g"] * 9) ** 0.5)
    b = torch.randn(c["O"], device="cuda", generator=g) if c["bias"] else None
    if zero_offsets:
        off = torch.zeros(c["N"], 2 * c["dg"] * 9, ho, wo, device="cuda")
        m = torch.ones(c["N"], c["dg"] * 9, ho, wo, device="cuda") if c["mask"] else None
    else:
        off = c["osc"] * torch.randn(c["N"], 2 * c["dg"] * 9, ho, wo, device="cuda", generator=g)
        m = (torch.sigmoid(torch.randn(c["N"], c["dg"] * 9, ho, wo, device="cuda", generator=g))
             if c["mask"] else None)
    go = torch.randn(c["N"], c["O"], ho, wo, device="cuda", generator=g)
    return x, w, b, off, m, go


def _fwd_bwd(c, x, w, b, off, m, go, flags):
    leaves = [t.clone().requires_grad_() if t is not None else None for t in (x, w, b, off, m)]
    xl, wl, bl, ol, ml = leaves
    out = deform_conv2d_ex(xl, ol, wl, bl, c["s"], c["p"], c["d"], ml, flags=flags)
    out.backward(go)
    return out.detach(), [t.grad if t is not None else None for t in leaves]


def _close(got, want, tol):
    return rel_norm_err(got.double().cpu().numpy(), want.double().cpu().numpy()) <= tol


# fp32 FFMA to 1e-5; 3xTF32 (the low x low product dropped) to the reference's
# fp32 tolerance 1e-4; TF32 to 2e-3
@pytest.mark.parametrize("flags,tol", [(MATH_FP32, 1e-5), (MATH_3XTF32, 1e-4),
                                       (MATH_TF32, 2e-3)], ids=["fp32", "3xtf32", "tf32"])
@pytest.mark.parametrize("name", sorted(CONFIGS))
def test_zero_offsets_equal_cudnn_conv(cuda_device, name, flags, tol):
    c = CONFIGS[name]
    x, w, b, off, m, go = _tensors(c, zero_offsets=True)
    out, (gx, gw, gb, _, _) = _fwd_bwd(c, x, w, b, off, m, go, flags)
    prev = torch.backends.cudnn.allow_tf32
    torch.backends.cudnn.allow_tf32 = False
    try:
        xr, wr = x.clone().requires_grad_(), w.clone().requires_grad_()
        ref = F.conv2d(xr, wr, b, c["s"], c["p"], c["d"], c["g"])
        ref.backward(go)
    finally:
        torch.backends.cudnn.allow_tf32 = prev
    assert _close(out, ref.detach(), tol)
    assert _close(gx, xr.grad, tol)
    assert _close(gw, wr.grad, tol)
    if b is not None:
        assert _close(gb, go.sum((0, 2, 3)), 1e-6)


@pytest.mark.parametrize("name", sorted(CONFIGS))
def test_batch_independence(cuda_device, name):
    c = CONFIGS[name]
    x, w, b, off, m, go = _tensors(c, zero_offsets=False, seed=1)
    out, grads = _fwd_bwd(c, x, w, b, off, m, go, MATH_TF32)
    n = c["N"] - 1
    sl = lambda t: None if t is None else t[n:n + 1].contiguous()
    out1, grads1 = _fwd_bwd(c, sl(x), w, b, sl(off), sl(m), sl(go), MATH_TF32)
    torch.testing.assert_close(out1, out[n:n + 1], rtol=1e-5, atol=1e-5)
    for k in (0, 3, 4):  # per-image gradients: input, offset, mask
        if grads[k] is not None:
            torch.testing.assert_close(grads1[k], grads[k][n:n + 1], rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("name", sorted(CONFIGS))
def test_math_modes_agree_on_the_workload(cuda_device, name):
    c = CONFIGS[name]
    x, w, b, off, m, go = _tensors(c, zero_offsets=False, seed=2)
    ref_out, ref_g = _fwd_bwd(c, x, w, b, off, m, go, MATH_FP32)
    for flags, out_tol, grad_tol in ((MATH_3XTF32, 1e-4, 1e-4), (MATH_TF32, 5e-3, 1e-3)):
        out, grads = _fwd_bwd(c, x, w, b, off, m, go, flags)
        assert _close(out, ref_out, out_tol), flags
        for k, (gt, gr) in enumerate(zip(grads, ref_g)):
            if gr is not None:
                assert _close(gt, gr, grad_tol), (flags, k)
