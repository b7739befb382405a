"""Stream order of a training step: steps queued back to back with no host
synchronization -- each backward (its prologue, then the fused tensor-core
kernel) right behind its forward, in the caller's stream, with the
library's side-stream forks and joins -- give the results of steps run one
call at a time with a synchronize around every call: TF32 and bf16
tensors, an input below and one above the side-stream threshold.  Any
change that lets a kernel start before the one ahead of it has finished
(programmatic dependent launch, more side streams) has to keep this."""
import pytest
import torch

import pytorch_mps_deform_conv2d_b200 as dcn
from pytorch_mps_deform_conv2d_b200 import _native

pytestmark = pytest.mark.gpu


def _inputs(dtype, C, H, W):
    g = torch.Generator().manual_seed(3)
    x = torch.randn(2, C, H, W, generator=g)
    off = 3 * torch.randn(2, 18, H, W, generator=g)
    m = torch.sigmoid(torch.randn(2, 9, H, W, generator=g))
    w = torch.randn(C, C, 3, 3, generator=g) / (3 * C ** 0.5)
    b = torch.randn(C, generator=g)
    gos = [torch.randn(2, C, H, W, generator=g) for _ in range(2)]
    leaves = [t.to("cuda", dtype).requires_grad_() for t in (x, off, m, w, b)]
    return leaves, [t.to("cuda", dtype) for t in gos]


def _step(leaves, go):
    x, off, m, w, b = leaves
    out = dcn.deform_conv2d(x, off, w, b, padding=1, mask=m)
    return [out.detach()] + list(torch.autograd.grad(out, leaves, go))


@pytest.mark.parametrize("dtype,C,H,W", [(torch.float32, 128, 40, 48),
                                         (torch.float32, 256, 90, 100),  # 18 MB: side streams
                                         (torch.bfloat16, 128, 40, 48)])
def test_queued_steps_match_synchronized_steps(cuda_device, dtype, C, H, W):
    leaves, gos = _inputs(dtype, C, H, W)
    dcn.set_math_mode("tf32")
    try:
        _native.profiler_read()
        _native.profiler_enable(True)
        try:
            _step(leaves, gos[0])
        finally:
            _native.profiler_enable(False)
        stats = _native.profiler_read()
        fused = [k for k in stats if k.startswith("bwd_fused_tc")]
        assert fused and any(k.startswith("bwd_prologue") for k in stats), sorted(stats)

        want = []
        for go in gos:  # one call at a time
            torch.cuda.synchronize()
            x, off, m, w, b = leaves
            out = dcn.deform_conv2d(x, off, w, b, padding=1, mask=m)
            torch.cuda.synchronize()
            grads = torch.autograd.grad(out, leaves, go)
            torch.cuda.synchronize()
            want.append([out.detach()] + list(grads))

        got = [_step(leaves, gos[i % 2]) for i in range(8)]  # queued, no synchronize
        torch.cuda.synchronize()
        for i, res in enumerate(got):
            for a, e in zip(res, want[i % 2]):
                a, e = a.float(), e.float()
                # the grad-input reductions sum in another order run to run
                tol = 1e-5 if dtype == torch.float32 else 1e-2
                torch.testing.assert_close(a, e, rtol=tol,
                                           atol=tol * max(1.0, float(e.abs().max())))
    finally:
        dcn.set_math_mode(None)
