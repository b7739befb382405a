"""CUDA graph capture of a whole forward + backward through the public
module: the library's launches, side-stream forks/joins and workspace
allocations are capturable, and replays with new input values match eager
execution (tensor-core path with and without side streams -- the library
uses them for inputs of 16 MB and more --, and the fp32 kernels)."""
import pytest
import torch

import pytorch_mps_deform_conv2d_b200 as dcn

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("mode,channels,H,W", [("tf32", 128, 10, 11), ("fp32", 8, 10, 11),
                                                ("3xtf32", 64, 10, 11),
                                                ("tf32", 256, 90, 100)])  # 18 MB: side streams
def test_graph_capture_matches_eager(cuda_device, mode, channels, H, W):
    torch.manual_seed(0)
    mod = dcn.DeformConv2d(channels, channels, 3, padding=1).cuda()
    shape = (2, channels, H, W)
    x = torch.randn(shape, device="cuda", requires_grad=True)
    off = (2 * torch.randn(2, 18, H, W, device="cuda")).requires_grad_()
    m = torch.rand(2, 9, H, W, device="cuda", requires_grad=True)
    go = torch.randn(2, channels, H, W, device="cuda")
    leaves = [x, off, m, mod.weight, mod.bias]

    def step():
        for t in leaves:
            t.grad = None
        out = mod(x, off, m)
        out.backward(go)
        return out

    dcn.set_math_mode(mode)
    try:
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):  # warm-up outside the capture
            for _ in range(3):
                step()
        torch.cuda.current_stream().wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        for t in leaves:
            t.grad = None
        with torch.cuda.graph(graph):
            out_static = step()
        grads_static = [t.grad for t in leaves]
        for rep in range(2):
            with torch.no_grad():  # new values in the captured input buffers
                x.copy_(torch.randn(shape, device="cuda"))
                off.copy_(2 * torch.randn(2, 18, H, W, device="cuda"))
                go.copy_(torch.randn_like(go))
            graph.replay()
            torch.cuda.synchronize()
            got = [out_static.detach().clone()] + [g.clone() for g in grads_static]
            want_out = step().detach()
            want = [want_out] + [t.grad.clone() for t in leaves]
            for a, b in zip(got, want):
                # atomics sum in another order run to run: scale to the values
                torch.testing.assert_close(a, b, rtol=1e-5,
                                           atol=1e-5 * max(1.0, float(b.abs().max())))
    finally:
        dcn.set_math_mode(None)
