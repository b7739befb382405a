"""Generate the golden vectors in this folder from the reference itself.

Run in a container that has the reference checkout (read-only) and
torchvision:

    python tests/golden/make_golden.py /path/to/pytorch_mps_deform_conv2d

It imports the reference package ``deform_conv2d_mps`` from ``<ref>/src`` and
runs its own public ``deform_conv2d`` on CPU tensors.  On CPU that function
routes to torchvision's kernel (``src/deform_conv2d_mps/ops.py:165-169``),
which is the reference's CPU implementation of the hot path.  Inputs are
seeded CPU tensors; forward output and all five gradients (for a random,
non-scalar upstream gradient) are saved per case as ``<case>.npz``.

The reference checkout is not needed afterwards: the tests read only the
``.npz`` files.
"""
from __future__ import annotations

import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))

# name -> geometry / distribution.  Each mirrors a case of the reference's
# own tests (tests/test_forward.py, tests/test_backward.py), its example
# (example/example01_deform_conv2d_cpu_mps.py:42-86) or a scaled-down member
# of a benchmarked shape family.
CASES = {
    # example01: N=2, C=4, outC=6, 10x12, k3, pad 1, offset*0.5, sigmoid
    # mask, seed 0 -> output mean -0.70549 on every recorded platform.
    "example01": dict(N=2, C=4, outC=6, H=10, W=12, k=(3, 3), pad=(1, 1),
                      offset_scale=0.5, mask="sigmoid", bias=True,
                      order="example01"),
    # The README usage case: x randn(2,4,16,16), w randn(6,4,3,3), no bias,
    # offset std 1, mask uniform[0,1).
    "readme_tiny": dict(N=2, C=4, outC=6, H=16, W=16, k=(3, 3), pad=(0, 0),
                        offset_scale=1.0, mask="rand", bias=False),
    "matrix_k3_s1_p1_d1_v2": dict(N=2, C=4, outC=6, H=9, W=9, k=(3, 3),
                                  pad=(1, 1), mask="rand", bias=True),
    "matrix_k1_s2_p0_d2_v1": dict(N=2, C=4, outC=6, H=9, W=9, k=(1, 1),
                                  stride=(2, 2), dil=(2, 2), mask=None,
                                  bias=True),
    "asym_everything": dict(N=2, C=4, outC=6, H=8, W=11, k=(1, 3),
                            stride=(2, 1), pad=(0, 2), dil=(2, 1),
                            mask="rand", bias=True),
    "boundary_stress_v1": dict(N=2, C=4, outC=6, H=9, W=9, k=(3, 3),
                               pad=(1, 1), offset_scale=8.0, mask=None,
                               bias=True),
    "dg2_cpg3": dict(N=2, C=6, outC=6, H=9, W=9, k=(3, 3), pad=(1, 1), dg=2,
                     mask="rand", bias=True),
    "g2_dg2": dict(N=2, C=4, outC=6, H=9, W=9, k=(3, 3), pad=(1, 1),
                   groups=2, dg=2, mask="rand", bias=True),
    "depthwise_g6": dict(N=2, C=6, outC=6, H=9, W=9, k=(3, 3), pad=(1, 1),
                         groups=6, mask="rand", bias=True),
    "n1_odd_nobias": dict(N=1, C=3, outC=5, H=9, W=9, k=(3, 3), pad=(1, 1),
                          mask="rand", bias=False),
    # Scaled-down members of the benchmarked shape families (channel counts
    # that take the tiled GEMM paths, offsets/masks drawn like the benchmark
    # workloads).
    "train_step_small": dict(N=2, C=32, outC=32, H=20, W=24, k=(3, 3),
                             pad=(1, 1), offset_scale=2.0, mask="sigmoid",
                             bias=True, weight="kaiming"),
    "grouped_small": dict(N=2, C=64, outC=64, H=12, W=12, k=(3, 3),
                          pad=(1, 1), groups=32, dg=4, offset_scale=2.0,
                          mask="sigmoid", bias=True, weight="kaiming"),
    "neck_small": dict(N=1, C=64, outC=64, H=13, W=19, k=(3, 3), pad=(1, 1),
                       offset_scale=4.0, mask="sigmoid", bias=True,
                       weight="kaiming"),
    "dcnv1_sweep_small": dict(N=2, C=64, outC=64, H=12, W=12, k=(3, 3),
                              stride=(2, 1), pad=(2, 1), dil=(2, 1), dg=8,
                              offset_scale=3.0, mask=None, bias=False,
                              weight="kaiming"),
}


def _make(case):
    N, C, outC, H, W = case["N"], case["C"], case["outC"], case["H"], case["W"]
    kh, kw = case["k"]
    sh, sw = case.get("stride", (1, 1))
    ph, pw = case.get("pad", (0, 0))
    dh, dw = case.get("dil", (1, 1))
    g = case.get("groups", 1)
    dg = case.get("dg", 1)
    Ho = (H + 2 * ph - dh * (kh - 1) - 1) // sh + 1
    Wo = (W + 2 * pw - dw * (kw - 1) - 1) // sw + 1
    osc = case.get("offset_scale", 1.0)
    torch.manual_seed(0)
    if case.get("order") == "example01":
        # example01_deform_conv2d_cpu_mps.py:77-86 draw order
        x = torch.randn(N, C, H, W)
        w = torch.randn(outC, C // g, kh, kw)
        b = torch.randn(outC)
        off = torch.randn(N, 2 * dg * kh * kw, Ho, Wo) * osc
        m = torch.sigmoid(torch.randn(N, dg * kh * kw, Ho, Wo))
    else:
        x = torch.randn(N, C, H, W)
        if case.get("weight") == "kaiming":
            w = torch.empty(outC, C // g, kh, kw)
            torch.nn.init.kaiming_uniform_(w, a=5 ** 0.5)
        else:
            w = torch.randn(outC, C // g, kh, kw)
        b = torch.randn(outC) if case["bias"] else None
        off = osc * torch.randn(N, 2 * dg * kh * kw, Ho, Wo)
        if case["mask"] == "rand":
            m = torch.rand(N, dg * kh * kw, Ho, Wo)
        elif case["mask"] == "sigmoid":
            m = torch.sigmoid(torch.randn(N, dg * kh * kw, Ho, Wo))
        else:
            m = None
    go = torch.randn(N, outC, Ho, Wo)
    return x, w, b, off, m, go, (sh, sw), (ph, pw), (dh, dw)


def main(ref_root: str) -> None:
    sys.path.insert(0, os.path.join(ref_root, "src"))
    from deform_conv2d_mps import deform_conv2d as ref_deform_conv2d

    index = {}
    for name, case in CASES.items():
        x, w, b, off, m, go, s, p, d = _make(case)
        leaves = [t.clone().requires_grad_(True) if t is not None else None
                  for t in (x, w, b, off, m)]
        xr, wr, br, offr, mr = leaves
        out = ref_deform_conv2d(xr, offr, wr, bias=br, stride=s, padding=p,
                                dilation=d, mask=mr)
        out.backward(go)
        arrays = dict(x=x.numpy(), weight=w.numpy(), offset=off.numpy(),
                      grad_out=go.numpy(), out=out.detach().numpy(),
                      grad_x=xr.grad.numpy(), grad_offset=offr.grad.numpy(),
                      grad_weight=wr.grad.numpy(),
                      stride=np.array(s), padding=np.array(p),
                      dilation=np.array(d))
        if b is not None:
            arrays.update(bias=b.numpy(), grad_bias=br.grad.numpy())
        if m is not None:
            arrays.update(mask=m.numpy(), grad_mask=mr.grad.numpy())
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **arrays)
        index[name] = dict(out_mean=float(out.detach().mean()),
                           out_shape=list(out.shape))
        print(f"{name:24s} out {tuple(out.shape)} mean {index[name]['out_mean']:+.5f}")
    with open(os.path.join(HERE, "index.json"), "w") as f:
        json.dump(dict(generator="reference deform_conv2d_mps CPU route "
                                 "(torchvision " + __import__("torchvision").__version__
                                 + ", torch " + torch.__version__ + ")",
                       cases=index), f, indent=1, sort_keys=True)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <reference checkout>")
    main(sys.argv[1])
