#!/usr/bin/env python
"""Benchmark: DCNv2 forward + backward on the detection-neck workload.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--math tf32|fp32|3xtf32] [--workload neck|train|grouped|dcnv1]

One step is one training pass of the deformable convolution over one batch:
forward, backward with a fixed upstream gradient, and (N > 1) the NCCL
all-reduce of grad_weight / grad_bias.  Each rank holds its own full batch
(weak scaling, data parallel), so `value` -- milliseconds per iteration of
the 2x256x100x152 workload for the whole job -- is the per-step time (max
over ranks) divided by the number of batches all ranks processed.

Inputs are synthetic, seeded CPU tensors with the workload's shapes and
distributions (x randn, weight kaiming_uniform(a=sqrt 5), bias randn, offset
N(0, 4^2), mask sigmoid(randn), grad_out randn), copied to the device before
timing.  L2 is flushed (a 256 MiB write) between timed iterations, outside
the timed events.

The printed JSON line carries the roofline of the dominant kernel (timed live
with the library's CUDA-event profiler), the CPU baseline (the reference
package's own CPU route -- torchvision's kernel -- on the whole workload: two
timed steps, all host threads), end-to-end numbers through the public module
API with host<->device copies inside the timed region (parameter gradients
read back, and the output with all five gradients read back), and the step
time of the other math modes.

`--impl reference` times the reference's CPU implementation alone on the
whole workload (rank 0): W untimed steps, then K timed ones.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

METRIC = ("DCNv2 fwd+bwd ms/iter (2×256×100×152) and % roofline at 1/2/4/8 "
          "B200 vs host CPU")

WORKLOADS = {
    "neck": dict(desc="detection-neck DCNv2 fwd+bwd: x 2x256x100x152, weight 256x256x3x3, "
                      "bias, stride 1, pad 1, dil 1, dg 1, offset N(0,4^2), mask sigmoid(randn)",
                 N=2, C=256, outC=256, H=100, W=152, k=3, stride=(1, 1), pad=(1, 1),
                 dil=(1, 1), groups=1, dg=1, offset_std=4.0, mask=True, bias=True),
    "train": dict(desc="DCNv2 training step: x 8x64x64x64, weight 64x64x3x3, bias, pad 1, "
                       "offset N(0,2^2), mask sigmoid(randn)",
                  N=8, C=64, outC=64, H=64, W=64, k=3, stride=(1, 1), pad=(1, 1), dil=(1, 1),
                  groups=1, dg=1, offset_std=2.0, mask=True, bias=True),
    "grouped": dict(desc="grouped DCNv2: x 8x64x64x64, weight 64x2x3x3 (groups 32), dg 4, pad 1, "
                         "offset N(0,2^2), mask sigmoid(randn), bias",
                    N=8, C=64, outC=64, H=64, W=64, k=3, stride=(1, 1), pad=(1, 1), dil=(1, 1),
                    groups=32, dg=4, offset_std=2.0, mask=True, bias=True),
    "dcnv1": dict(desc="DCNv1 sweep: x 64x512x28x28, weight 512x512x3x3, no bias, stride (2,1), "
                       "pad (2,1), dil (2,1), dg 8, offset N(0,3^2), no mask",
                  N=64, C=512, outC=512, H=28, W=28, k=3, stride=(2, 1), pad=(2, 1), dil=(2, 1),
                  groups=1, dg=8, offset_std=3.0, mask=False, bias=False),
}

FLUSH_BYTES = 256 << 20


def out_hw(wl):
    k = wl["k"]
    ho = (wl["H"] + 2 * wl["pad"][0] - wl["dil"][0] * (k - 1) - 1) // wl["stride"][0] + 1
    wo = (wl["W"] + 2 * wl["pad"][1] - wl["dil"][1] * (k - 1) - 1) // wl["stride"][1] + 1
    return ho, wo


def make_inputs(wl, seed=0, n=None, c_in=None):
    """Seeded CPU tensors in the order x, weight, bias, offset, mask, grad_out.
    `n` / `c_in` cut a sample: the first n images / first c_in input channels."""
    import torch
    torch.manual_seed(seed)
    N, C, O, H, W, k = wl["N"], wl["C"], wl["outC"], wl["H"], wl["W"], wl["k"]
    g, dg = wl["groups"], wl["dg"]
    ho, wo = out_hw(wl)
    x = torch.randn(N, C, H, W)
    w = torch.empty(O, C // g, k, k)
    torch.nn.init.kaiming_uniform_(w, a=math.sqrt(5))
    b = torch.randn(O) if wl["bias"] else None
    off = wl["offset_std"] * torch.randn(N, 2 * dg * k * k, ho, wo)
    m = torch.sigmoid(torch.randn(N, dg * k * k, ho, wo)) if wl["mask"] else None
    go = torch.randn(N, O, ho, wo)
    if n is not None:
        x, off, go = x[:n], off[:n], go[:n]
        m = m[:n] if m is not None else None
    if c_in is not None:
        assert g == 1
        x, w = x[:, :c_in].contiguous(), w[:, :c_in].contiguous()
    return x, w, b, off, m, go


def bench_config(wl, args=None):
    """The workload the metric is quoted on, the same for both arms: one
    iteration is forward + backward of this batch (how a run spreads its
    iterations over devices is under the line's "run" key)."""
    return {"workload": wl["desc"], "global_batch": wl["N"],
            "io_dtype": getattr(args, "dtype", "fp32"),
            "input_layout": getattr(args, "layout", "nchw")}


def algorithmic_work(wl):
    """FLOPs and compulsory HBM bytes of one fwd+bwd iteration."""
    N, C, O, k, g, dg = wl["N"], wl["C"], wl["outC"], wl["k"], wl["groups"], wl["dg"]
    ho, wo = out_hw(wl)
    P = ho * wo
    gemm = 2.0 * O * (C // g) * k * k * N * P
    x = N * C * wl["H"] * wl["W"]
    off = N * 2 * dg * k * k * P
    msk = N * dg * k * k * P if wl["mask"] else 0
    wts = O * (C // g) * k * k
    bia = O if wl["bias"] else 0
    out = N * O * P
    fwd = x + off + msk + wts + bia + out
    bwd = (out + x + off + msk + wts) + (x + off + msk + wts + bia)
    return dict(flops=3 * gemm, gemm_flops=gemm, bytes=4.0 * (fwd + bwd), P=P)


# tcgen05 kernels (TF32 operands; 3xTF32 issues three products per multiply-add)
TC_KERNELS = ("fwd_tc", "bwd_fused_tc", "bwd_data_tc", "bwd_weight_tc", "bwd_weight_col",
              "fwd_tc_bf16", "fwd_tc_f16", "bwd_fused_tc_bf16", "bwd_fused_tc_f16")
# kind::f16 with 16-bit operands
BF16_KERNELS = ("fwd_tc_bf16", "fwd_tc_f16", "bwd_fused_tc_bf16", "bwd_fused_tc_f16")
HALF = {"bf16": "bfloat16", "fp16": "float16"}


def kernel_work(name, wl):
    """(amount, unit, bound) of one launch of a library kernel."""
    w = algorithmic_work(wl)
    N, C = wl["N"], wl["C"]
    # (the helpers first: "fwd_prologue" shares the tensor-core kernels' prefix)
    if name in ("fwd_prologue", "bwd_finish"):  # a transpose + the weight read and rewritten
        wts = wl["outC"] * (C // wl["groups"]) * wl["k"] ** 2
        return 2.0 * 4 * (N * C * wl["H"] * wl["W"] + wts), "byte", "hbm"
    if name.startswith("bwd_fused_tc"):  # both backward GEMMs
        return 2.0 * w["gemm_flops"], "flop", "tensor"
    if name.startswith(("fwd_", "bwd_data", "bwd_weight")):
        return w["gemm_flops"], "flop", "tensor"
    if name in ("nchw_to_nhwc", "nhwc_to_nchw", "copy_nhwc"):
        return 2.0 * 4 * N * C * wl["H"] * wl["W"], "byte", "hbm"
    if name == "bwd_prologue":  # grad_out in + rows out, zeroed accumulators, packed weight
        ho, wo = out_hw(wl)
        O, k2, dg = wl["outC"], wl["k"] ** 2, wl["dg"]
        wts = O * (C // wl["groups"]) * k2
        zeroed = N * C * wl["H"] * wl["W"] + N * 3 * dg * k2 * ho * wo + wts
        return 4.0 * (2 * N * O * ho * wo + zeroed + 2 * wts), "byte", "hbm"
    if name == "grad_bias":
        return 4.0 * N * wl["outC"] * w["P"], "byte", "hbm"
    return None, None, None


# ---------------------------------------------------------------------------
# peaks
# ---------------------------------------------------------------------------
def measured_peaks_file():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            return json.load(f), "MEASURED_PEAKS.json"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}, "fallback"


def measure_matmul_tflops(dtype_mode, n=8192, reps=5):
    """cuBLAS burst throughput, best of `reps` (torch.matmul n^3, 2 n^3 flop)."""
    import torch
    prev = torch.backends.cuda.matmul.allow_tf32
    dt = torch.bfloat16 if dtype_mode == "bf16" else torch.float32
    torch.backends.cuda.matmul.allow_tf32 = dtype_mode == "tf32"
    try:
        a = torch.randn(n, n, device="cuda", dtype=dt)
        b = torch.randn(n, n, device="cuda", dtype=dt)
        for _ in range(2):
            torch.matmul(a, b)
        best = float("inf")
        for _ in range(reps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            torch.matmul(a, b)
            e1.record()
            torch.cuda.synchronize()
            best = min(best, e0.elapsed_time(e1))
        del a, b
        return 2.0 * n ** 3 / (best * 1e-3) / 1e12
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


def measure_l2_gbs(bytes_=64 << 20, passes=16, reps=5):
    """L2 <-> SM bandwidth of this GPU, best of `reps`: the library's probe
    (dcn_l2_probe) sweeping an L2-resident buffer with 16-byte loads cached
    in L2 only (kind 0, the corner gathers), with 16-byte fp32 reductions
    (kind 1, the col2im scatter), and with both in one loop, 5 loads to 2
    reductions (kind 2), and with 16-byte loads from random 128-byte lines
    (kind 3, the corner gathers' pattern) and 16-byte reductions into random
    lines (kind 4, the col2im scatter's pattern).  Returns {"l2_to_sm",
    "sm_to_l2_red", "mixed_5to2", "gather", "scatter_red"} in GB/s (kind 2:
    bytes read plus bytes reduced)."""
    import ctypes

    import torch
    from pytorch_mps_deform_conv2d_b200 import _native
    lib = _native.load_capi()
    buf = torch.zeros(bytes_ // 4, device="cuda")
    stream = torch.cuda.current_stream()
    out = {}
    warps = torch.cuda.get_device_properties(buf.device).multi_processor_count * 64
    for kind, name in ((0, "l2_to_sm"), (1, "sm_to_l2_red"), (2, "mixed_5to2"),
                       (3, "gather"), (4, "scatter_red")):
        def launch():
            rc = lib.dcn_l2_probe(kind, ctypes.c_void_p(buf.data_ptr()), bytes_, passes,
                                  ctypes.c_void_p(stream.cuda_stream))
            if rc != 0:
                raise RuntimeError(f"dcn_l2_probe({kind}) failed: {rc}")
        for _ in range(2):
            launch()
        best = float("inf")
        for _ in range(reps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            launch()
            e1.record()
            torch.cuda.synchronize()
            best = min(best, e0.elapsed_time(e1))
        moved = (bytes_ if kind < 2 else (bytes_ // 3584) * 3584 if kind == 2
                 else 512 * (bytes_ // 512 // warps // 4 * 4) * warps)
        out[name] = round(moved * passes / (best * 1e-3) / 1e9, 1)
    del buf
    return out


def gather_bytes(name, wl):
    """Corner-gather bytes of one launch of a tensor-core kernel that gathers
    (every sample reads 4 corner vectors of all its channels; dropped
    corners read the zero row): 4 x C x element size x taps x N x P."""
    if not name.startswith(("fwd_tc", "bwd_fused_tc")):
        return 0.0
    esize = 2 if name.endswith(("_bf16", "_f16")) else 4
    return 4.0 * wl["C"] * esize * wl["k"] ** 2 * wl["N"] * algorithmic_work(wl)["P"]


def binding_roofline(traffic, avg_ms, l2_peaks, gathered=0.0):
    """The dominant kernel against the L2 <-> SM crossbar.  Bytes it moved
    each way in one launch (ncu: l1tex__m_xbar2l1tex_read_bytes.sum and
    l1tex__m_l1tex2xbar_write_bytes.sum, from the committed profile of the
    same workload and mode), split into corner gathers (`gathered`, random
    128-byte lines) and streaming loads (the rest: TMA tiles, offsets).
    Floor model from the probes of this run: loads take gathers / gather
    rate + the rest / load rate, reductions take their bytes / scatter rate
    (16-byte reductions into random lines); the two directions overlap by the fraction `overlap` that the mixed
    probe (5:2 loads to reductions) shows between running them one after the
    other and fully side by side.  `frac` = floor / launch time."""
    if not traffic or "l2_to_sm_bytes" not in traffic or not l2_peaks:
        return None
    rd, wr = float(traffic["l2_to_sm_bytes"]), float(traffic.get("sm_to_l2_bytes", 0.0))
    gat = min(gathered, rd)
    t = avg_ms * 1e-3
    P_ld, P_red = l2_peaks["l2_to_sm"] * 1e9, l2_peaks["sm_to_l2_red"] * 1e9
    P_gat, P_mix = l2_peaks["gather"] * 1e9, l2_peaks["mixed_5to2"] * 1e9
    P_sct = l2_peaks.get("scatter_red", l2_peaks["sm_to_l2_red"]) * 1e9
    # overlap of the probe's own mix: 5 bytes loaded, 2 reduced
    ser, par, mix = 5 / P_ld + 2 / P_red, max(5 / P_ld, 2 / P_red), 7 / P_mix
    overlap = min(1.0, max(0.0, (ser - mix) / (ser - par)))
    t_ld = gat / P_gat + (rd - gat) / P_ld
    # the kernels' reductions land on lines that follow the sampling offsets
    t_red = wr / P_sct
    floor = t_ld + t_red - overlap * min(t_ld, t_red)
    return {"resource": "L2 <-> SM crossbar (gathers, tiles, fp32 reductions)",
            "unit": "GB/s", "l2_to_sm_bytes": rd, "gather_bytes": gat, "sm_to_l2_bytes": wr,
            "achieved": round((rd + wr) / t / 1e9, 1),
            "floor_ms": round(floor * 1e3, 4), "loads_ms": round(t_ld * 1e3, 4),
            "reductions_ms": round(t_red * 1e3, 4), "overlap": round(overlap, 3),
            "frac": round(floor / t, 3),
            "peaks_gbs": {k: l2_peaks.get(k) for k in ("l2_to_sm", "gather", "sm_to_l2_red",
                                                        "scatter_red", "mixed_5to2")},
            "peak_source": "dcn_l2_probe in this run (64 MiB L2-resident buffer, all SMs)",
            "bytes_source": traffic.get("source")}


# ---------------------------------------------------------------------------
# clocks
# ---------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [l for l in out.splitlines() if l.strip()]
        return False

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for name, val in zip(names, f[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------------------------
# CPU baseline: the reference's own CPU route on a bounded sample
# ---------------------------------------------------------------------------
def reference_cpu_op():
    """The reference package's public deform_conv2d (its CPU route calls
    torchvision's kernel, src/deform_conv2d_mps/ops.py:165-169); torchvision
    directly when the package is not installed under baseline/_ref."""
    ref_dir = os.path.join(ROOT, "baseline", "_ref")
    if os.path.isdir(os.path.join(ref_dir, "deform_conv2d_mps")):
        if ref_dir not in sys.path:
            sys.path.insert(0, ref_dir)
        from deform_conv2d_mps import deform_conv2d as ref_op
        return ref_op, "reference package deform_conv2d_mps 0.1.0 (CPU route -> torchvision)"
    from torchvision.ops import deform_conv2d as tv_op
    return tv_op, "torchvision.ops.deform_conv2d (the reference's CPU route)"


def cpu_sample_plan(wl):
    """A cut of the workload: one image and a slice of the input channels,
    1/scale of its work (every cost term of the op is linear in images x
    input channels).  Used only for the `sampled` cross-check figure."""
    n = 1
    c_in = wl["C"]
    if wl["groups"] == 1:
        while c_in > 32 and (wl["N"] // n) * (wl["C"] // c_in) < 16:
            c_in //= 2
    scale = (wl["N"] / n) * (wl["C"] / c_in)
    return n, c_in, scale


def cpu_reference_step_fn(wl, threads, sampled=False):
    """One fwd+bwd step of the reference's CPU route on the whole workload
    (or, with `sampled`, on the cut of cpu_sample_plan); returns the step,
    the factor from its time to a whole-workload time (1 unless sampled) and
    a description."""
    import torch
    torch.set_num_threads(threads)
    op, label = reference_cpu_op()
    n, c_in, scale = cpu_sample_plan(wl) if sampled else (None, None, 1.0)
    x, w, b, off, m, go = make_inputs(wl, n=n, c_in=c_in if c_in != wl["C"] else None)
    leaves = [t.clone().requires_grad_(True) if t is not None else None for t in (x, w, b, off, m)]

    def step():
        for t in leaves:
            if t is not None:
                t.grad = None
        xx, ww, bb, oo, mm = leaves
        out = op(xx, oo, ww, bias=bb, stride=wl["stride"], padding=wl["pad"],
                 dilation=wl["dil"], mask=mm)
        out.backward(go)

    if sampled:
        desc = (f"{n} of {wl['N']} images x {c_in} of {wl['C']} input channels of the workload "
                f"(1/{scale:g} of its work), fwd+bwd through {label}; x {scale:g}")
    else:
        desc = (f"the whole workload ({wl['N']} images, all five inputs requiring grad, a "
                f"fixed upstream gradient), fwd+bwd through {label}")
    return step, scale, desc


def time_cpu_steps(step, steps, warmup):
    for _ in range(warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(steps):
        step()
    return (time.perf_counter() - t0) / steps


def cpu_baseline(wl):
    """The reference's CPU route timed on the whole workload on this host:
    one untimed step, then two timed ones (about 25 s for the detection
    neck on 16 cores).  `sampled`: the same route on a 1/16 cut of the
    workload scaled back up, and its ratio to the measured figure (a check of
    the linear scaling older bench lines relied on)."""
    import torch
    threads = os.cpu_count() or 1
    step, _, desc = cpu_reference_step_fn(wl, threads)
    full_ms = time_cpu_steps(step, steps=2, warmup=1) * 1e3
    del step
    sstep, scale, sdesc = cpu_reference_step_fn(wl, threads, sampled=True)
    sample_ms = time_cpu_steps(sstep, steps=3, warmup=1) * 1e3 * scale
    return {"value": round(full_ms, 3), "unit": "ms/iter", "cores": torch.get_num_threads(),
            "kind": "reference", "sample": desc + "; 2 timed steps after 1 untimed, unscaled",
            "sampled": {"value": round(sample_ms, 3), "ratio_to_measured":
                        round(sample_ms / full_ms, 3), "sample": sdesc}}


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
def load_traffic():
    path = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(path):
        with open(path) as f:
            return json.load(f)
    return {}


def run_ours(args, wl):
    import torch
    import torch.distributed as dist
    import pytorch_mps_deform_conv2d_b200 as dcn
    from pytorch_mps_deform_conv2d_b200 import _native
    from pytorch_mps_deform_conv2d_b200.ops import _MODES, deform_conv2d_ex

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    flags = _MODES[args.math]

    strong = args.scaling == "strong"
    x, w, b, off, m, go = make_inputs(wl, seed=0 if strong else rank)
    row0, slabs, group = 0, 1, None
    if strong:
        # the one batch split over the ranks: images first, then row slabs
        from pytorch_mps_deform_conv2d_b200.distributed import (image_groups, image_slab,
                                                                 slab_rows)
        first, count, slab, slabs = image_slab(rank, world, wl["N"])
        groups = image_groups(world, wl["N"]) if world > 1 else []
        group = groups[first] if slabs > 1 else None
        rows = slab_rows(go.shape[2], slab, slabs)
        row0 = rows.start
        cut = lambda t: None if t is None else t[first:first + count, :, rows].contiguous()
        x = x[first:first + count].contiguous()
        off, m, go = cut(off), cut(m), cut(go)
    if args.dtype in HALF:  # 16-bit I/O: every tensor (and gradient) bf16 / fp16
        hdt = getattr(torch, HALF[args.dtype])
        x, w, b, off, m, go = (None if t is None else t.to(hdt)
                               for t in (x, w, b, off, m, go))
    if args.layout == "nhwc":  # channels-last input (and grad_input), same values
        x = x.contiguous(memory_format=torch.channels_last)
    xd, offd, md, god = (t.to(dev) if t is not None else None for t in (x, off, m, go))
    wd = w.to(dev).requires_grad_(True)
    bd = b.to(dev).requires_grad_(True) if b is not None else None
    xd.requires_grad_(True)
    offd.requires_grad_(True)
    if md is not None:
        md.requires_grad_(True)
    params = [p for p in (wd, bd) if p is not None]
    leaves = [t for t in (xd, offd, md, wd, bd) if t is not None]
    flush = torch.empty(FLUSH_BYTES // 4, device=dev)
    comm_stream = torch.cuda.current_stream(dev)

    from pytorch_mps_deform_conv2d_b200.distributed import allreduce_grads

    def allreduce(params_):
        if world > 1:
            allreduce_grads(params_)

    from pytorch_mps_deform_conv2d_b200.distributed import deform_conv2d_row_sharded

    def step_with_flags(fl):
        for t in leaves:
            t.grad = None
        if slabs > 1:  # this rank's output rows; grad_input summed over the image's ranks
            out = deform_conv2d_row_sharded(xd, offd, wd, bd, wl["stride"], wl["pad"],
                                            wl["dil"], md, row_begin=row0, group=group,
                                            flags=fl)
        else:
            out = deform_conv2d_ex(xd, offd, wd, bd, wl["stride"], wl["pad"], wl["dil"], md,
                                   flags=fl)
        out.backward(god)
        allreduce(params)

    def step():
        step_with_flags(flags)

    for _ in range(args.warmup):
        step()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()

    def timed_pass(profile):
        """K steps, L2 flushed before each (outside its events); the summed
        device time of the steps, the max over ranks.  With `profile`, the
        library's per-launch event pairs are on: its kernel table, at the cost
        of a gap at every recorded launch, so the headline pass runs without."""
        starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
        ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        _native.profiler_enable(profile)
        t0 = time.perf_counter()
        for i in range(args.steps):
            flush.zero_()
            starts[i].record()
            step()
            ends[i].record()
        torch.cuda.synchronize()
        wall_s = time.perf_counter() - t0
        _native.profiler_enable(False)
        if world > 1:
            dist.barrier()
        tot = sum(s.elapsed_time(e) for s, e in zip(starts, ends))
        if world > 1:
            t = torch.tensor([tot], device=dev, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            tot = float(t.item())
        return tot, wall_s

    _native.profiler_read()  # drop anything recorded before
    clocks = ClockSampler(local)
    with clocks:
        total_ms, wall = timed_pass(False)   # the headline
        prof_ms, _ = timed_pass(True)        # the kernel table
    kstats = _native.profiler_read()
    ms_per_step = total_ms / args.steps
    value = ms_per_step if strong else ms_per_step / world

    # ---- dominant kernel roofline ----
    kernels = {k: v for k, v in kstats.items() if k != "memset"}
    launches = sum(v[0] for v in kernels.values())
    # the dominant kernel among those with a work model (under a profiler the
    # small helpers can stretch past it)
    modelled = [k for k in kernels if kernel_work(k, wl)[0] is not None] or list(kernels)
    dom = max(modelled, key=lambda k: kernels[k][1])
    dom_launches, dom_ms = kernels[dom]
    avg_ms = dom_ms / dom_launches
    amount, unit, bound = kernel_work(dom, wl)
    if amount is None:
        amount, unit, bound = 0.0, "byte", "hbm"
    if strong:  # this rank's part of the batch: its images x its share of their rows
        amount *= xd.shape[0] / wl["N"] * god.shape[2] / out_hw(wl)[0]
    peaks, peaks_src = measured_peaks_file()
    if args.profile:
        peak_tf32 = 0.5 * peaks.get("bf16_tflops", 1590.0)
        peak_fp32 = peak_tf32 / 8.0
        l2_peaks = None
    else:
        peak_tf32 = measure_matmul_tflops("tf32")
        peak_fp32 = measure_matmul_tflops("fp32")
        l2_peaks = measure_l2_gbs()
    # TF32 denominator: the larger of this run's cuBLAS TF32 GEMM and half the
    # measured bf16 peak (TF32 runs at half the bf16 rate on these tensor cores)
    half_bf16 = 0.5 * float(peaks.get("bf16_tflops", 1590.0))
    peak_tf32_used = max(peak_tf32, half_bf16)
    roof = {"kernel": dom, "bound": bound, "share_of_step": round(dom_ms / prof_ms, 3)
            if world == 1 else None}
    if bound == "tensor":
        if dom in BF16_KERNELS:
            peak = float(peaks.get("bf16_tflops", 1590.0))
            src = f"{peaks_src} bf16_tflops (cuBLAS bf16 burst)"
        elif dom in TC_KERNELS:
            peak = peak_tf32_used
            src = (f"max(cuBLAS tf32 8192^3 burst in this run {peak_tf32:.1f}, half of "
                   f"{peaks_src} bf16_tflops {half_bf16:.1f}) TFLOP/s")
        else:
            peak = peak_fp32
            src = "cuBLAS fp32 (FFMA, no TF32) 8192^3 burst measured in this run"
        achieved = amount / (avg_ms * 1e-3) / 1e12
        roof.update(achieved=round(achieved, 2), peak=round(peak, 1), unit="TFLOP/s",
                    frac=round(achieved / peak, 3), peak_source=src,
                    flop_per_launch=amount)
    else:
        peak = peaks.get("hbm_gbs", 6650.0)
        achieved = amount / (avg_ms * 1e-3) / 1e9
        roof.update(achieved=round(achieved, 1), peak=peak, unit="GB/s",
                    frac=round(achieved / peak, 3), peak_source=f"{peaks_src} hbm_gbs",
                    bytes_per_launch=amount)
    traffic = load_traffic().get(f"{args.workload}:{args.math}:{dom}")
    roof["traffic"] = traffic["bytes_per_launch"] if traffic else None
    roof["binding"] = binding_roofline(traffic, avg_ms, l2_peaks, gather_bytes(dom, wl))
    work = algorithmic_work(wl)
    step_roof_ms = work["flops"] / ((peak_tf32_used if args.math != "fp32" else peak_fp32) * 1e12) * 1e3
    roof["step_roofline_ms"] = round(max(step_roof_ms, work["bytes"] / (peaks.get("hbm_gbs", 6650.0) * 1e9) * 1e3), 4)
    roof["step_frac"] = round(roof["step_roofline_ms"] / ms_per_step, 3)
    roof["peaks_measured_tflops"] = {"tf32": round(peak_tf32, 1), "fp32": round(peak_fp32, 1)}
    # the step against its binding resources: each kernel's crossbar floor
    # (committed profile + this run's probes) or, for the HBM-bound helpers,
    # its algorithmic bytes at the HBM peak; kernels without a model add 0
    if l2_peaks and world == 1:
        tr_all = load_traffic()
        floor_ms, parts = 0.0, {}
        for name, (n_launch, tot_ms) in kernels.items():
            tr = tr_all.get(f"{args.workload}:{args.math}:{name}")
            if tr is not None and "l2_to_sm_bytes" in tr:
                bnd = binding_roofline(tr, tot_ms / n_launch, l2_peaks, gather_bytes(name, wl))
                f = bnd["floor_ms"]
            else:
                amount, unit, _ = kernel_work(name, wl)
                f = amount / (peaks.get("hbm_gbs", 6650.0) * 1e9) * 1e3 if unit == "byte" else 0.0
            parts[name] = round(f * n_launch / args.steps, 4)
            floor_ms += f * n_launch / args.steps
        roof["step_floor_ms"] = round(floor_ms, 4)
        roof["step_floor_frac"] = round(floor_ms / ms_per_step, 3)
        roof["step_floor_parts_ms"] = parts

    # ---- end to end through the public module API, host buffers ----
    e2e = None if (args.profile or strong) else run_e2e(args, wl, x, w, b, off, m, go, dev, world, flags,
                                            allreduce, flush)

    kernel_table = {k: {"launches": v[0], "ms_per_launch": round(v[1] / v[0], 4)}
                    for k, v in sorted(kernels.items(), key=lambda kv: -kv[1][1])}
    line = {
        "metric": METRIC, "value": round(value, 4), "unit": "ms/iter", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4),
        "higher_is_better": False, "scaling": args.scaling, "vs_baseline": None,
        "dtype": (args.dtype if any(k in BF16_KERNELS for k in kernels) else
                  (f"{args.dtype} I/O, " if args.dtype in HALF else "") +
                  (args.math if any(k in TC_KERNELS for k in kernels) else "f32")),
        "data": "synthetic",
        "config": bench_config(wl, args),
        "run": {"per_step_batch": wl["N"] if strong else wl["N"] * world,
                "per_gpu_batch": xd.shape[0],
                "parallelism": (f"dp{world // slabs}x{slabs} row slabs" if strong
                                else f"dp{world}"),
                "math": args.math,
                "l2": "flushed between timed iterations (256 MiB write, outside the timed "
                      "events)",
                "wall_s": round(wall, 3),
                "kernel_table": ("a second pass of the same steps with a CUDA event pair "
                                 "around every library launch (gpu_launches, kernels, "
                                 "roofline.achieved); its ms/step: %.4f" %
                                 (prof_ms / args.steps))},
        "roofline": roof, "e2e": e2e, "gpu_launches": launches,
        "kernels": kernel_table,
    }
    if world == 1 and not args.profile:
        line["cuda_graph"] = graph_step_ms(step, leaves, flush, args.steps)
        line["math_modes"] = other_math_modes(args, step_with_flags, flush)
        line["e2e_full_readback"] = run_e2e(args, wl, x, w, b, off, m, go, dev, world, flags,
                                            allreduce, flush, full=True)
    if world == 1 and not (args.no_cpu_baseline or args.profile):
        line["cpu_baseline"] = cpu_baseline(wl)
    clk = clocks.summary()
    line["clocks"] = {"sm_mhz": clk["sm_mhz"], "sm_max_mhz": clk["sm_max_mhz"],
                      "reasons": clk["reasons"]}
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


def graph_step_ms(step, leaves, flush, steps):
    """The same step captured once in a CUDA graph and replayed (launch gaps
    removed): CUDA events around each replay, L2 flushed before each,
    inputs resident.  An extra figure beside the eager `value`."""
    import torch
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(2):
            step()
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    for t in leaves:
        t.grad = None
    with torch.cuda.graph(graph):
        step()
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    total = 0.0
    for _ in range(steps):
        flush.zero_()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        graph.replay()
        e1.record()
        e1.synchronize()
        total += e0.elapsed_time(e1)
    del graph
    return {"ms_per_step": round(total / steps, 4), "mode": "whole fwd+bwd step replayed"}


def other_math_modes(args, step_with_flags, flush):
    """ms per step of the same step in the other math modes (3xTF32: fp32
    accuracy on the tensor cores; fp32: FFMA on the CUDA cores, the strict
    parity mode), timed like the headline: 2 untimed steps, then K steps with
    CUDA events around each, L2 flushed before each."""
    import torch
    from pytorch_mps_deform_conv2d_b200.ops import _MODES
    res = {}
    for mode in ("3xtf32", "fp32"):
        if mode == args.math:
            continue
        fl = _MODES[mode]
        for _ in range(2):
            step_with_flags(fl)
        torch.cuda.synchronize()
        total = 0.0
        for _ in range(args.steps):
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            step_with_flags(fl)
            e1.record()
            e1.synchronize()
            total += e0.elapsed_time(e1)
        res[mode] = {"ms_per_step": round(total / args.steps, 4)}
    return res


def run_e2e(args, wl, x, w, b, off, m, go, dev, world, flags, allreduce, flush, full=False):
    """Same step through the public module API with the batch coming from
    pinned host memory and the parameter gradients read back each step (with
    `full`: the output and every gradient -- input, offset, mask, weight,
    bias -- read back, the op's whole result).

    Two measurements: `serial` -- each step copies its inputs, computes and
    reads back, alone, L2 flushed before it; `pipelined` (the reported value)
    -- the steps run back to back the way a data loader feeds training: step
    i+1's host-to-device copies run on a copy stream into a second set of
    buffers while step i computes.  Every step still moves all of its inputs
    over PCIe and reads its results back inside the timed region."""
    import torch
    import pytorch_mps_deform_conv2d_b200 as dcn
    mod = dcn.DeformConv2d(wl["C"], wl["outC"], wl["k"], stride=wl["stride"], padding=wl["pad"],
                           dilation=wl["dil"], groups=wl["groups"], bias=wl["bias"]).to(dev)
    if args.dtype in HALF:
        mod = mod.to(getattr(torch, HALF[args.dtype]))
    with torch.no_grad():
        mod.weight.copy_(w)
        if b is not None:
            mod.bias.copy_(b)
    dcn.set_math_mode(args.math)
    host = [t.pin_memory() if t is not None else None for t in (x, off, m, go)]
    params = [p for p in mod.parameters()]
    pdt = params[0].dtype
    # read back: the parameter gradients, and with `full` also the output and
    # the input, offset and mask gradients (shapes of x, off, m, go)
    back_shapes = [p.shape for p in params]
    if full:
        back_shapes += [t.shape for t in (go, x, off, m) if t is not None]
    outs = [torch.empty(s, dtype=pdt, pin_memory=True) for s in back_shapes]
    h2d = sum(t.numel() * t.element_size() for t in host if t is not None)
    d2h = sum(o.numel() * o.element_size() for o in outs)
    compute = torch.cuda.current_stream(dev)
    copier = torch.cuda.Stream(dev)
    slots = [[torch.empty_like(t, device=dev) if t is not None else None for t in host]
             for _ in range(2)]
    copied = [torch.cuda.Event() for _ in range(2)]
    used = [torch.cuda.Event() for _ in range(2)]

    def load(slot, stream):
        with torch.cuda.stream(stream):
            for d, h in zip(slots[slot], host):
                if d is not None:
                    d.copy_(h, non_blocking=True)
            copied[slot].record(stream)

    def run(slot):
        compute.wait_event(copied[slot])
        xd, od, md, gd = slots[slot]
        xd = xd.detach().requires_grad_(True)
        od = od.detach().requires_grad_(True)
        md = md.detach().requires_grad_(True) if md is not None else None
        for p in params:
            p.grad = None
        out = mod(xd, od, md)
        out.backward(gd)
        allreduce(params)
        results = [p.grad for p in params]
        if full:
            results += [out.detach()] + [t.grad for t in (xd, od, md) if t is not None]
        for r, o in zip(results, outs):
            o.copy_(r, non_blocking=True)
        used[slot].record(compute)

    try:
        for i in range(max(3, args.warmup)):
            load(i % 2, compute)
            run(i % 2)
        torch.cuda.synchronize()
        # serial: one step at a time
        serial = 0.0
        for _ in range(args.steps):
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(compute)
            load(0, compute)
            run(0)
            e1.record(compute)
            e1.synchronize()
            serial += e0.elapsed_time(e1)
        # pipelined: copies of step i+1 overlap the compute of step i
        flush.zero_()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(compute)
        copier.wait_stream(compute)
        load(0, copier)
        for i in range(args.steps):
            if i + 1 < args.steps:
                nxt = (i + 1) % 2
                copier.wait_event(used[nxt])  # the buffers' previous step is done
                load(nxt, copier)
            run(i % 2)
        e1.record(compute)
        e1.synchronize()
        piped = e0.elapsed_time(e1)
    finally:
        dcn.set_math_mode(None)
    if world > 1:
        import torch.distributed as dist
        t = torch.tensor([serial, piped], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        serial, piped = float(t[0].item()), float(t[1].item())
    return {"value": round(piped / args.steps / world, 4), "unit": "ms/iter",
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "mode": "pipelined",
            "serial_value": round(serial / args.steps / world, 4),
            "read_back": ("output and all five gradients" if full
                          else "grad_weight and grad_bias")}


# ---------------------------------------------------------------------------
# reference arm
# ---------------------------------------------------------------------------
def run_reference(args, wl):
    """The reference's own CPU implementation of the path (its public
    deform_conv2d on CPU tensors, which routes to torchvision's kernel) on the
    whole workload, all host threads, rank 0 only: `warmup` untimed steps,
    then `steps` timed ones (about 8.5 s a step for the detection neck on 16
    cores)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    step, _, desc = cpu_reference_step_fn(wl, threads)
    import torch
    t0 = time.perf_counter()
    value = time_cpu_steps(step, args.steps, args.warmup) * 1e3
    wall = time.perf_counter() - t0
    line = {
        "metric": METRIC, "impl": "reference", "value": round(value, 3), "unit": "ms/iter",
        "n_gpus": int(os.environ.get("WORLD_SIZE", "1")), "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(value, 3), "higher_is_better": False,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": bench_config(wl),
        "run": {"where": "host CPU, one process", "threads": torch.get_num_threads(),
                "wall_s": round(wall, 3)},
        "cpu_baseline": {"value": round(value, 3), "unit": "ms/iter",
                         "cores": torch.get_num_threads(), "kind": "reference",
                         "sample": desc + f"; {args.steps} timed steps after {args.warmup} "
                                          "untimed, unscaled"},
        "e2e": {"value": round(value, 3), "unit": "ms/iter", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--math", choices=["tf32", "fp32", "3xtf32"], default="tf32")
    ap.add_argument("--scaling", choices=["weak", "strong"], default="weak",
                    help="weak: every rank a whole batch; strong: the one batch split over the "
                         "ranks (images, then row slabs of each image)")
    ap.add_argument("--dtype", choices=["fp32", "bf16", "fp16"], default="fp32",
                    help="tensor dtype of the step (the reference and the headline: fp32)")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="neck")
    ap.add_argument("--layout", choices=["nchw", "nhwc"], default="nchw",
                    help="memory format of the input (nhwc: torch.channels_last)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--profile", action="store_true",
                    help="device steps only (no CPU baseline, no e2e pass, no cuBLAS peak "
                         "runs): the command the ncu captures wrap")
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "ours":
        args.warmup = 3
    wl = WORKLOADS[args.workload]
    if args.impl == "reference":
        run_reference(args, wl)
    else:
        run_ours(args, wl)


if __name__ == "__main__":
    main()
