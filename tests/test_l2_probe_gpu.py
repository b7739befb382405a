"""dcn_l2_probe, the L2 <-> SM bandwidth probe behind the bench line's
binding-resource roofline: the reduction kind adds exactly 1.0 per pass to
every float of the swept bytes (and nothing past them), the mixed kind to
every float of its reduced part only, the load kind leaves the buffer as it
was, bad arguments are refused, and all three report a bandwidth in a
plausible range."""
import ctypes

import pytest
import torch

from pytorch_mps_deform_conv2d_b200 import _native

pytestmark = pytest.mark.gpu


def _probe(kind, buf, nbytes, passes):
    lib = _native.load_capi()
    stream = torch.cuda.current_stream()
    return lib.dcn_l2_probe(kind, ctypes.c_void_p(buf.data_ptr()), nbytes, passes,
                            ctypes.c_void_p(stream.cuda_stream))


def test_reduction_probe_adds_one_per_pass(cuda_device):
    buf = torch.zeros(1 << 18, device="cuda")  # 1 MiB
    swept = (1 << 20) - 48  # not a multiple of the grid's stride
    assert _probe(1, buf, swept + 8, 3) == 0  # rounded down to 16 bytes
    torch.cuda.synchronize()
    n = swept // 4
    assert torch.all(buf[:n] == 3.0)
    assert torch.all(buf[n:] == 0.0)


def test_mixed_probe_adds_to_its_last_two_sevenths(cuda_device):
    blocks = 40
    buf = torch.zeros(blocks * 3584 // 4 + 64, device="cuda")
    assert _probe(2, buf, blocks * 3584 + 100, 2) == 0  # rounded down to 3584 bytes
    torch.cuda.synchronize()
    nr = blocks * 160 * 4  # floats read
    nw = blocks * 64 * 4   # floats reduced
    assert torch.all(buf[:nr] == 0.0)
    assert torch.all(buf[nr:nr + nw] == 2.0)
    assert torch.all(buf[nr + nw:] == 0.0)


def test_scatter_probe_adds_four_per_reduction(cuda_device):
    buf = torch.zeros(8 << 20, device="cuda")  # 32 MiB
    assert _probe(4, buf, buf.numel() * 4, 2) == 0
    torch.cuda.synchronize()
    warps = torch.cuda.get_device_properties(0).multi_processor_count * 64
    per_warp = buf.numel() * 4 // 16 // 32 // warps // 4 * 4
    expected = 2 * warps * per_warp * 32 * 4  # passes x reductions x 4 floats
    assert float(buf.double().sum()) == expected
    assert float(buf.max()) <= 2 * 32 * 4 * per_warp  # nothing outside the lines' floats


def test_load_probe_leaves_the_buffer(cuda_device):
    buf = torch.arange(1 << 18, device="cuda", dtype=torch.float32)
    ref = buf.clone()
    assert _probe(0, buf, buf.numel() * 4, 4) == 0
    torch.cuda.synchronize()
    assert torch.equal(buf, ref)


def test_bad_arguments_are_refused(cuda_device):
    buf = torch.zeros(1024, device="cuda")
    assert _probe(5, buf, 4096, 1) == 1
    assert _probe(4, buf, 4096, 1) == 1  # too small for one scatter round
    assert _probe(3, buf, 4096, 1) == 1  # too small for one gather round
    assert _probe(2, buf, 3568, 1) == 1  # under one mixed block
    assert _probe(0, buf, 4096, 0) == 1
    assert _probe(0, buf, 8, 1) == 1
    misaligned = buf[1:]
    assert _probe(0, misaligned, 1024, 1) == 1


def test_bandwidths_are_plausible(cuda_device):
    import bench
    peaks = bench.measure_l2_gbs(bytes_=32 << 20, passes=8, reps=3)
    # above HBM-class copy rates, below anything the crossbar could carry
    assert 2000.0 < peaks["l2_to_sm"] < 200000.0, peaks
    assert 500.0 < peaks["sm_to_l2_red"] < 200000.0, peaks
    assert 500.0 < peaks["mixed_5to2"] < 200000.0, peaks
    assert 500.0 < peaks["gather"] < 200000.0, peaks
    assert 200.0 < peaks["scatter_red"] < 200000.0, peaks
