"""GradAllReduce over NCCL (two GPUs, one process each): the hooks start one
coalesced asynchronous all-reduce of a DCN layer's grad_weight and grad_bias
once the backward has produced both, and wait() leaves each rank with the sum
of the ranks' gradients.  Skipped with fewer than two GPUs."""
import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, result_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        from _util import make_case
        from pytorch_mps_deform_conv2d_b200.distributed import GradAllReduce
        from pytorch_mps_deform_conv2d_b200.ops import MATH_TF32, deform_conv2d_ex
        case = make_case(N=2, inC=64, outC=64, H=12, W=14, offset_scale=2.0, seed=rank)
        dev = torch.device("cuda", rank)

        def step(w, b):
            out = deform_conv2d_ex(case["x"].to(dev), case["off"].to(dev), w, b, case["stride"],
                                   case["padding"], case["dilation"], case["m"].to(dev),
                                   flags=MATH_TF32)
            out.backward(case["go"].to(dev))

        # reference: this rank's gradients, summed by plain blocking all-reduces
        w0 = torch.nn.Parameter(case["w"].to(dev))
        b0 = torch.nn.Parameter(case["b"].to(dev))
        step(w0, b0)
        expect = [w0.grad, b0.grad]
        for t in expect:
            dist.all_reduce(t)
        # the hooks: the collective starts inside the backward
        w = torch.nn.Parameter(case["w"].to(dev))
        b = torch.nn.Parameter(case["b"].to(dev))
        sync = GradAllReduce([w, b])
        step(w, b)
        sync.wait()
        torch.cuda.synchronize()
        # the grad_weight reductions' order varies run to run: TF32 noise only
        ok = all(torch.allclose(a, e, rtol=1e-4, atol=1e-4 * float(e.abs().max()))
                 for a, e in zip((w.grad, b.grad), expect))
        sync.remove()
        result_q.put((rank, "ok" if ok else "mismatch"))
    except Exception as e:
        result_q.put((rank, "error: " + repr(e)))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def test_grad_allreduce_over_nccl():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = sorted([q.get(timeout=300) for _ in procs])
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert [r[1] for r in out] == ["ok", "ok"], out
