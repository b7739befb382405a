"""Batch-sharded data parallelism on CPU ranks (gloo, world size 2): sharded
forward/backward with the oracle plus the all-reduce of grad_weight /
grad_bias equals the single-process result; a rank that fails before the
collective makes the others fail on a short timeout instead of hanging."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from pytorch_mps_deform_conv2d_b200.distributed import allreduce_grads, shard_batch, shard_range


def test_shard_range_balanced():
    for n in range(0, 11):
        for w in range(1, 5):
            sl = [shard_range(n, r, w) for r in range(w)]
            assert sl[0].start == 0 and sl[-1].stop == n
            assert all(a.stop == b.start for a, b in zip(sl, sl[1:]))
            sizes = [s.stop - s.start for s in sl]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_range(4, 2, 2)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, case, result_q, fail_rank, adjacent=False):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=10))
    try:
        if rank == fail_rank:
            raise RuntimeError("injected failure before the collective")
        from oracle import oracle
        x, off, m, go = shard_batch([case["x"], case["off"], case["m"], case["go"]], rank, world)
        _, _, _, gw, gb = oracle.backward(go.numpy(), x.numpy(), off.numpy(), case["w"].numpy(),
                                          case["b"].numpy(), 1, 1, 1, m.numpy())
        w = torch.nn.Parameter(case["w"].clone())
        b = torch.nn.Parameter(case["b"].clone())
        if adjacent:  # grad_weight and grad_bias back to back in one buffer
            flat = torch.cat([torch.from_numpy(gw).reshape(-1), torch.from_numpy(gb)])
            w.grad = flat[:gw.size].view(gw.shape)
            b.grad = flat[gw.size:]
            allreduce_grads([w, b])
            assert w.grad.data_ptr() == flat.data_ptr()  # reduced in place
        else:
            w.grad, b.grad = torch.from_numpy(gw), torch.from_numpy(gb)
            allreduce_grads([w, b])
        result_q.put((rank, "ok", w.grad.numpy(), b.grad.numpy()))
    except Exception as e:  # report, then leave the group
        result_q.put((rank, "error", repr(e), None))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _case():
    torch.manual_seed(0)
    N, C, O, H, W = 4, 8, 6, 9, 10
    return dict(x=torch.randn(N, C, H, W), w=torch.randn(O, C, 3, 3), b=torch.randn(O),
                off=torch.randn(N, 18, H, W), m=torch.rand(N, 9, H, W), go=torch.randn(N, O, H, W))


def _run(world, fail_rank=-1, adjacent=False):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    case = _case()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, case, q, fail_rank, adjacent))
             for r in range(world)]
    for p in procs:
        p.start()
    out = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return case, sorted(out, key=lambda r: r[0])


@pytest.mark.parametrize("adjacent", [False, True], ids=["separate", "in-place"])
def test_sharded_grads_equal_full_batch(adjacent):
    from oracle import oracle
    case, out = _run(2, adjacent=adjacent)
    _, _, _, gw, gb = oracle.backward(case["go"].numpy(), case["x"].numpy(), case["off"].numpy(),
                                      case["w"].numpy(), case["b"].numpy(), 1, 1, 1,
                                      case["m"].numpy())
    for rank, status, rgw, rgb in out:
        assert status == "ok", rgw
        np.testing.assert_allclose(rgw, gw, rtol=1e-5, atol=1e-4)
        np.testing.assert_allclose(rgb, gb, rtol=1e-5, atol=1e-4)


def test_failed_rank_surfaces_as_error_not_hang():
    _, out = _run(2, fail_rank=1)
    assert out[1][1] == "error" and "injected" in out[1][2]
    assert out[0][1] == "error"  # the survivor's collective fails on the timeout


def _hook_worker(rank, world, port, result_q, bucketed=False):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=10))
    try:
        from pytorch_mps_deform_conv2d_b200.distributed import GradAllReduce, GradBucket
        w = torch.nn.Parameter(torch.zeros(4, 3))
        b = torch.nn.Parameter(torch.zeros(4))
        bucket = GradBucket([w, b]) if bucketed else None  # one flat collective
        sync = GradAllReduce([w, b], average=False)
        got = []
        for step in range(2):  # the hooks re-arm after wait()
            if bucket is not None:
                bucket.zero_()
            else:
                w.grad = b.grad = None
            xs = torch.full((4, 3), float(rank + 1 + 10 * step))
            ys = torch.full((4,), float(2 * (rank + 1) + 10 * step))
            ((w * xs).sum() + (b * ys).sum()).backward()
            sync.wait()
            got.append((w.grad.clone().numpy(), b.grad.clone().numpy()))
        sync.remove()
        result_q.put((rank, "ok", got))
    except Exception as e:
        result_q.put((rank, "error", repr(e)))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


@pytest.mark.parametrize("bucketed", [False, True], ids=["separate", "bucket"])
def test_grad_allreduce_hooks_sum_after_backward(bucketed):
    """GradAllReduce: the collective starts from the parameters' hooks once
    both gradients are accumulated, and wait() leaves the summed gradients
    (separate gradients, or a GradBucket's views reduced as one buffer)."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_hook_worker, args=(r, 2, port, q, bucketed))
             for r in range(2)]
    for p in procs:
        p.start()
    out = sorted([q.get(timeout=120) for _ in procs], key=lambda r: r[0])
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    for rank, status, got in out:
        assert status == "ok", got
        for step, (gw, gb) in enumerate(got):
            np.testing.assert_array_equal(gw, np.full((4, 3), 1 + 2 + 20 * step, np.float32))
            np.testing.assert_array_equal(gb, np.full((4,), 2 + 4 + 20 * step, np.float32))


def _bucket_worker(rank, world, port, result_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=10))
    try:
        from pytorch_mps_deform_conv2d_b200.distributed import GradBucket
        w = torch.nn.Parameter(torch.zeros(4, 3))
        b = torch.nn.Parameter(torch.zeros(4))
        bucket = GradBucket([w, b])
        got = []
        for step in range(2):
            bucket.zero_()
            xs = torch.full((4, 3), float(rank + 1 + 10 * step))
            ((w * xs).sum() + (b * (rank + 2)).sum()).backward()
            # accumulated in place into the bucket's views
            assert w.grad.data_ptr() == bucket.flat.data_ptr()
            allreduce_grads([w, b])
            got.append((w.grad.clone().numpy(), b.grad.clone().numpy()))
        result_q.put((rank, "ok", got))
    except Exception as e:
        result_q.put((rank, "error", repr(e)))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def test_grad_bucket_accumulates_in_place_and_reduces_once():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_bucket_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = sorted([q.get(timeout=120) for _ in procs], key=lambda r: r[0])
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    for rank, status, got in out:
        assert status == "ok", got
        for step, (gw, gb) in enumerate(got):
            np.testing.assert_array_equal(gw, np.full((4, 3), 1 + 2 + 20 * step, np.float32))
            np.testing.assert_array_equal(gb, np.full((4,), 2 + 3, np.float32))


def test_adjacent_view_takes_the_gradients_in_any_order():
    from pytorch_mps_deform_conv2d_b200.distributed import _adjacent_view
    flat = torch.arange(15, dtype=torch.float32)
    gw, gb = flat[:12].view(4, 3), flat[12:]
    for grads in ([gw, gb], [gb, gw]):  # hooks may deliver either first
        view = _adjacent_view(grads)
        assert view is not None and view.data_ptr() == flat.data_ptr()
        assert torch.equal(view, flat)
    assert _adjacent_view([gw, flat[13:]]) is None  # a gap
    assert _adjacent_view([gw, torch.zeros(3)]) is None  # another storage
