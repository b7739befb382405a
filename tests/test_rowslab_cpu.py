"""Row slabs (more ranks than images) on CPU ranks: the rank -> (image, slab)
map covers every output row of every image exactly once, and the gradient
exchange of the replicated input sums over the ranks of one image only
(gloo, world size 4, two images)."""
import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from pytorch_mps_deform_conv2d_b200.distributed import image_slab, slab_rows


@pytest.mark.parametrize("world", [1, 2, 4, 8])
@pytest.mark.parametrize("out_h", [1, 7, 100])
def test_image_slabs_cover_every_row_once(world, out_h):
    n_images = 2
    if world > n_images and out_h < world // n_images:
        pytest.skip("fewer rows than slabs")
    seen = {}
    for r in range(world):
        first, count, slab, slabs = image_slab(r, world, n_images)
        rows = slab_rows(out_h, slab, slabs)
        for n in range(first, first + count):
            for y in range(rows.start, rows.stop):
                assert (n, y) not in seen, (r, n, y)
                seen[(n, y)] = r
    assert len(seen) == n_images * out_h


def test_image_slab_rejects_uneven_split():
    with pytest.raises(ValueError):
        image_slab(0, 3, 2)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=20))
    try:
        from pytorch_mps_deform_conv2d_b200.distributed import _SumGradOver, image_groups
        groups = image_groups(world, 2)
        first, _, _, _ = image_slab(rank, world, 2)
        x = torch.ones(3, requires_grad=True)
        y = _SumGradOver.apply(x, groups[first])
        (y * float(rank + 1)).sum().backward()
        q.put((rank, x.grad.tolist()))
    except Exception as e:
        q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


def test_input_gradient_summed_over_the_image_ranks():
    world = 4
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    # ranks 0, 1 share image 0 (weights 1 + 2); ranks 2, 3 image 1 (3 + 4)
    assert results[0] == results[1] == [3.0, 3.0, 3.0], results
    assert results[2] == results[3] == [7.0, 7.0, 7.0], results
