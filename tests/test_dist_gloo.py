"""Multi-rank host logic on CPU (gloo): sharding balance, the all-gather of
pooled embeddings with un-permutation, and a rank that fails before the
collective (the others get an error from the short process-group timeout,
they do not hang)."""
import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from siglip2_b200 import workloads as W
from siglip2_b200.parallel import gather_pooled, image_cost, shard_images


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_shard_images_balanced_and_complete():
    shapes = W.sample_spatial_shapes("area_aspect", 512, 1024, seed=1337)
    for world in (2, 4, 8):
        owned = shard_images(shapes.tolist(), world)
        flat = sorted(i for o in owned for i in o)
        assert flat == list(range(512))
        loads = [sum(image_cost(*shapes[i].tolist()) for i in o) for o in owned]
        assert max(loads) / min(loads) < 1.01


def _worker(rank, world, port, shapes, fail_rank, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
    try:
        owned = shard_images(shapes, world)
        if rank == fail_rank:
            raise RuntimeError("injected failure before the collective")
        # a stand-in for the pooled embeddings: row i carries its global image index
        local = torch.tensor([[float(i)] * 4 for i in owned[rank]], dtype=torch.float32).reshape(-1, 4)
        out = gather_pooled(local, owned)
        ok = torch.equal(out[:, 0], torch.arange(len(shapes), dtype=torch.float32))
        q.put((rank, "ok" if ok else "mismatch"))
    except Exception as e:  # noqa: BLE001
        q.put((rank, f"error: {type(e).__name__}"))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:  # noqa: BLE001
            pass


def _run(world, fail_rank=-1):
    shapes = W.sample_spatial_shapes("area_aspect", 37, 1024, seed=5).tolist()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, shapes, fail_rank, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert not p.is_alive()
    return dict(q.get(timeout=5) for _ in range(world))


@pytest.mark.parametrize("world", [2, 4])
def test_gather_pooled_gloo(world):
    res = _run(world)
    assert all(v == "ok" for v in res.values()), res


def test_failed_rank_does_not_hang_peers():
    res = _run(2, fail_rank=1)
    assert res[1].startswith("error")
    assert res[0].startswith("error"), res  # the peer's collective ends with an error, not a hang
