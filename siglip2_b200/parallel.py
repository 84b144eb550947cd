"""Image-parallel sharding of a NaFlex batch across ranks (one process per
GPU) and the single collective of the path: an all-gather of the pooled
embeddings.

The tower has no cross-image interaction (the document mask is
block-diagonal, ``model.py:156-161``; the head pools per image), so each rank
runs the whole forward on its own images with replicated weights and no
collective inside the forward.
"""
from __future__ import annotations

import heapq

import torch
import torch.distributed as dist


def image_cost(h: int, w: int, d_model: int = 1152, mlp: int = 4304) -> float:
    """Relative forward cost of one image: linear terms (projections, MLP)
    plus the quadratic attention term, 4 L^2 D per layer."""
    L = h * w
    return L * (8 * d_model * d_model + 4 * d_model * mlp) + 4 * L * L * d_model


def shard_images(shapes, world: int, d_model: int = 1152, mlp: int = 4304) -> list[list[int]]:
    """Longest-processing-time-first assignment of images to ranks by cost.
    Returns, per rank, the global image indices it owns (ascending)."""
    costs = sorted(((image_cost(int(h), int(w), d_model, mlp), i) for i, (h, w) in enumerate(shapes)),
                   reverse=True)
    heap = [(0.0, r) for r in range(world)]
    owned = [[] for _ in range(world)]
    for c, i in costs:
        load, r = heapq.heappop(heap)
        owned[r].append(i)
        heapq.heappush(heap, (load + c, r))
    return [sorted(o) for o in owned]


class PooledGather:
    """The path's one collective, set up once per sharding: every rank's
    ``[B_r, D]`` pooled rows are padded to the largest shard, gathered with
    one ``all_gather_into_tensor`` and put back into global image order with
    one precomputed ``index_select`` (no host work or host-to-device copy per
    call)."""

    def __init__(self, owned: list[list[int]], dim: int, dtype, device, group=None):
        self.world = len(owned)
        self.bmax = max(len(o) for o in owned)
        self.group = group
        self.send = torch.zeros((self.bmax, dim), dtype=dtype, device=device)
        self.recv = torch.empty((self.world * self.bmax, dim), dtype=dtype, device=device)
        pos = {}
        for r, idx in enumerate(owned):
            for k, i in enumerate(idx):
                pos[i] = r * self.bmax + k
        total = sum(len(o) for o in owned)
        assert sorted(pos) == list(range(total)), "shards must cover every image exactly once"
        self.index = torch.tensor([pos[i] for i in range(total)], dtype=torch.int64, device=device)

    def __call__(self, pooled_local: torch.Tensor) -> torch.Tensor:
        n = pooled_local.shape[0]
        self.send[:n].copy_(pooled_local)
        dist.all_gather_into_tensor(self.recv, self.send, group=self.group)
        return self.recv.index_select(0, self.index)


def gather_pooled(pooled_local: torch.Tensor, owned: list[list[int]], group=None) -> torch.Tensor:
    """All-gather every rank's ``[B_r, D]`` pooled rows and return ``[B, D]``
    in global image order (one-shot form of ``PooledGather``)."""
    return PooledGather(owned, pooled_local.shape[1], pooled_local.dtype, pooled_local.device, group)(pooled_local)
