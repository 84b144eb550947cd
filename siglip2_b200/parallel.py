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


def gather_pooled(pooled_local: torch.Tensor, owned: list[list[int]], group=None) -> torch.Tensor:
    """All-gather every rank's ``[B_r, D]`` pooled rows and return ``[B, D]``
    in global image order.  Ranks are padded to the largest shard so one
    ``all_gather_into_tensor`` suffices."""
    world = len(owned)
    bmax = max(len(o) for o in owned)
    D = pooled_local.shape[1]
    send = torch.zeros((bmax, D), dtype=pooled_local.dtype, device=pooled_local.device)
    send[: pooled_local.shape[0]] = pooled_local
    recv = torch.empty((world * bmax, D), dtype=pooled_local.dtype, device=pooled_local.device)
    dist.all_gather_into_tensor(recv, send, group=group)
    total = sum(len(o) for o in owned)
    out = torch.empty((total, D), dtype=pooled_local.dtype, device=pooled_local.device)
    for r, idx in enumerate(owned):
        if idx:
            out[torch.tensor(idx, device=out.device)] = recv[r * bmax: r * bmax + len(idx)]
    return out
