"""Expert-parallel decode across ranks: the host side of hg_engine_ep_init.

One process per GPU, each with its own Engine and its own sequences. The routed experts of every MoE
layer are split evenly: rank q owns experts [q E/W, (q+1) E/W). Rank 0 creates the NCCL unique id
and every rank receives it over torch.distributed; the broadcast runs under the process group's
timeout, so a rank that never joins makes the others fail on the host (instead of blocking in the
NCCL rendezvous). Each engine then builds its communicator and, from the next decode step on,
exchanges its tokens' expert rows with the owners (include/hobbygpu.h).
"""
from __future__ import annotations

from typing import Callable


def experts_per_rank(n_experts: int, world: int) -> int:
    if world < 1 or n_experts % world:
        raise ValueError(f"{n_experts} experts do not split evenly over {world} ranks")
    return n_experts // world


def owner(expert: int, n_experts: int, world: int) -> int:
    """Rank that computes routed expert `expert`."""
    return expert // experts_per_rank(n_experts, world)


def local_experts(rank: int, n_experts: int, world: int) -> range:
    epr = experts_per_rank(n_experts, world)
    return range(rank * epr, (rank + 1) * epr)


def exchange_id(make_id: Callable[[], bytes], group=None) -> bytes:
    """Rank 0's id (make_id() there) on every rank of `group`; raises if a rank does not join
    within the process group's timeout."""
    import torch.distributed as dist

    obj = [make_id() if dist.get_rank(group) == 0 else None]
    dist.broadcast_object_list(obj, src=0, group=group)
    return obj[0]


def setup(engine, group=None) -> None:
    """Expert parallelism on `engine` over the ranks of `group` (torch.distributed must be
    initialized; one engine per rank, all loaded from the same model)."""
    import torch.distributed as dist

    from .engine import Engine

    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    experts_per_rank(engine.cfg["n_experts"], world)  # fail early, on every rank alike
    uid = exchange_id(Engine.ep_unique_id, group)
    engine.ep_init(uid, rank, world)
