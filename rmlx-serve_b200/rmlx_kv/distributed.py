"""Host-side helpers for a pool sharded over GPUs (one process per GPU).

The KV heads of a model are split over the ranks; the block manager, the
prefix cache and the block tables are replicated (every rank makes the same
decisions from the same inputs), so the per-step device work needs no
collective.  Two host exchanges remain:

* sharing the NCCL unique id that block migration uses;
* agreeing on a migration plan: how many blocks move, and where the
  receiver puts them (it allocates them in its own block manager).

Both run over an existing torch.distributed process group (gloo or NCCL),
which here is plumbing only; the block bytes move through the library's
own NCCL communicator (``NcclComm`` / ``KVPool.migrate``).
"""
from __future__ import annotations

from typing import List, Tuple

import numpy as np


def shard_heads(num_heads: int, world: int, rank: int) -> Tuple[int, int]:
    """(head_offset, heads_on_this_rank) for an even split of the KV heads."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    if num_heads % world:
        raise ValueError(f"{num_heads} KV heads do not split evenly over {world} ranks")
    per = num_heads // world
    return rank * per, per


def _dev(group):
    import torch
    import torch.distributed as dist
    backend = dist.get_backend(group)
    return torch.device("cuda", torch.cuda.current_device()) if backend == "nccl" else torch.device("cpu")


def share_nccl_id(group=None) -> bytes:
    """Rank 0 of `group` makes an NCCL unique id; every rank returns it."""
    import torch
    import torch.distributed as dist
    from .pool import NcclComm
    buf = torch.zeros(128, dtype=torch.uint8, device=_dev(group))
    if dist.get_rank(group) == 0:
        buf.copy_(torch.frombuffer(bytearray(NcclComm.unique_id()), dtype=torch.uint8))
    dist.broadcast(buf, src=dist.get_global_rank(group, 0) if group is not None else 0, group=group)
    return bytes(buf.cpu().numpy().tobytes())


def exchange_migration_plan(mgr, send_ids: List[int], peer: int, group=None) -> Tuple[List[int], int]:
    """Tell `peer` how many blocks this rank sends and learn how many it sends
    here; allocate that many destination blocks from `mgr` (this rank's block
    manager).  Returns (recv_ids, n_peer_sends).  Raises if this pool cannot
    hold the incoming blocks (nothing is allocated then)."""
    import torch
    import torch.distributed as dist
    dev = _dev(group)
    mine = torch.tensor([len(send_ids)], dtype=torch.int64, device=dev)
    theirs = torch.zeros(1, dtype=torch.int64, device=dev)
    me = dist.get_rank()
    # Deadlock-free pairwise exchange: the lower rank sends first.
    if me < peer:
        dist.send(mine, dst=peer, group=group)
        dist.recv(theirs, src=peer, group=group)
    else:
        dist.recv(theirs, src=peer, group=group)
        dist.send(mine, dst=peer, group=group)
    n_in = int(theirs.item())
    if n_in > mgr.num_free_blocks():
        raise RuntimeError(f"peer sends {n_in} blocks, only {mgr.num_free_blocks()} free here")
    recv_ids = mgr.allocate_n(n_in).tolist()
    return recv_ids, n_in


def remap_block_table(bt: np.ndarray, moved_from: List[int], moved_to: List[int]) -> np.ndarray:
    """Block table with every id in moved_from replaced by its moved_to twin."""
    lut = {int(a): int(b) for a, b in zip(moved_from, moved_to)}
    out = bt.copy()
    flat = out.reshape(-1)
    for i, x in enumerate(flat):
        y = lut.get(int(x))
        if y is not None:
            flat[i] = y
    return out
