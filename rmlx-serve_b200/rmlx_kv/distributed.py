"""Host-side helpers for a pool sharded over GPUs (one process per GPU).

The KV heads of a model are split over the ranks; the block manager, the
prefix cache and the block tables are replicated (every rank makes the same
decisions from the same inputs), so the per-step device work needs no
collective.  Two host exchanges remain:

* sharing the NCCL unique id that block migration uses;
* agreeing on a migration plan: how many blocks move, and where the
  receiver puts them (it allocates them in its own block manager).

The id travels over an existing torch.distributed process group (gloo or
NCCL); the plan travels through that group's host key-value store with a
bounded wait, so a rank that has left is found on the host before any
NCCL transfer is posted toward it.  torch.distributed is plumbing only; the
block bytes move through the library's own NCCL communicator (``NcclComm``
/ ``KVPool.migrate``).
"""
from __future__ import annotations

from typing import List, Optional, Tuple

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


_EPOCH = {}


def reset_plan_counts() -> None:
    """Forget this process's exchange counts (for a new job sharing the
    process with a new store and new peers)."""
    _EPOCH.clear()


def _default_store():
    from torch.distributed import distributed_c10d
    return distributed_c10d._get_default_store()


def depart(store=None, rank: Optional[int] = None) -> None:
    """Announce on the host that this rank leaves the job between steps.

    A rank calls this after its last collective has completed (nothing of
    its own in flight on the GPU).  A peer's next ``exchange_migration_plan``
    sees the mark and fails at once with RMLX_E_TIMEOUT instead of waiting
    out its deadline; it never enqueues an NCCL transfer toward the rank
    that left."""
    import torch.distributed as dist
    store = _default_store() if store is None else store
    me = dist.get_rank() if rank is None else rank
    store.set(f"rmlx_kv/departed/{me}", "1")


def exchange_migration_plan(mgr, send_ids: List[int], peer: int, group=None, *, store=None,
                            rank: Optional[int] = None, timeout_s: float = 60.0) -> Tuple[List[int], int]:
    """Tell `peer` how many blocks this rank sends and learn how many it sends
    here; allocate that many destination blocks from `mgr` (this rank's block
    manager).  Returns (recv_ids, n_peer_sends).

    This is the handshake that must complete before either rank calls
    ``KVPool.migrate``: it runs entirely on the host, through the key-value
    store of the process group (or `store`, with `rank` this rank's id), and
    every wait in it is bounded by `timeout_s`.  A peer that has left
    (``depart``) or does not answer by the deadline raises ``RmlxError`` with
    RMLX_E_TIMEOUT before anything is allocated or enqueued, so no NCCL
    transfer is ever posted toward a rank that will not post its half.
    Raises RMLX_E_EXHAUSTED, on both ranks, if either pool cannot hold the
    blocks coming to it (nothing is allocated then).

    Both ranks of a pair call this the same number of times in the same
    order; the n-th call of each is matched with the n-th call of the other
    (a per-process count of the pair's exchanges).  After an exchange has
    failed the two counts may disagree: treat the peer as gone, and pair a
    replacement process with this one only through a fresh store and a
    fresh process (or ``reset_plan_counts``).
    """
    import time
    import torch.distributed as dist
    from ._lib import RMLX_E_EXHAUSTED, RMLX_E_TIMEOUT, RmlxError
    store = _default_store() if store is None else store
    me = (dist.get_rank() if group is None else dist.get_global_rank(group, dist.get_rank(group))) \
        if rank is None else rank
    if peer == me:
        raise ValueError("a rank cannot migrate blocks to itself")
    epoch = _EPOCH.get((me, peer), 0)
    _EPOCH[(me, peer)] = epoch + 1
    deadline = time.monotonic() + timeout_s

    def post(phase, value):
        store.set(f"rmlx_kv/migrate/{me}->{peer}/{epoch}/{phase}", value)

    def hear(phase):
        key = f"rmlx_kv/migrate/{peer}->{me}/{epoch}/{phase}"
        while not store.check([key]):
            if store.check([f"rmlx_kv/departed/{peer}"]):
                raise RmlxError(RMLX_E_TIMEOUT, f"migration plan: rank {peer} has left the job")
            if time.monotonic() > deadline:
                raise RmlxError(RMLX_E_TIMEOUT, f"migration plan: rank {peer} did not answer within {timeout_s:g} s")
            time.sleep(0.005)
        v = store.get(key).decode()
        store.delete_key(key)  # this rank is its only reader
        return v

    # Phase 1: the block counts.  Phase 2: both sides confirm that they can
    # take what comes, so that neither posts its transfer while the other
    # has given up.
    post("count", str(len(send_ids)))
    n_in = int(hear("count"))
    fits = n_in <= mgr.num_free_blocks()
    post("ready", "1" if fits else "0")
    peer_ready = hear("ready") == "1"
    if not fits:
        raise RmlxError(RMLX_E_EXHAUSTED, f"peer sends {n_in} blocks, only {mgr.num_free_blocks()} free here")
    if not peer_ready:
        raise RmlxError(RMLX_E_EXHAUSTED, f"rank {peer} cannot hold the {len(send_ids)} blocks this rank sends")
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
