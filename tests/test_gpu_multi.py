"""Two-GPU block migration over NCCL (pack -> ncclSend/ncclRecv -> unpack).

Runs as two spawned child processes, one per GPU, and is skipped when fewer
than two GPUs are visible.  Each rank fills its pool with bytes derived
from its rank, the ranks agree on the migration plan through the host
handshake (a TCP key-value store), exchange blocks in both directions, and
every migrated block must arrive bit-identical; blocks that were not
targets must be untouched.

Then rank 1 leaves between steps: its migration has completed and its
communicator is closed, so nothing of it is in flight.  Rank 0's next plan
exchange must fail on the host with RMLX_E_TIMEOUT, promptly, before it
allocates or enqueues anything, and its GPU context must stay usable.  No
test here posts an NCCL transfer toward a rank that will not post its half.
"""
import multiprocessing as mp
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

L, H, D, BS, N = 2, 2, 128, 16, 64
SEND = {0: [3, 7, 9, 63], 1: [1, 2]}     # blocks each rank sends
RECV = {0: [20, 21], 1: [10, 11, 12, 0]}  # where each rank puts what it receives


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _pool_bytes(rank, nbytes):
    return np.random.default_rng(1000 + rank).integers(0, 256, size=nbytes, dtype=np.uint8)


def _worker(rank, uid_q, res_q, port, left_q):
    try:
        import datetime
        import sys
        import time
        root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
        sys.path.insert(0, os.path.join(root, "rmlx-serve_b200"))
        import torch
        import torch.distributed as dist
        import rmlx_kv
        from rmlx_kv import _lib
        from rmlx_kv import distributed as rd
        store = dist.TCPStore("127.0.0.1", port, 2, rank == 0, timeout=datetime.timedelta(seconds=60),
                              wait_for_workers=False)
        torch.cuda.set_device(rank)
        if rank == 0:
            uid = rmlx_kv.NcclComm.unique_id()
            uid_q.put(uid)
        else:
            uid = uid_q.get(timeout=60)
        pool = rmlx_kv.KVPool(L, H, D, BS, N, dtype=rmlx_kv.BF16, device=rank)
        bb = pool.layout.block_bytes
        mine = _pool_bytes(rank, pool.layout.bytes)
        pool.write(mine)
        comm = rmlx_kv.NcclComm(2, uid, rank, rank, timeout_ms=60000)
        peer = 1 - rank
        # the plan: counts through the host handshake (the destination ids
        # are fixed here instead of allocated, so the bytes are predictable)
        mgr = rmlx_kv.PagedCacheManager(BS, N)
        recv_ids, n_in = rd.exchange_migration_plan(mgr, SEND[rank], peer, store=store, rank=rank, timeout_s=60)
        assert n_in == len(RECV[rank]) == len(recv_ids)
        send = torch.tensor(SEND[rank], dtype=torch.int32, device="cuda")
        recv = torch.tensor(RECV[rank], dtype=torch.int32, device="cuda")
        s_st = torch.empty(len(SEND[rank]) * bb, dtype=torch.uint8, device="cuda")
        r_st = torch.empty(len(RECV[rank]) * bb, dtype=torch.uint8, device="cuda")
        pool.migrate(comm, peer, send, len(SEND[rank]), s_st, recv, len(RECV[rank]), r_st)
        comm.wait(timeout_ms=60000)
        got = pool.read()
        theirs = _pool_bytes(peer, pool.layout.bytes)
        want = mine.copy()
        for src, dst in zip(SEND[peer], RECV[rank]):
            want[dst * bb:(dst + 1) * bb] = theirs[src * bb:(src + 1) * bb]
        ok = bool(np.array_equal(got, want)) and pool.check() == 0
        comm.close()
        if rank == 1:
            # leaves between steps: its transfer is complete, its
            # communicator closed; the departure is announced on the host
            rd.depart(store=store, rank=1)
            left_q.put(1)
            pool.close()
            res_q.put((rank, ok, ""))
            return
        left_q.get(timeout=120)
        t0 = time.monotonic()
        code, free0 = None, mgr.num_free_blocks()
        try:
            rd.exchange_migration_plan(mgr, [5], peer, store=store, rank=rank, timeout_s=30)
        except rmlx_kv.RmlxError as e:
            code = e.status
        waited = time.monotonic() - t0
        # the context is still usable: a fresh append + gather round trip
        x = torch.arange(H * D, dtype=torch.float32, device="cuda").to(torch.bfloat16).reshape(1, 1, H, D)
        slot = torch.tensor([3 * BS], dtype=torch.int32, device="cuda")
        pool.append(x, x, slot, 1)
        ok_t = torch.empty(H * D, dtype=torch.bfloat16, device="cuda")
        ov_t = torch.empty_like(ok_t)
        pool.gather(0, torch.tensor([[3]], dtype=torch.int32, device="cuda"), 1,
                    torch.tensor([1], dtype=torch.int32, device="cuda"), 1, ok_t, ov_t)
        torch.cuda.synchronize()
        usable = bool(torch.equal(ok_t, x.reshape(-1))) and bool(torch.equal(ov_t, x.reshape(-1)))
        usable = usable and pool.check() == 0
        pool.close()
        fast = waited < 10.0  # the departure mark, not the 30 s deadline
        untouched = mgr.num_free_blocks() == free0
        ok = ok and code == _lib.RMLX_E_TIMEOUT and fast and usable and untouched
        res_q.put((rank, ok, f"code={code} waited={waited:.2f}s usable={usable} untouched={untouched}"))
    except Exception as e:  # reported to the parent, which fails the test
        res_q.put((rank, False, repr(e)))


def test_migrate_blocks_between_two_gpus_then_peer_leaves():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    uid_q, res_q, left_q = ctx.Queue(), ctx.Queue(), ctx.Queue()
    port = _free_port()
    env_keep = os.environ.get("NCCL_NVLS_ENABLE")
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    try:
        procs = [ctx.Process(target=_worker, args=(r, uid_q, res_q, port, left_q)) for r in range(2)]
        for p in procs:
            p.start()
        results = [res_q.get(timeout=240) for _ in range(2)]
        for p in procs:
            p.join(timeout=60)
    finally:
        if env_keep is None:
            os.environ.pop("NCCL_NVLS_ENABLE", None)
        else:
            os.environ["NCCL_NVLS_ENABLE"] = env_keep
        for p in procs:
            if p.is_alive():
                p.kill()
    for rank, ok, err in sorted(results):
        assert ok, f"rank {rank}: {err or 'migrated blocks differ'}"
