"""Two-GPU block migration over NCCL (pack -> ncclSend/ncclRecv -> unpack).

Runs as two spawned child processes, one per GPU, and is skipped when fewer
than two GPUs are visible.  Each rank fills its pool with bytes derived
from its rank, the ranks exchange blocks in both directions, and every
migrated block must arrive bit-identical; blocks that were not targets
must be untouched.
"""
import multiprocessing as mp
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

L, H, D, BS, N = 2, 2, 128, 16, 64
SEND = {0: [3, 7, 9, 63], 1: [1, 2]}     # blocks each rank sends
RECV = {0: [20, 21], 1: [10, 11, 12, 0]}  # where each rank puts what it receives


def _pool_bytes(rank, nbytes):
    return np.random.default_rng(1000 + rank).integers(0, 256, size=nbytes, dtype=np.uint8)


def _worker(rank, uid_q, res_q):
    try:
        import sys
        root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
        sys.path.insert(0, os.path.join(root, "rmlx-serve_b200"))
        import torch
        import rmlx_kv
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
        pool.close()
        res_q.put((rank, ok, ""))
    except Exception as e:  # reported to the parent, which fails the test
        res_q.put((rank, False, repr(e)))


def test_migrate_blocks_between_two_gpus():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    uid_q, res_q = ctx.Queue(), ctx.Queue()
    env_keep = os.environ.get("NCCL_NVLS_ENABLE")
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    try:
        procs = [ctx.Process(target=_worker, args=(r, uid_q, res_q)) for r in range(2)]
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


def _timeout_worker(rank, uid_q, res_q, go_q):
    """Rank 1 joins the communicator and never posts its half of the
    migration; rank 0's migration must end with RMLX_E_TIMEOUT after its
    deadline (the communicator's 20 s timeout), the communicator aborted and
    the GPU context still usable."""
    try:
        import sys
        import time
        root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
        sys.path.insert(0, os.path.join(root, "rmlx-serve_b200"))
        import torch
        import rmlx_kv
        from rmlx_kv import _lib
        torch.cuda.set_device(rank)
        if rank == 0:
            uid = rmlx_kv.NcclComm.unique_id()
            uid_q.put(uid)
        else:
            uid = uid_q.get(timeout=60)
        pool = rmlx_kv.KVPool(L, H, D, BS, N, dtype=rmlx_kv.BF16, device=rank)
        comm = rmlx_kv.NcclComm(2, uid, rank, rank, timeout_ms=20000)
        if rank == 1:
            go_q.get(timeout=120)  # stays up, posting nothing, until rank 0 is done
            try:
                comm.close()  # the peer aborted: a bounded finalize, then destroy
            except Exception:
                pass
            pool.close()
            res_q.put((rank, True, ""))
            return
        bb = pool.layout.block_bytes
        send = torch.tensor([1, 2], dtype=torch.int32, device="cuda")
        recv = torch.tensor([5, 6], dtype=torch.int32, device="cuda")
        s_st = torch.empty(2 * bb, dtype=torch.uint8, device="cuda")
        r_st = torch.empty(2 * bb, dtype=torch.uint8, device="cuda")
        t0 = time.monotonic()
        code = None
        try:
            # Point-to-point connections are set up lazily with the peer, so the
            # group end itself cannot complete: migrate's bounded wait (the
            # communicator's timeout) ends with the abort; a queued transfer
            # would end in comm.wait instead.
            pool.migrate(comm, 1, send, 2, s_st, recv, 2, r_st)
            comm.wait(timeout_ms=1500)
        except rmlx_kv.RmlxError as e:
            code = e.status
        waited = time.monotonic() - t0
        go_q.put(1)
        # the context is still usable: a fresh append + gather round trip
        torch.cuda.synchronize()
        x = torch.arange(H * D, dtype=torch.float32, device="cuda").to(torch.bfloat16).reshape(1, 1, H, D)
        slot = torch.tensor([3 * BS], dtype=torch.int32, device="cuda")
        pool.append(x, x, slot, 1)
        ok_t = torch.empty(H * D, dtype=torch.bfloat16, device="cuda")
        ov_t = torch.empty_like(ok_t)
        pool.gather(0, torch.tensor([[3]], dtype=torch.int32, device="cuda"), 1,
                    torch.tensor([1], dtype=torch.int32, device="cuda"), 1, ok_t, ov_t)
        torch.cuda.synchronize()
        usable = bool(torch.equal(ok_t, x.reshape(-1))) and pool.check() == 0
        try:
            comm.close()
        except Exception:
            pass
        pool.close()
        ok = code == _lib.RMLX_E_TIMEOUT and 1.0 < waited < 60.0 and usable
        res_q.put((rank, ok, f"code={code} waited={waited:.2f}s usable={usable}"))
    except Exception as e:
        res_q.put((rank, False, repr(e)))


def test_migrate_times_out_when_peer_never_posts():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    uid_q, res_q, go_q = ctx.Queue(), ctx.Queue(), ctx.Queue()
    env_keep = os.environ.get("NCCL_NVLS_ENABLE")
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    try:
        procs = [ctx.Process(target=_timeout_worker, args=(r, uid_q, res_q, go_q)) for r in range(2)]
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
        assert ok, f"rank {rank}: {err}"
