"""The N>1 host path on CPU: two gloo ranks (world size 2, 127.0.0.1).

Covers what runs on the host when the pool is sharded over GPUs: every
rank builds bit-identical replicated block tables and slot mappings from
the seeded workload, the head shards tile the heads exactly once, per-rank
algorithmic bytes sum to the single-GPU bytes, the max-over-ranks timing
reduction, the NCCL-id broadcast path (with a stand-in id), and the
pairwise migration-plan exchange with destination allocation and block
table remapping.
"""
import hashlib
import os
import socket
import sys

import numpy as np
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, out):
    sys.path.insert(0, os.path.join(ROOT, "rmlx-serve_b200"))
    sys.path.insert(0, ROOT)
    import datetime
    import torch
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        import bench
        import rmlx_kv
        from rmlx_kv import distributed as rd
        w = bench.WORKLOADS["decode"]
        wl = bench.make_workload(w, 8)
        digest = hashlib.sha256(wl["bt"].tobytes() + wl["slots"].tobytes()).hexdigest()
        digests = [None] * world
        dist.all_gather_object(digests, digest)
        off, per = rd.shard_heads(w.heads, world, rank)
        shards = [None] * world
        dist.all_gather_object(shards, (off, per))
        lens = (wl["lens0"] + 1).astype(np.int64)
        a1, g1 = bench.step_bytes(w, lens, w.heads)
        ar, gr = bench.step_bytes(w, lens, per)
        t = torch.tensor([float(rank + 1)], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        # NCCL-id broadcast path with a stand-in payload (no NCCL on CPU)
        buf = torch.zeros(128, dtype=torch.uint8)
        if rank == 0:
            buf[:] = torch.arange(128, dtype=torch.uint8)
        dist.broadcast(buf, src=0)
        # migration plan: rank 0 sends 5 blocks, rank 1 sends 2
        mgr = rmlx_kv.PagedCacheManager(16, 64)
        held = mgr.allocate_n(20).tolist()
        send = held[:5] if rank == 0 else held[:2]
        recv_ids, n_in = rd.exchange_migration_plan(mgr, send, 1 - rank)
        bt = np.array([held[:10], held[10:20]], dtype=np.int32)
        bt2 = rd.remap_block_table(bt, send, list(range(100, 100 + len(send))))
        table_reads = 4 * int(((lens + w.block - 1) // w.block).sum()) + 4 * w.batch
        out.put((rank, dict(digests=digests, shards=shards, bytes=(a1, g1, ar, gr, table_reads),
                            tmax=float(t.item()),
                            buf=bytes(buf.numpy().tobytes()), n_in=n_in, recv=recv_ids,
                            free=mgr.num_free_blocks(), bt_changed=int((bt2 != bt).sum()), nsend=len(send))))
    except Exception as e:
        out.put((rank, {"error": repr(e)}))
    finally:
        dist.destroy_process_group()


def test_two_rank_host_path():
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, out)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(out.get(timeout=240) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    for r in (0, 1):
        assert "error" not in res[r], res[r]
    a, b = res[0], res[1]
    assert a["digests"][0] == a["digests"][1] == b["digests"][0]
    assert sorted(a["shards"]) == [(0, 4), (4, 4)]
    a1, g1, ar, gr, tr = a["bytes"]
    assert 2 * ar == a1
    # gather bytes: the K/V rows split exactly over the ranks; every rank
    # reads the block tables and lengths itself
    assert 2 * gr - g1 == tr
    assert a["tmax"] == b["tmax"] == 2.0
    assert a["buf"] == b["buf"] == bytes(range(128))
    assert a["n_in"] == 2 and b["n_in"] == 5
    assert len(a["recv"]) == 2 and len(b["recv"]) == 5
    assert a["free"] == 64 - 20 - 2 and b["free"] == 64 - 20 - 5
    assert a["bt_changed"] == 5 and b["bt_changed"] == 2


def _handshake_worker(rank, world, port, out):
    """Failure paths of the migration-plan handshake, all on the host."""
    sys.path.insert(0, os.path.join(ROOT, "rmlx-serve_b200"))
    import datetime
    import time
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    res = {}
    try:
        import rmlx_kv
        from rmlx_kv import _lib
        from rmlx_kv import distributed as rd
        # (1) the receiver cannot hold what comes: both ranks fail, neither allocates
        mgr = rmlx_kv.PagedCacheManager(16, 8 if rank == 1 else 64)
        mgr.allocate_n(4)
        free0 = mgr.num_free_blocks()
        try:
            rd.exchange_migration_plan(mgr, list(range(6)) if rank == 0 else [0], 1 - rank, timeout_s=30)
            res["exhausted"] = None
        except rmlx_kv.RmlxError as e:
            res["exhausted"] = e.status
        res["untouched"] = mgr.num_free_blocks() == free0
        dist.barrier()
        # (2) a peer that stays up but never answers: the deadline
        if rank == 0:
            t0 = time.monotonic()
            try:
                rd.exchange_migration_plan(mgr, [1], 1, timeout_s=1.0)
                res["silent"] = None
            except rmlx_kv.RmlxError as e:
                res["silent"] = e.status
            res["silent_s"] = time.monotonic() - t0
        dist.barrier()
        # (3) a peer that leaves between steps: found at once through its mark
        if rank == 1:
            rd.depart()
        dist.barrier()
        if rank == 0:
            t0 = time.monotonic()
            try:
                rd.exchange_migration_plan(mgr, [1], 1, timeout_s=30)
                res["left"] = None
            except rmlx_kv.RmlxError as e:
                res["left"] = e.status
            res["left_s"] = time.monotonic() - t0
        res["timeout_code"] = _lib.RMLX_E_TIMEOUT
        res["exhausted_code"] = _lib.RMLX_E_EXHAUSTED
        out.put((rank, res))
    except Exception as e:
        out.put((rank, {"error": repr(e)}))
    finally:
        dist.barrier()
        dist.destroy_process_group()


def test_two_rank_plan_handshake_failures():
    """The migration-plan handshake fails on the host, on both ranks where
    both are present, with nothing allocated: a receiver that cannot hold
    the blocks (RMLX_E_EXHAUSTED on both), a peer that never answers
    (RMLX_E_TIMEOUT at the deadline) and a peer that left between steps
    (RMLX_E_TIMEOUT at once).  No GPU and no NCCL are involved."""
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_handshake_worker, args=(r, 2, port, out)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(out.get(timeout=240) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    for r in (0, 1):
        assert "error" not in res[r], res[r]
    a, b = res[0], res[1]
    assert a["exhausted"] == b["exhausted"] == a["exhausted_code"]
    assert a["untouched"] and b["untouched"]
    assert a["silent"] == a["timeout_code"] and 1.0 <= a["silent_s"] < 10.0
    assert a["left"] == a["timeout_code"] and a["left_s"] < 5.0
