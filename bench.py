#!/usr/bin/env python3
"""KV-cache step benchmark: paged append + per-layer paged gather.

Default workload (``--workload decode``): Llama-3.1-8B KV shape -- 32
layers, 8 KV heads, head_dim 128, block 16, bf16; batch 64, context lengths
uniform in [512, 4096]; every step appends one token per sequence to every
layer, then gathers every layer's K/V for all sequences through the block
tables.  Block tables are drawn from a seeded permutation of a pool sized
1.25x the blocks in use.

``--workload prefix``: prefix caching with eviction -- 512 requests, token
ids uniform over 128256; 60% start with one of 8 shared 1024-token prefixes
plus a unique 64-512-token suffix, 40% are unique with 256-2048 tokens;
per-block chain hashes on the GPU, then admission through the block manager
and the prefix cache with LRU eviction under a pool of 60% of the distinct
blocks the requests need.  Metric: admissions per second.

``--workload quant8`` / ``quant4``: the same layers and heads, batch 128,
contexts uniform in [1024, 8192], K/V N(0,1) with 1% outliers x8, stored as
8-bit / 4-bit group-affine codes (group 64 along head_dim, fp16 scale and
zero per group): quantise-on-append, dequantise-on-gather to bf16.

With N GPUs (one process per GPU under torchrun) the 8 KV heads are split
over the GPUs: each rank owns 8/N heads of every block and runs the same
step on them; there is no collective in the step.

Metric: algorithmic HBM GB/s of the step (bytes the append and the gathers
must read and write), whole job; also microseconds per step.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]
                  [--workload decode|quant8|quant4]
"""
import argparse
import contextlib
import json
import os
import shutil
import subprocess
import sys
import tempfile
import time
from dataclasses import dataclass

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "rmlx-serve_b200"))

F32, F16, BF16 = 0, 1, 2


@dataclass
class Workload:
    name: str
    metric: str
    desc: str
    seed: int
    layers: int = 32
    heads: int = 8
    head_dim: int = 128
    block: int = 16
    batch: int = 64
    ctx_lo: int = 512
    ctx_hi: int = 4096
    bits: int = 0
    group: int = 64
    meta: int = F16
    outliers: float = 0.0
    attn_g: int = 0  # > 0: decode attention with this many query heads per KV head instead of the gather
    dtype: int = BF16
    lens: tuple = ()  # fixed prompt lengths (instead of uniform in [ctx_lo, ctx_hi])
    min_blocks: int = 0  # pool at least this large
    graph: bool = False  # latency-bound: the timed steps are captured once in a CUDA graph and replayed

    # bytes of one token's rows of the local heads
    def in_row(self, h):
        return h * self.head_dim * 2

    def stored_row(self, h):
        return h * self.head_dim * self.bits // 8 if self.bits else self.in_row(h)

    def meta_row(self, h):
        return h * (self.head_dim // self.group) * 2 * (2 if self.meta == F16 else 4) if self.bits else 0

    @property
    def kernel(self):
        if self.attn_g:
            return "paged_decode_attn_codes_kernel" if self.bits else "paged_decode_attn_rows_kernel"
        return "gather_dequant_r1_kernel" if self.bits else "gather_rows_kernel"

    @property
    def profile(self):
        return f"{self.kernel}_llama8b_{self.name}.txt"


WORKLOADS = {
    "decode": Workload(
        "decode", "KV append+gather HBM GB/s (decode step, Llama-3.1-8B KV shape)",
        "decode-step KV ops: 32 layers x 8 KV heads x 128, block 16, bf16, batch 64, ctx U[512,4096], "
        "append 1 token/seq/layer then paged gather of every layer", seed=0x5EED + 2),
    "quant8": Workload(
        "quant8", "KV quant-append + dequant-gather HBM GB/s (8-bit, Llama-3.1-8B KV shape)",
        "quantised KV store: 32 layers x 8 KV heads x 128, block 16, 8-bit codes, group 64, fp16 scale/zero, "
        "batch 128, ctx U[1024,8192], 1% outliers x8; quantise-on-append 1 token/seq/layer, then "
        "dequantise-on-gather (bf16) of every layer", seed=0x5EED + 3, batch=128, ctx_lo=1024, ctx_hi=8192, bits=8,
        outliers=0.01),
    "quant4": Workload(
        "quant4", "KV quant-append + dequant-gather HBM GB/s (4-bit, Llama-3.1-8B KV shape)",
        "quantised KV store: 32 layers x 8 KV heads x 128, block 16, 4-bit codes (2 per byte), group 64, fp16 "
        "scale/zero, batch 128, ctx U[1024,8192], 1% outliers x8; quantise-on-append 1 token/seq/layer, then "
        "dequantise-on-gather (bf16) of every layer", seed=0x5EED + 3, batch=128, ctx_lo=1024, ctx_hi=8192, bits=4,
        outliers=0.01),
    "config1": Workload(
        "config1", "KV append+gather HBM GB/s (1 layer, 4 sequences; latency-bound: see us_per_step)",
        "the reference's own case: 1 layer x 8 KV heads x 128, block 16, fp16, pool 256 blocks, 4 sequences with "
        "prompts 37/128/255/512, 1 token appended per sequence per step, then the gather of the layer",
        seed=0x5EED + 1, layers=1, batch=4, lens=(37, 128, 255, 512), dtype=F16, min_blocks=256, graph=True),
    "attn": Workload(
        "attn", "KV append + paged decode attention HBM GB/s (decode step, Llama-3.1-8B shape)",
        "decode step with attention reading the pool in place: 32 layers x 8 KV heads x 128, block 16, bf16, "
        "32 query heads (4 per KV head), batch 64, ctx U[512,4096]; append 1 token/seq/layer, then paged decode "
        "attention of every layer (no gathered copy)", seed=0x5EED + 2, attn_g=4),
    "attn8": Workload(
        "attn8", "KV quant-append + paged decode attention over 8-bit codes HBM GB/s (decode step, Llama-3.1-8B shape)",
        "decode step with attention reading an 8-bit pool in place: 32 layers x 8 KV heads x 128, block 16, 8-bit "
        "codes, group 64, fp16 scale/zero, 32 query heads (4 per KV head), batch 64, ctx U[512,4096]; quantise-on-"
        "append 1 token/seq/layer, then paged decode attention of every layer (codes fed to the tensor cores)",
        seed=0x5EED + 2, attn_g=4, bits=8),
    "attn4": Workload(
        "attn4", "KV quant-append + paged decode attention over 4-bit codes HBM GB/s (decode step, Llama-3.1-8B shape)",
        "decode step with attention reading a 4-bit pool in place: 32 layers x 8 KV heads x 128, block 16, 4-bit "
        "codes (2 per byte), group 64, fp16 scale/zero, 32 query heads (4 per KV head), batch 64, ctx U[512,4096]; "
        "quantise-on-append 1 token/seq/layer, then paged decode attention of every layer (codes fed to the tensor "
        "cores)", seed=0x5EED + 2, attn_g=4, bits=4),
}


PREFIX_METRIC = "prefix-cache admissions/s (512 requests, 8 shared 1024-token prefixes, LRU at 60% budget)"
PREFIX_DESC = ("prefix caching + eviction: 512 requests, vocab 128256; 60% = one of 8 shared 1024-token prefixes + "
               "unique 64-512-token suffix, 40% unique 256-2048 tokens; chain hash per 16-token block + parent on the "
               "GPU; refcounted reuse; LRU eviction with a pool of 60% of the distinct blocks needed")


def prefix_requests(seed, n_req=512, n_prefix=8, prefix_len=1024, suffix=(64, 512), unique=(256, 2048),
                    vocab=128256, shared=0.6):
    """Seeded requests of the prefix-caching workload: (tokens, cu_tokens)."""
    rng = np.random.default_rng(seed)
    prefixes = [rng.integers(0, vocab, size=prefix_len, dtype=np.uint32) for _ in range(n_prefix)]
    reqs = []
    for _ in range(n_req):
        if rng.random() < shared:
            p = prefixes[int(rng.integers(n_prefix))]
            reqs.append(np.concatenate([p, rng.integers(0, vocab, size=int(rng.integers(suffix[0], suffix[1] + 1)),
                                                        dtype=np.uint32)]))
        else:
            reqs.append(rng.integers(0, vocab, size=int(rng.integers(unique[0], unique[1] + 1)), dtype=np.uint32))
    cu = np.zeros(n_req + 1, dtype=np.int64)
    cu[1:] = np.cumsum([len(r) for r in reqs])
    return np.concatenate(reqs).astype(np.uint32), cu


def prefix_pool_size(toks, cu, cub, hashes, block=16, impl=None):
    """60% of the distinct blocks the requests need (a dry run with room for
    all).  `impl`: the module whose block manager, prefix cache and
    admission run it (the product's by default; the reference arm passes the
    oracle)."""
    if impl is None:
        import rmlx_kv as impl
    m, p = impl.PagedCacheManager(block, int(cub[-1])), impl.PrefixCacheManager(int(cub[-1]))
    st = impl.prefix_admit(m, p, toks, cu, hashes, cub)[2]
    return int(np.ceil(0.6 * st["new_blocks"]))


def run_prefix(args, rank, world):
    """GPU chain hash of every block + native admission; rank 0 only (the
    prefix cache is replicated on every rank, so the work does not shard)."""
    if rank != 0:
        return
    import torch
    import rmlx_kv
    torch.cuda.set_device(0)
    seed = 0x5EED + 4
    toks, cu = prefix_requests(seed)
    nb = (np.diff(cu) + 15) // 16
    cub = np.zeros(len(cu), dtype=np.int64)
    cub[1:] = np.cumsum(nb)
    n_req = len(cu) - 1
    stream = torch.cuda.current_stream()
    d_t, d_cu, d_cub = (torch.from_numpy(toks.view(np.int32)).cuda(), torch.from_numpy(cu).cuda(),
                        torch.from_numpy(cub).cuda())
    d_h = torch.empty(int(cub[-1]), dtype=torch.int64, device="cuda")
    for _ in range(args.warmup):
        rmlx_kv.hash_block_chains(d_t, d_cu, None, n_req, 16, d_cub, d_h)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        rmlx_kv.hash_block_chains(d_t, d_cu, None, n_req, 16, d_cub, d_h)
    e1.record(stream)
    torch.cuda.synchronize()
    hash_ms = e0.elapsed_time(e1) / args.steps
    hashes = d_h.cpu().numpy().view(np.uint64)
    pool = prefix_pool_size(toks, cu, cub, hashes)
    admit_s, stats = [], None
    for i in range(args.warmup + args.steps):
        m, p = rmlx_kv.PagedCacheManager(16, pool), rmlx_kv.PrefixCacheManager(pool)
        t0 = time.perf_counter()
        _, ev, stats = rmlx_kv.prefix_admit(m, p, toks, cu, hashes, cub)
        if i >= args.warmup:
            admit_s.append(time.perf_counter() - t0)
        hit = p.hit_rate()
    admit = float(np.median(admit_s))
    # e2e: tokens H2D, hash kernel, hashes D2H, admission -- per batch of requests
    pin_t = torch.from_numpy(toks.view(np.int32)).pin_memory()
    pin_h = torch.empty(int(cub[-1]), dtype=torch.int64, pin_memory=True)
    e2e = []
    for i in range(args.warmup + args.steps):
        m, p = rmlx_kv.PagedCacheManager(16, pool), rmlx_kv.PrefixCacheManager(pool)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        d_t.copy_(pin_t, non_blocking=True)
        rmlx_kv.hash_block_chains(d_t, d_cu, None, n_req, 16, d_cub, d_h)
        pin_h.copy_(d_h, non_blocking=True)
        torch.cuda.synchronize()
        rmlx_kv.prefix_admit(m, p, toks, cu, pin_h.numpy().view(np.uint64), cub)
        if i >= args.warmup:
            e2e.append(time.perf_counter() - t0)
    e2e_s = float(np.median(e2e))
    cpu = None
    if not args.no_cpu_baseline:
        gbs, sec = prefix_cpu(toks, cu, cub, pool)
        cpu = {"value": round(n_req / sec, 2), "unit": "admissions/s", "cores": 1, "kind": "port",
               "sample": "oracle chain hash + admission of all 512 requests (single thread, as the reference)"}
    hash_bytes = 4 * len(toks) + 8 * int(cub[-1])
    print(json.dumps({
        "metric": PREFIX_METRIC, "value": round(n_req / (hash_ms * 1e-3 + admit), 2), "unit": "admissions/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(hash_ms + admit * 1e3, 4), "us_per_admission": round(admit / n_req * 1e6, 2),
        "higher_is_better": True, "scaling": "replicas", "vs_baseline": None, "dtype": "u32", "data": "synthetic",
        "config": {"workload": PREFIX_DESC, "requests": n_req, "tokens": int(len(toks)), "blocks": int(cub[-1]),
                   "pool_blocks": pool},
        "hash_kernel": {"ms": round(hash_ms, 4), "gbs": round(hash_bytes / (hash_ms * 1e-3) / 1e9, 2)},
        "admission": {"ms": round(admit * 1e3, 3), **stats, "hit_rate": round(hit, 4)},
        "e2e": {"value": round(n_req / e2e_s, 2), "unit": "admissions/s", "h2d_bytes_per_step": 4 * len(toks),
                "d2h_bytes_per_step": 8 * int(cub[-1])},
        "gpu_launches": args.steps, "cpu_baseline": cpu,
    }), flush=True)


def prefix_cpu(toks, cu, cub, pool):
    """The oracle's chain hash and admission (the reference's O(trie) LRU scan)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as orc
    t0 = time.perf_counter()
    hashes, _ = orc.hash_chains(toks, cu, np.zeros(len(cu) - 1, dtype=np.uint64), 16)
    m, p = orc.PagedCacheManager(16, pool), orc.PrefixCacheManager(pool)
    orc.prefix_admit(m, p, toks, cu, hashes, cub)
    sec = time.perf_counter() - t0
    return 0.0, sec


def run_prefix_reference(args, world):
    """--impl reference for the prefix workload: the oracle's chain hash and
    admission of all 512 requests per step, single thread (as the
    reference), W warm-up and K timed steps; the pool size comes from the
    oracle's own dry run.  The product library is not loaded."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as orc
    toks, cu = prefix_requests(0x5EED + 4)
    cub = np.zeros(len(cu), dtype=np.int64)
    cub[1:] = np.cumsum((np.diff(cu) + 15) // 16)
    hashes, _ = orc.hash_chains(toks, cu, np.zeros(len(cu) - 1, dtype=np.uint64), 16)
    pool = prefix_pool_size(toks, cu, cub, hashes, impl=orc)
    secs = []
    for i in range(args.warmup + args.steps):
        _, sec = prefix_cpu(toks, cu, cub, pool)
        if i >= args.warmup:
            secs.append(sec)
    sec = float(np.median(secs))
    v = round((len(cu) - 1) / sec, 2)
    print(json.dumps({"impl": "reference", "metric": PREFIX_METRIC, "value": v, "unit": "admissions/s",
                      "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                      "ms_per_step": round(sec * 1e3, 2), "higher_is_better": True, "scaling": "replicas",
                      "vs_baseline": None, "dtype": "u32", "data": "synthetic",
                      "config": {"workload": PREFIX_DESC, "requests": len(cu) - 1, "tokens": int(len(toks)),
                                 "blocks": int(cub[-1]), "pool_blocks": pool},
                      "cpu_baseline": {"value": v, "unit": "admissions/s", "cores": 1, "kind": "port",
                                       "sample": "oracle chain hash + admission of all 512 requests per step, "
                                                 "single thread"},
                      "e2e": {"value": v, "unit": "admissions/s", "h2d_bytes_per_step": 0,
                              "d2h_bytes_per_step": 0}}), flush=True)


L70_METRIC = "KV fork/COW + append + gather HBM GB/s (Llama-3-70B KV shape, KV heads sharded over GPUs)"
L70_DESC = ("Llama-3-70B KV: 80 layers x 8 KV heads x 128, block 16, bf16; batch 256, ctx log-uniform [2048,32768]; "
            "per step 5% of sequences fork (copy-on-write of the shared partial tail), 1 token appended per "
            "sequence, then a paged gather of every resident layer; 2% of blocks migrated between rank pairs "
            "over NVLink (NCCL), timed separately")


def l70_plan(seed, steps, batch=256, block=16, fork_frac=0.05):
    """Host plan of the fork/append steps, identical on every rank, made by
    the library's batch planner (rmlx_kv_batch_*): per step a few sequences
    are replaced by forks of others (remove, then fork into the freed row),
    then each sequence appends one token (copy-on-write of a shared tail).
    Returns per step the copy pairs, slots, block table and lengths after
    the append; the pool size; the block manager and the planner (which
    holds the sequences' block references while it lives)."""
    import rmlx_kv
    from rmlx_kv.batch import KVBatch
    rng = np.random.default_rng(seed)
    lens = np.exp(rng.uniform(np.log(2048), np.log(32768), size=batch)).astype(np.int64)
    nfork = max(1, int(round(fork_frac * batch)))
    # in use at the start, plus at most one new block per sequence and one
    # copy-on-write block per fork each step
    num_blocks = int(((lens + block - 1) // block).sum()) + (steps + 1) * (batch + nfork)
    mgr = rmlx_kv.PagedCacheManager(block, num_blocks)
    mgr.free_n(rng.permutation(mgr.allocate_n(num_blocks)))  # scatter the free list
    planner = KVBatch(mgr, None, batch)
    uids = np.arange(1, batch + 1, dtype=np.uint64)  # uids[row]
    for r in range(batch):
        row, _, _ = planner.add(int(uids[r]), rng.integers(0, 128256, size=int(lens[r]), dtype=np.uint32))
        assert row == r
    next_uid = batch + 1
    plan = []
    for _ in range(steps):
        idx = rng.permutation(batch)
        for parent, child in zip(idx[:nfork], idx[nfork:2 * nfork]):
            planner.remove(int(uids[child]))
            row = planner.fork(int(uids[parent]), next_uid)
            assert row == child
            uids[child] = next_uid
            next_uid += 1
        slots, cow_src, cow_dst = planner.step(uids, rng.integers(0, 128256, size=batch, dtype=np.uint32))
        bt, ln = planner.tables()
        plan.append(dict(cow_src=cow_src.copy(), cow_dst=cow_dst.copy(), slots=slots.copy(), bt=bt.copy(),
                         lens=ln.copy()))
    return plan, num_blocks, mgr, planner


def run_llama70b(args, rank, world):
    import datetime
    import torch
    import rmlx_kv
    from rmlx_kv import _lib
    from rmlx_kv import distributed as rd
    dist = None
    if world > 1:
        import torch.distributed as dist
        torch.cuda.set_device(env_int("LOCAL_RANK", 0))
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
                                device_id=torch.device("cuda", torch.cuda.current_device()))
    else:
        torch.cuda.set_device(0)
    dev = torch.cuda.current_device()
    LAYERS_FULL, HEADS, D, BS, B = 80, 8, 128, 16, 256
    w = Workload("llama70b", L70_METRIC, L70_DESC, 0x5EED + 5, layers=LAYERS_FULL, batch=B, bits=args.bits)
    off, H = rd.shard_heads(HEADS, world, rank)
    W, K = args.warmup, args.steps
    plan, num_blocks, mgr, planner = l70_plan(w.seed, W + K)
    qkw = dict(quant_bits=w.bits, group_size=w.group, meta_dtype=w.meta) if w.bits else {}
    probe = rmlx_kv.KVPool(1, H, D, BS, 1, dtype=rmlx_kv.BF16, head_offset=off, device=dev, **qkw)
    tile = probe.layout.tile_bytes
    probe.close()
    per_layer = num_blocks * 2 * H * tile
    budget = 130e9
    L = int(min(LAYERS_FULL, max(1, budget // per_layer)))
    if args.layers:
        L = min(L, args.layers)
    pool = rmlx_kv.KVPool(L, H, D, BS, num_blocks, dtype=rmlx_kv.BF16, head_offset=off, device=dev, **qkw)
    h, lib = pool.handle, _lib.lib
    gen = torch.Generator(device="cuda").manual_seed(0x5EED + 5 + rank)
    if w.bits:
        # random codes with small positive scales: any byte pattern is a valid code
        view = torch.as_tensor(DevView(pool.layout.base, pool.layout.bytes), device="cuda")
        for o in range(0, view.numel(), 1 << 30):
            view[o:o + (1 << 30)].random_(0, 256, generator=gen)
        meta = pool.layout.meta_row_bytes
        if meta:
            tiles = view.view(-1, pool.layout.tile_bytes)
            codes = BS * pool.layout.row_bytes
            tiles[:, codes:codes + BS * meta].view(torch.float16).uniform_(0.001, 0.05, generator=gen)
    else:
        view = torch.as_tensor(DevView(pool.layout.base, pool.layout.bytes), device="cuda").view(torch.bfloat16)
        for o in range(0, view.numel(), 1 << 28):
            view[o:o + (1 << 28)].normal_(generator=gen)
    del view
    stream = torch.cuda.current_stream()
    sp = stream.cuda_stream
    new_k = torch.randn((W + K, L, B, H, D), device="cuda", dtype=torch.bfloat16, generator=gen)
    new_v = torch.randn_like(new_k)
    dev_plan = []
    for st in plan:
        dev_plan.append(dict(src=torch.from_numpy(st["cow_src"]).cuda() if len(st["cow_src"]) else None,
                             dst=torch.from_numpy(st["cow_dst"]).cuda() if len(st["cow_dst"]) else None,
                             n=len(st["cow_src"]), slots=torch.from_numpy(st["slots"]).cuda(),
                             bt=torch.from_numpy(st["bt"]).cuda(), width=st["bt"].shape[1],
                             lens=torch.from_numpy(st["lens"]).cuda()))
    max_tok = max(int(st["lens"].sum()) for st in plan)
    out_k = torch.empty(max_tok * H * D, device="cuda", dtype=torch.bfloat16)
    out_v = torch.empty_like(out_k)
    ts, ls = H * D, B * H * D

    def launch(si, ev=None):
        d = dev_plan[si]
        rc = 0
        if d["n"]:
            rc |= lib.rmlx_kv_copy_blocks(h, d["src"].data_ptr(), d["dst"].data_ptr(), d["n"], sp)
        rc |= lib.rmlx_kv_append(h, 0, L, new_k[si].data_ptr(), new_v[si].data_ptr(), ls, ts, D,
                                 d["slots"].data_ptr(), B, sp)
        if ev is not None:
            ev[0].record(stream)
        for layer in range(L):
            rc |= lib.rmlx_kv_gather(h, layer, d["bt"].data_ptr(), d["width"], d["lens"].data_ptr(), B,
                                     out_k.data_ptr(), out_v.data_ptr(), sp)
        if ev is not None:
            ev[1].record(stream)
        return rc

    def barrier():
        if dist is not None:
            dist.barrier()

    def max_over_ranks(x):
        if dist is None:
            return x
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    rc = 0
    for si in range(W):
        rc |= launch(si)
    if rc or pool.check():
        raise SystemExit("error during warm-up")
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(K)]
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = Clocks(dev)
    clocks.start()
    barrier()
    torch.cuda.synchronize()
    e0.record(stream)
    for i in range(K):
        rc |= launch(W + i, evs[i])
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    clk = clocks.stop()
    ms = max_over_ranks(e0.elapsed_time(e1))
    if rc or pool.check():
        raise SystemExit("error in the timed region")
    tot, cows, gbytes = 0, 0, []
    for i in range(K):
        st = plan[W + i]
        n = len(st["cow_src"])
        cows += n
        append, g1 = step_bytes(w, st["lens"].astype(np.int64), H, L)
        tot += 2 * n * L * 2 * H * tile + append + L * g1  # copy-on-write: read + write each tile
        gbytes.append(g1)
    tot *= world
    value = tot / (ms * 1e-3) / 1e9
    g_ms = float(np.mean([a.elapsed_time(b) for a, b in evs])) / L
    achieved = float(np.mean(gbytes)) / (g_ms * 1e-3) / 1e9
    mig = None
    if world > 1:
        # 2% of the blocks in use, exchanged with the paired rank into free blocks
        peer = rank ^ 1 if (rank ^ 1) < world else rank
        uid = rd.share_nccl_id()
        comm = rmlx_kv.NcclComm(world, uid, rank, dev, timeout_ms=120000)
        if peer != rank:
            in_use = [b for b in range(num_blocks) if mgr.ref_count(b) > 0]
            nmov = max(1, int(0.02 * len(in_use)))
            send = torch.tensor(in_use[:nmov], dtype=torch.int32, device="cuda")
            recv_ids, n_in = rd.exchange_migration_plan(mgr, in_use[:nmov], peer)
            recv = torch.tensor(recv_ids, dtype=torch.int32, device="cuda")
            bb = pool.layout.block_bytes
            s_st = torch.empty(nmov * bb, dtype=torch.uint8, device="cuda")
            r_st = torch.empty(n_in * bb, dtype=torch.uint8, device="cuda")
            m0, m1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            pool.migrate(comm, peer, send, nmov, s_st, recv, n_in, r_st)  # warm-up
            comm.wait()
            barrier()
            m0.record(stream)
            pool.migrate(comm, peer, send, nmov, s_st, recv, n_in, r_st)
            m1.record(stream)
            comm.wait()
            mig_ms = max_over_ranks(m0.elapsed_time(m1))
            moved = (nmov + n_in) * bb
            mig = {"blocks_per_rank": nmov, "bytes_per_rank": moved, "ms": round(mig_ms, 3),
                   "gbs_per_rank": round(moved / (mig_ms * 1e-3) / 1e9, 1),
                   "gbs_per_direction": round(nmov * bb / (mig_ms * 1e-3) / 1e9, 1),
                   "what": "pack + ncclSend/ncclRecv + unpack, rank pairs (r, r^1) exchanging at once; "
                           "bytes_per_rank counts sent + received, gbs_per_direction the sent bytes alone"}
        comm.close()
    if rank == 0:
        peak, kind = measured_peak()
        print(json.dumps({
            "metric": L70_METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": K,
            "warmup": W, "ms_per_step": round(ms / K, 4), "us_per_step_80_layers": round(ms / K * 1e3 * 80 / L, 1),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": f"u{w.bits}+bf16" if w.bits else "bf16", "data": "synthetic",
            "config": {"workload": L70_DESC + (f"; {w.bits}-bit codes, group 64, fp16 scale/zero" if w.bits else ""),
                       "batch": B, "inputs": "larger than L2 (each layer gather reads GBs)", "layers": 80, "layers_resident": L, "kv_heads_per_gpu": H,
                       "pool_blocks": num_blocks, "cow_copies_per_step": round(cows / K, 2),
                       "note": "fewer than 80 layers are resident when the 80-layer pool does not fit in "
                               "130 GB; GB/s counts the bytes of the resident layers"},
            "roofline": {"bound": "hbm", "kernel": w.kernel, "achieved": round(achieved, 1), "peak": peak,
                         "peak_kind": kind, "unit": "GB/s", "frac": round(achieved / peak, 4),
                         "launch_ms": round(g_ms, 4)},
            "migration": mig, "gpu_launches": K * (2 + L), "clocks": clk,
        }), flush=True)
    pool.close()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def env_int(name, default):
    try:
        return int(os.environ.get(name, default))
    except ValueError:
        return default


def measured_peak():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def profile_traffic(name, algorithmic_bytes):
    """DRAM bytes (read + write) per launch from the kernel's committed ncu
    summary, scaled from the captured launch to this launch by algorithmic
    bytes (the traffic of a gather grows in proportion to the rows moved)."""
    vals = {}
    try:
        for line in open(os.path.join(ROOT, "profiles", name)):
            if line.startswith("traffic_"):
                k, v = line.split(":", 1)
                vals[k.strip()] = float(v)
    except OSError:
        return None
    if "traffic_bytes_per_launch" not in vals or "traffic_algorithmic_bytes" not in vals:
        return None
    return round(vals["traffic_bytes_per_launch"] / vals["traffic_algorithmic_bytes"] * algorithmic_bytes)


def _allocate_n(mgr, n):
    if hasattr(mgr, "allocate_n"):
        return np.asarray(mgr.allocate_n(n))
    return np.array([mgr.allocate() for _ in range(n)], dtype=np.int64)


def _free_n(mgr, ids):
    if hasattr(mgr, "free_n"):
        return mgr.free_n(ids)
    for b in ids:
        mgr.free(int(b))


def make_workload(w, steps_total, manager=None):
    """Seeded lengths, block tables and per-step slot mappings for
    `steps_total` steps.  `manager(block_size, num_blocks)` makes the block
    manager that hands out the blocks: the product's by default; the
    reference arm passes the oracle's, which gives the same tables (FIFO
    reuse of the same permuted free list)."""
    if manager is None:
        import rmlx_kv
        manager = rmlx_kv.PagedCacheManager
    rng = np.random.default_rng(w.seed)
    if w.lens:
        lens0 = np.array(w.lens, dtype=np.int64)
    else:
        lens0 = rng.integers(w.ctx_lo, w.ctx_hi + 1, size=w.batch).astype(np.int64)
    need = (lens0 + steps_total + w.block - 1) // w.block
    num_blocks = max(int(np.ceil(1.25 * need.sum())), w.min_blocks)
    mgr = manager(w.block, num_blocks)
    # Make the free list a seeded permutation of the pool: allocate all, free
    # in permuted order (FIFO reuse hands them out in that order).
    _free_n(mgr, rng.permutation(_allocate_n(mgr, num_blocks)))
    bt = np.zeros((w.batch, int(need.max())), dtype=np.int32)
    nblk = np.zeros(w.batch, dtype=np.int64)
    for s in range(w.batch):
        n0 = (int(lens0[s]) + w.block - 1) // w.block
        bt[s, :n0] = _allocate_n(mgr, n0)
        nblk[s] = n0
    slots = np.zeros((steps_total, w.batch), dtype=np.int32)
    for st in range(steps_total):
        for s in range(w.batch):
            p = int(lens0[s]) + st
            while p // w.block >= nblk[s]:
                bt[s, nblk[s]] = _allocate_n(mgr, 1)[0]
                nblk[s] += 1
            slots[st, s] = bt[s, p // w.block] * w.block + p % w.block
    return dict(lens0=lens0, bt=bt, slots=slots, num_blocks=num_blocks, mgr=mgr)


def step_bytes(w, lens, heads, layers=None, batch=None):
    """Algorithmic bytes of one step.  Append: read every new row, write its
    stored form (and its scale/zero).  Gather of one layer: read every stored
    row (and meta) of every sequence, write it out in the input type; plus
    the block-table entries and lengths the gather reads.  K and V both.
    `batch`: sequences appended (default: the workload's batch)."""
    layers = w.layers if layers is None else layers
    batch = w.batch if batch is None else batch
    i, s, m = w.in_row(heads), w.stored_row(heads), w.meta_row(heads)
    append = 2 * batch * layers * (i + s + m)
    blocks = int(((lens + w.block - 1) // w.block).sum())
    if w.attn_g:
        # attention reads every stored row once (no gathered copy written),
        # plus the queries it reads and the outputs it writes
        qo = 2 * batch * w.attn_g * i
        return append, 2 * int(lens.sum()) * (s + m) + 4 * blocks + 4 * batch + qo
    gather_one = 2 * int(lens.sum()) * (s + m + i) + 4 * blocks + 4 * batch
    return append, gather_one


class DevView:
    """Zero-copy torch view of raw device memory (for filling the pool)."""

    def __init__(self, ptr, nbytes):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False),
                                         "version": 3}


class Clocks:
    """nvidia-smi sampling of SM clocks and throttle reasons during timing."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap,clocks.mem")

    def __init__(self, device):
        self.device = device
        self.proc = None
        self.path = None

    def start(self):
        if not shutil.which("nvidia-smi"):
            return
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        self.f = open(self.path, "w")
        self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.device}", f"--query-gpu={self.Q}",
                                      "--format=csv,noheader,nounits", "-lms", "100"], stdout=self.f,
                                     stderr=subprocess.DEVNULL)
        time.sleep(0.3)

    def stop(self):
        if not self.proc:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.f.close()
        sm, mem, mx, reasons = [], [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in open(self.path):
            p = [x.strip() for x in ln.split(",")]
            if len(p) < 9:
                continue
            try:
                sm.append(float(p[1]))
                mx = max(mx, float(p[2]))
            except ValueError:
                continue
            for n, v in zip(names, p[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
            if len(p) > 9:
                try:
                    mem.append(float(p[9]))
                except ValueError:
                    pass
        os.unlink(self.path)
        self.proc = None
        if not sm:
            return None
        out = {"sm_mhz": float(np.median(sm)), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}
        if mem:
            out["mem_mhz"] = float(np.median(mem))
            out["mem_mhz_min"] = float(min(mem))
        return out


def cpu_sample(w, steps, warm, threads, lens0, bt, slots, num_blocks, seqs=None):
    """The oracle (CPU restatement of the reference) on the host cores: one
    layer of every step -- append 1 token per sequence (quantising it for the
    quantised workloads), then the full gather (dequantise) of that layer,
    sequences split over `threads`.  `seqs`: only the first `seqs` sequences
    (a bounded sample for slow legs).  Returns (GB/s, seconds per sample)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as orc
    H, D = w.heads, w.head_dim
    nseq = w.batch if seqs is None else min(seqs, w.batch)
    g = orc.Geo(1, H, D, w.block, num_blocks, 2, bits=w.bits, group_size=w.group,
                meta_bytes=2 if w.meta == F16 else 4)
    rng = np.random.default_rng(w.seed + 1)
    pool = rng.integers(0, 256, size=g.pool_bytes(), dtype=np.uint8)
    if w.bits:
        # sane scale/zero so that the CPU does not run on random subnormals
        tb = g.tile_bytes()
        rb, mrb = D * w.bits // 8, (D // w.group) * 2 * (2 if w.meta == F16 else 4)
        tiles = pool.reshape(-1, tb)
        meta = np.tile(np.array([0.02, -2.5], dtype=np.float16 if w.meta == F16 else np.float32),
                       (tiles.shape[0], w.block * (D // w.group)))
        tiles[:, w.block * rb:w.block * rb + w.block * mrb] = meta.view(np.uint8)
    bt = np.ascontiguousarray(bt[:nseq])
    tot = int((lens0[:nseq] + slots.shape[0]).sum()) * H * D
    ok = np.empty(tot, dtype=np.uint16)
    ov = np.empty(tot, dtype=np.uint16)
    kin = orc.f32_to_dtype(rng.standard_normal((nseq, H, D), dtype=np.float32), orc.BF16)
    total_bytes, t_total = 0, 0.0
    for st in range(warm + steps):
        lens = (lens0[:nseq] + st + 1).astype(np.int32)
        sl = slots[st, :nseq].astype(np.int64)
        t0 = time.perf_counter()
        if w.bits:
            orc.paged_append_quant(pool, g, 0, 1, kin, kin, orc.BF16, 0, H * D, D, sl)
            orc.paged_gather_dequant(pool, g, 0, bt, bt.shape[1], lens, ok, ov, orc.BF16, threads=threads)
        else:
            orc.paged_append(pool, g, 0, 1, kin, kin, 0, H * D, D, sl)
            orc.paged_gather(pool, g, 0, bt, bt.shape[1], lens, ok, ov, threads=threads)
        dt = time.perf_counter() - t0
        if st >= warm:
            a, gth = step_bytes(w, lens.astype(np.int64), H, layers=1, batch=nseq)
            total_bytes += a + gth
            t_total += dt
    return total_bytes / t_total / 1e9, t_total / steps


def single_thread_leg(w, steps_available):
    """Sequences and steps of the single-thread oracle leg: the reference is
    single-threaded (`&mut self` throughout paged_cache.rs), so this is the
    reference-faithful CPU figure; bounded to about 10-20 s of work (one
    step of the workload's steps is its warm-up)."""
    seqs, steps = (max(1, w.batch // 16), 3) if w.bits else (w.batch, 10)
    return seqs, max(1, min(steps, steps_available - 1))


def run_reference(args, w, rank, world):
    """--impl reference: the reference's CPU path on the host cores.  The
    Rust reference cannot be built in this image, so this is the oracle
    (its C++ restatement, oracle/): block tables from the oracle's block
    manager, the oracle's row-copy append and gather.  The product library
    is not loaded.  The driver's --steps/--warmup are honoured, each step a
    sample of one of the layers at the full batch; the pool is sized from
    the same warm-up + timed steps as the product's arm, so the config is
    the same."""
    if rank != 0:
        return
    if w.attn_g:
        print(json.dumps({"impl": "reference", "unavailable": "the reference has no attention of its own on this "
                          "path (it runs inside the external rmlx-nn Metal layer cache)"}))
        return
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as orc
    threads = os.cpu_count() or 1
    K, W = args.steps, args.warmup
    wl = make_workload(w, W + K, manager=orc.PagedCacheManager)
    gbs, sec = cpu_sample(w, K, W, threads, wl["lens0"], wl["bt"], wl["slots"], wl["num_blocks"])
    s1, k1 = single_thread_leg(w, W + K)
    gbs1, _ = cpu_sample(w, k1, 1, 1, wl["lens0"], wl["bt"], wl["slots"], wl["num_blocks"], seqs=s1)
    sample = (f"oracle append + gather, 1 of {w.layers} layers per step at the full batch {w.batch}, "
              f"{K} timed steps after {W} warm-up, {threads} threads (sequences split over them); GB/s is per "
              f"sampled byte, ms_per_step the sampled layer's time x{w.layers}")
    print(json.dumps({
        "impl": "reference", "metric": w.metric, "value": round(gbs, 2), "unit": "GB/s", "n_gpus": world,
        "steps": K, "warmup": W, "ms_per_step": round(sec * w.layers * 1e3, 3), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f16" if w.dtype == F16 else "bf16", "data": "synthetic",
        "config": config_of(w, w.heads // world, wl["num_blocks"], world,
                            not w.attn_g and not w.bits and args.gather == "layers"),
        "cpu_baseline": {"value": round(gbs, 2), "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": sample},
        "single_thread": {"value": round(gbs1, 2), "unit": "GB/s", "cores": 1, "kind": "port",
                          "sample": f"the reference-faithful figure (the reference is single-threaded): oracle "
                                    f"append + gather, 1 layer per step, first {s1} of {w.batch} sequences, "
                                    f"{k1} timed steps after 1 warm-up, 1 thread"},
        "e2e": {"value": round(gbs, 2), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def config_of(w, H, num_blocks, world, multi=None):
    c = {"workload": w.desc, "batch": w.batch, "layers": w.layers, "kv_heads": w.heads, "kv_heads_per_gpu": H,
         "head_dim": w.head_dim, "block_size": w.block, "pool_blocks": num_blocks, "sharding": f"kv-head x{world}",
         "l2": ("inputs larger than L2: each gather launch moves >0.1 GB, no flush" if not w.lens else
                "L2-resident (a few MB per step): a latency-bound case, reported as us_per_step")}
    if w.bits:
        c.update({"quant_bits": w.bits, "group_size": w.group, "meta": "f16" if w.meta == F16 else "f32",
                  "outliers": w.outliers})
    if multi is not None and not w.attn_g:
        c["gather"] = ("one rmlx_kv_gather_layers launch per step for all layers, each layer into its own output"
                       if multi else "one rmlx_kv_gather launch per layer, into a reused per-layer output")
    if w.graph:
        c["launch"] = ("device-timed steps replayed from one CUDA graph of the K steps' library launches; "
                       "the e2e loop runs the planner and stages each step's inputs on the host, then replays "
                       "its buffer set's captured step (H2D copies, C-ABI launches, status read)")
    return c


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="decode", choices=sorted(WORKLOADS) + ["prefix", "llama70b"])
    ap.add_argument("--bits", type=int, default=0, choices=[0, 8],
                    help="llama70b workload: 0 = bf16 pool, 8 = 8-bit codes")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--kv-heads", type=int, default=None,
                    help="override the workload's KV heads (e.g. 1: one GPU's shard of an 8-GPU run)")
    ap.add_argument("--layers", type=int, default=None,
                    help="layers in the pool (profiling runs only; a gather moves the same bytes per layer)")
    ap.add_argument("--quick", action="store_true", help="device-timed loop only (profiling runs)")
    ap.add_argument("--gather", default="layers", choices=["layers", "per-layer"],
                    help="plain pools: one multi-layer gather launch per step, or one launch per layer")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    rank, world = env_int("RANK", 0), env_int("WORLD_SIZE", 1)
    if args.workload == "prefix":
        if args.impl == "reference":
            if rank == 0:
                run_prefix_reference(args, world)
            return
        return run_prefix(args, rank, world)
    if args.workload == "llama70b":
        if args.impl == "reference":
            if rank == 0:
                print(json.dumps({"impl": "reference", "unavailable": "the fork/COW/migration workload has no CPU "
                                  "path in the reference (its caches are single-sequence CPU f32)"}))
            return
        return run_llama70b(args, rank, world)
    w = WORKLOADS[args.workload]
    if args.layers:
        w.layers = args.layers
    if args.kv_heads:
        w.heads = args.kv_heads

    rank, world, local = env_int("RANK", 0), env_int("WORLD_SIZE", 1), env_int("LOCAL_RANK", 0)
    if args.impl == "reference":
        return run_reference(args, w, rank, world)

    import torch
    import rmlx_kv
    from rmlx_kv import _lib

    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    dev = torch.cuda.current_device()
    if w.heads % world:
        raise SystemExit(f"{w.heads} KV heads do not split over {world} GPUs")
    H, D, L, B, BS = w.heads // world, w.head_dim, w.layers, w.batch, w.block
    W, K = args.warmup, args.steps
    wl = make_workload(w, W + K)
    lens0, bt, slots, num_blocks = wl["lens0"], wl["bt"], wl["slots"], wl["num_blocks"]

    tdt = torch.float16 if w.dtype == F16 else torch.bfloat16
    pool = rmlx_kv.KVPool(L, H, D, BS, num_blocks, dtype=w.dtype, quant_bits=w.bits, group_size=w.group,
                          meta_dtype=w.meta, head_offset=rank * H, device=dev)
    h = pool.handle
    lib = _lib.lib
    stream = torch.cuda.current_stream()
    sp = stream.cuda_stream
    gen = torch.Generator(device="cuda").manual_seed(w.seed + rank)

    def rand_rows(shape):
        x = torch.randn(shape, device="cuda", dtype=torch.float32, generator=gen)
        if w.outliers:
            x = torch.where(torch.rand(shape, device="cuda", generator=gen) < w.outliers, x * 8.0, x)
        return x.to(tdt)

    ts, hs = H * D, D
    bt_d = torch.from_numpy(bt).cuda()
    if w.bits:
        # Prompt K/V ~ N(0,1) (+outliers) quantised into the pool through the
        # product's own quantise-on-append, a chunk of tokens at a time.
        pos = [(s, p) for s in range(B) for p in range(int(lens0[s]))]
        chunk = 4096
        for o in range(0, len(pos), chunk):
            part = pos[o:o + chunk]
            T = len(part)
            sl = torch.tensor([bt[s, p // BS] * BS + p % BS for s, p in part], dtype=torch.int32, device="cuda")
            kk, vv = rand_rows((L, T, H, D)), rand_rows((L, T, H, D))
            _lib.check(lib.rmlx_kv_append(h, 0, L, kk.data_ptr(), vv.data_ptr(), T * ts, ts, hs, sl.data_ptr(), T,
                                          sp))
        del kk, vv
    else:
        view = torch.as_tensor(DevView(pool.layout.base, pool.layout.bytes), device="cuda").view(tdt)
        step = 1 << 28
        for o in range(0, view.numel(), step):
            view[o:o + step].normal_(generator=gen)
        del view

    kv_shape = (W + K, L, B, H, D)
    new_k, new_v = rand_rows(kv_shape), rand_rows(kv_shape)
    slots_d = torch.from_numpy(slots).cuda()
    lens_steps = np.stack([(lens0 + s + 1).astype(np.int32) for s in range(W + K)])
    lens_d = torch.from_numpy(lens_steps).cuda()
    G = w.attn_g
    # one rmlx_kv_gather_layers launch per step for all layers, each into its
    # own output, instead of one rmlx_kv_gather per layer into a reused buffer
    multi = not G and not w.bits and args.gather == "layers"
    if G:
        # per-layer queries of the step, attention output, split workspace
        q_d = rand_rows((L, B, H * G, D))
        att_out = torch.empty((B, H * G, D), device="cuda", dtype=tdt)
        ws_bytes = pool.attention_workspace_size(G, B, int(lens_steps[-1].sum()))
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
        scale = 1.0 / float(np.sqrt(D))
        out_k = out_v = None
    else:
        out_k = torch.empty(int(lens_steps[-1].sum()) * H * D * (L if multi else 1), device="cuda", dtype=tdt)
        out_v = torch.empty_like(out_k)
    layer_elems = int(lens_steps[-1].sum()) * H * D  # each layer's gathered K (or V), elements
    ls = B * H * D

    def launch_step(s, sp=sp, gathers_only=False):
        """The append, then the gather of every layer (or its attention)."""
        rc = 0
        if not gathers_only:
            rc = lib.rmlx_kv_append(h, 0, L, new_k[s].data_ptr(), new_v[s].data_ptr(), ls, ts, hs,
                                    slots_d[s].data_ptr(), B, sp)
        if multi:
            rc |= lib.rmlx_kv_gather_layers(h, 0, L, bt_d.data_ptr(), bt.shape[1], lens_d[s].data_ptr(), B,
                                            out_k.data_ptr(), out_v.data_ptr(), layer_elems, sp)
        for layer in range(0 if multi else L):
            if G:
                rc |= lib.rmlx_kv_decode_attention(h, layer, q_d[layer].data_ptr(), G, bt_d.data_ptr(), bt.shape[1],
                                                   lens_d[s].data_ptr(), B, scale, att_out.data_ptr(),
                                                   ws.data_ptr(), ws_bytes, sp)
            else:
                rc |= lib.rmlx_kv_gather(h, layer, bt_d.data_ptr(), bt.shape[1], lens_d[s].data_ptr(), B,
                                         out_k.data_ptr(), out_v.data_ptr(), sp)
        return rc

    def barrier():
        if dist is not None:
            dist.barrier()

    def max_over_ranks(x):
        if dist is None:
            return x
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    rc = 0
    for s in range(W):
        rc |= launch_step(s)
    if rc or pool.check() != 0:
        raise SystemExit("launch or device-side validation error during warm-up")

    clocks = Clocks(dev)
    clocks.start()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))]
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if w.graph:
        # Latency-bound steps: issuing them from Python leaves the GPU idle
        # between launches, so the K steps' library launches are captured
        # once (same arguments as the loop below would pass) and replayed.
        g_steps, g_gathers = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_steps, capture_error_mode="relaxed"):
            cap = torch.cuda.current_stream().cuda_stream
            for i in range(K):
                rc |= launch_step(W + i, sp=cap)
        with torch.cuda.graph(g_gathers, capture_error_mode="relaxed"):
            cap = torch.cuda.current_stream().cuda_stream
            for i in range(K):
                rc |= launch_step(W + i, sp=cap, gathers_only=True)
        torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    e0.record(stream)
    if w.graph:
        g_steps.replay()
    else:
        for i in range(K):
            rc |= launch_step(W + i)
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    elapsed_ms = max_over_ranks(e0.elapsed_time(e1))
    # The gather (or attention) launch time: the K steps' gathers alone, back
    # to back after the timed region, events around them all (events between
    # launches inside the timed steps would stop consecutive kernels from
    # overlapping their launch with the previous one's tail).
    ev[0][0].record(stream)
    if w.graph:
        g_gathers.replay()
    else:
        for i in range(K):
            rc |= launch_step(W + i, gathers_only=True)
    ev[0][1].record(stream)
    torch.cuda.synchronize()
    gather_ms = [ev[0][0].elapsed_time(ev[0][1]) / (K * (1 if multi else L))]
    if rc or pool.check() != 0:
        raise SystemExit("launch or device-side validation error in the timed region")

    # Algorithmic bytes over the timed steps, all ranks.
    tot_bytes, gather_bytes = 0, []
    for i in range(K):
        a, g1 = step_bytes(w, lens_steps[W + i].astype(np.int64), H)
        tot_bytes += a + L * g1
        gather_bytes += [L * g1] if multi else [g1] * L
    tot_bytes *= world
    value = tot_bytes / (elapsed_ms * 1e-3) / 1e9
    ms_per_step = elapsed_ms / K
    g_bytes = float(np.mean(gather_bytes))
    g_ms = float(np.mean(gather_ms))

    # The append alone: the K timed steps' appends again, back to back,
    # captured once in a CUDA graph and replayed between CUDA events (issued
    # one by one from Python, each launch would wait for the host: the
    # append's device time is a few microseconds); average launch = span / K.
    a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    g_app = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g_app, capture_error_mode="relaxed"):
        cap = torch.cuda.current_stream().cuda_stream
        for i in range(K):
            rc |= lib.rmlx_kv_append(h, 0, L, new_k[W + i].data_ptr(), new_v[W + i].data_ptr(), ls, ts, hs,
                                     slots_d[W + i].data_ptr(), B, cap)
    torch.cuda.synchronize()
    a0.record(stream)
    g_app.replay()
    a1.record(stream)
    torch.cuda.synchronize()
    del g_app
    if rc or pool.check() != 0:
        raise SystemExit("launch or device-side validation error in the append timing")
    append_ms = a0.elapsed_time(a1) / K
    append_bytes = step_bytes(w, lens_steps[W].astype(np.int64), H)[0]

    if args.quick:
        clocks.stop()
        if rank == 0:
            print(json.dumps({"quick": True, "workload": w.name, "layers": L, "ms_per_step": round(ms_per_step, 4),
                              "append_ms": round(append_ms, 4),
                              "append_gbs": round(append_bytes / (append_ms * 1e-3) / 1e9, 1),
                              "value": round(value, 2), "gather_launch_ms": round(g_ms, 4),
                              "gather_gbs": round(g_bytes / (g_ms * 1e-3) / 1e9, 1)}))
        pool.close()
        if dist is not None:
            dist.destroy_process_group()
        return

    # ---- e2e: the same steps through the public API with host buffers ----
    # Per step: the batch planner (rmlx_kv_batch_step) gives each sequence's
    # slot, new blocks and block tables; H2D of the new K/V (pinned), slots,
    # block tables and lengths; the append and the per-layer gathers (or
    # attention); a D2H read of the step's status word.  The gathered K/V stay
    # in HBM for the attention that consumes them.  Inputs are double-
    # buffered: step i + 1's copies run on a copy stream while step i
    # computes, and each step's status word is read asynchronously
    # (rmlx_kv_pool_status_async) and checked on the host two steps later,
    # when its buffers are reused.
    from rmlx_kv.batch import KVBatch
    mgr = rmlx_kv.PagedCacheManager(BS, num_blocks)
    rng = np.random.default_rng(w.seed + 7)
    mgr.free_n(rng.permutation(mgr.allocate_n(num_blocks)))
    planner = KVBatch(mgr, None, B)
    uids = np.arange(1, B + 1, dtype=np.uint64)
    for s in range(B):  # prompts as long as the sequences are when the timed steps start
        planner.add(int(uids[s]), rng.integers(0, 128256, size=int(lens0[s]) + W, dtype=np.uint32))
    step_tokens = rng.integers(0, 128256, size=(K, B), dtype=np.uint32)
    host_bt = np.zeros_like(bt)
    pin_k = torch.empty((K, L, B, H, D), dtype=tdt, pin_memory=True)
    pin_v = torch.empty_like(pin_k, pin_memory=True)
    pin_k.copy_(new_k[W:W + K].cpu())
    pin_v.copy_(new_v[W:W + K].cpu())
    # two sets of host (pinned) and device buffers, used by alternate steps
    pin_bt = [torch.from_numpy(host_bt.copy()).pin_memory() for _ in range(2)]
    pin_slots = [torch.empty(B, dtype=torch.int32, pin_memory=True) for _ in range(2)]
    pin_lens = [torch.empty(B, dtype=torch.int32, pin_memory=True) for _ in range(2)]
    pin_status = [torch.zeros(1, dtype=torch.int32, pin_memory=True) for _ in range(2)]
    dk = [torch.empty((L, B, H, D), device="cuda", dtype=tdt) for _ in range(2)]
    dv = [torch.empty_like(dk[0]) for _ in range(2)]
    d_slots = [torch.empty(B, dtype=torch.int32, device="cuda") for _ in range(2)]
    d_lens = [torch.empty(B, dtype=torch.int32, device="cuda") for _ in range(2)]
    d_bt = [torch.empty_like(bt_d) for _ in range(2)]
    h2d = 2 * dk[0].numel() * 2 + 2 * B * 4 + host_bt.nbytes
    if G:
        # the step's queries for every layer come from the host too
        pin_q = q_d.cpu().pin_memory()
        dq = [torch.empty_like(q_d) for _ in range(2)]
        h2d += q_d.numel() * 2
    copy_stream = torch.cuda.Stream()
    copied = [torch.cuda.Event() for _ in range(2)]
    done = [torch.cuda.Event() for _ in range(2)]

    def status_seen(b):
        """The status word of the step that last used buffer set b (its
        event has completed)."""
        done[b].synchronize()
        return int(pin_status[b][0])

    def step_ops(b, sp_b, src_k, src_v, copies_on=None):
        """The step's H2D copies into buffer set b, its library launches and
        its asynchronous status read.  copies_on: a side stream for the
        copies (the compute stream waits for them)."""
        nonlocal rc
        ctx = torch.cuda.stream(copies_on) if copies_on is not None else contextlib.nullcontext()
        with ctx:
            dk[b].copy_(src_k, non_blocking=True)
            dv[b].copy_(src_v, non_blocking=True)
            d_slots[b].copy_(pin_slots[b], non_blocking=True)
            d_lens[b].copy_(pin_lens[b], non_blocking=True)
            d_bt[b].copy_(pin_bt[b], non_blocking=True)
            if G:
                dq[b].copy_(pin_q, non_blocking=True)
            if copies_on is not None:
                copied[b].record(copies_on)
        if copies_on is not None:
            torch.cuda.current_stream().wait_event(copied[b])
        rc |= lib.rmlx_kv_append(h, 0, L, dk[b].data_ptr(), dv[b].data_ptr(), ls, ts, hs, d_slots[b].data_ptr(), B,
                                 sp_b)
        if multi:
            rc |= lib.rmlx_kv_gather_layers(h, 0, L, d_bt[b].data_ptr(), bt.shape[1], d_lens[b].data_ptr(), B,
                                            out_k.data_ptr(), out_v.data_ptr(), layer_elems, sp_b)
        for layer in range(0 if multi else L):
            if G:
                rc |= lib.rmlx_kv_decode_attention(h, layer, dq[b][layer].data_ptr(), G, d_bt[b].data_ptr(),
                                                   bt.shape[1], d_lens[b].data_ptr(), B, scale, att_out.data_ptr(),
                                                   ws.data_ptr(), ws_bytes, sp_b)
            else:
                rc |= lib.rmlx_kv_gather(h, layer, d_bt[b].data_ptr(), bt.shape[1], d_lens[b].data_ptr(), B,
                                         out_k.data_ptr(), out_v.data_ptr(), sp_b)
        # the step's status word, read back to the host without waiting
        rc |= lib.rmlx_kv_pool_status_async(h, pin_status[b].data_ptr(), sp_b)

    graphs = None
    if w.graph:
        # Latency-bound steps: each buffer set's step (copies from fixed
        # pinned staging, launches, status read) captured once and replayed;
        # the host stages each step's K/V and the planner's tables into the
        # set's pinned buffers before the replay.
        stage_k = [torch.empty_like(pin_k[0]).pin_memory() for _ in range(2)]
        stage_v = [torch.empty_like(pin_k[0]).pin_memory() for _ in range(2)]
        graphs = []
        for b in range(2):
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr, capture_error_mode="relaxed"):
                step_ops(b, torch.cuda.current_stream().cuda_stream, stage_k[b], stage_v[b])
            graphs.append(gr)
        torch.cuda.synchronize()

    barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for i in range(K):
        b = i % 2
        slots_i, _, _ = planner.step(uids, step_tokens[i])
        tb, ln = planner.tables()
        if i >= 2 and status_seen(b):  # step i - 2 finished with set b: its status word
            raise SystemExit("device-side validation error in the e2e loop")
        pin_slots[b].numpy()[:] = slots_i
        pin_lens[b].numpy()[:] = ln
        pin_bt[b].numpy()[:, :tb.shape[1]] = tb
        if graphs is not None:
            stage_k[b].copy_(pin_k[i])
            stage_v[b].copy_(pin_v[i])
            graphs[b].replay()
        else:
            step_ops(b, sp, pin_k[i], pin_v[i], copies_on=copy_stream)
        done[b].record(stream)
        if rc:
            raise SystemExit("launch error in the e2e loop")
    if any(status_seen(b) for b in range(min(K, 2))):
        raise SystemExit("device-side validation error in the e2e loop")
    torch.cuda.synchronize()
    barrier()
    e2e_s = max_over_ranks(time.perf_counter() - t0)
    if pool.check():
        raise SystemExit("device-side validation error in the e2e loop")
    clk = clocks.stop()
    e2e_value = tot_bytes / e2e_s / 1e9

    peak, peak_kind = measured_peak()
    achieved = g_bytes / (g_ms * 1e-3) / 1e9
    traffic = profile_traffic(w.profile, g_bytes)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and not G:
        threads = os.cpu_count() or 1
        steps = min(8 if not w.bits else 3, W + K - 1)
        gbs, _ = cpu_sample(w, steps, 1, threads, lens0, bt, slots, num_blocks)
        s1, k1 = single_thread_leg(w, W + K)
        gbs1, _ = cpu_sample(w, k1, 1, 1, lens0, bt, slots, num_blocks, seqs=s1)
        cpu = {"value": round(gbs, 2), "unit": "GB/s", "cores": threads, "kind": "port",
               "sample": f"oracle append+gather, 1 of {L} layers per step, batch {B}, {steps} timed steps, "
                         f"sequences split over {threads} threads",
               "single_thread": {"value": round(gbs1, 2), "unit": "GB/s", "cores": 1,
                                 "sample": f"reference-faithful (the reference is single-threaded): 1 layer per "
                                           f"step, first {s1} of {B} sequences, {k1} timed steps, 1 thread"}}

    if rank == 0:
        print(json.dumps({
            "metric": w.metric, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": K,
            "warmup": W, "ms_per_step": round(ms_per_step, 4), "us_per_step": round(ms_per_step * 1e3, 1),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "f16" if w.dtype == F16 else "bf16",
            "data": "synthetic", "config": config_of(w, H, num_blocks, world, multi),
            "roofline": {"bound": "hbm", "kernel": w.kernel, "achieved": round(achieved, 1), "peak": peak,
                         "peak_kind": peak_kind, "unit": "GB/s", "frac": round(achieved / peak, 4),
                         "frac_of_8000_nominal": round(achieved / 8000.0, 4), "traffic": traffic,
                         "algorithmic_bytes_per_launch": int(g_bytes), "launch_ms": round(g_ms, 4)},
            "append": {"kernel": "append_quant_kernel" if w.bits else "append_rows_kernel",
                       "algorithmic_bytes_per_launch": int(append_bytes), "launch_ms": round(append_ms, 4),
                       "achieved": round(append_bytes / (append_ms * 1e-3) / 1e9, 1),
                       "frac": round(append_bytes / (append_ms * 1e-3) / 1e9 / peak, 4),
                       "what": "the timed steps' appends again, back to back from one CUDA graph (all layers, "
                               "one launch per step)"},
            "e2e": {"value": round(e2e_value, 2), "unit": "GB/s", "h2d_bytes_per_step": int(h2d),
                    "d2h_bytes_per_step": 4, "ms_per_step": round(e2e_s / K * 1e3, 4)},
            "gpu_launches": K * (1 + (1 if multi else (2 if G else 1) * L)),
            "cpu_baseline": cpu,
            "clocks": clk,
        }), flush=True)
    planner.close()
    pool.close()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
