"""GPU parity at the benchmarked shapes, through the launches the bench times.

Each test builds the bench's own seeded workload (block tables, slot
mappings, lengths) at full size, runs one decode step of one layer through
the same C-ABI calls the bench makes (rmlx_kv_copy_blocks, rmlx_kv_append,
rmlx_kv_gather / rmlx_kv_decode_attention, with the bench's strides), and
compares with the oracle on the same inputs:

* the decode step at the Llama-3.1-8B KV shape (batch 64, ctx U[512,4096],
  bf16): pool bytes after the append and the gathered K/V, byte for byte;
  and the multi-layer gather (rmlx_kv_gather_layers) at that shape;
* the quantised store (batch 128, ctx U[1024,8192], 8- and 4-bit codes,
  group 64, fp16 scale/zero, N(0,1) with 1% outliers x8): the prompts are
  quantised on append on both sides, then one decode step; codes, scales,
  zeros and the dequantised K/V byte for byte;
* the Llama-3-70B fork/copy-on-write step on one GPU's shard of an 8-GPU
  run (1 KV head, batch 256, ctx log-uniform [2048,32768], bf16 and 8-bit):
  two steps of forks, tile copies, appends and gathers, byte for byte;
* decode attention at the Llama-3.1-8B shape (4 query heads per KV head)
  over bf16, 8-bit and 4-bit pools against float64 attention over the
  oracle's rows, with the tolerances of test_gpu_attention.py.

The oracle runs its gathers on all host threads; the prompts of the
quantised store are quantised by the oracle in parallel chunks.
"""
import os
from concurrent.futures import ThreadPoolExecutor

import numpy as np
import pytest

import bench
import oracle as orc
import rmlx_kv
from rmlx_kv import _lib
from helpers import to_dev

pytestmark = pytest.mark.gpu

THREADS = os.cpu_count() or 1


def _sp():
    import torch
    return torch.cuda.current_stream().cuda_stream


def _view(pool, dtype):
    import torch
    return torch.as_tensor(bench.DevView(pool.layout.base, pool.layout.bytes), device="cuda").view(dtype)


def _same(got, want, what):
    assert got.shape == want.shape, what
    if not np.array_equal(got, want):
        bad = np.flatnonzero(got != want)
        raise AssertionError(f"{what}: {bad.size} of {want.size} differ, first at {bad[0]}")


def _slots_of_prompts(bt, lens0, bs):
    """Slots of every prompt token, sequence by sequence (the prefill)."""
    seq = np.repeat(np.arange(len(lens0)), lens0)
    pos = np.concatenate([np.arange(n) for n in lens0])
    return (bt[seq, pos // bs].astype(np.int64) * bs + pos % bs).astype(np.int32)


def _rand_rows(gen, shape, outliers):
    """The bench's rows: N(0,1) with optional outliers x8, as bf16 (device)."""
    import torch
    x = torch.randn(shape, device="cuda", dtype=torch.float32, generator=gen)
    if outliers:
        x = torch.where(torch.rand(shape, device="cuda", generator=gen) < outliers, x * 8.0, x)
    return x.to(torch.bfloat16)


def _host16(t):
    """A 16-bit device tensor's bits on the host (uint16)."""
    import torch
    return np.ascontiguousarray(t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16))


def _append_both(pool, host, g, k, v, slots, T, quant):
    """One rmlx_kv_append of T tokens (1 layer, [T][H][D] rows, the bench's
    strides) on the device and the oracle's append of the same rows."""
    lib = _lib.lib
    H, D = g.heads, g.hd
    sd = to_dev(slots)
    _lib.check(lib.rmlx_kv_append(pool.handle, 0, 1, k.data_ptr(), v.data_ptr(), T * H * D, H * D, D,
                                  sd.data_ptr(), T, _sp()))
    kh, vh = _host16(k), _host16(v)
    if quant:
        assert orc.paged_append_quant(host, g, 0, 1, kh, vh, orc.BF16, T * H * D, H * D, D, slots) == 0
    else:
        assert orc.paged_append(host, g, 0, 1, kh, vh, T * H * D, H * D, D, slots) == 0
    return sd


def _gather_both(pool, host, g, bt, lens, quant):
    """One rmlx_kv_gather of the layer on the device (bf16 out) and the
    oracle's gather (dequantise) on all host threads; returns both."""
    import torch
    lib = _lib.lib
    tot = int(lens.sum()) * g.heads * g.hd
    ok = torch.empty(max(tot, 8), dtype=torch.int16, device="cuda")
    ov = torch.empty_like(ok)
    btd, lnd = to_dev(bt), to_dev(lens.astype(np.int32))
    _lib.check(lib.rmlx_kv_gather(pool.handle, 0, btd.data_ptr(), bt.shape[1], lnd.data_ptr(), len(lens),
                                  ok.data_ptr(), ov.data_ptr(), _sp()))
    ek, ev = np.empty(tot, np.uint16), np.empty(tot, np.uint16)
    if quant:
        rc = orc.paged_gather_dequant(host, g, 0, bt, bt.shape[1], lens.astype(np.int32), ek, ev, orc.BF16,
                                      threads=THREADS)
    else:
        rc = orc.paged_gather(host, g, 0, bt, bt.shape[1], lens.astype(np.int32), ek, ev, threads=THREADS)
    assert rc == 0
    torch.cuda.synchronize()
    return (ok.cpu().numpy().view(np.uint16)[:tot], ov.cpu().numpy().view(np.uint16)[:tot]), (ek, ev)


def _prefill_quant(pool, host, g, bt, lens0, gen, outliers, chunk=16384):
    """The prompts, N(0,1) with outliers, quantised on append on the device
    and by the oracle (chunks in parallel: their slots are disjoint)."""
    import torch
    H, D = g.heads, g.hd
    slots = _slots_of_prompts(bt, lens0, g.bs)
    futs = []
    with ThreadPoolExecutor(max_workers=THREADS) as ex:
        for o in range(0, len(slots), chunk):
            sl = np.ascontiguousarray(slots[o:o + chunk])
            T = len(sl)
            k, v = _rand_rows(gen, (T, H, D), outliers), _rand_rows(gen, (T, H, D), outliers)
            sd = to_dev(sl)
            _lib.check(_lib.lib.rmlx_kv_append(pool.handle, 0, 1, k.data_ptr(), v.data_ptr(), T * H * D, H * D, D,
                                               sd.data_ptr(), T, _sp()))
            kh, vh = _host16(k), _host16(v)
            futs.append(ex.submit(orc.paged_append_quant, host, g, 0, 1, kh, vh, orc.BF16, T * H * D, H * D, D,
                                  sl))
            if len(futs) >= 2 * THREADS:
                assert futs.pop(0).result() == 0
        for f in futs:
            assert f.result() == 0
    torch.cuda.synchronize()


def test_decode_step_llama8b_layer(cuda):
    """Config 2: batch 64, ctx U[512,4096], 8 KV heads x 128, block 16, bf16."""
    import torch
    w = bench.WORKLOADS["decode"]
    wl = bench.make_workload(w, 1)
    H, D, BS, B, N = w.heads, w.head_dim, w.block, w.batch, wl["num_blocks"]
    pool = rmlx_kv.KVPool(1, H, D, BS, N, dtype=rmlx_kv.BF16)
    gen = torch.Generator(device="cuda").manual_seed(w.seed)
    _view(pool, torch.bfloat16).normal_(generator=gen)
    torch.cuda.synchronize()
    host = pool.read()
    g = orc.Geo(1, H, D, BS, N, 2)
    k, v = _rand_rows(gen, (B, H, D), 0.0), _rand_rows(gen, (B, H, D), 0.0)
    keep = _append_both(pool, host, g, k, v, wl["slots"][0], B, quant=False)
    lens = wl["lens0"] + 1
    (gk, gv), (ek, ev) = _gather_both(pool, host, g, wl["bt"], lens, quant=False)
    del keep
    assert pool.check() == 0
    _same(pool.read(), host, "pool after the append")
    _same(gk, ek, "gathered K")
    _same(gv, ev, "gathered V")
    pool.close()


def test_gather_layers_llama8b(cuda):
    """rmlx_kv_gather_layers at the decode shape (batch 64, ctx U[512,4096],
    8 KV heads x 128, bf16) over 4 layers in one launch, each layer's output
    at its own offset, against the oracle's per-layer gathers."""
    import torch
    w = bench.WORKLOADS["decode"]
    wl = bench.make_workload(w, 1)
    L, H, D, BS, B, N = 4, w.heads, w.head_dim, w.block, w.batch, wl["num_blocks"]
    pool = rmlx_kv.KVPool(L, H, D, BS, N, dtype=rmlx_kv.BF16)
    gen = torch.Generator(device="cuda").manual_seed(w.seed + 1)
    _view(pool, torch.bfloat16).normal_(generator=gen)
    torch.cuda.synchronize()
    host = pool.read()
    g = orc.Geo(L, H, D, BS, N, 2)
    lens = (wl["lens0"] + 1).astype(np.int32)
    bt = wl["bt"]
    tot = int(lens.sum()) * H * D
    ok = torch.empty(L * tot, dtype=torch.int16, device="cuda")
    ov = torch.empty_like(ok)
    btd, lnd = to_dev(bt), to_dev(lens)
    _lib.check(_lib.lib.rmlx_kv_gather_layers(pool.handle, 0, L, btd.data_ptr(), bt.shape[1], lnd.data_ptr(), B,
                                              ok.data_ptr(), ov.data_ptr(), tot, _sp()))
    torch.cuda.synchronize()
    assert pool.check() == 0
    for layer in range(L):
        ek, ev = np.empty(tot, np.uint16), np.empty(tot, np.uint16)
        assert orc.paged_gather(host, g, layer, bt, bt.shape[1], lens, ek, ev, threads=THREADS) == 0
        _same(ok[layer * tot:(layer + 1) * tot].cpu().numpy().view(np.uint16), ek, f"layer {layer} K")
        _same(ov[layer * tot:(layer + 1) * tot].cpu().numpy().view(np.uint16), ev, f"layer {layer} V")
    pool.close()


@pytest.mark.parametrize("bits", [8, 4])
def test_quant_step_llama8b_layer(cuda, bits):
    """Config 3: batch 128, ctx U[1024,8192], group 64, fp16 scale/zero,
    1% outliers x8; quantise-on-append of the prompts and of one step,
    dequantise-on-gather to bf16."""
    import torch
    w = bench.WORKLOADS["quant8" if bits == 8 else "quant4"]
    wl = bench.make_workload(w, 1)
    H, D, BS, B, N = w.heads, w.head_dim, w.block, w.batch, wl["num_blocks"]
    pool = rmlx_kv.KVPool(1, H, D, BS, N, dtype=rmlx_kv.BF16, quant_bits=bits, group_size=w.group,
                          meta_dtype=rmlx_kv.F16)
    g = orc.Geo(1, H, D, BS, N, 2, bits=bits, group_size=w.group, meta_bytes=2)
    host = np.zeros(g.pool_bytes(), dtype=np.uint8)
    assert host.size == pool.layout.bytes
    gen = torch.Generator(device="cuda").manual_seed(w.seed)
    _prefill_quant(pool, host, g, wl["bt"], wl["lens0"], gen, w.outliers)
    k, v = _rand_rows(gen, (B, H, D), w.outliers), _rand_rows(gen, (B, H, D), w.outliers)
    keep = _append_both(pool, host, g, k, v, wl["slots"][0], B, quant=True)
    (gk, gv), (ek, ev) = _gather_both(pool, host, g, wl["bt"], wl["lens0"] + 1, quant=True)
    del keep
    assert pool.check() == 0
    _same(pool.read(), host, "codes and scale/zero")
    _same(gk, ek, "dequantised K")
    _same(gv, ev, "dequantised V")
    pool.close()


@pytest.mark.parametrize("bits", [0, 8])
def test_fork_step_llama70b_one_head_shard(cuda, bits):
    """Config 5 on one GPU's shard at 8 GPUs (1 KV head, head offset 7):
    batch 256, ctx log-uniform [2048,32768]; two steps of forks (tile copies
    of shared tails), appends and gathers, as the bench plans them."""
    import torch
    B, D, BS = 256, 128, 16
    plan, N, _, _planner = bench.l70_plan(0x5EED + 5, 2)
    qkw = dict(quant_bits=8, group_size=64, meta_dtype=rmlx_kv.F16) if bits else {}
    pool = rmlx_kv.KVPool(1, 1, D, BS, N, dtype=rmlx_kv.BF16, head_offset=7, **qkw)
    g = orc.Geo(1, 1, D, BS, N, 2, bits=bits, group_size=64, meta_bytes=2)
    assert g.pool_bytes() == pool.layout.bytes
    gen = torch.Generator(device="cuda").manual_seed(0x5EED + 5 + 7)
    if bits:
        view = _view(pool, torch.uint8)
        view.random_(0, 256, generator=gen)
        tiles = view.view(-1, pool.layout.tile_bytes)
        codes = BS * pool.layout.row_bytes
        # (scale, zero) f16 pairs, written through views of the pool
        meta = tiles[:, codes:codes + BS * pool.layout.meta_row_bytes].unflatten(1, (-1, 4))
        meta[..., 0:2].view(torch.float16).uniform_(0.001, 0.05, generator=gen)
        meta[..., 2:4].view(torch.float16).uniform_(-3.0, -1.0, generator=gen)
        del view, tiles, meta
    else:
        _view(pool, torch.bfloat16).normal_(generator=gen)
    torch.cuda.synchronize()
    host = pool.read()
    lib = _lib.lib
    for step in plan:
        n = len(step["cow_src"])
        if n:
            src, dst = to_dev(step["cow_src"]), to_dev(step["cow_dst"])
            _lib.check(lib.rmlx_kv_copy_blocks(pool.handle, src.data_ptr(), dst.data_ptr(), n, _sp()))
            assert orc.copy_blocks(host, g, step["cow_src"], step["cow_dst"]) == 0
        k, v = _rand_rows(gen, (B, 1, D), 0.0), _rand_rows(gen, (B, 1, D), 0.0)
        keep = _append_both(pool, host, g, k, v, step["slots"], B, quant=bool(bits))
        (gk, gv), (ek, ev) = _gather_both(pool, host, g, step["bt"], step["lens"].astype(np.int64),
                                          quant=bool(bits))
        del keep
        _same(gk, ek, "gathered K")
        _same(gv, ev, "gathered V")
    assert pool.check() == 0
    _same(pool.read(), host, "pool after the steps")
    pool.close()


@pytest.mark.parametrize("bits", [0, 8, 4])
def test_attention_llama8b_layer(cuda, bits):
    """Decode attention at the Llama-3.1-8B shape (batch 64, ctx U[512,4096],
    8 KV heads x 128, 4 query heads per KV head), bf16 / 8-bit / 4-bit pools
    with fp16 scale/zero, against float64 attention over the oracle's rows
    (bf16 rows; the exact f32 dequantisation for quantised pools)."""
    import torch
    from test_gpu_attention import TOL, _attend
    w = bench.WORKLOADS["attn" if not bits else f"attn{bits}"]
    wl = bench.make_workload(w, 1)
    H, D, BS, B, N, G = w.heads, w.head_dim, w.block, w.batch, wl["num_blocks"], w.attn_g
    qkw = dict(quant_bits=bits, group_size=w.group, meta_dtype=rmlx_kv.F16) if bits else {}
    pool = rmlx_kv.KVPool(1, H, D, BS, N, dtype=rmlx_kv.BF16, **qkw)
    gen = torch.Generator(device="cuda").manual_seed(w.seed)
    lens = (wl["lens0"] + 1).astype(np.int32)
    bt = wl["bt"]
    if bits:
        slots = _slots_of_prompts(bt, lens, BS)
        for o in range(0, len(slots), 16384):
            sl = to_dev(np.ascontiguousarray(slots[o:o + 16384]))
            T = sl.numel()
            k, v = _rand_rows(gen, (T, H, D), 0.0), _rand_rows(gen, (T, H, D), 0.0)
            _lib.check(_lib.lib.rmlx_kv_append(pool.handle, 0, 1, k.data_ptr(), v.data_ptr(), T * H * D, H * D, D,
                                               sl.data_ptr(), T, _sp()))
            torch.cuda.synchronize()
    else:
        _view(pool, torch.bfloat16).normal_(generator=gen)
    q = _rand_rows(gen, (B, H * G, D), 0.0)
    scale = 1.0 / float(np.sqrt(D))
    ws_bytes = pool.attention_workspace_size(G, B, int(lens.sum()))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    out = torch.full((B, H * G, D), -7, dtype=torch.int16, device="cuda")
    btd, lnd = to_dev(bt), to_dev(lens)
    _lib.check(_lib.lib.rmlx_kv_decode_attention(pool.handle, 0, q.data_ptr(), G, btd.data_ptr(), bt.shape[1],
                                                 lnd.data_ptr(), B, scale, out.data_ptr(), ws.data_ptr(), ws_bytes,
                                                 _sp()))
    torch.cuda.synchronize()
    assert pool.check() == 0
    got = orc.dtype_to_f32(out.cpu().numpy().view(np.uint16), orc.BF16).astype(np.float64)
    host = pool.read()
    g = orc.Geo(1, H, D, BS, N, 2, bits=bits, group_size=w.group, meta_bytes=2)
    tot = int(lens.sum()) * H * D
    if bits:
        ek, ev = np.empty(tot, np.float32), np.empty(tot, np.float32)
        assert orc.paged_gather_dequant(host, g, 0, bt, bt.shape[1], lens, ek, ev, orc.F32, threads=THREADS) == 0
        kf, vf = ek.astype(np.float64), ev.astype(np.float64)
    else:
        ek, ev = np.empty(tot, np.uint16), np.empty(tot, np.uint16)
        assert orc.paged_gather(host, g, 0, bt, bt.shape[1], lens, ek, ev, threads=THREADS) == 0
        kf = orc.dtype_to_f32(ek, orc.BF16).astype(np.float64)
        vf = orc.dtype_to_f32(ev, orc.BF16).astype(np.float64)
    want = _attend(kf, vf, _host16(q), G, lens, scale, orc.BF16, H, D)
    err = np.abs(got - want)
    mx, rms = TOL[orc.BF16]
    assert np.isfinite(got).all()
    assert err.max() <= mx, f"max abs error {err.max()}"
    assert np.sqrt((err ** 2).mean()) <= rms, f"rms error {np.sqrt((err ** 2).mean())}"
    pool.close()
