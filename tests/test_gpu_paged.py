"""GPU parity: paged append (reshape-and-cache) and block-table gather.

The CUDA path (through the C ABI) and the oracle run on the same seeded
inputs; the pool bytes and the gathered K/V must be bit-identical.  The
semantics are RotatingKVCache's row copy (rotating_cache.rs:126-136,
162-197) placed by block tables.
"""
import numpy as np
import pytest

import oracle as orc
import rmlx_kv
from helpers import ESIZE, NP_DT, block_tables, rand_rows, slots_for, to_dev, to_host

pytestmark = pytest.mark.gpu


def run_case(cuda, L, H, D, bs, N, dt, prompt_lens, new_tokens=1, seed=0, layout="THD"):
    """Prefill every sequence, append `new_tokens` decode tokens, gather all
    layers; compare pool and outputs with the oracle."""
    rng = np.random.default_rng(seed)
    lens = np.array(prompt_lens, dtype=np.int64)
    bt, _ = block_tables(rng, lens, bs, N, extra=new_tokens)
    g = orc.Geo(L, H, D, bs, N, ESIZE[dt])
    host_pool = np.zeros(g.pool_bytes(), dtype=np.uint8)
    pool = rmlx_kv.KVPool(L, H, D, bs, N, dtype=dt, device=0)
    assert pool.layout.bytes == host_pool.size

    def append(positions):
        T = len(positions)
        if layout == "THD":
            shape, ls, ts, hs = (L, T, H, D), T * H * D, H * D, D
        else:  # the reference's [heads, tokens, head_dim] per layer
            shape, ls, ts, hs = (L, H, T, D), H * T * D, D, T * D
        k = rand_rows(rng, shape, dt)
        v = rand_rows(rng, shape, dt)
        slots = slots_for(bt, bs, positions) if T else np.zeros(0, dtype=np.int32)
        assert orc.paged_append(host_pool, g, 0, L, k, v, ls, ts, hs, slots) == 0
        if T:
            pool.append(to_dev(k), to_dev(v), to_dev(slots), T, layer_stride=ls, token_stride=ts, head_stride=hs)

    append([(s, p) for s in range(len(lens)) for p in range(lens[s])])
    for step in range(new_tokens):
        append([(s, int(lens[s]) + step) for s in range(len(lens))])
    final = (lens + new_tokens).astype(np.int32)
    assert pool.check() == 0
    np.testing.assert_array_equal(pool.read(), host_pool)

    tot = int(final.sum()) * H * D
    npdt = NP_DT[dt]
    bt_d, lens_d = to_dev(bt), to_dev(final)
    import torch
    ok = torch.empty(max(tot * ESIZE[dt], 16), dtype=torch.uint8, device=cuda)
    ov = torch.empty_like(ok)
    for layer in range(L):
        ek = np.zeros(tot, dtype=npdt)
        ev = np.zeros(tot, dtype=npdt)
        assert orc.paged_gather(host_pool, g, layer, bt, bt.shape[1], final, ek, ev) == 0
        pool.gather(layer, bt_d, bt.shape[1], lens_d, len(final), ok, ov)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(to_host(ok, npdt)[:tot], ek)
        np.testing.assert_array_equal(to_host(ov, npdt)[:tot], ev)
    assert pool.check() == 0
    pool.close()


def test_config1_fp16(cuda):
    """1 layer, 8 heads, 128, block 16, fp16, pool 256; prompts 37/128/255/512 + 1 token."""
    run_case(cuda, 1, 8, 128, 16, 256, orc.F16, [37, 128, 255, 512], seed=0x5EED + 1)


def test_reference_layout_bf16(cuda):
    run_case(cuda, 2, 4, 128, 16, 64, orc.BF16, [5, 16, 17, 40], new_tokens=3, seed=1, layout="HTD")


@pytest.mark.parametrize("dt,D", [(orc.F32, 64), (orc.BF16, 256), (orc.F16, 8)])
def test_dtypes_and_head_dims(cuda, dt, D):
    run_case(cuda, 2, 2, D, 16, 40, dt, [1, 15, 16, 33, 0], new_tokens=2, seed=2)


@pytest.mark.parametrize("bs", [1, 8, 32])
def test_block_sizes(cuda, bs):
    run_case(cuda, 1, 3, 64, bs, 200, orc.BF16, [3, 31, 32, 65], new_tokens=1, seed=3)


def test_ragged_and_empty_sequences(cuda):
    run_case(cuda, 3, 1, 128, 16, 64, orc.BF16, [0, 0, 1, 2, 15, 16, 17, 0, 31], new_tokens=0, seed=4)


def test_empty_calls_are_noops(cuda):
    import torch
    pool = rmlx_kv.KVPool(1, 1, 128, 16, 4, dtype=orc.BF16)
    pool.append(None, None, None, 0)
    dummy = torch.zeros(16, dtype=torch.uint8, device=cuda)
    pool.gather(0, dummy, 0, dummy, 0, dummy, dummy)
    assert pool.check() == 0
    assert not pool.read().any()


def test_many_sequences_per_launch(cuda):
    """8192 sequences (the per-launch maximum): the shared-memory scan path."""
    rng = np.random.default_rng(5)
    lens = rng.integers(0, 4, size=8192)
    run_case(cuda, 1, 1, 64, 4, 8192 * 2, orc.BF16, lens.tolist(), new_tokens=1, seed=5)


def test_negative_slot_skips_token(cuda):
    import torch
    L, H, D, bs, N = 1, 2, 64, 16, 8
    pool = rmlx_kv.KVPool(L, H, D, bs, N, dtype=orc.BF16)
    rng = np.random.default_rng(6)
    k = rand_rows(rng, (L, 3, H, D), orc.BF16)
    slots = np.array([5, -1, 17], dtype=np.int32)
    pool.append(to_dev(k), to_dev(k), to_dev(slots), 3)
    g = orc.Geo(L, H, D, bs, N, 2)
    host = np.zeros(g.pool_bytes(), dtype=np.uint8)
    orc.paged_append(host, g, 0, L, k, k, 3 * H * D, H * D, D, slots)
    assert pool.check() == 0
    np.testing.assert_array_equal(pool.read(), host)
    del torch


def test_out_of_pool_ids_are_flagged_not_written(cuda):
    """A slot or block-table entry outside the pool latches the device error
    word and skips only that row/tile (the reference panics on range)."""
    import torch
    L, H, D, bs, N = 1, 1, 64, 4, 4
    pool = rmlx_kv.KVPool(L, H, D, bs, N, dtype=orc.BF16)
    rng = np.random.default_rng(7)
    k = rand_rows(rng, (L, 2, H, D), orc.BF16)
    slots = np.array([3, N * bs], dtype=np.int32)  # second is one past the end
    pool.append(to_dev(k), to_dev(k), to_dev(slots), 2)
    assert pool.check() & 1  # DEV_ERR_SLOT
    g = orc.Geo(L, H, D, bs, N, 2)
    host = np.zeros(g.pool_bytes(), dtype=np.uint8)
    assert orc.paged_append(host, g, 0, L, k, k, 2 * H * D, H * D, D, slots) == 1
    np.testing.assert_array_equal(pool.read(), host)
    bt = np.array([[0, N + 3], [1, 0]], dtype=np.int32)
    lens = np.array([8, 4], dtype=np.int32)
    out = torch.full((12 * D,), 7, dtype=torch.int16, device=cuda)
    out2 = out.clone()
    pool.gather(0, to_dev(bt), 2, to_dev(lens), 2, out, out2)
    assert pool.check() & 2  # DEV_ERR_BLOCK
    ek = np.full(12 * D, 7, dtype=np.uint16)
    ev = ek.copy()
    assert orc.paged_gather(host, g, 0, bt, 2, lens, ek, ev) == 1
    np.testing.assert_array_equal(to_host(out, np.uint16), ek)


def test_status_async_reads_without_clearing(cuda):
    """rmlx_kv_pool_status_async copies the error word on a stream without
    waiting and without clearing it: 0 on a clean pool, the latched bit after
    an out-of-pool slot (once an event after it has completed), and the word
    is still there for the synchronous check, which clears it."""
    import torch
    from rmlx_kv import _lib
    L, H, D, bs, N = 1, 1, 64, 4, 4
    pool = rmlx_kv.KVPool(L, H, D, bs, N, dtype=orc.BF16)
    stream = torch.cuda.current_stream()
    word = torch.full((1,), -1, dtype=torch.int32).pin_memory()

    def read_async():
        pool.status_async(word, stream)
        ev = torch.cuda.Event()
        ev.record(stream)
        ev.synchronize()
        return int(word[0])

    assert read_async() == 0
    k = rand_rows(np.random.default_rng(9), (L, 1, H, D), orc.BF16)
    pool.append(to_dev(k), to_dev(k), to_dev(np.array([N * bs], dtype=np.int32)), 1)
    assert read_async() & 1  # DEV_ERR_SLOT
    assert read_async() & 1  # not cleared by the asynchronous read
    assert pool.check() & 1
    assert read_async() == 0
    assert _lib.lib.rmlx_kv_pool_status_async(pool.handle, None, stream.cuda_stream) == _lib.RMLX_E_BAD_ARG
    pool.close()


def test_bad_arguments_rejected(cuda):
    with pytest.raises(rmlx_kv.RmlxError):
        rmlx_kv.KVPool(1, 1, 12, 16, 4, dtype=orc.BF16)  # 24-byte rows are not 16-byte multiples
    pool = rmlx_kv.KVPool(2, 1, 64, 16, 4, dtype=orc.BF16)
    import torch
    d = torch.zeros(64, dtype=torch.int32, device=cuda)
    with pytest.raises(rmlx_kv.RmlxError):
        pool.gather(2, d, 1, d, 1, d, d)  # layer out of range
    with pytest.raises(rmlx_kv.RmlxError):
        pool.append(d, d, d, 1, layer_begin=1, num_layers=2)
    with pytest.raises(rmlx_kv.RmlxError):
        pool.gather(0, d, 1, d, 8193, d, d)  # too many sequences for one launch


def _gather_layers_case(cuda, L, H, D, bs, N, dt, lens, l0, nl, seed, bits=0, gs=64, meta=orc.F16):
    """rmlx_kv_gather_layers over layers [l0, l0 + nl) equals the oracle's
    per-layer gathers, each at its layer offset, with padding between the
    layers' outputs left untouched."""
    import torch
    rng = np.random.default_rng(seed)
    lens = np.array(lens, dtype=np.int64)
    bt, _ = block_tables(rng, lens, bs, N)
    qkw = dict(quant_bits=bits, group_size=gs, meta_dtype=meta) if bits else {}
    pool = rmlx_kv.KVPool(L, H, D, bs, N, dtype=dt, **qkw)
    g = orc.Geo(L, H, D, bs, N, ESIZE[dt], bits=bits, group_size=gs, meta_bytes=4 if meta == orc.F32 else 2)
    if bits:
        host = np.zeros(g.pool_bytes(), dtype=np.uint8)
        pos = [(s, p) for s in range(len(lens)) for p in range(lens[s])]
        k = rand_rows(rng, (L, len(pos), H, D), dt, 0.01)
        v = rand_rows(rng, (L, len(pos), H, D), dt, 0.01)
        slots = slots_for(bt, bs, pos)
        assert orc.paged_append_quant(host, g, 0, L, k, v, dt, len(pos) * H * D, H * D, D, slots) == 0
        pool.append(to_dev(k), to_dev(v), to_dev(slots), len(pos))
    else:
        host = rng.integers(0, 256, size=g.pool_bytes(), dtype=np.uint8)
        pool.write(host)
    final = lens.astype(np.int32)
    tot = int(final.sum()) * H * D
    npdt = NP_DT[dt]
    stride = tot + 24  # elements between layers: 16-byte multiple, with a gap
    ok = torch.full((nl * stride * ESIZE[dt],), 0x5A, dtype=torch.uint8, device=cuda)
    ov = torch.full_like(ok, 0x5A)
    pool.gather_layers(l0, nl, to_dev(bt), bt.shape[1], to_dev(final), len(final), ok, ov, stride)
    torch.cuda.synchronize()
    assert pool.check() == 0
    gk, gv = to_host(ok, npdt).reshape(nl, stride), to_host(ov, npdt).reshape(nl, stride)
    pad = np.full(24 * ESIZE[dt], 0x5A, dtype=np.uint8).view(npdt)
    for i in range(nl):
        ek, ev = np.zeros(tot, dtype=npdt), np.zeros(tot, dtype=npdt)
        if bits:
            assert orc.paged_gather_dequant(host, g, l0 + i, bt, bt.shape[1], final, ek, ev, dt) == 0
        else:
            assert orc.paged_gather(host, g, l0 + i, bt, bt.shape[1], final, ek, ev) == 0
        np.testing.assert_array_equal(gk[i, :tot], ek)
        np.testing.assert_array_equal(gv[i, :tot], ev)
        np.testing.assert_array_equal(gk[i, tot:], pad)
    pool.close()


@pytest.mark.parametrize("l0,nl", [(0, 4), (1, 2), (3, 1)])
def test_gather_layers(cuda, l0, nl):
    _gather_layers_case(cuda, 4, 3, 128, 16, 96, orc.BF16, [1, 15, 16, 17, 0, 300, 33], l0, nl, seed=20 + l0 + nl)


@pytest.mark.parametrize("dt,D,bs", [(orc.F32, 64, 8), (orc.F16, 256, 32), (orc.BF16, 64, 1)])
def test_gather_layers_dtypes(cuda, dt, D, bs):
    _gather_layers_case(cuda, 3, 2, D, bs, 400 // bs + 40, dt, [5, 0, 40, 129], 0, 3, seed=25)


@pytest.mark.parametrize("bits", [8, 4])
def test_gather_layers_quantised(cuda, bits):
    """Quantised pools: one dequantising launch per layer, same offsets."""
    _gather_layers_case(cuda, 3, 2, 128, 16, 64, orc.BF16, [3, 64, 100], 0, 3, seed=27, bits=bits)


def test_gather_layers_bad_arguments(cuda):
    import torch
    pool = rmlx_kv.KVPool(4, 1, 64, 16, 4, dtype=orc.BF16)
    d = torch.zeros(256, dtype=torch.int32, device=cuda)
    with pytest.raises(rmlx_kv.RmlxError):
        pool.gather_layers(2, 3, d, 1, d, 1, d, d, 64)  # past the last layer
    with pytest.raises(rmlx_kv.RmlxError):
        pool.gather_layers(0, 2, d, 1, d, 1, d, d, 4)  # 8-byte layer stride
    with pytest.raises(rmlx_kv.RmlxError):
        pool.gather_layers(0, 2, d, 1, d, 1, d, d, 0)
    pool.gather_layers(0, 0, d, 1, d, 1, d, d, 64)  # no layers: a no-op
    assert pool.check() == 0
    pool.close()
