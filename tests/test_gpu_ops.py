"""GPU parity: block copy (copy-on-write data move), pack/unpack for
migration, the prefix-block chain hash, and the device-backed
QuantizedKVCache drop-in."""
import numpy as np
import pytest

import oracle as orc
import rmlx_kv
from helpers import to_dev

pytestmark = pytest.mark.gpu


def _filled_pool(L, H, D, bs, N, seed, **kw):
    pool = rmlx_kv.KVPool(L, H, D, bs, N, **kw)
    rng = np.random.default_rng(seed)
    data = rng.integers(0, 256, size=pool.layout.bytes, dtype=np.uint8)
    pool.write(data)
    return pool, data


def test_copy_blocks_matches_oracle(cuda):
    L, H, D, bs, N = 4, 8, 128, 16, 64
    pool, host = _filled_pool(L, H, D, bs, N, 21, dtype=orc.BF16)
    g = orc.Geo(L, H, D, bs, N, 2)
    src = np.array([3, 7, 9, 0, 63], dtype=np.int32)
    dst = np.array([10, 11, 40, 62, 1], dtype=np.int32)
    pool.copy_blocks(to_dev(src), to_dev(dst), len(src))
    assert orc.copy_blocks(host, g, src, dst) == 0
    assert pool.check() == 0
    np.testing.assert_array_equal(pool.read(), host)


def test_copy_blocks_quantised_pool(cuda):
    pool, host = _filled_pool(2, 2, 128, 16, 16, 22, dtype=orc.BF16, quant_bits=4, group_size=64,
                              meta_dtype=orc.F16)
    g = orc.Geo(2, 2, 128, 16, 16, 2, bits=4, group_size=64, meta_bytes=2)
    src, dst = np.array([1, 2], np.int32), np.array([5, 6], np.int32)
    pool.copy_blocks(to_dev(src), to_dev(dst), 2)
    orc.copy_blocks(host, g, src, dst)
    np.testing.assert_array_equal(pool.read(), host)


def test_copy_blocks_bad_id_flagged(cuda):
    pool, host = _filled_pool(1, 1, 64, 16, 4, 23, dtype=orc.BF16)
    pool.copy_blocks(to_dev(np.array([0, 9], np.int32)), to_dev(np.array([1, 2], np.int32)), 2)
    assert pool.check() & 2
    g = orc.Geo(1, 1, 64, 16, 4, 2)
    orc.copy_blocks(host, g, [0, 9], [1, 2])
    np.testing.assert_array_equal(pool.read(), host)


def test_pack_unpack_roundtrip(cuda):
    import torch
    L, H, D, bs, N = 3, 4, 128, 16, 32
    a, host_a = _filled_pool(L, H, D, bs, N, 24, dtype=orc.BF16)
    b, host_b = _filled_pool(L, H, D, bs, N, 25, dtype=orc.BF16)
    ids = np.array([5, 0, 31, 17], dtype=np.int32)
    dst = np.array([1, 2, 3, 30], dtype=np.int32)
    bb = a.layout.block_bytes
    staging = torch.empty(len(ids) * bb, dtype=torch.uint8, device=cuda)
    a.pack_blocks(to_dev(ids), len(ids), staging)
    torch.cuda.synchronize()
    st = staging.cpu().numpy()
    for i, blk in enumerate(ids):
        np.testing.assert_array_equal(st[i * bb:(i + 1) * bb], host_a[blk * bb:(blk + 1) * bb])
    b.unpack_blocks(to_dev(dst), len(dst), staging)
    for i, blk in enumerate(dst):
        host_b[blk * bb:(blk + 1) * bb] = host_a[ids[i] * bb:(ids[i] + 1) * bb]
    assert b.check() == 0
    np.testing.assert_array_equal(b.read(), host_b)


@pytest.mark.parametrize("bs", [16, 1, 5])
def test_chain_hash_matches_oracle(cuda, bs):
    import torch
    rng = np.random.default_rng(26)
    lens = [0, 1, 15, 16, 17, 33, 2048, 100, 64]
    cu = np.zeros(len(lens) + 1, dtype=np.int64)
    cu[1:] = np.cumsum(lens)
    toks = rng.integers(0, 128256, size=int(cu[-1]), dtype=np.uint32)
    roots = rng.integers(0, 2 ** 63, size=len(lens), dtype=np.uint64)
    roots[0] = 0
    want, cub = orc.hash_chains(toks, cu, roots, bs)
    out = torch.zeros(max(len(want), 1), dtype=torch.int64, device=cuda)
    rmlx_kv.hash_block_chains(to_dev(toks), to_dev(cu), to_dev(roots), len(lens), bs, to_dev(cub), out)
    torch.cuda.synchronize()
    got = out.cpu().numpy().view(np.uint64)[:len(want)]
    np.testing.assert_array_equal(got, want)


def test_chain_hash_shared_prefix_is_shared(cuda):
    """Two requests with the same first 2 blocks get the same first 2 hashes."""
    import torch
    rng = np.random.default_rng(27)
    pre = rng.integers(0, 1000, size=32, dtype=np.uint32)
    a = np.concatenate([pre, rng.integers(0, 1000, size=20, dtype=np.uint32)])
    b = np.concatenate([pre, rng.integers(0, 1000, size=16, dtype=np.uint32)])
    toks = np.concatenate([a, b])
    cu = np.array([0, len(a), len(a) + len(b)], dtype=np.int64)
    want, cub = orc.hash_chains(toks, cu, np.zeros(2, np.uint64), 16)
    out = torch.zeros(len(want), dtype=torch.int64, device=cuda)
    rmlx_kv.hash_block_chains(to_dev(toks), to_dev(cu), None, 2, 16, to_dev(cub), out)
    got = out.cpu().numpy().view(np.uint64)
    np.testing.assert_array_equal(got, want)
    na = int(cub[1])
    assert got[0] == got[na] and got[1] == got[na + 1] and got[2] != got[na + 2]


# ---- QuantizedKVCache drop-in (quantized_cache.rs) ------------------------

def test_qcache_reference_tests(cuda):  # quantized_cache.rs:304-386
    c = rmlx_kv.QuantizedKVCache(32, 8, 128, 4, 32)
    assert (c.seq_len(), c.num_layers(), c.bits(), c.group_size()) == (0, 32, 4, 32)
    c = rmlx_kv.QuantizedKVCache(1, 1, 8, 8, 8)  # :344-365
    keys = np.arange(8, dtype=np.float32)
    c.append(0, keys, keys * 10, 1)
    assert c.seq_len() == 1
    dk = c.get_keys_dequantized(0)
    assert len(dk) == 8 and np.abs(dk - keys).max() < 0.1
    with pytest.raises(rmlx_kv.RmlxError, match="bits must be 4 or 8"):  # :383-386
        rmlx_kv.QuantizedKVCache(1, 1, 8, 3, 8)


@pytest.mark.parametrize("bits,gs,D,H", [(8, 64, 128, 8), (4, 64, 128, 8), (8, 32, 64, 2), (4, 5, 10, 3),
                                         (8, 7, 14, 1), (4, 64, 32, 1)])
def test_qcache_matches_oracle(cuda, bits, gs, D, H):
    rng = np.random.default_rng(28)
    L = 2
    mine = rmlx_kv.QuantizedKVCache(L, H, D, bits, gs)
    ref = orc.QuantizedKVCache(L, H, D, bits, gs)
    single_partial = gs > D
    for step, T in enumerate([5, 1, 1, 3] if not single_partial else [1]):
        for layer in range(L):
            k = rng.standard_normal(H * T * D).astype(np.float32)
            v = (rng.standard_normal(H * T * D) * 3).astype(np.float32)
            mine.append(layer, k, v, T)
            ref.append(layer, k, v, T)
    assert mine.seq_len() == ref.seq_len()
    for layer in range(L):
        for which in (0, 1):
            for a, b in zip(mine.raw(layer, which), ref.raw(layer, which)):
                np.testing.assert_array_equal(a, b)
        np.testing.assert_array_equal(mine.get_keys_dequantized(layer), ref.get_keys_dequantized(layer))
        np.testing.assert_array_equal(mine.get_values_dequantized(layer), ref.get_values_dequantized(layer))


def test_qcache_partial_groups_reproduce_reference_panic(cuda):
    """group_size > head_dim: the second append leaves a partial group mid-
    stream and dequantize_data's slice panics (start > end); both refuse."""
    mine = rmlx_kv.QuantizedKVCache(1, 1, 8, 8, 32)
    ref = orc.QuantizedKVCache(1, 1, 8, 8, 32)
    x = np.arange(8, dtype=np.float32)
    for c in (mine, ref):
        c.append(0, x, x, 1)
    np.testing.assert_array_equal(mine.get_keys_dequantized(0), ref.get_keys_dequantized(0))
    for c in (mine, ref):
        c.append(0, x + 1, x, 1)
    with pytest.raises(orc.OracleError):
        ref.get_keys_dequantized(0)
    with pytest.raises(rmlx_kv.RmlxError):
        mine.get_keys_dequantized(0)


def test_qcache_length_mismatch(cuda):
    c = rmlx_kv.QuantizedKVCache(1, 2, 8, 8, 8)
    with pytest.raises(rmlx_kv.RmlxError, match="length mismatch"):
        c.append(0, np.zeros(8, np.float32), np.zeros(8, np.float32), 1)


def test_chain_hash_full_prefix_workload(cuda):
    """All blocks of the prefix-caching workload (512 requests, ~640k tokens)."""
    import torch
    from helpers import prefix_workload
    rng = np.random.default_rng(0x5EED + 4)
    toks, cu = prefix_workload(rng, 512, 8, 1024, (64, 512), (256, 2048))
    roots = np.zeros(512, dtype=np.uint64)
    want, cub = orc.hash_chains(toks, cu, roots, 16)
    out = torch.zeros(len(want), dtype=torch.int64, device=cuda)
    rmlx_kv.hash_block_chains(to_dev(toks), to_dev(cu), None, 512, 16, to_dev(cub), out)
    np.testing.assert_array_equal(out.cpu().numpy().view(np.uint64), want)
