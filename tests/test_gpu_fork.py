"""GPU parity of a forked decode batch: per step the copy-on-write tile
copies, the one-token append and the gather of every layer, on the device
and in the oracle, with block tables from SequenceBlocks.  bf16 and 8-bit
pools; gathered K/V and final pool bytes bit-exact."""
import numpy as np
import pytest

import oracle as orc
import rmlx_kv
from helpers import ESIZE, NP_DT, rand_rows, to_dev, to_host
from rmlx_kv.batch import SequenceBlocks

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("bits", [0, 8])
def test_fork_cow_append_gather(cuda, bits):
    import torch
    L, H, D, bs, B, steps, nfork = 2, 2, 128, 16, 12, 6, 3
    dt = orc.BF16
    rng = np.random.default_rng(50 + bits)
    lens = rng.integers(1, 100, size=B)
    nb = int(((lens + bs - 1) // bs).sum()) + (steps + 1) * (B + nfork)
    qkw = dict(quant_bits=bits, group_size=64, meta_dtype=orc.F16) if bits else {}
    g = orc.Geo(L, H, D, bs, nb, ESIZE[dt], **(dict(bits=8, group_size=64, meta_bytes=2) if bits else {}))
    pool = rmlx_kv.KVPool(L, H, D, bs, nb, dtype=dt, **qkw)
    host = np.zeros(g.pool_bytes(), dtype=np.uint8)
    mgr = rmlx_kv.PagedCacheManager(bs, nb)
    mgr.free_n(rng.permutation(mgr.allocate_n(nb)))  # scattered block ids
    seqs = SequenceBlocks(mgr, bs, lens)
    pos = [(s, p) for s in range(B) for p in range(int(lens[s]))]
    bt0 = seqs.block_table()
    slots0 = np.array([bt0[s, p // bs] * bs + p % bs for s, p in pos], dtype=np.int32)

    def append(slots):
        T = len(slots)
        k = rand_rows(rng, (L, T, H, D), dt, 0.01)
        v = rand_rows(rng, (L, T, H, D), dt, 0.01)
        ls, ts, hs = T * H * D, H * D, D
        if bits:
            assert orc.paged_append_quant(host, g, 0, L, k, v, dt, ls, ts, hs, slots) == 0
        else:
            assert orc.paged_append(host, g, 0, L, k, v, ls, ts, hs, slots) == 0
        pool.append(to_dev(k), to_dev(v), to_dev(slots), T)

    append(slots0)
    npdt = NP_DT[dt]
    for step in range(steps):
        idx = rng.permutation(B)
        for p, c in zip(idx[:nfork], idx[nfork:2 * nfork]):
            seqs.fork(int(p), int(c))
        src, dst, slots = seqs.append_slots()
        if len(src):
            assert orc.copy_blocks(host, g, src, dst) == 0
            pool.copy_blocks(to_dev(src), to_dev(dst), len(src))
        append(slots)
        bt, final = seqs.block_table(), seqs.seq_lens()
        tot = int(final.sum()) * H * D
        ok = torch.empty(tot * ESIZE[dt], dtype=torch.uint8, device=cuda)
        ov = torch.empty_like(ok)
        bt_d, lens_d = to_dev(bt), to_dev(final)
        for layer in range(L):
            ek, ev = np.zeros(tot, dtype=npdt), np.zeros(tot, dtype=npdt)
            if bits:
                assert orc.paged_gather_dequant(host, g, layer, bt, bt.shape[1], final, ek, ev, dt) == 0
            else:
                assert orc.paged_gather(host, g, layer, bt, bt.shape[1], final, ek, ev) == 0
            pool.gather(layer, bt_d, bt.shape[1], lens_d, B, ok, ov)
            torch.cuda.synchronize()
            np.testing.assert_array_equal(to_host(ok, npdt)[:tot], ek)
            np.testing.assert_array_equal(to_host(ov, npdt)[:tot], ev)
    assert pool.check() == 0
    np.testing.assert_array_equal(pool.read(), host)
    pool.close()
