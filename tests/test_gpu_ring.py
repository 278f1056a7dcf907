"""GPU parity of the sliding-window ring: random appends and trims driven by
RotatingBlocks on a device pool (rmlx_kv_append, rmlx_kv_move_rows,
rmlx_kv_gather_ring) against the oracle's RotatingKVCache, one oracle cache
per layer.  f32 pools compare bit for bit with the reference's f32 rows;
bf16 pools with the same rows rounded to bf16.  Decode attention over the
ring's rows [0, seq_len) equals attention over the oracle's logical rows
(attention does not depend on row order)."""
import numpy as np
import pytest

import oracle as orc
import rmlx_kv
from helpers import to_dev
from rmlx_kv.batch import RotatingBlocks

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dt,bs,max_size,keep", [(orc.F32, 16, 40, 4), (orc.BF16, 8, 37, 0), (orc.F32, 5, 23, 22),
                                                 (orc.BF16, 16, 64, 16)])
def test_ring_matches_oracle(cuda, dt, bs, max_size, keep):
    import torch
    L, H, D, B = 2, 2, 64, 3
    N = B * (-(-max_size // bs)) + 4
    pool = rmlx_kv.KVPool(L, H, D, bs, N, dtype=dt)
    pool.write(np.zeros(pool.layout.bytes, np.uint8))
    mgr = rmlx_kv.PagedCacheManager(bs, N)
    rings = [RotatingBlocks(mgr, bs, max_size, keep) for _ in range(B)]
    refs = [[orc.RotatingKVCache(1, H, D, max_size, keep) for _ in range(L)] for _ in range(B)]
    rng = np.random.default_rng(70 + bs)
    npdt = np.float32 if dt == orc.F32 else np.uint16
    for step in range(25):
        for s in range(B):
            if rng.random() < 0.2 and rings[s].can_trim():
                n = int(rng.integers(0, rings[s].seq_len() - keep + 1))
                src, dst = rings[s].trim(n)
                for r in refs[s]:
                    r.trim(n)
                if len(src):
                    pool.move_rows(to_dev(src), to_dev(dst), len(src))
            else:
                T = int(rng.integers(1, max_size + 5))
                x = rng.standard_normal((L, H, T, D), dtype=np.float32)
                xq = orc.dtype_to_f32(orc.f32_to_dtype(x, dt), dt) if dt != orc.F32 else x
                slots = rings[s].append_slots(T)
                for l in range(L):
                    refs[s][l].append(0, xq[l].reshape(-1), -xq[l].reshape(-1), T)
                k = orc.f32_to_dtype(x, dt) if dt != orc.F32 else x
                v = orc.f32_to_dtype(-x, dt) if dt != orc.F32 else -x
                pool.append(to_dev(k), to_dev(v), to_dev(slots), T, layer_stride=H * T * D, token_stride=D,
                            head_stride=T * D)
        lens = np.array([r.seq_len() for r in rings], np.int32)
        offs = np.array([r.ring_offset() for r in rings], np.int32)
        width = max(max(len(r.table) for r in rings), 1)
        bt = np.zeros((B, width), np.int32)
        for s, r in enumerate(rings):
            bt[s, :len(r.table)] = r.table
        tot = int(lens.sum()) * H * D
        ok = torch.empty(max(tot, 4), dtype=torch.float32 if dt == orc.F32 else torch.int16, device=cuda)
        ov = torch.empty_like(ok)
        for l in range(L):
            pool.gather_ring(l, to_dev(bt), width, to_dev(lens), to_dev(offs), B, keep, max_size, ok, ov)
            torch.cuda.synchronize()
            gk = ok.cpu().numpy().view(npdt)[:tot]
            gv = ov.cpu().numpy().view(npdt)[:tot]
            if dt != orc.F32:
                gk, gv = orc.dtype_to_f32(gk, dt), orc.dtype_to_f32(gv, dt)
            o = 0
            for s in range(B):
                n = int(lens[s]) * H * D
                want_k = np.concatenate([np.asarray(h, np.float32) for h in refs[s][l].get_keys(0)])
                want_v = np.concatenate([np.asarray(h, np.float32) for h in refs[s][l].get_values(0)])
                np.testing.assert_array_equal(gk[o:o + n], want_k)
                np.testing.assert_array_equal(gv[o:o + n], want_v)
                o += n
        assert pool.check() == 0
    pool.close()


def test_ring_decode_attention_order_free(cuda):
    """Attention over a rotated ring's physical rows equals attention over
    the logical rows."""
    import torch
    L, H, D, bs, max_size, keep, G = 1, 2, 128, 16, 100, 10, 4
    pool = rmlx_kv.KVPool(L, H, D, bs, 16, dtype=orc.BF16)
    mgr = rmlx_kv.PagedCacheManager(bs, 16)
    ring = RotatingBlocks(mgr, bs, max_size, keep)
    rng = np.random.default_rng(77)
    T = 257  # wraps the ring twice
    x = orc.f32_to_dtype(rng.standard_normal((L, H, T, D), dtype=np.float32), orc.BF16)
    slots = ring.append_slots(T)
    pool.append(to_dev(x), to_dev(x), to_dev(slots), T, layer_stride=H * T * D, token_stride=D, head_stride=T * D)
    assert ring.ring_offset() > 0
    bt = np.array([ring.table], np.int32)
    lens = np.array([ring.seq_len()], np.int32)
    q = torch.from_numpy(orc.f32_to_dtype(rng.standard_normal((1, H * G, D), dtype=np.float32), orc.BF16)
                         .view(np.int16)).to(cuda)
    ws = torch.empty(pool.attention_workspace_size(G, 1, max_size), dtype=torch.uint8, device=cuda)
    out = torch.empty((1, H * G, D), dtype=torch.int16, device=cuda)
    pool.decode_attention(0, q, G, to_dev(bt), bt.shape[1], to_dev(lens), 1, 1 / np.sqrt(D), out, ws)
    ok = torch.empty(max_size * H * D, dtype=torch.int16, device=cuda)
    ov = torch.empty_like(ok)
    pool.gather_ring(0, to_dev(bt), bt.shape[1], to_dev(lens), to_dev(np.array([ring.ring_offset()], np.int32)), 1,
                     keep, max_size, ok, ov)
    torch.cuda.synchronize()
    k = orc.dtype_to_f32(ok.cpu().numpy().view(np.uint16), orc.BF16).astype(np.float64).reshape(H, max_size, D)
    qf = orc.dtype_to_f32(q.cpu().numpy().view(np.uint16), orc.BF16).astype(np.float64).reshape(H * G, D)
    want = np.zeros((H * G, D))
    for j in range(H * G):
        sc = k[j // G] @ qf[j] / np.sqrt(D)
        p = np.exp(sc - sc.max())
        want[j] = (p / p.sum()) @ k[j // G]
    got = orc.dtype_to_f32(out.cpu().numpy().view(np.uint16), orc.BF16).reshape(H * G, D)
    assert np.abs(got - want).max() < 0.03
    pool.close()
