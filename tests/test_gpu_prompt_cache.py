"""Prompt cache save/load through a device pool (prompt_cache.rs:63-210).

save: the file equals, byte for byte, what the safetensors library writes
for the sequence's rows as the oracle gathers them from the same pool
bytes.  load: the blocks it fills hold exactly the rows the oracle's append
writes (a quantised pool quantises them on the way in), and a pool that
holds a shard of the heads loads its own heads from a full file.
"""
import numpy as np
import pytest

import oracle as orc
import rmlx_kv
from helpers import ESIZE, NP_DT, block_tables, rand_rows
from rmlx_kv import prompt_cache as pc

pytestmark = pytest.mark.gpu
st = pytest.importorskip("safetensors.torch")


def _torch_view(a, dt):
    import torch
    t = torch.from_numpy(np.ascontiguousarray(a).view(np.int16 if a.dtype == np.uint16 else a.dtype))
    return t.view(torch.bfloat16 if dt == orc.BF16 else torch.float16) if dt != orc.F32 else t


def _filled(L, H, D, bs, N, dt, seed, **kw):
    pool = rmlx_kv.KVPool(L, H, D, bs, N, dtype=dt, **kw)
    rng = np.random.default_rng(seed)
    vals = rng.standard_normal(pool.layout.bytes // ESIZE[dt], dtype=np.float32)
    host = orc.f32_to_dtype(vals, dt).view(np.uint8).copy() if not kw.get("quant_bits") else None
    if host is not None:
        pool.write(host)
    return pool, host, rng


@pytest.mark.parametrize("dt", [orc.BF16, orc.F16])
def test_save_matches_safetensors(cuda, tmp_path, dt):
    L, H, D, bs, N = 3, 4, 128, 16, 64
    pool, host, rng = _filled(L, H, D, bs, N, dt, 80)
    seq = 37
    bt, _ = block_tables(rng, [seq], bs, N)
    ids = bt[0, :3]
    path = tmp_path / "s.safetensors"
    meta = {"model": "llama"}
    pc.save_prompt_cache(path, pool, ids, seq, metadata=meta)
    g = orc.Geo(L, H, D, bs, N, ESIZE[dt])
    ref = {}
    lens = np.array([seq], np.int32)
    for l in range(L):
        ek, ev = np.zeros(seq * H * D, NP_DT[dt]), np.zeros(seq * H * D, NP_DT[dt])
        assert orc.paged_gather(host, g, l, bt, bt.shape[1], lens, ek, ev) == 0
        for h in range(H):
            ref[f"layer_{l}_head_{h}_keys"] = _torch_view(ek.reshape(H, seq, D)[h], dt)
            ref[f"layer_{l}_head_{h}_values"] = _torch_view(ev.reshape(H, seq, D)[h], dt)
    assert path.read_bytes() == st.save(ref, metadata=meta)
    pool.close()


@pytest.mark.parametrize("bits", [0, 8, 4])
def test_load_writes_the_oracle_rows(cuda, tmp_path, bits):
    L, H, D, bs, N, dt, seq = 2, 4, 128, 16, 32, orc.BF16, 70
    rng = np.random.default_rng(81 + bits)
    k = rand_rows(rng, (L, H, seq, D), dt, 0.01)
    v = rand_rows(rng, (L, H, seq, D), dt, 0.01)
    path = tmp_path / "l.safetensors"
    pc.write_prompt_cache(path, k, v, dt)
    qkw = dict(quant_bits=bits, group_size=64, meta_dtype=orc.F16) if bits else {}
    pool = rmlx_kv.KVPool(L, H, D, bs, N, dtype=dt, **qkw)
    pool.write(np.zeros(pool.layout.bytes, np.uint8))
    ids = rng.permutation(N)[:5].astype(np.int32)
    assert pc.load_prompt_cache(path, pool, ids) == seq
    assert pool.check() == 0
    g = orc.Geo(L, H, D, bs, N, ESIZE[dt], **(dict(bits=bits, group_size=64, meta_bytes=2) if bits else {}))
    host = np.zeros(g.pool_bytes(), np.uint8)
    slots = np.array([ids[t // bs] * bs + t % bs for t in range(seq)], np.int32)
    # the file's [layer][head][token][dim] rows: head stride seq*D, token stride D
    ls, ts, hs = H * seq * D, D, seq * D
    if bits:
        assert orc.paged_append_quant(host, g, 0, L, k, v, dt, ls, ts, hs, slots) == 0
    else:
        assert orc.paged_append(host, g, 0, L, k, v, ls, ts, hs, slots) == 0
    np.testing.assert_array_equal(pool.read(), host)
    if not bits:  # and saving it back gives the same file
        p2 = tmp_path / "l2.safetensors"
        pc.save_prompt_cache(p2, pool, ids, seq)
        assert p2.read_bytes() == path.read_bytes()
    pool.close()


def test_sharded_pools_load_their_heads(cuda, tmp_path):
    L, H, D, bs, N, dt, seq = 2, 8, 64, 16, 16, orc.F16, 33
    rng = np.random.default_rng(83)
    k = rand_rows(rng, (L, H, seq, D), dt)
    v = rand_rows(rng, (L, H, seq, D), dt)
    path = tmp_path / "full.safetensors"
    pc.write_prompt_cache(path, k, v, dt, metadata={"shards": "2"})
    ids = np.array([3, 9, 1], np.int32)
    for r in range(2):
        pool = rmlx_kv.KVPool(L, H // 2, D, bs, N, dtype=dt, head_offset=r * (H // 2))
        assert pc.load_prompt_cache(path, pool, ids) == seq
        out = tmp_path / f"shard{r}.safetensors"
        pc.save_prompt_cache(out, pool, ids, seq)
        sk, sv = pc.read_prompt_cache(out, L, H // 2, D, dt, head_offset=r * (H // 2))
        np.testing.assert_array_equal(sk, k[:, r * 4:(r + 1) * 4])
        np.testing.assert_array_equal(sv, v[:, r * 4:(r + 1) * 4])
        pool.close()


def test_empty_and_bad_calls(cuda, tmp_path):
    pool = rmlx_kv.KVPool(1, 2, 64, 16, 8, dtype=orc.BF16)
    p = tmp_path / "e.safetensors"
    pc.save_prompt_cache(p, pool, [], 0, metadata={"k": "v"})
    assert p.read_bytes() == st.save({}, metadata={"k": "v"})
    assert pc.load_prompt_cache(p, pool, []) == 0
    with pytest.raises(rmlx_kv.RmlxError, match="fewer"):
        pc.save_prompt_cache(p, pool, [0], 17)
    with pytest.raises(rmlx_kv.RmlxError):
        pc.save_prompt_cache(p, pool, [0, 99], 20)  # block 99 is outside the pool
    k = np.zeros((1, 2, 20, 64), np.uint16)
    pc.write_prompt_cache(p, k, k, orc.BF16)
    with pytest.raises(rmlx_kv.RmlxError, match="fewer"):
        pc.load_prompt_cache(p, pool, [0])
    with pytest.raises(rmlx_kv.RmlxError, match="out of range"):
        pc.load_prompt_cache(p, pool, [0, 8])
    pool.close()
