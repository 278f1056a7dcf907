"""Prompt cache files (prompt_cache.rs:63-233) on the host, no GPU.

The reference writes its file with the safetensors crate
(safetensors::tensor::serialize; Cargo.lock pins 0.4.5).  The Python package
`safetensors` installed here binds the same Rust crate (0.7.0), so it is the
checker: files written by rmlx_prompt_cache_write must be byte-identical to
its output for the same tensors and metadata, and files it writes must read
back exactly.  Where the metadata has several keys the crate writes them in
hash-map order, so those files are compared by content instead of bytes.
"""
import numpy as np
import pytest

import rmlx_kv
from rmlx_kv import prompt_cache as pc
from rmlx_kv.batch import SequenceBlocks

st = pytest.importorskip("safetensors.torch")
torch = pytest.importorskip("torch")

TORCH_DT = {rmlx_kv.F32: torch.float32, rmlx_kv.F16: torch.float16, rmlx_kv.BF16: torch.bfloat16}
NP_DT = {rmlx_kv.F32: np.float32, rmlx_kv.F16: np.uint16, rmlx_kv.BF16: np.uint16}


def _arrays(L, H, S, D, dt, seed):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((2, L, H, S, D), dtype=np.float32)
    t = torch.from_numpy(x).to(TORCH_DT[dt])
    if dt == rmlx_kv.F32:
        return t[0].numpy(), t[1].numpy(), t
    return t[0].view(torch.int16).numpy().view(np.uint16), t[1].view(torch.int16).numpy().view(np.uint16), t


def _as_reference(t, L, H, S, head_offset=0):
    """The tensors save_prompt_cache writes (prompt_cache.rs:76-96)."""
    out = {}
    if S == 0:
        return out
    for l in range(L):
        for h in range(H):
            out[f"layer_{l}_head_{head_offset + h}_keys"] = t[0, l, h].contiguous()
            out[f"layer_{l}_head_{head_offset + h}_values"] = t[1, l, h].contiguous()
    return out


@pytest.mark.parametrize("dt", [rmlx_kv.BF16, rmlx_kv.F16, rmlx_kv.F32])
@pytest.mark.parametrize("meta", [None, {"model": "llama-3.1-8b"}, {"note": "quote \" backslash \\ tab\t é"}])
def test_bytes_match_safetensors(tmp_path, dt, meta):
    L, H, S, D = 12, 3, 5, 64  # 12 layers: names sort "layer_10" before "layer_2"
    k, v, t = _arrays(L, H, S, D, dt, 1)
    path = tmp_path / "c.safetensors"
    pc.write_prompt_cache(path, k, v, dt, metadata=meta)
    assert path.read_bytes() == st.save(_as_reference(t, L, H, S), metadata=meta)


def test_head_offset_names_and_empty_cache(tmp_path):
    k, v, t = _arrays(2, 2, 3, 64, rmlx_kv.BF16, 2)
    p = tmp_path / "shard.safetensors"
    pc.write_prompt_cache(p, k, v, rmlx_kv.BF16, head_offset=4)
    assert p.read_bytes() == st.save(_as_reference(t, 2, 2, 3, head_offset=4))
    e = tmp_path / "empty.safetensors"
    z = np.zeros((2, 2, 0, 64), np.uint16)
    pc.write_prompt_cache(e, z, z, rmlx_kv.BF16, metadata={"a": "b"})
    assert e.read_bytes() == st.save({}, metadata={"a": "b"})
    info = pc.prompt_cache_info(e)
    assert info["seq_len"] == 0 and info["dtype"] == -1 and info["metadata"] == {"a": "b"}
    # as load_prompt_cache (max index starts at 0), an empty file reads as 1 layer x 1 head
    assert (info["num_layers"], info["num_kv_heads"]) == (1, 1)


@pytest.mark.parametrize("dt", [rmlx_kv.BF16, rmlx_kv.F32])
def test_read_files_written_by_safetensors(tmp_path, dt):
    L, H, S, D = 3, 8, 37, 128
    k, v, t = _arrays(L, H, S, D, dt, 3)
    p = tmp_path / "ref.safetensors"
    meta = {"model": "x", "tokenizer": "y", "n": "3"}
    st.save_file(_as_reference(t, L, H, S), str(p), metadata=meta)
    info = pc.prompt_cache_info(p)
    assert info == {"num_layers": L, "num_kv_heads": H, "seq_len": S, "head_dim": D, "dtype": dt, "metadata": meta}
    rk, rv = pc.read_prompt_cache(p, L, H, D, dt)
    np.testing.assert_array_equal(rk, k)
    np.testing.assert_array_equal(rv, v)
    # a shard of the heads (a pool holding heads 4..7)
    sk, sv = pc.read_prompt_cache(p, L, 4, D, dt, head_offset=4)
    np.testing.assert_array_equal(sk, k[:, 4:])
    np.testing.assert_array_equal(sv, v[:, 4:])
    # a cache with more layers than the file: the file's layers are read
    mk, _ = pc.read_prompt_cache(p, L + 2, H, D, dt)
    np.testing.assert_array_equal(mk, k)


def test_roundtrip_through_own_writer(tmp_path):
    k, v, _ = _arrays(4, 2, 100, 128, rmlx_kv.F16, 4)
    p = tmp_path / "rt.safetensors"
    pc.write_prompt_cache(p, k, v, rmlx_kv.F16, metadata={"a": "1", "b": "2"})
    rk, rv = pc.read_prompt_cache(p, 4, 2, 128, rmlx_kv.F16)
    np.testing.assert_array_equal(rk, k)
    np.testing.assert_array_equal(rv, v)
    assert pc.prompt_cache_info(p)["metadata"] == {"a": "1", "b": "2"}
    loaded = st.load_file(str(p))  # the library reads our file too
    np.testing.assert_array_equal(loaded["layer_3_head_1_values"].view(torch.int16).numpy().view(np.uint16), v[3, 1])


def test_rejections(tmp_path):
    L, H, S, D = 2, 2, 4, 64
    k, v, t = _arrays(L, H, S, D, rmlx_kv.BF16, 5)
    good = tmp_path / "g.safetensors"
    pc.write_prompt_cache(good, k, v, rmlx_kv.BF16)
    with pytest.raises(rmlx_kv.RmlxError, match="dtype"):
        pc.read_prompt_cache(good, L, H, D, rmlx_kv.F16)
    with pytest.raises(rmlx_kv.RmlxError, match="head_dim"):
        pc.read_prompt_cache(good, L, H, 128, rmlx_kv.BF16)
    with pytest.raises(rmlx_kv.RmlxError, match="layers"):
        pc.read_prompt_cache(good, 1, H, D, rmlx_kv.BF16)
    with pytest.raises(rmlx_kv.RmlxError, match="lacks"):
        pc.read_prompt_cache(good, L, 3, D, rmlx_kv.BF16)  # head 2 is not in the file
    bad = tmp_path / "b.safetensors"
    st.save_file({"layer_0_head_0_keys": torch.zeros(2, 64, dtype=torch.bfloat16),
                  "weights": torch.zeros(2, dtype=torch.bfloat16)}, str(bad))
    with pytest.raises(rmlx_kv.RmlxError, match="not layer_"):
        pc.prompt_cache_info(bad)
    mixed = tmp_path / "m.safetensors"
    st.save_file({"layer_0_head_0_keys": torch.zeros(2, 64, dtype=torch.bfloat16),
                  "layer_0_head_0_values": torch.zeros(3, 64, dtype=torch.bfloat16)}, str(mixed))
    with pytest.raises(rmlx_kv.RmlxError, match="shapes"):
        pc.prompt_cache_info(mixed)
    trunc = tmp_path / "t.safetensors"
    trunc.write_bytes(good.read_bytes()[:-10])
    with pytest.raises(rmlx_kv.RmlxError, match="data_offsets"):
        pc.prompt_cache_info(trunc)
    junk = tmp_path / "j.safetensors"
    junk.write_bytes(b"\xff" * 16)
    with pytest.raises(rmlx_kv.RmlxError, match="header"):
        pc.prompt_cache_info(junk)
    with pytest.raises(rmlx_kv.RmlxError, match="cannot open"):
        pc.prompt_cache_info(tmp_path / "missing.safetensors")


def test_trim_prompt_cache():
    """prompt_cache.rs:265-281 (test_trim_prompt_cache) on block tables."""
    m = rmlx_kv.PagedCacheManager(4, 64)
    seqs = SequenceBlocks(m, 4, [10, 10])
    assert pc.can_trim_prompt_cache(seqs)
    held = [list(t) for t in seqs.tables]
    freed = pc.trim_prompt_cache(seqs, 3)  # 10 -> 7 tokens: 3 -> 2 blocks of 4
    assert seqs.lens == [7, 7] and freed == [held[0][2], held[1][2]] and m.num_free_blocks() == 64 - 4
    freed = pc.trim_prompt_cache(seqs, 100)
    assert seqs.lens == [0, 0] and len(freed) == 4 and m.num_free_blocks() == 64
    assert not pc.can_trim_prompt_cache(seqs)


def test_trim_keeps_shared_blocks_of_a_fork():
    m = rmlx_kv.PagedCacheManager(4, 16)
    seqs = SequenceBlocks(m, 4, [9, 0])
    seqs.fork(0, 1)
    seqs.trim(1, 6)  # the branch keeps 3 tokens: block 0 stays shared
    assert seqs.lens == [9, 3] and m.ref_count(seqs.tables[0][0]) == 2
    assert all(m.ref_count(b) == 1 for b in seqs.tables[0][1:])
