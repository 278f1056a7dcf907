"""Oracle pinning for the quantiser and the chain hash (CPU only).

* quantized_cache.rs:299-387 restated against the oracle;
* known-answer codes derived from those tests' inputs by the reference's
  formula (quantize_group, quantized_cache.rs:232-273);
* XXH64 published test values (the chain hash's mixing function).
"""
import numpy as np
import pytest

import oracle as orc


def _hexf(x):
    return float(np.float32(x)).hex()


def test_known_answer_8bit_halves():
    b, s, z = orc.quantize_group([0, .5, 1, 1.5, 2, 2.5, 3, 3.5], 8)
    assert list(b) == [0, 36, 73, 109, 146, 182, 219, 255]
    assert _hexf(s) == "0x1.c1c1c20000000p-7" and z == 0.0


def test_known_answer_4bit_packing_low_nibble_first():
    b, s, z = orc.quantize_group(list(range(8)), 4)
    assert [int(x) for x in b] == [0x20, 0x64, 0xB9, 0xFD]
    assert _hexf(s) == "0x1.ddddde0000000p-2" and z == 0.0


def test_known_answer_constant_group():
    b, s, z = orc.quantize_group([42.0] * 8, 8)
    assert list(b) == [0] * 8 and s == 1.0 and z == 42.0


def test_known_answer_8bit_integers():
    b, s, _ = orc.quantize_group(list(range(8)), 8)
    assert list(b) == [0, 36, 73, 109, 146, 182, 219, 255]
    assert _hexf(s) == "0x1.c1c1c20000000p-6"


def test_odd_4bit_group_pads_high_nibble():  # quantized_cache.rs:261-265
    b, s, z = orc.quantize_group([0.0, 1.0, 2.0], 4)
    assert len(b) == 2 and (int(b[1]) >> 4) == 0
    # dequantize_group emits two values per byte (:284-292): 4 values back
    assert len(orc.dequantize_group(b, s, z, 4)) == 4


def test_8bit_roundtrip():  # :313-325
    data = [0.0, 0.5, 1.0, 1.5, 2.0, 2.5, 3.0, 3.5]
    b, s, z = orc.quantize_group(data, 8)
    rec = orc.dequantize_group(b, s, z, 8)
    assert len(rec) == len(data) and np.abs(np.array(data) - rec).max() < 0.02


def test_4bit_roundtrip():  # :328-341
    data = [float(i) for i in range(8)]
    b, s, z = orc.quantize_group(data, 4)
    rec = orc.dequantize_group(b, s, z, 4)
    assert len(rec) == 8 and np.abs(np.array(data) - rec).max() < 0.6


def test_append_and_retrieve():  # :344-365
    c = orc.QuantizedKVCache(1, 1, 8, 8, 8)
    keys = np.arange(8, dtype=np.float32)
    c.append(0, keys, keys * 10, 1)
    assert c.seq_len() == 1
    dk = c.get_keys_dequantized(0)
    assert len(dk) == 8 and np.abs(dk - keys).max() < 0.1


def test_constant_values():  # :368-380
    b, s, z = orc.quantize_group([42.0] * 8, 8)
    assert np.abs(orc.dequantize_group(b, s, z, 8) - 42.0).max() < 0.01


def test_invalid_bits():  # :383-386 (should_panic "bits must be 4 or 8")
    with pytest.raises(RuntimeError):
        orc.QuantizedKVCache(1, 1, 8, 3, 8)


def test_seq_len_counts_layer0_only():  # :121-126
    c = orc.QuantizedKVCache(2, 1, 8, 8, 8)
    x = np.zeros(8, np.float32)
    c.append(1, x, x, 1)
    assert c.seq_len() == 0
    c.append(0, x, x, 1)
    assert c.seq_len() == 1


@pytest.mark.parametrize("msg,want", [
    (b"", 0xEF46DB3751D8E999),
    (b"a", 0xD24EC4F1A98C6E5B),
    (b"abc", 0x44BC2CF5AD770999),
    (b"Nobody inspects the spammish repetition", 0xFBCEA83C8A378BF1),
])
def test_xxh64_published_values(msg, want):
    assert orc.xxh64(msg) == want


def test_chain_hash_definition():
    """hash[b] = XXH64(le64(parent) || le32(tokens of block b)), parent of
    block 0 = the root; a partial last block hashes only its tokens."""
    toks = np.arange(40, dtype=np.uint32) * 7 + 3
    root = 0x1234_5678_9ABC_DEF0
    got, cub = orc.hash_chains(toks, [0, 40], [root], 16)
    assert list(cub) == [0, 3]
    parent = root
    for b in range(3):
        chunk = toks[b * 16:(b + 1) * 16]
        msg = np.uint64(parent).tobytes() + chunk.astype("<u4").tobytes()
        parent = orc.xxh64(msg)
        assert int(got[b]) == parent
