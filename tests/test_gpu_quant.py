"""GPU parity: group-affine quantise-on-append and dequantise-on-gather.

Codes, scales and zeros must be bit-identical to the oracle's restatement of
quantize_group (quantized_cache.rs:232-273); dequantised rows must be
bit-identical to dequantize_group's f32 `code * scale + zero`
(quantized_cache.rs:278-296) rounded to the output type, i.e. within 0.5 ulp
of the reference's f32 value.  With f16 metadata the codes are still exact,
the dequantised rows are bit-identical to the oracle's `code * scale16 +
zero16`, and their distance from the f32-metadata value is measured in f16
ulps of the group's magnitude against a stated bound.
"""
import numpy as np
import pytest

import oracle as orc
import rmlx_kv
from helpers import ESIZE, NP_DT, block_tables, rand_rows, slots_for, to_dev, to_host

pytestmark = pytest.mark.gpu


def run_quant_case(cuda, L, H, D, bs, N, dt, bits, gs, meta, prompt_lens, new_tokens=1, seed=0, outliers=0.01):
    import torch
    rng = np.random.default_rng(seed)
    lens = np.array(prompt_lens, dtype=np.int64)
    bt, _ = block_tables(rng, lens, bs, N, extra=new_tokens)
    g = orc.Geo(L, H, D, bs, N, ESIZE[dt], bits=bits, group_size=gs, meta_bytes=4 if meta == orc.F32 else 2)
    host = np.zeros(g.pool_bytes(), dtype=np.uint8)
    pool = rmlx_kv.KVPool(L, H, D, bs, N, dtype=dt, quant_bits=bits, group_size=gs, meta_dtype=meta)
    assert pool.layout.bytes == host.size

    def append(positions):
        T = len(positions)
        if T == 0:
            return
        k = rand_rows(rng, (L, T, H, D), dt, outliers)
        v = rand_rows(rng, (L, T, H, D), dt, outliers)
        slots = slots_for(bt, bs, positions)
        assert orc.paged_append_quant(host, g, 0, L, k, v, dt, T * H * D, H * D, D, slots) == 0
        pool.append(to_dev(k), to_dev(v), to_dev(slots), T)

    append([(s, p) for s in range(len(lens)) for p in range(lens[s])])
    for step in range(new_tokens):
        append([(s, int(lens[s]) + step) for s in range(len(lens))])
    assert pool.check() == 0
    np.testing.assert_array_equal(pool.read(), host)  # codes + meta bit-exact

    final = (lens + new_tokens).astype(np.int32)
    tot = int(final.sum()) * H * D
    npdt = NP_DT[dt]
    ok = torch.empty(max(tot * ESIZE[dt], 16), dtype=torch.uint8, device=cuda)
    ov = torch.empty_like(ok)
    bt_d, lens_d = to_dev(bt), to_dev(final)
    for layer in range(L):
        ek = np.zeros(tot, dtype=npdt)
        ev = np.zeros(tot, dtype=npdt)
        assert orc.paged_gather_dequant(host, g, layer, bt, bt.shape[1], final, ek, ev, dt) == 0
        pool.gather(layer, bt_d, bt.shape[1], lens_d, len(final), ok, ov)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(to_host(ok, npdt)[:tot], ek)
        np.testing.assert_array_equal(to_host(ov, npdt)[:tot], ev)
    assert pool.check() == 0
    pool.close()


@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("meta", [orc.F32, orc.F16])
def test_llama_shape_small_batch(cuda, bits, meta):
    """8 heads x 128, group 64, bf16, 1% outliers x8 (the quantised-store config), small batch."""
    run_quant_case(cuda, 2, 8, 128, 16, 128, orc.BF16, bits, 64, meta, [37, 128, 255, 300], seed=11)


@pytest.mark.parametrize("dt", [orc.F32, orc.F16])
@pytest.mark.parametrize("gs", [8, 16, 32, 128])
def test_group_sizes_and_dtypes(cuda, dt, gs):
    run_quant_case(cuda, 1, 2, 128, 16, 32, dt, 8 if gs != 16 else 4, gs, orc.F32, [1, 17, 40], seed=12)


def test_4bit_small_groups_split_chunks(cuda):
    """group 8 < 32 codes per 16-byte chunk: per-element group lookup path."""
    run_quant_case(cuda, 1, 1, 64, 8, 16, orc.BF16, 4, 8, orc.F16, [9, 30], new_tokens=2, seed=13)


def test_constant_groups_use_unit_scale(cuda):
    """range == 0 -> scale 1.0, zero = the value, codes 0 (quantized_cache.rs:242, :368-380)."""
    import torch
    L, H, D, bs, N = 1, 1, 64, 4, 4
    pool = rmlx_kv.KVPool(L, H, D, bs, N, dtype=orc.F32, quant_bits=8, group_size=64)
    k = np.full((1, 1, H, D), 42.0, dtype=np.float32)
    pool.append(to_dev(k), to_dev(k), to_dev(np.array([0], dtype=np.int32)), 1)
    raw = pool.read(0, pool.layout.tile_bytes)
    assert not raw[:64].any()
    meta = raw[bs * 64:bs * 64 + 8].view(np.float32)
    assert meta[0] == 1.0 and meta[1] == 42.0
    out = torch.empty(D, dtype=torch.float32, device=cuda)
    out2 = torch.empty_like(out)
    pool.gather(0, to_dev(np.zeros((1, 1), np.int32)), 1, to_dev(np.array([1], np.int32)), 1, out, out2)
    assert (out.cpu().numpy() == 42.0).all()


@pytest.mark.parametrize("bits", [8, 4])
def test_f16_meta_ulp_vs_f32_reference(cuda, bits):
    """fp16 scale/zero on the GPU: bit-exact to the oracle with either
    metadata, and within the stated bound (f16 ulps of the group's largest
    |value|) of the reference's f32 `code * scale + zero`, with the figure
    test_f16_meta_ulp.py reports for the same rows."""
    import torch
    from test_f16_meta_ulp import BOUND, MEASURED, dequant_both, rows, ulp_error
    T, H, D, bs = 8192, 8, 128, 16
    N = T // bs
    x = rows(T, H, D, 0x5EED + 3)
    want32, want16 = dequant_both(bits, T, H, D)
    got = {}
    for meta in (orc.F32, orc.F16):
        pool = rmlx_kv.KVPool(1, H, D, bs, N, dtype=orc.F32, quant_bits=bits, group_size=64, meta_dtype=meta)
        pool.append(to_dev(x), to_dev(x), to_dev(np.arange(T, dtype=np.int32)), T)
        o = torch.empty(T * H * D, dtype=torch.float32, device=cuda)
        pool.gather(0, to_dev(np.arange(N, dtype=np.int32).reshape(1, N)), N, to_dev(np.array([T], np.int32)), 1,
                    o, torch.empty_like(o))
        torch.cuda.synchronize()
        assert pool.check() == 0
        got[meta] = o.cpu().numpy()
        pool.close()
    np.testing.assert_array_equal(got[orc.F32], want32)
    np.testing.assert_array_equal(got[orc.F16], want16)
    e = ulp_error(got[orc.F32], got[orc.F16])
    assert e <= BOUND and e == MEASURED[bits]


# (head_dim, block_size, out dtype, group): every dequant kernel path.
#  r1 = single-round kernel (tasks per row a power of two <= 32, block_size * tasks <= 256);
#  the general kernel: multi-round, shift indexing (tasks per row > 32), division (not a power of two).
DISPATCH = [
    (128, 16, orc.BF16, 64),   # r1
    (64, 8, orc.F32, 32),      # r1, f32 output
    (128, 32, orc.BF16, 64),   # general, 2 rounds per tile
    (128, 16, orc.F32, 64),    # general, f32 output, 2 rounds
    (512, 16, orc.BF16, 128),  # general, 64 tasks per row (shifts)
    (96, 16, orc.F16, 32),     # general, 12 tasks per row (division)
    (96, 4, orc.BF16, 32),     # general, division, short blocks
]


@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("meta", [orc.F16, orc.F32])
@pytest.mark.parametrize("D,bs,dt,gs", DISPATCH)
def test_dequant_dispatch_paths(cuda, bits, meta, D, bs, dt, gs):
    run_quant_case(cuda, 2, 2, D, bs, 48, dt, bits, gs, meta, [1, bs - 1 if bs > 1 else 1, 3 * bs + 5, 70],
                   new_tokens=2, seed=15 + D + bs)
