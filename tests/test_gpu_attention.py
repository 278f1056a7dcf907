"""GPU numerics of the paged decode attention against a float64 reference.

The reference computes softmax(scale * q K^T) V in float64 from the K/V rows
that the gather returns for the same block tables (the gather itself is
bit-exact against the oracle in test_gpu_paged.py).  Tolerances, from the
kernel's arithmetic: scores and sums in f32 from exact products of the
16-bit inputs; the exponentiated scores P are rounded to the pool's type
before P V (relative error 2^-9 for bf16, 2^-12 for f16 per weight), and the
output is rounded to the pool's type.  With |V| <~ 4.5 that bounds the
error by about 4 * 2^-9 * 4.5 = 0.035 (bf16) and 0.005 (f16); the tests use
max-abs 0.03 / 0.004 and an RMS bound ten times tighter.

Quantised pools with group_size >= 16 (8-bit) or >= 32 (4-bit) are read as
codes: the queries are rounded to f16 after division by their row's max
|q| (2^-12), the products of codes and queries are exact, and the weights
P s / smax are rounded to f16 (2^-12) instead of P to the pool's type; the
dequantised rows themselves are never rounded, while the reference reads
them rounded to the pool's type (2^-9 for bf16, 2^-12 for f16).  The same
bounds hold.

Value-range cases (K/V scaled by 1e-3 or 300, or offset by 40) compare with
float64 attention over the oracle's exact f32 dequantisation instead; their
bounds scale with the largest |V|, and the RMS bound adds half an ulp of the
largest output, which the output's own rounding to the pool's type costs.
"""
import numpy as np
import pytest

import oracle as orc
import rmlx_kv
from helpers import ESIZE, block_tables, to_dev

pytestmark = pytest.mark.gpu

TOL = {orc.BF16: (0.03, 0.003), orc.F16: (0.004, 0.0004)}


def _pool(L, H, D, bs, N, dt, seed):
    pool = rmlx_kv.KVPool(L, H, D, bs, N, dtype=dt)
    rng = np.random.default_rng(seed)
    vals = rng.standard_normal(pool.layout.bytes // 2, dtype=np.float32)
    pool.write(orc.f32_to_dtype(vals, dt).view(np.uint8))
    return pool, rng


def _reference(pool, layer, q, G, bt, lens, scale, dt, cuda):
    """float64 attention over the gathered K/V: out [B, H*G, D]."""
    import torch
    H, D = pool.cfg.num_kv_heads, pool.cfg.head_dim
    tot = int(lens.sum())
    ok = torch.empty(max(tot * H * D, 8), dtype=torch.int16, device=cuda)
    ov = torch.empty_like(ok)
    pool.gather(layer, to_dev(bt), bt.shape[1], to_dev(lens.astype(np.int32)), len(lens), ok, ov)
    torch.cuda.synchronize()
    k = orc.dtype_to_f32(ok.cpu().numpy().view(np.uint16)[:tot * H * D], dt).astype(np.float64)
    v = orc.dtype_to_f32(ov.cpu().numpy().view(np.uint16)[:tot * H * D], dt).astype(np.float64)
    return _attend(k, v, q, G, lens, scale, dt, H, D)


def _reference_exact(pool, layer, q, G, bt, lens, scale, dt, bits, gs, meta):
    """float64 attention over the oracle's f32 dequantisation of the pool's
    bytes (the dequantised rows are not rounded to the pool's type)."""
    c = pool.cfg
    H, D = c.num_kv_heads, c.head_dim
    g = orc.Geo(c.num_layers, H, D, c.block_size, c.num_blocks, ESIZE[dt], bits=bits, group_size=gs,
                meta_bytes=4 if meta == orc.F32 else 2)
    host = pool.read()
    tot = int(lens.sum())
    ek, ev = np.zeros(max(tot * H * D, 1), np.float32), np.zeros(max(tot * H * D, 1), np.float32)
    assert orc.paged_gather_dequant(host, g, layer, bt, bt.shape[1], lens.astype(np.int32), ek, ev, orc.F32) == 0
    return _attend(ek[:tot * H * D].astype(np.float64), ev[:tot * H * D].astype(np.float64), q, G, lens, scale, dt,
                   H, D)


def _attend(k, v, q, G, lens, scale, dt, H, D):
    """softmax(scale q K^T) V per sequence and query head in float64, from
    K/V gathered as [sequence][head][token][dim]."""
    qf = orc.dtype_to_f32(q, dt).astype(np.float64).reshape(len(lens), H * G, D)
    out = np.zeros_like(qf)
    o = 0
    for s, n in enumerate(lens):
        n = int(n)
        ks = k[o * H * D:(o + n) * H * D].reshape(H, n, D)
        vs = v[o * H * D:(o + n) * H * D].reshape(H, n, D)
        o += n
        if n == 0:
            continue
        for j in range(H * G):
            sc = ks[j // G] @ qf[s, j] * scale
            p = np.exp(sc - sc.max())
            out[s, j] = (p / p.sum()) @ vs[j // G]
    return out


def run_attn(cuda, L, H, D, bs, N, dt, G, lens, seed, layer=0, extra_tokens=0):
    import torch
    pool, rng = _pool(L, H, D, bs, N, dt, seed)
    lens = np.array(lens, dtype=np.int64)
    bt, _ = block_tables(rng, lens, bs, N)
    q = orc.f32_to_dtype(rng.standard_normal((len(lens), H * G, D), dtype=np.float32), dt)
    scale = 1.0 / np.sqrt(D)
    ws_bytes = pool.attention_workspace_size(G, len(lens), int(lens.sum()) + extra_tokens)
    ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=cuda)
    out = torch.full((len(lens), H * G, D), -7, dtype=torch.int16, device=cuda)
    pool.decode_attention(layer, to_dev(q), G, to_dev(bt), bt.shape[1], to_dev(lens.astype(np.int32)), len(lens),
                          scale, out, ws)
    torch.cuda.synchronize()
    assert pool.check() == 0
    got = orc.dtype_to_f32(out.cpu().numpy().view(np.uint16), dt).astype(np.float64)
    want = _reference(pool, layer, q, G, bt, lens, scale, dt, cuda)
    err = np.abs(got - want)
    mx, rms = TOL[dt]
    assert np.isfinite(got).all()
    assert err.max() <= mx, f"max abs error {err.max()}"
    assert np.sqrt((err ** 2).mean()) <= rms, f"rms error {np.sqrt((err ** 2).mean())}"
    zero = lens == 0
    assert (got[zero] == 0).all()
    pool.close()
    return err


@pytest.mark.parametrize("dt", [orc.BF16, orc.F16])
def test_config1_shape(cuda, dt):
    """8 KV heads x 128, block 16, 4 query heads per KV head, prompts 37/128/255/512 (+1)."""
    run_attn(cuda, 1, 8, 128, 16, 256, dt, 4, [38, 129, 256, 513], seed=60)


@pytest.mark.parametrize("G", [1, 8, 16])
def test_group_sizes(cuda, G):
    run_attn(cuda, 2, 2, 128, 16, 128, orc.BF16, G, [1, 17, 300, 700], seed=61 + G, layer=1)


@pytest.mark.parametrize("bs", [1, 8, 32, 48])
def test_block_sizes(cuda, bs):
    """bs 1 and 8: a 16-token chunk spans several blocks (row-by-row copies);
    32 and 48: several chunks per block."""
    N = 600 // bs + 80
    run_attn(cuda, 1, 2, 128, bs, N, orc.BF16, 4, [3, 16, 31, 257], seed=62 + bs)


@pytest.mark.parametrize("dt", [orc.BF16, orc.F16])
def test_head_dim_64_and_ragged(cuda, dt):
    run_attn(cuda, 1, 4, 64, 16, 256, dt, 2, [0, 1, 15, 16, 17, 255, 256, 257, 1000], seed=63)


def test_long_sequences_many_splits(cuda):
    """8192 and 5000 tokens: 32 and 20 splits combined per query head."""
    run_attn(cuda, 1, 1, 128, 16, 900, orc.BF16, 8, [8192, 5000, 3], seed=64)


def test_many_sequences(cuda):
    rng = np.random.default_rng(65)
    lens = rng.integers(0, 200, size=300).tolist()
    run_attn(cuda, 1, 2, 64, 16, int(sum(lens) // 16 + 400), orc.F16, 4, lens, seed=66)


def test_workspace_too_small_is_flagged(cuda):
    import torch
    pool, rng = _pool(1, 2, 128, 16, 64, orc.BF16, 67)
    lens = np.array([600, 300], dtype=np.int32)
    bt, _ = block_tables(rng, lens, 16, 64)
    q = torch.zeros((2, 8, 128), dtype=torch.bfloat16, device=cuda)
    need = pool.attention_workspace_size(4, 2, 900)
    small = 2 * 4 * (128 + 2) * 4  # one split: 2 KV heads x 4 query heads x (head_dim + max, sum) f32
    assert 0 < small < need
    ws = torch.empty(small, dtype=torch.uint8, device=cuda)
    out = torch.full((2, 8, 128), 3.0, dtype=torch.bfloat16, device=cuda)
    pool.decode_attention(0, q, 4, to_dev(bt), bt.shape[1], to_dev(lens), 2, 0.1, out, ws)
    assert pool.check() & 4
    assert (out.float() == 3.0).all()  # left unwritten
    pool.close()


def test_bad_block_id_flagged(cuda):
    import torch
    pool, rng = _pool(1, 1, 128, 16, 8, orc.BF16, 68)
    bt = np.array([[0, 1, 99]], dtype=np.int32)
    q = torch.zeros((1, 4, 128), dtype=torch.bfloat16, device=cuda)
    ws = torch.empty(pool.attention_workspace_size(4, 1, 40), dtype=torch.uint8, device=cuda)
    out = torch.empty((1, 4, 128), dtype=torch.bfloat16, device=cuda)
    pool.decode_attention(0, q, 4, to_dev(bt), 3, to_dev(np.array([40], np.int32)), 1, 0.1, out, ws)
    assert pool.check() & 2
    pool.close()


def run_attn_quant(cuda, L, H, D, bs, N, dt, G, lens, seed, bits, gs, meta, layer=0, kscale=1.0, vscale=1.0,
                   shift=0.0, exact_ref=False):
    """Quantised pool filled through the quantise-on-append path; the
    reference reads the rows the dequantising gather returns (rounded to the
    pool's type), or with exact_ref the oracle's f32 dequantisation of the
    same pool bytes.  K = kscale N(0,1) + shift, V = vscale N(0,1) + shift,
    and the queries are divided by kscale so that the logits stay of order
    one.  The tolerances grow with the largest |V|, and the RMS bound also
    allows for the output's own rounding to the pool's type."""
    import torch
    from helpers import slots_for
    rng = np.random.default_rng(seed)
    pool = rmlx_kv.KVPool(L, H, D, bs, N, dtype=dt, quant_bits=bits, group_size=gs, meta_dtype=meta)
    pool.write(np.zeros(pool.layout.bytes, np.uint8))
    lens = np.array(lens, dtype=np.int64)
    bt, _ = block_tables(rng, lens, bs, N)
    pos = [(s, p) for s in range(len(lens)) for p in range(int(lens[s]))]
    if pos:
        T = len(pos)
        def vals(sc):
            x = rng.standard_normal((L, T, H, D), dtype=np.float32) * np.float32(sc) + np.float32(shift)
            return orc.f32_to_dtype(x, dt)
        k = vals(kscale)  # N(0,1) at scale 1, shift 0: the tolerance above assumes |V| <~ 4.5
        v = vals(vscale)
        pool.append(to_dev(k), to_dev(v), to_dev(slots_for(bt, bs, pos)), T)
    q = orc.f32_to_dtype(rng.standard_normal((len(lens), H * G, D), dtype=np.float32) / np.float32(kscale), dt)
    sm_scale = 1.0 / np.sqrt(D)
    ws = torch.empty(max(pool.attention_workspace_size(G, len(lens), int(lens.sum())), 16), dtype=torch.uint8,
                     device=cuda)
    out = torch.full((len(lens), H * G, D), -7, dtype=torch.int16, device=cuda)
    pool.decode_attention(layer, to_dev(q), G, to_dev(bt), bt.shape[1], to_dev(lens.astype(np.int32)), len(lens),
                          sm_scale, out, ws)
    torch.cuda.synchronize()
    assert pool.check() == 0
    got = orc.dtype_to_f32(out.cpu().numpy().view(np.uint16), dt).astype(np.float64)
    if exact_ref:
        want = _reference_exact(pool, layer, q, G, bt, lens, sm_scale, dt, bits, gs, meta)
    else:
        want = _reference(pool, layer, q, G, bt, lens, sm_scale, dt, cuda)
    err = np.abs(got - want)
    mx, rms = TOL[dt]
    grow = (4.5 * abs(vscale) + abs(shift)) / 4.5
    out_ulp = (2.0 ** -8 if dt == orc.BF16 else 2.0 ** -11) * np.abs(want).max()  # of the largest output
    assert np.isfinite(got).all()
    assert err.max() <= mx * grow, f"max abs error {err.max()}"
    assert np.sqrt((err ** 2).mean()) <= rms * grow + out_ulp / 2, f"rms error {np.sqrt((err ** 2).mean())}"
    assert (got[lens == 0] == 0).all()
    pool.close()


@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("meta", [orc.F16, orc.F32])
def test_quantised_pool(cuda, bits, meta):
    """8 KV heads x 128, group 64, 4 query heads per KV head; K/V rows as
    the dequantising gather returns them (codes read in place)."""
    run_attn_quant(cuda, 2, 8, 128, 16, 256, orc.BF16, 4, [38, 129, 256, 513, 0, 1000], 70 + bits, bits, 64, meta,
                   layer=1)


@pytest.mark.parametrize("bs,D,gs,dt", [(8, 128, 32, orc.BF16), (1, 64, 16, orc.F16), (32, 64, 64, orc.F16),
                                        (5, 128, 128, orc.BF16), (16, 128, 8, orc.BF16)])
def test_quantised_block_sizes_and_groups(cuda, bs, D, gs, dt):
    """bs 8, 1 and 5: chunks span blocks (row-by-row copies of codes and of
    4-, 8- or 16-byte scale/zero rows); 32: two chunks per block.  Groups of
    8 (both widths) and of 16 at 4 bits are below what the codes kernel
    takes: the kernel that dequantises into a tile serves them."""
    N = 700 // bs + 40
    for bits in (8, 4):
        run_attn_quant(cuda, 1, 2, D, bs, N, dt, 8, [3, 16, 31, 300], 80 + bs + bits, bits, gs, orc.F16)


@pytest.mark.parametrize("kscale,vscale,shift,meta", [(1e-3, 1e-3, 0.0, orc.F32), (1e-3, 1e-3, 0.0, orc.F16),
                                                       (300.0, 300.0, 0.0, orc.F32), (1.0, 1.0, 40.0, orc.F16)])
def test_quantised_value_ranges(cuda, kscale, vscale, shift, meta):
    """K/V far from unit scale (with f16 scale/zero, 1e-3 values give
    scales below f16's normal range) and a large common offset: the
    scale/zero folds and the per-chunk normalisation of the weights keep
    the error relative to |V|.  The reference is the oracle's exact
    dequantisation."""
    for bits in (8, 4):
        run_attn_quant(cuda, 1, 2, 128, 16, 120, orc.BF16, 4, [7, 100, 500], 95 + bits, bits, 64, meta,
                       kscale=kscale, vscale=vscale, shift=shift, exact_ref=True)


@pytest.mark.parametrize("G", [1, 12, 16])
def test_quantised_query_groups(cuda, G):
    """One query head per KV head, and 12 or 16 (two 8-wide head tiles in
    the kernel that reads codes)."""
    for bits in (8, 4):
        run_attn_quant(cuda, 1, 4, 128, 16, 200, orc.BF16, G, [5, 77, 300, 0], 90 + G + bits, bits, 64, orc.F16)


def test_bad_arguments(cuda):
    import torch
    q = torch.zeros(4096, dtype=torch.bfloat16, device=cuda)
    ws = torch.empty(1 << 20, dtype=torch.uint8, device=cuda)
    bt = to_dev(np.zeros((1, 1), np.int32))
    ln = to_dev(np.array([1], np.int32))
    quant = rmlx_kv.KVPool(1, 1, 256, 16, 4, dtype=orc.BF16, quant_bits=8, group_size=64)
    with pytest.raises(rmlx_kv.RmlxError, match="head_dim"):
        quant.decode_attention(0, q, 1, bt, 1, ln, 1, 0.1, q, ws)
    p256 = rmlx_kv.KVPool(1, 1, 256, 16, 4, dtype=orc.BF16)
    with pytest.raises(rmlx_kv.RmlxError, match="head_dim"):
        p256.decode_attention(0, q, 1, bt, 1, ln, 1, 0.1, q, ws)
    p = rmlx_kv.KVPool(1, 1, 128, 16, 4, dtype=orc.BF16)
    with pytest.raises(rmlx_kv.RmlxError, match="q_heads_per_kv"):
        p.decode_attention(0, q, 17, bt, 1, ln, 1, 0.1, q, ws)
    with pytest.raises(rmlx_kv.RmlxError):
        p.decode_attention(3, q, 1, bt, 1, ln, 1, 0.1, q, ws)
    with pytest.raises(rmlx_kv.RmlxError, match="softmax_scale"):
        p.decode_attention(0, q, 1, bt, 1, ln, 1, 0.0, q, ws)
    pf32 = rmlx_kv.KVPool(1, 1, 128, 16, 4, dtype=orc.F32)
    with pytest.raises(rmlx_kv.RmlxError, match="F16 or BF16"):
        pf32.decode_attention(0, q, 1, bt, 1, ln, 1, 0.1, q, ws)
    for x in (quant, p256, p, pf32):
        x.close()
