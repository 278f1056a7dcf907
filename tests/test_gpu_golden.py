"""The device path through the C ABI against the committed golden
fixtures (tests/golden/golden.json): pool bytes, gathered K/V, copied
blocks, chain hashes and the flat quantised cache, all as SHA-256 digests
of bit-exact outputs.  No oracle runs here."""
import json
import os
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))

import cases as C  # noqa: E402
import rmlx_kv  # noqa: E402
from helpers import to_dev  # noqa: E402

GOLD = json.load(open(os.path.join(HERE, "golden", "golden.json")))
NPDT = {C.F32: np.float32, C.F16: np.uint16, C.BF16: np.uint16}

pytestmark = pytest.mark.gpu


def _device_case(cuda, L, H, D, bs, N, dt, lens, new, seed, bits=0, gs=64, meta=C.F32):
    import torch
    bt, calls, final = C.paged_inputs(L, H, D, bs, N, dt, lens, new, seed, outliers=0.01 if bits else 0.0)
    qkw = dict(quant_bits=bits, group_size=gs, meta_dtype=meta) if bits else {}
    pool = rmlx_kv.KVPool(L, H, D, bs, N, dtype=dt, **qkw)
    pool.write(np.zeros(pool.layout.bytes, dtype=np.uint8))
    for k, v, slots in calls:
        if len(slots):
            pool.append(to_dev(k), to_dev(v), to_dev(slots), len(slots))
    tot = int(final.sum()) * H * D
    esz = C.ESIZE[dt]
    ok = torch.empty(max(tot * esz, 16), dtype=torch.uint8, device=cuda)
    ov = torch.empty_like(ok)
    bt_d, lens_d = to_dev(bt), to_dev(final)
    gathers = []
    for layer in range(L):
        pool.gather(layer, bt_d, bt.shape[1], lens_d, len(final), ok, ov)
        torch.cuda.synchronize()
        gathers.append([C.sha(ok.cpu().numpy()[:tot * esz]), C.sha(ov.cpu().numpy()[:tot * esz])])
    assert pool.check() == 0
    out = {"inputs": C.sha(bt, *[a for c in calls for a in c]), "pool": C.sha(pool.read()), "gather": gathers}
    pool.close()
    return out


@pytest.mark.parametrize("case", C.PAGED, ids=[c[0] for c in C.PAGED])
def test_paged_golden(cuda, case):
    name, L, H, D, bs, N, dt, lens, new, seed = case
    assert _device_case(cuda, L, H, D, bs, N, dt, lens, new, seed) == GOLD["paged"][name]


@pytest.mark.parametrize("case", C.QUANT, ids=[c[0] for c in C.QUANT])
def test_quant_golden(cuda, case):
    name, L, H, D, bs, N, dt, bits, gs, meta, lens, new, seed = case
    assert _device_case(cuda, L, H, D, bs, N, dt, lens, new, seed, bits, gs, meta) == GOLD["quant"][name]


def test_copy_golden(cuda):
    (L, H, D, bs, N), data, src, dst = C.copy_inputs()
    pool = rmlx_kv.KVPool(L, H, D, bs, N, dtype=C.BF16)
    pool.write(data)
    pool.copy_blocks(to_dev(src), to_dev(dst), len(src))
    assert pool.check() == 0
    assert {"inputs": C.sha(data, src, dst), "pool": C.sha(pool.read())} == GOLD["copy"]
    pool.close()


@pytest.mark.parametrize("bs", [16, 1, 5])
def test_hash_golden(cuda, bs):
    import torch
    g = GOLD["hash"][f"bs{bs}"]
    toks, cu, roots = C.hash_inputs(bs)
    assert C.sha(toks, cu, roots) == g["inputs"]
    cub = np.array(g["cu_blocks"], dtype=np.int64)
    out = torch.zeros(int(cub[-1]), dtype=torch.int64, device=cuda)
    rmlx_kv.hash_block_chains(to_dev(toks), to_dev(cu), to_dev(roots), len(cu) - 1, bs, to_dev(cub), out)
    got = out.cpu().numpy().view(np.uint64)
    assert C.sha(got) == g["sha"]
    if "hashes" in g:
        assert [f"{int(x):016x}" for x in got] == g["hashes"]


@pytest.mark.parametrize("case", C.QCACHE, ids=[c[0] for c in C.QCACHE])
def test_qcache_golden(cuda, case):
    name, L, H, D, bits, gs, seed = case
    g = GOLD["qcache"][name]
    q = rmlx_kv.QuantizedKVCache(L, H, D, bits, gs)
    app = C.qcache_appends(L, H, D, gs, seed)
    for layer, k, v, T in app:
        q.append(layer, k, v, T)
    raw, deq = [], []
    for layer in range(L):
        for which in (0, 1):
            raw.append(C.sha(*q.raw(layer, which)))
            deq.append(C.sha(q.get_keys_dequantized(layer) if which == 0 else q.get_values_dequantized(layer)))
    assert q.seq_len() == g["seq_len"]
    assert raw == g["raw"] and deq == g["dequant"]
