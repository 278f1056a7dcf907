"""Writes tests/golden/golden.json: digests (and, where small, the values)
of the oracle's outputs on the seeded cases of cases.py.

The oracle is the CPU restatement of rmlx-serve-cache (oracle/), pinned by
the reference's own unit tests (restated in
tests/test_reference_unit_tests.py), the quantiser's known-answer vectors
and XXH64's published test values.  The reference itself is a Rust crate
and has no toolchain here, so these fixtures freeze the pinned oracle: the
CPU suite re-derives them from the oracle (any drift fails), and the GPU
suite checks the device path against them without running the oracle.

    python tests/golden/make_golden.py          # rewrite golden.json
"""
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(HERE)), "oracle"))

import cases as C  # noqa: E402


def _geo(orc, L, H, D, bs, N, dt, bits=0, gs=64, meta=C.F32):
    if bits:
        return orc.Geo(L, H, D, bs, N, C.ESIZE[dt], bits=bits, group_size=gs, meta_bytes=C.ESIZE[meta])
    return orc.Geo(L, H, D, bs, N, C.ESIZE[dt])


NPDT = {C.F32: np.float32, C.F16: np.uint16, C.BF16: np.uint16}


def paged_case(orc, L, H, D, bs, N, dt, lens, new, seed, bits=0, gs=64, meta=C.F32):
    bt, calls, final = C.paged_inputs(L, H, D, bs, N, dt, lens, new, seed, outliers=0.01 if bits else 0.0)
    g = _geo(orc, L, H, D, bs, N, dt, bits, gs, meta)
    pool = np.zeros(g.pool_bytes(), dtype=np.uint8)
    for k, v, slots in calls:
        T = len(slots)
        if T == 0:
            continue
        ls, ts, hs = T * H * D, H * D, D
        if bits:
            rc = orc.paged_append_quant(pool, g, 0, L, k, v, dt, ls, ts, hs, slots)
        else:
            rc = orc.paged_append(pool, g, 0, L, k, v, ls, ts, hs, slots)
        assert rc == 0
    tot = int(final.sum()) * H * D
    gathers = []
    for layer in range(L):
        ek, ev = np.zeros(tot, dtype=NPDT[dt]), np.zeros(tot, dtype=NPDT[dt])
        if bits:
            assert orc.paged_gather_dequant(pool, g, layer, bt, bt.shape[1], final, ek, ev, dt) == 0
        else:
            assert orc.paged_gather(pool, g, layer, bt, bt.shape[1], final, ek, ev) == 0
        gathers.append([C.sha(ek), C.sha(ev)])
    inputs = C.sha(bt, *[a for c in calls for a in c])
    return {"inputs": inputs, "pool": C.sha(pool), "gather": gathers}


def compute(orc):
    out = {}
    out["paged"] = {name: paged_case(orc, L, H, D, bs, N, dt, lens, new, seed)
                    for name, L, H, D, bs, N, dt, lens, new, seed in C.PAGED}
    out["quant"] = {name: paged_case(orc, L, H, D, bs, N, dt, lens, new, seed, bits, gs, meta)
                    for name, L, H, D, bs, N, dt, bits, gs, meta, lens, new, seed in C.QUANT}
    (L, H, D, bs, N), data, src, dst = C.copy_inputs()
    pool = data.copy()
    assert orc.copy_blocks(pool, _geo(orc, L, H, D, bs, N, C.BF16), src, dst) == 0
    out["copy"] = {"inputs": C.sha(data, src, dst), "pool": C.sha(pool)}
    out["hash"] = {}
    for bs in (16, 1, 5):
        toks, cu, roots = C.hash_inputs(bs)
        h, cub = orc.hash_chains(toks, cu, roots, bs)
        ent = {"inputs": C.sha(toks, cu, roots), "cu_blocks": cub.tolist(), "sha": C.sha(h)}
        if bs == 16:
            ent["hashes"] = [f"{int(x):016x}" for x in h]
        out["hash"][f"bs{bs}"] = ent
    out["admit"] = {}
    for name, seed, budget in C.ADMIT:
        toks, cu = C.prefix_requests(seed)
        h, cub = orc.hash_chains(toks, cu, np.zeros(len(cu) - 1, np.uint64), 16)
        pool_blocks = max(int(budget * int(cub[-1])), 1)
        m, p = orc.PagedCacheManager(16, pool_blocks), orc.PrefixCacheManager(pool_blocks)
        ids, ev, st, nev = orc.prefix_admit(m, p, toks, cu, h, cub)
        out["admit"][name] = {"inputs": C.sha(toks, cu), "pool_blocks": pool_blocks,
                              "block_ids": ids.tolist(), "evicted": ev.tolist(), "stats": st}
    out["qcache"] = {}
    for name, L, H, D, bits, gs, seed in C.QCACHE:
        q = orc.QuantizedKVCache(L, H, D, bits, gs)
        app = C.qcache_appends(L, H, D, gs, seed)
        for layer, k, v, T in app:
            q.append(layer, k, v, T)
        raw, deq = [], []
        for layer in range(L):
            for which in (0, 1):
                raw.append(C.sha(*q.raw(layer, which)))
                deq.append(C.sha(q._get(layer, which)))
        out["qcache"][name] = {"inputs": C.sha(*[a for _, k, v, _ in app for a in (k, v)]), "seq_len": q.seq_len(),
                               "raw": raw, "dequant": deq}
    return out


def main():
    import oracle as orc
    data = compute(orc)
    data["_about"] = ("SHA-256 digests of the oracle's outputs on the seeded cases of tests/golden/cases.py; "
                      "written by tests/golden/make_golden.py")
    with open(os.path.join(HERE, "golden.json"), "w") as f:
        json.dump(data, f, indent=1, sort_keys=True)
        f.write("\n")


if __name__ == "__main__":
    main()
