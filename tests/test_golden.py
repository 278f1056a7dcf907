"""The committed golden fixtures (tests/golden/golden.json) against the
oracle and against this package's host-side code (no GPU).

Each case's inputs are rebuilt from its seed and must hash to the recorded
input digest first, so a change in numpy's random streams reads as such
and not as a wrong result."""
import json
import os
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))

import cases as C  # noqa: E402
import make_golden  # noqa: E402
import oracle as orc  # noqa: E402
import rmlx_kv  # noqa: E402

GOLD = json.load(open(os.path.join(HERE, "golden", "golden.json")))


@pytest.fixture(scope="module")
def derived():
    return make_golden.compute(orc)


@pytest.mark.parametrize("section", ["paged", "quant", "copy", "hash", "admit", "qcache"])
def test_oracle_reproduces_golden(derived, section):
    assert derived[section] == GOLD[section]


def test_golden_chain_hashes_follow_definition():
    """First blocks of the bs-16 case, recomputed from the hash definition
    (XXH64 of le64(parent) || le32(tokens), seed 0) one by one."""
    toks, cu, roots = C.hash_inputs(16)
    want = GOLD["hash"]["bs16"]["hashes"]
    cub = GOLD["hash"]["bs16"]["cu_blocks"]
    for r in range(len(cu) - 1):
        parent = int(roots[r])
        for b in range(cub[r + 1] - cub[r]):
            lo, hi = int(cu[r]) + 16 * b, min(int(cu[r]) + 16 * (b + 1), int(cu[r + 1]))
            msg = parent.to_bytes(8, "little") + toks[lo:hi].astype("<u4").tobytes()
            parent = orc.xxh64(msg, 0)
            assert f"{parent:016x}" == want[cub[r] + b]


@pytest.mark.parametrize("name,seed,budget", C.ADMIT)
def test_product_admission_matches_golden(name, seed, budget):
    g = GOLD["admit"][name]
    toks, cu = C.prefix_requests(seed)
    assert C.sha(toks, cu) == g["inputs"]
    h, cub = orc.hash_chains(toks, cu, np.zeros(len(cu) - 1, np.uint64), 16)
    m, p = rmlx_kv.PagedCacheManager(16, g["pool_blocks"]), rmlx_kv.PrefixCacheManager(g["pool_blocks"])
    ids, ev, st = rmlx_kv.prefix_admit(m, p, toks, cu, h, cub)
    assert ids.astype(np.int64).tolist() == g["block_ids"]
    assert ev.astype(np.int64).tolist() == g["evicted"]
    assert st == g["stats"]


def test_golden_inputs_are_stable():
    for name, L, H, D, bs, N, dt, lens, new, seed in C.PAGED:
        bt, calls, _ = C.paged_inputs(L, H, D, bs, N, dt, lens, new, seed)
        assert C.sha(bt, *[a for c in calls for a in c]) == GOLD["paged"][name]["inputs"], name
