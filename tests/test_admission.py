"""Prefix-cache admission (rmlx_prefix_admit) against the oracle's
restatement of the same policy, on the prefix-caching workload's shape
scaled down to sizes the oracle's O(trie) eviction scan finishes quickly:
identical block assignments, eviction sequence and statistics, and the
reference-count invariants of the policy."""
import numpy as np
import pytest

import oracle as orc
import rmlx_kv
from helpers import prefix_workload

BS = 16


def _run(n_req, n_prefix, prefix_len, suffix_range, unique_range, budget, seed, vocab=128256):
    rng = np.random.default_rng(seed)
    toks, cu = prefix_workload(rng, n_req, n_prefix, prefix_len, suffix_range, unique_range, vocab)
    roots = np.zeros(n_req, dtype=np.uint64)
    hashes, cub = orc.hash_chains(toks, cu, roots, BS)
    demand = int(cub[-1])
    pool = max(int(budget * demand), 1)
    pm, pp = rmlx_kv.PagedCacheManager(BS, pool), rmlx_kv.PrefixCacheManager(pool)
    om, op = orc.PagedCacheManager(BS, pool), orc.PrefixCacheManager(pool)
    ids_p, ev_p, st_p = rmlx_kv.prefix_admit(pm, pp, toks, cu, hashes, cub)
    ids_o, ev_o, st_o, nev = orc.prefix_admit(om, op, toks, cu, hashes, cub)
    return dict(ids_p=ids_p, ev_p=ev_p, st_p=st_p, ids_o=ids_o, ev_o=ev_o, st_o=st_o, nev=nev, pm=pm, pp=pp, om=om,
                op=op, pool=pool, demand=demand)


@pytest.mark.parametrize("seed,budget", [(0, 0.6), (1, 0.3), (2, 1.2), (3, 0.05)])
def test_admission_matches_oracle(seed, budget):
    r = _run(64, 4, 256, (16, 128), (64, 512), budget, seed)
    np.testing.assert_array_equal(r["ids_p"].astype(np.int64), r["ids_o"])
    assert r["st_p"] == r["st_o"]
    assert len(r["ev_p"]) == r["nev"]
    np.testing.assert_array_equal(r["ev_p"].astype(np.int64), r["ev_o"])
    # what stays allocated is exactly what the prefix cache holds, once each
    assert r["pm"].num_allocated_blocks() == r["pp"].num_blocks() == r["op"].num_blocks()
    assert r["pm"].num_free_blocks() == r["om"].num_free_blocks()
    for b in range(r["pool"]):
        assert r["pm"].ref_count(b) in (0, 1)
    st = r["st_p"]
    assert st["requests"] == 64 and st["admitted"] + st["rejected"] == 64
    assert st["hit_blocks"] + st["new_blocks"] == int((r["ids_p"] >= 0).sum())


def test_shared_prefixes_are_reused():
    """With room for everything, every request after the first of its prefix
    reuses the prefix's full blocks."""
    r = _run(32, 2, 128, (1, 40), (20, 60), 4.0, 7)
    assert r["st_p"]["evictions"] == 0 and r["st_p"]["rejected"] == 0
    assert r["st_p"]["hit_blocks"] > 0


def test_unaligned_prefix_boundaries_and_tiny_pool():
    """Prefix lengths that end mid-block, and a pool too small for the
    largest request (rejections)."""
    r = _run(48, 3, 100, (1, 30), (1, 200), 0.02, 9)
    np.testing.assert_array_equal(r["ids_p"].astype(np.int64), r["ids_o"])
    assert r["st_p"] == r["st_o"] and r["st_p"]["rejected"] > 0
    np.testing.assert_array_equal(r["ev_p"].astype(np.int64), r["ev_o"])


def test_bad_layout_rejected():
    m, p = rmlx_kv.PagedCacheManager(BS, 8), rmlx_kv.PrefixCacheManager(8)
    with pytest.raises(rmlx_kv.RmlxError):
        rmlx_kv.prefix_admit(m, p, np.zeros(20, np.uint32), [0, 20], np.zeros(3, np.uint64), [0, 3])
