"""Seeded workload builders shared by the tests (inputs only; no checking)."""
import numpy as np

import oracle as orc

NP_DT = {orc.F32: np.float32, orc.F16: np.uint16, orc.BF16: np.uint16}
ESIZE = {orc.F32: 4, orc.F16: 2, orc.BF16: 2}


def rand_rows(rng, shape, dt, outliers=0.0):
    """N(0,1) values (optionally 1%-style outliers x8) stored as `dt` bits."""
    x = rng.standard_normal(shape, dtype=np.float32)
    if outliers:
        x = np.where(rng.random(shape) < outliers, x * 8.0, x).astype(np.float32)
    return orc.f32_to_dtype(x, dt)


def block_tables(rng, lens, bs, num_blocks, extra=0):
    """Per-sequence block lists drawn from a seeded permutation of the pool.

    Returns (bt [B, max_blocks] int32 padded with 0, blocks per sequence).
    `extra` reserves room for that many more tokens per sequence.
    """
    need = [(int(L) + extra + bs - 1) // bs for L in lens]
    assert sum(need) <= num_blocks, "pool too small"
    perm = rng.permutation(num_blocks).astype(np.int32)
    width = max(max(need), 1)
    bt = np.zeros((len(lens), width), dtype=np.int32)
    o = 0
    for s, n in enumerate(need):
        bt[s, :n] = perm[o:o + n]
        o += n
    return bt, need


def slots_for(bt, bs, seq_pos):
    """slot = block * bs + offset for each (seq, position) pair."""
    return np.array([int(bt[s, p // bs]) * bs + p % bs for s, p in seq_pos], dtype=np.int32)


def to_dev(a, device="cuda"):
    import torch
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:
        a = a.view(np.int16)
    if a.dtype == np.uint64:
        a = a.view(np.int64)
    if a.dtype == np.uint32:
        a = a.view(np.int32)
    return torch.from_numpy(a.copy()).to(device)


def to_host(t, dtype):
    return t.cpu().numpy().view(dtype)


def prefix_workload(rng, n_req, n_prefix, prefix_len, suffix_range, unique_range, vocab=128256, shared=0.6):
    """Requests for the prefix-caching workload: a fraction `shared` start with
    one of `n_prefix` shared prefixes of `prefix_len` tokens plus a unique
    suffix (length uniform in suffix_range), the rest are unique (length
    uniform in unique_range).  Token ids uniform over `vocab`.
    Returns (tokens uint32, cu_tokens int64)."""
    prefixes = [rng.integers(0, vocab, size=prefix_len, dtype=np.uint32) for _ in range(n_prefix)]
    reqs = []
    for _ in range(n_req):
        if rng.random() < shared:
            p = prefixes[int(rng.integers(n_prefix))]
            suf = rng.integers(0, vocab, size=int(rng.integers(suffix_range[0], suffix_range[1] + 1)), dtype=np.uint32)
            reqs.append(np.concatenate([p, suf]))
        else:
            reqs.append(rng.integers(0, vocab, size=int(rng.integers(unique_range[0], unique_range[1] + 1)),
                                     dtype=np.uint32))
    cu = np.zeros(n_req + 1, dtype=np.int64)
    cu[1:] = np.cumsum([len(r) for r in reqs])
    return np.concatenate(reqs).astype(np.uint32), cu
