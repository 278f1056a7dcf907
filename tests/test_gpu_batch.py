"""The batch planner driving a device pool end to end: prompts admitted with
prefix-cache reuse (only the uncached tokens are appended), forks, decode
steps with copy-on-write tile copies, removals into the prefix cache.  Row t
of a sequence holds values that depend on its tokens 0..t (as a model's K/V
do), so every gathered row can be checked against the host's expectation:
a reused or shared block must hold exactly what the sequence would have
written itself."""
import numpy as np
import pytest

import oracle as orc
import rmlx_kv
from helpers import to_dev
from rmlx_kv.batch import KVBatch

pytestmark = pytest.mark.gpu

L, H, D, BS, NB = 2, 2, 64, 4, 160


def _rows(tokens, t0, t1):
    """K and V rows (f32 storage) of positions [t0, t1): a function of the prefix."""
    out_k = np.empty((L, t1 - t0, H, D), np.float32)
    h = 1469598103934665603
    for t, tok in enumerate(tokens[:t1]):
        h = ((h ^ int(tok)) * 1099511628211) & (2 ** 64 - 1)
        if t >= t0:
            rng = np.random.default_rng(h)
            out_k[:, t - t0] = rng.standard_normal((L, H, D), dtype=np.float32)
    return out_k, -out_k


def test_planner_drives_pool(cuda):
    import torch
    pool = rmlx_kv.KVPool(L, H, D, BS, NB, dtype=orc.F32)
    m, p = rmlx_kv.PagedCacheManager(BS, NB), rmlx_kv.PrefixCacheManager(NB)
    batch = KVBatch(m, p, 8)
    rng = np.random.default_rng(90)
    seqs, uid = {}, 0
    base = [rng.integers(0, 9, size=n).tolist() for n in (11, 23)]

    def append(tokens, t0, slots):
        k, v = _rows(tokens, t0, t0 + len(slots))
        pool.append(to_dev(k), to_dev(v), to_dev(np.asarray(slots, np.int32)), len(slots))

    for it in range(60):
        r = rng.random()
        if r < 0.2 and len(seqs) < 8:
            uid += 1
            prompt = base[int(rng.integers(2))][:int(rng.integers(5, 24))] + rng.integers(0, 9, size=2).tolist()
            _, cached, slots = batch.add(uid, prompt)
            if len(slots):
                append(prompt, cached, slots)
            seqs[uid] = list(prompt)
        elif r < 0.3 and seqs and len(seqs) < 8:
            parent = list(seqs)[int(rng.integers(len(seqs)))]
            uid += 1
            batch.fork(parent, uid)
            seqs[uid] = list(seqs[parent])
        elif r < 0.4 and seqs:
            u = list(seqs)[int(rng.integers(len(seqs)))]
            batch.remove(u, cache_prefix=True)
            del seqs[u]
        elif seqs:
            uids = list(seqs)
            toks = rng.integers(0, 9, size=len(uids)).tolist()
            slots, src, dst = batch.step(uids, toks)
            if len(src):
                pool.copy_blocks(to_dev(src), to_dev(dst), len(src))
            for u, tok in zip(uids, toks):
                seqs[u].append(int(tok))
            for i, u in enumerate(uids):
                append(seqs[u], len(seqs[u]) - 1, [slots[i]])
        # every live sequence reads back what it would have written itself
        bt, lens = batch.tables()
        if len(lens) == 0:
            continue
        tot = int(lens.sum()) * H * D
        ok = torch.empty(max(tot, 4), dtype=torch.float32, device=cuda)
        ov = torch.empty_like(ok)
        for layer in range(L):
            pool.gather(layer, to_dev(bt), bt.shape[1], to_dev(lens), len(lens), ok, ov)
            torch.cuda.synchronize()
            gk, gv = ok.cpu().numpy(), ov.cpu().numpy()
            o = 0
            for row in range(len(lens)):
                n = int(lens[row])
                if n == 0:
                    continue
                u = next(x for x in seqs if batch.seq(x)[0] == row)
                k, v = _rows(seqs[u], 0, n)
                np.testing.assert_array_equal(gk[o:o + n * H * D], k[layer].transpose(1, 0, 2).reshape(-1))
                np.testing.assert_array_equal(gv[o:o + n * H * D], v[layer].transpose(1, 0, 2).reshape(-1))
                o += n * H * D
    assert pool.check() == 0
    st = batch.stats()
    assert st["cached_tokens"] > 0 and st["cow_copies"] > 0
    batch.close()
    pool.close()
