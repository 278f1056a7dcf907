"""Restatement of the batch planner's policy (rmlx_kv_batch_*, kv_batch.cc)
over the oracle's block manager, prefix trie and XXH64, for the parity
tests.  Same rows, same allocation order, same references."""
import numpy as np

import oracle as orc


class Exhausted(Exception):
    pass


def chain_hash(parent, toks):
    msg = int(parent).to_bytes(8, "little") + np.asarray(toks, dtype="<u4").tobytes()
    return orc.xxh64(msg, 0)


class BatchModel:
    def __init__(self, mgr, prefix, max_seqs, bs):
        self.m, self.p, self.bs = mgr, prefix, bs
        self.rows = [None] * max_seqs
        self.stats = dict(admitted=0, rejected=0, prompt_tokens=0, cached_tokens=0, new_blocks=0, evictions=0,
                          cow_copies=0)

    def _row_of(self, uid):
        for i, r in enumerate(self.rows):
            if r is not None and r["uid"] == uid:
                return i
        return None

    def _take(self):
        while True:
            b = self.m.allocate()
            if b is not None:
                self.stats["new_blocks"] += 1
                return b
            v = self.p.evict_lru() if self.p is not None else None
            if v is None:
                return None
            self.m.free(v)
            self.stats["evictions"] += 1

    def _cache(self, toks, nfull, ids):
        if self.p is None or nfull <= 0:
            return
        att, rep = self.p.insert_report(np.asarray(toks[:nfull * self.bs], np.uint32), ids[:nfull])
        for b in range(nfull):
            if att[b] or rep[b] >= 0:
                self.m.increment_ref(int(ids[b]))
            if rep[b] >= 0:
                self.m.free(int(rep[b]))

    def add(self, uid, prompt):
        n, bs = len(prompt), self.bs
        if n == 0 or self._row_of(uid) is not None:
            raise ValueError
        r = next((i for i, x in enumerate(self.rows) if x is None), None)
        if r is None:
            raise Exhausted
        nb, nfull = -(-n // bs), n // bs
        hashes, h = [], 0
        for k in range(nfull):
            h = chain_hash(h, prompt[k * bs:(k + 1) * bs])
            hashes.append(h)
        blocks, reuse = [], 0
        if self.p is not None:
            self.p.lookup(np.asarray(prompt[:nfull * bs], np.uint32))
            while reuse < (n - 1) // bs:
                b = self.m.lookup_hash(hashes[reuse])
                if b is None:
                    break
                self.m.increment_ref(b)
                blocks.append(b)
                reuse += 1
        for k in range(reuse, nb):
            b = self._take()
            if b is None:
                for x in blocks:
                    self.m.free(x)
                self.stats["rejected"] += 1
                raise Exhausted
            blocks.append(b)
            self.m.append_tokens(b, np.asarray(prompt[k * bs:min(n, (k + 1) * bs)], np.uint32))
            if k < nfull:
                self.m.register_hash(b, hashes[k])
        self._cache(prompt, nfull, blocks)
        cached = reuse * bs
        slots = [blocks[t // bs] * bs + t % bs for t in range(cached, n)]
        self.rows[r] = dict(uid=uid, blocks=blocks, tokens=list(prompt), hashes=hashes)
        self.stats["admitted"] += 1
        self.stats["prompt_tokens"] += n
        self.stats["cached_tokens"] += cached
        return r, cached, slots

    def fork(self, parent, child):
        i = self._row_of(parent)
        if i is None or self._row_of(child) is not None:
            raise ValueError
        r = next((k for k, x in enumerate(self.rows) if x is None), None)
        if r is None:
            raise Exhausted
        src = self.rows[i]
        for b in src["blocks"]:
            self.m.increment_ref(b)
        self.rows[r] = dict(uid=child, blocks=list(src["blocks"]), tokens=list(src["tokens"]),
                            hashes=list(src["hashes"]))
        return r

    def remove(self, uid, cache):
        i = self._row_of(uid)
        if i is None:
            raise ValueError
        row = self.rows[i]
        if cache:
            self._cache(row["tokens"], len(row["hashes"]), row["blocks"])
        for b in row["blocks"]:
            self.m.free(b)
        self.rows[i] = None

    def step(self, uids, tokens):
        bs = self.bs
        idx = [self._row_of(u) for u in uids]
        if any(i is None for i in idx) or len(set(uids)) != len(uids):
            raise ValueError
        need, got, copies = [], [], {}
        for i in idx:
            row = self.rows[i]
            ln = len(row["tokens"])
            nd = 1 if ln % bs == 0 else 0
            if not nd:
                tail = row["blocks"][-1]
                if self.m.ref_count(tail) - copies.get(tail, 0) > 1:
                    nd = 2
                    copies[tail] = copies.get(tail, 0) + 1
            need.append(nd)
            if nd:
                b = self._take()
                if b is None:
                    for x in got:
                        self.m.free(x)
                    self.stats["new_blocks"] -= len(got)
                    raise Exhausted
                got.append(b)
        slots, src, dst, k = [], [], [], 0
        for i, nd, tok in zip(idx, need, tokens):
            row = self.rows[i]
            ln = len(row["tokens"])
            if nd == 1:
                row["blocks"].append(got[k])
                k += 1
            elif nd == 2:
                s, d = row["blocks"][-1], got[k]
                k += 1
                _, _, toks, _ = self.m.get_block(s)
                self.m.append_tokens(d, np.asarray(toks, np.uint32))
                self.m.free(s)
                row["blocks"][-1] = d
                src.append(s)
                dst.append(d)
                self.stats["cow_copies"] += 1
            b = row["blocks"][-1]
            slots.append(b * bs + ln % bs)
            self.m.append_tokens(b, np.asarray([tok], np.uint32))
            row["tokens"].append(int(tok))
            if (ln + 1) % bs == 0:
                parent = row["hashes"][-1] if row["hashes"] else 0
                h = chain_hash(parent, row["tokens"][ln + 1 - bs:ln + 1])
                row["hashes"].append(h)
                self.m.register_hash(b, h)
        return slots, src, dst

    def tables(self):
        nr = max([i + 1 for i, r in enumerate(self.rows) if r is not None] + [0])
        mb = max([len(r["blocks"]) for r in self.rows if r is not None] + [0])
        bt = np.zeros((nr, max(mb, 1)), np.int32)
        lens = np.zeros(nr, np.int32)
        for i in range(nr):
            r = self.rows[i]
            if r is not None:
                bt[i, :len(r["blocks"])] = r["blocks"]
                lens[i] = len(r["tokens"])
        return bt[:, :mb] if mb else bt[:, :0], lens
