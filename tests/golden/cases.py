"""Seeded inputs of the golden cases (shared by make_golden.py and the
tests that check against golden.json).

Every case is rebuilt from its seed here; golden.json records a SHA-256 of
the inputs (so a change in numpy's random streams is caught rather than
mistaken for a wrong result) and of every output.
"""
import hashlib

import numpy as np

F32, F16, BF16 = 0, 1, 2
ESIZE = {F32: 4, F16: 2, BF16: 2}


def sha(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def bits_of(x: np.ndarray, dt: int) -> np.ndarray:
    """f32 -> storage bits of dt, round-to-nearest-even (numpy only)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    if dt == F32:
        return x
    if dt == F16:
        return x.astype(np.float16).view(np.uint16)
    u = x.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    nan = np.isnan(x)
    r[nan] = 0x7FC0
    return r


# Paged append + gather cases: (name, L, H, D, bs, N, dtype, prompt lengths, new tokens, seed)
PAGED = [
    ("config1_fp16", 1, 8, 128, 16, 256, F16, [37, 128, 255, 512], 1, 101),
    ("ragged_bf16", 2, 2, 64, 16, 64, BF16, [0, 1, 16, 17, 100, 15], 2, 102),
    ("f32_bs8", 1, 3, 32, 8, 40, F32, [5, 64, 9], 3, 103),
]

# Quantised pool cases: (name, L, H, D, bs, N, dtype, bits, group, meta dtype, lens, new tokens, seed)
QUANT = [
    ("q8_llama_f16meta", 1, 8, 128, 16, 128, BF16, 8, 64, F16, [37, 128, 255, 300], 1, 111),
    ("q4_llama_f16meta", 1, 8, 128, 16, 128, BF16, 4, 64, F16, [37, 128, 255, 300], 1, 112),
    ("q8_f32meta_g32", 2, 2, 128, 16, 32, F16, 8, 32, F32, [1, 17, 40], 2, 113),
    ("q4_f32meta_g8", 1, 1, 64, 8, 16, BF16, 4, 8, F32, [9, 30], 2, 114),
]


def block_tables(rng, lens, bs, num_blocks, extra):
    need = [(int(n) + extra + bs - 1) // bs for n in lens]
    perm = rng.permutation(num_blocks).astype(np.int32)
    bt = np.zeros((len(lens), max(max(need), 1)), dtype=np.int32)
    o = 0
    for s, n in enumerate(need):
        bt[s, :n] = perm[o:o + n]
        o += n
    return bt


def paged_inputs(L, H, D, bs, N, dt, lens, new, seed, outliers=0.0):
    """Block table, then one batch of rows per append call: the prompt
    tokens of every sequence, then `new` single-token decode steps.
    Rows are [L, T, H, D] in dt's storage bits; values N(0,1) (with a
    fraction `outliers` scaled x8)."""
    rng = np.random.default_rng(seed)
    lens = np.asarray(lens, dtype=np.int64)
    bt = block_tables(rng, lens, bs, N, new)
    calls = []
    positions = [[(s, p) for s in range(len(lens)) for p in range(int(lens[s]))]]
    positions += [[(s, int(lens[s]) + i) for s in range(len(lens))] for i in range(new)]
    for pos in positions:
        T = len(pos)
        kv = []
        for _ in range(2):
            x = rng.standard_normal((L, T, H, D), dtype=np.float32)
            if outliers:
                x = np.where(rng.random(x.shape) < outliers, x * 8.0, x).astype(np.float32)
            kv.append(bits_of(x, dt))
        slots = np.array([int(bt[s, p // bs]) * bs + p % bs for s, p in pos], dtype=np.int32)
        calls.append((kv[0], kv[1], slots))
    final = (lens + new).astype(np.int32)
    return bt, calls, final


def copy_inputs():
    """Pool bytes of a 4-layer bf16 pool and copy pairs.  The destination
    set does not meet the source set (the copy contract: the pairs run in
    parallel, so a chain would have no defined result)."""
    rng = np.random.default_rng(121)
    L, H, D, bs, N = 4, 8, 128, 16, 64
    tile = bs * D * 2
    data = rng.integers(0, 256, size=N * L * 2 * H * tile, dtype=np.uint8)
    src = np.array([3, 7, 9, 0, 63, 20], dtype=np.int32)
    dst = np.array([10, 11, 40, 62, 1, 12], dtype=np.int32)
    return (L, H, D, bs, N), data, src, dst


HASH_LENS = [0, 1, 15, 16, 17, 33, 2048, 100, 64]


def hash_inputs(bs):
    rng = np.random.default_rng(131)
    cu = np.zeros(len(HASH_LENS) + 1, dtype=np.int64)
    cu[1:] = np.cumsum(HASH_LENS)
    toks = rng.integers(0, 128256, size=int(cu[-1]), dtype=np.uint32)
    roots = rng.integers(0, 2 ** 63, size=len(HASH_LENS), dtype=np.uint64)
    roots[0] = 0
    return toks, cu, roots


def prefix_requests(seed, n_req=64, n_prefix=4, prefix_len=256, suffix=(16, 128), unique=(64, 512), vocab=128256,
                    shared=0.6):
    """The prefix-caching workload's request mix, scaled down."""
    rng = np.random.default_rng(seed)
    prefixes = [rng.integers(0, vocab, size=prefix_len, dtype=np.uint32) for _ in range(n_prefix)]
    reqs = []
    for _ in range(n_req):
        if rng.random() < shared:
            p = prefixes[int(rng.integers(n_prefix))]
            s = rng.integers(0, vocab, size=int(rng.integers(suffix[0], suffix[1] + 1)), dtype=np.uint32)
            reqs.append(np.concatenate([p, s]))
        else:
            reqs.append(rng.integers(0, vocab, size=int(rng.integers(unique[0], unique[1] + 1)), dtype=np.uint32))
    cu = np.zeros(n_req + 1, dtype=np.int64)
    cu[1:] = np.cumsum([len(r) for r in reqs])
    return np.concatenate(reqs).astype(np.uint32), cu


ADMIT = [("admit_30pct", 201, 0.3), ("admit_5pct", 202, 0.05)]

# Flat QuantizedKVCache cases: (name, layers, heads, head_dim, bits, group, seed)
QCACHE = [("qc8_g64", 2, 8, 128, 8, 64, 301), ("qc4_g5", 2, 3, 10, 4, 5, 302), ("qc4_g64_d32", 2, 1, 32, 4, 64, 303)]
QCACHE_STEPS = [5, 1, 1, 3]


def qcache_appends(L, H, D, gs, seed):
    """Append calls (layer, keys, values, tokens).  With group > head_dim a
    second append would leave a partial group mid-stream, which the
    reference's dequantize refuses, so that case appends once."""
    rng = np.random.default_rng(seed)
    out = []
    for T in (QCACHE_STEPS if gs <= D else [1]):
        for layer in range(L):
            k = rng.standard_normal(H * T * D).astype(np.float32)
            v = (rng.standard_normal(H * T * D) * 3).astype(np.float32)
            out.append((layer, k, v, T))
    return out
