"""Prompt cache files (crates/rmlx-serve-cache/src/prompt_cache.rs).

``save_prompt_cache`` / ``load_prompt_cache`` keep the reference's file:
a safetensors file with one ``[seq_len, head_dim]`` tensor per (layer, head)
named ``layer_{l}_head_{h}_{keys|values}`` and optional string metadata.
Here the cache is a sequence's blocks in a device pool; the host-array
forms (``write_prompt_cache`` / ``read_prompt_cache``) take
``[layers, heads, seq_len, head_dim]`` arrays.  ``trim_prompt_cache`` and
``can_trim_prompt_cache`` act on a batch's block tables
(:class:`rmlx_kv.batch.SequenceBlocks`), where a sequence's length lives.
"""
from __future__ import annotations

import ctypes as C
import json
import os
from typing import Dict, List, Optional, Sequence

import numpy as np

from . import _lib
from ._lib import check, lib

_ESIZE = {_lib.F32: 4, _lib.F16: 2, _lib.BF16: 2}


def _meta(metadata: Optional[Dict[str, str]]):
    items = list((metadata or {}).items())
    keys = (C.c_char_p * max(len(items), 1))(*[k.encode() for k, _ in items])
    vals = (C.c_char_p * max(len(items), 1))(*[v.encode() for _, v in items])
    return keys, vals, len(items)


def _path(path) -> bytes:
    return os.fsencode(os.fspath(path))


def prompt_cache_info(path) -> dict:
    """Layers, heads (largest index + 1), seq_len, head_dim, dtype (-1 when
    empty) and metadata of a prompt cache file."""
    L, H, S, D, dt = (C.c_int32() for _ in range(5))
    n = C.c_size_t()
    check(lib.rmlx_prompt_cache_info(_path(path), C.byref(L), C.byref(H), C.byref(S), C.byref(D), C.byref(dt), None,
                                     0, C.byref(n)))
    buf = C.create_string_buffer(n.value + 1)
    check(lib.rmlx_prompt_cache_info(_path(path), C.byref(L), C.byref(H), C.byref(S), C.byref(D), C.byref(dt), buf,
                                     n.value + 1, C.byref(n)))
    meta = json.loads(buf.value.decode()) if n.value else None
    return {"num_layers": L.value, "num_kv_heads": H.value, "seq_len": S.value, "head_dim": D.value,
            "dtype": dt.value, "metadata": meta}


def write_prompt_cache(path, keys: np.ndarray, values: np.ndarray, dtype: int, head_offset: int = 0,
                       metadata: Optional[Dict[str, str]] = None) -> None:
    """keys/values: [layers, heads, seq_len, head_dim] arrays holding the
    storage bits of `dtype` (uint16 for F16/BF16, float32 for F32)."""
    k = np.ascontiguousarray(keys)
    v = np.ascontiguousarray(values)
    if k.shape != v.shape or k.ndim != 4:
        raise ValueError("keys and values must be [layers, heads, seq_len, head_dim] of one shape")
    if k.itemsize != _ESIZE[dtype] or v.itemsize != _ESIZE[dtype]:
        raise ValueError("array element size does not match dtype")
    mk, mv, nm = _meta(metadata)
    L, H, S, D = k.shape
    check(lib.rmlx_prompt_cache_write(_path(path), L, H, head_offset, S, D, dtype, k.ctypes.data, v.ctypes.data, mk,
                                      mv, nm))


def read_prompt_cache(path, num_layers: int, num_kv_heads: int, head_dim: int, dtype: int, head_offset: int = 0):
    """(keys, values) as [layers in the file, num_kv_heads, seq_len, head_dim]
    arrays of dtype's storage bits, for heads [head_offset, head_offset +
    num_kv_heads)."""
    info = prompt_cache_info(path)
    S, L = info["seq_len"], min(info["num_layers"], num_layers)
    npdt = np.float32 if dtype == _lib.F32 else np.uint16
    k = np.zeros((max(L, 1), num_kv_heads, S, head_dim), dtype=npdt)
    v = np.zeros_like(k)
    got = C.c_int32()
    check(lib.rmlx_prompt_cache_read(_path(path), num_layers, num_kv_heads, head_offset, head_dim, dtype,
                                     k.ctypes.data, v.ctypes.data, k.nbytes, C.byref(got)))
    if got.value == 0:
        return k[:0], v[:0]
    return k[:info["num_layers"]], v[:info["num_layers"]]


def save_prompt_cache(path, pool, block_ids: Sequence[int], seq_len: int,
                      metadata: Optional[Dict[str, str]] = None, stream=None) -> None:
    """prompt_cache.rs:63-127: the sequence held in `block_ids` (block-table
    order) of every layer of `pool`."""
    from .pool import _stream
    ids = np.ascontiguousarray(np.asarray(block_ids, dtype=np.int32))
    mk, mv, nm = _meta(metadata)
    check(lib.rmlx_prompt_cache_save(pool.handle, ids.ctypes.data_as(_lib.i32p), len(ids), seq_len, _path(path),
                                     mk, mv, nm, _stream(stream, pool.device)))


def load_prompt_cache(path, pool, block_ids: Sequence[int], stream=None) -> int:
    """prompt_cache.rs:137-210: the file's rows into the caller's blocks
    (ceil(seq_len / block_size) of them); returns seq_len."""
    from .pool import _stream
    ids = np.ascontiguousarray(np.asarray(block_ids, dtype=np.int32))
    got = C.c_int32()
    check(lib.rmlx_prompt_cache_load(pool.handle, _path(path), ids.ctypes.data_as(_lib.i32p), len(ids), C.byref(got),
                                     _stream(stream, pool.device)))
    return got.value


def trim_prompt_cache(seqs, n: int, which: Optional[List[int]] = None) -> List[int]:
    """prompt_cache.rs:218-226: drop the last `n` tokens of each sequence
    (all, or those in `which`) of a SequenceBlocks; blocks that no longer
    hold a token are released.  Returns the freed block ids."""
    freed = []
    for s in (range(len(seqs.lens)) if which is None else which):
        freed += seqs.trim(s, n)
    return freed


def can_trim_prompt_cache(seqs) -> bool:
    """prompt_cache.rs:231-233: some sequence holds a token."""
    return any(n > 0 for n in seqs.lens)
