"""rmlx_qcache_get_dequantized_static: dequantise without allocating.

Callers that must not call cudaMalloc while they run -- an engine that gave
nearly all free GPU memory to its KV pool at start-up, or code on the
per-step path that cannot take the device-wide synchronisation an
allocation may cause -- read a QuantizedKVCache layer back through this
entry point.  It stages the values in a fixed device array the library
holds on every GPU it is loaded on, so its results must equal the oracle's
dequantisation (the reference's `dequantize_data`) and those of the
allocating getters, call after call, even though each call reuses the
array the previous call left behind; and it must not move the device's
free memory.

This file is collected last on purpose, and it does not depend on any
state the other tests leave behind.
"""
import ctypes as C
import os
import re

import numpy as np
import pytest

import oracle as orc
import rmlx_kv
from rmlx_kv import _lib

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _header_max_floats():
    """RMLX_QCACHE_STATIC_MAX_FLOATS as the header defines it."""
    text = open(os.path.join(ROOT, "include", "rmlx_kv.h")).read()
    m = re.search(r"#define\s+RMLX_QCACHE_STATIC_MAX_FLOATS\s+\(\(size_t\)([0-9*\s]+)\)", text)
    assert m, "RMLX_QCACHE_STATIC_MAX_FLOATS not found in include/rmlx_kv.h"
    n = 1
    for f in m.group(1).split("*"):
        n *= int(f)
    return n


MAX_FLOATS = _header_max_floats()

_fn = _lib.lib.rmlx_qcache_get_dequantized_static
_fn.restype = C.c_int
_fn.argtypes = [C.c_void_p, C.c_size_t, C.c_int32, _lib.f32p, C.c_size_t, C.POINTER(C.c_size_t)]


def static_get(q, layer, which):
    n = C.c_size_t()
    _lib.check(_fn(q._h, layer, which, None, 0, C.byref(n)))
    out = np.full(n.value, np.nan, dtype=np.float32)
    _lib.check(_fn(q._h, layer, which, out.ctypes.data_as(_lib.f32p), n.value, C.byref(n)))
    assert n.value == out.size
    return out


def _filled(bits, gs, heads, head_dim, steps, seed, layers=2):
    """The same appends into the product's cache and the oracle's."""
    rng = np.random.default_rng(seed)
    q = rmlx_kv.QuantizedKVCache(layers, heads, head_dim, bits, gs)
    o = orc.QuantizedKVCache(layers, heads, head_dim, bits, gs)
    for T in steps:
        for layer in range(layers):
            k = rng.standard_normal(heads * T * head_dim).astype(np.float32)
            v = (rng.standard_normal(heads * T * head_dim) * 4).astype(np.float32)
            q.append(layer, k, v, T)
            o.append(layer, k, v, T)
    return q, o


@pytest.mark.parametrize("bits", [8, 4])
def test_static_matches_oracle_and_allocating_getters_two_calls_in_a_row(cuda, bits):
    """Bit-exact (the tolerance every dequantisation test here uses)."""
    q, o = _filled(bits, 64, 8, 128, [40, 1, 1, 7], seed=bits)
    # Two calls in a row on the shared array: a large read, then a different
    # layer and side, then the first again.
    a = static_get(q, 0, 0)
    b = static_get(q, 1, 1)
    np.testing.assert_array_equal(a, o.get_keys_dequantized(0))
    np.testing.assert_array_equal(b, o.get_values_dequantized(1))
    np.testing.assert_array_equal(a, q.get_keys_dequantized(0))
    np.testing.assert_array_equal(b, q.get_values_dequantized(1))
    np.testing.assert_array_equal(static_get(q, 0, 0), a)


def test_static_smaller_read_after_larger(cuda):
    big, obig = _filled(8, 32, 8, 128, [64], seed=11)
    small, osmall = _filled(8, 32, 2, 64, [3], seed=12)
    x = static_get(big, 1, 0)
    y = static_get(small, 0, 1)
    np.testing.assert_array_equal(x, obig.get_keys_dequantized(1))
    np.testing.assert_array_equal(y, osmall.get_values_dequantized(0))


def test_static_at_exactly_its_array(cuda):
    """A layer of exactly RMLX_QCACHE_STATIC_MAX_FLOATS values is served."""
    heads, hd = 8, 128
    assert MAX_FLOATS % (heads * hd) == 0
    T = MAX_FLOATS // (heads * hd)
    q, o = _filled(8, 64, heads, hd, [T], seed=21, layers=1)
    got = static_get(q, 0, 1)
    assert got.size == MAX_FLOATS
    np.testing.assert_array_equal(got, o.get_values_dequantized(0))


def test_static_rejects_more_than_its_array(cuda):
    heads, hd = 8, 128
    T = MAX_FLOATS // (heads * hd) + 1
    q = rmlx_kv.QuantizedKVCache(1, heads, hd, 8, 64)
    x = np.zeros(heads * T * hd, dtype=np.float32)
    q.append(0, x, x, T)
    n = C.c_size_t()
    assert _fn(q._h, 0, 0, None, 0, C.byref(n)) == _lib.OK and n.value > MAX_FLOATS
    out = np.empty(n.value, dtype=np.float32)
    rc = _fn(q._h, 0, 0, out.ctypes.data_as(_lib.f32p), n.value, C.byref(n))
    assert rc == _lib.E_BAD_ARG
    assert "static scratch" in _lib.lib.rmlx_last_error().decode()


def test_static_empty_layer(cuda):
    q = rmlx_kv.QuantizedKVCache(2, 1, 8, 8, 8)
    assert static_get(q, 1, 0).size == 0


def test_static_allocates_no_device_memory(cuda):
    """Free device memory is the same before and after static reads of a
    large layer (after one warm-up call, which looks the array's address up);
    the allocating getter on a fresh cache is what moves it."""
    import torch
    heads, hd = 8, 128
    T = MAX_FLOATS // (heads * hd)
    q, _ = _filled(8, 64, heads, hd, [T], seed=31, layers=1)
    static_get(q, 0, 0)
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    for which in (0, 1, 0, 1):
        static_get(q, 0, which)
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free0
    q2, _ = _filled(8, 64, heads, hd, [T], seed=32, layers=1)
    torch.cuda.synchronize()
    free1 = torch.cuda.mem_get_info()[0]
    q2.get_keys_dequantized(0)  # stages through scratch it allocates
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] < free1
