"""fp16 scale/zero: how far the dequantised values sit from the reference's
f32 `code * scale + zero` (quantized_cache.rs:284-293).

The reference keeps scale and zero in f32.  A pool with fp16 metadata keeps
the reference's codes (bit-exact: they are computed from the f32 scale and
zero) and stores scale and zero rounded to f16; dequantisation is then
`code * scale16 + zero16` in f32 (mul then add), which is the reference's
formula over f16 metadata, bit-exact on the GPU against the oracle
(test_gpu_quant.py, test_gpu_fullshape.py).  Against the f32-metadata value
the difference comes from the two roundings: at most half an f16 ulp of
|zero| (|zero| <= the group's magnitude) plus code x half an f16 ulp of
scale (code x scale <= the group's range <= twice its magnitude), so below
2.5 f16 ulps of the group's largest |value| while the scale is a normal f16
number.  Measured on the oracle (the GPU is bit-exact to it) over 8192
tokens of rows like the quantised store's (N(0,1), 1% outliers x8, group
64 along head_dim 128, seed 0x5EED + 3), in f16 ulps of the group's
largest |value|:

    8-bit: max 1.53      4-bit: max 2.36

Per element, relative to the element's own f16 ulp, the difference is not
bounded: an element near zero (code * scale cancelling zero) keeps the
absolute error of the zero's rounding while its own ulp shrinks.
"""
import numpy as np
import pytest

import oracle as orc

# max |f16-meta value - f32-meta value| in f16 ulps of the group's max |value|:
# the analytic bound, and the measured maxima of the docstring
BOUND = 2.5
MEASURED = {8: 1.525390625, 4: 2.3603515625}


def ulp16(x):
    """Spacing of f16 numbers at |x| (subnormal spacing below 2^-14)."""
    a = np.abs(np.asarray(x, dtype=np.float64))
    return 2.0 ** (np.floor(np.log2(np.maximum(a, 2.0 ** -14))) - 10)


def rows(T, H, D, seed):
    """[1][T][H][D] f32 rows: N(0,1) with 1% outliers x8."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((1, T, H, D), dtype=np.float32)
    return np.where(rng.random(x.shape) < 0.01, x * 8.0, x).astype(np.float32)


def dequant_both(bits, T=8192, H=8, D=128, gs=64, seed=0x5EED + 3):
    """Oracle dequantisation of the same rows with f32 and with f16 metadata
    (f32 in and out): (f32-meta values, f16-meta values), [H][T][D]."""
    x = rows(T, H, D, seed)
    bs = 16
    N = T // bs
    out = {}
    for mb in (4, 2):
        g = orc.Geo(1, H, D, bs, N, 4, bits=bits, group_size=gs, meta_bytes=mb)
        host = np.zeros(g.pool_bytes(), np.uint8)
        assert orc.paged_append_quant(host, g, 0, 1, x, x, orc.F32, T * H * D, H * D, D,
                                      np.arange(T, dtype=np.int64)) == 0
        ok, ov = np.empty(T * H * D, np.float32), np.empty(T * H * D, np.float32)
        assert orc.paged_gather_dequant(host, g, 0, np.arange(N, dtype=np.int32).reshape(1, N), N,
                                        np.array([T], np.int32), ok, ov, orc.F32) == 0
        out[mb] = ok
    return out[4], out[2]


def ulp_error(ref32, got16, gs=64):
    err = np.abs(got16.astype(np.float64) - ref32.astype(np.float64)).reshape(-1, gs)
    mag = np.abs(ref32.astype(np.float64)).reshape(-1, gs).max(axis=1, keepdims=True)
    return float((err / ulp16(mag)).max())


@pytest.mark.parametrize("bits", [8, 4])
def test_f16_meta_within_bound_of_f32_reference(bits):
    ref, got = dequant_both(bits)
    e = ulp_error(ref, got)
    assert e <= BOUND, f"{bits}-bit: {e:.3f} f16 ulps of the group's magnitude"
    assert e == MEASURED[bits]  # the figure reported for this sample


def test_codes_equal_with_either_metadata():
    """The codes do not depend on how scale/zero are stored."""
    rng = np.random.default_rng(5)
    T, H, D, bs = 64, 2, 128, 16
    x = rng.standard_normal((1, T, H, D), dtype=np.float32)
    codes = []
    for mb in (4, 2):
        g = orc.Geo(1, H, D, bs, T // bs, 4, bits=8, group_size=64, meta_bytes=mb)
        host = np.zeros(g.pool_bytes(), np.uint8)
        orc.paged_append_quant(host, g, 0, 1, x, x, orc.F32, T * H * D, H * D, D, np.arange(T, dtype=np.int64))
        tiles = host.reshape(-1, g.tile_bytes())
        codes.append(tiles[:, :bs * D].copy())
    np.testing.assert_array_equal(codes[0], codes[1])
