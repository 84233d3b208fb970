"""The float -> xlns16 table splits into an exponent part and a per-mantissa
part for every normal float; the tiled weight conversion on the GPU
(k_to_lns16_typed_tiled) computes it that way instead of gathering from the
table, and its launcher re-checks the split on the library's own table before
using it (conv16_splits).

The table is indexed by a float's upper 17 bits u = bits >> 15 (the sign,
the biased exponent e and the top 8 mantissa bits m).  For e in 1..254 the
code is
    clamp(128 (e - 127) + G[m] + 0x4000, 0, 0x7FFF) | sign,
with G[m] = 128 log2(1 + m/256) truncated toward zero: floored for |x| >= 1
(read off the entries at e = 127), rounded up below (entries at e = 126,
plus 128).  Subnormals, infinities and NaNs (e = 0 or 255) keep the table.
The GPU parity tests show the device table equals this oracle's table."""
import numpy as np


def test_conv16_splits_into_exponent_and_mantissa(orc):
    u = np.arange(131072, dtype=np.uint32)
    code = orc.from_f32_16((u << 15).view(np.float32)).astype(np.int64)
    e = ((u >> 8) & 0xFF).astype(np.int64)
    m = (u & 0xFF).astype(np.int64)
    gp = code[(127 << 8) | np.arange(256)] - 0x4000               # |x| >= 1
    gn = code[(126 << 8) | np.arange(256)] - 0x4000 + 128         # |x| < 1
    assert gp.min() >= 0 and gp.max() <= 255 and gn.min() >= 0 and gn.max() <= 255
    normal = (e >= 1) & (e <= 254)
    g = np.where(e < 127, gn[m], gp[m])
    split = np.clip(128 * (e - 127) + g + 0x4000, 0, 0x7FFF) | ((u >> 16) << 15)
    assert np.array_equal(code[normal], split[normal])
    # the floor and the rounded-up part differ by one wherever the log is not an integer
    assert gp[0] == gn[0] == 0 and np.all(gn[1:] == gp[1:] + 1)


def test_conv16_low_mantissa_bits_ignored(orc):
    """the table sees only the top 8 mantissa bits: every float in a bucket
    converts like the bucket's lower edge"""
    rng = np.random.default_rng(0)
    hi = rng.integers(0, 1 << 17, 100000, dtype=np.uint32) << 15
    lo = rng.integers(0, 1 << 15, 100000, dtype=np.uint32)
    a = orc.from_f32_16(hi.view(np.float32))
    b = orc.from_f32_16((hi | lo).view(np.float32))
    nan = np.isnan((hi | lo).view(np.float32))
    assert np.array_equal(a[~nan], b[~nan])
