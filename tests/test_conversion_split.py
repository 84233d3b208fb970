"""The float -> xlns16 table splits into an exponent part and a per-mantissa
part for every normal float; the tiled weight conversion on the GPU
(k_to_lns16_typed_tiled) computes it that way instead of gathering from the
65,536-entry table, and its launcher re-checks the split on the library's own
table before using it (conv16_splits).

For a float with biased exponent e in 1..254 and top mantissa bits m (the
table is indexed by the float's upper 16 bits), the code is
    clamp(128 (e - 127) + G[m] + 0x4000, 0, 0x7FFF) | sign,
with G[m] = 128 log2(1 + m/128) truncated toward zero: floored for |x| >= 1
(read off the entries at e = 127), rounded up below (entries at e = 126,
plus 128).  Subnormals, infinities and NaNs (e = 0 or 255) keep the table.
The GPU parity tests show the device table equals this oracle's table."""
import numpy as np


def test_conv16_splits_into_exponent_and_mantissa(orc):
    u = np.arange(65536, dtype=np.uint32)
    code = orc.from_f32_16((u << 16).view(np.float32)).astype(np.int64)
    e = ((u >> 7) & 0xFF).astype(np.int64)
    m = (u & 0x7F).astype(np.int64)
    gp = code[(127 << 7) | np.arange(128)] - 0x4000               # |x| >= 1
    gn = code[(126 << 7) | np.arange(128)] - 0x4000 + 128         # |x| < 1
    assert gp.min() >= 0 and gp.max() <= 255 and gn.min() >= 0 and gn.max() <= 255
    normal = (e >= 1) & (e <= 254)
    g = np.where(e < 127, gn[m], gp[m])
    split = np.clip(128 * (e - 127) + g + 0x4000, 0, 0x7FFF) | ((u >> 15) << 15)
    assert np.array_equal(code[normal], split[normal])
    # the floor and the rounded-up part differ by one wherever the log is not an integer
    assert gp[0] == gn[0] == 0 and np.all(gn[1:] == gp[1:] + 1)
