"""The NF4 code table of the quantize kernel (quant_kernels.cu, QTab): for
bf16 / f16 inputs the kernel looks the code of the rounded x / absmax up by
its 16-bit pattern instead of searching the thresholds.  This restates the
table's construction and index rule in numpy and checks it against the
oracle's quantize (the reference's 16-way argmin, quant_ops.py:80-126) for
every pattern the kernel can meet: all values in [-1, 1].  NaN (code 0) is
checked by the rule alone.
"""
import numpy as np
import pytest

from oracle import oracle as orc

# (dtype, lowest pattern with |value| >= 2^-5, pattern of 1.0, sign bit of the index)
RULES = {orc.BF16: (0x3D00, 0x3F80, 0x400), orc.F16: (0x2800, 0x3C00, 0x2000)}


def _value(bits, dt):
    return orc.to_f32(np.asarray(bits, np.uint16), dt)


def _oracle_codes(vals, dt):
    """code of each v in [-1, 1] from the oracle: block [1.0, v, 0, ...] has
    absmax 1, so x / absmax is v itself; the code is byte 0's high nibble."""
    n = vals.size
    x = np.zeros((n, 64), np.float32)
    x[:, 0] = 1.0
    x[:, 1] = vals
    bits = orc.f32_to_bf16_bits(x) if dt == orc.BF16 else x.astype(np.float16).view(np.uint16)
    packed, _ = orc.nf4_quantize(bits.reshape(-1), dt, 64)
    return (packed.reshape(n, 32)[:, 0] >> 4).astype(np.int64)


def _table(dt):
    lo, one, sgn = RULES[dt]
    tab = np.zeros(2 * sgn, np.int64)
    for neg in (0, sgn):
        tab[neg] = 7
        a = np.arange(lo, one + 1, dtype=np.uint32)
        pat = (a | (0x8000 if neg else 0)).astype(np.uint16)
        tab[neg + 1 + (a - lo)] = _oracle_codes(_value(pat, dt), dt)
        tab[neg + one - lo + 2] = 0
    return tab


def _lookup(bits, dt, tab):
    lo, one, sgn = RULES[dt]
    b = bits.astype(np.int64)
    a = b & 0x7FFF
    j = np.clip(a - (lo - 1), 0, one - lo + 2)
    s = ((b >> 5) & sgn) if dt == orc.BF16 else ((b >> 2) & sgn)
    return tab[j | s]


@pytest.mark.parametrize("dt", [orc.BF16, orc.F16])
def test_code_table_equals_argmin_on_every_pattern(dt):
    tab = _table(dt)
    bits = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    vals = _value(bits, dt)
    reach = np.abs(vals) <= 1.0  # every value x / absmax can take (NaN aside)
    got = _lookup(bits[reach], dt, tab)
    want = _oracle_codes(vals[reach], dt)
    assert np.array_equal(got, want)
    # every |value| < 2^-5 sits between the thresholds of code 7
    small = reach & (np.abs(vals) < 2.0 ** -5)
    assert np.all(_oracle_codes(vals[small], dt) == 7)
    # NaN patterns land on the code-0 entries
    nan = np.isnan(vals)
    assert np.all(_lookup(bits[nan], dt, tab) == 0)
