"""Matmul parity tolerance shared by the CPU oracle tests and the GPU tests.

The north-star bar is: max-abs error <= 1e-2 x RMS(reference output), for bf16
inputs with fp32 accumulation.  Outputs are stored in the activation dtype, so
two correct implementations whose fp32 sums differ slightly (summation order,
or where in the chain a weight is rounded) land one output ulp apart wherever
the sum sits next to a rounding boundary -- and the reference rounds more
than once: LoRALinear rounds the base output, then rounds again after adding
the adapter term, so a one-ulp move of the base can become two when the
adapter term is an exact half ulp (ties-to-even).  For bf16 one ulp exceeds
1e-2 x RMS as soon as |y| >= 2 x RMS.  The check is therefore

    |y - y_ref| <= 1e-2 * rms(y_ref) + roundings * ulp   (elementwise)

with `roundings` the number of output roundings after the accumulation in
the reference's op sequence (1 for QuantLinear alone, 2 with the adapter),
ulp = one unit in the last place of the stored dtype at the larger of |y|
and |y_ref| (0 for fp32): two values on either side of a power of two are
one rounding apart at the upper binade's ulp.
``matmul_error`` reports the plain max-abs / RMS figure alongside.
"""
import numpy as np

RTOL_RMS = 1e-2
F32, BF16, F16 = 0, 1, 2
_MANT = {BF16: 7, F16: 10}


def ulp(y, dtype):
    if dtype not in _MANT:
        return np.zeros_like(y, dtype=np.float64)
    a = np.abs(y.astype(np.float64))
    e = np.floor(np.log2(np.where(a > 0, a, 1.0)))
    if dtype == F16:
        e = np.maximum(e, -14)
    return np.where(a > 0, np.exp2(e - _MANT[dtype]), 0.0)


def matmul_error(y, y_ref):
    y = np.asarray(y, np.float64)
    y_ref = np.asarray(y_ref, np.float64)
    rms = float(np.sqrt(np.mean(y_ref ** 2))) if y_ref.size else 0.0
    err = float(np.max(np.abs(y - y_ref))) if y_ref.size else 0.0
    return err, rms


# (label, max-abs / RMS, outputs that needed the ulp allowance, outputs) of
# the checks that asked to be recorded; the test session prints them.
RECORDED = []


def assert_matmul_close(y, y_ref, dtype, roundings=2, label=None):
    """Elementwise check against the bound above.  Returns the plain figures:
    max-abs / RMS and how many outputs exceeded the bare 1e-2 x RMS bar and
    passed only through the ulp allowance.  Where that count is 0 the bare
    north-star bar holds for the whole output.  With a `label` the figures
    are also recorded for the session summary."""
    y = np.asarray(y, np.float64)
    y_ref = np.asarray(y_ref, np.float64)
    assert y.shape == y_ref.shape, (y.shape, y_ref.shape)
    assert np.all(np.isfinite(y)), "non-finite output"
    err, rms = matmul_error(y, y_ref)
    diff = np.abs(y - y_ref)
    # the rounding that produced an output erred by at most half an ulp of
    # the output's own binade: next to a power of two the larger of the two
    # values' ulps is the one that applies
    bound = RTOL_RMS * rms + roundings * np.maximum(ulp(y_ref, dtype), ulp(y, dtype))
    bad = diff > bound
    if bad.any():
        i = np.argmax(diff - bound)
        raise AssertionError(
            f"{int(bad.sum())}/{y.size} outputs outside 1e-2*RMS + {roundings} ulp: max-abs {err:.4g}, "
            f"rms {rms:.4g}; worst at flat {i}: {y.reshape(-1)[i]!r} vs {y_ref.reshape(-1)[i]!r}")
    n_ulp = int(np.count_nonzero(diff > RTOL_RMS * rms))
    if n_ulp == 0:
        assert err <= RTOL_RMS * rms
    stats = {"max_abs_over_rms": err / rms if rms > 0 else 0.0, "n_ulp": n_ulp, "n": int(y.size)}
    if label is not None:
        RECORDED.append((label, stats["max_abs_over_rms"], n_ulp, int(y.size)))
    return stats
