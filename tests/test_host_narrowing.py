"""pkv_f32_to_bf16: the host-side f32 -> bf16 narrowing that the host stager
applies to f32 rows bound for a bf16 pool. Pure host code, so it runs without
a GPU: round to nearest even on every non-NaN f32 class, checked against the
oracle's bit-level restatement; NaNs stay NaNs. (Equality with the device's
own conversion, NaNs included, is a GPU test.)"""

import numpy as np

from pagedkv import _lib
from pagedkv.workloads import f32_to_bf16_bits


def narrow(x):
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.zeros(x.size, np.uint16)
    assert _lib.lib.pkv_f32_to_bf16(x.ctypes.data, out.ctypes.data, x.size) == 0
    return out


def test_round_to_nearest_even_on_random_bit_patterns():
    bits = np.random.default_rng(0).integers(0, 2**32, 1 << 20, dtype=np.uint64).astype(np.uint32)
    bits = bits[(bits & 0x7fffffff) <= 0x7f800000]  # no NaNs
    x = bits.view(np.float32)
    np.testing.assert_array_equal(narrow(x), f32_to_bf16_bits(x))


def test_ties_subnormals_overflow_and_signed_zero():
    fmax = np.finfo(np.float32).max
    x = np.array([0.0, -0.0, np.inf, -np.inf, fmax, -fmax, 1.00390625, 1.01171875, -2.00390625,
                  3.0e-39, -3.0e-39, 1e-45, 3.3895e38, 3.39617e38], np.float32)
    got = narrow(x)
    np.testing.assert_array_equal(got, f32_to_bf16_bits(x))
    assert got[0] == 0 and got[1] == 0x8000 and got[2] == 0x7f80 and got[3] == 0xff80
    assert got[4] == 0x7f80 and got[5] == 0xff80   # past the largest bf16: infinity
    assert got[6] == 0x3f80 and got[7] == 0x3f82   # ties to even


def test_nan_stays_nan():
    nan = np.array([0x7fc00000, 0xffc00000, 0x7f800001, 0xff800001, 0x7fffffff],
                   np.uint32).view(np.float32)
    got = narrow(np.concatenate([nan, np.ones(100, np.float32)]))
    assert np.all((got[:5] & 0x7f80) == 0x7f80) and np.all(got[:5] & 0x7f)
    assert np.all(got[5:] == 0x3f80)


def test_empty_and_null():
    assert _lib.lib.pkv_f32_to_bf16(None, None, 0) == 0
    assert _lib.lib.pkv_f32_to_bf16(None, None, 4) == 9
