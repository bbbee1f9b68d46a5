"""The integer form of the tf32 split's rounding (tc::to_tf32_int in
model_b200/csrc/tc_common.cuh, used by the operand-splitting GEMM's
converters and the balance backward's d cos split):

    bits(round(x)) = (bits(x) + 0x1000) & 0xFFFFE000

checked on the host against round-to-nearest, ties away from zero, to 10
mantissa bits, computed in exact float64 arithmetic from the value (the
rounding rule of cvt.rna.tf32.f32).  No GPU: this pins the formula the
device code applies, including ties, carries into the exponent, negative
values, subnormals and the overflow to infinity at the top of the range."""

import numpy as np


def _int_form(x: np.ndarray) -> np.ndarray:
    b = x.astype(np.float32).view(np.uint32)
    return ((b + np.uint32(0x1000)) & np.uint32(0xFFFFE000)).view(np.float32)


def _rna_tf32(x: np.ndarray) -> np.ndarray:
    x64 = x.astype(np.float64)
    a = np.abs(x64)
    out = np.zeros_like(x64)
    nz = a > 0
    # quantum: 2^(exponent - 10), subnormals sharing the smallest normal exponent's
    e = np.floor(np.log2(a[nz]))
    # log2 can land one off at exact powers of two after rounding; correct it
    e = np.where(np.exp2(e) > a[nz], e - 1, e)
    e = np.where(np.exp2(e + 1) <= a[nz], e + 1, e)
    q = np.exp2(np.maximum(e, -126.0) - 10.0)
    r = np.floor(a[nz] / q + 0.5) * q
    out[nz] = np.sign(x64[nz]) * r
    out[~nz] = x64[~nz]   # +-0 kept
    with np.errstate(over="ignore"):
        return out.astype(np.float32)   # >= 2^128 becomes inf


def _bits(x):
    return np.asarray(x, np.float32).view(np.uint32)


def test_random_values_match_round_to_nearest_ties_away():
    rng = np.random.default_rng(0)
    x = (rng.standard_normal(200_000) * np.exp2(rng.integers(-60, 60, 200_000))).astype(np.float32)
    np.testing.assert_array_equal(_bits(_int_form(x)), _bits(_rna_tf32(x)))


def test_every_low_bit_pattern_of_one_mantissa():
    # all 2^13 dropped-bit patterns below one kept mantissa, both signs
    base = np.uint32(0x3FA5A000)   # 1.29...: kept bits set, dropped bits zero
    low = np.arange(0x2000, dtype=np.uint32)
    for sign in (np.uint32(0), np.uint32(0x80000000)):
        x = ((base | low) | sign).view(np.float32)
        np.testing.assert_array_equal(_bits(_int_form(x)), _bits(_rna_tf32(x)))


def test_ties_round_away_from_zero():
    x = np.array([0x3F801000, 0xBF801000, 0x3F803000, 0xBF803000], np.uint32).view(np.float32)
    got = _int_form(x)
    # 1 + 2^-11 (a tie) -> 1 + 2^-10; 1 + 3 * 2^-11 (a tie) -> 1 + 2^-9
    np.testing.assert_array_equal(got, np.array([1 + 2.0**-10, -(1 + 2.0**-10), 1 + 2.0**-9, -(1 + 2.0**-9)],
                                                np.float32))


def test_carry_into_the_exponent_and_overflow():
    x = np.array([np.nextafter(np.float32(2.0), np.float32(0)),   # all mantissa bits set -> 2.0
                  np.float32(np.finfo(np.float32).max),             # rounds up past the largest tf32 -> inf
                  np.float32(-np.finfo(np.float32).max)], np.float32)
    got = _int_form(x)
    assert got[0] == 2.0
    assert np.isposinf(got[1]) and np.isneginf(got[2])
    np.testing.assert_array_equal(_bits(got), _bits(_rna_tf32(x)))


def test_zeros_and_subnormals():
    tiny = np.finfo(np.float32).tiny
    x = np.array([0.0, -0.0, tiny, -tiny, tiny / 3, tiny / 1000, -tiny / 7, np.float32(2.0**-149)], np.float32)
    np.testing.assert_array_equal(_bits(_int_form(x)), _bits(_rna_tf32(x)))


def test_split_reconstructs_three_term_operand():
    # hi + lo carries x to within 2^-22 relative: the 3xTF32 products' basis
    rng = np.random.default_rng(1)
    x = rng.standard_normal(100_000).astype(np.float32)
    hi = _int_form(x)
    lo = _int_form((x - hi).astype(np.float32))
    err = np.abs((hi.astype(np.float64) + lo) - x) / np.abs(x)
    assert err.max() <= 2.0**-21
