"""The exact integer <-> f32 conversions the Q8_0 decode kernels use instead of
the conversion instructions, checked bit for bit over their input ranges.
CPU only (numpy on the same IEEE bit patterns).

* int8 -> f32 (attention_decode.cu, s8x4_to_f32): the byte with its sign bit
  flipped (b + 128) becomes the low mantissa byte of 2^23 (bits 0x4B0000xx);
  subtracting 2^23 + 128 leaves b.
* int32 -> f32 for |x| < 2^22 (attention_decode_q8tc.cu, i22f): x added to the
  bit pattern of 1.5 * 2^23, whose spacing is 1, is 1.5 * 2^23 + x;
  subtracting 1.5 * 2^23 leaves x.
* y in [0, 1] -> round(y (2^22 - 1)) (the P digits): fma(y, 2^22 - 1,
  1.5 * 2^23) read back as bits minus the bit pattern of 1.5 * 2^23.
"""
import numpy as np


def as_f32(bits):
    return np.asarray(bits, dtype=np.uint32).view(np.float32)


def as_bits(f):
    return np.asarray(f, dtype=np.float32).view(np.uint32)


def test_int8_through_the_mantissa_of_2_pow_23():
    b = np.arange(-128, 128, dtype=np.int32)
    byte = (b.astype(np.uint32) ^ 0x80) & 0xFF
    f = as_f32(0x4B000000 | byte) - np.float32(8388736.0)
    assert f.dtype == np.float32 and np.array_equal(f, b.astype(np.float32))


def test_int22_through_one_and_a_half_times_2_pow_23():
    x = np.concatenate([np.arange(-(2 ** 22) + 1, -(2 ** 22) + 5000), np.arange(-5000, 5000),
                        np.arange(2 ** 22 - 5000, 2 ** 22),
                        np.random.default_rng(0).integers(-(2 ** 22) + 1, 2 ** 22, 200000)]).astype(np.int64)
    bits = ((x + 0x4B400000) & 0xFFFFFFFF).astype(np.uint32)
    f = as_f32(bits) - np.float32(12582912.0)
    assert np.array_equal(f.astype(np.int64), x)


def test_p_digits_round_to_nearest_even():
    # y on f32's grid in [0, 1] with spacing >= 2^-24: y (2^22 - 1) + 1.5 * 2^23 is exact in f64, so
    # one rounding to f32 is what the fused multiply-add produces
    rng = np.random.default_rng(1)
    y = np.concatenate([np.arange(0, 2 ** 24 + 1, 4099), rng.integers(0, 2 ** 24 + 1, 200000)]) / 2.0 ** 24
    y = y.astype(np.float32)
    p_one = np.float32(4194303.0)
    fused = (y.astype(np.float64) * np.float64(p_one) + 12582912.0).astype(np.float32)
    got = as_bits(fused).astype(np.int64) - 0x4B400000
    want = np.rint(y.astype(np.float64) * np.float64(p_one)).astype(np.int64)
    assert np.array_equal(got, want)
    assert got.min() >= 0 and got.max() <= 2 ** 22 - 1  # three unsigned base-256 digits
