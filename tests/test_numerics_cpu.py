"""CPU restatement, in exact rational arithmetic, of the integer and rounding
identities the kernels' requantisation and short exp2 rely on.

The GPU self-checks (``q3_quant_selfcheck``, ``q3_exp2_selfcheck``) compare
the device code with the reference forms over every float32 input; these tests
pin the same mathematics on the host, independently of any GPU:

* an int8 code from a shared reciprocal of the scale with Markstein's
  correction, unclamped, equals the code from the IEEE quotient, clipped to
  +-127 (ref_qwen3.py:69-76), whenever the scale is amax * RN(1/127) of an
  absolute maximum amax >= |x| and lies in [2^-100, 2^100];
* rounding a quotient in [-127.5, 127.5] to an integer by adding 1.5 * 2^23
  in float32 is rint (ties to even), and the sum's low byte is the code's;
* the byte permutes that pack four codes gather those low bytes;
* the exp2 shifter's bit pattern u = 0x4B400000 + k gives the table index
  k & 255 as u & 255 and the exponent step (k >> 8) << 23 as
  (u << 15) & 0xFF800000 (mod 2^32).

Each float32 operation is computed exactly with ``fractions.Fraction`` and
rounded once to the nearest float32, ties to even (``rn32``), which is what an
IEEE single operation (or a fused multiply-add) returns.
"""

from __future__ import annotations

from fractions import Fraction

import numpy as np

F = np.float32
TWO = Fraction(2)


def rn32(v: Fraction) -> Fraction:
    """v rounded to the nearest float32 (ties to even), as an exact Fraction;
    +-inf beyond the largest finite float32 (returned as None)."""
    if v == 0:
        return Fraction(0)
    sign = -1 if v < 0 else 1
    a = -v if v < 0 else v
    e = a.numerator.bit_length() - a.denominator.bit_length()
    while TWO ** e > a:
        e -= 1
    while TWO ** (e + 1) <= a:
        e += 1
    q = max(e - 23, -149)                      # exponent of the ulp at a
    m = a / TWO ** q
    n = m.numerator // m.denominator
    rem = m - n
    if rem > Fraction(1, 2) or (rem == Fraction(1, 2) and n % 2 == 1):
        n += 1
    r = n * TWO ** q
    if r >= TWO ** 128:
        return None
    return sign * r


def f32(v: Fraction) -> float:
    return float(F(float(v)))                  # exact: v is a float32 value


def rint_even(v: Fraction) -> int:
    n = v.numerator // v.denominator
    rem = v - n
    if rem > Fraction(1, 2) or (rem == Fraction(1, 2) and n % 2 == 1):
        n += 1
    return n


KINV127 = rn32(Fraction(1, 127))               # the kernels' 1.0f / 127.0f


def code_quotient(x: Fraction, s: Fraction) -> int:
    """ref_qwen3.py:69-76: rint(RN(x / s)) clipped to +-127."""
    return max(-127, min(127, rint_even(rn32(x / s))))


def code_reciprocal(x: Fraction, s: Fraction) -> int:
    """quant1_rcp_absmax: r = RN(1/s), q0 = RN(x r), e = RN(x - q0 s) (fma),
    q = RN(e r + q0) (fma), then rint without a clamp."""
    r = rn32(1 / s)
    q0 = rn32(x * r)
    e = rn32(x - q0 * s)
    q = rn32(e * r + q0)
    return rint_even(q)


def _fr(v) -> Fraction:
    return Fraction(float(F(v)))


def test_rn32_matches_numpy_single_operations():
    """rn32 agrees with numpy's float32 arithmetic (IEEE single, RN-even)."""
    rng = np.random.default_rng(1)
    a = (rng.standard_normal(400) * 10.0 ** rng.integers(-30, 30, 400)).astype(F)
    b = (rng.standard_normal(400) * 10.0 ** rng.integers(-30, 30, 400)).astype(F)
    with np.errstate(all="ignore"):
        for x, y in zip(a, b):
            for got, want in ((rn32(Fraction(float(x)) * Fraction(float(y))), x * y),
                              (rn32(Fraction(float(x)) + Fraction(float(y))), x + y),
                              (rn32(Fraction(float(x)) / Fraction(float(y))), x / y)):
                if got is None:
                    assert np.isinf(want)
                else:
                    assert f32(got) == float(want)


def _amaxes(rng, n):
    out = [Fraction(1), Fraction(127), TWO ** -93, TWO ** 106, _fr(np.nextafter(F(1), F(2))),
           _fr(np.nextafter(F(1), F(0))), _fr(F(2) - F(2) ** F(-23))]
    for m, e in zip(rng.uniform(1.0, 2.0, n), rng.integers(-90, 105, n)):
        out.append(_fr(F(m) * F(2.0) ** F(e)))
    return out


def test_reciprocal_requantisation_matches_quotient():
    """Markstein's correction from one reciprocal, unclamped, gives the
    quotient's clipped code for |x| <= amax: random x, +-amax, tiny and zero x,
    and x at and next to every half-integer multiple of the scale (the
    double-rounding ties)."""
    rng = np.random.default_rng(11)
    checked = 0
    for amax in _amaxes(rng, 24):
        s = rn32(amax * KINV127)
        if not (TWO ** -100 <= s <= TWO ** 100):
            continue
        xs = [amax, -amax, Fraction(0), _fr(np.float32(float(amax)) * F(1e-30))]
        xs += [_fr(F(float(amax)) * F(u)) for u in rng.uniform(-1.0, 1.0, 60)]
        for k in rng.integers(-127, 127, 40):
            t = f32(rn32((Fraction(int(k)) + Fraction(1, 2)) * s))
            for v in (t, float(np.nextafter(F(t), F(np.inf))), float(np.nextafter(F(t), F(-np.inf)))):
                xv = Fraction(v)
                if abs(xv) <= amax:
                    xs.append(xv)
        for x in xs:
            c = code_reciprocal(x, s)
            assert -127 <= c <= 127, (float(x), float(s))
            assert c == code_quotient(x, s), (float(x), float(amax), float(s))
            checked += 1
    assert checked > 3000


def test_absmax_scale_bounds_the_quotient():
    """|x / s| <= amax / s = 127 / ((1 + d1)(1 + d2)) <= 127 / (1 - 2^-24)^2,
    below 127.5, for a scale in [2^-100, 2^100] (d1, d2 the relative errors of
    the two roundings): the reciprocal form needs no clamp."""
    rng = np.random.default_rng(5)
    for amax in _amaxes(rng, 200):
        s = rn32(amax * KINV127)
        if TWO ** -100 <= s <= TWO ** 100:
            assert amax / s < Fraction(255, 2)
            assert amax / s <= 127 / (1 - TWO ** -24) ** 2


def test_shifter_rounding_is_rint_and_keeps_the_low_byte():
    """float32(q + 1.5 * 2^23) - 0x4B400000 is rint(q) (ties to even) for q in
    [-127.5, 127.5]; its low byte is the code's two's-complement byte."""
    halves = np.arange(-255, 256, dtype=np.float64) / 2.0
    q = np.concatenate([halves.astype(F), np.nextafter(halves.astype(F), F(np.inf)),
                        np.nextafter(halves.astype(F), F(-np.inf)),
                        np.random.default_rng(3).uniform(-127.5, 127.5, 20000).astype(F)])
    q = q[np.abs(q) <= F(127.5)]
    bits = (q + F(12582912.0)).view(np.int32)
    code = bits - np.int32(0x4B400000)
    assert np.array_equal(code, np.rint(q).astype(np.int32))
    assert np.array_equal(bits & 0xFF, code & 0xFF)


def _byte_perm(x: int, y: int, s: int) -> int:
    """CUDA __byte_perm: result byte n is byte (s >> 4n) & 7 of the 64-bit
    value {y, x} (x in bytes 0-3)."""
    v = (y << 32) | x
    return sum(((v >> (8 * ((s >> (4 * n)) & 7))) & 0xFF) << (8 * n) for n in range(4))


def test_byte_permutes_pack_the_low_bytes():
    rng = np.random.default_rng(9)
    for w in rng.integers(0, 2 ** 32, size=(500, 4), dtype=np.uint64):
        b0, b1, b2, b3 = (int(v) for v in w)
        packed = _byte_perm(_byte_perm(b0, b1, 0x0040), _byte_perm(b2, b3, 0x0040), 0x5410)
        assert packed == (b0 & 0xFF) | (b1 & 0xFF) << 8 | (b2 & 0xFF) << 16 | (b3 & 0xFF) << 24


def test_exp2_shifter_index_and_exponent_step():
    """For every k = rint(256 x) with x in [-125, 128): u = 0x4B400000 + k
    gives k & 255 as u & 255 and (k >> 8) << 23 as (u << 15) & 0xFF800000,
    mod 2^32; and the shifter's float32 sum is that u."""
    k = np.arange(-32000, 32769, dtype=np.int64)
    u = (0x4B400000 + k).astype(np.uint64)
    assert np.array_equal(u & 255, (k & 255).astype(np.uint64))
    step = ((k >> 8) << 23) & 0xFFFFFFFF
    assert np.array_equal((u << 15) & 0xFF800000, step.astype(np.uint64))
    x = (k.astype(np.float64) / 256.0).astype(F)
    x = x[(x >= F(-125)) & (x < F(128))]
    sh = ((x * F(256.0)) + F(12582912.0)).view(np.uint32).astype(np.int64) - 0x4B400000
    assert np.array_equal(sh, np.rint(x.astype(np.float64) * 256.0).astype(np.int64))
