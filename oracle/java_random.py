"""Restatement of ``java.util.Random`` (test infrastructure, oracle only).

The reference seeds ``new java.util.Random(seed)`` in its sampler
(inference/Sampler.java:313-316) and in its unit tests
(test quant/Q4_0Test.java:22, inference/SamplerTest.java). The generator is the
48-bit linear congruential generator whose every step is specified in the Java
SE API documentation of ``java.util.Random`` (``next``, ``nextInt(bound)``,
``nextFloat``, ``nextDouble``, ``nextGaussian``). This module restates that
published specification; it is not derived from any JDK source.
"""
from __future__ import annotations

import math

_MULT = 0x5DEECE66D
_ADD = 0xB
_MASK = (1 << 48) - 1


def _to_int32(v: int) -> int:
    v &= 0xFFFFFFFF
    return v - (1 << 32) if v >= (1 << 31) else v


class JavaRandom:
    """``java.util.Random`` with the documented LCG (seed scrambled by 0x5DEECE66D)."""

    def __init__(self, seed: int):
        self._seed = (seed ^ _MULT) & _MASK
        self._next_gaussian: float | None = None

    def next_bits(self, bits: int) -> int:
        self._seed = (self._seed * _MULT + _ADD) & _MASK
        return _to_int32(self._seed >> (48 - bits))

    def next_int(self, bound: int | None = None) -> int:
        if bound is None:
            return self.next_bits(32)
        if bound <= 0:
            raise ValueError("bound must be positive")
        if bound & (-bound) == bound:  # power of two
            return _to_int32((bound * self.next_bits(31)) >> 31)
        while True:
            bits = self.next_bits(31)
            val = bits % bound
            if _to_int32(bits - val + (bound - 1)) >= 0:
                return val

    def next_float(self) -> float:
        # next(24) / 2^24, exactly representable in float32.
        return self.next_bits(24) / float(1 << 24)

    def next_double(self) -> float:
        return ((self.next_bits(26) << 27) + self.next_bits(27)) * (2.0 ** -53)

    def next_gaussian(self) -> float:
        # Marsaglia polar method, as the Java SE documentation specifies.
        if self._next_gaussian is not None:
            g, self._next_gaussian = self._next_gaussian, None
            return g
        while True:
            v1 = 2.0 * self.next_double() - 1.0
            v2 = 2.0 * self.next_double() - 1.0
            s = v1 * v1 + v2 * v2
            if 0.0 < s < 1.0:
                break
        mul = math.sqrt(-2.0 * math.log(s) / s)
        self._next_gaussian = v2 * mul
        return v1 * mul
