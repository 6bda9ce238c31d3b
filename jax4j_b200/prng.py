"""PrngKey (core/tensor/PrngKey.java:27-112): immutable counter-based keys on the host.

Values themselves are drawn on the device by j4b_random_uniform / j4b_random_normal (the
splitmix64 counter streams of ComputeBackend.java:51-76); this module only derives keys.
"""
from __future__ import annotations

from dataclasses import dataclass

_M64 = (1 << 64) - 1
_PHI = 0x9E3779B97F4A7C15


def _signed(v: int) -> int:
    return v - (1 << 64) if v >= 1 << 63 else v


def mix64(v: int) -> int:
    """ComputeBackend.java:290-295 / PrngKey.java:102-107 (splitmix64 finaliser)."""
    v &= _M64
    v = ((v ^ (v >> 30)) * 0xBF58476D1CE4E5B9) & _M64
    v = ((v ^ (v >> 27)) * 0x94D049BB133111EB) & _M64
    return v ^ (v >> 31)


@dataclass(frozen=True)
class PrngKey:
    seed: int
    counter: int = 0

    @staticmethod
    def of(seed: int) -> "PrngKey":
        return PrngKey(seed, 0)

    def advance(self, amount: int) -> "PrngKey":
        if amount < 0:
            raise ValueError("PRNG counter advance must be non-negative")
        return PrngKey(self.seed, self.counter + amount)

    def fold_in(self, data: int) -> "PrngKey":
        return PrngKey(_signed(mix64(self.seed ^ mix64(data))), self.counter)

    def split(self, count: int) -> list["PrngKey"]:
        if count < 1:
            raise ValueError("PRNG split count must be positive")
        return [PrngKey(_signed(mix64(self.seed + _PHI * (self.counter + i + 1))), 0)
                for i in range(count)]
