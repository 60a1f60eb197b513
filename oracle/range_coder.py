"""Range coder of the reference, restated in Python -- TEST INFRASTRUCTURE ONLY.

Only tests/ import this module: it turns the CDFs that the device computes into the archive bytes
the reference host would write, so tests can check archive round trips and byte parity.

  RangeEncoder (shift_low, encode, finish)   src/domain/coder.rs:114-196
  RangeDecoder (new, get_freq, update)       src/domain/coder.rs:198-290
  Cdf::uniform / Cdf::range                  src/domain/coder.rs:84-98

24-bit normalisation (TOP = 2^24), 64-bit low with Schindler carry propagation, and the
decoder's cumulative-frequency clamp to total - 1.
"""
from __future__ import annotations

from typing import List, Tuple

TOP = 1 << 24
M32 = 0xFFFFFFFF


def uniform(n: int) -> Tuple[List[int], int]:
    """Cdf::uniform(n): every symbol gets TOP // n; total = (TOP // n) * n."""
    f = TOP // n
    return [i * f for i in range(n + 1)], f * n


class RangeEncoder:
    def __init__(self) -> None:
        self.low = 0          # u64
        self.range = M32      # u32
        self.cache = 0
        self.ff_count = 0
        self.first = True
        self.out = bytearray()

    def _shift_low(self) -> None:
        low32 = self.low & M32
        if low32 < 0xFF000000 or (self.low >> 32) != 0:
            carry = (self.low >> 32) & 0xFF
            if not self.first:
                self.out.append((self.cache + carry) & 0xFF)
            self.first = False
            for _ in range(self.ff_count):
                self.out.append((0xFF + carry) & 0xFF)
            self.ff_count = 0
            self.cache = (self.low >> 24) & 0xFF
        else:
            self.ff_count += 1
        self.low = (self.low & 0x00FFFFFF) << 8

    def encode(self, lo: int, hi: int, total: int) -> None:
        r = self.range // total
        assert r > 0, "range underflow"
        self.low += lo * r
        if hi < total:
            self.range = (r * (hi - lo)) & M32
        else:
            self.range = (self.range - ((r * lo) & M32)) & M32
        while self.range < TOP:
            self._shift_low()
            self.range = (self.range << 8) & M32

    def finish(self) -> bytes:
        for _ in range(5):
            self._shift_low()
        if not self.first:
            self.out.append(self.cache)
            self.out.extend(b"\xff" * self.ff_count)
        return bytes(self.out)


class RangeDecoder:
    def __init__(self, data: bytes) -> None:
        self.low = 0
        self.range = M32
        self.code = 0
        self.data = data
        self.pos = 0
        for _ in range(4):
            self.code = ((self.code << 8) | self._next()) & M32

    def _next(self) -> int:
        if self.pos < len(self.data):
            b = self.data[self.pos]
            self.pos += 1
            return b
        return 0

    def get_freq(self, total: int) -> int:
        r = self.range // total
        if r == 0:
            raise ValueError("decoder range underflow")
        return min(((self.code - self.low) & M32) // r, total - 1)

    def update(self, lo: int, hi: int, total: int) -> None:
        r = self.range // total
        self.low = (self.low + r * lo) & M32
        if hi < total:
            self.range = (r * (hi - lo)) & M32
        else:
            self.range = (self.range - r * lo) & M32
        while self.range < TOP:
            self.code = ((self.code << 8) | self._next()) & M32
            self.low = (self.low << 8) & M32
            self.range = (self.range << 8) & M32


def lookup(cdf, cum: int) -> int:
    """Cdf::lookup (coder.rs:100-114) on a list or array of n + 1 entries."""
    lo, hi = 0, len(cdf) - 1
    while lo < hi:
        mid = (lo + hi) // 2
        if cdf[mid + 1] <= cum:
            lo = mid + 1
        else:
            hi = mid
    return lo
