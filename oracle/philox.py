"""Philox4x32-10 counter-based generator (TEST INFRASTRUCTURE).

The published algorithm of Salmon, Moraes, Dror and Shaw, "Parallel random numbers: as easy as
1, 2, 3" (SC'11): a 4x32-bit counter is pushed through 10 rounds of two 32x32->64 multiplies and
xors with a 2x32-bit key that is bumped by the Weyl constants between rounds.

The speculative step's uniform stream is defined on top of it (the CUDA kernel implements the
same definition independently):

    uniform(seed, index) = (philox(counter=(index_lo, index_hi, 0, 0), key=(seed_lo, seed_hi))[0] >> 8)
                           * 2**-24

which is a float32-exact value in [0, 1). ``index`` is the per-request draw counter, advanced by
one for every uniform the acceptance consumes (in the reference's data-dependent order).
"""

from __future__ import annotations

MULT0 = 0xD2511F53
MULT1 = 0xCD9E8D57
WEYL0 = 0x9E3779B9
WEYL1 = 0xBB67AE85
MASK = 0xFFFFFFFF


def philox4x32_10(counter: tuple[int, int, int, int], key: tuple[int, int]) -> tuple[int, int, int, int]:
    c0, c1, c2, c3 = (x & MASK for x in counter)
    k0, k1 = (x & MASK for x in key)
    for round_index in range(10):
        p0 = MULT0 * c0
        p1 = MULT1 * c2
        hi0, lo0 = (p0 >> 32) & MASK, p0 & MASK
        hi1, lo1 = (p1 >> 32) & MASK, p1 & MASK
        c0, c1, c2, c3 = hi1 ^ c1 ^ k0, lo1, hi0 ^ c3 ^ k1, lo0
        if round_index != 9:
            k0 = (k0 + WEYL0) & MASK
            k1 = (k1 + WEYL1) & MASK
    return c0, c1, c2, c3


def uniform(seed: int, index: int) -> float:
    word = philox4x32_10((index & MASK, (index >> 32) & MASK, 0, 0), (seed & MASK, (seed >> 32) & MASK))[0]
    return (word >> 8) * (1.0 / (1 << 24))


class UniformStream:
    """Iterator over ``uniform(seed, start), uniform(seed, start + 1), ...``; ``index`` is the next."""

    def __init__(self, seed: int, start: int = 0) -> None:
        self.seed = seed
        self.index = start

    def __iter__(self):
        return self

    def __next__(self) -> float:
        value = uniform(self.seed, self.index)
        self.index += 1
        return value
