"""MT19937 and torch's CPU ``randperm`` — TEST INFRASTRUCTURE ONLY (oracle).

The routing maps of the reference (attention/precision_maps.py) draw random
permutations from torch's CPU generator: ``torch.manual_seed(42)`` followed by
``torch.randperm(n)`` (the global generator, :537-540, :580-601) and
``torch.randperm(n, generator=g)`` with ``g.manual_seed(42)`` (:307-309).

torch's CPU generator is the published Mersenne Twister MT19937 (Matsumoto &
Nishimura 1998): state initialised from the 32-bit seed with the standard
``init_genrand`` recurrence, 32-bit outputs tempered as in the paper. For
n below 2^32/20 torch's ``randperm`` (ATen ``randperm_cpu``) starts from the
identity and, for i = 0 .. n-2, swaps element i with element i + (r mod (n-i))
where r is the next 32-bit output. This module restates both; the unit tests
compare it with ``torch.randperm`` for many n and seeds.
"""
from __future__ import annotations

import numpy as np

N, M = 624, 397
MATRIX_A = 0x9908B0DF
UPPER, LOWER = 0x80000000, 0x7FFFFFFF


class MT19937:
    """Mersenne Twister with the reference initialisation (seed -> 624 words)."""

    def __init__(self, seed: int):
        mt = [0] * N
        mt[0] = seed & 0xFFFFFFFF
        for i in range(1, N):
            mt[i] = (1812433253 * (mt[i - 1] ^ (mt[i - 1] >> 30)) + i) & 0xFFFFFFFF
        self.mt = mt
        self.idx = N

    def _twist(self) -> None:
        mt = self.mt
        for i in range(N):
            y = (mt[i] & UPPER) | (mt[(i + 1) % N] & LOWER)
            mt[i] = mt[(i + M) % N] ^ (y >> 1) ^ (MATRIX_A if (y & 1) else 0)
        self.idx = 0

    def next_u32(self) -> int:
        if self.idx >= N:
            self._twist()
        y = self.mt[self.idx]
        self.idx += 1
        y ^= y >> 11
        y ^= (y << 7) & 0x9D2C5680
        y ^= (y << 15) & 0xEFC60000
        y ^= y >> 18
        return y & 0xFFFFFFFF


def randperm(n: int, gen: MT19937) -> np.ndarray:
    """torch CPU randperm(n) for n < 2^32 / 20, drawing from ``gen``."""
    if n >= (2**32) // 20:
        raise ValueError("large-n randperm path not restated")
    perm = np.arange(n, dtype=np.int64)
    for i in range(n - 1):
        z = gen.next_u32() % (n - i)
        perm[i], perm[i + z] = perm[i + z], perm[i]
    return perm
