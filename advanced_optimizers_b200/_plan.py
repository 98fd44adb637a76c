"""Host planner: cuts a parameter group's tensors into pieces and gives every
CTA of the persistent elementwise launch a contiguous run with an equal share
of elements.

A piece is [begin, end) of one tensor's flat elements:
  * begin is a multiple of 2048 (one int8_sr block, state_util.py:10), so a
    CTA always owns whole quantisation blocks;
  * for factored_2nd tensors both ends also sit on row boundaries of the
    effective shape (d1, d2), so every row's sum is finished inside one CTA
    (factorization_util.py:68) and each piece writes one row of column
    partials ("slot");
  * factored pieces hold at most ``MAX_ROWS`` rows, which bounds the float32
    column partials' accumulation depth before the float64 slot reduction.
"""
from __future__ import annotations

import math

import numpy as np

from ._lib import PIECE_DT

CHUNK = 2048
MAX_ROWS = 64


def effective_shape(numel: int):
    """factorization_util._get_effective_shape (factorization_util.py:43-50)."""
    if numel <= 0:
        return (0, 0)
    for i in range(math.isqrt(numel), 0, -1):
        if numel % i == 0:
            return (numel // i, i)
    return (numel, 1)


def unit_of(numel: int, d2: int) -> int:
    """Smallest piece granule: one chunk, or lcm(d2, 2048) for factored tensors."""
    if d2 <= 0:
        return CHUNK
    return d2 * CHUNK // math.gcd(d2, CHUNK)


def plan(numels, d2s, grid: int):
    """numels[i], d2s[i] (0 = not factored) -> (pieces, cta_offsets, n_slots).

    The last CTA takes whatever remains, so len(cta_offsets) == grid + 1 and
    every CTA index in [0, grid) is valid (some may own no piece)."""
    total = int(sum(int(n) for n in numels))
    grid = max(1, int(grid))
    target = max(CHUNK, -(-total // grid))
    pieces = []
    offsets = [0]
    n_slots = [0] * len(numels)
    budget = target
    cta = 0

    def close():
        nonlocal budget, cta
        offsets.append(len(pieces))
        cta += 1
        budget = target

    for t, (n, d2) in enumerate(zip(numels, d2s)):
        n, d2 = int(n), int(d2)
        if n <= 0:
            continue
        unit = unit_of(n, d2)
        cap = max(unit, (MAX_ROWS * d2 // unit) * unit) if d2 > 0 else 1 << 62
        pos = 0
        while pos < n:
            take = min(n - pos, cap)
            last_cta = cta >= grid - 1
            if not last_cta and take > budget:
                fit = (budget // unit) * unit
                if fit == 0:
                    if offsets[-1] != len(pieces):       # CTA already has work: next CTA
                        close()
                        continue
                    fit = unit
                take = min(take, fit)
            pieces.append((pos, pos + take, t, n_slots[t]))
            n_slots[t] += 1
            pos += take
            budget -= take
            if not last_cta and budget < CHUNK:
                close()
    while len(offsets) < grid + 1:
        offsets.append(len(pieces))
    offsets = offsets[: grid + 1]
    offsets[-1] = len(pieces)
    arr = np.zeros(len(pieces), PIECE_DT)
    if pieces:
        p = np.array(pieces, dtype=np.int64)
        arr["begin"], arr["end"], arr["tensor"], arr["slot"] = p[:, 0], p[:, 1], p[:, 2], p[:, 3]
    return arr, np.asarray(offsets, np.int32), n_slots
