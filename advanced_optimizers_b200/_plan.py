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

    All tensors are laid end to end; CTA c owns the elements between global
    cut points c and c+1, where cut point c is c*total/grid rounded to the
    nearest position a piece may start at (a multiple of the tensor's unit, or
    a tensor boundary).  Rounding errors therefore never accumulate: every CTA
    holds its share to within one unit.  len(cta_offsets) == grid + 1."""
    grid = max(1, int(grid))
    starts = []
    total = 0
    for n in numels:
        starts.append(total)
        total += max(0, int(n))
    units = [unit_of(int(n), int(d2)) for n, d2 in zip(numels, d2s)]

    def snap(x):
        """nearest allowed cut position to global element x"""
        if x <= 0:
            return 0
        if x >= total:
            return total
        # tensor containing x
        lo, hi = 0, len(starts) - 1
        while lo < hi:
            mid = (lo + hi + 1) // 2
            if starts[mid] <= x:
                lo = mid
            else:
                hi = mid - 1
        t = lo
        while t < len(numels) and int(numels[t]) <= 0:
            t += 1
        s0, n, u = starts[t], int(numels[t]), units[t]
        off = x - s0
        down = (off // u) * u
        up = min(n, down + u)
        return s0 + (down if off - down <= up - off else up)

    cuts = [0]
    for c in range(1, grid):
        cuts.append(max(cuts[-1], snap((c * total) // grid)))
    cuts.append(total)

    pieces = []
    offsets = [0]
    n_slots = [0] * len(numels)
    t = 0
    for c in range(grid):
        a, b = cuts[c], cuts[c + 1]
        while a < b:
            while t < len(numels) and starts[t] + int(numels[t]) <= a:
                t += 1
            s0, n, d2, u = starts[t], int(numels[t]), int(d2s[t]), units[t]
            end = min(b, s0 + n)
            pos = a - s0
            stop = end - s0
            cap = max(u, (MAX_ROWS * d2 // u) * u) if d2 > 0 else stop - pos
            while pos < stop:
                take = min(stop - pos, cap)
                pieces.append((pos, pos + take, t, n_slots[t]))
                n_slots[t] += 1
                pos += take
            a = end
        offsets.append(len(pieces))
    arr = np.zeros(len(pieces), PIECE_DT)
    if pieces:
        p = np.array(pieces, dtype=np.int64)
        arr["begin"], arr["end"], arr["tensor"], arr["slot"] = p[:, 0], p[:, 1], p[:, 2], p[:, 3]
    return arr, np.asarray(offsets, np.int32), n_slots
