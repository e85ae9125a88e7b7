"""NumPy restatement of the diagonal packing and BSGS plaintext semantics -- TEST INFRASTRUCTURE ONLY.

* ``diagonal_rows`` follows ``llama3fhe/operators/linear/weight.py:122-154`` (``_cpu_packer``):
  ``row(g, b)[s] = W[(f - g B) mod D, (f + b + lane_shift * lane) mod D]`` with ``f = s // lanes``,
  ``lane = s % lanes``, rows ordered giant-major over one chunk.
* ``bsgs_matvec`` follows ``llama3fhe/layouts/shifted_lane.py:201-268``: baby rotations by
  ``b * lanes`` slots, giant rotations by ``g * B * lanes`` slots, rotation ``np.roll(v, -r)``.
"""
from __future__ import annotations

import numpy as np


def rotate(v: np.ndarray, r: int) -> np.ndarray:
    return np.roll(np.asarray(v), -int(r))


def diagonal_rows(weight: np.ndarray, *, dimension: int, token_lanes: int, baby_steps: int, giant_base: int,
                  giant_count: int, lane_shift: int = 0, slots: int | None = None) -> np.ndarray:
    slots = dimension * token_lanes if slots is None else int(slots)
    s = np.arange(slots, dtype=np.int64)
    f = s // token_lanes
    lane = s % token_lanes
    rows = []
    for gr in range(giant_count):
        g = giant_base + gr
        out_f = (f - g * baby_steps) % dimension
        for b in range(baby_steps):
            in_f = (f + b + lane_shift * lane) % dimension
            rows.append(np.asarray(weight)[out_f, in_f])
    return np.asarray(rows)


def bsgs_matvec(weight: np.ndarray, carrier: np.ndarray, *, dimension: int, token_lanes: int, baby_steps: int,
                lane_shift: int = 0) -> np.ndarray:
    diagonals = dimension if lane_shift == 0 else lane_shift
    giants = diagonals // baby_steps
    carrier = np.asarray(carrier)
    babies = [rotate(carrier, b * token_lanes) for b in range(baby_steps)]
    rows = diagonal_rows(weight, dimension=dimension, token_lanes=token_lanes, baby_steps=baby_steps,
                         giant_base=0, giant_count=giants, lane_shift=lane_shift, slots=carrier.size)
    out = np.zeros(carrier.shape, dtype=np.result_type(carrier, weight))
    for g in range(giants):
        acc = np.zeros_like(out)
        for b in range(baby_steps):
            acc = acc + babies[b] * rows[g * baby_steps + b]
        out = out + rotate(acc, g * baby_steps * token_lanes)
    return out
