"""Shifted-lane (SL) decode packing: the numpy carrier layout and the two rotation stages around the MAC.

Mirrors ``llama3fhe/layouts/shifted_lane.py:41-175`` (the layout) and ``llama3fhe/operators/linear/shifted_lane.py``
(``lane0_mask_vector``, ``mask_lane0``, ``expand_lane0_to_shifted_lanes``, ``fold_shifted_lanes``): same names,
argument meaning and errors, on this engine's primitives.

Layout: slot ``(c, l) = c * lanes + l`` of a ``slots``-slot carrier holds ``x[(c + shift * l) mod D]`` with
``lanes = slots / D`` and ``shift = D / lanes``; a linear whose plan has ``lane_shift = shift`` then needs only
``shift`` diagonals, and the lanes of its output are partial products over the input blocks ``[shift l,
shift (l + 1))``, summed into lane 0 by ``fold_shifted_lanes``.  Ciphertext inputs are not consumed.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from . import fhe

__all__ = ["ShiftedLaneLayout", "lane0_mask_vector", "mask_lane0", "expand_lane0_to_shifted_lanes",
           "fold_shifted_lanes"]


def _power_of_two(v: int, name: str) -> None:
    if int(v) <= 0 or int(v) & (int(v) - 1):
        raise ValueError(f"{name} must be a positive power of two, got {v}.")


@dataclass(frozen=True)
class ShiftedLaneLayout:
    """One-token shifted-lane carrier (``lanes = slots / hidden_dim``)."""

    hidden_dim: int = 4096
    slots: int = 32768

    def __post_init__(self) -> None:
        _power_of_two(self.hidden_dim, "hidden_dim")
        _power_of_two(self.slots, "slots")
        if int(self.slots) % int(self.hidden_dim):
            raise ValueError(f"shifted-lane layout requires slots divisible by hidden_dim, got slots={self.slots}, "
                             f"hidden_dim={self.hidden_dim}.")
        if int(self.hidden_dim) % self.lanes:
            raise ValueError(f"hidden_dim={self.hidden_dim} must be divisible by lanes={self.lanes}.")

    @property
    def lanes(self) -> int:
        return int(self.slots) // int(self.hidden_dim)

    @property
    def shift(self) -> int:
        return int(self.hidden_dim) // self.lanes

    def slot(self, channel: int, lane: int) -> int:
        return int(channel) * self.lanes + int(lane)

    def pack(self, x, *, dtype=np.float64) -> np.ndarray:
        """SL carrier of ``x``: slot (c, l) holds x[(c + shift l) mod D]."""
        x = np.asarray(x, dtype=dtype).reshape(-1)
        if x.shape != (int(self.hidden_dim),):
            raise ValueError(f"pack expects shape {(int(self.hidden_dim),)}, got {x.shape}.")
        s = np.arange(int(self.slots))
        return x[(s // self.lanes + self.shift * (s % self.lanes)) % int(self.hidden_dim)]

    def pack_lane0(self, x, *, dtype=np.float64) -> np.ndarray:
        """Lane-0 carrier of ``x``: lane 0 holds x, the other lanes are zero."""
        x = np.asarray(x, dtype=dtype).reshape(-1)
        if x.shape != (int(self.hidden_dim),):
            raise ValueError(f"lane-0 pack expects shape {(int(self.hidden_dim),)}, got {x.shape}.")
        out = np.zeros((int(self.slots),), dtype=x.dtype)
        out[:: self.lanes] = x
        return out

    def unpack(self, carrier, *, lane: int = 0) -> np.ndarray:
        """``x`` read back from one lane (that lane's shift undone)."""
        carrier = np.asarray(carrier)
        if carrier.shape != (int(self.slots),):
            raise ValueError(f"shifted-lane carrier must have shape {(int(self.slots),)}, got {carrier.shape}.")
        return np.roll(carrier[int(lane):: self.lanes], self.shift * int(lane))

    def is_shifted_lane(self, carrier, *, atol: float = 1e-9) -> bool:
        ref = self.unpack(carrier, lane=0)
        return all(np.allclose(self.unpack(carrier, lane=l), ref, atol=atol) for l in range(1, self.lanes))

    def lane0_to_shifted_offsets(self) -> tuple[int, ...]:
        """slot(c, l) receives x[c + shift l] from slot(c + shift l, 0): a rotation by (D - 1) l."""
        return tuple((int(self.hidden_dim) - 1) * l for l in range(1, self.lanes))

    def fold_offsets(self) -> tuple[int, ...]:
        return tuple(1 << i for i in range(int(self.lanes).bit_length() - 1))


def lane0_mask_vector(plan, *, slots: int) -> np.ndarray:
    """Plaintext vector selecting lane 0 of every channel."""
    slots = int(slots)
    if slots != int(plan.dimension) * int(plan.token_lanes):
        raise ValueError(f"lane mask expects slots={plan.dimension * plan.token_lanes}, got {slots}.")
    mask = np.zeros((slots,), dtype=np.float64)
    mask[:: int(plan.token_lanes)] = 1.0
    return mask


def mask_lane0(cipher, *, plan, crypto_context):
    """``cipher * lane0_mask``, rescaled (one level)."""
    level = int(crypto_context.level_for_cipher(cipher))
    plain = crypto_context.plaintext(lane0_mask_vector(plan, slots=int(crypto_context.max_slots)),
                                     name=f"sl.lane0_mask.{plan.dimension}x{plan.token_lanes}", level=level)
    ctx = crypto_context.context
    return fhe.rescale(fhe.homo_mul_pt(cipher, plain, ctx), ctx)


def expand_lane0_to_shifted_lanes(cipher, *, plan, crypto_context, mask: bool = False):
    """SL carrier from a carrier whose lane 0 holds x: ``token_lanes - 1`` hoisted rotations (one ModUp) and adds;
    ``mask=True`` first zeroes lanes 1.. (one level)."""
    if not plan.shifted_lanes:
        raise ValueError("expand_lane0_to_shifted_lanes needs a shifted-lane plan.")
    ctx = crypto_context.context
    source = mask_lane0(cipher, plan=plan, crypto_context=crypto_context) if mask else cipher
    out = source.deep_copy()
    for term in fhe.unpack_cipher_batch(fhe.fast_rotate(source, tuple(plan.lane_expand_offsets), ctx)):
        out = fhe.homo_add(out, term, ctx)
    return out


def fold_shifted_lanes(cipher, *, plan, crypto_context):
    """Rotate-and-add by 1, 2, 4, ... so lane 0 holds the lane sum (lanes 1.. hold garbage afterwards)."""
    if not plan.shifted_lanes:
        raise ValueError("fold_shifted_lanes needs a shifted-lane plan.")
    ctx = crypto_context.context
    out = cipher.deep_copy()
    for offset in plan.fold_offsets:
        out = fhe.homo_add(out, fhe.homo_rotate(out, int(offset), ctx), ctx)
    return out
