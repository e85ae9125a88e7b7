"""Diagonal (BSGS) linear layers over libholmes_cuda: a batched schedule behind the reference's operator calls.

The reference's own ``LinearOperator`` (``llama3fhe/operators/linear/operator.py:58-639``) runs unchanged on this
engine through :mod:`holmes_b200.easyfhe_compat`; it loops over inputs inside every chunk (``_mac_chunk``: one
``hoisted_mac_sum`` plus a giant alignment rotation per input).  This module is the engine's faster schedule of
the same computation, with call names a caller of the reference recognises (``LinearOperator.apply`` / ``project``
/ ``prepare_baby_rotations`` / ``cache_info``, ``LinearWeight``) and its own geometry types: :class:`BsgsSchedule`
(the schedule knobs; the reference's ``LinearOperatorConfig`` objects are accepted and read by attribute name) and
:class:`BsgsLayout` (babies, giants, chunks and the exact rotation-key set).  All inputs of a call move together:

* baby basis: one batched ModUp of every input, then one key switch per baby offset over all inputs
  (each rotation key is read from HBM once per offset, not once per input);
* per chunk: the diagonal rows are packed and encoded on the GPU (``holmes_pack_diagonals`` ->
  special FFT -> rounding + NTT), one multi-input BSGS MAC produces every input's partial sums, and
  the Horner giant chain runs as batched key switches whose "+ partial[g]" is fused into ModDown;
* the chunk alignment rotation is fused with the running accumulation the same way;
* one batched rescale at the end.

Per input, this is the same sequence of modular operations as the reference's loop (Horner order,
alignment, accumulation, rescale), so the result is residue-for-residue what a per-input run gives.
"""
from __future__ import annotations

import hashlib

import os
import time
from dataclasses import dataclass, field

import numpy as np
import torch

from . import _lib
from . import fhe as F

HOIST_MODES = ("normal", "ext_normal", "ext_double_hoist")
CACHE_MODES = ("none", "middle", "plain", "both")


@dataclass(frozen=True)
class BsgsSchedule:
    """How one square diagonal linear is evaluated: the knobs of the reference's ``LinearOperatorConfig``
    (``llama3fhe/operators/linear/config.py:49-121``) under this engine's own names.

    ``babies`` B baby steps; ``anchor`` babies per anchored block (>= 2; -1 or >= B: one block); ``chunk_rows``
    diagonal rows encoded and multiplied per chunk (at least B); ``reuse_babies`` keeps an input's baby basis for
    the next apply; ``hoist`` the giant-step strategy; ``cache`` which encode stage a weight keeps ("middle": FFT'd
    rows, "plain": NTT plaintexts); ``weight_on_device`` keeps the weight page in HBM; ``lane_shift`` > 0 selects the
    shifted-lane packing (D / lanes diagonals)."""

    babies: int = 32
    anchor: int = 32
    chunk_rows: int = 512
    reuse_babies: bool = True
    hoist: str = "normal"
    cache: str = "none"
    weight_on_device: bool = True
    lane_shift: int = 0

    def __post_init__(self) -> None:
        problems = []
        if int(self.babies) < 1:
            problems.append(f"babies={self.babies} (need >= 1)")
        if int(self.anchor) != -1 and int(self.anchor) < 2:
            problems.append(f"anchor={self.anchor} (need -1 or >= 2)")
        if int(self.chunk_rows) < int(self.babies):
            problems.append(f"chunk_rows={self.chunk_rows} below babies={self.babies}")
        if int(self.lane_shift) < 0:
            problems.append(f"lane_shift={self.lane_shift} (need >= 0)")
        if str(self.hoist).lower() not in HOIST_MODES:
            problems.append(f"hoist={self.hoist!r} (one of {HOIST_MODES})")
        if str(self.cache) not in CACHE_MODES:
            problems.append(f"cache={self.cache!r} (one of {CACHE_MODES})")
        if problems:
            raise ValueError("invalid BSGS schedule: " + "; ".join(problems))

    @classmethod
    def coerce(cls, config) -> "BsgsSchedule":
        """This schedule from a ``BsgsSchedule``, None (the defaults) or any object with the attribute names of the
        reference's ``LinearOperatorConfig`` (its own instances included), read field by field."""
        if config is None:
            return cls()
        if isinstance(config, cls):
            return config
        return cls(babies=int(config.baby_steps), anchor=int(config.baby_anchor_step),
                   chunk_rows=int(config.max_plaintext_rows),
                   reuse_babies=bool(getattr(config, "reuse_baby_rotations", True)),
                   hoist=str(getattr(config, "hoist_strategy", "normal")).lower(),
                   cache=str(getattr(config, "constant_cache_mode", "none")),
                   weight_on_device=str(getattr(config, "raw_weight_policy", "device")) == "device",
                   lane_shift=int(getattr(config, "lane_shift", 0)))

    def layout(self, dimension: int, lanes: int) -> "BsgsLayout":
        return BsgsLayout(int(dimension), int(lanes), int(self.babies), int(self.anchor), int(self.chunk_rows),
                          int(self.lane_shift))

    def rotation_keys(self, dimension: int, lanes: int, conjugation_slots: int | None = None) -> tuple[int, ...]:
        return self.layout(dimension, lanes).rotation_keys(self.hoist, conjugation_slots)


#: the reference's production schedule for every Llama-3 projection (QKV, W_O, gate/up, down): 64 babies, one
#: anchor block, 512 rows per chunk (``llama3fhe/operators/linear/config.py:123-134``)
PRODUCTION = BsgsSchedule(babies=64, anchor=64, chunk_rows=512)


@dataclass(frozen=True)
class Chunk:
    """Giants ``first .. first + count - 1`` of a layout, encoded and multiplied together."""

    index: int
    first: int
    count: int

    @property
    def name(self) -> str:
        return f"chunk.{int(self.index)}"


class BsgsLayout:
    """BSGS geometry of one D x D diagonal page over ``lanes`` token lanes (feature-major slot f * lanes + t).

    Diagonal row (g, b) holds ``W[(f - g B) mod D, (f + b + lane_shift t) mod D]`` at slot (f, t); the matvec is
    ``sum_g rot(sum_b row(g, b) * rot(x, b lanes), g B lanes)``: babies at strides ``b lanes``, giants at stride
    ``B lanes``, the giants split into chunks of ``chunk_rows / B``.  ``rotation_keys`` is the exact key set a
    schedule needs (pinned against the reference's ``linear_rotations``, ``config.py:338-380``, by the golden
    fixtures)."""

    def __init__(self, dimension: int, lanes: int, babies: int, anchor: int, chunk_rows: int, lane_shift: int = 0):
        if dimension < 1 or lanes < 1 or babies < 1:
            raise ValueError(f"layout needs positive dimension, lanes and babies, got {dimension}, {lanes}, {babies}")
        if lane_shift and lane_shift * lanes != dimension:
            raise ValueError(f"lane_shift={lane_shift} must be dimension / lanes = {dimension} / {lanes} "
                             f"for the shifted-lane packing")
        self.dimension, self.lanes, self.babies = dimension, lanes, babies
        self.anchor, self.chunk_rows, self.lane_shift = anchor, chunk_rows, lane_shift
        self.diagonals = lane_shift if lane_shift else dimension
        if self.diagonals % babies:
            raise ValueError(f"babies={babies} does not divide the {self.diagonals} diagonals")
        self.giants = self.diagonals // babies
        self.giant_stride = babies * lanes
        self.baby_strides = tuple(b * lanes for b in range(babies))
        per = max(1, chunk_rows // babies)
        self.chunks = tuple(Chunk(i, first, min(per, self.giants - first))
                            for i, first in enumerate(range(0, self.giants, per)))
        width = anchor if 2 <= anchor < babies else babies
        #: baby blocks (start, width): anchored blocks reach their babies through one anchor rotation
        self.blocks = tuple((b0, min(width, babies - b0)) for b0 in range(0, babies, width))
        keys = {s * lanes for s in range(1, width)}
        if len(self.blocks) > 1:
            keys.add(anchor * lanes)
        self.baby_keys = tuple(sorted(keys))
        #: shifted lanes: the lane-fold rotations (1, 2, 4, ...) and the lane-0 -> all-lanes expansion rotations
        self.fold_strides = tuple(1 << i for i in range(lanes.bit_length() - 1)) if lane_shift else ()
        self.expand_strides = tuple((dimension - 1) * t for t in range(1, lanes)) if lane_shift else ()
        self.key = (dimension, lanes, babies, chunk_rows, lane_shift, anchor)

    def rotation_keys(self, hoist: str = "normal", conjugation_slots: int | None = None) -> tuple[int, ...]:
        keys = set(self.baby_keys)
        widest = max(c.count for c in self.chunks)
        if widest > 1:                                 # giant steps inside a chunk
            if str(hoist).lower() == "ext_double_hoist":
                keys.update(s * self.giant_stride for s in range(1, widest))
            else:
                keys.add(self.giant_stride)
        keys.update(c.first * self.giant_stride for c in self.chunks if c.first)   # chunk alignment
        keys.update(self.fold_strides)
        keys.update(self.expand_strides)
        if conjugation_slots is not None:
            keys.add(4 * int(conjugation_slots) - 1)
        keys.discard(0)
        return tuple(sorted(keys))


# ----------------------------------------------------------------------------------------------------- session


class Session:
    """The ``crypto_context`` object the operators receive (reference: backend.py:249-396)."""

    def __init__(self, client: F.Client, context: F.Context) -> None:
        self.tensor = torch
        self.fhe = F
        self.client = client
        self.context = context
        self.max_slots = int(context.max_slots)

    @property
    def device(self) -> str:
        return str(self.context.device)

    def level_for_cipher(self, cipher) -> int:
        return int(self.context.L) - int(cipher.state.cur_limbs)

    def encrypt(self, values, *, level: int, slots: int | None = None, counter: int | None = None):
        cur = int(self.context.L) - int(level)
        return self.client.encrypt(np.asarray(values).reshape(-1), slots=self.max_slots if slots is None else slots,
                                   cur_limbs=cur, scaling_factor=self.context.scale_at(cur), counter=counter)

    def decrypt(self, cipher, item: int = 0) -> np.ndarray:
        return np.asarray(self.client.decrypt(cipher, item)).reshape(-1)

    def plaintext(self, values, *, name: str, level: int, slots: int | None = None, dtype=np.float64,
                  is_ext: bool = False) -> F.Plaintext:
        """A public vector encoded at ``level``'s limbs and scale (reference: backend.py:303-330), cached per
        name, level, slot count and contents."""
        array = np.ascontiguousarray(np.asarray(values, dtype=dtype).reshape(-1))
        slots = self.max_slots if slots is None else int(slots)
        key = (str(name), int(level), slots, bool(is_ext), hashlib.sha1(array.tobytes()).hexdigest())
        cache = self.__dict__.setdefault("_plaintexts", {})
        hit = cache.get(key)
        if hit is not None:
            return hit
        ctx = self.context
        cur = int(ctx.L) - int(level)
        if is_ext:   # the extended basis Q u P (operators/attention/prefill/input.py:1013-1018)
            z = torch.from_numpy(array.astype(np.complex128)).reshape(1, slots)
            pv = F.encode_rows(ctx, z, cur, ctx.scale_at(cur), slots, ext=True)
            pt = F.Plaintext([pv], F.CipherState(cur, 1, ctx.scale_at(cur)), slots, True, 1, ctx)
        else:
            bundle = F.ConstantBundle({"value": F.PackedRaw(torch.from_numpy(array.astype(np.complex128)))})
            pt = bundle.plaintext("value", state=F.CipherState(cur, 1, ctx.scale_at(cur)), slots=slots, context=ctx)
        ctx.check_encode_range()
        cache[key] = pt
        return pt


def create_session(spec: F.CKKSContextSpec, device: str = "cuda") -> Session:
    client, context = F.generate_client_context(spec, device)
    return Session(client, context)


# ----------------------------------------------------------------------------------------------------- weight


def pack_chunk(ctx: F.Context, weight: torch.Tensor, layout: BsgsLayout, chunk: Chunk, slots: int) -> torch.Tensor:
    """Diagonal rows of ``chunk`` as complex128 [rows][slots] (the rows of the reference's packers,
    ``llama3fhe/operators/linear/weight.py:122-154``)."""
    rows = chunk.count * layout.babies
    out = torch.empty((rows, slots), dtype=torch.complex128, device=ctx.device)
    w = weight
    cplx = bool(w.is_complex())
    src = torch.view_as_real(w) if cplx else w
    _lib.call("holmes_pack_diagonals", src.data_ptr(), int(cplx), layout.dimension, layout.lanes, layout.babies,
              chunk.first, chunk.count, layout.lane_shift, int(slots),
              torch.view_as_real(out).data_ptr(), 2 * slots, F._stream())
    return out


class LinearWeight:
    """One square physical weight page and its per-chunk constant bundles (reference: weight.py:232-659)."""

    def __init__(self, weight, *, dtype, crypto_context) -> None:
        self.dtype = np.dtype(dtype)
        self.crypto_context = crypto_context
        if torch.is_tensor(weight):
            w = weight
            shape = tuple(int(v) for v in w.shape)
        else:
            w = np.asarray(weight)
            shape = w.shape
        if len(shape) != 2 or shape[0] != shape[1]:
            raise ValueError(f"linear weight must be one square physical page, got {shape}.")
        self._weight = w
        self._dimension = int(shape[0])
        self._device_source = None
        self._upload_event = None
        self._bundles: dict = {}
        self._closed = False
        self.setup_seconds = 0.0

    @property
    def dimension(self) -> int:
        return self._dimension

    @property
    def closed(self) -> bool:
        return self._closed

    def prepare(self, schedule=None) -> float:
        """Upload the page to HBM (once); returns the seconds spent.  ``schedule`` is accepted for the reference's
        signature and not needed."""
        if self._closed:
            raise RuntimeError("the weight page has been closed")
        del schedule
        start = time.perf_counter()
        if self._device_source is None:
            ctx = self.crypto_context.context
            cplx = np.issubdtype(self.dtype, np.complexfloating)
            tdtype = torch.complex128 if cplx else torch.float64
            w = self._weight
            if not torch.is_tensor(w):
                w = torch.from_numpy(np.ascontiguousarray(np.asarray(w, dtype=self.dtype)))
            if w.device.type == "cpu" and w.is_pinned() and w.dtype == tdtype and w.is_contiguous():
                # A pinned host page is uploaded on a side stream, so the copy overlaps what the caller's stream
                # runs before the first encode (the baby rotations of apply); plaintext() waits for it.
                main = torch.cuda.current_stream(ctx.device)
                up = getattr(ctx, "_upload_stream", None)
                if up is None:
                    up = ctx._upload_stream = torch.cuda.Stream(device=ctx.device)
                dev = torch.empty(w.shape, dtype=tdtype, device=ctx.device)
                up.wait_stream(main)
                with torch.cuda.stream(up):
                    dev.copy_(w, non_blocking=True)
                dev.record_stream(up)
                self._upload_event = torch.cuda.Event()
                self._upload_event.record(up)
                self._device_source = dev
            else:
                self._device_source = w.to(device=ctx.device, dtype=tdtype).contiguous()
        elapsed = time.perf_counter() - start
        self.setup_seconds += elapsed
        return elapsed

    def _bundle(self, layout: BsgsLayout, chunk: Chunk, schedule: BsgsSchedule) -> F.ConstantBundle:
        key = (*layout.key, chunk.index, schedule.cache)
        bundle = self._bundles.get(key)
        if bundle is None:
            self.prepare()
            ctx = self.crypto_context.context

            def packer(source, slots, context, layout=layout, chunk=chunk):
                del context
                return pack_chunk(ctx, source, layout, chunk, slots)

            bundle = F.ConstantBundle(vectors={chunk.name: F.UnpackedRaw(self._device_source, packer)},
                                      cache_mode=schedule.cache)
            if schedule.cache != "none":
                self._bundles[key] = bundle
        return bundle

    def plaintext(self, layout: BsgsLayout, chunk: Chunk, *, level: int, schedule) -> F.Plaintext:
        """The NTT plaintexts of ``chunk``'s diagonal rows at ``level`` (over Q u P for the extended hoists)."""
        schedule = BsgsSchedule.coerce(schedule)
        if self._closed:
            raise RuntimeError("the weight page has been closed")
        if layout.dimension != self.dimension:
            raise ValueError(f"layout of dimension {layout.dimension} applied to a {self.dimension}-wide page")
        ctx = self.crypto_context.context
        cur = int(ctx.L) - int(level)
        bundle = self._bundle(layout, chunk, schedule)
        if self._upload_event is not None:
            torch.cuda.current_stream(ctx.device).wait_event(self._upload_event)
        return bundle.plaintext(chunk.name, state=F.CipherState(cur, 1, ctx.scale_at(cur)),
                                slots=int(self.crypto_context.max_slots), context=ctx,
                                is_ext=schedule.hoist != "normal", cache=True)

    def cache_info(self) -> dict:
        totals: dict = {"bundle_count": len(self._bundles)}
        for b in self._bundles.values():
            for k, v in b.cache_info().items():
                totals[k] = totals.get(k, 0) + int(v)
        for k in ("middle_entries", "plain_entries", "middle_bytes", "plain_bytes", "total_bytes", "middle_hits",
                  "middle_misses", "plain_hits", "plain_misses"):
            totals.setdefault(k, 0)
        return totals

    def clear_cache(self) -> None:
        for b in self._bundles.values():
            b.clear_cache()
        self._bundles.clear()

    def close(self) -> None:
        self.clear_cache()
        self._device_source = None
        self._upload_event = None
        self._weight = None
        self._closed = True

    def __enter__(self) -> "LinearWeight":
        if self._closed:
            raise RuntimeError("the weight page has been closed")
        return self

    def __exit__(self, *exc) -> None:
        self.close()


# ----------------------------------------------------------------------------------------------------- operator


_EMPTY_PROFILE = {"weight_prepare_cpu": 0.0, "weight_upload": 0.0, "baby_precompute": 0.0,
                  "baby_precompute_enqueue": 0.0, "baby_cache_hits": 0.0, "baby_cache_misses": 0.0,
                  "pack_encode": 0.0, "online": 0.0, "rescale": 0.0}


class _Babies:
    """Baby basis of a batch of inputs: storage [B][2][I][cur][N] (baby-major, so a contiguous range of babies is
    one contiguous block for the sharded build's all-gather; input i's babies are strided by 2 I cur N); with
    ``ext`` the babies are over the extended basis Q u P, [cur + K] limbs."""

    def __init__(self, sources, level: int, storage: torch.Tensor, state: F.CipherState, slots: int,
                 ext: bool = False) -> None:
        self.sources = tuple(sources)
        self.level = level
        self.storage = storage
        self.state = state
        self.slots = slots
        self.ext = bool(ext)
        self.pending = None  # all-gather still filling other ranks' babies (sharded build)

    def ready(self) -> None:
        """Make the current stream wait for the sharded build's all-gather."""
        if self.pending is not None:
            self.pending.wait()
            self.pending = None

    def blocks(self, ctx: F.Context) -> list[F.Cipher]:
        B, inputs = int(self.storage.shape[0]), int(self.storage.shape[2])
        out = []
        for i in range(inputs):
            c0 = self.storage[:, 0, i]
            c1 = self.storage[:, 1, i]
            out.append(F.Cipher([c0, c1], self.state, self.slots, self.ext, B, ctx))
        return out


class LinearOperator:
    """A reusable BSGS schedule with an operator-local baby cache (reference: operator.py:58-639)."""

    def __init__(self, *, crypto_context, token_lanes: int, config=None, baby_shard=None) -> None:
        """``config``: a :class:`BsgsSchedule`, or the reference's ``LinearOperatorConfig`` (read by attribute name).
        ``baby_shard = (rank, world, group)`` splits the baby key switches over the ranks of ``group`` (each rank
        holding the same inputs) and all-gathers the basis; None builds it locally."""
        self.crypto_context = crypto_context
        self.baby_shard = None if baby_shard is None else (int(baby_shard[0]), int(baby_shard[1]), baby_shard[2])
        self.token_lanes = int(token_lanes)
        if self.token_lanes <= 0:
            raise ValueError(f"token_lanes={token_lanes} must be positive")
        self.config = BsgsSchedule.coerce(config)
        self._baby_cache: dict = {}
        self._baby_hits = 0
        self._baby_misses = 0
        self._closed = False

    @property
    def closed(self) -> bool:
        return self._closed

    def layout(self, dimension: int) -> BsgsLayout:
        return self.config.layout(int(dimension), self.token_lanes)

    # -- baby basis ----------------------------------------------------------------------------------------
    def _baby_key(self, inputs, plan: BsgsLayout):
        return (tuple(id(c) for c in inputs), plan.key)

    def _lookup_babies(self, inputs, plan: BsgsLayout, level: int):
        key = self._baby_key(inputs, plan)
        entry = self._baby_cache.get(key)
        if entry is not None and all(a is b for a, b in zip(entry.sources, inputs)) and entry.level == level:
            self._baby_hits += len(inputs)
            return entry
        if entry is not None:
            del self._baby_cache[key]
        self._baby_misses += len(inputs)
        return None

    def _build_babies(self, inputs, plan: BsgsLayout, level: int) -> _Babies:
        """All B baby rotations of every input.  With a baby shard (rank, world, group) set, this rank key-switches
        only its contiguous range of babies and an all-gather over the group fills in the rest: every rank then
        holds the whole basis at 1 / world of the key switches."""
        ctx = self.crypto_context.context
        cur = int(inputs[0].state.cur_limbs)
        n_in = len(inputs)
        B = plan.babies
        ext = self.config.hoist != "normal"
        limbs = cur + (ctx.K if ext else 0)
        storage = torch.empty((B, 2, n_in, limbs, ctx.N), dtype=torch.uint64, device=ctx.device)
        c0 = torch.stack([c.cv[0][0, :cur] for c in inputs])
        c1 = torch.stack([c.cv[1][0, :cur] for c in inputs])
        lo, hi = 0, B
        shard = self.baby_shard
        if shard is not None and B % shard[1] == 0 and shard[1] > 1:
            lo, hi = shard[0] * B // shard[1], (shard[0] + 1) * B // shard[1]
        if lo == 0:
            if ext:   # baby 0 over Q u P: (P c0, P c1), zero on the special limbs
                pm = ctx.p_mod_q_dev(cur)
                for c, src in ((0, c0), (1, c1)):
                    storage[0, c, :, cur:].zero_()
                    _lib.call("holmes_mul_const", ctx.handle, src.data_ptr(), pm.data_ptr(), storage[0, c].data_ptr(),
                              n_in, cur, F._item_stride(src), F._item_stride(storage[0, c]), F._stream())
            else:
                storage[0, 0].copy_(c0)
                storage[0, 1].copy_(c1)
        if max(lo, 1) < hi:
            digits, dig_item = F._modup(ctx, c1, cur, n_in, True)
            for b in range(max(lo, 1), hi):
                g = ctx.galois(plan.baby_strides[b])
                if ext:
                    key_t, cap = ctx.switch_key(g, cur)
                    _lib.call("holmes_keyswitch_ext", ctx.handle, digits.data_ptr(), dig_item, cur, key_t.data_ptr(),
                              cap, int(g), c0.data_ptr(), F._item_stride(c0), storage[b, 0].data_ptr(),
                              storage[b, 1].data_ptr(), F._item_stride(storage[b, 0]), n_in, F._stream())
                else:
                    F._keyswitch(ctx, digits, dig_item, cur, g, ctx.switch_key(g, cur), c0, None, F._item_stride(c0),
                                 storage[b, 0], storage[b, 1], n_in)
        entry = _Babies(inputs, level, storage, inputs[0].state, int(inputs[0].slots), ext)
        if (lo, hi) != (0, B):
            from .collectives import all_gather_rows
            # asynchronous: the first chunk's encode (which needs no babies) overlaps the transfer
            entry.pending = all_gather_rows(storage, lo, hi, shard[1], shard[2], async_op=True)
        if self.config.reuse_babies:
            self._baby_cache[self._baby_key(inputs, plan)] = entry
        return entry

    def prepare_baby_rotations(self, input_ciphers, *, dimension: int) -> dict:
        if self._closed:
            raise RuntimeError("the linear operator has been closed")
        inputs = tuple(input_ciphers)
        profile = {"baby_precompute": 0.0, "baby_precompute_enqueue": 0.0, "baby_cache_hits": 0.0,
                   "baby_cache_misses": 0.0}
        if not inputs or not self.config.reuse_babies:
            return profile
        plan = self.layout(int(dimension))
        levels = {int(self.crypto_context.level_for_cipher(c)) for c in inputs}
        if len(levels) != 1:
            raise ValueError(f"the inputs of one apply must share a level, got levels {sorted(levels)}")
        level = levels.pop()
        hits, misses = self._baby_hits, self._baby_misses
        start = time.perf_counter()
        if self._lookup_babies(inputs, plan, level) is None:
            self._build_babies(inputs, plan, level)
            torch.cuda.synchronize(self.crypto_context.context.device)
            profile["baby_precompute"] = time.perf_counter() - start
            profile["baby_precompute_enqueue"] = profile["baby_precompute"]
        profile["baby_cache_hits"] = float(self._baby_hits - hits)
        profile["baby_cache_misses"] = float(self._baby_misses - misses)
        return profile

    def clear_baby_cache(self) -> None:
        self._baby_cache.clear()

    def cache_info(self) -> dict:
        return {"baby_entries": sum(len(e.sources) for e in self._baby_cache.values()),
                "baby_hits": int(self._baby_hits), "baby_misses": int(self._baby_misses)}

    # -- apply ---------------------------------------------------------------------------------------------
    def apply(self, input_ciphers, weight: LinearWeight, *, chunk_indices=None, rescale: bool = True):
        """W x for every input (single non-extended ciphertexts at one level, at most 32); ``chunk_indices`` limits
        the sum to those chunks (a partial at scale degree 2 without ``rescale``).  Returns (outputs, stage
        seconds)."""
        if self._closed:
            raise RuntimeError("the linear operator has been closed")
        strategy = self.config.hoist
        ext = strategy != "normal"
        double = strategy == "ext_double_hoist"
        inputs = tuple(input_ciphers)
        if not inputs:
            return (), dict(_EMPTY_PROFILE)
        if weight.closed:
            raise RuntimeError("the weight page has been closed")
        if weight.crypto_context is not self.crypto_context:
            raise ValueError("the operator and the weight page belong to different sessions")
        if len(inputs) > 32:
            raise ValueError(f"{len(inputs)} inputs in one apply; the multi-input MAC takes at most 32")
        plan = self.layout(weight.dimension)
        if chunk_indices is None:
            chunks = plan.chunks
        else:
            wanted = tuple(int(i) for i in chunk_indices)
            if not wanted or len(set(wanted)) != len(wanted):
                raise ValueError(f"chunk_indices {wanted} must name distinct chunks, at least one")
            for i in wanted:
                if i < 0 or i >= len(plan.chunks):
                    raise IndexError(f"chunk index {i} outside [0, {len(plan.chunks)})")
            chunks = tuple(plan.chunks[i] for i in wanted)
        levels = {int(self.crypto_context.level_for_cipher(c)) for c in inputs}
        if len(levels) != 1:
            raise ValueError(f"the inputs of one apply must share a level, got levels {sorted(levels)}")
        level = levels.pop()
        if any(c.batch_size != 1 or c.is_ext for c in inputs):
            raise ValueError("every input must be one non-extended ciphertext")
        ctx = self.crypto_context.context
        stage = dict(_EMPTY_PROFILE)
        stage["weight_upload"] = float(weight.prepare(self.config))
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
        ev[0].record()
        babies = self._lookup_babies(inputs, plan, level) if self.config.reuse_babies else None
        if babies is None:
            babies = self._build_babies(inputs, plan, level)
        ev[1].record()
        cur = int(inputs[0].state.cur_limbs)
        n_in = len(inputs)
        blocks = babies.blocks(ctx)
        acc0 = acc1 = None
        pt_state = None
        encode_events = []
        for chunk in chunks:
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
            pts = weight.plaintext(plan, chunk, level=level, schedule=self.config)
            e1.record()
            pt_state = pts.state
            babies.ready()
            res = F.bsgs_partial_sums(ctx, blocks, pts, chunk.count)
            del pts
            if ext:   # babies and MAC over Q u P, one ModDown per giant partial
                G = int(res.shape[1])
                down = torch.empty((2, G, n_in, cur, ctx.N), dtype=torch.uint64, device=ctx.device)
                scratch = ctx.workspace("ks", G * n_in * 2 * (ctx.K + cur) * ctx.N)
                _lib.call("holmes_moddown", ctx.handle, res[0].data_ptr(), res[1].data_ptr(), (cur + ctx.K) * ctx.N,
                          cur, down[0].data_ptr(), down[1].data_ptr(), cur * ctx.N, G * n_in, scratch.data_ptr(),
                          F._stream())
                res = down
            if double:   # ext_double_hoist: every giant rotated directly over Q u P, summed, one ModDown
                g0, g1 = F.giant_double_hoist(ctx, res, plan.giant_stride)
            else:        # normal / ext_normal: the Horner chain
                g0, g1 = F.giant_horner(ctx, res, plan.giant_stride)
            shift = chunk.first * plan.giant_stride
            if acc0 is None:
                if shift:
                    n0, n1 = torch.empty_like(g0), torch.empty_like(g1)
                    F.rotate_batch(ctx, g0, g1, cur, shift, n0, n1, reuse=False)
                    acc0, acc1 = n0, n1
                else:
                    acc0, acc1 = g0.clone(), g1.clone()
            else:
                n0, n1 = torch.empty_like(acc0), torch.empty_like(acc1)
                if shift:
                    F.rotate_batch(ctx, g0, g1, cur, shift, n0, n1, post0=acc0, post1=acc1, reuse=False)
                else:
                    F._ew(ctx, 0, g0, acc0, n0, cur)
                    F._ew(ctx, 0, g1, acc1, n1, cur)
                acc0, acc1 = n0, n1
            encode_events.append((e0, e1))  # read after the final synchronisation
        ev[2].record()
        sf = None
        if babies.state.scaling_factor is not None and pt_state.scaling_factor is not None:
            sf = float(babies.state.scaling_factor) * float(pt_state.scaling_factor)
        state = F.CipherState(cur, int(babies.state.scale_degree) + int(pt_state.scale_degree), sf)
        batch = F.Cipher([acc0, acc1], state, inputs[0].slots, False, n_in, ctx)
        if rescale:
            batch = F.rescale(batch, ctx)
        ev[3].record()
        ctx.check_encode_range()   # one device read per apply (the encoder's 2^61 limit)
        outputs = tuple(batch.cipher_like([batch.cv[0][i:i + 1], batch.cv[1][i:i + 1]], batch_size=1)
                        for i in range(n_in))
        stage["baby_precompute"] = ev[0].elapsed_time(ev[1]) / 1e3
        stage["online"] = ev[1].elapsed_time(ev[2]) / 1e3
        stage["rescale"] = ev[2].elapsed_time(ev[3]) / 1e3
        stage["pack_encode"] = sum(a.elapsed_time(b) for a, b in encode_events) / 1e3
        return outputs, stage

    def project(self, input_ciphers, weight, *, dtype, chunk_indices=None, rescale: bool = True):
        start = time.perf_counter()
        with LinearWeight(weight, dtype=np.dtype(dtype), crypto_context=self.crypto_context) as prepared:
            prep = time.perf_counter() - start
            outputs, profile = self.apply(input_ciphers, prepared, chunk_indices=chunk_indices, rescale=rescale)
            profile["weight_prepare_cpu"] = float(prep)
            return outputs, profile

    def close(self) -> None:
        self.clear_baby_cache()
        self._closed = True

    def __enter__(self) -> "LinearOperator":
        if self._closed:
            raise RuntimeError("the linear operator has been closed")
        return self

    def __exit__(self, *exc) -> None:
        self.close()
