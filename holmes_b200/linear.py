"""Diagonal (BSGS) linear layers over libholmes_cuda, with the reference's operator API.

Public names, arguments and validation follow ``llama3fhe/operators/linear`` (config.py:49-380,
operator.py:58-639, weight.py:232-659): ``LinearOperatorConfig``, ``LinearPlan``, ``LinearChunk``,
``BabyBlock``, ``linear_rotations``, ``LLAMA3_LINEAR_SCHEDULES``, ``LinearWeight`` and
``LinearOperator`` (``apply`` / ``project`` / ``prepare_baby_rotations`` / ``cache_info``).

What differs is the schedule underneath ``apply``.  The reference loops over inputs inside every
chunk (``_mac_chunk``: one ``hoisted_mac_sum`` plus a giant alignment rotation per input).  Here all
inputs of a call move together:

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

_CACHE_MODES = {"none", "middle", "plain", "both"}
_HOIST_STRATEGIES = {"normal", "ext_normal", "ext_double_hoist"}
_RAW_WEIGHT_POLICIES = {"device", "host"}


def default_linear_encode_depth() -> int:
    raw = os.environ.get("LLAMA_FHE_LINEAR_ENCODE_DEPTH", "0").strip()
    try:
        depth = int(raw or "0")
    except ValueError as exc:
        raise ValueError(f"LLAMA_FHE_LINEAR_ENCODE_DEPTH must be a non-negative integer, got {raw!r}.") from exc
    if depth < 0:
        raise ValueError(f"LLAMA_FHE_LINEAR_ENCODE_DEPTH must be a non-negative integer, got {raw!r}.")
    return depth


@dataclass(frozen=True)
class LinearOperatorConfig:
    """Schedule and cache policy of one diagonal linear (reference: config.py:49-121)."""

    baby_steps: int = 32
    baby_anchor_step: int = 32
    max_plaintext_rows: int = 512
    reuse_baby_rotations: bool = True
    hoist_strategy: str = "normal"
    constant_cache_mode: str = "none"
    raw_weight_policy: str = "device"
    lane_shift: int = 0
    encode_depth: int = field(default_factory=default_linear_encode_depth)

    def __post_init__(self) -> None:
        if int(self.baby_steps) <= 0:
            raise ValueError("baby_steps must be positive.")
        if int(self.encode_depth) < 0:
            raise ValueError("encode_depth must be zero or positive.")
        if int(self.baby_anchor_step) in (0, 1):
            raise ValueError("baby_anchor_step must be at least two or -1.")
        if int(self.baby_anchor_step) < -1:
            raise ValueError("baby_anchor_step must be positive or -1.")
        if int(self.max_plaintext_rows) < int(self.baby_steps):
            raise ValueError("max_plaintext_rows must hold one baby-step group.")
        if int(self.lane_shift) < 0:
            raise ValueError("lane_shift must be zero or positive.")
        if str(self.hoist_strategy).lower() not in _HOIST_STRATEGIES:
            raise ValueError("hoist_strategy must be 'normal', 'ext_normal', or 'ext_double_hoist'.")
        if str(self.constant_cache_mode) not in _CACHE_MODES:
            raise ValueError(f"constant_cache_mode must be one of {sorted(_CACHE_MODES)}, "
                             f"got {self.constant_cache_mode!r}.")
        if str(self.raw_weight_policy) not in _RAW_WEIGHT_POLICIES:
            raise ValueError(f"raw_weight_policy must be 'device' or 'host', got {self.raw_weight_policy!r}.")

    def plan(self, *, dimension: int, token_lanes: int) -> "LinearPlan":
        return LinearPlan(dimension=int(dimension), token_lanes=int(token_lanes), baby_steps=int(self.baby_steps),
                          baby_anchor_step=int(self.baby_anchor_step),
                          max_plaintext_rows=int(self.max_plaintext_rows), lane_shift=int(self.lane_shift))


def _production_linear_config() -> LinearOperatorConfig:
    return LinearOperatorConfig(baby_steps=64, baby_anchor_step=64, max_plaintext_rows=512, reuse_baby_rotations=True,
                                hoist_strategy="normal", constant_cache_mode="none", raw_weight_policy="device")


@dataclass(frozen=True)
class Llama3LinearSchedules:
    qkv: LinearOperatorConfig = field(default_factory=_production_linear_config)
    w_o: LinearOperatorConfig = field(default_factory=_production_linear_config)
    gate_up: LinearOperatorConfig = field(default_factory=_production_linear_config)
    down: LinearOperatorConfig = field(default_factory=_production_linear_config)


LLAMA3_LINEAR_SCHEDULES = Llama3LinearSchedules()


@dataclass(frozen=True)
class LinearChunk:
    index: int
    giant_base: int
    giant_count: int

    @property
    def name(self) -> str:
        return f"chunk.{int(self.index)}"


@dataclass(frozen=True)
class BabyBlock:
    start: int
    width: int


@dataclass(frozen=True)
class LinearPlan:
    """BSGS geometry of one square diagonal block (reference: config.py:150-336)."""

    dimension: int
    token_lanes: int
    baby_steps: int
    baby_anchor_step: int
    max_plaintext_rows: int
    lane_shift: int = 0

    def __post_init__(self) -> None:
        if int(self.dimension) <= 0:
            raise ValueError("dimension must be positive.")
        if int(self.token_lanes) <= 0:
            raise ValueError("token_lanes must be positive.")
        if int(self.baby_steps) <= 0:
            raise ValueError("baby_steps must be positive.")
        if int(self.lane_shift) < 0:
            raise ValueError("lane_shift must be zero or positive.")
        if int(self.lane_shift) and int(self.lane_shift) * int(self.token_lanes) != int(self.dimension):
            raise ValueError("shifted-lane packing requires lane_shift * token_lanes == dimension, got "
                             f"{self.lane_shift} * {self.token_lanes} != {self.dimension}.")
        if int(self.diagonals) % int(self.baby_steps):
            raise ValueError(f"baby_steps={self.baby_steps} must divide diagonals={self.diagonals} "
                             f"(dimension={self.dimension}, lane_shift={self.lane_shift}).")
        if int(self.baby_anchor_step) in (0, 1) or int(self.baby_anchor_step) < -1:
            raise ValueError("baby_anchor_step must be at least two or -1.")
        if int(self.max_plaintext_rows) < int(self.baby_steps):
            raise ValueError("max_plaintext_rows must hold one baby-step group.")

    @property
    def shifted_lanes(self) -> bool:
        return int(self.lane_shift) > 0

    @property
    def diagonals(self) -> int:
        return int(self.lane_shift) if self.shifted_lanes else int(self.dimension)

    @property
    def giant_steps(self) -> int:
        return self.diagonals // int(self.baby_steps)

    @property
    def fold_offsets(self) -> tuple[int, ...]:
        if not self.shifted_lanes:
            return ()
        return tuple(1 << i for i in range(int(self.token_lanes).bit_length() - 1))

    @property
    def lane_expand_offsets(self) -> tuple[int, ...]:
        if not self.shifted_lanes:
            return ()
        return tuple((int(self.dimension) - 1) * lane for lane in range(1, int(self.token_lanes)))

    @property
    def chunk_giants(self) -> int:
        return max(1, int(self.max_plaintext_rows) // int(self.baby_steps))

    @property
    def giant_offset(self) -> int:
        return int(self.baby_steps) * int(self.token_lanes)

    @property
    def baby_offsets(self) -> tuple[int, ...]:
        return tuple(b * int(self.token_lanes) for b in range(int(self.baby_steps)))

    @property
    def anchor_enabled(self) -> bool:
        return int(self.baby_anchor_step) >= 2 and int(self.baby_steps) > int(self.baby_anchor_step)

    @property
    def baby_blocks(self) -> tuple[BabyBlock, ...]:
        width = int(self.baby_anchor_step) if self.anchor_enabled else int(self.baby_steps)
        return tuple(BabyBlock(start=s, width=min(width, int(self.baby_steps) - s))
                     for s in range(0, int(self.baby_steps), width))

    @property
    def baby_rotation_count(self) -> int:
        return max(0, int(self.baby_steps) - 1)

    @property
    def baby_key_offsets(self) -> tuple[int, ...]:
        width = int(self.baby_blocks[0].width)
        keys = {s * int(self.token_lanes) for s in range(1, width)}
        if len(self.baby_blocks) > 1:
            keys.add(int(self.baby_anchor_step) * int(self.token_lanes))
        return tuple(sorted(keys))

    @property
    def chunks(self) -> tuple[LinearChunk, ...]:
        bases = range(0, self.giant_steps, self.chunk_giants)
        return tuple(LinearChunk(index=i, giant_base=b, giant_count=min(self.chunk_giants, self.giant_steps - b))
                     for i, b in enumerate(bases))

    @property
    def chunk_sizes(self) -> tuple[int, ...]:
        return tuple(c.giant_count for c in self.chunks)

    @property
    def plaintext_chunks(self) -> int:
        return len(self.chunks)

    @property
    def cache_key(self) -> tuple[int, ...]:
        return (int(self.dimension), int(self.token_lanes), int(self.baby_steps), int(self.max_plaintext_rows),
                int(self.lane_shift))


def linear_rotations(*, dimension: int, token_lanes: int, slots: int | None = None,
                     include_conjugation: bool = False,
                     operator_config: LinearOperatorConfig | None = None) -> tuple[int, ...]:
    """Exact rotation-key set of one schedule (reference: config.py:338-380)."""
    cfg = LinearOperatorConfig() if operator_config is None else operator_config
    plan = cfg.plan(dimension=int(dimension), token_lanes=int(token_lanes))
    keys = set(plan.baby_key_offsets)
    most = max(c.giant_count for c in plan.chunks)
    if most > 1:
        if str(cfg.hoist_strategy).lower() == "ext_double_hoist":
            keys.update(step * plan.giant_offset for step in range(1, most))
        else:
            keys.add(plan.giant_offset)
    keys.update(c.giant_base * plan.giant_offset for c in plan.chunks if c.giant_base)
    keys.update(plan.fold_offsets)
    keys.update(plan.lane_expand_offsets)
    if include_conjugation:
        if slots is None:
            raise ValueError("slots are required when conjugation is requested.")
        keys.add(4 * int(slots) - 1)
    return tuple(sorted(int(v) for v in keys if int(v)))


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


def pack_chunk(ctx: F.Context, weight: torch.Tensor, plan: LinearPlan, chunk: LinearChunk, slots: int) -> torch.Tensor:
    """Diagonal rows of ``chunk`` as complex128 [rows][slots] (reference: weight.py:122-154)."""
    rows = int(chunk.giant_count) * int(plan.baby_steps)
    out = torch.empty((rows, slots), dtype=torch.complex128, device=ctx.device)
    w = weight
    cplx = bool(w.is_complex())
    src = torch.view_as_real(w) if cplx else w
    _lib.call("holmes_pack_diagonals", src.data_ptr(), int(cplx), int(plan.dimension), int(plan.token_lanes),
              int(plan.baby_steps), int(chunk.giant_base), int(chunk.giant_count), int(plan.lane_shift), int(slots),
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

    def prepare(self, operator_config: LinearOperatorConfig) -> float:
        if self._closed:
            raise RuntimeError("linear weight is closed.")
        del operator_config
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

    def _bundle(self, plan: LinearPlan, chunk: LinearChunk, operator_config: LinearOperatorConfig) -> F.ConstantBundle:
        key = (*plan.cache_key, int(chunk.index), str(operator_config.constant_cache_mode))
        bundle = self._bundles.get(key)
        if bundle is None:
            self.prepare(operator_config)
            ctx = self.crypto_context.context

            def packer(source, slots, context, plan=plan, chunk=chunk):
                del context
                return pack_chunk(ctx, source, plan, chunk, slots)

            bundle = F.ConstantBundle(vectors={chunk.name: F.UnpackedRaw(self._device_source, packer)},
                                      cache_mode=str(operator_config.constant_cache_mode))
            if str(operator_config.constant_cache_mode) != "none":
                self._bundles[key] = bundle
        return bundle

    def plaintext(self, plan: LinearPlan, chunk: LinearChunk, *, level: int,
                  operator_config: LinearOperatorConfig) -> F.Plaintext:
        if self._closed:
            raise RuntimeError("linear weight is closed.")
        if int(plan.dimension) != self.dimension:
            raise ValueError(f"linear plan dimension={plan.dimension} does not match weight "
                             f"dimension={self.dimension}.")
        ctx = self.crypto_context.context
        cur = int(ctx.L) - int(level)
        bundle = self._bundle(plan, chunk, operator_config)
        if self._upload_event is not None:
            torch.cuda.current_stream(ctx.device).wait_event(self._upload_event)
        return bundle.plaintext(chunk.name, state=F.CipherState(cur, 1, ctx.scale_at(cur)),
                                slots=int(self.crypto_context.max_slots), context=ctx,
                                is_ext=str(operator_config.hoist_strategy).lower() != "normal", cache=True)

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
            raise RuntimeError("cannot enter a closed linear weight.")
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

    def __init__(self, *, crypto_context, token_lanes: int, config: LinearOperatorConfig | None = None,
                 baby_shard=None) -> None:
        """``baby_shard = (rank, world, group)`` splits the baby key switches over the ranks of ``group`` (each
        rank holding the same inputs) and all-gathers the basis; None builds it locally."""
        self.crypto_context = crypto_context
        self.baby_shard = None if baby_shard is None else (int(baby_shard[0]), int(baby_shard[1]), baby_shard[2])
        self.token_lanes = int(token_lanes)
        if self.token_lanes <= 0:
            raise ValueError("token_lanes must be positive.")
        self.config = LinearOperatorConfig() if config is None else config
        self._baby_cache: dict = {}
        self._baby_hits = 0
        self._baby_misses = 0
        self._closed = False

    @property
    def closed(self) -> bool:
        return self._closed

    def plan(self, dimension: int) -> LinearPlan:
        return self.config.plan(dimension=int(dimension), token_lanes=int(self.token_lanes))

    # -- baby basis ----------------------------------------------------------------------------------------
    def _baby_key(self, inputs, plan: LinearPlan):
        return (tuple(id(c) for c in inputs), plan.cache_key + (int(plan.baby_anchor_step),))

    def _lookup_babies(self, inputs, plan: LinearPlan, level: int):
        key = self._baby_key(inputs, plan)
        entry = self._baby_cache.get(key)
        if entry is not None and all(a is b for a, b in zip(entry.sources, inputs)) and entry.level == level:
            self._baby_hits += len(inputs)
            return entry
        if entry is not None:
            del self._baby_cache[key]
        self._baby_misses += len(inputs)
        return None

    def _build_babies(self, inputs, plan: LinearPlan, level: int) -> _Babies:
        """All B baby rotations of every input.  With a baby shard (rank, world, group) set, this rank key-switches
        only its contiguous range of babies and an all-gather over the group fills in the rest: every rank then
        holds the whole basis at 1 / world of the key switches."""
        ctx = self.crypto_context.context
        cur = int(inputs[0].state.cur_limbs)
        n_in = len(inputs)
        B = int(plan.baby_steps)
        ext = str(self.config.hoist_strategy).lower() != "normal"
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
                pm = torch.tensor(ctx.p_mod_q(cur), dtype=torch.uint64, device=ctx.device)
                for c, src in ((0, c0), (1, c1)):
                    storage[0, c, :, cur:].zero_()
                    _lib.call("holmes_mul_const", ctx.handle, src.data_ptr(), pm.data_ptr(), storage[0, c].data_ptr(),
                              n_in, cur, F._item_stride(src), F._item_stride(storage[0, c]), F._stream())
            else:
                storage[0, 0].copy_(c0)
                storage[0, 1].copy_(c1)
        if max(lo, 1) < hi:
            digits, dig_item = F._modup(ctx, c1, cur, n_in)
            for b in range(max(lo, 1), hi):
                g = ctx.galois(plan.baby_offsets[b])
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
        if bool(self.config.reuse_baby_rotations):
            self._baby_cache[self._baby_key(inputs, plan)] = entry
        return entry

    def prepare_baby_rotations(self, input_ciphers, *, dimension: int) -> dict:
        if self._closed:
            raise RuntimeError("linear operator is closed.")
        inputs = tuple(input_ciphers)
        profile = {"baby_precompute": 0.0, "baby_precompute_enqueue": 0.0, "baby_cache_hits": 0.0,
                   "baby_cache_misses": 0.0}
        if not inputs or not bool(self.config.reuse_baby_rotations):
            return profile
        plan = self.plan(int(dimension))
        levels = {int(self.crypto_context.level_for_cipher(c)) for c in inputs}
        if len(levels) != 1:
            raise ValueError("linear inputs must enter at one common level.")
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
        if self._closed:
            raise RuntimeError("linear operator is closed.")
        strategy = str(self.config.hoist_strategy).lower()
        if strategy not in _HOIST_STRATEGIES:
            raise ValueError(f"unknown hoist_strategy {strategy!r}")
        ext = strategy != "normal"
        double = strategy == "ext_double_hoist"
        inputs = tuple(input_ciphers)
        if not inputs:
            return (), dict(_EMPTY_PROFILE)
        if weight.closed:
            raise RuntimeError("cannot apply a closed linear weight.")
        if weight.crypto_context is not self.crypto_context:
            raise ValueError("linear operator and weight must share one context.")
        if len(inputs) > 32:
            raise ValueError("at most 32 inputs per apply (split the batch)")
        plan = self.plan(weight.dimension)
        if chunk_indices is None:
            chunks = plan.chunks
        else:
            wanted = tuple(int(i) for i in chunk_indices)
            if not wanted:
                raise ValueError("chunk_indices must select at least one chunk.")
            if len(set(wanted)) != len(wanted):
                raise ValueError("chunk_indices must not repeat a chunk.")
            for i in wanted:
                if i < 0 or i >= len(plan.chunks):
                    raise IndexError(f"chunk index {i} outside [0, {len(plan.chunks)})")
            chunks = tuple(plan.chunks[i] for i in wanted)
        levels = {int(self.crypto_context.level_for_cipher(c)) for c in inputs}
        if len(levels) != 1:
            raise ValueError("linear inputs must enter at one common level.")
        level = levels.pop()
        if any(c.batch_size != 1 or c.is_ext for c in inputs):
            raise ValueError("linear inputs must be single non-extended ciphertexts.")
        ctx = self.crypto_context.context
        stage = dict(_EMPTY_PROFILE)
        stage["weight_upload"] = float(weight.prepare(self.config))
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
        ev[0].record()
        babies = self._lookup_babies(inputs, plan, level) if bool(self.config.reuse_baby_rotations) else None
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
            pts = weight.plaintext(plan, chunk, level=level, operator_config=self.config)
            e1.record()
            pt_state = pts.state
            babies.ready()
            res = F.bsgs_partial_sums(ctx, blocks, pts, int(chunk.giant_count))
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
                g0, g1 = F.giant_double_hoist(ctx, res, int(plan.giant_offset))
            else:        # normal / ext_normal: the Horner chain
                g0, g1 = F.giant_horner(ctx, res, int(plan.giant_offset))
            shift = int(chunk.giant_base) * int(plan.giant_offset)
            if acc0 is None:
                if shift:
                    n0, n1 = torch.empty_like(g0), torch.empty_like(g1)
                    F.rotate_batch(ctx, g0, g1, cur, shift, n0, n1)
                    acc0, acc1 = n0, n1
                else:
                    acc0, acc1 = g0.clone(), g1.clone()
            else:
                n0, n1 = torch.empty_like(acc0), torch.empty_like(acc1)
                if shift:
                    F.rotate_batch(ctx, g0, g1, cur, shift, n0, n1, post0=acc0, post1=acc1)
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
            raise RuntimeError("cannot enter a closed linear operator.")
        return self

    def __exit__(self, *exc) -> None:
        self.close()
