"""Device-payload transport between ranks over torch.distributed: ciphertext packets move GPU to GPU through NCCL
(NVLink / NVSwitch), never through host staging.

Mirrors the reference's ``Transport`` protocol (``llama3fhe/parallel/prefill/transport.py:449-611``: ``rank``,
``stats``, ``device_payloads``, ``world_size``, ``peers``, ``send``, ``recv``, ``all_gather``, ``all_to_all``, the
split-phase ``*_isend`` + ``wait()``, ``barrier``, ``gather_to``, ``close``; same argument meaning and errors:
``ValueError`` for a send to self or a wrong payload count, ``IndexError`` for a rank outside the world,
``TimeoutError`` when a receive outlives its limit, ``RuntimeError`` when a collective round starts while an
earlier split-phase round is still unwaited).  It is the backend the reference's host and pinned staging
transports would be replaced by (``build_transport(kind="nccl")``); payloads are whatever the stations send,
normally ``wire.CipherPacket`` with device components (``pack_cipher(host=False)``).

Wire format, per message: a payload is pickled with every tensor (and every NumPy array above 64 KiB) taken out by
``persistent_id``; the message is ``[skeleton length]`` (int64), the skeleton (pickle of tag, byte sizes and the
body), then each tensor as raw bytes, all on the process group's device (CUDA for NCCL).  Tensors travel as
``uint8`` views, so any dtype (``uint64`` residues, ``complex128``) moves bit for bit.

Ordering.  Point-to-point messages and collective rounds use two process groups created together in the
constructor (every rank constructs the transport at the same point), so a pending point-to-point message can never
be mistaken for a collective's.  ``recv(src, tag)`` takes the next message from ``src``; one with another tag is
received whole and kept for the ``recv`` that asks for it.  Collectives post all their sends and receives of a phase
as one NCCL group (``batch_isend_irecv``), so symmetric exchanges cannot deadlock.  ``send`` posts its NCCL sends at
once and returns; as NCCL point-to-point sends complete only against the peer's receive, two ranks that send each
other large payloads before receiving must use ``all_to_all``.
"""
from __future__ import annotations

import datetime
import io
import os
import pickle
import time
from collections import defaultdict, deque
from dataclasses import dataclass, field
from typing import Any, Sequence

import numpy as np
import torch
import torch.distributed as dist

__all__ = ["TransportStats", "NcclTransport", "NcclCollectiveHandle", "build_transport", "TRANSPORT_BACKENDS",
           "CipherPacket", "pack_cipher", "unpack_cipher"]

TRANSPORT_BACKENDS: tuple[str, ...] = ("nccl",)
_INLINE_ARRAY_BYTES = 64 << 10
_POLL_SECONDS = 1e-4


@dataclass
class TransportStats:
    """Counters with the reference's names (``transport.py:449-467``)."""

    messages_sent: int = 0
    messages_received: int = 0
    bytes_sent: int = 0
    bytes_received: int = 0
    send_seconds: float = 0.0
    recv_wait_seconds: float = 0.0
    collectives: int = 0

    def to_dict(self) -> dict:
        return {k: getattr(self, k) for k in ("messages_sent", "messages_received", "bytes_sent", "bytes_received",
                                                "send_seconds", "recv_wait_seconds", "collectives")}


# ----------------------------------------------------------------------------------------------------- encoding


class _Pickler(pickle.Pickler):
    def __init__(self, f, out: list) -> None:
        super().__init__(f, protocol=pickle.HIGHEST_PROTOCOL)
        self.out = out

    def persistent_id(self, obj):
        if torch.is_tensor(obj):
            self.out.append(obj.detach())
            return ("t", len(self.out) - 1, str(obj.dtype).removeprefix("torch."), tuple(obj.shape), obj.device.type)
        if isinstance(obj, np.ndarray) and obj.dtype != object and obj.nbytes > _INLINE_ARRAY_BYTES:
            self.out.append(torch.from_numpy(np.ascontiguousarray(obj)))
            return ("a", len(self.out) - 1, obj.dtype.str, tuple(obj.shape), "cpu")
        return None


class _Unpickler(pickle.Unpickler):
    def __init__(self, f, tensors: list) -> None:
        super().__init__(f)
        self.tensors = tensors

    def persistent_load(self, pid):
        kind, index, dtype, shape, where = pid
        raw = self.tensors[index]
        if kind == "a":
            return raw.cpu().numpy().view(np.dtype(dtype)).reshape(shape).copy()
        t = raw.view(getattr(torch, dtype)).reshape(shape)
        return t.cpu() if where == "cpu" and t.device.type != "cpu" else t


def _as_bytes(t: torch.Tensor, device: torch.device) -> torch.Tensor:
    b = t.contiguous().reshape(-1).view(torch.uint8)
    return b if b.device == device else b.to(device, non_blocking=True)


def _encode(tag: str, payload: Any, device: torch.device) -> tuple[torch.Tensor, list, int]:
    """(skeleton bytes on ``device``, payload byte tensors on ``device``, payload bytes)."""
    found: list = []
    body = io.BytesIO()
    _Pickler(body, found).dump(payload)
    parts = [_as_bytes(t, device) for t in found]
    sizes = [int(p.numel()) for p in parts]
    skeleton = pickle.dumps((str(tag), sizes, body.getvalue()), protocol=pickle.HIGHEST_PROTOCOL)
    sk = torch.frombuffer(bytearray(skeleton), dtype=torch.uint8).to(device)
    return sk, parts, sum(sizes)


def _decode(skeleton: torch.Tensor) -> tuple[str, list, bytes]:
    return pickle.loads(skeleton.cpu().numpy().tobytes())


def _finish(body: bytes, parts: list) -> Any:
    return _Unpickler(io.BytesIO(body), parts).load()


# ----------------------------------------------------------------------------------------------------- transport


@dataclass
class NcclCollectiveHandle:
    """The receive half of a split-phase collective; ``wait()`` returns the payloads indexed by rank."""

    transport: "NcclTransport"
    sequence: int
    finish: Any
    _result: Any = None
    _done: bool = False

    def wait(self) -> list:
        if not self._done:
            self._result = self.transport._collective_wait(self)
            self._done = True
        return self._result

    @property
    def done(self) -> bool:
        return bool(self._done)


@dataclass
class NcclTransport:
    """Point-to-point plus the collectives for one rank, over the default (or a given) process group."""

    rank: int | None = None
    group: Any = None
    #: seconds a receive may wait before ``TimeoutError`` (None = forever)
    default_timeout: float | None = 900.0
    device: Any = None
    stats: TransportStats = field(default_factory=TransportStats)
    #: components may stay on the device: they travel GPU to GPU
    device_payloads: bool = True

    def __post_init__(self) -> None:
        if not dist.is_initialized():
            raise RuntimeError("NcclTransport needs an initialised torch.distributed process group")
        world = dist.get_world_size(self.group)
        me = dist.get_rank(self.group)
        if self.rank is None:
            self.rank = me
        self.rank = int(self.rank)
        if self.rank < 0 or self.rank >= world:
            raise IndexError(f"rank {self.rank} outside world of size {world}")
        if self.rank != me:
            raise ValueError(f"rank {self.rank} is not this process's rank {me}")
        self._world = int(world)
        ranks = list(range(self._world)) if self.group is None else dist.get_process_group_ranks(self.group)
        self._globals = ranks
        self._p2p = dist.new_group(ranks)
        self._coll = dist.new_group(ranks)
        backend = dist.get_backend(self._p2p)
        if self.device is None:
            self.device = (torch.device("cuda", torch.cuda.current_device()) if backend == "nccl"
                           else torch.device("cpu"))
        self.device = torch.device(self.device)
        self._stash: dict = defaultdict(deque)
        self._inflight: list = []
        self._sequence = 0
        self._gather_sequence = 0
        self._open_round = None
        self._broken = False
        self._closed = False

    def __enter__(self) -> "NcclTransport":
        return self

    def __exit__(self, *_exc) -> None:
        self.close()

    @property
    def world_size(self) -> int:
        return self._world

    @property
    def peers(self) -> tuple:
        return tuple(r for r in range(self._world) if r != self.rank)

    # -------------------------------------------------------------------------------------------- plumbing
    def _check(self) -> None:
        if self._closed:
            raise RuntimeError("transport is closed")
        if self._broken:
            raise RuntimeError("transport is unusable after a receive timed out with its receive still posted")

    def _g(self, r: int) -> int:
        return int(self._globals[r])

    def _reap(self) -> None:
        """Drop finished sends.  gloo reports a send finished only through ``wait``: past 64 pending sends the
        oldest are waited for, which bounds the buffers kept alive."""
        self._inflight = [(w, keep) for w, keep in self._inflight if not w.is_completed()]
        if self.device.type != "cuda" and len(self._inflight) > 64:
            for w, _ in self._inflight[:-64]:
                w.wait()
            self._inflight = self._inflight[-64:]

    def _wait(self, works: list, deadline: float | None, what: str) -> None:
        """Wait for ``works`` until ``deadline``: NCCL works are polled (their completion is a CUDA event); gloo's
        point-to-point works report completion only through ``wait``, which takes the remaining time."""
        for w in works:
            if self.device.type == "cuda":
                while not w.is_completed():
                    if deadline is not None and time.perf_counter() > deadline:
                        self._broken = True
                        raise TimeoutError(f"rank {self.rank}: {what} did not arrive in time")
                    time.sleep(_POLL_SECONDS)
                w.wait()
            elif deadline is None:
                w.wait()
            else:
                left = max(deadline - time.perf_counter(), 1e-3)
                try:
                    w.wait(timeout=datetime.timedelta(seconds=left))
                except RuntimeError as exc:
                    if "imed out" not in str(exc):
                        raise
                    self._broken = True
                    raise TimeoutError(f"rank {self.rank}: {what} did not arrive in time") from exc

    def _deadline(self, timeout: float | None) -> float | None:
        limit = self.default_timeout if timeout is None else timeout
        return None if limit is None else time.perf_counter() + float(limit)

    # -------------------------------------------------------------------------------------------- p2p
    def send(self, dst: int, tag: str, payload: Any) -> None:
        self._check()
        dst = int(dst)
        if dst < 0 or dst >= self._world:
            raise IndexError(f"destination {dst} outside world of size {self._world}")
        if dst == self.rank:
            raise ValueError("use local hand-off instead of sending to self")
        started = time.perf_counter()
        sk, parts, nbytes = _encode(tag, payload, self.device)
        head = torch.tensor([sk.numel()], dtype=torch.int64).to(self.device)
        works = [dist.isend(head, self._g(dst), group=self._p2p), dist.isend(sk, self._g(dst), group=self._p2p)]
        works += [dist.isend(p, self._g(dst), group=self._p2p) for p in parts if p.numel()]
        self._inflight += [(w, (head, sk, parts)) for w in works]
        self._reap()
        self.stats.messages_sent += 1
        self.stats.bytes_sent += nbytes
        self.stats.send_seconds += time.perf_counter() - started

    def _recv_next(self, src: int, deadline: float | None) -> tuple:
        head = torch.empty(1, dtype=torch.int64, device=self.device)
        self._wait([dist.irecv(head, self._g(src), group=self._p2p)], deadline, f"a message from {src}")
        sk = torch.empty(int(head.item()), dtype=torch.uint8, device=self.device)
        self._wait([dist.irecv(sk, self._g(src), group=self._p2p)], deadline, f"a message body from {src}")
        tag, sizes, body = _decode(sk)
        parts = [torch.empty(n, dtype=torch.uint8, device=self.device) for n in sizes]
        self._wait([dist.irecv(p, self._g(src), group=self._p2p) for p in parts if p.numel()], deadline,
                   f"payload tensors from {src}")
        return tag, body, parts, sum(sizes)

    def recv(self, src: int, tag: str, *, timeout: float | None = None) -> Any:
        self._check()
        src = int(src)
        if src < 0 or src >= self._world or src == self.rank:
            raise IndexError(f"source {src} is not a peer of rank {self.rank}")
        key = (src, str(tag))
        if self._stash[key]:
            body, parts, nbytes = self._stash[key].popleft()
            return self._accept(body, parts, nbytes)
        deadline = self._deadline(timeout)
        started = time.perf_counter()
        while True:
            got, body, parts, nbytes = self._recv_next(src, deadline)
            if got == str(tag):
                self.stats.recv_wait_seconds += time.perf_counter() - started
                return self._accept(body, parts, nbytes)
            self._stash[(src, got)].append((body, parts, nbytes))

    def _accept(self, body: bytes, parts: list, nbytes: int) -> Any:
        self.stats.messages_received += 1
        self.stats.bytes_received += nbytes
        return _finish(body, parts)

    # -------------------------------------------------------------------------------------------- collectives
    def _begin_round(self) -> int:
        if self._open_round is not None:
            raise RuntimeError(f"rank {self.rank}: collective round #{self._open_round} is still in flight; wait() "
                               "for it before issuing the next collective")
        self._sequence += 1
        self.stats.collectives += 1
        return self._sequence

    def _exchange(self, tag: str, payloads_by_dst: Sequence[Any], deadline: float | None):
        """Phase 1 (lengths) and phase 2 (skeletons) now; phase 3 (tensors) posted, waited for in ``finish``."""
        if not self.peers:
            return lambda own: [own]
        started = time.perf_counter()
        enc = {d: _encode(tag, payloads_by_dst[d], self.device) for d in self.peers}
        heads_out = {d: torch.tensor([enc[d][0].numel()], dtype=torch.int64).to(self.device) for d in self.peers}
        heads_in = {s: torch.empty(1, dtype=torch.int64, device=self.device) for s in self.peers}
        ops = [dist.P2POp(dist.isend, heads_out[d], self._g(d), self._coll) for d in self.peers]
        ops += [dist.P2POp(dist.irecv, heads_in[s], self._g(s), self._coll) for s in self.peers]
        self._wait(dist.batch_isend_irecv(ops), deadline, "collective lengths")
        sk_in = {s: torch.empty(int(heads_in[s].item()), dtype=torch.uint8, device=self.device) for s in self.peers}
        ops = [dist.P2POp(dist.isend, enc[d][0], self._g(d), self._coll) for d in self.peers]
        ops += [dist.P2POp(dist.irecv, sk_in[s], self._g(s), self._coll) for s in self.peers]
        self._wait(dist.batch_isend_irecv(ops), deadline, "collective skeletons")
        meta = {s: _decode(sk_in[s]) for s in self.peers}
        for s in self.peers:
            if meta[s][0] != str(tag):
                raise RuntimeError(f"rank {self.rank}: collective {tag!r} met {meta[s][0]!r} from rank {s}: the ranks "
                                   "issued their collectives in different orders")
        parts_in = {s: [torch.empty(n, dtype=torch.uint8, device=self.device) for n in meta[s][1]] for s in self.peers}
        ops = [dist.P2POp(dist.isend, p, self._g(d), self._coll) for d in self.peers for p in enc[d][1] if p.numel()]
        ops += [dist.P2POp(dist.irecv, p, self._g(s), self._coll) for s in self.peers for p in parts_in[s]
                if p.numel()]
        works = dist.batch_isend_irecv(ops) if ops else []
        for d in self.peers:
            self.stats.bytes_sent += enc[d][2]
        self.stats.send_seconds += time.perf_counter() - started
        keep = [enc, heads_out]   # the send buffers live until the payload phase completes

        def finish(own) -> list:
            t0 = time.perf_counter()
            self._wait(works, deadline, "collective payloads")
            keep.clear()
            self.stats.recv_wait_seconds += time.perf_counter() - t0
            out: list = [None] * self._world
            out[self.rank] = own
            for s in self.peers:
                self.stats.bytes_received += sum(meta[s][1])
                out[s] = _finish(meta[s][2], parts_in[s])
            return out

        return finish

    def all_to_all_isend(self, tag: str, payloads_by_dst: Sequence[Any], *,
                         timeout: float | None = None) -> NcclCollectiveHandle:
        self._check()
        if len(payloads_by_dst) != self._world:
            raise ValueError("all_to_all needs exactly one payload per rank")
        seq = self._begin_round()
        fin = self._exchange(f"{tag}#{seq}", payloads_by_dst, self._deadline(timeout))
        own = payloads_by_dst[self.rank]
        self._open_round = seq
        return NcclCollectiveHandle(self, seq, lambda: fin(own))

    def all_gather_isend(self, tag: str, payload: Any, *, timeout: float | None = None) -> NcclCollectiveHandle:
        return self.all_to_all_isend(tag, [payload] * self._world, timeout=timeout)

    def _collective_wait(self, handle: NcclCollectiveHandle) -> list:
        if self._open_round != handle.sequence:
            raise RuntimeError(f"rank {self.rank}: round #{handle.sequence} is not the open collective round")
        try:
            return handle.finish()
        finally:
            self._open_round = None

    def all_to_all(self, tag: str, payloads_by_dst: Sequence[Any], *, timeout: float | None = None) -> list:
        return self.all_to_all_isend(tag, payloads_by_dst, timeout=timeout).wait()

    def all_gather(self, tag: str, payload: Any, *, timeout: float | None = None) -> list:
        return self.all_gather_isend(tag, payload, timeout=timeout).wait()

    def barrier(self, tag: str = "barrier", *, timeout: float | None = None) -> None:
        self.all_gather(tag, None, timeout=timeout)

    def gather_to(self, root: int, tag: str, payload: Any, *, timeout: float | None = None):
        """One payload per rank on ``root`` (the others return None); point-to-point, no collective round."""
        root = int(root)
        if root < 0 or root >= self._world:
            raise IndexError(f"root {root} outside world of size {self._world}")
        self._gather_sequence += 1
        self.stats.collectives += 1
        gtag = f"{tag}#g{self._gather_sequence}"
        if self.rank != root:
            self.send(root, gtag, payload)
            return None
        out: list = [None] * self._world
        out[self.rank] = payload
        for s in self.peers:
            out[s] = self.recv(s, gtag, timeout=timeout)
        return out

    def close(self) -> None:
        if self._closed:
            return
        if not self._broken:
            for w, _ in self._inflight:
                w.wait()
        self._inflight = []
        self._stash.clear()
        self._closed = True


def build_transport(rank: int | None = None, endpoints=None, *, kind: str | None = None, **options: Any):
    """The device-payload backend (``kind="nccl"``, or ``T2_TRANSPORT=nccl``): the reference's factory
    (``transport.py:538-566``) gains this name; ``endpoints`` (the host backends' queues) is not used."""
    del endpoints
    name = str(kind if kind is not None else os.environ.get("T2_TRANSPORT", "nccl")).lower()
    if name != "nccl":
        raise ValueError(f"unknown transport backend {name!r}; choose from {TRANSPORT_BACKENDS}")
    return NcclTransport(rank, **options)


# ----------------------------------------------------------------------------------------------------- packets


@dataclass
class CipherPacket:
    """A ciphertext for the wire (``llama3fhe/parallel/wire.py:282-303``): its components by reference plus the
    state and the encoding contract."""

    components: tuple
    cur_limbs: int
    scale_degree: int
    scaling_factor: float | None
    slots: int
    batch_size: int
    is_ext: bool
    tag: str = ""

    @property
    def nbytes(self) -> int:
        return int(sum(int(c.numel()) * c.element_size() for c in self.components))


def pack_cipher(cipher, *, tag: str = "") -> CipherPacket:
    """The device components by reference (``pack_cipher(host=False)``); the cipher is not consumed."""
    s = cipher.state
    return CipherPacket(tuple(cipher.cv), int(s.cur_limbs), int(s.scale_degree),
                        None if s.scaling_factor is None else float(s.scaling_factor), int(cipher.slots),
                        int(cipher.batch_size), bool(cipher.is_ext), str(tag))


def unpack_cipher(packet: CipherPacket, context):
    """A ``fhe.Cipher`` on ``context``'s device from a received packet (components moved there if needed)."""
    from . import fhe

    cv = [c.to(context.device) if c.device != torch.device(context.device) else c for c in packet.components]
    state = fhe.CipherState(packet.cur_limbs, packet.scale_degree, packet.scaling_factor)
    return fhe.Cipher(cv, state, packet.slots, packet.is_ext, packet.batch_size, context)
