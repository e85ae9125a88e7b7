"""Multi-GPU exchange for the linear path: one process per GPU, ``torch.distributed`` for the plumbing.

The reference moves ciphertexts between ranks through host shared memory and adds partial sums only on the
owning rank, with the FHE add (``parallel/prefill/transport.py:36-47``, ``parallel/wire.py:1-20``,
``parallel/decode/decode_collectives.py:59-195``).  Here:

* ``token_shard`` / ``chunk_shard`` partition the work the way the reference's ownership does
  (``parallel/prefill/ownership.py:1-44``: adjacent ciphertexts per rank; ``parallel/decode/decode_ownership.py``:
  BSGS chunks per rank);
* ``exchange_partials`` sends every rank's partial sums of the items another rank owns to that owner with one
  ``all_to_all`` of raw uint64 limbs (bit copies are a valid transport for residues);
* ``modular_reduce_scatter`` then adds the received partials modulo q on the owner with ``holmes_modsum`` --
  NCCL's own sum is not modular, so the collective moves data and the engine adds.

``exchange_partials`` is plain ``torch.distributed`` and runs on any backend (the CPU tests use gloo);
``modular_reduce_scatter`` needs the CUDA engine.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from . import _lib


def token_shard(n_items: int, world: int, rank: int) -> range:
    """Adjacent items per rank: rank r owns [r n / W, (r + 1) n / W)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    return range(rank * n_items // world, (rank + 1) * n_items // world)


def chunk_shard(n_chunks: int, world: int, rank: int) -> tuple[int, ...]:
    """BSGS chunks per rank, contiguous, as even as possible."""
    return tuple(token_shard(n_chunks, world, rank))


def owner_of(item: int, n_items: int, world: int) -> int:
    for r in range(world):
        if item in token_shard(n_items, world, r):
            return r
    raise IndexError(item)


def exchange_partials(partials: torch.Tensor, world: int, group=None) -> torch.Tensor:
    """``partials`` [n_items][...] on every rank -> [world][n_owned][...]: the partial sums of this rank's owned
    items from every rank (rank order), via one all_to_all.  Items are token-sharded; ``n_items`` must divide
    evenly over the ranks so every rank sends and receives equal blocks."""
    n = int(partials.shape[0])
    if n % world:
        raise ValueError(f"{n} items do not split evenly over {world} ranks")
    per = n // world
    send = partials.contiguous().reshape(world, per, *partials.shape[1:])
    recv = torch.empty_like(send)
    if world == 1:
        recv.copy_(send)
        return recv
    # residues travel as their bit pattern (int64 view): backends need not support uint64
    dist.all_to_all_single(recv.reshape(-1).view(torch.int64), send.reshape(-1).view(torch.int64), group=group)
    return recv


def all_gather_rows(storage: torch.Tensor, lo: int, hi: int, world: int, group=None, async_op: bool = False):
    """In-place all-gather along dim 0: this rank filled rows [lo, hi) of ``storage`` (equal contiguous ranges
    per rank, in rank order); afterwards every rank holds every row.  Residues travel as their bit pattern.
    With ``async_op`` the work handle is returned: ``storage`` may not be read before ``handle.wait()``."""
    rows = int(storage.shape[0])
    if rows % world or hi - lo != rows // world:
        raise ValueError(f"rows [{lo}, {hi}) are not this rank's equal share of {rows} over {world}")
    flat = storage.view(torch.int64).reshape(-1)
    per = flat.numel() // world
    r = lo // (hi - lo)
    if world > 1:
        return dist.all_gather_into_tensor(flat, flat[r * per:(r + 1) * per], group=group, async_op=async_op)
    return None


def modsum(ctx, buffers: torch.Tensor, limbs: int) -> torch.Tensor:
    """Sum [k][items][limbs][N] buffers modulo q limb-wise on the GPU -> [items][limbs][N]."""
    k, items = int(buffers.shape[0]), int(buffers.shape[1])
    out = torch.empty(buffers.shape[1:], dtype=torch.uint64, device=buffers.device)
    srcs = _lib.ptr_array([buffers[i].data_ptr() for i in range(k)])
    _lib.call("holmes_modsum", ctx.handle, srcs, k, out.data_ptr(), items, int(limbs), int(buffers[0].stride(0)),
              torch.cuda.current_stream().cuda_stream)
    return out


def modular_reduce_scatter(ctx, partials: torch.Tensor, world: int, group=None) -> torch.Tensor:
    """Owner-side mod-q sum of every rank's partial sums: [n_items][limbs][N] per rank -> [n_owned][limbs][N]
    on each rank (the rank's token shard of the items)."""
    recv = exchange_partials(partials, world, group)
    return modsum(ctx, recv, int(partials.shape[1]))


# ----------------------------------------------------------------------------------------------------- peer memory


class PeerReduceScatter:
    """Modular reduce-scatter of token-sharded partial sums over peer memory, one kernel per step.

    Every rank owns a ``partials`` buffer [n_items][limbs][N] that the other ranks map once at construction (CUDA IPC
    handles travel through ``group`` with ``all_gather_object``; each rank opens its peers' handles with its own device
    current).  ``reduce()`` is device-side only, on the current stream:

    1. signal "my partials of this epoch are written" (flag 0 of this rank's flag block);
    2. wait (bounded) until every rank's flag 0 reaches the epoch;
    3. sum every rank's partials of this rank's token shard modulo q into ``out`` -- plain loads from peer memory;
    4. signal "I have read your partials" into every peer's flag 2 + rank, and wait (bounded) until every peer has
       done the same in this rank's block, so the next step may overwrite ``partials``.

    A wait that runs out sets a device status word and the sum is skipped; ``check()`` (one device read) raises
    ``TimeoutError`` naming the flag.  The reference's partial reduces are host-staged sends plus an owner-side
    ``homo_add`` (``parallel/prefill/stations.py:1565-1596``, ``parallel/decode/decode_collectives.py:59-195``)."""

    FLAGS_PER_RANK = 2

    def __init__(self, ctx, n_items: int, limbs: int, world: int, rank: int, group=None,
                 timeout_s: float = 2.0, clock_hz: float = 1.965e9) -> None:
        if world < 1 or world > 16 or not 0 <= rank < world:
            raise ValueError(f"rank {rank} of world {world} (1 .. 16 ranks)")
        if n_items % world:
            raise ValueError(f"{n_items} items do not split evenly over {world} ranks")
        self.ctx, self.world, self.rank, self.group = ctx, int(world), int(rank), group
        self.n_items, self.limbs, self.per = int(n_items), int(limbs), int(n_items) // int(world)
        self.budget = int(timeout_s * clock_hz)
        self.timeout_s = float(timeout_s)
        dev = ctx.device
        self._owned: list[int] = []
        self._mapped: list[int] = []
        self.partials = self._alloc((self.n_items, self.limbs, ctx.N))
        self.flags = self._alloc((self.FLAGS_PER_RANK + self.world,))
        self.status = torch.zeros(1, dtype=torch.int32, device=dev)
        self.epoch = 0
        handles = (self._export(self.partials), self._export(self.flags))
        if self.world > 1:
            every = [None] * self.world
            dist.all_gather_object(every, handles, group=group)
        else:
            every = [handles]
        torch.cuda.synchronize(dev)
        self.peer_partials, self.peer_flags = [], []
        for r, (hp, hf) in enumerate(every):
            if r == self.rank:
                self.peer_partials.append(self.partials.data_ptr())
                self.peer_flags.append(self.flags.data_ptr())
            else:
                self.peer_partials.append(self._import(hp))
                self.peer_flags.append(self._import(hf))

    def _alloc(self, shape) -> torch.Tensor:
        """A zeroed uint64 tensor on its own cudaMalloc allocation (IPC handles name whole allocations)."""
        n = 1
        for d in shape:
            n *= int(d)
        ptr = _lib.ctypes.c_void_p()
        _lib.call("holmes_peer_alloc", n * 8, _lib.ctypes.byref(ptr))
        self._owned.append(int(ptr.value))

        class _View:
            __cuda_array_interface__ = {"shape": tuple(int(d) for d in shape), "typestr": "<u8",
                                        "data": (int(ptr.value), False), "version": 3, "strides": None}

        return torch.as_tensor(_View(), device=self.ctx.device)

    @staticmethod
    def _export(t: torch.Tensor) -> bytes:
        buf = (_lib.ctypes.c_ubyte * 64)()
        _lib.call("holmes_ipc_export", t.data_ptr(), buf)
        return bytes(buf)

    def _import(self, handle: bytes) -> int:
        ptr = _lib.ctypes.c_void_p()
        _lib.call("holmes_ipc_import", (_lib.ctypes.c_ubyte * 64).from_buffer_copy(handle), _lib.ctypes.byref(ptr))
        self._mapped.append(int(ptr.value))
        return int(ptr.value)

    def _ptrs(self, ptrs) -> "_lib.ctypes.Array":
        return _lib.ptr_array([int(p) for p in ptrs])

    def reduce(self, out: torch.Tensor | None = None) -> torch.Tensor:
        """Sum of every rank's ``partials`` rows of this rank's token shard, modulo q -> [n_items / world][limbs][N]."""
        ctx, N, L = self.ctx, self.ctx.N, self.limbs
        item = L * N
        if out is None:
            out = torch.empty((self.per, L, N), dtype=torch.uint64, device=ctx.device)
        if tuple(out.shape) != (self.per, L, N) or not out.is_contiguous():
            raise ValueError(f"out must be a contiguous [{self.per}][{L}][{N}] tensor")
        self.epoch += 1
        e, s = self.epoch, torch.cuda.current_stream().cuda_stream
        F = self.FLAGS_PER_RANK
        own = self.flags.data_ptr()
        _lib.call("holmes_peer_signal", self._ptrs([own]), 1, e, s)
        _lib.call("holmes_peer_wait", self._ptrs(self.peer_flags), self.world, e, self.budget, self.status.data_ptr(), s)
        off = self.rank * self.per * item * 8
        srcs = self._ptrs([p + off for p in self.peer_partials])
        _lib.call("holmes_modreduce_scatter", ctx.handle, srcs, self.world, out.data_ptr(), self.per, L, item,
                  self.status.data_ptr(), s)
        done = [p + 8 * (F + self.rank) for p in self.peer_flags]
        _lib.call("holmes_peer_signal", self._ptrs(done), self.world, e, s)
        mine = [own + 8 * (F + r) for r in range(self.world)]
        _lib.call("holmes_peer_wait", self._ptrs(mine), self.world, e, self.budget, self.status.data_ptr(), s)
        return out

    def check(self) -> None:
        """Raise if a wait of an earlier step ran out (one device read)."""
        st = int(self.status.item())
        if st:
            self.status.zero_()
            raise TimeoutError(f"peer reduce-scatter: a flag wait of rank {self.rank} ran out after "
                               f"{self.timeout_s:.1f} s (flag {st - 1}); a peer did not reach epoch {self.epoch}")

    def close(self) -> None:
        """Unmap the peers' buffers, then (after every rank has unmapped this one's: a barrier over ``group``) free
        this rank's.  Collective: every rank calls it once, after its last step."""
        torch.cuda.synchronize(self.ctx.device)
        for p in self._mapped:
            _lib.call("holmes_ipc_close", p)
        self._mapped.clear()
        self.partials = self.flags = None
        if self.world > 1:
            dist.barrier(group=self.group)
        for p in self._owned:
            _lib.call("holmes_peer_free", _lib.ctypes.c_void_p(p))
        self._owned.clear()
        for p in self._owned:
            _lib.call("holmes_peer_free", p)
        self._owned.clear()
