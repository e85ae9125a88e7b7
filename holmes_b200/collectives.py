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
