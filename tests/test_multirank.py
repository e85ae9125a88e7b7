"""N > 1 host logic on CPU: world-size-2 gloo process groups exchange partial sums the way the multi-GPU path
does (raw uint64 limbs, owner-side modular sum).  The modular sum itself is the engine's GPU kernel; here the
oracle's CPU add stands in as the checker, so the test covers the sharding and the exchange protocol."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from holmes_b200 import collectives as C


def _port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_shards_partition_work():
    for n, w in ((16, 1), (16, 2), (16, 4), (16, 8), (8, 8), (7, 3)):
        seen = []
        for r in range(w):
            seen += list(C.token_shard(n, w, r))
        assert seen == list(range(n))
        assert all(C.owner_of(i, n, w) == next(r for r in range(w) if i in C.token_shard(n, w, r)) for i in range(n))
    assert [C.chunk_shard(8, 4, r) for r in range(4)] == [(0, 1), (2, 3), (4, 5), (6, 7)]
    with pytest.raises(ValueError):
        C.token_shard(4, 2, 2)


def _worker(rank, world, port, q, out_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(100 + rank)
        items, limbs, n = 4, 3, 16
        partials = np.stack([rng.integers(0, q[l], (items, n), dtype=np.uint64) for l in range(limbs)], axis=1)
        np.save(os.path.join(out_dir, f"p{rank}.npy"), partials)
        recv = C.exchange_partials(torch.from_numpy(partials), world)
        np.save(os.path.join(out_dir, f"r{rank}.npy"), recv.numpy())
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_exchange_partials_gloo_world2(tmp_path):
    from oracle.oracle import lib, _p

    q = [(1 << 40) - 87, (1 << 40) - 167, (1 << 40) - 195]
    world = 2
    mp.spawn(_worker, args=(world, _port(), q, str(tmp_path)), nprocs=world, join=True)
    parts = [np.load(tmp_path / f"p{r}.npy") for r in range(world)]
    for r in range(world):
        recv = np.load(tmp_path / f"r{r}.npy")        # [world][owned][limbs][N]
        owned = list(C.token_shard(4, world, r))
        for k in range(world):
            np.testing.assert_array_equal(recv[k], parts[k][owned])
        # owner-side modular sum (the engine does this with holmes_modsum on the GPU)
        total = recv[0].copy()
        for k in range(1, world):
            for li in range(3):
                for i in range(len(owned)):
                    a = np.ascontiguousarray(total[i, li])
                    b = np.ascontiguousarray(recv[k][i, li])
                    lib().orc_add(_p(a), _p(b), _p(a), a.size, q[li])
                    total[i, li] = a
        want = sum(p[owned].astype(object) for p in parts)
        for li in range(3):
            assert np.array_equal(total[:, li].astype(object), want[:, li] % q[li])


def _gather_worker(rank, world, port, out_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rows, per_row = 8, 5
        storage = torch.zeros((rows, per_row), dtype=torch.uint64)
        lo, hi = rank * rows // world, (rank + 1) * rows // world
        for r in range(lo, hi):  # this rank's babies: row r holds 1000 r + k, with the top bit set in some words
            storage[r] = torch.tensor([(1000 * r + k) | ((k % 2) << 63) for k in range(per_row)], dtype=torch.uint64)
        C.all_gather_rows(storage, lo, hi, world)
        np.save(os.path.join(out_dir, f"g{rank}.npy"), storage.numpy())
    finally:
        dist.destroy_process_group()


def test_all_gather_rows_gloo_world2(tmp_path):
    """The sharded baby-basis build: each rank fills its contiguous rows, the in-place all-gather fills the rest
    bit for bit (uint64 through int64 views)."""
    world = 2
    mp.spawn(_gather_worker, args=(world, _port(), str(tmp_path)), nprocs=world, join=True)
    want = np.array([[(1000 * r + k) | ((k % 2) << 63) for k in range(5)] for r in range(8)], dtype=np.uint64)
    for r in range(world):
        np.testing.assert_array_equal(np.load(tmp_path / f"g{r}.npy"), want)
