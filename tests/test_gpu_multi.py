"""Two GPUs over NCCL: the modular reduce-scatter of partial sums (raw limbs over all_to_all, owner-side mod-q sum
with holmes_modsum, and the peer-memory PeerReduceScatter) equals the exact sum.  Skipped with fewer than two GPUs."""
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, out_dir):
    from datetime import timedelta

    import torch.distributed as dist

    from holmes_b200 import collectives as C
    from tests.gpu_helpers import make_pair

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        _, _, ctx = make_pair(log_n=12, limbs=4, dnum=2, dcrt=45, first=55, special=55)
        rng = np.random.default_rng(7 + rank)
        items, limbs, n = 4, 4, ctx.N
        parts = np.stack([rng.integers(0, ctx.moduli[l], (items, n), dtype=np.uint64) for l in range(limbs)], axis=1)
        np.save(os.path.join(out_dir, f"p{rank}.npy"), parts)
        got = C.modular_reduce_scatter(ctx, torch.from_numpy(parts).cuda(), world)
        torch.cuda.synchronize()
        np.save(os.path.join(out_dir, f"s{rank}.npy"), got.cpu().numpy())
        np.save(os.path.join(out_dir, "q.npy"), np.array(ctx.moduli[:limbs], dtype=np.uint64))
        # the same reduce over peer memory (IPC-mapped partials, flag waits, one summing kernel), two epochs
        prs = C.PeerReduceScatter(ctx, items, limbs, world, rank, timeout_s=10.0)
        for step, data in enumerate((parts, parts[::-1].copy())):
            prs.partials.copy_(torch.from_numpy(data).cuda())
            out = prs.reduce()
            torch.cuda.synchronize()
            prs.check()
            np.save(os.path.join(out_dir, f"peer{step}_{rank}.npy"), out.cpu().numpy())
            np.save(os.path.join(out_dir, f"pin{step}_{rank}.npy"), data)
        dist.barrier()
        prs.close()
        dist.barrier()
        ctx.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_modular_reduce_scatter_two_gpus(tmp_path):
    import torch.multiprocessing as mp

    from holmes_b200 import collectives as C

    world = 2
    mp.spawn(_worker, args=(world, _port(), str(tmp_path)), nprocs=world, join=True)
    parts = [np.load(tmp_path / f"p{r}.npy") for r in range(world)]
    q = [int(v) for v in np.load(tmp_path / "q.npy")]
    for r in range(world):
        got = np.load(tmp_path / f"s{r}.npy")
        owned = list(C.token_shard(4, world, r))
        want = sum(p[owned].astype(object) for p in parts)
        for li, ql in enumerate(q):
            assert np.array_equal(got[:, li].astype(object), want[:, li] % ql)
    # peer-memory reduce-scatter: word for word the same sums, on both epochs
    for step in range(2):
        ins = [np.load(tmp_path / f"pin{step}_{r}.npy") for r in range(world)]
        for r in range(world):
            got = np.load(tmp_path / f"peer{step}_{r}.npy")
            owned = list(C.token_shard(4, world, r))
            want = sum(p[owned].astype(object) for p in ins)
            for li, ql in enumerate(q):
                assert np.array_equal(got[:, li].astype(object), want[:, li] % ql), (step, r, li)


def _linear_worker(rank, world, port, out_dir):
    from datetime import timedelta

    import torch.distributed as dist

    from holmes_b200 import collectives as C
    from holmes_b200 import fhe as F
    from holmes_b200 import linear as LN
    from tests.gpu_helpers import make_pair

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        _, client, ctx = make_pair(log_n=11, limbs=4, dnum=2, dcrt=45, first=55, special=55)
        session = LN.Session(client, ctx)
        dim, lanes = 64, 16
        cfg = LN.BsgsSchedule(babies=8, anchor=8, chunk_rows=16)
        rng = np.random.default_rng(26081431)
        w = rng.normal(scale=0.02, size=(dim, dim))
        xs = rng.normal(size=(4, lanes, dim))
        cts = [client.encrypt(x.T.reshape(-1), cur_limbs=ctx.L, counter=100 + i) for i, x in enumerate(xs)]
        op = LN.LinearOperator(crypto_context=session, token_lanes=lanes, config=cfg, baby_shard=(rank, world, None))
        lw = LN.LinearWeight(w, dtype=w.dtype, crypto_context=session)
        chunks = C.chunk_shard(len(op.layout(dim).chunks), world, rank)
        parts, _ = op.apply(cts, lw, chunk_indices=chunks, rescale=False)
        s0 = C.modular_reduce_scatter(ctx, torch.cat([p.cv[0] for p in parts]), world)
        s1 = C.modular_reduce_scatter(ctx, torch.cat([p.cv[1] for p in parts]), world)
        mine = list(C.token_shard(4, world, rank))
        res = F.rescale(F.Cipher([s0, s1], parts[0].state, parts[0].slots, False, len(mine), ctx), ctx)
        torch.cuda.synchronize()
        np.save(os.path.join(out_dir, f"lin{rank}.npy"), torch.stack([res.cv[0], res.cv[1]]).cpu().numpy())
        dist.barrier()
        ctx.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_chunk_sharded_linear_with_baby_all_gather_two_gpus(tmp_path):
    """Chunk sharding with the baby key switches split over the ranks and all-gathered: every owner's rescaled
    output equals the oracle's single-process linear residue for residue."""
    import torch.multiprocessing as mp

    from holmes_b200 import collectives as C
    from holmes_b200 import linear as LN
    from tests.gpu_helpers import make_pair
    from tests.test_gpu_parity import _oracle_linear

    world = 2
    mp.spawn(_linear_worker, args=(world, _port(), str(tmp_path)), nprocs=world, join=True)
    o, _, ctx = make_pair(log_n=11, limbs=4, dnum=2, dcrt=45, first=55, special=55)
    try:
        dim, lanes = 64, 16
        plan = LN.BsgsSchedule(babies=8, anchor=8, chunk_rows=16).layout(dim, lanes)
        rng = np.random.default_rng(26081431)
        w = rng.normal(scale=0.02, size=(dim, dim))
        xs = rng.normal(size=(4, lanes, dim))
        refs = [o.encrypt(x.T.reshape(-1), ctx.L, counter=100 + i) for i, x in enumerate(xs)]
        expect = _oracle_linear(o, refs, w, plan, ctx.L, ctx.scale)
        for r in range(world):
            got = np.load(tmp_path / f"lin{r}.npy")
            for k, i in enumerate(C.token_shard(4, world, r)):
                np.testing.assert_array_equal(got[0, k], expect[i][0])
                np.testing.assert_array_equal(got[1, k], expect[i][1])
    finally:
        ctx.close()


def _transport_worker(rank, world, port, out_dir):
    import time
    from datetime import timedelta

    import torch.distributed as dist

    from holmes_b200 import transport as T
    from tests.gpu_helpers import make_pair

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        _, client, ctx = make_pair(log_n=12, limbs=4, dnum=2, dcrt=45, first=55, special=55)
        tr = T.build_transport(kind="nccl", default_timeout=60.0)
        assert tr.device_payloads and tr.device.type == "cuda"
        z = np.random.default_rng(rank).normal(size=ctx.max_slots) * 0.5
        ct = client.encrypt(z, cur_limbs=4, counter=rank)
        mine = [c.clone() for c in ct.cv]
        # point to point: rank 0 -> 1, received out of order
        if rank == 0:
            tr.send(1, "late", T.pack_cipher(ct, tag="late"))
            tr.send(1, "early", {"n": 7})
        else:
            first = tr.recv(0, "early")
            got = T.unpack_cipher(tr.recv(0, "late"), ctx)
            assert first == {"n": 7} and got.cv[0].device.type == "cuda"
            np.save(os.path.join(out_dir, "p2p.npy"), torch.stack([c[0] for c in got.cv]).cpu().numpy())
        # all_to_all of packets (device to device), then a timed page-sized exchange: 16 ciphertexts at 13 limbs
        # of N = 2^16 (218 MB) split over the ranks
        got = tr.all_to_all("cts", [T.pack_cipher(ct) for _ in range(world)])
        np.save(os.path.join(out_dir, f"a2a{rank}.npy"),
                np.stack([torch.stack([c[0] for c in g.components]).cpu().numpy() for g in got]))
        np.save(os.path.join(out_dir, f"mine{rank}.npy"), torch.stack([m[0] for m in mine]).cpu().numpy())
        big = torch.randint(0, 2**62, (16 // world, 2, 13, 1 << 16), dtype=torch.int64, device="cuda")
        for _ in range(2):
            tr.all_to_all("warm", [big] * world)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        reps = 5
        for _ in range(reps):
            tr.all_to_all("page", [big] * world)
        torch.cuda.synchronize()
        dt = (time.perf_counter() - t0) / reps
        with open(os.path.join(out_dir, f"gbs{rank}.txt"), "w") as f:
            f.write(f"{big.numel() * 8 * (world - 1) / dt / 1e9:.1f}")
        tr.close()
        dist.barrier()
        ctx.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_nccl_transport_two_gpus(tmp_path):
    """The reference's Transport protocol over NCCL: ciphertext packets move GPU to GPU bit for bit (point to point
    with out-of-order tags, all_to_all); a page-sized all_to_all reports its per-rank send bandwidth."""
    import torch.multiprocessing as mp

    world = 2
    mp.spawn(_transport_worker, args=(world, _port(), str(tmp_path)), nprocs=world, join=True)
    mine = [np.load(tmp_path / f"mine{r}.npy") for r in range(world)]
    np.testing.assert_array_equal(np.load(tmp_path / "p2p.npy"), mine[0])
    for r in range(world):
        got = np.load(tmp_path / f"a2a{r}.npy")
        for s in range(world):
            np.testing.assert_array_equal(got[s], mine[s])
    gbs = [float((tmp_path / f"gbs{r}.txt").read_text()) for r in range(world)]
    print("transport all_to_all GB/s per rank:", gbs)
    assert min(gbs) > 1.0
