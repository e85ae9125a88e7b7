"""The device-payload transport (holmes_b200/transport.py) on CPU: world-size-2 gloo process groups run the
reference's Transport protocol (llama3fhe/parallel/prefill/transport.py:480-611; its contract test
tests/test_parallel_transport.py:205-273): tagged point-to-point with out-of-order receives, all_gather, all_to_all,
the split-phase variants and their in-flight rule, gather_to, barrier, the errors, and payloads that keep uint64 /
complex128 tensors and large NumPy arrays bit for bit."""
import os
import pickle
import socket
from dataclasses import dataclass

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from holmes_b200 import transport as T


def _port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@dataclass
class Packet:
    components: tuple
    state: tuple
    tag: str = ""


def _payload(rank: int, salt: int) -> Packet:
    g = torch.Generator().manual_seed(1000 * rank + salt)
    c0 = torch.randint(0, 2**62, (2, 3, 64), generator=g, dtype=torch.int64).view(torch.uint64)
    c1 = torch.randn(5, generator=g, dtype=torch.complex128)
    big = np.random.default_rng(rank + salt).integers(0, 2**63, size=20000, dtype=np.uint64)  # 160 KB: travels
    return Packet((c0, c1, big, np.arange(3)), (13, 1, 2.0**50 + rank), tag=f"r{rank}")


def _same(a: Packet, b: Packet) -> bool:
    return (a.state == b.state and a.tag == b.tag and torch.equal(a.components[0], b.components[0])
            and a.components[0].dtype == torch.uint64 and torch.equal(a.components[1], b.components[1])
            and np.array_equal(a.components[2], b.components[2]) and a.components[2].dtype == np.uint64
            and np.array_equal(a.components[3], b.components[3]))


def _worker(rank, world, port, out_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    log = {}
    try:
        tr = T.build_transport(kind="nccl", default_timeout=30.0)
        assert tr.rank == rank and tr.world_size == world and tr.peers == (1 - rank,) and tr.device_payloads
        peer = 1 - rank
        # point to point, received in the other order than sent
        if rank == 0:
            tr.send(1, "a", _payload(0, 1))
            tr.send(1, "b", _payload(0, 2))
            tr.send(1, "none", None)
        else:
            log["b"] = _same(tr.recv(0, "b"), _payload(0, 2))
            log["a"] = _same(tr.recv(0, "a"), _payload(0, 1))
            log["none"] = tr.recv(0, "none") is None
        # collectives
        got = tr.all_gather("ag", _payload(rank, 3))
        log["all_gather"] = all(_same(got[r], _payload(r, 3)) for r in range(world))
        got = tr.all_to_all("a2a", [_payload(rank, 10 + d) for d in range(world)])
        log["all_to_all"] = all(_same(got[s], _payload(s, 10 + rank)) for s in range(world))
        h = tr.all_gather_isend("split", {"x": torch.full((4,), rank)})
        try:
            tr.all_gather("too-early", 1)
            log["in_flight_rule"] = False
        except RuntimeError:
            log["in_flight_rule"] = True
        got = h.wait()
        log["split"] = h.done and all(torch.equal(got[r]["x"], torch.full((4,), r)) for r in range(world))
        got = tr.gather_to(0, "g", (rank, "x" * rank))
        log["gather_to"] = got == [(0, ""), (1, "x")] if rank == 0 else got is None
        tr.barrier()
        # errors
        for bad, exc in ((lambda: tr.send(rank, "self", None), ValueError), (lambda: tr.send(5, "oob", None), IndexError),
                         (lambda: tr.all_to_all("bad", [None]), ValueError)):
            try:
                bad()
                log.setdefault("errors", []).append(False)
            except exc:
                log.setdefault("errors", []).append(True)
        stats = tr.stats.to_dict()
        log["stats"] = stats["collectives"] >= 5 and stats["bytes_sent"] > 0 and stats["bytes_received"] > 0
        tr.barrier()
        if rank == 1:
            try:
                tr.recv(0, "never", timeout=0.2)
                log["timeout"] = False
            except TimeoutError:
                log["timeout"] = True
        else:
            log["timeout"] = True
        dist.barrier()
    finally:
        with open(os.path.join(out_dir, f"log{rank}.pkl"), "wb") as f:
            pickle.dump(log, f)
        dist.destroy_process_group()


def test_transport_protocol_gloo_world2(tmp_path):
    mp.spawn(_worker, args=(2, _port(), str(tmp_path)), nprocs=2, join=True)
    for r in range(2):
        with open(tmp_path / f"log{r}.pkl", "rb") as f:
            log = pickle.load(f)
        assert log.pop("errors") == [True, True, True], log
        assert all(log.values()), (r, log)
        if r == 1:
            assert {"a", "b", "none"} <= set(log)


def test_factory_and_packets():
    with pytest.raises(ValueError):
        T.build_transport(kind="host")
    with pytest.raises(RuntimeError):
        T.NcclTransport()   # no process group
    from holmes_b200 import fhe as F

    cv = [torch.arange(12, dtype=torch.int64).view(torch.uint64).reshape(1, 3, 4) for _ in range(2)]
    ct = F.Cipher(cv, F.CipherState(3, 1, 2.0**40), 2, False, 1, None)
    pk = T.pack_cipher(ct, tag="x")
    assert pk.nbytes == 2 * 12 * 8 and pk.components[0] is cv[0]
