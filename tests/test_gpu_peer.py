"""The peer-memory reduce-scatter's building blocks on one GPU.

* world 1: ``PeerReduceScatter.reduce`` over its own IPC-shareable buffer returns the partials word for word, on
  two epochs in a row;
* failure detection without a fault: a flag wait on a flag that nothing sets runs out after a short cycle budget,
  writes the flag's index + 1 into the status word and returns; the summing kernel after it does nothing; the host
  reads the status and raises; the context stays usable (a following sum is exact).
"""
import ctypes

import numpy as np
import pytest
import torch

from tests.gpu_helpers import dev, host, make_pair, residues

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def pair():
    o, client, ctx = make_pair(log_n=12, limbs=3, dnum=1, dcrt=45, first=55, special=55)
    yield o, client, ctx
    ctx.close()


def test_world_one_reduce_is_identity(pair):
    from holmes_b200 import collectives as C

    o, _, ctx = pair
    prs = C.PeerReduceScatter(ctx, 2, 3, 1, 0, timeout_s=1.0)
    try:
        rng = np.random.default_rng(1)
        for _ in range(2):
            parts = np.stack([residues(o.pr.q, 3, o.pr.n, rng) for _ in range(2)])
            prs.partials.copy_(dev(parts))
            out = prs.reduce()
            np.testing.assert_array_equal(host(out), parts)
            prs.check()
        assert prs.epoch == 2
    finally:
        prs.close()


def test_flag_wait_runs_out_and_reports(pair):
    from holmes_b200 import _lib as L

    o, _, ctx = pair
    flags = torch.zeros(2, dtype=torch.uint64, device=ctx.device)
    flags[0] = 5                                        # flag 0 is at epoch 5; flag 1 is never set
    status = torch.zeros(1, dtype=torch.int32, device=ctx.device)
    ptrs = L.ptr_array([flags.data_ptr(), flags.data_ptr() + 8])
    L.call("holmes_peer_wait", ptrs, 2, 5, 20_000_000, status.data_ptr(), 0)   # ~10 ms at the SM clock
    torch.cuda.synchronize()
    assert int(status.item()) == 2                      # flag 1 (index + 1) gave up
    # the summing kernel does nothing while the status is set ...
    rng = np.random.default_rng(2)
    a = dev(residues(o.pr.q, 3, o.pr.n, rng)[None])
    out = torch.full_like(a, 7)
    srcs = L.ptr_array([a.data_ptr()])
    L.call("holmes_modreduce_scatter", ctx.handle, srcs, 1, out.data_ptr(), 1, 3, 3 * o.pr.n, status.data_ptr(), 0)
    assert int(host(out).max()) == 7 and int(host(out).min()) == 7
    # ... and sums once it is cleared; the context is still usable
    status.zero_()
    L.call("holmes_modreduce_scatter", ctx.handle, srcs, 1, out.data_ptr(), 1, 3, 3 * o.pr.n, status.data_ptr(), 0)
    np.testing.assert_array_equal(host(out), host(a))
    # a satisfied wait leaves the status alone
    L.call("holmes_peer_wait", L.ptr_array([flags.data_ptr()]), 1, 5, 20_000_000, status.data_ptr(), 0)
    torch.cuda.synchronize()
    assert int(status.item()) == 0


def test_peer_reduce_scatter_check_raises_on_timeout(pair):
    from holmes_b200 import collectives as C

    _, _, ctx = pair
    prs = C.PeerReduceScatter(ctx, 1, 3, 1, 0, timeout_s=1.0)
    try:
        prs.status.fill_(3)
        with pytest.raises(TimeoutError):
            prs.check()
        assert int(prs.status.item()) == 0
    finally:
        prs.close()
