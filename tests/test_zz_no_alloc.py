"""holmes_rescale_noalloc: the rescale entry point that allocates nothing.

Callers such as a serving runtime that owns the entire device memory pool, or a latency-critical loop that
must not let cudaMalloc synchronise the device, cannot hand holmes_rescale a scratch buffer on demand.  The
no-alloc variant takes its scratch from a fixed array inside the library.  This test calls it through the
C ABI twice in a row, on different ciphertexts, and requires residue-for-residue equality with
holmes_rescale given caller scratch; it also checks that a request larger than the fixed array is refused.
The file is named so that pytest collects it last; it builds its own context, so it passes alone too.
"""
import numpy as np
import pytest
import torch

from tests.gpu_helpers import host, make_pair

pytestmark = pytest.mark.gpu


def test_rescale_noalloc_matches_rescale_on_two_calls():
    from holmes_b200 import _lib as L

    _, client, ctx = make_pair(log_n=16, limbs=4, dnum=2, dcrt=50, first=55, special=55, K=2, hamming=64)
    rng = np.random.default_rng(11)
    cur = ctx.L
    for call in range(2):
        z = rng.normal(size=ctx.max_slots) + 1j * rng.normal(size=ctx.max_slots)
        ct = client.encrypt(z, cur_limbs=cur, counter=40 + call)
        src = torch.stack([ct.cv[0][0], ct.cv[1][0]])                  # [2][cur][N]
        want = torch.empty((2, cur - 1, ctx.N), dtype=torch.uint64, device=ctx.device)
        got = torch.full((2, cur - 1, ctx.N), 7, dtype=torch.uint64, device=ctx.device)
        scratch = torch.empty(2 * ctx.N, dtype=torch.uint64, device=ctx.device)
        L.call("holmes_rescale", ctx.handle, src.data_ptr(), cur * ctx.N, want.data_ptr(), (cur - 1) * ctx.N, cur, 2,
               scratch.data_ptr(), 0)
        L.call("holmes_rescale_noalloc", ctx.handle, src.data_ptr(), cur * ctx.N, got.data_ptr(), (cur - 1) * ctx.N,
               cur, 2, 0)
        np.testing.assert_array_equal(host(got), host(want))
    # five 2^16-word polynomials do not fit the 4 * 2^16-word array: refused before any launch
    big = torch.empty((5, cur, ctx.N), dtype=torch.uint64, device=ctx.device)
    out = torch.empty((5, cur - 1, ctx.N), dtype=torch.uint64, device=ctx.device)
    rc = L.load().holmes_rescale_noalloc(ctx.handle, big.data_ptr(), cur * ctx.N, out.data_ptr(), (cur - 1) * ctx.N,
                                         cur, 5, None)
    assert rc == -6
    torch.cuda.synchronize()
    ctx.close()
