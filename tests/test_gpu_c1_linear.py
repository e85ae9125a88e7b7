"""BASELINE config 1 (the reference's CPU-path linear), end to end on the GPU, residue for residue against the
oracle's restatement of LinearOperator.apply and decoded against the plaintext matvec.

N = 2^13 (4096 slots), 8 Q limbs of ~50-bit primes, dnum 2 (alpha 4) with K = alpha = 4 special primes (one
special prime against 4-limb digits would drown Delta = 2^40 in key-switch noise), Delta = 2^40, one ciphertext
x ~ N(0, 1)^4096, W ~ N(0, 0.02^2)^{4096 x 4096} times a seeded +-1 diagonal and the normalised Walsh-Hadamard
transform, lanes 1, baby 64, giant 64 in 512-row chunks, one rescale."""
import numpy as np
import pytest

from tests.gpu_helpers import host, make_pair
from tests.test_gpu_parity import _oracle_linear

pytestmark = pytest.mark.gpu


def _fwht_rows(a: np.ndarray) -> np.ndarray:
    """Normalised Walsh-Hadamard transform of every row (the butterfly recursion of the published algorithm)."""
    a = a.copy()
    n = a.shape[1]
    h = 1
    while h < n:
        b = a.reshape(a.shape[0], n // (2 * h), 2, h)
        x, y = b[:, :, 0, :].copy(), b[:, :, 1, :].copy()
        b[:, :, 0, :], b[:, :, 1, :] = x + y, x - y
        h *= 2
    return a / np.sqrt(n)


def test_config1_linear_bitexact_and_decodes():
    from holmes_b200 import linear as LN

    o, client, ctx = make_pair(log_n=13, limbs=8, dnum=2, dcrt=50, first=50, special=50, K=4, hamming=0, seed=0,
                               scale_bits=40)
    try:
        dim = 4096
        rng = np.random.default_rng(0)
        signs = rng.choice([-1.0, 1.0], size=dim)
        w = _fwht_rows(rng.normal(scale=0.02, size=(dim, dim)) * signs[None, :])
        x = rng.normal(size=dim)
        cfg = LN.BsgsSchedule(babies=64, anchor=64, chunk_rows=512)
        plan = cfg.layout(dim, 1)
        assert (plan.babies, plan.giants, len(plan.chunks)) == (64, 64, 8)
        session = LN.Session(client, ctx)
        cur = ctx.L
        ct = client.encrypt(x, cur_limbs=cur, counter=7)
        ref = o.encrypt(x, cur, counter=7)
        with LN.LinearOperator(crypto_context=session, token_lanes=1, config=cfg) as op, \
                LN.LinearWeight(w, dtype=w.dtype, crypto_context=session) as lw:
            outs, _ = op.apply([ct], lw)
        got = outs[0]
        expect = _oracle_linear(o, [ref], w, plan, cur, ctx.scale)[0]
        np.testing.assert_array_equal(host(got.cv[0][0]), expect[0])
        np.testing.assert_array_equal(host(got.cv[1][0]), expect[1])
        dec = client.decrypt(got).real
        want = x @ w.T
        assert np.abs(dec - want).max() < 1e-4 * np.abs(want).max()
    finally:
        ctx.close()
