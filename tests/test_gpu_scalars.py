"""Scalar and plaintext-addend operations of the EasyFHE surface (encode_scalar, homo_mul_scalar[_rescale],
homo_add_scalar, homo_add_pt): residues against the oracle's exact modular arithmetic, values against NumPy."""
import numpy as np
import pytest
import torch

from tests.gpu_helpers import host, make_pair

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def env():
    o, client, ctx = make_pair(log_n=12, limbs=6, dnum=2, dcrt=50, first=55, special=55, hamming=64, seed=4)
    yield o, client, ctx
    ctx.close()


def test_mul_scalar_residues_and_value(env):
    from holmes_b200 import fhe as F

    o, client, ctx = env
    rng = np.random.default_rng(0)
    z = rng.normal(size=ctx.max_slots) * 0.5
    ct = client.encrypt(z, cur_limbs=5, counter=1)
    enc = F.encode_scalar(-0.375, cur_limbs=5, scaling_factor=float(ctx.q(4)), context=ctx)
    raw = F.homo_mul_scalar(ct, enc, ctx)
    k = [enc.integer % ctx.q(i) for i in range(5)]
    for c in range(2):
        want = o.mul_scalar(host(ct.cv[c][0, :5]), k, list(range(5)))
        np.testing.assert_array_equal(host(raw.cv[c][0, :5]), want)
    out = F.homo_mul_scalar_rescale(ct, enc, ctx)
    assert int(out.state.cur_limbs) == 4
    assert np.abs(client.decrypt(out) - (-0.375) * z).max() < 1e-6


def test_add_scalar_and_pt(env):
    from holmes_b200 import fhe as F

    _, client, ctx = env
    rng = np.random.default_rng(1)
    z = rng.normal(size=ctx.max_slots) * 0.5
    w = rng.normal(size=ctx.max_slots) * 0.5 + 1j * rng.normal(size=ctx.max_slots) * 0.5
    ct = client.encrypt(z, cur_limbs=4, counter=2)
    out = F.homo_add_scalar(ct, 0.8125, ctx)
    assert np.abs(client.decrypt(out) - (z + 0.8125)).max() < 1e-6
    sf = float(ct.state.scaling_factor)
    pv = F.encode_rows(ctx, torch.from_numpy(w[None, :]).to(ctx.device), 4, sf, ctx.max_slots)
    pt = F.Plaintext([pv], F.CipherState(4, 1, sf), ctx.max_slots, False, 1, ctx)
    out = F.homo_add_pt(ct, pt, ctx)
    assert np.abs(client.decrypt(out) - (z + w)).max() < 1e-6
    with pytest.raises(ValueError):
        F.encode_scalar(1j, cur_limbs=4, context=ctx)


def test_grouped_scalar_weighted_acc_matches_the_loop():
    """polynomial.py:255-300: the weight table through one launch equals the scalar-multiply-and-add loop residue for
    residue (20 terms: the kernel's sums restart after 16)."""
    from holmes_b200 import fhe as F

    o, client, ctx = make_pair(log_n=10, limbs=4, dnum=2, dcrt=40, first=50, special=50)
    try:
        rng = np.random.default_rng(11)
        n, cur = 20, 3
        cts = [client.encrypt(rng.normal(size=ctx.max_slots) * 0.3, cur_limbs=cur, counter=60 + i) for i in range(n)]
        batch = F.pack_cipher_batch(cts)
        weights = rng.normal(size=(2, n))
        sf = float(cts[0].state.scaling_factor)
        bundle = F.ConstantBundle(scalars={f"w{g}_{k}": weights[g, k] for g in range(2) for k in range(n)})
        tables = [bundle.encoded_scalars([f"w{g}_{k}" for k in range(n)], cur_limbs=cur, scale_degree=1, context=ctx,
                                         scaling_factor=sf) for g in range(2)]
        table = F.EncodedScalar(F.torch.stack([t.residues for t in tables]), cur, 1, sf)
        acc = F.grouped_scalar_weighted_acc(batch, table, ctx)
        assert acc.batch_size == 2
        for g in range(2):
            loop = None
            for k in range(n):
                term = F.homo_mul_scalar(cts[k], F.encode_scalar(weights[g, k], cur, 1, sf, ctx), ctx)
                loop = term if loop is None else F.homo_add(loop, term, ctx)
            for c in range(2):
                np.testing.assert_array_equal(host(acc.cv[c][g]), host(loop.cv[c][0, :cur]))
    finally:
        ctx.close()
