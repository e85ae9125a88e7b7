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


def test_const_op_abi_host_constants(env):
    """holmes_const_op (per-limb constants by value from host memory): add, multiply and multiply-accumulate against the
    oracle's modular arithmetic, over both components in one launch (a run of 2 x batch items) and component by
    component (separate storages); limbs beyond the parameter table are refused."""
    import ctypes

    from holmes_b200 import _lib
    from holmes_b200 import fhe as F

    o, client, ctx = env
    rng = np.random.default_rng(7)
    cts = [client.encrypt(rng.normal(size=ctx.max_slots) * 0.3, cur_limbs=5, counter=40 + i) for i in range(3)]
    src = F.pack_cipher_batch(cts)
    n = src.batch_size
    assert F._run(src.cv, n) is not None       # a packed batch is one run of 2 x n items
    apart = F.Cipher([src.cv[0].clone(), src.cv[1].clone()], src.state, src.slots, False, n, ctx)
    assert F._run(apart.cv, n) is None
    ids = list(range(5))
    k1 = [int(v) for v in rng.integers(0, 2 ** 62, 5, dtype=np.uint64)]
    k1 = [v % ctx.q(i) for i, v in enumerate(k1)]
    k2 = [(3 * v + 11) % ctx.q(i) for i, v in enumerate(k1)]
    run = F._new_cipher(ctx, n, 5, src.state, src.slots)
    F.const_cv(ctx, F.CONST_MUL, src.cv, k1, run.cv, n, 5)
    split = F.Cipher([torch.empty_like(run.cv[0]), torch.empty_like(run.cv[1])], run.state, run.slots, False, n, ctx)
    F.const_cv(ctx, F.CONST_MUL, apart.cv, k1, split.cv, n, 5)
    F.const_cv(ctx, F.CONST_AXPY, src.cv, k2, run.cv, n, 5)
    added = F._new_cipher(ctx, n, 5, src.state, src.slots)
    F.const_cv(ctx, F.CONST_ADD, src.cv, k2, added.cv, n, 5)
    for c in range(2):
        for i in range(n):
            x = host(src.cv[c][i, :5])
            m1 = o.mul_scalar(x, k1, ids)
            np.testing.assert_array_equal(host(split.cv[c][i]), m1)
            np.testing.assert_array_equal(host(run.cv[c][i]), o.add(m1, o.mul_scalar(x, k2, ids), ids))
            want = np.stack([(x[l].astype(object) + k2[l]) % ctx.q(l) for l in ids]).astype(np.uint64)
            np.testing.assert_array_equal(host(added.cv[c][i]), want)
    # rescale, add and multiply-by-i: one launch over the run and one per component give the same words
    for fn in (lambda x: F.rescale(x, ctx), lambda x: F.homo_add(x, x, ctx), lambda x: F.homo_mul_i(x, ctx, True)):
        a, b = fn(src), fn(apart)
        for c in range(2):
            np.testing.assert_array_equal(host(a.cv[c]), host(b.cv[c]))
    r = F.rescale(src, ctx)
    for c in range(2):
        np.testing.assert_array_equal(host(r.cv[c][1]), o.rescale((host(src.cv[0][1, :5]), host(src.cv[1][1, :5])))[c])
    host_k = (ctypes.c_uint64 * 65)(*([1] * 65))
    rc = _lib.load().holmes_const_op(ctx.handle, 1, src.cv[0].data_ptr(), host_k, run.cv[0].data_ptr(), 1, 65,
                                     F._item_stride(src.cv[0]), F._item_stride(run.cv[0]), F._stream())
    assert rc == -2
