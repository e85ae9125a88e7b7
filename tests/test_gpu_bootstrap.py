"""CKKS bootstrapping on the GPU: residue-for-residue against the CPU restatement (oracle/bootstrap_oracle.py),
decoded against the input message, and batched refresh (refresh_many) identical to one-at-a-time refresh.

Ring N = 2^12 (2^11 slots), 20 limbs of 59/60-bit primes (the reference's production prime sizes), level budget
(3, 3): depth 3 + 10 + 3 = 16, so 4 limbs remain."""
import numpy as np
import pytest

from tests.gpu_helpers import host, make_pair

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def boot():
    from holmes_b200 import bootstrap as BS
    from holmes_b200 import linear as LN

    o, client, ctx = make_pair(log_n=12, limbs=20, dnum=4, dcrt=59, first=60, special=60, hamming=64, seed=1)
    session = LN.Session(client, ctx)
    cfg = BS.BootstrapConfig(log_slots=11, level_budget=(3, 3), k_bound=12)
    op = BS.BootstrapOperator.prepare(session, cfg)
    yield o, client, ctx, op
    ctx.close()


def test_bootstrap_decodes_to_the_message(boot):
    _, client, ctx, op = boot
    rng = np.random.default_rng(0)
    z = (rng.normal(size=ctx.max_slots) + 1j * rng.normal(size=ctx.max_slots)) * 0.5
    ct = client.encrypt(z, cur_limbs=3, counter=5)
    out = op.refresh(ct)
    assert int(out.state.cur_limbs) == op.program.output_limbs == ctx.L - 16
    err = np.abs(client.decrypt(out) - z).max()
    assert err < 1e-6, err


def test_bootstrap_bitexact_vs_oracle(boot):
    from oracle.bootstrap_oracle import OracleBootstrap

    o, client, ctx, op = boot
    rng = np.random.default_rng(1)
    z = rng.normal(size=ctx.max_slots) * 0.3
    ct = client.encrypt(z, cur_limbs=2, counter=9)
    ref = o.encrypt(z, 2, counter=9)
    got = op.refresh(ct)
    e0, e1, esf = OracleBootstrap(o, op.program).bootstrap(ref, s_in=float(ct.state.scaling_factor))
    np.testing.assert_array_equal(host(got.cv[0][0]), e0)
    np.testing.assert_array_equal(host(got.cv[1][0]), e1)
    assert float(got.state.scaling_factor) == esf


def test_refresh_many_matches_single(boot):
    _, client, ctx, op = boot
    rng = np.random.default_rng(2)
    cts = [client.encrypt(rng.normal(size=ctx.max_slots) * 0.4, cur_limbs=3, counter=20 + i) for i in range(3)]
    many = op.refresh_many(cts)
    for ct, m in zip(cts, many):
        one = op.refresh(ct)
        np.testing.assert_array_equal(host(m.cv[0][0]), host(one.cv[0][0]))
        np.testing.assert_array_equal(host(m.cv[1][0]), host(one.cv[1][0]))
    assert op.batch_calls >= 1


def test_meta_bts_correction(boot):
    """The two-pass Meta-BTS correction (iterations = 2): residue for residue against the oracle, output at the
    input's scale with one limb fewer than a single refresh, and a smaller error than one refresh."""
    from oracle.bootstrap_oracle import OracleBootstrap

    o, client, ctx, op = boot
    rng = np.random.default_rng(5)
    z = rng.normal(size=ctx.max_slots) * 0.4
    ct = client.encrypt(z, cur_limbs=3, counter=60)
    ref = o.encrypt(z, 3, counter=60)
    one = op.refresh(ct)
    two = op.refresh(ct, iterations=2, precision_bits=8)
    assert int(two.state.cur_limbs) == int(one.state.cur_limbs) - 1
    assert float(two.state.scaling_factor) == float(ct.state.scaling_factor)
    e0, e1, esf = OracleBootstrap(o, op.program).refresh(ref, float(ct.state.scaling_factor), 2, 8)
    np.testing.assert_array_equal(host(two.cv[0][0]), e0)
    np.testing.assert_array_equal(host(two.cv[1][0]), e1)
    err1 = np.abs(client.decrypt(one) - z).max()
    err2 = np.abs(client.decrypt(two) - z).max()
    assert err2 < err1 / 8, (err1, err2)
    many = op.refresh_many([ct, ct], iterations=2, precision_bits=8)
    np.testing.assert_array_equal(host(many[1].cv[0][0]), host(two.cv[0][0]))
    with pytest.raises(ValueError):
        op.refresh(ct, iterations=3)


def test_pair_bootstrap_and_halve(boot):
    """Two real ciphertexts through one refresh as a + i b (stations.pair_bootstrap), unpacked with the
    conjugation to (2a, 2b), then halved."""
    from holmes_b200 import refresh as R

    _, client, ctx, op = boot
    rng = np.random.default_rng(3)
    a, b = rng.normal(size=ctx.max_slots) * 0.3, rng.normal(size=ctx.max_slots) * 0.3
    cts = [client.encrypt(a, cur_limbs=3, counter=40), client.encrypt(b, cur_limbs=3, counter=41)]
    out, factor = R.pair_bootstrap(cts, context=ctx, bootstrap_operator=op)
    assert factor == 2.0 and len(out) == 2
    assert np.abs(client.decrypt(out[0]) - 2 * a).max() < 1e-5
    assert np.abs(client.decrypt(out[1]) - 2 * b).max() < 1e-5
    half = R.halve(out, context=ctx)
    assert np.abs(client.decrypt(half[0]) - a).max() < 1e-5
    assert np.abs(client.decrypt(half[1]) - b).max() < 1e-5
    with pytest.raises(ValueError):
        R.pair_bootstrap(cts[:1], context=ctx, bootstrap_operator=op)


def test_bootstrap_rejects_bad_input(boot):
    _, client, ctx, op = boot
    ct = client.encrypt(np.zeros(ctx.max_slots), cur_limbs=1, counter=30)
    with pytest.raises(ValueError):
        op.refresh(ct)


@pytest.fixture(scope="module")
def sparse_boot():
    from holmes_b200 import bootstrap as BS
    from holmes_b200 import linear as LN

    o, client, ctx = make_pair(log_n=12, limbs=20, dnum=4, dcrt=59, first=60, special=60, hamming=64, seed=2)
    session = LN.Session(client, ctx)
    cfg = BS.BootstrapConfig(log_slots=8, level_budget=(3, 3), k_bound=12)   # 256 slots of 2048: gap 8
    op = BS.BootstrapOperator.prepare(session, cfg)
    yield o, client, ctx, op
    ctx.close()


def test_sparse_slot_bootstrap_decodes_and_matches_oracle(sparse_boot):
    """Sparse slots (the reference's 2^3 .. 2^12-slot programs): subsum over the rotations by n j, then the
    n-point CoeffsToSlots / EvalMod / SlotsToCoeffs; decoded against the message, residues against the oracle."""
    from oracle.bootstrap_oracle import OracleBootstrap

    o, client, ctx, op = sparse_boot
    n = op.program.n
    assert op.program.gap == ctx.N // (2 * n) == 8
    rng = np.random.default_rng(3)
    z = (rng.normal(size=n) + 1j * rng.normal(size=n)) * 0.5
    ct = client.encrypt(z, slots=n, cur_limbs=3, counter=31)
    out = op.refresh(ct)
    assert int(out.slots) == n
    err = np.abs(client.decrypt(out) - z).max()
    assert err < 1e-6, err
    ref = o.encrypt(z, 3, counter=31, slots=n)
    e0, e1, esf = OracleBootstrap(o, op.program).bootstrap(ref, s_in=float(ct.state.scaling_factor))
    np.testing.assert_array_equal(host(out.cv[0][0]), e0)
    np.testing.assert_array_equal(host(out.cv[1][0]), e1)
    assert float(out.state.scaling_factor) == esf
