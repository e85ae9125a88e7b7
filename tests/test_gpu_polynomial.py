"""The fused homo_mul_relin_rescale_postop and the Paterson-Stockmeyer evaluator (holmes_b200/polynomial.py, mirror of
llama3fhe/operators/nonlinear/polynomial.py:469-562) on the GPU: residues of the fused post-operations against the
oracle, decoded Chebyshev series against NumPy at the stated tolerance."""
import numpy as np
import pytest
from numpy.polynomial import chebyshev as C

from tests.gpu_helpers import host, make_pair

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def deep():
    o, client, ctx = make_pair(log_n=12, limbs=12, dnum=3, dcrt=50, first=58, special=58, hamming=64, seed=5)
    yield o, client, ctx
    ctx.close()


def test_postop_residues_match_the_oracle(deep):
    """rescale(a b), doubled, minus a deeper ciphertext read at the output's limbs, plus a scalar: the oracle's
    multiply, relinearise, rescale, add, subtract and constant add, residue for residue."""
    from holmes_b200 import fhe as F
    from holmes_b200.polynomial import _post_scalar

    o, client, ctx = deep
    rng = np.random.default_rng(3)
    za, zb, zs = (rng.normal(size=ctx.max_slots) * 0.5 for _ in range(3))
    cur = 6
    a, ra = client.encrypt(za, cur_limbs=cur, counter=1), o.encrypt(za, cur, counter=1)
    b, rb = client.encrypt(zb, cur_limbs=cur, counter=2), o.encrypt(zb, cur, counter=2)
    s, rs = client.encrypt(zs, cur_limbs=9, counter=3), o.encrypt(zs, 9, counter=3)
    enc = _post_scalar(-0.75, a, b, ctx)
    out = F.homo_mul_relin_rescale_postop(a, b, ctx, apply_double=True, sub=s, scalar=enc)
    assert int(out.state.cur_limbs) == cur - 1 and int(out.state.scale_degree) == 1
    ids = list(range(cur - 1))
    e = o.rescale(o.mul_relin(ra, rb))
    e = [o.add(e[c], e[c], ids) for c in range(2)]
    e = [o.sub(e[c], np.ascontiguousarray(rs[c][: cur - 1]), ids) for c in range(2)]
    konst = np.stack([np.full(ctx.N, enc.integer % ctx.q(i), dtype=np.uint64) for i in ids])
    e[0] = o.add(e[0], konst, ids)
    for c in range(2):
        np.testing.assert_array_equal(host(out.cv[c][0, : cur - 1]), e[c])
    got = client.decrypt(out)
    assert np.abs(got - (2 * za * zb - zs - 0.75)).max() < 1e-6
    # the unfused sequence gives the same residues; a batch shares one broadcast sub
    plain = F.rescale(F.homo_mul_relin(a, b, ctx), ctx)
    ref = F.homo_add_scalar(F.homo_sub(F.homo_add(plain, plain, ctx), F.align_to(s, plain.state, ctx), ctx), enc, ctx)
    for c in range(2):
        np.testing.assert_array_equal(host(ref.cv[c][0]), host(out.cv[c][0]))
    ab = F.pack_cipher_batch([a, b])
    both = F.homo_mul_relin_rescale_postop(ab, ab, ctx, apply_double=True, sub=s)
    sq = F.homo_mul_relin_rescale_postop(b, b, ctx, apply_double=True, sub=s)
    for c in range(2):
        np.testing.assert_array_equal(host(both.cv[c][1]), host(sq.cv[c][0]))


def test_postop_refuses_mismatched_inputs(deep):
    from holmes_b200 import fhe as F

    _, client, ctx = deep
    a = client.encrypt(np.ones(ctx.max_slots) * 0.1, cur_limbs=6, counter=7)
    shallow = client.encrypt(np.ones(ctx.max_slots) * 0.1, cur_limbs=4, counter=8)
    with pytest.raises(ValueError):
        F.homo_mul_relin_rescale_postop(a, a, ctx, sub=shallow)


def _ref_coeffs(f, a, b, degree):
    std = C.chebinterpolate(lambda y: f((y * (b - a) + (a + b)) / 2), degree)
    ref = std.copy()
    ref[0] *= 2.0  # the reference's convention: c_0 halved at evaluation
    return std, ref


def test_silu_degree59_on_a_batch(deep):
    """SiLU on [-8, 8] at degree 59 (k = 4, m = 4: 6 levels + 1 for the map) on two ciphertexts at once; decoded
    against the same series in float64 to 1e-6 (50-bit scale)."""
    from holmes_b200 import fhe as F
    from holmes_b200.polynomial import chebyshev_ps_mul_depth, eval_chebyshev_series_cipher

    _, client, ctx = deep
    rng = np.random.default_rng(59)
    a, b = -8.0, 8.0
    std, ref = _ref_coeffs(lambda v: v / (1 + np.exp(-v)), a, b, 59)
    xs = [rng.uniform(a, b, size=ctx.max_slots) for _ in range(2)]
    batch = F.pack_cipher_batch([client.encrypt(x, cur_limbs=12, counter=20 + i) for i, x in enumerate(xs)])
    out = eval_chebyshev_series_cipher(batch, ref, lower_bound=a, upper_bound=b, crypto_context=ctx)
    assert int(out.state.cur_limbs) == 12 - 1 - chebyshev_ps_mul_depth(ref)
    for i, x in enumerate(xs):
        want = C.chebval((2 * x - (a + b)) / (b - a), std)
        err = np.abs(client.decrypt(out, item=i).real - want).max()
        assert err < 1e-6, err
        assert np.abs(want - x / (1 + np.exp(-x))).max() < 1e-3  # the fit itself


def test_degree236_mapped_input(deep):
    """Degree 236 (the SiLU degree of the model; k = 16, m = 4: 8 levels) on an input already in [-1, 1]."""
    from holmes_b200.polynomial import eval_chebyshev_series_cipher

    _, client, ctx = deep
    rng = np.random.default_rng(236)
    ref = rng.normal(size=237) / np.arange(1, 238)
    std = ref.copy()
    std[0] *= 0.5
    x = rng.uniform(-1, 1, size=ctx.max_slots)
    ct = client.encrypt(x, cur_limbs=12, counter=40)
    out = eval_chebyshev_series_cipher(ct, ref, lower_bound=-1.0, upper_bound=1.0, crypto_context=ctx,
                                       input_is_chebyshev_mapped=True)
    assert int(out.state.cur_limbs) == 4
    err = np.abs(client.decrypt(out).real - C.chebval(x, std)).max()
    assert err < 1e-6, err


def test_too_shallow_input_is_refused(deep):
    from holmes_b200.polynomial import eval_chebyshev_series_cipher

    _, client, ctx = deep
    ct = client.encrypt(np.zeros(ctx.max_slots), cur_limbs=5, counter=50)
    with pytest.raises(ValueError):
        eval_chebyshev_series_cipher(ct, np.ones(60), lower_bound=-1.0, upper_bound=1.0, crypto_context=ctx)
