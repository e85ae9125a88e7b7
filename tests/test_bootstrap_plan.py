"""Bootstrapping host logic on CPU: the level-grouped butterfly factorisation of CoeffsToSlots / SlotsToCoeffs
against the oracle's special FFT, the Chebyshev cosine, and the key / depth requirements."""
import numpy as np
import pytest

from holmes_b200 import bootstrap as BS
from oracle.oracle import Oracle, OracleParams, _p, lib


def _bitrev(v):
    n = v.size
    bits = n.bit_length() - 1
    idx = np.array([int(format(i, f"0{bits}b")[::-1], 2) for i in range(n)])
    return v[idx]


@pytest.mark.parametrize(("log_n", "budget", "sparse"), [(10, 3, 1), (12, 3, 1), (12, 4, 1), (13, 5, 1), (12, 3, 4),
                                                     (13, 2, 64)])
def test_transform_levels_match_special_fft(log_n, budget, sparse):
    o = Oracle(OracleParams(log_n=log_n, limbs=2, dnum=1, dcrt_bits=40, first_mod_bits=50, special_bits=50))
    n, M = o.pr.n // 2 // sparse, 2 * o.pr.n
    rng = np.random.default_rng(log_n)
    v = rng.normal(size=n) + 1j * rng.normal(size=n)
    # oracle special inverse FFT (with bit reversal and 1/n)
    re, im = np.ascontiguousarray(v.real), np.ascontiguousarray(v.imag)
    lib().orc_fft_special_inv(_p(re), _p(im), n, M, _p(o.rot_group), _p(o.ksi_re), _p(o.ksi_im))
    inv = re + 1j * im
    c2s = BS.fft_levels(n, M, budget, inverse=True)
    assert len(c2s) == budget
    np.testing.assert_allclose(BS.apply_levels_numpy(c2s, v), n * _bitrev(inv), atol=1e-8 * n)
    # forward: butterflies after bit reversal
    re, im = np.ascontiguousarray(v.real), np.ascontiguousarray(v.imag)
    lib().orc_fft_special(_p(re), _p(im), n, M, _p(o.rot_group), _p(o.ksi_re), _p(o.ksi_im))
    fwd = re + 1j * im
    s2c = BS.fft_levels(n, M, budget, inverse=False)
    np.testing.assert_allclose(BS.apply_levels_numpy(s2c, _bitrev(v)), fwd, atol=1e-8 * n)
    # diagonal counts: a level of s stages has at most 2^(s+1) - 1 diagonals
    stages = int(np.log2(n))
    for lvl in c2s + s2c:
        assert len(lvl) <= 2 ** (int(np.ceil(stages / budget)) + 1) - 1


def test_chebyshev_cosine_accuracy():
    B, r = 13.0, 3
    c = BS.chebyshev_cos(B, r, 63)
    w = np.linspace(-1, 1, 2001)
    got = np.polynomial.chebyshev.chebval(w, c)
    assert np.abs(got - np.cos(2 * np.pi * B * w / 2 ** r)).max() < 1e-12
    # r double angles of cos(2 pi (v - 1/4) / 2^r) give sin(2 pi v)
    v = np.linspace(-12.4, 12.4, 997)
    x = np.polynomial.chebyshev.chebval((v - 0.25) / B, c)
    for _ in range(r):
        x = 2 * x * x - 1
    assert np.abs(x - np.sin(2 * np.pi * v)).max() < 1e-9


def test_requirements_and_depth():
    spec = BS.BootstrapSpec(log_slots=11, level_budget=(3, 3), k_bound=12)
    req = BS.requirements([spec], log_n=12)
    assert spec.depth == 3 + 10 + 3 == req.depth
    assert (2 << 12) - 1 in req.rotations
    assert all(0 < r < (1 << 11) or r == (2 << 12) - 1 for r in req.rotations)
    with pytest.raises(ValueError):
        BS.BootstrapSpec(mode="slots_first")


def _automorph(t: np.ndarray, k: int) -> np.ndarray:
    """sigma_k(t)(X) = t(X^k) in Z[X]/(X^N + 1)."""
    N = t.size
    out = np.zeros_like(t)
    for i, c in enumerate(t):
        e = (i * k) % (2 * N)
        if e < N:
            out[e] += c
        else:
            out[e - N] -= c
    return out


@pytest.mark.parametrize("log_slots", [6, 8])
def test_sparse_subsum_is_gap_times_the_subring_part(log_slots):
    """Rotations by n j (j < gap) are the automorphisms X -> X^(5^(n j)) fixing X^gap: the log2(gap) rotate-and-add
    steps of the sparse-slot bootstrap leave gap times the coefficients at multiples of gap, the rest cancels."""
    N, n = 1 << 10, 1 << log_slots
    gap = N // (2 * n)
    t = np.random.default_rng(log_slots).integers(-1000, 1000, size=N)
    acc = t.copy()
    g = 1
    while g < gap:
        acc = acc + _automorph(acc, pow(5, n * g, 2 * N))
        g *= 2
    want = np.zeros_like(t)
    want[::gap] = gap * t[::gap]
    np.testing.assert_array_equal(acc, want)
    spec = BS.BootstrapSpec(log_slots=log_slots, level_budget=(2, 2))
    req = BS.requirements([spec], log_n=10)
    assert {n << i for i in range(int(np.log2(gap)))} <= set(req.rotations)


def test_refresh_iterations_validated_on_host():
    """Meta-BTS accepts one or two iterations; the check runs before any device work."""
    from holmes_b200 import bootstrap as BS

    calls = []
    with pytest.raises(ValueError):
        BS.with_correction(object(), None, lambda c: calls.append(c), 3, 8)
    assert not calls


@pytest.mark.parametrize("degree", [7, 8, 31, 63, 64, 100])
def test_paterson_stockmeyer_split_reproduces_the_series(degree):
    """EvalMod's Chebyshev-basis split p = q T_n + r (bootstrap.cheb_split), applied recursively down to leaves of
    ps_baby(degree) coefficients exactly as bootstrap._chebyshev / OracleBootstrap.chebyshev do, evaluates to the
    series itself; and it never needs more than log2(degree + 1) + 1 levels."""
    from numpy.polynomial import chebyshev as C

    rng = np.random.default_rng(degree)
    c = list(rng.normal(size=degree + 1) / (1 + np.arange(degree + 1)))
    x = np.linspace(-1, 1, 257)
    m = BS.ps_baby(degree)
    T = lambda k: C.chebval(x, [0] * k + [1])  # noqa: E731

    def depth_of(k):   # levels T_k costs in the power tree (T_2k = 2 T_k^2 - 1, T_2k+1 = 2 T_k T_k+1 - T_1)
        return 0 if k <= 1 else int(np.ceil(np.log2(k)))

    def evalp(cs):
        if len(cs) <= m:
            lvl = max(depth_of(k) for k in range(1, len(cs))) + 1 if len(cs) > 1 else 1
            return C.chebval(x, cs), lvl
        n = 1 << (int(np.ceil(np.log2(len(cs)))) - 1)
        q, r = BS.cheb_split(cs, n)
        (qv, ql), (rv, rl) = evalp(q), evalp(r)
        return qv * T(n) + rv, max(max(ql, depth_of(n)) + 1, rl)

    val, levels = evalp(c)
    np.testing.assert_allclose(val, C.chebval(x, c), atol=1e-12)
    assert levels <= int(np.ceil(np.log2(degree + 1))) + 1
    assert m == 1 << max(1, int(np.ceil(np.log2(degree + 1) / 2)))
