"""Host side of the Paterson-Stockmeyer evaluator (holmes_b200/polynomial.py) against the reference's own coefficient
algebra (llama3fhe/approx/chebyshev.py, fixtures made by tests/golden/make_poly_golden.py)."""
import json
import os

import numpy as np
import pytest
from numpy.polynomial import chebyshev as C

from holmes_b200.polynomial import chebyshev_ps_mul_depth, compute_degrees_ps, evaluate_tree_numpy, ps_tree

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "poly_golden.json")


@pytest.fixture(scope="module")
def golden():
    with open(GOLDEN, encoding="utf-8") as f:
        return json.load(f)


def test_split_table_matches_reference(golden):
    """compute_degrees_ps for every degree of the table (1..2204) and the search beyond it."""
    bad = [(n, k, m, compute_degrees_ps(n)) for n, k, m in golden["degrees_ps"] if compute_degrees_ps(n) != (k, m)]
    assert not bad, bad[:5]


def test_tree_reproduces_the_reference_direct_evaluation(golden):
    """The split, evaluated in float64, equals eval_chebyshev_series_direct (c_0 halved, [a, b] mapped onto [-1, 1];
    the reference returns float32)."""
    for case in golden["direct"]:
        coeffs = np.asarray(case["coefficients"])
        a, b = case["a"], case["b"]
        x = np.asarray(case["x"])
        k, m, tree = ps_tree(coeffs)
        assert chebyshev_ps_mul_depth(coeffs) == case["depth"]
        got = evaluate_tree_numpy(tree, k, m, (2.0 * x - (a + b)) / (b - a))
        want = np.asarray(case["y"])
        assert np.allclose(got, want, rtol=2e-6, atol=2e-6 * np.abs(want).max()), (case["degree"],
                                                                                   np.abs(got - want).max())


def test_silu_fit_convention(golden):
    """A Chebyshev-Gauss fit in NumPy's convention is the reference's fit with c_0 doubled."""
    s = golden["silu59"]
    a, b = s["a"], s["b"]
    std = C.chebinterpolate(lambda y: (v := (y * (b - a) + (a + b)) / 2) / (1 + np.exp(-v)), 59)
    ref = np.asarray(s["coefficients"])
    assert np.allclose(std[1:], ref[1:], atol=1e-12) and abs(2 * std[0] - ref[0]) < 1e-12


@pytest.mark.parametrize("n", [1, 2, 3, 12, 17, 60, 236, 247, 1000])
def test_tree_is_exact_and_leaves_fit_the_baby_basis(n):
    rng = np.random.default_rng(n)
    coeffs = rng.normal(size=n + 1) / np.arange(1, n + 2)
    k, m, tree = ps_tree(coeffs)
    assert len(tree.leaves) == (1 << m) - 1
    assert all(leaf.weights.shape == (k + 1,) for leaf in tree.leaves)
    y = np.linspace(-1, 1, 513)
    std = coeffs.copy()
    std[0] *= 0.5
    assert np.abs(evaluate_tree_numpy(tree, k, m, y) - C.chebval(y, std)).max() < 1e-12


def test_degree_zero_refused():
    with pytest.raises(ValueError):
        ps_tree([1.0, 0.0])
    with pytest.raises(ValueError):
        compute_degrees_ps(0)
