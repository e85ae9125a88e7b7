"""Generate ``poly_golden.json`` by running the reference's own Chebyshev / Paterson-Stockmeyer coefficient algebra.

Run once, in a checkout that has the reference tree available (the fixture is committed; the tests only read it):

    python tests/golden/make_poly_golden.py /path/to/holmes

Pins, from ``llama3fhe/approx/chebyshev.py``:

* ``compute_degrees_ps`` (lines 79-108): the (k, m) split for every degree 1..2204 and a few beyond the table;
* ``chebyshev_ps_mul_depth`` (lines 111-121);
* ``eval_chebyshev_series_direct`` (lines 136-163): the coefficient convention (c_0 halved) and the map of
  [a, b] onto [-1, 1], on seeded coefficients and points;
* ``eval_chebyshev_coefficients`` (lines 22-48): the fit of SiLU on [-8, 8] at degree 59.
"""
from __future__ import annotations

import json
import math
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
from make_golden import _StubFinder  # noqa: E402


def main(reference_root: str) -> None:
    sys.meta_path.insert(0, _StubFinder())
    sys.path.insert(0, reference_root)
    from llama3fhe.approx import chebyshev as ch

    rng = np.random.default_rng(2024)
    meta = {}
    degrees = list(range(1, 2205)) + [2205, 2500, 3000, 4095]
    meta["degrees_ps"] = [[n, *ch.compute_degrees_ps(n)] for n in degrees]
    cases = []
    for n, a, b in ((5, -1.0, 1.0), (59, -8.0, 8.0), (119, 0.5, 40.0), (236, -20.0, 20.0)):
        coeffs = rng.normal(size=n + 1) / np.arange(1, n + 2)
        x = rng.uniform(a, b, size=64)
        y = ch.eval_chebyshev_series_direct(x, coeffs, a, b)
        cases.append({"degree": n, "a": a, "b": b, "coefficients": coeffs.tolist(), "x": x.tolist(),
                      "y": np.asarray(y, dtype=np.float64).tolist(), "depth": ch.chebyshev_ps_mul_depth(coeffs)})
    meta["direct"] = cases
    silu = ch.eval_chebyshev_coefficients(lambda v: v / (1.0 + math.exp(-v)), -8.0, 8.0, 59)
    meta["silu59"] = {"a": -8.0, "b": 8.0, "coefficients": np.asarray(silu).tolist()}
    with open(os.path.join(HERE, "poly_golden.json"), "w", encoding="utf-8") as f:
        json.dump(meta, f)
    print("wrote", len(meta["degrees_ps"]), "splits and", len(cases), "direct cases")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("HOLMES_REFERENCE", "../holmes"))
