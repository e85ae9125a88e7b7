"""The three hoist strategies of the linear operator (operators/linear/config.py:9, 354-359) restated on the CPU
oracle at N = 2^10: "normal" (Horner over Q), "ext_normal" (babies and MAC over Q u P, a ModDown per giant partial)
and "ext_double_hoist" (every giant rotated over Q u P, one ModDown of the sum) all decode to W x at the reference's
linear tolerance.  The GPU tests hold the engine to these restatements residue for residue; this pins the
restatements themselves to the plaintext product."""
import numpy as np

from holmes_b200 import linear as LN
from oracle.oracle import Oracle, OracleParams
from tests.test_gpu_parity import _oracle_linear, _oracle_linear_ext


def test_hoist_strategy_restatements_decode_to_the_product():
    o = Oracle(OracleParams(log_n=10, limbs=4, dnum=2, dcrt_bits=45, first_mod_bits=55, special_bits=55,
                            hamming=32, seed=3))
    dim, lanes = 32, 16
    rng = np.random.default_rng(5)
    w = rng.normal(scale=0.02, size=(dim, dim))
    x = rng.normal(size=(lanes, dim))
    cur = o.pr.limbs
    scale = o.pr.scale()
    ref = o.encrypt(x.T.reshape(-1), cur, counter=1)
    want = x @ w.T
    out_scale = scale * scale / o.pr.q[cur - 1]
    got = {}
    for strategy in ("normal", "ext_normal", "ext_double_hoist"):
        cfg = LN.BsgsSchedule(babies=4, anchor=4, chunk_rows=16,
                                      hoist=strategy)
        plan = cfg.layout(dim, lanes)
        assert plan.chunks[0].count == 4
        if strategy == "normal":
            (res,) = _oracle_linear(o, [ref], w, plan, cur, scale)
        else:
            (res,) = _oracle_linear_ext(o, [ref], w, plan, cur, scale, double=strategy == "ext_double_hoist")
        dec = o.decrypt(res[0], res[1], out_scale).real.reshape(dim, lanes).T
        np.testing.assert_allclose(dec, want, atol=2e-8 * 50, rtol=2e-6)
        got[strategy] = dec
    assert np.abs(got["ext_double_hoist"] - got["normal"]).max() < 1e-6
