"""The CPU restatement of bootstrapping (oracle/bootstrap_oracle.py, the checker of the GPU bootstrap) on its own:
N = 2^12, 20 limbs of 59/60-bit primes, level budget (3, 3), the program planned by holmes_b200.bootstrap.generate
for a host-only stand-in of the context.  The refreshed ciphertext has the program's output level and the fixed
scale Delta, and decrypts to the message; this pins the Paterson-Stockmeyer EvalMod and the one-rescale sums of the
restatement without a GPU."""
import types

import numpy as np

from holmes_b200 import bootstrap as BS
from oracle.bootstrap_oracle import OracleBootstrap
from oracle.oracle import Oracle, OracleParams


def test_oracle_bootstrap_refreshes_to_the_message():
    o = Oracle(OracleParams(log_n=12, limbs=20, dnum=4, dcrt_bits=59, first_mod_bits=60, special_bits=60,
                            special_limbs=None, hamming=64, seed=1, scale_bits=None))
    q = list(o.pr.q)
    n = 1 << 12
    ctx = types.SimpleNamespace(N=n, M=2 * n, L=20, logN=12, scale=float(2.0 ** o.pr.scale_bits),
                                q=lambda i: q[i])
    prog = BS.generate(ctx, BS.BootstrapSpec(log_slots=11, level_budget=(3, 3), k_bound=12))
    rng = np.random.default_rng(1)
    z = rng.normal(size=n // 2) * 0.3
    c0, c1, scale = OracleBootstrap(o, prog).bootstrap(o.encrypt(z, 2, counter=9), s_in=float(ctx.scale))
    assert c0.shape[0] == prog.output_limbs == 20 - prog.spec.depth
    assert scale == float(ctx.scale)
    err = np.abs(o.decrypt(c0, c1, scale) - z).max()
    assert err < 1e-6, err
