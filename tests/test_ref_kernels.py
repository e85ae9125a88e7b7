"""Pin the oracle -- and the engine's drop-in entry points -- to the reference's own CUDA kernels.

``make -C oracle ref`` compiles ``bench/cmp/kernels/holmes_encode.cu`` and ``holmes_mac.cu`` from the
reference tree into ``oracle/_ref/`` (sm_100a).  These are the only reference binaries that exist (the
rest of the arithmetic lives in EasyFHE, which is not distributed), and they document EasyFHE's
conventions: NTT root order, encode rounding / reduction, the plaintext MAC.  Both are N = 2^16.

* encode stage 2 (llround(v sf) + per-limb reduction + NTT, holmes_encode.cu:115-226) is compared
  with the oracle's rounding + NTT and with libholmes_cuda's ``holmes_encode_fft``;
* ``holmes_mac_multi`` (holmes_mac.cu:116-274, 359-402) is compared with the oracle's MAC and with
  libholmes_cuda's same-signature drop-in.
"""
import ctypes
import os

import numpy as np
import pytest
import torch

from tests.gpu_helpers import dev, host, make_pair, residues

pytestmark = pytest.mark.gpu

REF = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle", "_ref")
K_MAX64 = 9223372036854775295  # Encode.cu MAX_64BIT_VALUE (holmes_encode.cu:14)


def _ref(name):
    path = os.path.join(REF, name)
    if not os.path.exists(path):
        pytest.skip(f"{path} not built (make -C oracle ref)")
    return ctypes.CDLL(path)


@pytest.fixture(scope="module")
def big():
    o, client, ctx = make_pair(log_n=16, limbs=3, dnum=1, dcrt=59, first=60, special=60, K=1, hamming=0)
    yield o, client, ctx
    ctx.close()


def _root_tables(o, limbs):
    """power_of_roots / power_of_roots_shoup in the reference layout [limbs][N] (separate arrays)."""
    roots = np.stack([o.roots[i] for i in range(limbs)])
    shoup = np.stack([np.array([(int(w) << 64) // o.pr.q[i] for w in o.roots[i]], dtype=np.uint64)
                      for i in range(limbs)])
    return roots, shoup


def test_reference_encode_stage2_pins_oracle_and_engine(big):
    o, _, ctx = big
    lib = _ref("libholmes_encode_ref.so")
    p = ctypes.c_void_p
    lib.holmes_encode_stage2.argtypes = [p, p, ctypes.c_longlong, ctypes.c_int, ctypes.c_double, ctypes.c_int, p, p, p,
                                         p, p, p, p, ctypes.c_int, ctypes.c_int, ctypes.c_int]
    lib.holmes_encode_stage2.restype = ctypes.c_int
    n, limbs, rows = o.pr.n, 3, 2
    rng = np.random.default_rng(1)
    vals = rng.normal(scale=3.0, size=(rows, n))
    vals[0, :8] = [0.0, -0.0, 0.5, -0.5, 1.5, -2.5, 1e-12, -1e-12]
    sf = float(2.0 ** 50)
    q = [o.pr.q[i] for i in range(limbs)]
    diffs = np.array([K_MAX64 % qi for qi in q], dtype=np.uint64)
    ks = np.array([qi.bit_length() - 1 + 63 for qi in q], dtype=np.uint64)
    ratios = np.array([(1 << int(k)) // qi for k, qi in zip(ks, q)], dtype=np.uint64)
    roots, shoup = _root_tables(o, limbs)
    d_in = dev(vals)
    d_out = torch.empty((rows, limbs, n), dtype=torch.uint64, device="cuda")
    tabs = [dev(np.array(q, dtype=np.uint64)), dev(diffs), dev(ratios), dev(ks), dev(roots), dev(shoup)]
    rc = lib.holmes_encode_stage2(d_out.data_ptr(), d_in.data_ptr(), n, rows, sf, limbs,
                                  *[t.data_ptr() for t in tabs], 0, 0, 3, 0)
    assert rc == 0
    ref_out = host(d_out)
    # oracle: coefficient n < N/2 is in[2n], n >= N/2 is in[2(n - N/2) + 1], llround(v sf), reduce, NTT
    for r in range(rows):
        coeff = np.empty(n, dtype=np.int64)
        half = n // 2
        re = vals[r, 0::2] * sf
        im = vals[r, 1::2] * sf
        coeff[:half] = np.array([_llround(v) for v in re], dtype=np.int64)
        coeff[half:] = np.array([_llround(v) for v in im], dtype=np.int64)
        expect = o.ntt(o.reduce_signed(coeff, range(limbs)), range(limbs))
        np.testing.assert_array_equal(ref_out[r], expect)
    # engine: the same doubles through holmes_encode_fft (rounding + NTT of already transformed slots)
    from holmes_b200 import _lib as L

    eng = torch.empty((rows, limbs, n), dtype=torch.uint64, device="cuda")
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    L.call("holmes_encode_fft", ctx.handle, d_in.data_ptr(), n, rows, n // 2, sf, limbs, eng.data_ptr(), limbs * n,
           flag.data_ptr(), 0)
    np.testing.assert_array_equal(host(eng), ref_out)
    assert int(flag.item()) == 0


def _llround(v: float) -> int:
    """C llround: round half away from zero.  abs(v) - floor(abs(v)) is exact, so no double rounding
    (floor(abs(v) + 0.5) would round ties to even for odd integers in [2^52, 2^53))."""
    import math

    a = abs(float(v))
    f = math.floor(a)
    r = int(f) + (1 if a - f >= 0.5 else 0)
    return r if v >= 0 else -r


def test_reference_mac_multi_pins_oracle_and_engine(big):
    o, _, ctx = big
    lib = _ref("libholmes_mac_ref.so")
    p, i, ll = ctypes.c_void_p, ctypes.c_int, ctypes.c_longlong
    lib.holmes_mac_multi.argtypes = [p, p, p, ll, i, i, p, ll, i, i, i, p, p, p, p]
    lib.holmes_mac_multi.restype = i
    n, limbs, nb, groups, inputs = o.pr.n, 2, 8, 2, 3
    rng = np.random.default_rng(2)
    q = [o.pr.q[k] for k in range(limbs)]
    pts = np.stack([residues(q, limbs, n, rng) for _ in range(groups * nb)])
    babies = [[(residues(q, limbs, n, rng), residues(q, limbs, n, rng)) for _ in range(nb)] for _ in range(inputs)]
    store = [[dev(np.stack([b[c] for b in babies[k]])) for c in range(2)] for k in range(inputs)]
    d_pts = dev(pts)
    ks = np.array([qq.bit_length() - 1 + 63 for qq in q], dtype=np.uint64)
    ratios = np.array([(1 << int(k)) // qq for k, qq in zip(ks, q)], dtype=np.uint64)
    tabs = [dev(np.array(q, dtype=np.uint64)), dev(ratios), dev(ks)]
    from holmes_b200 import _lib as L

    c0s = L.ptr_array([s[0].data_ptr() for s in store])
    c1s = L.ptr_array([s[1].data_ptr() for s in store])
    outs = {}
    for who, fn in (("ref", lib.holmes_mac_multi), ("engine", L.load().holmes_mac_multi)):
        for ti in (10108, 408):
            res = torch.zeros((2, groups, inputs, limbs, n), dtype=torch.uint64, device="cuda")
            rc = fn(res.data_ptr(), c0s, c1s, limbs * n, nb, inputs, d_pts.data_ptr(), limbs * n, groups, ti, limbs,
                    *[t.data_ptr() for t in tabs], None)
            assert rc == 0, (who, ti, rc)
            outs[(who, ti)] = host(res)
    for k in range(inputs):
        e = o.bsgs_mac(pts, babies[k], groups)
        for c in range(2):
            for key, got in outs.items():
                np.testing.assert_array_equal(got[c, :, k], e[c], err_msg=str(key))
    # argument errors follow the reference's codes
    bad = L.load().holmes_mac_multi(None, c0s, c1s, 0, nb, 33, None, 0, groups, 10108, limbs, None, None, None, None)
    assert bad == -1
    assert L.load().holmes_mac_multi(None, c0s, c1s, 0, 0, 1, None, 0, groups, 10108, limbs, None, None, None,
                                     None) == -2
    assert L.load().holmes_mac_multi(None, c0s, c1s, 0, nb, 1, None, 0, 16, 10108, limbs, None, None, None,
                                     None) == -3
    assert L.load().holmes_mac_multi(None, c0s, c1s, 0, nb, 1, None, 0, 2, 7, limbs, None, None, None, None) == -4
