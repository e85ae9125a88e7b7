"""Residue-for-residue pins at the parameter sets the benchmark and BASELINE.json actually use.

* Production chain (``llama3fhe/parallel/presets.py:63-127``): N = 2^16, 38 limbs of 59/60-bit primes, dnum 5 ->
  alpha 8, K 8, sparse ternary secret (h = 192), rotation keys trimmed to the 13 limbs of the linear entry level
  (``llama3fhe/parallel/prefill/stations.py:190``; key tiers ``parallel/prefill/keys.py:118-140``).  Ciphertexts at 13
  limbs: one ``homo_rotate`` (positive and negative offsets, normalised as N/2 + r, ``keys.py:91-102``), one hoisted set
  of 4 baby offsets (one ModUp), a Horner giant chain of 8 giants with the production giant offset 512, one rescale
  and one relinearised product of two different ciphertexts.
* N = 2^16, ~50-bit primes, dnum 3 (36 limbs -> alpha = K = 12), residues uniform in [0, q_i)
  at L = 1, 13 and 36 active limbs: batched NTT / iNTT, rotation, plaintext x ciphertext product and rescale.

Every engine output is compared word for word with the CPU oracle on the same inputs and keys."""
import numpy as np
import pytest
import torch

from tests.gpu_helpers import dev, host, make_pair, residues

pytestmark = pytest.mark.gpu

PROD_CUR = 13
BABY = (0, 8, 16, 24)          # baby offsets b * lanes with 8 token lanes (operators/linear/config.py:256-263)
GIANT_OFFSET = 512             # 64 babies x 8 lanes


@pytest.fixture(scope="module")
def production():
    rots = (1, 513, -8, GIANT_OFFSET) + BABY[1:]
    o, client, ctx = make_pair(log_n=16, limbs=38, dnum=5, dcrt=59, first=60, special=60, K=8, hamming=192,
                               key_limits={r: PROD_CUR for r in rots})
    assert (ctx.L, ctx.K, ctx.alpha) == (38, 8, 8)
    assert ctx.moduli == o.pr.q
    yield o, client, ctx
    ctx.close()


def _enc(o, client, seed, counter):
    from holmes_b200 import fhe as F

    rng = np.random.default_rng(seed)
    z = (rng.normal(size=client.context.max_slots) + 1j * rng.normal(size=client.context.max_slots)) * 0.1
    ct = client.encrypt(z, cur_limbs=PROD_CUR, counter=counter)
    ref = o.encrypt(z, PROD_CUR, counter=counter)
    np.testing.assert_array_equal(host(ct.cv[0][0]), ref[0])
    np.testing.assert_array_equal(host(ct.cv[1][0]), ref[1])
    assert isinstance(ct, F.Cipher)
    return z, ct, ref


def _same(got, want):
    np.testing.assert_array_equal(host(got.cv[0][0]), want[0])
    np.testing.assert_array_equal(host(got.cv[1][0]), want[1])


@pytest.mark.parametrize("rotation", [513, -8])
def test_production_rotation(production, rotation):
    from holmes_b200 import fhe as F

    o, client, ctx = production
    z, ct, ref = _enc(o, client, 1, 101)
    got = F.homo_rotate(ct, rotation, ctx)
    _same(got, o.rotate(ref, rotation, cap=PROD_CUR))
    assert np.abs(client.decrypt(got) - np.roll(z, -rotation)).max() < 1e-7


def test_production_hoisted_babies(production):
    from holmes_b200 import fhe as F

    o, client, ctx = production
    _, ct, ref = _enc(o, client, 2, 102)
    (block,) = F.prepare_hoisted_baby_rotations(ct, BABY, ctx)
    want = o.hoisted_rotations(ref, BABY, cap=PROD_CUR)
    for b in range(len(BABY)):
        np.testing.assert_array_equal(host(block.cv[0][b]), want[b][0])
        np.testing.assert_array_equal(host(block.cv[1][b]), want[b][1])


def test_production_giant_horner_8(production):
    """Horner over 8 giant partials of 2 inputs (batched key switches with ``+ partial[g]`` fused into ModDown)."""
    from holmes_b200 import fhe as F

    o, _, ctx = production
    rng = np.random.default_rng(3)
    G, items = 8, 2
    part = np.stack([np.stack([np.stack([residues(o.pr.q, PROD_CUR, o.pr.n, rng) for _ in range(items)])
                               for _ in range(G)]) for _ in range(2)])        # [2][G][items][cur][N]
    a0, a1 = F.giant_horner(ctx, dev(part), GIANT_OFFSET)
    for i in range(items):
        w0, w1 = o.giant_horner((part[0, :, i], part[1, :, i]), GIANT_OFFSET, cap=PROD_CUR)
        np.testing.assert_array_equal(host(a0[i]), w0)
        np.testing.assert_array_equal(host(a1[i]), w1)


def test_production_rescale(production):
    from holmes_b200 import fhe as F

    o, client, ctx = production
    _, a, ra = _enc(o, client, 4, 104)
    _, b, rb = _enc(o, client, 5, 105)
    prod = F.homo_mul_relin(a, b, ctx)
    want = o.mul_relin(ra, rb)
    _same(prod, want)
    _same(F.rescale(prod, ctx), o.rescale(want))


def test_production_mul_relin_distinct_operands(production):
    """a * b with a != b: a wiring slip that read a's components in place of b's would show here (a square
    cannot tell the operands apart)."""
    from holmes_b200 import fhe as F

    o, client, ctx = production
    za, a, ra = _enc(o, client, 6, 106)
    zb, b, rb = _enc(o, client, 7, 107)
    ab = F.homo_mul_relin(a, b, ctx)
    ba = F.homo_mul_relin(b, a, ctx)
    _same(ab, o.mul_relin(ra, rb))
    _same(ba, o.mul_relin(rb, ra))
    dec = client.decrypt(F.rescale(ab, ctx))
    assert np.abs(dec - za * zb).max() < 1e-6


# ------------------------------------------------------------------------------------------ BASELINE config 2


@pytest.fixture(scope="module")
def config2():
    o, client, ctx = make_pair(log_n=16, limbs=36, dnum=3, dcrt=50, first=50, special=50, hamming=192)
    assert (ctx.alpha, ctx.K) == (12, 12)
    assert ctx.moduli == o.pr.q
    yield o, client, ctx
    ctx.close()


def _uniform_ct(o, limbs, rng):
    return residues(o.pr.q, limbs, o.pr.n, rng), residues(o.pr.q, limbs, o.pr.n, rng)


@pytest.mark.parametrize("limbs", [1, 13, 36])
def test_config2_ntt_batch(config2, limbs):
    from holmes_b200 import _lib

    o, _, ctx = config2
    rng = np.random.default_rng(limbs)
    items = 3
    a = np.stack([residues(o.pr.q, limbs, o.pr.n, rng) for _ in range(items)])
    t = dev(a)
    _lib.call("holmes_ntt", ctx.handle, t.data_ptr(), items, limbs, limbs * o.pr.n, 0, 0, 0)
    got = host(t)
    for i in range(items):
        np.testing.assert_array_equal(got[i], o.ntt(a[i], range(limbs)))
    _lib.call("holmes_ntt", ctx.handle, t.data_ptr(), items, limbs, limbs * o.pr.n, 0, 1, 0)
    np.testing.assert_array_equal(host(t), a)


@pytest.mark.parametrize("limbs", [1, 13, 36])
@pytest.mark.parametrize("rotation", [1, -(1 << 14)])
def test_config2_rotation(config2, limbs, rotation):
    """A batch of two ciphertexts with uniform limbs sharing one key: each equals the oracle's rotation."""
    from holmes_b200 import fhe as F

    o, _, ctx = config2
    rng = np.random.default_rng(100 + limbs)
    cts = [_uniform_ct(o, limbs, rng) for _ in range(2)]
    c0 = dev(np.stack([c[0] for c in cts]))
    c1 = dev(np.stack([c[1] for c in cts]))
    o0, o1 = torch.empty_like(c0), torch.empty_like(c1)
    F.rotate_batch(ctx, c0, c1, limbs, rotation, o0, o1)
    for i, ct in enumerate(cts):
        w0, w1 = o.rotate(ct, rotation)
        np.testing.assert_array_equal(host(o0[i]), w0)
        np.testing.assert_array_equal(host(o1[i]), w1)


@pytest.mark.parametrize("limbs", [1, 13, 36])
def test_config2_mul_pt_and_rescale(config2, limbs):
    from holmes_b200 import fhe as F

    o, _, ctx = config2
    rng = np.random.default_rng(200 + limbs)
    c0, c1 = _uniform_ct(o, limbs, rng)
    pt = residues(o.pr.q, limbs, o.pr.n, rng)
    ids = list(range(limbs))
    ct = F.Cipher([dev(c0[None]), dev(c1[None])], F.CipherState(limbs, 1, ctx.scale), ctx.max_slots, False, 1, ctx)
    p = F.Plaintext([dev(pt[None])], F.CipherState(limbs, 1, ctx.scale), ctx.max_slots, False, 1, ctx)
    got = F.homo_mul_pt(ct, p, ctx)
    w0, w1 = o.mul(c0, pt, ids), o.mul(c1, pt, ids)
    _same(got, (w0, w1))
    if limbs >= 2:
        _same(F.rescale(got, ctx), o.rescale((w0, w1)))
