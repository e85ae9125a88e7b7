"""Extended-basis primitives of the attention transforms (operators/attention/prefill/input.py:1007-1031,
1198-1236): fast_rotate(output_ext=True), grouped_pairwise_mac over Q u P, moddown_from_ext; residue for residue
against the oracle, ModDown of an extended rotation equal to the plain rotation, decoded against NumPy."""
import numpy as np
import pytest

from tests.gpu_helpers import host, make_pair

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def pair():
    o, client, ctx = make_pair(log_n=11, limbs=5, dnum=2, dcrt=45, first=50, special=55, hamming=32)
    yield o, client, ctx
    ctx.close()


def test_ext_rotations_match_oracle_and_moddown_to_rotations(pair):
    o, client, ctx = pair
    from holmes_b200 import fhe as F

    z = np.random.default_rng(1).normal(size=ctx.max_slots) * 0.5
    ct = client.encrypt(z, cur_limbs=4, counter=3)
    ref = o.encrypt(z, 4, counter=3)
    offsets = (3, 0, -5, 2 * ctx.N - 1)
    ext = F.fast_rotate(ct, offsets, ctx, output_ext=True)
    assert ext.is_ext and ext.batch_size == len(offsets) and int(ext.cv[0].shape[1]) == 4 + ctx.K
    down = F.moddown_from_ext(ext, ctx)
    for b, r in enumerate(offsets):
        e0, e1 = o.rotate_ext(ref, r)
        np.testing.assert_array_equal(host(ext.cv[0][b]), e0)
        np.testing.assert_array_equal(host(ext.cv[1][b]), e1)
        plain = F.homo_rotate(ct, r, ctx) if r else ct
        np.testing.assert_array_equal(host(down.cv[0][b]), host(plain.cv[0][0, :4]))
        np.testing.assert_array_equal(host(down.cv[1][b]), host(plain.cv[1][0, :4]))


def test_grouped_pairwise_mac_ext_matches_oracle_and_decodes(pair):
    o, client, ctx = pair
    from holmes_b200 import fhe as F
    from holmes_b200 import linear as LN

    session = LN.Session(client, ctx)
    rng = np.random.default_rng(2)
    z = rng.normal(size=ctx.max_slots) * 0.5
    cur = 4
    ct = client.encrypt(z, cur_limbs=cur, counter=5)
    ref = o.encrypt(z, cur, counter=5)
    offsets = (0, 1, 7)
    w = rng.normal(size=(len(offsets), ctx.max_slots)) * 0.3
    ext = F.fast_rotate(ct, offsets, ctx, output_ext=True)
    level = ctx.L - cur
    pts = [session.plaintext(w[b], name=f"t{b}", level=level, is_ext=True) for b in range(len(offsets))]
    stacked = F.Plaintext([F.torch.cat([p.cv[0] for p in pts])], pts[0].state, pts[0].slots, True, len(pts), ctx)
    prod = F.grouped_pairwise_mac(ext, stacked, 1, ctx)
    assert prod.is_ext and prod.batch_size == 1
    out = F.rescale(F.moddown_from_ext(prod, ctx), ctx)
    # oracle: sum_b pt_ext[b] * rot_ext[b] over Q u P, ModDown, rescale
    ids = o.ext_ids(cur)
    acc = None
    for b, r in enumerate(offsets):
        e0, e1 = o.rotate_ext(ref, r)
        pt = o.encode_ext(w[b], cur, ctx.scale)
        t = (o.mul(e0, pt, ids), o.mul(e1, pt, ids))
        acc = t if acc is None else (o.add(acc[0], t[0], ids), o.add(acc[1], t[1], ids))
    d0, d1 = o.rescale((o.moddown(acc[0], cur), o.moddown(acc[1], cur)))
    np.testing.assert_array_equal(host(out.cv[0][0, :cur - 1]), d0)
    np.testing.assert_array_equal(host(out.cv[1][0, :cur - 1]), d1)
    want = sum(np.roll(z, -r) * w[b] for b, r in enumerate(offsets))
    assert np.abs(client.decrypt(out).real - want).max() < 1e-4


def test_grouped_pairwise_mac_plain_groups(pair):
    o, client, ctx = pair
    from holmes_b200 import fhe as F

    rng = np.random.default_rng(3)
    cur = 3
    zs = [rng.normal(size=ctx.max_slots) * 0.5 for _ in range(2)]
    cts = [client.encrypt(z, cur_limbs=cur, counter=40 + i) for i, z in enumerate(zs)]
    batch = F.pack_cipher_batch(cts)
    w = rng.normal(size=(4, ctx.max_slots)) * 0.3      # 2 groups x 2 ciphertexts
    pv = F.encode_rows(ctx, F.torch.from_numpy(w.astype(np.complex128)), cur, ctx.scale, ctx.max_slots)
    pts = F.Plaintext([pv], F.CipherState(cur, 1, ctx.scale), ctx.max_slots, False, 4, ctx)
    prod = F.grouped_pairwise_mac(batch, pts, 2, ctx)
    assert prod.batch_size == 2 and not prod.is_ext
    for g in range(2):
        want = w[2 * g] * zs[0] + w[2 * g + 1] * zs[1]
        got = client.decrypt(prod.cipher_like([prod.cv[0][g:g + 1], prod.cv[1][g:g + 1]], batch_size=1)).real
        assert np.abs(got - want).max() < 1e-3
