"""CUDA path vs the CPU oracle, residue for residue (bit-exact), through the C ABI.

Small rings (N = 2^10 .. 2^13, single-CTA NTT) and cluster rings (N = 2^14 .. 2^16, DSMEM NTT) are both
covered.  Decoded values are additionally checked against NumPy at the tolerances of the reference's own
GPU tests (tests/test_linear.py:280-340: 2e-8 relative to the weight scale)."""
import numpy as np
import pytest
import torch

from oracle import packing
from tests.gpu_helpers import dev, host, make_pair, residues

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def pair():
    o, client, ctx = make_pair(log_n=10, limbs=5, dnum=2, dcrt=40, first=50, special=50)
    yield o, client, ctx
    ctx.close()


def _lib():
    from holmes_b200 import _lib

    return _lib


def test_context_tables_match_oracle(pair):
    import ctypes

    o, _, ctx = pair
    assert ctx.moduli == o.pr.q
    ptr = ctypes.c_void_p()
    _lib().call("holmes_ctx_secret", ctx.handle, ctypes.byref(ptr))
    n = (ctx.L + ctx.K) * ctx.N
    buf = torch.empty(n, dtype=torch.uint64, device=ctx.device)
    torch.cuda.synchronize()
    _copy_ptr(ptr.value, buf, n * 8)
    np.testing.assert_array_equal(host(buf).reshape(ctx.L + ctx.K, ctx.N), o.secret)


def _copy_ptr(src_ptr: int, dst: torch.Tensor, nbytes: int) -> None:
    import ctypes

    cudart = ctypes.CDLL("libcudart.so.12") if _has("libcudart.so.12") else ctypes.CDLL("libcudart.so")
    cudart.cudaMemcpy.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int]
    assert cudart.cudaMemcpy(ctypes.c_void_p(dst.data_ptr()), ctypes.c_void_p(src_ptr), nbytes, 3) == 0


def _has(name: str) -> bool:
    import ctypes

    try:
        ctypes.CDLL(name)
        return True
    except OSError:
        return False


@pytest.mark.parametrize("log_n", [10, 12, 13, 14, 15, 16])
def test_ntt_forward_inverse_bitexact(log_n):
    o, _, ctx = make_pair(log_n=log_n, limbs=3, dnum=1, dcrt=59, first=60, special=60, K=1)
    rng = np.random.default_rng(log_n)
    items, limbs = 3, 3
    a = np.stack([residues(o.pr.q, limbs, o.pr.n, rng) for _ in range(items)])
    t = dev(a)
    _lib().call("holmes_ntt", ctx.handle, t.data_ptr(), items, limbs, limbs * o.pr.n, 0, 0, 0)
    got = host(t)
    for i in range(items):
        np.testing.assert_array_equal(got[i], o.ntt(a[i], range(limbs)))
    _lib().call("holmes_ntt", ctx.handle, t.data_ptr(), items, limbs, limbs * o.pr.n, 0, 1, 0)
    np.testing.assert_array_equal(host(t), a)
    # special-prime moduli (index L .. L + K - 1)
    b = residues(o.pr.q, 1, o.pr.n, rng, limb_ids=[3])
    tb = dev(b)
    _lib().call("holmes_ntt", ctx.handle, tb.data_ptr(), 1, 1, o.pr.n, 3, 0, 0)
    np.testing.assert_array_equal(host(tb), o.ntt(b, [3]))
    ctx.close()


def test_keys_bitexact(pair):
    o, _, ctx = pair
    for galois, cap in ((5, ctx.L), (pow(5, 7, 2 * ctx.N), 3), (2 * ctx.N - 1, ctx.L), (0, ctx.L)):
        key = torch.empty(ctx.key_words(cap), dtype=torch.uint64, device=ctx.device)
        _lib().call("holmes_keygen", ctx.handle, galois, cap, key.data_ptr(), 0)
        kb, ka = o.relin_key(cap) if galois == 0 else o.rotation_key(galois, cap)
        got = host(key).reshape(2, *kb.shape)
        np.testing.assert_array_equal(got[1], ka)
        np.testing.assert_array_equal(got[0], kb)


def test_encrypt_bitexact_and_decrypts(pair):
    o, client, ctx = pair
    rng = np.random.default_rng(7)
    z = rng.normal(size=ctx.max_slots) + 1j * rng.normal(size=ctx.max_slots)
    for cur in (ctx.L, 2):
        ct = client.encrypt(z, cur_limbs=cur, counter=11)
        r0, r1 = o.encrypt(z, cur, counter=11)
        np.testing.assert_array_equal(host(ct.cv[0][0]), r0)
        np.testing.assert_array_equal(host(ct.cv[1][0]), r1)
        assert np.abs(client.decrypt(ct) - z).max() < 1e-6


@pytest.mark.parametrize("slots", [512, 64, 4])
def test_encode_bitexact(pair, slots):
    o, _, ctx = pair
    from holmes_b200 import fhe as F

    rng = np.random.default_rng(slots)
    rows = rng.normal(size=(3, slots)) + 1j * rng.normal(size=(3, slots))
    pt = F.encode_rows(ctx, torch.from_numpy(rows).to(ctx.device), 4, ctx.scale, slots)
    got = host(pt)
    for r in range(3):
        np.testing.assert_array_equal(got[r], o.encode(rows[r], 4, ctx.scale, slots))


@pytest.mark.parametrize("log_n,slots", [(12, 2048), (14, 1024)])
def test_encode_bitexact_production_width_primes(log_n, slots):
    """59/60-bit moduli take the encoder's direct signed load (8 q > 2^61); 2^14 runs the cluster NTT.  Values
    near the 2^61 limit (coefficients up to 2^60.8 of either sign) exercise the widest inputs."""
    o, _, ctx = make_pair(log_n=log_n, limbs=3, dnum=1, dcrt=59, first=60, special=60)
    try:
        from holmes_b200 import fhe as F

        rng = np.random.default_rng(log_n)
        rows = (rng.uniform(-1, 1, size=(2, slots)) + 1j * rng.uniform(-1, 1, size=(2, slots))) * 56.0
        rows[1] *= 2.0 ** -30
        pt = F.encode_rows(ctx, torch.from_numpy(rows).to(ctx.device), 3, ctx.scale, slots)
        ctx.check_encode_range()
        got = host(pt)
        for r in range(2):
            np.testing.assert_array_equal(got[r], o.encode(rows[r], 3, ctx.scale, slots))
    finally:
        ctx.close()


def test_encode_range_error_is_raised(pair):
    _, _, ctx = pair
    from holmes_b200 import fhe as F

    big = np.full((1, ctx.max_slots), 1e9, dtype=np.complex128)
    F.encode_rows(ctx, torch.from_numpy(big).to(ctx.device), 2, ctx.scale, ctx.max_slots)
    with pytest.raises(ValueError):
        ctx.check_encode_range()


def _cipher(o, client, z, cur, counter):
    ct = client.encrypt(z, cur_limbs=cur, counter=counter)
    return ct, o.encrypt(z, cur, counter=counter)


@pytest.mark.parametrize("cur", [5, 3, 1])
def test_rotation_and_conjugation_bitexact(pair, cur):
    o, client, ctx = pair
    from holmes_b200 import fhe as F

    rng = np.random.default_rng(cur)
    z = rng.normal(size=ctx.max_slots) * 0.5
    ct, ref = _cipher(o, client, z, cur, 3)
    for r in (1, 7, -5, ctx.max_slots - 1, 2 * ctx.N - 1):
        out = F.homo_rotate(ct, r, ctx)
        e0, e1 = o.rotate(ref, r)
        np.testing.assert_array_equal(host(out.cv[0][0]), e0)
        np.testing.assert_array_equal(host(out.cv[1][0]), e1)
    want = np.roll(z, -7)
    assert np.abs(client.decrypt(F.homo_rotate(ct, 7, ctx)) - want).max() < 1e-5


def test_modup_digit_reuse_follows_writes(pair):
    """Rotations of one ciphertext by several offsets share its ModUp digits; a torch in-place write to the
    ciphertext (version counter) and a raw write by rotate_batch into its memory both retire them."""
    o, client, ctx = pair
    from holmes_b200 import fhe as F

    rng = np.random.default_rng(41)
    ct, ref = _cipher(o, client, rng.normal(size=ctx.max_slots) * 0.5, 5, 21)
    other, ref2 = _cipher(o, client, rng.normal(size=ctx.max_slots) * 0.5, 5, 22)
    for r in (3, 5, 3):
        out = F.homo_rotate(ct, r, ctx)
        e0, e1 = o.rotate(ref, r)
        np.testing.assert_array_equal(host(out.cv[0][0]), e0)
        np.testing.assert_array_equal(host(out.cv[1][0]), e1)
    assert any(v[0] is ct.cv[1] for v in ctx._modup_cache.values())
    ct.cv[0].copy_(other.cv[0])
    ct.cv[1].copy_(other.cv[1])
    out = F.homo_rotate(ct, 3, ctx)
    e0, e1 = o.rotate(ref2, 3)
    np.testing.assert_array_equal(host(out.cv[0][0]), e0)
    np.testing.assert_array_equal(host(out.cv[1][0]), e1)
    F.rotate_batch(ctx, other.cv[0], other.cv[1], 5, 7, ct.cv[0], ct.cv[1])   # raw write into ct's memory
    out = F.homo_rotate(ct, 3, ctx)
    e0, e1 = o.rotate(o.rotate(ref2, 7), 3)
    np.testing.assert_array_equal(host(out.cv[0][0]), e0)
    np.testing.assert_array_equal(host(out.cv[1][0]), e1)


@pytest.mark.parametrize("dnum", [7, 3])
def test_rotation_bitexact_many_digits(dnum):
    """beta = ceil(cur / alpha) above the key-switch inner product's register-cached key counts (2 and 5): seven
    one-limb digits, and three digits of three limbs."""
    o, client, ctx = make_pair(log_n=11, limbs=7, dnum=dnum, dcrt=45, first=50, special=50, K=1 if dnum == 7 else 3)
    try:
        from holmes_b200 import fhe as F

        z = np.random.default_rng(dnum).normal(size=ctx.max_slots) * 0.5
        ct, ref = _cipher(o, client, z, 7, 9)
        for r in (3, 2 * ctx.N - 1):
            out = F.homo_rotate(ct, r, ctx)
            e0, e1 = o.rotate(ref, r)
            np.testing.assert_array_equal(host(out.cv[0][0]), e0)
            np.testing.assert_array_equal(host(out.cv[1][0]), e1)
    finally:
        ctx.close()


def test_hoisted_babies_bitexact(pair):
    o, client, ctx = pair
    from holmes_b200 import fhe as F

    z = np.random.default_rng(4).normal(size=ctx.max_slots)
    ct, ref = _cipher(o, client, z, 4, 5)
    offsets = [0, 3, 6, 9, 12]
    (block,) = F.prepare_hoisted_baby_rotations(ct, offsets, ctx)
    expect = o.hoisted_rotations(ref, offsets)
    for b in range(len(offsets)):
        np.testing.assert_array_equal(host(block.cv[0][b]), expect[b][0])
        np.testing.assert_array_equal(host(block.cv[1][b]), expect[b][1])


def test_elementwise_rescale_mul_i_relin_bitexact(pair):
    o, client, ctx = pair
    from holmes_b200 import fhe as F

    rng = np.random.default_rng(9)
    za = rng.normal(size=ctx.max_slots) * 0.5
    zb = rng.normal(size=ctx.max_slots) * 0.5
    a, ra = _cipher(o, client, za, 5, 21)
    b, rb = _cipher(o, client, zb, 5, 22)
    ids = range(5)
    s = F.homo_add(a, b, ctx)
    np.testing.assert_array_equal(host(s.cv[0][0]), o.add(ra[0], rb[0], ids))
    d = F.homo_sub(a, b, ctx)
    np.testing.assert_array_equal(host(d.cv[1][0]), o.sub(ra[1], rb[1], ids))
    mi = F.homo_mul_i(a, ctx)
    e = o.mul_i(ra)
    np.testing.assert_array_equal(host(mi.cv[0][0]), e[0])
    np.testing.assert_array_equal(host(mi.cv[1][0]), e[1])
    rs = F.rescale(a, ctx)
    e = o.rescale(ra)
    np.testing.assert_array_equal(host(rs.cv[0][0]), e[0])
    np.testing.assert_array_equal(host(rs.cv[1][0]), e[1])
    prod = F.homo_mul_relin(a, b, ctx)
    e = o.mul_relin(ra, rb)
    np.testing.assert_array_equal(host(prod.cv[0][0]), e[0])
    np.testing.assert_array_equal(host(prod.cv[1][0]), e[1])
    got = client.decrypt(F.rescale(prod, ctx))
    assert np.abs(got - za * zb).max() < 1e-4


@pytest.mark.parametrize("inputs,G,nb", [(3, 3, 5), (1, 8, 19), (1, 1, 9), (2, 9, 8), (5, 2, 17)])
def test_bsgs_mac_bitexact(pair, inputs, G, nb):
    """Every tile the MAC dispatches by input count (one, two, four inputs per block), with giant counts below, at
    and above the block's 8 and baby counts that leave a short last stage."""
    o, _, ctx = pair
    rng = np.random.default_rng(12 + inputs + G)
    cur = 4
    pts = np.stack([residues(o.pr.q, cur, o.pr.n, rng) for _ in range(G * nb)])
    babies = [[(residues(o.pr.q, cur, o.pr.n, rng), residues(o.pr.q, cur, o.pr.n, rng)) for _ in range(nb)]
              for _ in range(inputs)]
    from holmes_b200 import _lib as L

    store = [torch.stack([torch.stack([dev(b[c]) for b in babies[i]]) for c in range(2)]) for i in range(inputs)]
    res = torch.empty((2, G, inputs, cur, ctx.N), dtype=torch.uint64, device=ctx.device)
    pt = dev(pts)
    c0s = L.ptr_array([s[0].data_ptr() for s in store])
    c1s = L.ptr_array([s[1].data_ptr() for s in store])
    L.call("holmes_bsgs_mac", ctx.handle, res.data_ptr(), c0s, c1s, cur * ctx.N, nb, inputs, pt.data_ptr(),
           cur * ctx.N, G, cur, 0)
    got = host(res)
    for i in range(inputs):
        e = o.bsgs_mac(pts, babies[i], G)
        for c in range(2):
            np.testing.assert_array_equal(got[c, :, i], e[c])


def _oracle_linear(o, ref_inputs, weight, plan, cur, scale):
    """Per-input restatement of LinearOperator.apply (reference: operator.py:203-467)."""
    outs = []
    for ref in ref_inputs:
        babies = o.hoisted_rotations(ref, plan.baby_strides)
        acc = None
        for chunk in plan.chunks:
            rows = packing.diagonal_rows(weight, dimension=plan.dimension, token_lanes=plan.lanes,
                                         baby_steps=plan.babies, giant_base=chunk.first,
                                         giant_count=chunk.count, lane_shift=plan.lane_shift)
            pts = np.stack([o.encode(r, cur, scale) for r in rows])
            part = o.bsgs_mac(pts, babies, chunk.count)
            res = o.giant_horner(part, plan.giant_stride)
            if chunk.first:
                res = o.rotate(res, chunk.first * plan.giant_stride)
            acc = res if acc is None else (o.add(acc[0], res[0], range(cur)), o.add(acc[1], res[1], range(cur)))
        outs.append(o.rescale(acc))
    return outs


def _oracle_linear_ext(o, ref_inputs, weight, plan, cur, scale, double=False):
    """ext_normal restatement: babies and MAC over Q u P, one ModDown per giant partial, then the plain Horner.
    ``double`` (ext_double_hoist): every giant partial rotated by g giant_offset before its ModDown (giant 0 lifted
    as P times itself), the rotations summed over Q u P, one ModDown."""
    ids = o.ext_ids(cur)
    moduli = [o.pr.q[i] for i in ids]
    outs = []
    for ref in ref_inputs:
        babies = [o.rotate_ext(ref, r) for r in plan.baby_strides]
        acc = None
        for chunk in plan.chunks:
            rows = packing.diagonal_rows(weight, dimension=plan.dimension, token_lanes=plan.lanes,
                                         baby_steps=plan.babies, giant_base=chunk.first,
                                         giant_count=chunk.count, lane_shift=plan.lane_shift)
            pts = np.stack([o.encode_ext(r, cur, scale) for r in rows])
            part = o.bsgs_mac(pts, babies, chunk.count, moduli=moduli)
            down = [np.stack([o.moddown(part[c][g], cur) for g in range(chunk.count)]) for c in range(2)]
            if double:
                terms = [o.rotate_ext((down[0][g], down[1][g]), g * plan.giant_stride)
                         for g in range(chunk.count)]
                tot = terms[0]
                for t in terms[1:]:
                    tot = (o.add(tot[0], t[0], ids), o.add(tot[1], t[1], ids))
                res = (o.moddown(tot[0], cur), o.moddown(tot[1], cur))
            else:
                res = o.giant_horner(down, plan.giant_stride)
            if chunk.first:
                res = o.rotate(res, chunk.first * plan.giant_stride)
            acc = res if acc is None else (o.add(acc[0], res[0], range(cur)), o.add(acc[1], res[1], range(cur)))
        outs.append(o.rescale(acc))
    return outs


def test_linear_operator_ext_double_hoist_bitexact_and_decodes():
    """hoist_strategy "ext_double_hoist" (4 giants per chunk, each rotated with its own key over Q u P, one ModDown of
    their sum): residue for residue against its restatement, decoded like "normal"."""
    from holmes_b200 import linear as LN

    o, client, ctx = make_pair(log_n=11, limbs=4, dnum=2, dcrt=45, first=55, special=55)
    session = LN.Session(client, ctx)
    dim, lanes = 64, 16
    cfg = LN.BsgsSchedule(babies=8, anchor=8, chunk_rows=32,
                                  hoist="ext_double_hoist")
    plan = cfg.layout(dim, lanes)
    assert plan.chunks[0].count == 4
    rng = np.random.default_rng(17)
    w = rng.normal(scale=0.02, size=(dim, dim))
    xs = rng.normal(size=(2, lanes, dim))
    cur = ctx.L
    cts, refs = [], []
    for i, x in enumerate(xs):
        ct, ref = _cipher(o, client, x.T.reshape(-1), cur, 300 + i)
        cts.append(ct)
        refs.append(ref)
    from holmes_b200 import fhe as F

    with LN.LinearOperator(crypto_context=session, token_lanes=lanes, config=cfg) as op, \
            LN.LinearWeight(w, dtype=w.dtype, crypto_context=session) as lw:
        outs, _ = op.apply(cts, lw)
        # the single-input EasyFHE call takes the same path
        pts = lw.plaintext(plan, plan.chunks[1], level=0, schedule=cfg)
        one = F.hoisted_mac_sum(cts[0], plan.baby_strides, pts, plan.giant_stride, plan.chunks[1].count, ctx,
                                strategy="ext_double_hoist")
        assert int(one.state.cur_limbs) == cur and not one.is_ext
    expect = _oracle_linear_ext(o, refs, w, plan, cur, ctx.scale, double=True)
    for got, e, x in zip(outs, expect, xs):
        np.testing.assert_array_equal(host(got.cv[0][0]), e[0])
        np.testing.assert_array_equal(host(got.cv[1][0]), e[1])
        dec = client.decrypt(got).reshape(dim, lanes).T
        np.testing.assert_allclose(dec, x @ w.T, atol=2e-8 * 50, rtol=2e-6)
    ctx.close()


def test_linear_operator_ext_normal_bitexact_and_decodes():
    """hoist_strategy "ext_normal": the same page residue for residue against its restatement, decoded like
    "normal" (the ModDowns move, the rounding differs by noise only)."""
    from holmes_b200 import linear as LN

    o, client, ctx = make_pair(log_n=11, limbs=4, dnum=2, dcrt=45, first=55, special=55)
    session = LN.Session(client, ctx)
    dim, lanes = 64, 16
    cfg = LN.BsgsSchedule(babies=8, anchor=8, chunk_rows=16, hoist="ext_normal")
    plan = cfg.layout(dim, lanes)
    rng = np.random.default_rng(7)
    w = rng.normal(scale=0.02, size=(dim, dim))
    xs = rng.normal(size=(2, lanes, dim))
    cur = ctx.L
    cts, refs = [], []
    for i, x in enumerate(xs):
        ct, ref = _cipher(o, client, x.T.reshape(-1), cur, 200 + i)
        cts.append(ct)
        refs.append(ref)
    with LN.LinearOperator(crypto_context=session, token_lanes=lanes, config=cfg) as op, \
            LN.LinearWeight(w, dtype=w.dtype, crypto_context=session) as lw:
        outs, _ = op.apply(cts, lw)
    expect = _oracle_linear_ext(o, refs, w, plan, cur, ctx.scale)
    for got, e, x in zip(outs, expect, xs):
        np.testing.assert_array_equal(host(got.cv[0][0]), e[0])
        np.testing.assert_array_equal(host(got.cv[1][0]), e[1])
        dec = client.decrypt(got).reshape(dim, lanes).T
        np.testing.assert_allclose(dec, x @ w.T, atol=2e-8 * 50, rtol=2e-6)
    ctx.close()


@pytest.mark.parametrize("complex_weight", [False, True])
def test_linear_operator_bitexact_and_decodes(complex_weight):
    from holmes_b200 import linear as LN

    o, client, ctx = make_pair(log_n=11, limbs=4, dnum=2, dcrt=45, first=55, special=55)
    session = LN.Session(client, ctx)
    dim, lanes = 64, 16            # slots = 1024 = dim * lanes
    cfg = LN.BsgsSchedule(babies=8, anchor=8, chunk_rows=16)
    plan = cfg.layout(dim, lanes)
    rng = np.random.default_rng(26081431)
    w = rng.normal(scale=0.02, size=(dim, dim))
    if complex_weight:
        w = w + 1j * rng.normal(scale=0.02, size=(dim, dim))
    xs = rng.normal(size=(3, lanes, dim))
    cur = ctx.L
    cts, refs = [], []
    for i, x in enumerate(xs):
        carrier = x.T.reshape(-1)            # slot(d, t) = d * lanes + t
        ct, ref = _cipher(o, client, carrier, cur, 100 + i)
        cts.append(ct)
        refs.append(ref)
    with LN.LinearOperator(crypto_context=session, token_lanes=lanes, config=cfg) as op, \
            LN.LinearWeight(w, dtype=w.dtype, crypto_context=session) as lw:
        outs, profile = op.apply(cts, lw)
        again, _ = op.apply(cts, lw)
        assert op.cache_info()["baby_hits"] == 3
    expect = _oracle_linear(o, refs, w, plan, cur, ctx.scale)
    for got, e, x in zip(outs, expect, xs):
        np.testing.assert_array_equal(host(got.cv[0][0]), e[0])
        np.testing.assert_array_equal(host(got.cv[1][0]), e[1])
        dec = client.decrypt(got).reshape(dim, lanes).T
        np.testing.assert_allclose(dec, x @ w.T, atol=2e-8 * 50, rtol=2e-6)
    for a, b in zip(outs, again):
        np.testing.assert_array_equal(host(a.cv[0]), host(b.cv[0]))
    assert profile["online"] > 0
    # a pinned host page is uploaded on a side stream behind the babies: same residues
    pinned = torch.from_numpy(np.ascontiguousarray(w)).pin_memory()
    with LN.LinearOperator(crypto_context=session, token_lanes=lanes, config=cfg) as op, \
            LN.LinearWeight(pinned, dtype=w.dtype, crypto_context=session) as lw:
        via_host, _ = op.apply(cts, lw)
    for a, b in zip(outs, via_host):
        np.testing.assert_array_equal(host(a.cv[0]), host(b.cv[0]))
        np.testing.assert_array_equal(host(a.cv[1]), host(b.cv[1]))
    ctx.close()


def test_full_ring_rotation_round_trip_and_linearity():
    """N = 2^16 with 59/60-bit primes on a 13-limb chain with dnum 2 (alpha 7, K 7): rotation by r then -r and
    conjugation twice return the message; rotation is linear (size-independent properties).  The production chain
    itself (38 limbs, dnum 5, keys trimmed to 13 limbs) is pinned in tests/test_gpu_production_chain.py."""
    from holmes_b200 import fhe as F

    o, client, ctx = make_pair(log_n=16, limbs=13, dnum=2, dcrt=59, first=60, special=60, K=7, hamming=192)
    rng = np.random.default_rng(0)
    za = rng.normal(size=ctx.max_slots) * 0.1
    zb = rng.normal(size=ctx.max_slots) * 0.1
    a = client.encrypt(za, counter=1)
    b = client.encrypt(zb, counter=2)
    r = F.homo_rotate(F.homo_rotate(a, 513, ctx), -513, ctx)
    assert np.abs(client.decrypt(r) - za).max() < 1e-9
    c = F.homo_rotate(F.homo_rotate(a, 2 * ctx.N - 1, ctx), 2 * ctx.N - 1, ctx)
    assert np.abs(client.decrypt(c) - za).max() < 1e-9
    lhs = F.homo_rotate(F.homo_add(a, b, ctx), 4096, ctx)
    rhs = F.homo_add(F.homo_rotate(a, 4096, ctx), F.homo_rotate(b, 4096, ctx), ctx)
    assert np.abs(client.decrypt(lhs) - client.decrypt(rhs)).max() < 1e-9
    assert np.abs(client.decrypt(lhs) - np.roll(za + zb, -4096)).max() < 1e-9
    # one rotation against the oracle at full size
    ra = o.encrypt(za, ctx.L, counter=1)
    e0, e1 = o.rotate(ra, 513)
    g = F.homo_rotate(a, 513, ctx)
    np.testing.assert_array_equal(host(g.cv[0][0]), e0)
    np.testing.assert_array_equal(host(g.cv[1][0]), e1)
    ctx.close()


def test_reference_encode_stage2_abi_matches_encode():
    """holmes_encode_stage2 with the reference's signature (bench/cmp/kernels/holmes_encode.cu:240-285): the caller's
    primes / Barrett tables and psi^bitrev root tables, interleaved stage-1 doubles in; the same plaintexts as
    holmes_encode_fft (N = 2^16, full slots, values of both signs)."""
    from holmes_b200 import fhe as F

    o, _, ctx = make_pair(log_n=16, limbs=3, dnum=1, dcrt=59, first=60, special=60)
    try:
        n, limbs, rows = o.pr.n, 3, 2
        rng = np.random.default_rng(12)
        z = F.torch.from_numpy(rng.normal(size=(rows, n // 2)) + 1j * rng.normal(size=(rows, n // 2))).to(ctx.device)
        mid = F.fft_special_inv_rows(ctx, z, n // 2)
        want = F.encode_rows(ctx, mid, limbs, ctx.scale, n // 2, already_transformed=True)
        bits = o.pr.log_n
        rev = np.array([int(format(k, f"0{bits}b")[::-1], 2) for k in range(n)])
        roots = np.empty((limbs, n), dtype=np.uint64)
        shoup = np.empty((limbs, n), dtype=np.uint64)
        for li in range(limbs):
            q, psi = o.pr.q[li], o.pr.psi[li]
            pw = [1] * n
            for k in range(1, n):
                pw[k] = pw[k - 1] * psi % q
            r = [pw[int(rev[k])] for k in range(n)]
            roots[li] = np.array(r, dtype=np.uint64)
            shoup[li] = np.array([(v << 64) // q for v in r], dtype=np.uint64)
        rt, st = dev(roots), dev(shoup)
        out = F.torch.empty((rows, limbs, n), dtype=F.torch.uint64, device=ctx.device)
        zr = F.torch.view_as_real(mid)
        rc = _lib().load().holmes_encode_stage2(out.data_ptr(), zr.data_ptr(), n, rows, float(ctx.scale), limbs,
                                               ctx.primes.data_ptr(), 0, ctx.barret_ratio.data_ptr(),
                                               ctx.barret_k.data_ptr(), rt.data_ptr(), st.data_ptr(), 0, 0, 3, 0)
        assert rc == 0
        np.testing.assert_array_equal(host(out), host(want))
    finally:
        ctx.close()


@pytest.mark.parametrize("ti", [1, 2, 4])
def test_reference_mac_gather_abi(ti):
    """holmes_mac_gather with the reference's signature (bench/cmp/kernels/holmes_mac.cu:404-428): segmented rows of
    gathered (plaintext row, baby) pairs; exact against Python integers at sampled coefficients (a 20-row segment
    crosses the 16-row fold)."""
    import ctypes
    from holmes_b200 import fhe as F

    o, _, ctx = make_pair(log_n=16, limbs=2, dnum=1, dcrt=59, first=60, special=60)
    try:
        n, limbs, inputs, nb, npt = o.pr.n, 2, 3, 6, 10
        rng = np.random.default_rng(ti)
        babies = [np.stack([np.stack([residues(o.pr.q, limbs, n, rng) for _ in range(2)]) for _ in range(nb)])
                  for _ in range(inputs)]                                   # [nb][2][limbs][N] per input
        pts = np.stack([residues(o.pr.q, limbs, n, rng) for _ in range(npt)])   # [npt][limbs][N]
        seg = np.array([0, 4, 9, 29], dtype=np.int32)
        rows = int(seg[-1])
        idx = rng.integers(0, nb, rows).astype(np.int32)
        prow = rng.integers(0, npt, rows).astype(np.int32)
        K = len(seg) - 1
        bt = [dev(b) for b in babies]
        bstride = 2 * limbs * n
        c0s = F._lib.ptr_array([b[:, 0].data_ptr() for b in bt])
        c1s = F._lib.ptr_array([b[:, 1].data_ptr() for b in bt])
        pt_d, idx_d, prow_d, seg_d = dev(pts), dev(idx), dev(prow), dev(seg)
        res = F.torch.empty((2, K, inputs, limbs, n), dtype=F.torch.uint64, device=ctx.device)
        rc = _lib().load().holmes_mac_gather(res.data_ptr(), c0s, c1s, bstride, idx_d.data_ptr(), prow_d.data_ptr(),
                                             seg_d.data_ptr(), inputs, K, pt_d.data_ptr(), limbs * n, ti, limbs,
                                             ctx.primes.data_ptr(), ctx.barret_ratio.data_ptr(),
                                             ctx.barret_k.data_ptr(), 0)
        assert rc == 0
        got = host(res)
        for j in (0, 7, 40000, n - 1):
            for k in range(K):
                for i in range(inputs):
                    for c in range(2):
                        for l in range(limbs):
                            want = sum(int(pts[prow[r], l, j]) * int(babies[i][idx[r], c, l, j])
                                       for r in range(seg[k], seg[k + 1])) % o.pr.q[l]
                            assert int(got[c, k, i, l, j]) == want
    finally:
        ctx.close()


def test_composed_rotate_and_encode_entry_points():
    """holmes_rotate (ModUp and key switch in one C call, two ciphertexts) equals fhe.homo_rotate word for word, and
    holmes_encode_diag_rows (pack and encode in one C call) equals the linear operator's plaintexts for a chunk."""
    import ctypes

    from holmes_b200 import _lib as L
    from holmes_b200 import fhe as F
    from holmes_b200 import linear as LN

    o, client, ctx = make_pair(log_n=11, limbs=4, dnum=2, dcrt=45, first=55, special=55)
    try:
        rng = np.random.default_rng(33)
        cur, N = 3, ctx.N
        cts = [client.encrypt(rng.normal(size=ctx.max_slots) * 0.5, cur_limbs=cur, counter=70 + i) for i in range(2)]
        batch = F.pack_cipher_batch(cts)
        for r in (5, 2 * N - 1):
            g = ctx.galois(r)
            key, cap = ctx.switch_key(g, cur)
            words = ctypes.c_longlong()
            L.call("holmes_rotate_scratch_words", ctx.handle, cur, 2, ctypes.byref(words))
            scratch = torch.empty(words.value, dtype=torch.uint64, device=ctx.device)
            out = torch.empty((2, 2, cur, N), dtype=torch.uint64, device=ctx.device)
            L.call("holmes_rotate", ctx.handle, batch.cv[0].data_ptr(), batch.cv[1].data_ptr(),
                   int(batch.cv[0].stride(0)), cur, key.data_ptr(), cap, g, out[0].data_ptr(), out[1].data_ptr(),
                   cur * N, 2, scratch.data_ptr(), 0)
            for i, ct in enumerate(cts):
                want = F.homo_rotate(ct, r, ctx)
                for c in range(2):
                    np.testing.assert_array_equal(host(out[c, i]), host(want.cv[c][0]))
        # hoisted rotations (offsets 0, 3, 9): one ModUp, three keys
        offs = (0, 3, 9)
        gal = [ctx.galois(r) for r in offs]
        keys = [ctx.switch_key(g, cur) if g > 1 else (torch.empty(1, dtype=torch.uint64, device=ctx.device), 0)
                for g in gal]
        hout = torch.empty((2, len(offs), 2, cur, N), dtype=torch.uint64, device=ctx.device)
        kp = (ctypes.c_void_p * 3)(*[k[0].data_ptr() for k in keys])
        caps = (ctypes.c_int * 3)(*[k[1] for k in keys])
        gals = (ctypes.c_uint64 * 3)(*gal)
        L.call("holmes_hoisted_rotations", ctx.handle, batch.cv[0].data_ptr(), batch.cv[1].data_ptr(),
               int(batch.cv[0].stride(0)), cur, 2, 3, kp, caps, gals, hout[0].data_ptr(), hout[1].data_ptr(), cur * N,
               2 * cur * N, scratch.data_ptr(), 0)
        for b, r in enumerate(offs):
            for i, ct in enumerate(cts):
                want = F.homo_rotate(ct, r, ctx)
                for c in range(2):
                    np.testing.assert_array_equal(host(hout[c, b, i]), host(want.cv[c][0]))
        # relinearised product of the two ciphertexts with themselves (items 0, 1)
        rkey, rcap = ctx.switch_key(0, cur)
        ms = torch.empty(words.value + 4 * 2 * cur * N, dtype=torch.uint64, device=ctx.device)
        mout = torch.empty((2, 2, cur, N), dtype=torch.uint64, device=ctx.device)
        L.call("holmes_mul_relin", ctx.handle, batch.cv[0].data_ptr(), batch.cv[1].data_ptr(), batch.cv[0].data_ptr(),
               batch.cv[1].data_ptr(), int(batch.cv[0].stride(0)), cur, 2, rkey.data_ptr(), rcap, mout[0].data_ptr(),
               mout[1].data_ptr(), cur * N, ms.data_ptr(), 0)
        for i, ct in enumerate(cts):
            want = F.homo_mul_relin(ct, ct, ctx)
            for c in range(2):
                np.testing.assert_array_equal(host(mout[c, i]), host(want.cv[c][0]))
        # giant sum over 3 partials (the hoisted outputs) with offset 16: the Python Horner chain
        g16 = ctx.galois(16)
        key16, cap16 = ctx.switch_key(g16, cur)
        L.call("holmes_rotate_scratch_words", ctx.handle, cur, 2, ctypes.byref(words))
        gs = torch.empty(words.value + 2 * 2 * cur * N, dtype=torch.uint64, device=ctx.device)
        gout = torch.empty((2, 2, cur, N), dtype=torch.uint64, device=ctx.device)
        L.call("holmes_giant_sum", ctx.handle, hout[0].data_ptr(), hout[1].data_ptr(), cur * N, 2 * cur * N, cur, 2, 3,
               key16.data_ptr(), cap16, g16, gout[0].data_ptr(), gout[1].data_ptr(), cur * N, gs.data_ptr(), 0)
        h0, h1 = F.giant_horner(ctx, hout.clone(), 16)
        np.testing.assert_array_equal(host(gout[0]), host(h0))
        np.testing.assert_array_equal(host(gout[1]), host(h1))
        session = LN.Session(client, ctx)
        dim, lanes = 64, 16
        cfg = LN.BsgsSchedule(babies=8, anchor=8, chunk_rows=16)
        plan = cfg.layout(dim, lanes)
        w = rng.normal(scale=0.02, size=(dim, dim))
        chunk = plan.chunks[1]
        rows = chunk.count * plan.babies
        slots = int(session.max_slots)
        with LN.LinearWeight(w, dtype=w.dtype, crypto_context=session) as lw:
            want = lw.plaintext(plan, chunk, level=ctx.L - cur, schedule=cfg)
            wd = torch.from_numpy(w).to(ctx.device)
            out = torch.empty((rows, cur, N), dtype=torch.uint64, device=ctx.device)
            scratch = torch.empty((rows, slots, 2), dtype=torch.float64, device=ctx.device)
            flag = torch.zeros(1, dtype=torch.int32, device=ctx.device)
            L.call("holmes_encode_diag_rows", ctx.handle, wd.data_ptr(), 0, dim, lanes, plan.babies,
                   chunk.first, chunk.count, plan.lane_shift, slots, float(ctx.scale_at(cur)), cur,
                   out.data_ptr(), cur * N, scratch.data_ptr(), flag.data_ptr(), 0)
            np.testing.assert_array_equal(host(out), host(want.cv[0][:, :cur]))
            assert int(flag.item()) == 0
    finally:
        ctx.close()


@pytest.mark.parametrize("giants", [1, 2, 4])
def test_giant_sum_abi_giant_counts_and_mul_relin_distinct(giants):
    """holmes_giant_sum with an odd and even number of Horner steps (the ping-pong's two parities, and the single-giant
    copy) against fhe.giant_horner; holmes_mul_relin of two DIFFERENT ciphertext batches against fhe.homo_mul_relin;
    scratch sized by holmes_scratch_words."""
    import ctypes

    from holmes_b200 import _lib as L
    from holmes_b200 import fhe as F

    o, client, ctx = make_pair(log_n=11, limbs=4, dnum=2, dcrt=45, first=55, special=55)
    try:
        rng = np.random.default_rng(50 + giants)
        cur, N, items = 3, ctx.N, 2
        part = np.stack([np.stack([np.stack([residues(o.pr.q, cur, N, rng) for _ in range(items)])
                                   for _ in range(giants)]) for _ in range(2)])   # [2][G][items][cur][N]
        pd = dev(part)
        g16 = ctx.galois(16)
        key16, cap16 = ctx.switch_key(g16, cur)
        words = ctypes.c_longlong()
        L.call("holmes_scratch_words", ctx.handle, 1, cur, items, ctypes.byref(words))
        gs = torch.empty(words.value, dtype=torch.uint64, device=ctx.device)
        gout = torch.empty((2, items, cur, N), dtype=torch.uint64, device=ctx.device)
        L.call("holmes_giant_sum", ctx.handle, pd[0].data_ptr(), pd[1].data_ptr(), cur * N, items * cur * N, cur, items,
               giants, key16.data_ptr(), cap16, g16, gout[0].data_ptr(), gout[1].data_ptr(), cur * N, gs.data_ptr(), 0)
        h0, h1 = F.giant_horner(ctx, pd.clone(), 16)
        np.testing.assert_array_equal(host(gout[0]), host(h0))
        np.testing.assert_array_equal(host(gout[1]), host(h1))
        for i in range(items):
            w0, w1 = o.giant_horner((part[0, :, i], part[1, :, i]), 16)
            np.testing.assert_array_equal(host(gout[0, i]), w0)
            np.testing.assert_array_equal(host(gout[1, i]), w1)
        # relinearised products a_i * b_i of two different batches
        a = F.pack_cipher_batch([client.encrypt(rng.normal(size=ctx.max_slots) * 0.5, cur_limbs=cur, counter=90 + i)
                                 for i in range(items)])
        b = F.pack_cipher_batch([client.encrypt(rng.normal(size=ctx.max_slots) * 0.5, cur_limbs=cur, counter=95 + i)
                                 for i in range(items)])
        assert a.cv[0].stride(0) == b.cv[0].stride(0)
        rkey, rcap = ctx.switch_key(0, cur)
        L.call("holmes_scratch_words", ctx.handle, 2, cur, items, ctypes.byref(words))
        ms = torch.empty(words.value, dtype=torch.uint64, device=ctx.device)
        mout = torch.empty((2, items, cur, N), dtype=torch.uint64, device=ctx.device)
        L.call("holmes_mul_relin", ctx.handle, a.cv[0].data_ptr(), a.cv[1].data_ptr(), b.cv[0].data_ptr(),
               b.cv[1].data_ptr(), int(a.cv[0].stride(0)), cur, items, rkey.data_ptr(), rcap, mout[0].data_ptr(),
               mout[1].data_ptr(), cur * N, ms.data_ptr(), 0)
        want = F.homo_mul_relin(a, b, ctx)
        np.testing.assert_array_equal(host(mout[0]), host(want.cv[0]))
        np.testing.assert_array_equal(host(mout[1]), host(want.cv[1]))
        for i in range(items):
            ra = (host(a.cv[0][i]), host(a.cv[1][i]))
            rb = (host(b.cv[0][i]), host(b.cv[1][i]))
            w0, w1 = o.mul_relin(ra, rb)
            np.testing.assert_array_equal(host(mout[0, i]), w0)
            np.testing.assert_array_equal(host(mout[1, i]), w1)
        assert L.load().holmes_scratch_words(ctx.handle, 7, cur, items, ctypes.byref(words)) == -4
    finally:
        ctx.close()
