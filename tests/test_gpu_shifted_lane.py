"""Shifted-lane decode linear on the GPU (mirrors the reference's tests/test_shifted_lane.py:100-152): lane-0
carrier -> SL form (hoisted batch rotation) -> linear over two chunk subsets summed before the rescale -> lane
fold -> lane-0 mask, decoded against W @ x at the reference's 1e-5 tolerance."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_shifted_lane_linear_matches_numpy_on_gpu():
    from holmes_b200 import fhe as F
    from holmes_b200 import linear as LN
    from holmes_b200.shifted_lane import (ShiftedLaneLayout, expand_lane0_to_shifted_lanes, fold_shifted_lanes,
                                          mask_lane0)

    dimension, lanes = 1024, 8  # 8192 slots (N = 2^14)
    config = LN.LinearOperatorConfig(baby_steps=16, baby_anchor_step=16, max_plaintext_rows=32,
                                     lane_shift=dimension // lanes)
    spec = F.CKKSContextSpec(depth=4, log_n=14, dnum=1, dcrt_bits=59, first_mod=60, seed=0, auto_load_keys=False)
    session = LN.create_session(spec)
    try:
        layout = ShiftedLaneLayout(hidden_dim=dimension, slots=8192)
        rng = np.random.default_rng(5)
        weight = rng.normal(scale=0.05, size=(dimension, dimension))
        x = rng.normal(scale=1.0, size=dimension)
        expected = weight @ x
        plan = config.plan(dimension=dimension, token_lanes=lanes)
        assert len(plan.chunks) == 4
        cipher = session.encrypt(layout.pack_lane0(x), level=0)
        with LN.LinearOperator(crypto_context=session, token_lanes=lanes, config=config) as op, \
                LN.LinearWeight(weight, dtype=np.float64, crypto_context=session) as prepared:
            sl_input = expand_lane0_to_shifted_lanes(cipher, plan=plan, crypto_context=session)
            assert layout.is_shifted_lane(session.decrypt(sl_input).real, atol=1e-6)
            part_a, _ = op.apply((sl_input,), prepared, chunk_indices=(0, 1), rescale=False)
            part_b, _ = op.apply((sl_input,), prepared, chunk_indices=(2, 3), rescale=False)
            summed = F.rescale(F.homo_add(part_a[0], part_b[0], session.context), session.context)
            folded = fold_shifted_lanes(summed, plan=plan, crypto_context=session)
            clean = mask_lane0(folded, plan=plan, crypto_context=session)
        got = session.decrypt(folded).real
        np.testing.assert_allclose(got[::lanes], expected, atol=1e-5, rtol=1e-5)
        masked = session.decrypt(clean).real
        np.testing.assert_allclose(masked[::lanes], expected, atol=1e-5, rtol=1e-5)
        assert np.abs(masked.reshape(dimension, lanes)[:, 1:]).max() < 1e-5
    finally:
        session.context.close()


def test_fast_rotate_batch_matches_single_rotations():
    from holmes_b200 import fhe as F
    from tests.gpu_helpers import host, make_pair

    _, client, ctx = make_pair(log_n=12, limbs=3, dnum=1, dcrt=50, first=50, special=50)
    try:
        z = np.random.default_rng(3).normal(size=ctx.max_slots)
        ct = client.encrypt(z, cur_limbs=3, counter=1)
        batch = F.fast_rotate(ct, (5, 0, -7), ctx)
        items = F.unpack_cipher_batch(batch)
        assert len(items) == 3
        for off, item in zip((5, 0, -7), items):
            single = F.homo_rotate(ct, off, ctx) if off else ct
            for c in range(2):
                np.testing.assert_array_equal(host(item.cv[c][0, :3]), host(single.cv[c][0, :3]))
        again = F.pack_cipher_batch(items)
        for c in range(2):
            np.testing.assert_array_equal(host(again.cv[c][:, :3]), host(batch.cv[c][:, :3]))
    finally:
        ctx.close()
