"""Host-side logic without a GPU: the linear plan geometry and rotation-key sets against the reference's
own values (golden fixtures + the counts asserted in tests/test_linear.py:21-165 of the reference),
configuration validation, and the C ABI (library loads, every declared symbol is exported)."""
import ctypes
import json
import os
import re

import pytest

from holmes_b200 import linear as LN

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")


@pytest.fixture(scope="module")
def plans():
    with open(os.path.join(GOLDEN, "linear_golden.json"), encoding="utf-8") as f:
        return json.load(f)["plans"]


def test_plan_geometry_matches_reference(plans):
    for p in plans:
        cfg = LN.LinearOperatorConfig(baby_steps=p["baby_steps"], baby_anchor_step=p["baby_anchor_step"],
                                      max_plaintext_rows=p["max_plaintext_rows"], hoist_strategy=p["hoist_strategy"],
                                      lane_shift=p["lane_shift"])
        plan = cfg.plan(dimension=p["dimension"], token_lanes=p["token_lanes"])
        assert plan.giant_steps == p["giant_steps"]
        assert plan.chunk_giants == p["chunk_giants"]
        assert plan.giant_offset == p["giant_offset"]
        assert list(plan.baby_offsets) == p["baby_offsets"]
        assert [[c.index, c.giant_base, c.giant_count] for c in plan.chunks] == p["chunks"]
        assert list(plan.baby_key_offsets) == p["baby_key_offsets"]
        assert [[b.start, b.width] for b in plan.baby_blocks] == p["baby_blocks"]
        assert list(plan.fold_offsets) == p["fold_offsets"]
        assert list(plan.lane_expand_offsets) == p["lane_expand_offsets"]
        rot = LN.linear_rotations(dimension=p["dimension"], token_lanes=p["token_lanes"], operator_config=cfg)
        assert list(rot) == p["rotations"]
        slots = p["dimension"] * p["token_lanes"]
        rc = LN.linear_rotations(dimension=p["dimension"], token_lanes=p["token_lanes"], slots=slots,
                                 include_conjugation=True, operator_config=cfg)
        assert list(rc) == p["rotations_conj"]


@pytest.mark.parametrize(("strategy", "baby", "anchor", "expected"), [
    ("normal", 32, 32, 39), ("ext_normal", 32, 32, 39), ("ext_double_hoist", 32, 32, 53),
    ("normal", 64, 64, 71), ("ext_normal", 64, 64, 71), ("ext_double_hoist", 64, 64, 77),
    ("normal", 128, 64, 72), ("ext_normal", 128, 64, 72), ("ext_double_hoist", 128, 64, 74)])
def test_rotation_key_counts(strategy, baby, anchor, expected):
    cfg = LN.LinearOperatorConfig(baby_steps=baby, baby_anchor_step=anchor, max_plaintext_rows=512,
                                  hoist_strategy=strategy)
    assert len(LN.linear_rotations(dimension=4096, token_lanes=8, operator_config=cfg)) == expected


def test_production_schedule():
    for cfg in (LN.LLAMA3_LINEAR_SCHEDULES.qkv, LN.LLAMA3_LINEAR_SCHEDULES.w_o, LN.LLAMA3_LINEAR_SCHEDULES.gate_up,
                LN.LLAMA3_LINEAR_SCHEDULES.down):
        assert (cfg.baby_steps, cfg.baby_anchor_step, cfg.max_plaintext_rows) == (64, 64, 512)
        assert cfg.hoist_strategy == "normal" and cfg.reuse_baby_rotations
    plan = LN.LLAMA3_LINEAR_SCHEDULES.qkv.plan(dimension=4096, token_lanes=8)
    assert plan.giant_offset == 512 and plan.chunk_sizes == (8,) * 8 and plan.plaintext_chunks == 8


@pytest.mark.parametrize("kwargs", [dict(baby_steps=0), dict(baby_anchor_step=1), dict(baby_anchor_step=-2),
                                    dict(max_plaintext_rows=8, baby_steps=16), dict(hoist_strategy="fast"),
                                    dict(constant_cache_mode="all"), dict(raw_weight_policy="disk"),
                                    dict(lane_shift=-1), dict(encode_depth=-1)])
def test_config_validation(kwargs):
    with pytest.raises(ValueError):
        LN.LinearOperatorConfig(**kwargs)


def test_unknown_strategies_are_refused():
    """The config accepts the reference's three names and nothing else."""
    with pytest.raises(ValueError):
        LN.LinearOperatorConfig(hoist_strategy="double")


def test_plan_validation():
    with pytest.raises(ValueError):
        LN.LinearOperatorConfig(baby_steps=48).plan(dimension=4096, token_lanes=8)
    with pytest.raises(ValueError):
        LN.LinearOperatorConfig(baby_steps=16, lane_shift=100).plan(dimension=4096, token_lanes=8)
    with pytest.raises(ValueError):
        LN.linear_rotations(dimension=64, token_lanes=4, include_conjugation=True)


def test_rotation_normalisation_and_key_size_match_reference():
    with open(os.path.join(GOLDEN, "linear_golden.json"), encoding="utf-8") as f:
        meta = json.load(f)
    for r, n, norm in meta["normalize_rotation"]:
        assert (n // 2 + r if r < 0 else r) == norm
    for n, limbs, alpha, k, nbytes in meta["rotation_key_bytes"]:
        beta = -(-limbs // alpha)
        assert 2 * 8 * beta * (limbs + k) * n == nbytes


def _declared_symbols():
    with open(os.path.join(ROOT, "include", "holmes_cuda.h"), encoding="utf-8") as f:
        text = f.read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\bint\s+(holmes_\w+)\s*\(", text)))


def test_c_abi_exports_every_declared_symbol():
    from holmes_b200 import _lib

    lib = _lib.load()
    names = _declared_symbols()
    assert len(names) >= 20
    for name in names:
        assert hasattr(lib, name), name
        assert name in _lib.SIGNATURES, name
    # and the shared object exports them under C linkage (no mangling)
    raw = ctypes.CDLL(_lib.LIB_PATH)
    for name in names:
        getattr(raw, name)


def test_shifted_lane_layout_matches_golden_semantics():
    """Carrier layout (layouts/shifted_lane.py:41-175): pack, lane-0 pack, unpack per lane, expansion offsets."""
    import numpy as np
    from holmes_b200.shifted_lane import ShiftedLaneLayout, lane0_mask_vector

    lay = ShiftedLaneLayout(hidden_dim=64, slots=512)
    assert (lay.lanes, lay.shift) == (8, 8)
    x = np.arange(64, dtype=np.float64)
    sl = lay.pack(x)
    assert lay.is_shifted_lane(sl)
    for lane in range(8):
        np.testing.assert_array_equal(lay.unpack(sl, lane=lane), x)
    assert sl[lay.slot(3, 2)] == x[(3 + 8 * 2) % 64]
    lr = lay.pack_lane0(x)
    # rotating the lane-0 carrier by each expansion offset and adding builds the SL carrier
    built = lr.copy()
    for off in lay.lane0_to_shifted_offsets():
        built = built + np.roll(lr, -off)
    np.testing.assert_array_equal(built, sl)
    assert lay.fold_offsets() == (1, 2, 4)
    plan = LN.LinearOperatorConfig(baby_steps=16, lane_shift=128).plan(dimension=1024, token_lanes=8)
    mask = lane0_mask_vector(plan, slots=8192)
    assert mask.sum() == 1024 and mask[::8].all()
    assert plan.lane_expand_offsets == tuple(1023 * l for l in range(1, 8))
    with pytest.raises(ValueError):
        ShiftedLaneLayout(hidden_dim=48, slots=512)


def test_cipher_batch_pack_unpack_on_host_tensors():
    import torch
    from holmes_b200 import fhe as F

    st = F.CipherState(2, 1, 2.0 ** 40)
    a = F.Cipher([torch.zeros((1, 3, 8), dtype=torch.int64), torch.ones((1, 3, 8), dtype=torch.int64)], st, 4)
    b = F.Cipher([torch.full((1, 2, 8), 2, dtype=torch.int64), torch.full((1, 2, 8), 3, dtype=torch.int64)], st, 4)
    batch = F.pack_cipher_batch([a, b])
    assert batch.batch_size == 2 and tuple(batch.cv[0].shape) == (2, 2, 8)
    items = F.unpack_cipher_batch(batch)
    assert [int(i.cv[1][0, 0, 0]) for i in items] == [1, 3]
    with pytest.raises(ValueError):
        F.pack_cipher_batch([a, a.cipher_like(a.cv, state=F.CipherState(3, 1, 2.0 ** 40))])
