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


def _schedule(p):
    return LN.BsgsSchedule(babies=p["baby_steps"], anchor=p["baby_anchor_step"], chunk_rows=p["max_plaintext_rows"],
                           hoist=p["hoist_strategy"], lane_shift=p["lane_shift"])


def test_plan_geometry_matches_reference(plans):
    """The engine's own layout type gives the reference's LinearPlan geometry and key sets for every fixture."""
    for p in plans:
        sched = _schedule(p)
        lay = sched.layout(p["dimension"], p["token_lanes"])
        assert lay.giants == p["giant_steps"]
        assert lay.chunks[0].count == p["chunk_giants"]
        assert lay.giant_stride == p["giant_offset"]
        assert list(lay.baby_strides) == p["baby_offsets"]
        assert [[c.index, c.first, c.count] for c in lay.chunks] == p["chunks"]
        assert list(lay.baby_keys) == p["baby_key_offsets"]
        assert [list(b) for b in lay.blocks] == p["baby_blocks"]
        assert list(lay.fold_strides) == p["fold_offsets"]
        assert list(lay.expand_strides) == p["lane_expand_offsets"]
        assert list(sched.rotation_keys(p["dimension"], p["token_lanes"])) == p["rotations"]
        slots = p["dimension"] * p["token_lanes"]
        assert list(sched.rotation_keys(p["dimension"], p["token_lanes"], conjugation_slots=slots)) == \
            p["rotations_conj"]


@pytest.mark.parametrize(("strategy", "baby", "anchor", "expected"), [
    ("normal", 32, 32, 39), ("ext_normal", 32, 32, 39), ("ext_double_hoist", 32, 32, 53),
    ("normal", 64, 64, 71), ("ext_normal", 64, 64, 71), ("ext_double_hoist", 64, 64, 77),
    ("normal", 128, 64, 72), ("ext_normal", 128, 64, 72), ("ext_double_hoist", 128, 64, 74)])
def test_rotation_key_counts(strategy, baby, anchor, expected):
    sched = LN.BsgsSchedule(babies=baby, anchor=anchor, chunk_rows=512, hoist=strategy)
    assert len(sched.rotation_keys(4096, 8)) == expected


def test_production_schedule():
    sched = LN.PRODUCTION
    assert (sched.babies, sched.anchor, sched.chunk_rows, sched.hoist, sched.reuse_babies) == (64, 64, 512, "normal",
                                                                                              True)
    lay = sched.layout(4096, 8)
    assert lay.giant_stride == 512 and [c.count for c in lay.chunks] == [8] * 8


def test_reference_config_objects_are_read_by_name():
    """A reference-style LinearOperatorConfig (any object with its attribute names) becomes the same schedule."""
    import types

    ref = types.SimpleNamespace(baby_steps=16, baby_anchor_step=8, max_plaintext_rows=64, reuse_baby_rotations=False,
                                hoist_strategy="EXT_NORMAL", constant_cache_mode="plain", raw_weight_policy="host",
                                lane_shift=0)
    assert LN.BsgsSchedule.coerce(ref) == LN.BsgsSchedule(babies=16, anchor=8, chunk_rows=64, reuse_babies=False,
                                                          hoist="ext_normal", cache="plain", weight_on_device=False)
    assert LN.BsgsSchedule.coerce(None) == LN.BsgsSchedule()


@pytest.mark.parametrize("kwargs", [dict(babies=0), dict(anchor=1), dict(anchor=-2), dict(chunk_rows=8, babies=16),
                                    dict(hoist="fast"), dict(hoist="double"), dict(cache="all"), dict(lane_shift=-1)])
def test_schedule_validation(kwargs):
    with pytest.raises(ValueError):
        LN.BsgsSchedule(**kwargs)


def test_layout_validation():
    with pytest.raises(ValueError):
        LN.BsgsSchedule(babies=48).layout(4096, 8)
    with pytest.raises(ValueError):
        LN.BsgsSchedule(babies=16, lane_shift=100).layout(4096, 8)


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
