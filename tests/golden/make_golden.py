"""Generate the golden fixtures in this folder by running the reference's own Python.

Run once, in a checkout that has the reference tree available (it is *not* needed afterwards: the
fixtures are committed and the tests only read them):

    python tests/golden/make_golden.py /path/to/holmes

The reference's ``llama3fhe`` imports EasyFHE at module scope; EasyFHE is a compiled package that
is not distributed with the reference, so a stub module stands in for it here.  None of the code
paths exercised below touch the stub: they are the reference's pure-NumPy / pure-Python parts
of the linear hot path --

* ``llama3fhe/operators/linear/weight.py:122-154`` ``_cpu_packer`` (diagonal rows of a chunk);
* ``llama3fhe/layouts/shifted_lane.py:177-268`` ``diagonal_plaintext`` / ``bsgs_matvec`` /
  ``shifted_lane_linear`` (BSGS plaintext semantics and the decoded-value oracle);
* ``llama3fhe/operators/linear/config.py:150-380`` ``LinearPlan`` geometry and
  ``linear_rotations`` key sets;
* ``llama3fhe/parallel/prefill/keys.py:91-118`` rotation normalisation and key sizes;
* ``llama3fhe/layouts/feature_major.py:10-120`` feature-major packing.
"""
from __future__ import annotations

import importlib.abc
import importlib.machinery
import json
import os
import sys
import types
from unittest import mock

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


class _StubFinder(importlib.abc.MetaPathFinder, importlib.abc.Loader):
    """Every ``easyfhe`` / ``sylph_easy`` import resolves to an inert mock module."""

    ROOTS = ("easyfhe", "sylph_easy", "triton")

    def find_spec(self, fullname, path, target=None):
        if fullname.split(".")[0] in self.ROOTS:
            return importlib.machinery.ModuleSpec(fullname, self, is_package=True)
        return None

    def create_module(self, spec):
        module = mock.MagicMock(name=spec.name)
        module.__path__ = []
        module.__spec__ = spec
        return module

    def exec_module(self, module):
        return None


def main(reference_root: str) -> None:
    sys.meta_path.insert(0, _StubFinder())
    sys.path.insert(0, reference_root)
    from llama3fhe.layouts import shifted_lane as sl
    from llama3fhe.layouts.feature_major import FeatureMajorPrefillLayout
    from llama3fhe.operators.linear import weight as weight_mod
    from llama3fhe.operators.linear.config import LinearOperatorConfig, linear_rotations
    from llama3fhe.parallel.prefill.keys import normalize_rotation, rotation_key_bytes

    rng = np.random.default_rng(20260101)
    arrays: dict[str, np.ndarray] = {}
    meta: dict[str, object] = {}

    # ---- diagonal packing (_cpu_packer), lane-replicated and shifted-lane, real and complex weights
    class _Ctx:
        tensor = types.SimpleNamespace(from_numpy=lambda a: a)
        device = "cpu"

    packer_cases = []
    for name, dim, lanes, baby, rows, lane_shift, cplx in (
        ("lr_real", 64, 4, 8, 32, 0, False),
        ("lr_complex", 32, 8, 4, 16, 0, True),
        ("sl_real", 64, 4, 4, 8, 16, False),
    ):
        cfg = LinearOperatorConfig(baby_steps=baby, baby_anchor_step=baby if baby >= 2 else -1,
                                   max_plaintext_rows=rows, lane_shift=lane_shift)
        plan = cfg.plan(dimension=dim, token_lanes=lanes)
        w = rng.normal(scale=0.02, size=(dim, dim))
        if cplx:
            w = w + 1j * rng.normal(scale=0.02, size=(dim, dim))
        arrays[f"pack_{name}_weight"] = w
        for chunk in plan.chunks:
            rows_out = weight_mod._cpu_packer(w, plan=plan, chunk=chunk, slots=dim * lanes,
                                              dtype=w.dtype, crypto_context=_Ctx())
            arrays[f"pack_{name}_chunk{chunk.index}"] = np.asarray(rows_out)
        packer_cases.append({
            "name": name, "dimension": dim, "token_lanes": lanes, "baby_steps": baby,
            "max_plaintext_rows": rows, "lane_shift": lane_shift, "complex": cplx,
            "chunks": [[c.index, c.giant_base, c.giant_count] for c in plan.chunks],
        })
    meta["packer_cases"] = packer_cases

    # ---- BSGS decoded-value oracle (shifted_lane.bsgs_matvec / shifted_lane_linear)
    bsgs_cases = []
    for name, hidden, slots, baby, lane_shift_mode in (
        ("lr", 32, 256, 4, "lr"),
        ("sl", 32, 256, 2, "sl"),
    ):
        layout = sl.ShiftedLaneLayout(hidden_dim=hidden, slots=slots)
        w = rng.normal(scale=0.02, size=(hidden, hidden))
        carrier = rng.normal(size=slots)
        shift = 0 if lane_shift_mode == "lr" else layout.shift
        out = sl.bsgs_matvec(w, carrier, layout=layout, baby_steps=baby, lane_shift=shift)
        arrays[f"bsgs_{name}_weight"] = w
        arrays[f"bsgs_{name}_carrier"] = carrier
        arrays[f"bsgs_{name}_out"] = np.asarray(out)
        rows = [sl.diagonal_plaintext(w, layout=layout, baby=b, giant=g, baby_steps=baby, lane_shift=shift)
                for g in range((hidden if shift == 0 else shift) // baby) for b in range(baby)]
        arrays[f"bsgs_{name}_rows"] = np.asarray(rows)
        bsgs_cases.append({"name": name, "hidden": hidden, "slots": slots, "baby": baby, "lane_shift": shift})
        if lane_shift_mode == "sl":
            x = rng.normal(size=hidden)
            arrays["sl_linear_x"] = x
            arrays["sl_linear_out"] = np.asarray(sl.shifted_lane_linear(w, x, layout=layout, baby_steps=baby))
    meta["bsgs_cases"] = bsgs_cases

    # ---- plan geometry and exact rotation-key sets
    plans = []
    for dim, lanes, baby, anchor, rows, strategy, lane_shift in (
        (4096, 8, 64, 64, 512, "normal", 0),
        (4096, 8, 32, 32, 512, "normal", 0),
        (4096, 8, 32, 32, 512, "ext_double_hoist", 0),
        (4096, 8, 128, 64, 512, "normal", 0),
        (4096, 8, 128, 64, 512, "ext_double_hoist", 0),
        (4096, 1, 64, 64, 512, "normal", 0),
        (4096, 8, 16, 16, 512, "normal", 512),
        (256, 8, 16, 16, 64, "normal", 0),
        (64, 128, 8, -1, 64, "normal", 0),
    ):
        cfg = LinearOperatorConfig(baby_steps=baby, baby_anchor_step=anchor, max_plaintext_rows=rows,
                                   hoist_strategy=strategy, lane_shift=lane_shift)
        plan = cfg.plan(dimension=dim, token_lanes=lanes)
        slots = dim * lanes if lane_shift == 0 else dim * lanes
        plans.append({
            "dimension": dim, "token_lanes": lanes, "baby_steps": baby, "baby_anchor_step": anchor,
            "max_plaintext_rows": rows, "hoist_strategy": strategy, "lane_shift": lane_shift,
            "giant_steps": plan.giant_steps, "chunk_giants": plan.chunk_giants,
            "giant_offset": plan.giant_offset, "baby_offsets": list(plan.baby_offsets),
            "chunks": [[c.index, c.giant_base, c.giant_count] for c in plan.chunks],
            "baby_key_offsets": list(plan.baby_key_offsets),
            "baby_blocks": [[b.start, b.width] for b in plan.baby_blocks],
            "fold_offsets": list(plan.fold_offsets), "lane_expand_offsets": list(plan.lane_expand_offsets),
            "rotations": list(linear_rotations(dimension=dim, token_lanes=lanes, operator_config=cfg)),
            "rotations_conj": list(linear_rotations(dimension=dim, token_lanes=lanes, slots=slots // 1,
                                                    include_conjugation=True, operator_config=cfg)),
        })
    meta["plans"] = plans
    meta["normalize_rotation"] = [[r, 65536, normalize_rotation(r, ring_dim=65536)] for r in (-1, -512, 0, 7, 32767)]
    meta["rotation_key_bytes"] = [[n, l, a, k, rotation_key_bytes(ring_dim=n, limbs=l, alpha=a, special_limbs=k)]
                                  for n, l, a, k in ((65536, 38, 8, 8), (65536, 13, 8, 8), (65536, 36, 12, 12),
                                                     (8192, 8, 4, 4))]

    # ---- feature-major packing
    fm = FeatureMajorPrefillLayout(seq_len=12, hidden_dim=16, slots=64)
    rows = rng.normal(size=(12, 16))
    arrays["fm_rows"] = rows
    arrays["fm_packed"] = fm.pack(rows)
    meta["fm"] = {"seq_len": 12, "hidden_dim": 16, "slots": 64, "cipher_count": fm.cipher_count}

    np.savez_compressed(os.path.join(HERE, "linear_golden.npz"), **arrays)
    with open(os.path.join(HERE, "linear_golden.json"), "w", encoding="utf-8") as f:
        json.dump(meta, f, indent=1, sort_keys=True)
    print("wrote", len(arrays), "arrays")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("HOLMES_REFERENCE", "../holmes"))
