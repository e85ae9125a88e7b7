"""Shared set-up for the GPU parity tests: an engine context and an oracle with identical parameters."""
from __future__ import annotations

import numpy as np
import torch

from oracle.oracle import Oracle, OracleParams


def make_pair(log_n=10, limbs=4, dnum=2, dcrt=40, first=50, special=50, K=None, hamming=32, seed=0, scale_bits=None,
              key_limits=None):
    """``key_limits``: rotation -> the largest limb count its key serves (keys trimmed to that many Q limbs, as the
    reference's key tiers do, ``llama3fhe/parallel/prefill/keys.py:118-140``)."""
    from holmes_b200 import fhe as F

    op = OracleParams(log_n=log_n, limbs=limbs, dnum=dnum, dcrt_bits=dcrt, first_mod_bits=first, special_bits=special,
                      special_limbs=K, hamming=hamming, seed=seed, scale_bits=scale_bits)
    spec = F.CKKSContextSpec(depth=limbs - 1, log_n=log_n, dnum=dnum, dcrt_bits=dcrt, first_mod=first,
                             special_bits=special, special_limbs=K, hamming_weight=hamming, seed=seed,
                             scale_bits=scale_bits,
                             secret_key_dist="SPARSE_TERNARY" if hamming else "UNIFORM_TERNARY",
                             auto_load_keys=False, rotation_key_limb_limits=dict(key_limits or {}))
    client, ctx = F.generate_client_context(spec)
    return Oracle(op), client, ctx


def residues(ctx_or_oracle_q, rows: int, n: int, rng, limb_ids=None) -> np.ndarray:
    qs = list(ctx_or_oracle_q)
    ids = range(rows) if limb_ids is None else limb_ids
    return np.stack([rng.integers(0, qs[i], n, dtype=np.uint64) for i in ids]).astype(np.uint64)


def dev(a: np.ndarray, device="cuda") -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a)).to(device)


def host(t: torch.Tensor) -> np.ndarray:
    torch.cuda.synchronize()
    return t.cpu().numpy()
