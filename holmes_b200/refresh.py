"""Pair refresh: two real ciphertexts through one bootstrap as ``left + i right``.

Mirrors the reference's residual-refresh helpers (``llama3fhe/operators/norm/refresh.py:21-60``) and the
station-level ``pair_bootstrap`` / ``halve`` (``llama3fhe/parallel/prefill/stations.py:102-190``): same names,
argument meaning and error behaviour, on this engine's primitives (``holmes_b200.fhe``) and bootstrap operator
(``holmes_b200.bootstrap.BootstrapOperator``).  Inputs are not consumed.
"""
from __future__ import annotations

from . import fhe


def _ctx_of(crypto_context):
    return getattr(crypto_context, "context", crypto_context)


def _half_rescale(cipher, *, crypto_context):
    """Public 0.5 multiplication with one rescale (``refresh.py:21-31``)."""
    ctx = _ctx_of(crypto_context)
    encoded = fhe.encode_scalar(0.5, cur_limbs=int(cipher.state.cur_limbs), scale_degree=1,
                                scaling_factor=float(ctx.q(int(cipher.state.cur_limbs) - 1)), context=ctx)
    out = fhe.homo_mul_scalar_rescale(cipher, encoded, ctx)
    out.state = out.state.replace(scaling_factor=cipher.state.scaling_factor)
    return out


def _pack_complex_pair(left, right, *, crypto_context):
    """Pack two real streams as ``left + i*right`` so one bootstrap serves both."""
    ctx = _ctx_of(crypto_context)
    return fhe.homo_add(left, fhe.homo_mul_i(right, ctx), ctx)


def _unpack_complex_pair(value, *, crypto_context):
    """Split a refreshed complex cipher into ``(2*real, 2*imaginary)`` with the conjugation (rotation index
    M - 1); the factor 2 is the caller's to undo (``_half_rescale``) or absorb."""
    ctx = _ctx_of(crypto_context)
    conjugated = fhe.homo_rotate(value, int(ctx.M) - 1, ctx)
    real_twice = fhe.homo_add(value, conjugated, ctx)
    imaginary_twice = fhe.homo_mul_i(fhe.homo_sub(conjugated, value, ctx), ctx)
    return real_twice, imaginary_twice


def pair_bootstrap(ciphers, *, context, bootstrap_operator, iterations: int = 1, precision_bits: int = 14,
                   synchronize: bool = True):
    """Refresh an even list of real ciphertexts two at a time via ``a + i*b``; returns ``(refreshed, 2.0)``.

    All pairs go through the operator's batched ``refresh_many`` when it has one (one C2S / EvalMod / S2C pass
    for the whole batch), else through ``refresh`` one pair at a time.
    """
    ciphers = tuple(ciphers)
    if len(ciphers) % 2:
        raise ValueError("pair_bootstrap needs an even number of ciphertexts")
    packed = [_pack_complex_pair(ciphers[k], ciphers[k + 1], crypto_context=context)
              for k in range(0, len(ciphers), 2)]
    many = getattr(bootstrap_operator, "refresh_many", None)
    kw = dict(iterations=int(iterations), precision_bits=int(precision_bits), synchronize=bool(synchronize))
    if many is not None:
        refreshed = list(many(packed, **kw))
    else:
        refreshed = [bootstrap_operator.refresh(p, **kw) for p in packed]
    out = []
    for r in refreshed:
        out.extend(_unpack_complex_pair(r, crypto_context=context))
    return tuple(out), 2.0


def halve(ciphers, *, context):
    """Public 0.5 multiplication (one rescale) undoing a pair-refresh doubling."""
    return tuple(_half_rescale(c, crypto_context=context) for c in ciphers)


__all__ = ["_pack_complex_pair", "_unpack_complex_pair", "_half_rescale", "pair_bootstrap", "halve"]
