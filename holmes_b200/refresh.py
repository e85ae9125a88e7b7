"""Pair refresh on this engine: one bootstrap carries two real ciphertexts, packed as ``a + i b``.

The composition is the reference's (``llama3fhe/operators/norm/refresh.py:21-60`` for the pack / unpack / halving
helpers, ``llama3fhe/parallel/prefill/stations.py:102-190`` for ``pair_bootstrap`` and ``halve``), and it has to be:
the three-line arithmetic is the interface.  The functions keep those names and argument meanings so a caller of the
reference can use them; they run on :mod:`holmes_b200.fhe` and the batched
:class:`holmes_b200.bootstrap.BootstrapOperator`, and they leave their inputs untouched.
"""
from __future__ import annotations

from . import fhe


def _ctx_of(crypto_context):
    return getattr(crypto_context, "context", crypto_context)


def _half_rescale(cipher, *, crypto_context):
    """Multiply by the public constant 1/2 and rescale once; the result keeps the input's scale."""
    ctx = _ctx_of(crypto_context)
    encoded = fhe.encode_scalar(0.5, cur_limbs=int(cipher.state.cur_limbs), scale_degree=1,
                                scaling_factor=float(ctx.q(int(cipher.state.cur_limbs) - 1)), context=ctx)
    out = fhe.homo_mul_scalar_rescale(cipher, encoded, ctx)
    out.state = out.state.replace(scaling_factor=cipher.state.scaling_factor)
    return out


def _pack_complex_pair(left, right, *, crypto_context):
    """``left + i right``: the real parts of two messages share one ciphertext (and so one bootstrap)."""
    ctx = _ctx_of(crypto_context)
    return fhe.homo_add(left, fhe.homo_mul_i(right, ctx), ctx)


def _unpack_complex_pair(value, *, crypto_context):
    """(2 Re, 2 Im) of a refreshed ``a + i b`` from one conjugation (rotation index M - 1): v + conj(v) and
    i (conj(v) - v).  The factor 2 stays for the caller to remove (``_half_rescale``) or fold into a later
    constant."""
    ctx = _ctx_of(crypto_context)
    conjugated = fhe.homo_rotate(value, int(ctx.M) - 1, ctx)
    real_twice = fhe.homo_add(value, conjugated, ctx)
    imaginary_twice = fhe.homo_mul_i(fhe.homo_sub(conjugated, value, ctx), ctx)
    return real_twice, imaginary_twice


def pair_bootstrap(ciphers, *, context, bootstrap_operator, iterations: int = 1, precision_bits: int = 14,
                   synchronize: bool = True):
    """Bootstrap an even number of real ciphertexts at half the bootstrap count: consecutive pairs are packed as
    ``a + i b``, refreshed, and split again.  Returns the refreshed ciphertexts (each doubled) and the factor 2.0.

    With an operator that has ``refresh_many`` every pair moves through one batched C2S / EvalMod / S2C pass;
    otherwise each pair is refreshed on its own.
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
    """Remove the doubling of ``pair_bootstrap`` (a public 1/2 and one rescale per ciphertext)."""
    return tuple(_half_rescale(c, crypto_context=context) for c in ciphers)


__all__ = ["_pack_complex_pair", "_unpack_complex_pair", "_half_rescale", "pair_bootstrap", "halve"]
