"""Paterson-Stockmeyer evaluation of Chebyshev series on CKKS ciphertexts (the SiLU, rsqrt and exp of the model).

Mirrors ``llama3fhe/operators/nonlinear/polynomial.py:469-562`` (``eval_chebyshev_series_cipher``: same name and
arguments, coefficient convention ``f = c_0 / 2 + sum_j c_j T_j`` on ``[lower_bound, upper_bound]``, and
multiplicative depth ``ceil(log2 k) + m`` with the split ``(k, m)`` of ``approx/chebyshev.py:51-121``).

The split is the published Paterson-Stockmeyer scheme for Chebyshev series with the monic padding
``g = f + T_M``, ``M = k (2^m - 1)`` (Chen, Chillotti, Song, "Improved bootstrapping for approximate homomorphic
encryption", EUROCRYPT 2019, Alg. 2), restated as a tree built on the host before any ciphertext work::

    node(g, 1) = g                                        (degree <= k: a leaf, sum_i w_i T_i)
    node(g, j) = (T_G + c) node(q, j - 1) + node(s, j - 1)   G = k 2^(j-1), X = G - k,
                 g = q T_G + r,  r - T_X = c q + (s - T_X)  (deg c < k, s monic of degree X)

and ``f = node(g, m) - T_M``.  Every leaf is a combination of the baby basis ``T_0 .. T_k``, so on the GPU the whole
tree costs: the baby basis and the giants ``T_{k 2^i}`` from the fused multiply-relinearise-rescale-double-subtract
kernel (``fhe.homo_mul_relin_rescale_postop``), ALL ``2^m - 1`` leaves from one weighted-sum launch per input and
component (``holmes_weighted_acc``, one group per leaf, constants through a trivial ``T_0``) plus one batched
rescale, then one product per inner node.  Inputs may be batches of ciphertexts; every operation runs on the batch.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np
from numpy.polynomial import chebyshev as npcheb

from . import _lib
from . import fhe

__all__ = ["compute_degrees_ps", "chebyshev_ps_mul_depth", "eval_chebyshev_series_cipher", "ps_tree",
           "evaluate_tree_numpy", "PSTree"]

# Degree ranges -> m of the Paterson-Stockmeyer split (k = floor(n / (2^m - 1)) + 1).  This is OpenFHE's
# table as the reference uses it (approx/chebyshev.py:51-76); it is kept identical so that a caller's level budget,
# computed with the reference's chebyshev_ps_mul_depth, matches the depth this evaluator consumes.
_M_BY_DEGREE = ((2, 1), (11, 2), (13, 3), (17, 2), (55, 3), (59, 4), (76, 3), (239, 4), (247, 5), (284, 4),
                (991, 5), (1007, 6), (1083, 5), (2015, 6), (2031, 7), (2204, 6))


def _degree(c) -> int:
    nz = np.flatnonzero(np.asarray(c, dtype=np.float64))
    return int(nz[-1]) if nz.size else 0


def compute_degrees_ps(n: int) -> tuple[int, int]:
    """``(k, m)`` for a Chebyshev series of degree ``n`` (the reference's ``compute_degrees_ps``)."""
    n = int(n)
    if n <= 0:
        raise ValueError("degree must be positive")
    for top, m in _M_BY_DEGREE:
        if n <= top:
            return n // ((1 << m) - 1) + 1, m
    # beyond the table: the fewest non-scalar products k + 2m + 2^(m-1) - 4 over the (k, m) that cover n, with
    # log2 k within one of log2 sqrt(n / 2)
    target = math.floor(math.log2(math.sqrt(n / 2)))
    best = None
    for k in range(1, n + 1):
        if abs(math.floor(math.log2(k)) - target) > 1:
            continue
        for m in range(1, math.ceil(math.log2(n / k) + 1) + 2):
            if k * ((1 << m) - 1) > n:
                cost = k + 2 * m + (1 << (m - 1)) - 4
                if best is None or cost < best[0]:
                    best = (cost, k, m)
    if best is None:
        raise ValueError("No valid (k, m) pairs found")
    return best[1], best[2]


def chebyshev_ps_mul_depth(coefficients) -> int:
    """Levels the evaluation consumes (not counting the map to [-1, 1]): ``ceil(log2 k) + m``."""
    n = _degree(coefficients)
    if n <= 0:
        return 0
    k, m = compute_degrees_ps(n)
    return math.ceil(math.log2(k)) + m


# ----------------------------------------------------------------------------------------------------- the tree


def _t(j: int) -> np.ndarray:
    e = np.zeros(j + 1)
    e[j] = 1.0
    return e


def _pad(c, size: int) -> np.ndarray:
    out = np.zeros(size)
    c = np.asarray(c, dtype=np.float64)[:size]
    out[: c.size] = c
    return out


@dataclass
class PSTree:
    """A node of the split.  Leaves hold standard-convention Chebyshev weights ``w[0..k]`` (``sum_i w_i T_i``);
    inner nodes hold the giant index ``G`` and the leaf ``c`` added to ``T_G`` plus the two children."""

    level: int
    weights: np.ndarray | None = None
    giant: int = 0
    c: "PSTree | None" = None
    q: "PSTree | None" = None
    s: "PSTree | None" = None
    leaves: list = field(default_factory=list)


def _node(g: np.ndarray, j: int, k: int, leaves: list) -> PSTree:
    if j == 1:
        w = _pad(g, k + 1)
        if _degree(g) > k:
            raise AssertionError("leaf of degree above k")
        leaf = PSTree(level=1, weights=w)
        leaves.append(leaf)
        return leaf
    G = k << (j - 1)
    X = G - k
    q, r = npcheb.chebdiv(g, _t(G))
    q = _pad(q, X + 1)
    r2 = _pad(r, G) - _pad(_t(X), G)
    c, s = npcheb.chebdiv(r2, q)
    s = _pad(s, X + 1) + _t(X)
    c_leaf = _node(_pad(c, k), 1, k, leaves)
    return PSTree(level=j, giant=G, c=c_leaf, q=_node(q, j - 1, k, leaves), s=_node(s, j - 1, k, leaves))


def ps_tree(coefficients) -> tuple[int, int, PSTree]:
    """``(k, m, root)`` for reference-convention coefficients (``c_0`` halved).  For ``m > 1`` the root evaluates
    ``f + T_M``; ``m = 1`` is one leaf of ``f`` itself."""
    c = np.asarray(coefficients, dtype=np.float64)
    n = _degree(c)
    if n < 1:
        raise ValueError(f"degree must be >= 1, got {n}.")
    f = np.array(c[: n + 1], copy=True)
    f[0] *= 0.5
    k, m = compute_degrees_ps(n)
    leaves: list = []
    if m == 1:
        root = _node(f, 1, k, leaves)
    else:
        M = k * ((1 << m) - 1)
        g = _pad(f, M + 1)
        g[M] = 1.0
        root = _node(g, m, k, leaves)
    root.leaves = leaves
    return k, m, root


def evaluate_tree_numpy(tree: PSTree, k: int, m: int, y: np.ndarray) -> np.ndarray:
    """The tree evaluated in float64 at ``y`` in [-1, 1] (host check of the split)."""
    def ev(node: PSTree):
        if node.weights is not None:
            return npcheb.chebval(y, node.weights)
        return (npcheb.chebval(y, _t(node.giant)) + ev(node.c)) * ev(node.q) + ev(node.s)

    out = ev(tree)
    if m > 1:
        out = out - npcheb.chebval(y, _t(k * ((1 << m) - 1)))
    return out


# ----------------------------------------------------------------------------------------------------- ciphers


def _add(a: fhe.Cipher, b: fhe.Cipher, ctx) -> fhe.Cipher:
    cur = min(int(a.state.cur_limbs), int(b.state.cur_limbs))
    return fhe.homo_add(fhe._drop_limbs(a, cur), fhe._drop_limbs(b, cur), ctx)


def _sub(a: fhe.Cipher, b: fhe.Cipher, ctx) -> fhe.Cipher:
    cur = min(int(a.state.cur_limbs), int(b.state.cur_limbs))
    return fhe.homo_sub(fhe._drop_limbs(a, cur), fhe._drop_limbs(b, cur), ctx)


def _post_scalar(value: float, a: fhe.Cipher, b: fhe.Cipher, ctx) -> fhe.EncodedScalar:
    """A scalar encoded for the output state of the fused product of ``a`` and ``b``."""
    out = min(int(a.state.cur_limbs), int(b.state.cur_limbs)) - 1
    scale = float(a.state.scaling_factor) * float(b.state.scaling_factor) / float(ctx.rescale_divisor_at(out))
    return fhe.encode_scalar(float(value), cur_limbs=out, scale_degree=1, scaling_factor=scale, context=ctx)


def _baby_basis(y: fhe.Cipher, k: int, ctx) -> list:
    """``[T_1 .. T_k]``: T_2j = 2 T_j^2 - 1 and T_2j+1 = 2 T_j T_j+1 - T_1, each one fused product."""
    T = [y]
    for j in range(2, k + 1):
        lhs, rhs = T[j // 2 - 1], T[(j + 1) // 2 - 1]
        if j & 1:
            T.append(fhe.homo_mul_relin_rescale_postop(lhs, rhs, ctx, apply_double=True, sub=T[0]))
        else:
            T.append(fhe.homo_mul_relin_rescale_postop(lhs, rhs, ctx, apply_double=True,
                                                       scalar=_post_scalar(-1.0, lhs, rhs, ctx)))
    return T


def _leaf_table(leaves: list, basis_limbs: int, scale: float, ctx) -> "fhe.torch.Tensor":
    """``[groups][k + 1][limbs]`` residues of round(w * scale) for every leaf weight."""
    qs = [ctx.q(i) for i in range(basis_limbs)]
    rows = []
    for leaf in leaves:
        ints = [int(round(float(w) * scale)) for w in leaf.weights]
        rows.append([[v % q for q in qs] for v in ints])
    return ctx.device_u64(np.array(rows, dtype=np.uint64))


def _leaves(T: list, leaves: list, ctx) -> list:
    """All leaves of the tree: one weighted-sum launch per input and component over ``[T_0 .. T_k]`` (``T_0`` the
    trivial encryption of 1), then one rescale of all of them."""
    torch = fhe.torch
    k = len(T)
    limbs = int(T[-1].state.cur_limbs)
    B = int(T[0].batch_size)
    N = ctx.N
    scale = float(T[-1].state.scaling_factor)
    basis = torch.empty((2, k + 1, B, limbs, N), dtype=torch.uint64, device=ctx.device)
    basis[:, 0].zero_()
    one = fhe.encode_scalar(1.0, cur_limbs=limbs, scale_degree=1, scaling_factor=scale, context=ctx)
    _lib.call("holmes_add_const", ctx.handle, basis[0, 0].data_ptr(), one.residues(ctx, limbs).data_ptr(),
              basis[0, 0].data_ptr(), B, limbs, limbs * N, limbs * N, fhe._stream())
    for i, t in enumerate(T):
        for c in range(2):
            basis[c, i + 1].copy_(t.cv[c][:, :limbs])
    groups = len(leaves)
    table = _leaf_table(leaves, limbs, scale, ctx)
    acc = torch.empty((2, groups, B, limbs, N), dtype=torch.uint64, device=ctx.device)
    for b in range(B):
        for c in range(2):
            _lib.call("holmes_weighted_acc", ctx.handle, basis[c, 0, b].data_ptr(), B * limbs * N, k + 1,
                      table.data_ptr(), acc[c, 0, b].data_ptr(), B * limbs * N, groups, limbs, fhe._stream())
    state = fhe.CipherState(limbs, 2, scale * scale)
    raw = fhe.Cipher([acc[0].view(groups * B, limbs, N), acc[1].view(groups * B, limbs, N)], state, T[0].slots,
                     False, groups * B, ctx)
    out = fhe.rescale(raw, ctx)
    return [out.cipher_like([cv[g * B:(g + 1) * B] for cv in out.cv], batch_size=B) for g in range(groups)]


def _map_to_chebyshev_domain(x: fhe.Cipher, a: float, b: float, ctx) -> fhe.Cipher:
    """``[a, b]`` onto ``[-1, 1]``: one scalar multiply (a level) unless the slope is 1, one scalar add."""
    alpha = 2.0 / (b - a)
    beta = -1.0 - 2.0 * a / (b - a)
    y = x
    if not math.isclose(alpha, 1.0):
        enc = fhe.encode_scalar(alpha, cur_limbs=int(y.state.cur_limbs), scale_degree=1,
                                scaling_factor=y.state.scaling_factor, context=ctx)
        y = fhe.homo_mul_scalar_rescale(y, enc, ctx)
    if not math.isclose(beta, 0.0):
        y = fhe.homo_add_scalar(y, beta, ctx)
    return y


def eval_chebyshev_series_cipher(input_cipher, coefficients, *, lower_bound: float, upper_bound: float,
                                 crypto_context, input_is_chebyshev_mapped: bool = False):
    """Evaluate pre-fitted Chebyshev coefficients (``c_0`` halved) on a ciphertext or a batch of ciphertexts.

    Consumes ``ceil(log2 k) + m`` levels (plus one for the map to [-1, 1] unless the input is already mapped or
    the interval's slope is 1)."""
    ctx = fhe._ctx(crypto_context)
    coeffs = np.asarray(coefficients, dtype=np.float64)
    n = _degree(coeffs)
    if n < 1:
        raise ValueError(f"degree must be >= 1, got {n}.")
    a, b = float(lower_bound), float(upper_bound)
    k, m, tree = ps_tree(coeffs)
    y = input_cipher if input_is_chebyshev_mapped else _map_to_chebyshev_domain(input_cipher, a, b, ctx)
    need = math.ceil(math.log2(k)) + m + 1
    if int(y.state.cur_limbs) < need:
        raise ValueError(f"degree {n} needs {need - 1} levels and one limb left: the input has "
                         f"{y.state.cur_limbs} limbs")
    T = _baby_basis(y, k, ctx)
    basis_limbs = int(T[-1].state.cur_limbs)
    T = [fhe._drop_limbs(t, basis_limbs) for t in T]
    giants = {k: T[-1]}
    for i in range(1, m):
        prev = giants[k << (i - 1)]
        giants[k << i] = fhe.homo_mul_relin_rescale_postop(prev, prev, ctx, apply_double=True,
                                                           scalar=_post_scalar(-1.0, prev, prev, ctx))
    leaf_values = dict(zip(map(id, tree.leaves), _leaves(T, tree.leaves, ctx)))

    def ev(node: PSTree):
        if node.weights is not None:
            return leaf_values[id(node)]
        head = _add(giants[node.giant], ev(node.c), ctx)
        qv = ev(node.q)
        return _add(fhe.homo_mul_relin_rescale_postop(head, qv, ctx), ev(node.s), ctx)

    out = ev(tree)
    if m > 1:
        # T_M = T_k(2^m - 1) by T_(2^i+1 - 1)k = 2 T_(2^i - 1)k T_2^i k - T_k
        tm = T[-1]
        for i in range(1, m):
            tm = fhe.homo_mul_relin_rescale_postop(tm, giants[k << i], ctx, apply_double=True, sub=T[-1])
        out = _sub(out, tm, ctx)
    return out
