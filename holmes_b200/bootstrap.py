"""CKKS bootstrapping over libholmes_cuda (full-slot, "modraise first").

The reference runs EasyFHE's OpenFHE-style bootstrap (``easyfhe.bs.openfhe``: ``BootstrapSpec``, ``generate``,
``bootstrap``, ``requirements``; used by ``llama3fhe/operators/nonlinear/bootstrap.py:119-159, 249-294, 626-711``)
in the pass order ModRaise -> CoeffsToSlots -> conjugate / real / imaginary -> EvalMod x 2 -> recombine ->
SlotsToCoeffs (``bench/cmp/holmes_batch_bs.py:65-118``).  This module implements that pipeline from the
published algorithm (Cheon-Han-Kim-Kim-Song 2018; cosine + double-angle EvalMod, Han-Ki 2020):

* **ModRaise** -- the ciphertext is scaled by 2^-cf (one level) and brought to q0; ``holmes_modraise`` reads it as
  centred integers modulo q_0..q_{raise-1}.  It now decrypts to t = m' + q0 I with |I| <= ``k_bound``.
* **CoeffsToSlots** -- the special inverse FFT (without its bit reversal and 1/n) factored into log2(n) butterfly
  stages with diagonals {0, +-len/2}, grouped into ``level_budget[0]`` levels; each level is one hoisted set of
  rotations (one ModUp, one key switch per diagonal), one multi-diagonal MAC and one rescale.  The constant
  Delta / (2 n q0 B) is spread evenly over the levels so no plaintext diagonal loses precision.
* **EvalMod** -- the real and imaginary parts (one conjugation) are each mapped to sin(2 pi v) with
  v = t_j / q0: cos(2 pi B w / 2^r) as a Chebyshev series on w = (v - 1/4) / B in [-1, 1], then r double-angle
  steps c <- 2 c^2 - 1.
* **SlotsToCoeffs** -- the forward special FFT stages with q0 2^cf / (2 pi Delta) spread over
  ``level_budget[1]`` levels.

Scales follow the reference's FIXEDMANUAL policy (``llama3fhe/config.py:15-25``): every ciphertext carries the
nominal scale Delta = 2^dcrt_bits at every level; plaintext constants are encoded at the scale of the limb the
next rescale drops, so a multiply-then-rescale returns to Delta.

EasyFHE's constants, level split and EvalMod polynomial are not available, so residues are not comparable to the
reference's; the result is checked at the decoded level (``tests/test_gpu_bootstrap.py``).
"""
from __future__ import annotations

import math
import time
from dataclasses import dataclass, field

import numpy as np
import torch

from . import _lib
from . import fhe as F

# --------------------------------------------------------------------------------------------------------- spec


@dataclass(frozen=True)
class BootstrapSpec:
    log_slots: int = 15
    level_budget: tuple = (4, 4)
    output_levels: int = 24
    strategy: str = "double_hoist"
    mode: str = "modraise_first"
    dim1: tuple | None = None
    baby_step: tuple | None = None
    # engine parameters
    k_bound: int = 24            # bound on |I| in t = m' + q0 I after ModRaise (sparse secret)
    cheb_degree: int = 63        # Chebyshev degree of the cosine
    double_angles: int = 3       # r
    correction_bits: int | None = None   # cf; default makes q0 2^cf / Delta ~ 2^10

    def __post_init__(self) -> None:
        if self.mode != "modraise_first":
            raise ValueError(f"unsupported bootstrap mode {self.mode!r}")
        if len(tuple(self.level_budget)) != 2 or min(self.level_budget) < 1:
            raise ValueError("level_budget must be two positive integers")

    @property
    def evalmod_depth(self) -> int:
        return int(math.ceil(math.log2(self.cheb_degree + 1))) + 1 + int(self.double_angles)

    @property
    def depth(self) -> int:
        return int(self.level_budget[0]) + self.evalmod_depth + int(self.level_budget[1])


@dataclass(frozen=True)
class Requirements:
    rotations: tuple
    depth: int


# --------------------------------------------------------------------------------------------------------- matrices


def _rot_group(n: int, M: int) -> np.ndarray:
    out = np.empty(n // 2 if n >= 2 else 1, dtype=np.int64)
    r = 1
    for j in range(out.size):
        out[j] = r
        r = (r * 5) % M
    return out


def _stage(n: int, length: int, M: int, inverse: bool) -> dict:
    """One butterfly stage of the special FFT as {offset: diagonal} with out[p] = sum_r d_r[p] v[p + r]."""
    half = length // 2
    lenq = 4 * length
    rot = _rot_group(max(length, 2), M)[:half]
    p = np.arange(n)
    j = p % length
    lower = j < half
    jj = np.where(lower, j, j - half)
    if inverse:
        k = (lenq - (rot[jj] % lenq)) * (M // lenq)
    else:
        k = (rot[jj] % lenq) * (M // lenq)
    w = np.exp(2j * np.pi * k / M)
    d0 = np.where(lower, 1.0 + 0j, -w)
    if inverse:
        dp = np.where(lower, 1.0 + 0j, 0j)
        dm = np.where(lower, 0j, w)
    else:
        dp = np.where(lower, w, 0j)
        dm = np.where(lower, 0j, 1.0 + 0j)
    out = {0: d0}
    for r, d in ((half % n, dp), ((-half) % n, dm)):  # +len/2 and -len/2 coincide when len = n
        out[r] = out.get(r, 0) + d
    return out


def _compose(a: dict, b: dict, n: int) -> dict:
    """Diagonals of A o B (apply B first): (A B)_{r+s} += A_r * rot(B_s, r)."""
    out: dict = {}
    for r, da in a.items():
        for s, db in b.items():
            key = (r + s) % n
            term = da * np.roll(db, -r)
            out[key] = out.get(key, 0) + term
    return {k: v for k, v in out.items() if np.abs(v).max() > 0}


def fft_levels(n: int, M: int, budget: int, inverse: bool) -> list[dict]:
    """CoeffsToSlots (inverse=True: stages len = n .. 2) or SlotsToCoeffs (len = 2 .. n) grouped into ``budget``
    levels, each the product of consecutive stages."""
    lengths = [n >> i for i in range(int(math.log2(n)))] if inverse else [2 << i for i in range(int(math.log2(n)))]
    stages = [_stage(n, ln, M, inverse) for ln in lengths]
    groups = np.array_split(np.arange(len(stages)), budget)
    levels = []
    for g in groups:
        mat = {0: np.ones(n, dtype=np.complex128)}
        for idx in g:
            mat = _compose(stages[idx], mat, n)
        levels.append(mat)
    return levels


def apply_levels_numpy(levels: list[dict], v: np.ndarray, scales=None) -> np.ndarray:
    """Plaintext application of grouped levels (host reference for the homomorphic transform)."""
    out = np.asarray(v, dtype=np.complex128)
    for i, mat in enumerate(levels):
        acc = np.zeros_like(out)
        for r, d in mat.items():
            acc += d * np.roll(out, -r)
        out = acc * (1.0 if scales is None else scales[i])
    return out


def chebyshev_cos(B: float, r: int, degree: int) -> np.ndarray:
    """Chebyshev coefficients of cos(2 pi B w / 2^r) on w in [-1, 1]."""
    f = lambda w: np.cos(2 * np.pi * B * w / (1 << r))  # noqa: E731
    return np.polynomial.chebyshev.chebinterpolate(f, degree)


# --------------------------------------------------------------------------------------------------------- program


@dataclass
class BootstrapProgram:
    spec: BootstrapSpec
    context: object
    n: int
    raise_to_limbs: int
    output_limbs: int
    cf: int
    B: float
    c2s: list
    s2c: list
    c2s_scale: float
    s2c_scale: float
    cheb: np.ndarray
    rotations: tuple
    gap: int = 1             # N / (2 n): sparse slots when > 1
    s2c_int: int = 1         # exact integer factor applied before SlotsToCoeffs (keeps its diagonals encodable)
    _plain: dict = field(default_factory=dict)
    _diag: dict = field(default_factory=dict)
    setup_seconds: float = 0.0
    cache_mode: str = "plain"   # "plain": keep encoded diagonals across refreshes; "none": encode per use

    @property
    def constants(self) -> "BootstrapProgram":
        """The program's constant store (EasyFHE ``program.constants``; ``set_cache_mode`` / ``clear_cache``)."""
        return self

    def set_cache_mode(self, mode: str, clear: bool = False) -> None:
        mode = str(mode)
        if mode not in ("none", "middle", "plain", "both"):
            raise ValueError(f"unknown bootstrap constant cache mode {mode!r}")
        self.cache_mode = mode
        if clear:
            self._plain.clear()

    def clear_cache(self) -> None:
        self._plain.clear()

    @property
    def output_state(self) -> F.CipherState:
        return F.CipherState(self.output_limbs, 1, self.context.scale)

    def diagonal_plaintexts(self, which: str, level: int, cur: int, adjust: float = 1.0):
        """Encoded diagonals of one transform level at ``cur`` limbs, scale q_{cur-1}, times ``adjust`` (cached)."""
        key = (which, level, cur, float(adjust))
        hit = self._plain.get(key)
        if hit is not None:
            return hit
        ctx = self.context
        mats = self.c2s if which == "c2s" else self.s2c
        factor = (self.c2s_scale if which == "c2s" else self.s2c_scale) * float(adjust)
        mat = mats[level]
        offsets = sorted(mat)
        # the level's diagonals stay on the device; the factor is applied there (the same double products as
        # mat[r] * factor on the host), so a per-call factor costs no host-to-device copy
        dkey = (which, level)
        raw = self._diag.get(dkey)
        if raw is None:
            host = torch.from_numpy(np.stack([mat[r] for r in offsets]).astype(np.complex128)).pin_memory()
            raw = self._diag[dkey] = host.to(ctx.device, non_blocking=True)
        rows = raw * factor
        scale = float(ctx.q(cur - 1))
        pv = F.encode_rows(ctx, rows, cur, scale, self.n)
        try:
            # a level encoded once (cached) is checked now; a per-call level (SlotsToCoeffs' rho, which the host-side
            # DIAGONAL_LIMIT bound already keeps in range) is checked without draining the stream
            ctx.check_encode_range(wait=float(adjust) == 1.0)
        except ValueError as exc:
            raise ValueError(f"{which} level {level} of the {self.n}-slot bootstrap: diagonals up to "
                             f"{float(np.max(np.abs(np.stack(list(mat.values()))))) * factor:.4g} at scale "
                             f"2^{math.log2(scale):.2f} "
                             f"(factor {factor:.4g}, adjust {float(adjust):.4g}): {exc}") from None
        pt = F.Plaintext([pv], F.CipherState(cur, 1, scale), self.n, False, len(offsets), ctx)
        # a level carrying a per-call factor (SlotsToCoeffs' rho) is encoded per call: caching it would keep one
        # entry per refresh
        if self.cache_mode in ("plain", "both") and float(adjust) == 1.0:
            self._plain[key] = (offsets, pt)
        return offsets, pt


def requirements(specs, log_n: int) -> Requirements:
    rots: set = set()
    depth = 0
    for spec in specs:
        n = 1 << int(spec.log_slots)
        M = 2 << int(log_n)
        for inverse, budget in ((True, spec.level_budget[0]), (False, spec.level_budget[1])):
            for mat in fft_levels(n, M, int(budget), inverse):
                rots.update(int(r) for r in mat if int(r))
        rots.add(M - 1)
        rots.update(n << i for i in range(int(log_n) - 1 - int(spec.log_slots)))  # sparse-slot subsum
        depth = max(depth, spec.depth)
    return Requirements(tuple(sorted(rots)), depth)


#: largest |diagonal value| a transform level may hold: plaintexts are encoded at the scale of the limb the next
#: rescale drops (~2^59), and the encoder's range is 2^61
DIAGONAL_LIMIT = 3.0


def s2c_integer_factor(levels: list[dict], total: float) -> int:
    """The power of two c that SlotsToCoeffs takes as an exact integer multiply (no level) so that its remaining
    constant total / c, spread evenly over the levels, keeps every diagonal below DIAGONAL_LIMIT.  Small level
    budgets (the sparse-slot programs clamp the budget to log2 of their slots) would otherwise put more than the
    encoder's range on each level: q0 2^cf / (2 pi Delta) ~ 163 over 3 levels is 5.5 per level."""
    peak = max(float(np.max(np.abs(np.stack(list(m.values()))))) for m in levels)
    c = 1
    while peak * (total / c) ** (1.0 / len(levels)) > DIAGONAL_LIMIT and c < (1 << 20):
        c *= 2
    return c


def generate(context, spec: BootstrapSpec) -> BootstrapProgram:
    """Precompute one bootstrap program for ``context`` (``bs.generate``)."""
    start = time.perf_counter()
    ctx = context
    n = 1 << int(spec.log_slots)
    if not 2 <= n <= ctx.N // 2:
        raise ValueError(f"bootstrap slots must be a power of two in [2, {ctx.N // 2}], got {n}")
    gap = ctx.N // (2 * n)
    raise_to = ctx.L
    out_limbs = raise_to - spec.depth
    if out_limbs < 2:
        raise ValueError(f"bootstrap depth {spec.depth} leaves {out_limbs} limbs of {raise_to}")
    q0 = ctx.q(0)
    delta = ctx.scale
    cf = spec.correction_bits
    if cf is None:
        cf = max(0, int(round(10 - math.log2(q0 / delta))))
    B = float(spec.k_bound + 1)
    c2s = fft_levels(n, ctx.M, int(spec.level_budget[0]), True)
    s2c = fft_levels(n, ctx.M, int(spec.level_budget[1]), False)
    c2s_total = delta / (2.0 * n * gap * q0 * B)  # the sparse subsum multiplies the message by gap
    s2c_total = q0 * (2.0 ** cf) / (2.0 * math.pi * delta)
    cheb = chebyshev_cos(B, int(spec.double_angles), int(spec.cheb_degree))
    req = requirements([spec], ctx.logN)
    s2c_int = s2c_integer_factor(s2c, s2c_total)
    prog = BootstrapProgram(spec=spec, context=ctx, n=n, raise_to_limbs=raise_to, output_limbs=out_limbs, cf=cf, B=B,
                            c2s=c2s, s2c=s2c, c2s_scale=c2s_total ** (1.0 / len(c2s)),
                            s2c_scale=(s2c_total / s2c_int) ** (1.0 / len(s2c)), cheb=cheb, rotations=req.rotations,
                            gap=gap, s2c_int=s2c_int)
    prog.setup_seconds = time.perf_counter() - start
    return prog


# --------------------------------------------------------------------------------------------------------- helpers
# Exact scales.  A ciphertext's state.scaling_factor is always its true scale.  Inside EvalMod every ciphertext at
# l limbs carries the canonical scale S[l], S[l-1] = S[l]^2 / q_{l-1}: a product of two level-l ciphertexts lands
# on S[l-1] by itself, and level drops and scalar products multiply by an integer chosen to land on S exactly.
# (Treating every scale as the nominal 2^59 would be off by the primes' distance from 2^59, about 2^-32 at
# N = 2^16, and EvalMod multiplies that by the q0 * I overflow term it removes.)


_stream = F._stream


def scale_table(top_limbs: int, top_scale: float, ctx) -> dict:
    S = {int(top_limbs): float(top_scale)}
    for lv in range(int(top_limbs), 1, -1):
        S[lv - 1] = S[lv] * S[lv] / float(ctx.q(lv - 1))
    return S


def mul_int(ct: F.Cipher, k: int) -> F.Cipher:
    """ct * k for an integer k, no rescale: the message is multiplied by k at the same declared scale."""
    ctx = ct.context
    cur = int(ct.state.cur_limbs)
    out = F._new_cipher(ctx, ct.batch_size, cur, ct.state, ct.slots)
    F.const_cv(ctx, F.CONST_MUL, ct.cv[:2], ctx.residues(k, cur), out.cv, ct.batch_size, cur)
    return out


def int_mul_rescale(ct: F.Cipher, k: int, new_scale: float) -> F.Cipher:
    """ct * k (an integer) then rescale; the result is declared at ``new_scale``."""
    ctx = ct.context
    cur = int(ct.state.cur_limbs)
    out = F._new_cipher(ctx, ct.batch_size, cur, F.CipherState(cur, 2, None), ct.slots)
    F.const_cv(ctx, F.CONST_MUL, ct.cv[:2], ctx.residues(k, cur), out.cv, ct.batch_size, cur)
    r = F.rescale(out, ctx)
    r.state = F.CipherState(cur - 1, 1, float(new_scale))
    return r


def mul_scalar_to(ct: F.Cipher, value: float, target: float) -> F.Cipher:
    """value * ct at one limb fewer, landing on scale ``target``."""
    q = float(ct.context.q(int(ct.state.cur_limbs) - 1))
    k = int(round(float(value) * target * q / float(ct.state.scaling_factor)))
    return int_mul_rescale(ct, k, target)


def _drop_view(ct: F.Cipher, limbs: int) -> F.Cipher:
    """The first ``limbs`` limbs of ``ct`` (a view, scale kept): a modulus drop costs no copy."""
    if int(ct.state.cur_limbs) == int(limbs):
        return ct
    return F.Cipher([c[:, :int(limbs)] for c in ct.cv[:2]], ct.state.replace(cur_limbs=int(limbs)), ct.slots, False,
                    ct.batch_size, ct.context)


def adjust(ct: F.Cipher, limbs: int, S: dict) -> F.Cipher:
    """Drop ``ct`` to ``limbs`` limbs, landing on the canonical scale S[limbs]: a modulus drop to ``limbs`` + 1 limbs
    (no arithmetic), then one integer multiply and rescale by q_limbs, k = round(S[limbs] q_limbs / scale)."""
    if int(ct.state.cur_limbs) <= int(limbs):
        return ct
    return mul_scalar_to(_drop_view(ct, int(limbs) + 1), 1.0, S[int(limbs)])


def lin_comb(terms: list, S: dict) -> F.Cipher:
    """sum_i c_i t_i over (ciphertext, coefficient) pairs on canonical scales, with ONE rescale: every t_i is dropped
    (modulus only) to lim + 1 limbs, lim = the lowest term's limbs - 1, and multiply-accumulated with the integer
    k_i = round(c_i S[lim] q_lim / scale_i), so that the rescale by q_lim lands the sum on S[lim]."""
    first = terms[0][0]
    ctx = first.context
    lim = min(int(t.state.cur_limbs) for t, _ in terms) - 1
    target = S[lim]
    q = float(ctx.q(lim))
    batch = first.batch_size
    acc = F._new_cipher(ctx, batch, lim + 1, F.CipherState(lim + 1, 2, None), first.slots)
    for i, (t, c) in enumerate(terms):
        k = int(round(float(c) * target * q / float(t.state.scaling_factor)))
        F.const_cv(ctx, F.CONST_MUL if i == 0 else F.CONST_AXPY, [x[:, :lim + 1] for x in t.cv[:2]],
                   ctx.residues(k, lim + 1), acc.cv, batch, lim + 1)
    r = F.rescale(acc, ctx)
    r.state = F.CipherState(lim, 1, target)
    return r


def add_scalar(ct: F.Cipher, value: float) -> F.Cipher:
    ctx = ct.context
    cur = int(ct.state.cur_limbs)
    v = int(round(float(value) * float(ct.state.scaling_factor)))
    out = F._new_cipher(ctx, ct.batch_size, cur, ct.state, ct.slots)
    F.const_cv(ctx, F.CONST_ADD, ct.cv[:1], ctx.residues(v, cur), out.cv[:1], ct.batch_size, cur)
    out.cv[1].copy_(ct.cv[1][:, :cur])
    return out


def drop_to(ct: F.Cipher, limbs: int) -> F.Cipher:
    """Modulus-only drop (the scale is kept)."""
    if int(ct.state.cur_limbs) == limbs:
        return ct
    return F.align_to(ct, ct.state.replace(cur_limbs=int(limbs)), ct.context)


def mul_rescale(a: F.Cipher, b: F.Cipher, S: dict) -> F.Cipher:
    lim = min(int(a.state.cur_limbs), int(b.state.cur_limbs))
    a, b = adjust(a, lim, S), adjust(b, lim, S)
    return F.rescale(F.homo_mul_relin(a, b, a.context), a.context)


def double(a: F.Cipher) -> F.Cipher:
    return F.homo_add(a, a, a.context)


def add(a: F.Cipher, b: F.Cipher, S: dict) -> F.Cipher:
    lim = min(int(a.state.cur_limbs), int(b.state.cur_limbs))
    return F.homo_add(adjust(a, lim, S), adjust(b, lim, S), a.context)


def sub(a: F.Cipher, b: F.Cipher, S: dict) -> F.Cipher:
    lim = min(int(a.state.cur_limbs), int(b.state.cur_limbs))
    return F.homo_sub(adjust(a, lim, S), adjust(b, lim, S), a.context)


def linear_level(ct: F.Cipher, offsets, pt: F.Plaintext) -> F.Cipher:
    """sum_r diag_r * rot(ct, r): hoisted rotations (one ModUp), one multi-diagonal MAC, one rescale.  The diagonals
    are encoded at the scale of the limb the rescale drops, so the scale is unchanged."""
    ctx = ct.context
    cur = int(ct.state.cur_limbs)
    items = ct.batch_size
    nb = len(offsets)
    store = torch.empty((2, nb, items, cur, ctx.N), dtype=torch.uint64, device=ctx.device)
    switches = []
    for b, off in enumerate(offsets):
        g = ctx.galois(int(off))
        if g == 1:
            store[0, b].copy_(ct.cv[0][:, :cur])
            store[1, b].copy_(ct.cv[1][:, :cur])
        else:
            switches.append((b, g, ctx.switch_key(g, cur)))
    if switches:
        digits, dig_item = F._modup(ctx, ct.cv[1], cur, items)
        lanes = F._ks_lanes(ctx, len(switches))   # the level's key switches are independent: spread over streams
        for i, (b, g, key) in enumerate(switches):
            k = i % len(lanes)
            with torch.cuda.stream(lanes[k]):
                F._keyswitch(ctx, digits, dig_item, cur, g, key, ct.cv[0], None, F._item_stride(ct.cv[0]),
                             store[0, b], store[1, b], items, workspace=f"ks{k}")
        F._ks_join(lanes)
    blocks = [F.Cipher([store[0, :, i], store[1, :, i]], ct.state, ct.slots, False, nb, ctx) for i in range(items)]
    res = F.bsgs_partial_sums(ctx, blocks, pt, 1)          # [2][1][items][cur][N]
    out = F.Cipher([res[0, 0], res[1, 0]], F.CipherState(cur, 2, float(ct.state.scaling_factor) * float(ctx.q(cur - 1))),
                   ct.slots, False, items, ctx)
    return F.rescale(out, ctx)


def ps_baby(degree: int) -> int:
    """Baby-step count m of the Paterson-Stockmeyer evaluation of a degree-``degree`` Chebyshev series:
    2^ceil(log2(degree + 1) / 2), at least 2."""
    return 1 << max(1, math.ceil(math.log2(int(degree) + 1) / 2))


def cheb_split(c: list, n: int) -> tuple:
    """p = q T_n + r for p = sum_k c_k T_k with len(c) <= 2n, from T_(n+j) = 2 T_n T_j - T_(n-j):
    q_0 = c_n, q_j = 2 c_(n+j); r_k = c_k - c_(2n-k) (the second term only where 2n - k < len(c))."""
    L = len(c)
    q = [c[n]] + [2.0 * c[n + j] for j in range(1, L - n)]
    r = [c[k] - (c[2 * n - k] if 2 * n - k < L else 0.0) for k in range(n)]
    return q, r


def _chebyshev(w: F.Cipher, coeffs: np.ndarray, S: dict) -> F.Cipher:
    """sum_k c_k T_k(w) by Paterson-Stockmeyer in the Chebyshev basis (canonical scales throughout): the baby powers
    T_1 .. T_(m-1) and the giant powers T_m, T_2m, ... (T_2k = 2 T_k^2 - 1, T_2k+1 = 2 T_k T_k+1 - T_1); the series
    split recursively as q T_n + r (``cheb_split``) down to leaves of m coefficients, each leaf one multiply-accumulate
    chain with one rescale (``lin_comb``).  Degree 63: 16 ciphertext products instead of 62, at the same depth
    (ceil(log2(d + 1)) + 1 levels)."""
    T: dict = {1: w}
    low: dict = {}

    def t1_at(limbs: int) -> F.Cipher:
        if limbs not in low:
            low[limbs] = adjust(w, limbs, S)
        return low[limbs]

    def get(k: int) -> F.Cipher:
        if k in T:
            return T[k]
        if k % 2 == 0:
            a = get(k // 2)
            T[k] = add_scalar(double(mul_rescale(a, a, S)), -1.0)
        else:
            p = double(mul_rescale(get(k // 2), get(k // 2 + 1), S))
            T[k] = F.homo_sub(p, t1_at(int(p.state.cur_limbs)), p.context)
        return T[k]

    m = ps_baby(len(coeffs) - 1)

    def leaf(c: list) -> F.Cipher:
        terms = [(get(k), float(c[k])) for k in range(1, len(c)) if abs(c[k]) >= 1e-18] or [(get(1), 0.0)]
        return add_scalar(lin_comb(terms, S), float(c[0]))

    def evalp(c: list) -> F.Cipher:
        if len(c) <= m:
            return leaf(c)
        n = 1 << (math.ceil(math.log2(len(c))) - 1)
        q, r = cheb_split(c, n)
        return add(mul_rescale(evalp(q), get(n), S), evalp(r), S)

    return evalp([float(v) for v in coeffs])


def eval_mod(x: F.Cipher, program: BootstrapProgram) -> F.Cipher:
    """x holds v / B (v = t_j / q0); returns sin(2 pi v)."""
    S = scale_table(int(x.state.cur_limbs), float(x.state.scaling_factor), x.context)
    w = add_scalar(x, -0.25 / program.B)
    c = _chebyshev(w, program.cheb, S)
    for _ in range(int(program.spec.double_angles)):
        c = add_scalar(double(mul_rescale(c, c, S)), -1.0)
    return c


def bootstrap(ct: F.Cipher, ctx, program: BootstrapProgram) -> F.Cipher:
    """Refresh ``ct`` (>= 2 limbs, scale degree 1) to ``program.output_limbs`` limbs (``bs.bootstrap``)."""
    ctx = F._ctx(ctx)
    if int(ct.state.cur_limbs) < 2:
        raise ValueError("bootstrap input needs at least two limbs")
    if int(ct.state.scale_degree) != 1 or ct.is_ext:
        raise ValueError("bootstrap input must be a non-extended degree-1 ciphertext")
    if int(ct.slots) != program.n:
        raise ValueError(f"bootstrap program is for {program.n} slots, ciphertext has {ct.slots}")
    s_in = float(ct.state.scaling_factor if ct.state.scaling_factor is not None else ctx.scale)
    x = drop_to(ct, 2).deep_copy() if int(ct.state.cur_limbs) > 2 else ct.deep_copy()
    x.state = F.CipherState(2, 1, s_in)
    k_pre = int(round(2.0 ** (-program.cf) * float(ctx.q(1))))
    x = int_mul_rescale(x, k_pre, s_in)                 # polynomial * k_pre / q1 ~ 2^-cf, now modulo q0 alone
    raise_to = program.raise_to_limbs
    items = x.batch_size
    raised = F._new_cipher(ctx, items, raise_to, F.CipherState(raise_to, 1, float(ctx.scale)), x.slots)
    scratch = ctx.workspace("modraise", 2 * items * ctx.N)
    for (src, n_src, si), (dst, _, so) in F._runs(items, x.cv[:2], raised.cv):
        _lib.call("holmes_modraise", ctx.handle, src.data_ptr(), si, dst.data_ptr(), so, raise_to, n_src,
                  scratch.data_ptr(), _stream())
    y = raised
    # Sparse slots (n < N/2): after ModRaise the overflow q0 I fills every coefficient, not only the multiples of
    # gap = N/(2n) that carry the n-slot message.  Summing the rotations by n j (j < gap), the automorphisms that
    # fix X^gap, keeps gap times the multiples-of-gap part: log2(gap) rotate-and-add steps, no level.
    g = 1
    while g < program.gap:
        y = F.homo_add(y, F.homo_rotate(y, program.n * g, ctx), ctx)
        g *= 2
    for lvl in range(len(program.c2s)):
        offsets, pt = program.diagonal_plaintexts("c2s", lvl, int(y.state.cur_limbs))
        y = linear_level(y, offsets, pt)
    x_c2s_scale = y.state.scaling_factor
    conj = F.homo_rotate(y, ctx.M - 1, ctx)
    re = F.homo_add(y, conj, ctx)
    im = F.homo_mul_i(F.homo_sub(conj, y, ctx), ctx)
    # the real and imaginary parts go through EvalMod as one batch (same level and scale; every op acts item by item,
    # so each part's residues are those of its own evaluation), half the launches of two evaluations
    items = re.batch_size
    both = eval_mod(F.pack_cipher_batch([re, im]), program)
    re = both.cipher_like([c[:items] for c in both.cv], batch_size=items)
    im = both.cipher_like([c[items:] for c in both.cv], batch_size=items)
    z = F.homo_add(re, F.homo_mul_i(im, ctx), ctx)
    # S2C's constant assumes the message at the nominal scale: z carries the input's message at scale
    # S_z Delta / m_scale.  The first S2C level also multiplies by rho = Delta / that, so the output lands exactly on
    # the context's fixed scale Delta, whatever scale the input arrived at (the reference's fixed-scale contexts,
    # scale_mode "fixed": every refresh restarts the scale bookkeeping at Delta, so the small per-level drift of
    # exactly tracked scales -- it doubles with every squaring -- cannot pile up from one refresh to the next).  For an
    # input at Delta, rho is within a few 2^-20 of 1; the diagonals absorb it, no level is spent.
    target = float(ctx.scale)
    m_scale = s_in * k_pre * 2.0 ** program.cf / float(ctx.q(1))
    rho = target / (float(z.state.scaling_factor) * float(ctx.scale) / m_scale)
    if not (math.isfinite(rho) and rho > 0):
        raise ValueError(f"bootstrap scale bookkeeping failed for the {program.n}-slot program: input scale {s_in!r} "
                         f"at {int(ct.state.cur_limbs)} limbs, CoeffsToSlots output scale {x_c2s_scale!r}, EvalMod "
                         f"output scale {z.state.scaling_factor!r} at {int(z.state.cur_limbs)} limbs")
    # exact integer part of the SlotsToCoeffs constant, applied without a level (message and noise alike): the
    # program's share, and the power of two that keeps rho * (per-level factor) encodable when the input arrives at a
    # scale well above its nominal one
    k_int = int(program.s2c_int)
    while rho * program.s2c_scale > DIAGONAL_LIMIT and k_int < (1 << 40):
        rho /= 2.0
        k_int *= 2
    if k_int > 1:
        z = mul_int(z, k_int)
    for lvl in range(len(program.s2c)):
        offsets, pt = program.diagonal_plaintexts("s2c", lvl, int(z.state.cur_limbs), rho if lvl == 0 else 1.0)
        z = linear_level(z, offsets, pt)
    z = drop_to(z, program.output_limbs)
    z.state = F.CipherState(int(z.state.cur_limbs), 1, target)
    return z


# --------------------------------------------------------------------------------------------------------- operator


def with_correction(cipher: F.Cipher, ctx, once, iterations: int, precision_bits: int) -> F.Cipher:
    """One bootstrap, or Meta-BTS: refresh, subtract the input from the refreshed value (both times 2^p, at the
    input's level), refresh that difference, subtract it, multiply by 2^-p with one rescale.  The output then has one
    limb fewer than a single refresh; as in the reference, a refresh that gained no limbs is returned unchanged.
    Names and steps follow the reference's _bootstrap_with_optional_correction (bootstrap.py:626-711)."""
    if int(iterations) not in (1, 2):
        raise ValueError("bootstrap iterations must be one or two.")
    first = once(cipher)
    if int(iterations) == 1:
        return first
    if int(first.state.cur_limbs) <= int(cipher.state.cur_limbs):
        return first
    if int(precision_bits) <= 0:
        first_down = F.align_to(first, cipher.state, ctx)
        error = once(F.homo_sub(first_down, F.align_to(cipher, first_down.state, ctx), ctx))
        return F.homo_sub(F.align_to(first, error.state, ctx), error, ctx)
    factor = F.encode_scalar(1 << int(precision_bits), cur_limbs=int(first.state.cur_limbs), scale_degree=0,
                             mode="integer", context=ctx)
    first_scaled = F.homo_mul_scalar(first, factor, ctx)
    first_down = F.align_to(first_scaled, cipher.state, ctx)
    original_scaled = F.homo_mul_scalar(cipher, factor, ctx)
    original_scaled = F.align_to(original_scaled, first_down.state, ctx)
    error = once(F.homo_sub(first_down, original_scaled, ctx))
    corrected = F.homo_sub(F.align_to(first_scaled, error.state, ctx), F.align_to(error, first_scaled.state, ctx), ctx)
    cur = int(corrected.state.cur_limbs)
    inv = F.encode_scalar(1.0 / float(1 << int(precision_bits)), cur_limbs=cur, scale_degree=1,
                          scaling_factor=float(ctx.q(cur - 1)), context=ctx)
    out = F.homo_mul_scalar_rescale(corrected, inv, ctx)
    out.state = out.state.replace(scaling_factor=first.state.scaling_factor)
    return out


@dataclass(frozen=True)
class BootstrapConfig:
    """Reference: ``llama3fhe/operators/nonlinear/bootstrap.py:47-159`` (full-slot program)."""

    log_slots: int = 15
    level_budget: tuple = (4, 4)
    output_levels: int = 24
    iterations: int = 1
    precision_bits: int = 8
    mode: str = "modraise_first"
    strategy: str = "double_hoist"
    k_bound: int = 24
    cheb_degree: int = 63
    double_angles: int = 3

    def spec(self) -> BootstrapSpec:
        return BootstrapSpec(log_slots=self.log_slots, level_budget=tuple(self.level_budget),
                             output_levels=self.output_levels, strategy=self.strategy, mode=self.mode,
                             k_bound=self.k_bound, cheb_degree=self.cheb_degree, double_angles=self.double_angles)


@dataclass
class BootstrapOperator:
    """Prepared bootstrap program (reference: ``BootstrapOperator.prepare / refresh / refresh_many``)."""

    crypto_context: object
    config: BootstrapConfig
    program: BootstrapProgram
    setup_seconds: float
    calls: int = 0
    batch_calls: int = 0

    @classmethod
    def prepare(cls, crypto_context, config: BootstrapConfig) -> "BootstrapOperator":
        start = time.perf_counter()
        ctx = crypto_context.context
        program = generate(ctx, config.spec())
        ctx.generate_rotation_keys(program.rotations, ctx.L)
        ctx.switch_key(0, ctx.L)
        return cls(crypto_context, config, program, time.perf_counter() - start)

    @staticmethod
    def required_rotations(*, log_n: int, log_slots: int = 15, level_budget: tuple = (4, 4), **_) -> tuple:
        return requirements([BootstrapSpec(log_slots=log_slots, level_budget=tuple(level_budget))], log_n).rotations

    def refresh(self, cipher, *, iterations: int | None = None, precision_bits: int | None = None, **_) -> F.Cipher:
        """One bootstrap, or the two-pass Meta-BTS correction (``iterations = 2``, reference bootstrap.py:626-711)."""
        it = int(self.config.iterations if iterations is None else iterations)
        bits = int(self.config.precision_bits if precision_bits is None else precision_bits)
        self.calls += 1
        ctx = self.crypto_context.context
        return with_correction(cipher, ctx, lambda c: bootstrap(c, ctx, self.program), it, bits)

    def refresh_many(self, ciphers, *, iterations: int | None = None, precision_bits: int | None = None,
                     **kw) -> list:
        """All ciphertexts of one state in one batched pass (every step runs on the batch)."""
        ciphers = list(ciphers)
        if not ciphers:
            return []
        if len(ciphers) == 1 or any(c.state != ciphers[0].state for c in ciphers):
            return [self.refresh(c, iterations=iterations, precision_bits=precision_bits, **kw) for c in ciphers]
        it = int(self.config.iterations if iterations is None else iterations)
        bits = int(self.config.precision_bits if precision_bits is None else precision_bits)
        ctx = self.crypto_context.context
        cur = int(ciphers[0].state.cur_limbs)
        c0 = torch.stack([c.cv[0][0, :cur] for c in ciphers])
        c1 = torch.stack([c.cv[1][0, :cur] for c in ciphers])
        batch = F.Cipher([c0, c1], ciphers[0].state, ciphers[0].slots, False, len(ciphers), ctx)
        out = with_correction(batch, ctx, lambda c: bootstrap(c, ctx, self.program), it, bits)
        self.calls += len(ciphers)
        self.batch_calls += 1
        return [out.cipher_like([out.cv[0][i:i + 1], out.cv[1][i:i + 1]], batch_size=1) for i in range(len(ciphers))]
