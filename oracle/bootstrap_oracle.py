"""CPU restatement of CKKS bootstrapping (full and sparse slots) -- TEST INFRASTRUCTURE ONLY.

Same pass order as the reference's batched bootstrap (``bench/cmp/holmes_batch_bs.py:65-118``: ModRaise ->
CoeffsToSlots -> conjugate / real / imaginary -> EvalMod x 2 -> recombine -> SlotsToCoeffs) and as
``holmes_b200.bootstrap``, on the oracle's exact CPU primitives (``oracle/oracle.py``), so the GPU result can be
compared residue for residue; scales are tracked exactly, with the same floating-point
steps as the GPU path, so the integer constants agree.  The transform diagonals and the Chebyshev coefficients are the host-side plan of
``holmes_b200.bootstrap`` (``fft_levels`` / ``chebyshev_cos``), which ``tests/test_bootstrap_plan.py`` checks
against the oracle's special FFT.  EasyFHE's own bootstrap constants are not available: parity with the
reference binary is unpinned here; the decoded result is checked against the input message.
"""
from __future__ import annotations

import math

import numpy as np

from .oracle import Oracle


class OracleBootstrap:
    def __init__(self, o: Oracle, program) -> None:
        self.o = o
        self.pr = o.pr
        self.prog = program
        self.delta = float(2.0 ** self.pr.scale_bits)

    # -- exact scales: a ciphertext is (c0, c1, scale); inside EvalMod the scale at l limbs is the canonical
    #    S[l], S[l-1] = S[l]^2 / q_{l-1}, reached by integer multiplies before each rescale
    def _ids(self, cur):
        return list(range(cur))

    def scale_table(self, top, s_top):
        S = {top: float(s_top)}
        for lv in range(top, 1, -1):
            S[lv - 1] = S[lv] * S[lv] / float(self.pr.q[lv - 1])
        return S

    def int_mul_rescale(self, ct, k, new_scale):
        c0, c1, _ = ct
        cur = c0.shape[0]
        r = [int(k) % self.pr.q[i] for i in range(cur)]
        o = self.o
        d0, d1 = o.rescale((o.mul_scalar(c0, r, self._ids(cur)), o.mul_scalar(c1, r, self._ids(cur))))
        return d0, d1, float(new_scale)

    def mul_scalar_to(self, ct, value, target):
        q = float(self.pr.q[ct[0].shape[0] - 1])
        return self.int_mul_rescale(ct, int(round(float(value) * target * q / float(ct[2]))), target)

    def adjust(self, ct, lim, S):
        # a modulus drop to lim + 1 limbs, then one integer multiply and rescale onto S[lim]
        if ct[0].shape[0] <= lim:
            return ct
        return self.mul_scalar_to(self.drop(ct, lim + 1), 1.0, S[lim])

    def lin_comb(self, terms, S):
        # sum c_i t_i: every t_i dropped to lim + 1 limbs and multiplied by k_i = round(c_i S[lim] q_lim / s_i), the
        # products summed, one rescale onto S[lim]
        o = self.o
        lim = min(t[0].shape[0] for t, _ in terms) - 1
        target = S[lim]
        q = float(self.pr.q[lim])
        ids = self._ids(lim + 1)
        acc = None
        for t, c in terms:
            k = int(round(float(c) * target * q / float(t[2])))
            r = [k % self.pr.q[i] for i in range(lim + 1)]
            m = (o.mul_scalar(t[0][:lim + 1], r, ids), o.mul_scalar(t[1][:lim + 1], r, ids))
            acc = m if acc is None else (o.add(acc[0], m[0], ids), o.add(acc[1], m[1], ids))
        d0, d1 = o.rescale(acc)
        return d0, d1, target

    def add_scalar(self, ct, value):
        c0, c1, sf = ct
        cur = c0.shape[0]
        v = int(round(float(value) * float(sf)))
        out = c0.copy()
        for i in range(cur):
            out[i] = ((out[i].astype(object) + v % self.pr.q[i]) % self.pr.q[i]).astype(np.uint64)
        return out, c1.copy(), sf

    @staticmethod
    def drop(ct, lim):
        return ct[0][:lim].copy(), ct[1][:lim].copy(), ct[2]

    def _add(self, a, b, sub=False):
        f = self.o.sub if sub else self.o.add
        lim = a[0].shape[0]
        return f(a[0], b[0], self._ids(lim)), f(a[1], b[1], self._ids(lim)), a[2]

    def mul_rescale(self, a, b, S):
        lim = min(a[0].shape[0], b[0].shape[0])
        a, b = self.adjust(a, lim, S), self.adjust(b, lim, S)
        d0, d1 = self.o.rescale(self.o.mul_relin(a[:2], b[:2]))
        return d0, d1, float(a[2]) * float(b[2]) / self.pr.q[lim - 1]

    def linear(self, ct, mat, factor):
        o = self.o
        c0, c1, sf = ct
        cur = c0.shape[0]
        offs = sorted(mat)
        rots = o.hoisted_rotations((c0, c1), offs)
        acc = None
        for r, (r0, r1) in zip(offs, rots):
            pt = o.encode(mat[r] * factor, cur, float(self.pr.q[cur - 1]), slots=len(mat[r]))
            t = (o.mul(r0, pt, self._ids(cur)), o.mul(r1, pt, self._ids(cur)))
            acc = t if acc is None else (o.add(acc[0], t[0], self._ids(cur)), o.add(acc[1], t[1], self._ids(cur)))
        d0, d1 = o.rescale(acc)
        return d0, d1, float(sf) * float(self.pr.q[cur - 1]) / self.pr.q[cur - 1]

    def add_adj(self, a, b, S):
        lim = min(a[0].shape[0], b[0].shape[0])
        return self._add(self.adjust(a, lim, S), self.adjust(b, lim, S))

    def chebyshev(self, w, S):
        # Paterson-Stockmeyer in the Chebyshev basis: babies T_1 .. T_(m-1), giants T_m, T_2m, ...; p = q T_n + r
        # recursively down to leaves of m coefficients, each one lin_comb (the split arithmetic is the plan's,
        # holmes_b200.bootstrap.ps_baby / cheb_split)
        from holmes_b200.bootstrap import cheb_split, ps_baby

        coeffs = self.prog.cheb
        T = {1: w}
        low = {}

        def t1_at(lim):
            if lim not in low:
                low[lim] = self.adjust(w, lim, S)
            return low[lim]

        def get(k):
            if k in T:
                return T[k]
            if k % 2 == 0:
                a = get(k // 2)
                s = self.mul_rescale(a, a, S)
                T[k] = self.add_scalar(self._add(s, s), -1.0)
            else:
                p = self.mul_rescale(get(k // 2), get(k // 2 + 1), S)
                T[k] = self._add(self._add(p, p), t1_at(p[0].shape[0]), sub=True)
            return T[k]

        m = ps_baby(len(coeffs) - 1)

        def leaf(c):
            terms = [(get(k), float(c[k])) for k in range(1, len(c)) if abs(c[k]) >= 1e-18] or [(get(1), 0.0)]
            return self.add_scalar(self.lin_comb(terms, S), float(c[0]))

        def evalp(c):
            if len(c) <= m:
                return leaf(c)
            n = 1 << (math.ceil(math.log2(len(c))) - 1)
            q, r = cheb_split(c, n)
            return self.add_adj(self.mul_rescale(evalp(q), get(n), S), evalp(r), S)

        return evalp([float(v) for v in coeffs])

    def eval_mod(self, x):
        S = self.scale_table(x[0].shape[0], x[2])
        c = self.chebyshev(self.add_scalar(x, -0.25 / self.prog.B), S)
        for _ in range(int(self.prog.spec.double_angles)):
            s = self.mul_rescale(c, c, S)
            c = self.add_scalar(self._add(s, s), -1.0)
        return c

    def modraise(self, ct, raise_to):
        o, q0 = self.o, self.pr.q[0]
        out = []
        for c in range(2):
            v = o.intt(ct[c][:1], [0])[0].astype(object)
            v = np.where(v > q0 // 2, v - q0, v)
            rows = np.stack([np.array([int(a) % self.pr.q[i] for a in v], dtype=np.uint64) for i in range(raise_to)])
            out.append(o.ntt(rows, self._ids(raise_to)))
        return out[0], out[1], self.delta

    def bootstrap(self, ct, s_in=None):
        """Refresh ``ct`` = (c0, c1) at scale ``s_in`` (default 2^scale_bits); returns (c0, c1, scale)."""
        o, prog = self.o, self.prog
        s_in = self.delta if s_in is None else float(s_in)
        x = (ct[0][:2].copy(), ct[1][:2].copy(), s_in)
        k_pre = int(round(2.0 ** (-prog.cf) * float(self.pr.q[1])))
        x = self.int_mul_rescale(x, k_pre, s_in)
        y = self.modraise(x, prog.raise_to_limbs)
        g = 1
        while g < getattr(prog, "gap", 1):   # sparse slots: sum of the rotations by n j, j < gap
            r0, r1 = o.rotate(y[:2], prog.n * g)
            ids = self._ids(y[0].shape[0])
            y = (o.add(y[0], r0, ids), o.add(y[1], r1, ids), y[2])
            g *= 2
        for lvl in prog.c2s:
            y = self.linear(y, lvl, prog.c2s_scale)
        cur = y[0].shape[0]
        c0, c1 = o.rotate(y[:2], 2 * self.pr.n - 1)          # conjugation: rotation index M - 1
        cj = (c0, c1, y[2])
        re = self._add(y, cj)
        d = self._add(cj, y, sub=True)
        i0, i1 = o.mul_i(d[:2])
        re, im = self.eval_mod(re), self.eval_mod((i0, i1, d[2]))
        j0, j1 = o.mul_i(im[:2])
        z = self._add(re, (j0, j1, im[2]))
        m_scale = s_in * k_pre * 2.0 ** prog.cf / float(self.pr.q[1])
        rho = self.delta / (float(z[2]) * self.delta / m_scale)   # output at the fixed scale Delta
        c_int = int(getattr(prog, "s2c_int", 1))
        while rho * prog.s2c_scale > 3.0 and c_int < (1 << 40):   # holmes_b200.bootstrap.DIAGONAL_LIMIT
            rho /= 2.0
            c_int *= 2
        if c_int > 1:   # the exact integer part of the SlotsToCoeffs constant (holmes_b200.bootstrap.mul_int)
            ids = self._ids(z[0].shape[0])
            r = [c_int % self.pr.q[i] for i in ids]
            z = (o.mul_scalar(z[0], r, ids), o.mul_scalar(z[1], r, ids), z[2])
        for k, lvl in enumerate(prog.s2c):
            z = self.linear(z, lvl, prog.s2c_scale * (rho if k == 0 else 1.0))
        z = self.drop(z, prog.output_limbs)
        return z[0], z[1], self.delta

    def refresh(self, ct, s_in, iterations=1, precision_bits=8):
        """One bootstrap or the Meta-BTS correction (same steps as holmes_b200.bootstrap.with_correction)."""
        o = self.o
        first = self.bootstrap(ct, s_in)
        cur_in = ct[0].shape[0]
        if iterations == 1 or first[0].shape[0] <= cur_in:
            return first

        def sub(a, b):
            ids = self._ids(a[0].shape[0])
            return o.sub(a[0], b[0], ids), o.sub(a[1], b[1], ids)

        def mul_int(c, k):
            ids = self._ids(c[0].shape[0])
            r = [int(k) % self.pr.q[i] for i in ids]
            return o.mul_scalar(c[0], r, ids), o.mul_scalar(c[1], r, ids)

        if precision_bits <= 0:
            first_down = (first[0][:cur_in], first[1][:cur_in])
            err = self.bootstrap(sub(first_down, (ct[0][:cur_in], ct[1][:cur_in])), s_in)
            lim = err[0].shape[0]
            d0, d1 = sub((first[0][:lim], first[1][:lim]), err)
            return d0, d1, self.delta
        f = 1 << int(precision_bits)
        fs = mul_int(first, f)
        first_down = (fs[0][:cur_in], fs[1][:cur_in])
        orig = mul_int((ct[0][:cur_in], ct[1][:cur_in]), f)
        err = self.bootstrap(sub(first_down, orig), s_in)
        lim = min(err[0].shape[0], fs[0].shape[0])
        c0, c1 = sub((fs[0][:lim], fs[1][:lim]), (err[0][:lim], err[1][:lim]))
        k = int(round(1.0 / float(f) * float(self.pr.q[lim - 1])))
        d0, d1 = o.rescale(mul_int((c0, c1), k))
        return d0, d1, self.delta


__all__ = ["OracleBootstrap"]
