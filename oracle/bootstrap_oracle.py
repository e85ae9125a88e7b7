"""CPU restatement of full-slot CKKS bootstrapping -- TEST INFRASTRUCTURE ONLY.

Same pass order as the reference's batched bootstrap (``bench/cmp/holmes_batch_bs.py:65-118``: ModRaise ->
CoeffsToSlots -> conjugate / real / imaginary -> EvalMod x 2 -> recombine -> SlotsToCoeffs) and as
``holmes_b200.bootstrap``, on the oracle's exact CPU primitives (``oracle/oracle.py``), so the GPU result can be
compared residue for residue.  The transform diagonals and the Chebyshev coefficients are the host-side plan of
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

    # -- FIXEDMANUAL helpers (nominal scale Delta after every rescale)
    def _ids(self, cur):
        return list(range(cur))

    def _res(self, value, scale, cur):
        v = int(round(float(value) * float(scale)))
        return [v % self.pr.q[i] for i in range(cur)]

    def mul_scalar_rescale(self, ct, value):
        cur = ct[0].shape[0]
        k = self._res(value, float(self.pr.q[cur - 1]), cur)
        o = self.o
        return o.rescale((o.mul_scalar(ct[0], k, self._ids(cur)), o.mul_scalar(ct[1], k, self._ids(cur))))

    def add_scalar(self, ct, value):
        cur = ct[0].shape[0]
        k = self._res(value, self.delta, cur)
        c0 = ct[0].copy()
        for i in range(cur):
            c0[i] = ((c0[i].astype(object) + k[i]) % self.pr.q[i]).astype(np.uint64)
        return c0, ct[1].copy()

    @staticmethod
    def drop(ct, lim):
        return ct[0][:lim].copy(), ct[1][:lim].copy()

    def mul_rescale(self, a, b):
        lim = min(a[0].shape[0], b[0].shape[0])
        return self.o.rescale(self.o.mul_relin(self.drop(a, lim), self.drop(b, lim)))

    def add(self, a, b):
        lim = min(a[0].shape[0], b[0].shape[0])
        a, b = self.drop(a, lim), self.drop(b, lim)
        return self.o.add(a[0], b[0], self._ids(lim)), self.o.add(a[1], b[1], self._ids(lim))

    def sub(self, a, b):
        lim = min(a[0].shape[0], b[0].shape[0])
        a, b = self.drop(a, lim), self.drop(b, lim)
        return self.o.sub(a[0], b[0], self._ids(lim)), self.o.sub(a[1], b[1], self._ids(lim))

    def linear(self, ct, mat, factor):
        o = self.o
        cur = ct[0].shape[0]
        offs = sorted(mat)
        rots = o.hoisted_rotations(ct, offs)
        acc = None
        for r, (c0, c1) in zip(offs, rots):
            pt = o.encode(mat[r] * factor, cur, float(self.pr.q[cur - 1]))
            t = (o.mul(c0, pt, self._ids(cur)), o.mul(c1, pt, self._ids(cur)))
            acc = t if acc is None else (o.add(acc[0], t[0], self._ids(cur)), o.add(acc[1], t[1], self._ids(cur)))
        return o.rescale(acc)

    def chebyshev(self, w):
        coeffs = self.prog.cheb
        T = {1: w}

        def get(k):
            if k in T:
                return T[k]
            if k % 2 == 0:
                a = get(k // 2)
                s = self.mul_rescale(a, a)
                T[k] = self.add_scalar(self.add(s, s), -1.0)
            else:
                a, b = get(k // 2), get(k // 2 + 1)
                p = self.mul_rescale(a, b)
                T[k] = self.sub(self.add(p, p), T[1])
            return T[k]

        terms = [self.mul_scalar_rescale(get(k), float(coeffs[k])) for k in range(1, len(coeffs))
                 if abs(coeffs[k]) >= 1e-18]
        acc = self.drop(terms[0], min(t[0].shape[0] for t in terms))
        for t in terms[1:]:
            acc = self.add(acc, t)
        return self.add_scalar(acc, float(coeffs[0]))

    def eval_mod(self, x):
        c = self.chebyshev(self.add_scalar(x, -0.25 / self.prog.B))
        for _ in range(int(self.prog.spec.double_angles)):
            s = self.mul_rescale(c, c)
            c = self.add_scalar(self.add(s, s), -1.0)
        return c

    def modraise(self, ct, raise_to):
        o, q0 = self.o, self.pr.q[0]
        out = []
        for c in range(2):
            v = o.intt(ct[c][:1], [0])[0].astype(object)
            v = np.where(v > q0 // 2, v - q0, v)
            rows = np.stack([np.array([int(a) % self.pr.q[i] for a in v], dtype=np.uint64) for i in range(raise_to)])
            out.append(o.ntt(rows, self._ids(raise_to)))
        return tuple(out)

    def bootstrap(self, ct):
        o, prog = self.o, self.prog
        x = self.drop(ct, 2) if ct[0].shape[0] > 2 else (ct[0].copy(), ct[1].copy())
        x = self.mul_scalar_rescale(x, 2.0 ** (-prog.cf))
        y = self.modraise(x, prog.raise_to_limbs)
        for lvl in prog.c2s:
            y = self.linear(y, lvl, prog.c2s_scale)
        cur = y[0].shape[0]
        cj = o.rotate(y, 2 * self.pr.n - 1)          # conjugation: rotation index M - 1
        re = (o.add(y[0], cj[0], self._ids(cur)), o.add(y[1], cj[1], self._ids(cur)))
        im = o.mul_i((o.sub(cj[0], y[0], self._ids(cur)), o.sub(cj[1], y[1], self._ids(cur))))
        re, im = self.eval_mod(re), self.eval_mod(im)
        z = self.add(re, o.mul_i(im))
        for lvl in prog.s2c:
            z = self.linear(z, lvl, prog.s2c_scale)
        return self.drop(z, prog.output_limbs)


__all__ = ["OracleBootstrap"]
