"""EasyFHE-shaped CKKS API over libholmes_cuda.

The reference's operators (``llama3fhe``) reach their engine through ``from easyfhe import fhe`` and
the session object's ``fhe`` / ``context`` / ``client`` fields (``llama3fhe/backend.py:249-396``).  This
module provides the subset of that surface the linear / key-switch hot path uses, with the same names,
argument meanings and error behaviour (``ValueError`` on state mismatches):

* ``CKKSContextSpec``, ``generate_client_context`` -> ``(Client, Context)``  (backend.py:556-596)
* ``CipherState``, ``Cipher`` (``cv`` = two uint64 tensors ``[batch][limbs][N]``, ``state``, ``slots``,
  ``is_ext``, ``batch_size``, ``cipher_like``, ``deep_copy``; parallel/wire.py:81-200)
* ``homo_add``, ``homo_sub``, ``homo_mul_i``, ``rescale``, ``align_to``, ``homo_rotate`` (rotation index
  ``M - 1`` = conjugation, qkv_kernel.py:832), ``prepare_hoisted_baby_rotations``, ``hoisted_mac_sum``,
  ``homo_mul_pt``, ``homo_mul_relin``, ``homo_mul_no_relin``, ``homo_relinearize``
* ``ConstantBundle`` / ``PackedRaw`` / ``UnpackedRaw`` (weight.py:471-545, backend.py:352-370)

Every arithmetic step runs in libholmes_cuda on the current torch CUDA stream; torch only owns the
device buffers.  There is no CPU path: without the library or a CUDA device these calls raise.
"""
from __future__ import annotations

import collections
import dataclasses
import gc
import math
import types
from dataclasses import dataclass, field

import numpy as np
import torch

from . import _lib

# ----------------------------------------------------------------------------------------------------- timing


class OpTimer:
    """CUDA-event timing of the engine's kernel families, with the algorithmic bytes each launch must move.

    Disabled by default; ``bench.py`` enables it over its timed region.  ``summary()`` synchronises."""

    def __init__(self) -> None:
        self.enabled = False
        self.records: dict = {}

    def start(self, name: str):
        if not self.enabled:
            return None
        e = torch.cuda.Event(enable_timing=True)
        e.record()
        return (name, e)

    def stop(self, token, nbytes: int) -> None:
        if token is None:
            return
        e = torch.cuda.Event(enable_timing=True)
        e.record()
        self.records.setdefault(token[0], []).append((token[1], e, int(nbytes)))

    def reset(self) -> None:
        self.records = {}

    def summary(self) -> dict:
        torch.cuda.synchronize()
        out = {}
        for name, recs in self.records.items():
            ms = sum(a.elapsed_time(b) for a, b, _ in recs)
            out[name] = {"launches": len(recs), "ms": ms, "bytes": sum(n for _, _, n in recs)}
        return out


OPTIMER = OpTimer()

# ----------------------------------------------------------------------------------------------------- state


@dataclass(frozen=True)
class CipherState:
    cur_limbs: int
    scale_degree: int = 1
    scaling_factor: float | None = None

    def replace(self, **changes) -> "CipherState":
        return dataclasses.replace(self, **changes)


class Cipher:
    """A CKKS ciphertext (two components) or a plaintext batch (one component).

    ``cv[c]`` is a ``torch.uint64`` tensor ``[batch][limbs_alloc][N]``; only the first
    ``state.cur_limbs`` limbs are meaningful.
    """

    def __init__(self, cv, state: CipherState, slots: int, is_ext: bool = False, batch_size: int | None = None,
                 context=None) -> None:
        self.cv = list(cv)
        self.state = state
        self.slots = int(slots)
        self.is_ext = bool(is_ext)
        self.batch_size = int(self.cv[0].shape[0] if batch_size is None else batch_size)
        self.context = context

    def cipher_like(self, cv, *, state=None, slots=None, is_ext=None, batch_size=None) -> "Cipher":
        return type(self)(cv, self.state if state is None else state, self.slots if slots is None else slots,
                          self.is_ext if is_ext is None else is_ext, batch_size, self.context)

    def deep_copy(self) -> "Cipher":
        return self.cipher_like([c.clone() for c in self.cv])

    @property
    def device(self):
        return self.cv[0].device

    def __repr__(self) -> str:
        return (f"Cipher(batch={self.batch_size}, limbs={self.state.cur_limbs}, degree={self.state.scale_degree}, "
                f"slots={self.slots})")


class Plaintext(Cipher):
    """One-component batch of NTT plaintexts ``cv[0]`` [rows][limbs][N]."""


# ----------------------------------------------------------------------------------------------------- context


@dataclass
class CKKSContextSpec:
    depth: int
    log_n: int
    dnum: int
    dcrt_bits: int
    first_mod: int
    secret_key_dist: str = "SPARSE_TERNARY"
    scale_mode: str = "fixed"
    rescale_policy: str = "manual"
    rotations: tuple = ()
    auto_load_keys: bool = True
    # engine parameters beyond the reference's spec
    special_bits: int = 60
    special_limbs: int | None = None
    hamming_weight: int = 192
    seed: int = 0
    scale_bits: int | None = None
    #: rotation -> largest limb count it is applied to (trimmed keys, parallel/prefill/keys.py:118-140)
    rotation_key_limb_limits: dict = field(default_factory=dict)
    relinearization: bool = True


_RAW_STREAM = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _stream() -> int:
    """The current CUDA stream of the current device, as the C ABI's ``void* stream``."""
    if _RAW_STREAM is not None:
        return _RAW_STREAM(torch._C._cuda_getDevice())
    return torch.cuda.current_stream().cuda_stream


class Context:
    """Evaluation context: moduli, device tables and switching keys (EasyFHE ``context``)."""

    def __init__(self, spec: CKKSContextSpec, device: str = "cuda") -> None:
        if not torch.cuda.is_available():
            raise _lib.HolmesError("libholmes_cuda needs a CUDA device")
        if torch.device(device).type != "cuda":
            raise _lib.HolmesError(f"libholmes_cuda has no CPU backend: device {device!r} is not a CUDA device")
        # contexts (keys, workspaces) that are no longer referenced may sit in reference cycles; free their device
        # memory before this one allocates (a caller that builds many contexts in one process relies on it)
        gc.collect()
        self.spec = spec
        self.device = torch.device(device if device != "cuda" else f"cuda:{torch.cuda.current_device()}")
        torch.cuda.set_device(self.device)
        params = _lib.HolmesParams()
        params.log_n = int(spec.log_n)
        params.limbs = int(spec.depth) + 1
        params.dnum = int(spec.dnum)
        params.dcrt_bits = int(spec.dcrt_bits)
        params.first_mod_bits = int(spec.first_mod)
        params.special_bits = int(spec.special_bits)
        params.special_limbs = int(spec.special_limbs or 0)
        dist = str(spec.secret_key_dist).upper()
        params.hamming = int(spec.hamming_weight) if dist.startswith("SPARSE") else 0
        params.seed = int(spec.seed)
        handle = _lib.ctypes.c_void_p()
        _lib.call("holmes_ctx_create", _lib.ctypes.byref(params), _lib.ctypes.byref(handle))
        self.handle = handle
        dims = (_lib.ctypes.c_int * 6)()
        _lib.call("holmes_ctx_dims", handle, dims)
        self.logN, self.L, self.K, self.alpha, self.dnum, self.beta_max = (int(v) for v in dims)
        self.N = 1 << self.logN
        self.M = 2 * self.N
        self.max_slots = self.N // 2
        moduli = (_lib.ctypes.c_uint64 * (self.L + self.K))()
        _lib.call("holmes_ctx_moduli", handle, moduli)
        self.moduli = [int(v) for v in moduli]
        self.scale = float(2.0 ** (spec.scale_bits if spec.scale_bits is not None else spec.dcrt_bits))
        # EasyFHE-style per-limb tables on the device (reference-ABI callers read these)
        ks = [q.bit_length() - 1 + 63 for q in self.moduli]
        self.primes = torch.tensor(self.moduli, dtype=torch.uint64, device=self.device)
        self.barret_k = torch.tensor(ks, dtype=torch.uint64, device=self.device)
        self.barret_ratio = torch.tensor([(1 << k) // q for k, q in zip(ks, self.moduli)], dtype=torch.uint64,
                                         device=self.device)
        self._keys: dict = {}
        self._caps = None
        self._galois_cache: dict = {}
        self._requested = set(int(r) for r in spec.rotations)
        self._work: dict = {}
        self._flag = torch.zeros(1, dtype=torch.int32, device=self.device)
        self._consts: collections.OrderedDict = collections.OrderedDict()
        self._modup_cache: collections.OrderedDict = collections.OrderedDict()
        self._modup_by_storage: dict = {}
        self._modup_cache_bytes = 0
        self._enc_counter = 0
        self.key_bytes = 0

    # -- bookkeeping ---------------------------------------------------------------------------------------
    def scale_at(self, cur_limbs: int) -> float:
        del cur_limbs
        return self.scale

    def q(self, i: int) -> int:
        return self.moduli[i]

    def rescale_divisor_at(self, cur_limbs: int) -> int:
        """The prime a rescale divides by when its output has ``cur_limbs`` limbs (the limb it drops)."""
        return self.moduli[int(cur_limbs)]

    def p_mod_q(self, cur: int) -> list:
        """P = product of the special primes, modulo q_0 .. q_{cur-1}."""
        P = math.prod(self.moduli[self.L:self.L + self.K])
        return [P % self.moduli[i] for i in range(int(cur))]

    def device_u64(self, rows) -> torch.Tensor:
        """A small uint64 table on this context's device, without a stream synchronisation: the copy starts from
        pinned host memory, and tables seen before come from a bounded cache (per-level constants recur in every
        bootstrap and polynomial)."""
        arr = np.ascontiguousarray(np.asarray(rows, dtype=np.uint64))
        key = (arr.shape, arr.tobytes()) if arr.nbytes <= 65536 else None
        if key is not None:
            hit = self._consts.get(key)
            if hit is not None:
                self._consts.move_to_end(key)
                return hit
        dev = torch.from_numpy(arr).pin_memory().to(self.device, non_blocking=True)
        if key is not None:
            self._consts[key] = dev
            if len(self._consts) > 8192:
                self._consts.popitem(last=False)
        return dev

    def forget_digits(self, *tensors) -> None:
        """Retire reused ModUp digits: of the inputs overlapping ``tensors``, or all of them when none are given.  A
        caller that overwrites a ciphertext's memory outside torch (its own kernel launches) calls this first; writes
        through torch ops and through this engine are tracked already."""
        if tensors:
            _modup_forget(self, *tensors)
        else:
            self._modup_cache.clear()
            self._modup_by_storage.clear()
            self._modup_cache_bytes = 0

    def p_mod_q_dev(self, cur: int) -> torch.Tensor:
        return self.device_u64(self.p_mod_q(cur))

    def residues(self, value: int, cur: int) -> list:
        """Canonical residues of an integer modulo q_0 .. q_{cur-1}."""
        v = int(value)
        return [v % q for q in self.moduli[:int(cur)]]

    def beta(self, cur: int) -> int:
        return -(-int(cur) // self.alpha)

    def galois(self, rotation: int) -> int:
        g = self._galois_cache.get(int(rotation))
        if g is None:
            out = _lib.ctypes.c_uint64()
            _lib.call("holmes_galois", self.handle, int(rotation), _lib.ctypes.byref(out))
            g = self._galois_cache[int(rotation)] = int(out.value)
        return g

    def workspace(self, name: str, words: int) -> torch.Tensor:
        buf = self._work.get(name)
        if buf is None or buf.numel() < words:
            buf = torch.empty(int(words), dtype=torch.uint64, device=self.device)
            self._work[name] = buf
        return buf

    def key_words(self, cap: int) -> int:
        out = _lib.ctypes.c_longlong()
        _lib.call("holmes_key_words", self.handle, int(cap), _lib.ctypes.byref(out))
        return int(out.value)

    def _make_key(self, galois: int, cap: int) -> torch.Tensor:
        key = torch.empty(self.key_words(cap), dtype=torch.uint64, device=self.device)
        _lib.call("holmes_keygen", self.handle, int(galois), int(cap), key.data_ptr(), _stream())
        self.key_bytes += key.numel() * 8
        return key

    def key_limit(self, galois: int) -> int | None:
        """The configured limb cap of a rotation's key (``rotation_key_limb_limits``), or None."""
        if self._caps is None:
            limits = self.spec.rotation_key_limb_limits or {}
            self._caps = {self.galois(int(r)): int(c) for r, c in limits.items()}
        return self._caps.get(galois) if galois else None

    def switch_key(self, galois: int, cur_limbs: int):
        """(key tensor, cap) for X -> X^galois (0 = relinearisation) usable at ``cur_limbs``.  A key is generated on
        first use, trimmed to the Q limbs it serves: the larger of ``cur_limbs`` and the rotation's configured limit
        (the key's rows for limbs below any cap are the same words, so a trimmed key gives the same residues).  A
        request above the cached key's cap replaces it with a wider one."""
        entry = self._keys.get(galois)
        if entry is not None and entry[1] >= cur_limbs:
            return entry
        limit = self.key_limit(galois)
        cap = min(self.L, max(int(cur_limbs), int(limit) if limit else int(cur_limbs)))
        if entry is not None:
            self.key_bytes -= entry[0].numel() * 8
        entry = (self._make_key(galois, cap), cap)
        self._keys[galois] = entry
        return entry

    def get_rotation_key_for_limbs(self, rotation: int, cur_limbs: int):
        return self.switch_key(self.galois(rotation), cur_limbs)

    def generate_rotation_keys(self, rotations, cur_limbs: int | None = None) -> None:
        for r in rotations:
            self.switch_key(self.galois(int(r)), self.L if cur_limbs is None else int(cur_limbs))

    def clear_cuda_rotation_cache(self, keep_rotations=()) -> None:
        keep = {self.galois(int(r)) for r in keep_rotations} | {0}
        for g in list(self._keys):
            if g not in keep:
                self.key_bytes -= self._keys[g][0].numel() * 8
                del self._keys[g]

    def check_encode_range(self, wait: bool = True) -> None:
        """Raise if any encode since the last check reached the 2^61 limit.  ``wait``: one device read now (the host
        waits for the stream); else the flag is copied back without waiting and the copy started by the previous
        such call is read if it has landed, so an overflow is reported one check late but the queue never drains."""
        if wait:
            if int(self._flag.item()):
                self._flag.zero_()
                raise ValueError("encoded value exceeds the 2^61 encoder range")
            return
        pending = getattr(self, "_flag_pending", None)
        if pending is not None:
            host, done = pending
            if not done.query():
                return
            self._flag_pending = None
            if int(host[0]):
                self._flag.zero_()
                raise ValueError("encoded value exceeds the 2^61 encoder range")
        host = torch.zeros(1, dtype=torch.int32).pin_memory()
        host.copy_(self._flag, non_blocking=True)
        done = torch.cuda.Event()
        done.record()
        self._flag_pending = (host, done)

    def close(self) -> None:
        if getattr(self, "handle", None) is not None:
            torch.cuda.synchronize(self.device)
            self._keys.clear()
            self._work.clear()
            self._consts.clear()
            self._modup_cache.clear()
            self._modup_by_storage.clear()
            self._modup_cache_bytes = 0
            self.__dict__.pop("_ones_rows", None)
            _lib.call("holmes_ctx_destroy", self.handle)
            self.handle = None

    def __del__(self):  # pragma: no cover - interpreter shutdown order varies
        try:
            self.close()
        except Exception:
            pass


# ----------------------------------------------------------------------------------------------------- encoding


def _as_slots(values, slots: int) -> np.ndarray:
    z = np.asarray(values)
    z = z.astype(np.complex128).reshape(-1)
    if z.size > slots:
        raise ValueError(f"{z.size} values do not fit {slots} slots")
    if z.size < slots:
        z = np.concatenate([z, np.zeros(slots - z.size, dtype=np.complex128)])
    return z


def encode_rows(ctx: Context, rows: torch.Tensor, cur_limbs: int, scale: float, slots: int,
                already_transformed: bool = False, ext: bool = False) -> torch.Tensor:
    """[rows][slots] complex128 (device) -> NTT plaintexts [rows][cur][N] (``ext``: [rows][cur + K][N] over the
    extended basis, the Q limbs first)."""
    if rows.dim() == 1:
        rows = rows.reshape(1, -1)
    nrows = int(rows.shape[0])
    if int(rows.shape[1]) != slots:
        raise ValueError(f"plaintext rows have {rows.shape[1]} slots, expected {slots}")
    z = rows.to(device=ctx.device, dtype=torch.complex128).contiguous()
    if z.data_ptr() == rows.data_ptr() and not already_transformed:
        z = z.clone()
    zr = torch.view_as_real(z)
    limbs = int(cur_limbs) + (ctx.K if ext else 0)
    out = torch.empty((nrows, limbs, ctx.N), dtype=torch.uint64, device=ctx.device)
    if not already_transformed:
        tok = OPTIMER.start("fft_special")
        _lib.call("holmes_fft_special_inv", ctx.handle, zr.data_ptr(), 2 * slots, nrows, slots, _stream())
        OPTIMER.stop(tok, 2 * nrows * slots * 16)
    tok = OPTIMER.start("encode_ntt")
    _lib.call("holmes_encode_fft_ext" if ext else "holmes_encode_fft", ctx.handle, zr.data_ptr(), 2 * slots, nrows,
              slots, float(scale), int(cur_limbs), out.data_ptr(), limbs * ctx.N, ctx._flag.data_ptr(), _stream())
    OPTIMER.stop(tok, nrows * slots * 16 + nrows * limbs * ctx.N * 8)
    return out


def fft_special_inv_rows(ctx: Context, rows: torch.Tensor, slots: int) -> torch.Tensor:
    z = rows.to(device=ctx.device, dtype=torch.complex128).reshape(-1, slots)
    if z.data_ptr() == rows.data_ptr():
        z = z.clone()
    zr = torch.view_as_real(z)
    tok = OPTIMER.start("fft_special")
    _lib.call("holmes_fft_special_inv", ctx.handle, zr.data_ptr(), 2 * slots, int(z.shape[0]), slots, _stream())
    OPTIMER.stop(tok, 2 * int(z.shape[0]) * slots * 16)
    return z


def _fft_special_np(z: np.ndarray, M: int) -> np.ndarray:
    """Forward CKKS embedding (decode) of one slot vector, vectorised per butterfly level."""
    n = z.size
    bits = n.bit_length() - 1
    idx = np.array([int(format(i, f"0{bits}b")[::-1], 2) if bits else 0 for i in range(n)])
    v = z[idx].copy()
    rot = np.array([pow(5, j, M) for j in range(max(1, n // 2))], dtype=np.int64)
    length = 2
    while length <= n:
        half = length // 2
        lenq = length * 4
        k = (rot[:half] % lenq) * (M // lenq)
        w = np.exp(2j * np.pi * k / M)
        v = v.reshape(-1, length)
        u = v[:, :half].copy()
        t = v[:, half:] * w
        v[:, :half] = u + t
        v[:, half:] = u - t
        v = v.reshape(-1)
        length *= 2
    return v


class Client:
    """Secret-key holder of a simulation context (EasyFHE ``client``)."""

    def __init__(self, context: Context) -> None:
        self.context = context

    def encrypt(self, values, device=None, slots: int | None = None, cur_limbs: int | None = None,
                scaling_factor: float | None = None, counter: int | None = None) -> Cipher:
        ctx = self.context
        del device
        slots = ctx.max_slots if slots is None else int(slots)
        cur = ctx.L if cur_limbs is None else int(cur_limbs)
        if not 1 <= cur <= ctx.L:
            raise ValueError(f"cur_limbs={cur} outside [1, {ctx.L}]")
        scale = ctx.scale_at(cur) if scaling_factor is None else float(scaling_factor)
        z = torch.from_numpy(_as_slots(values, slots)).to(ctx.device).reshape(1, slots)
        m = encode_rows(ctx, z, cur, scale, slots)
        ctx.check_encode_range()
        if counter is None:
            counter = ctx._enc_counter
            ctx._enc_counter += 1
        storage = torch.empty((2, 1, cur, ctx.N), dtype=torch.uint64, device=ctx.device)
        _lib.call("holmes_encrypt", ctx.handle, m.data_ptr(), cur, int(counter), storage[0].data_ptr(),
                  storage[1].data_ptr(), _stream())
        return Cipher([storage[0], storage[1]], CipherState(cur, 1, scale), slots, False, 1, ctx)

    def decrypt_coefficients(self, cipher: Cipher, item: int = 0) -> list[int]:
        ctx = self.context
        _valid(ctx, cipher, "decrypt")
        cur = int(cipher.state.cur_limbs)
        c0 = cipher.cv[0][item, :cur].contiguous()
        c1 = cipher.cv[1][item, :cur].contiguous()
        out = torch.empty((cur, ctx.N), dtype=torch.uint64, device=ctx.device)
        _lib.call("holmes_decrypt", ctx.handle, c0.data_ptr(), c1.data_ptr(), cur, out.data_ptr(), _stream())
        res = out.cpu().numpy()
        use = min(cur, 4)
        moduli = [ctx.q(i) for i in range(use)]
        Q = math.prod(moduli)
        acc = np.zeros(ctx.N, dtype=object)
        for i, qi in enumerate(moduli):
            hat = Q // qi
            inv = pow(hat % qi, -1, qi)
            acc = acc + ((res[i].astype(object) * inv) % qi) * hat
        acc = acc % Q
        return [int(v) - Q if int(v) > Q // 2 else int(v) for v in acc]

    def decrypt(self, cipher: Cipher, item: int = 0) -> np.ndarray:
        ctx = self.context
        coeffs = np.array([float(v) for v in self.decrypt_coefficients(cipher, item)], dtype=np.float64)
        slots = int(cipher.slots)
        gap = ctx.N // (2 * slots)
        scale = float(cipher.state.scaling_factor)
        z = coeffs[0:ctx.N // 2:gap][:slots] / scale + 1j * coeffs[ctx.N // 2::gap][:slots] / scale
        return _fft_special_np(z, ctx.M)


def generate_client_context(spec: CKKSContextSpec, device: str = "cuda"):
    ctx = Context(spec, device)
    if spec.auto_load_keys:   # eager: every requested key now, at its configured limit (else the full chain)
        for r in spec.rotations:
            g = ctx.galois(int(r))
            ctx.switch_key(g, ctx.key_limit(g) or ctx.L)
        if spec.relinearization:
            ctx.switch_key(0, ctx.L)
    return Client(ctx), ctx


# ----------------------------------------------------------------------------------------------------- helpers


def _new_cipher(ctx: Context, batch: int, limbs: int, state: CipherState, slots: int, comps: int = 2) -> Cipher:
    storage = torch.empty((comps, batch, limbs, ctx.N), dtype=torch.uint64, device=ctx.device)
    return Cipher([storage[c] for c in range(comps)], state, slots, False, batch, ctx)


def _item_stride(t: torch.Tensor) -> int:
    return int(t.stride(0))


def _check_same(a: Cipher, b: Cipher, what: str) -> None:
    if int(a.state.cur_limbs) != int(b.state.cur_limbs):
        raise ValueError(f"{what}: limb mismatch {a.state.cur_limbs} != {b.state.cur_limbs}")
    if int(a.state.scale_degree) != int(b.state.scale_degree):
        raise ValueError(f"{what}: scale degree mismatch {a.state.scale_degree} != {b.state.scale_degree}")
    if a.is_ext or b.is_ext:
        raise ValueError(f"{what}: extended ciphertexts are not supported")
    if a.batch_size != b.batch_size:
        raise ValueError(f"{what}: batch mismatch {a.batch_size} != {b.batch_size}")


def _valid(ctx: Context, a: Cipher, what: str) -> None:
    """Refuse, before any launch, a cipher or plaintext whose storage the kernels would read out of bounds or from the
    wrong device: every component must be a uint64 CUDA tensor on the context's device, [batch][>= limbs][N] with unit
    word stride and limb stride N (limbs = cur, or cur + K for the extended basis)."""
    limbs = int(a.state.cur_limbs) + (ctx.K if a.is_ext else 0)
    for c, t in enumerate(a.cv):
        if not torch.is_tensor(t) or t.device.type != "cuda" or t.device.index != ctx.device.index:
            raise ValueError(f"{what}: component {c} is not on {ctx.device}")
        if t.dtype != torch.uint64 or t.dim() != 3:
            raise ValueError(f"{what}: component {c} must be a uint64 [batch][limbs][N] tensor")
        if int(t.shape[0]) < int(a.batch_size) or int(t.shape[1]) < limbs or int(t.shape[2]) != ctx.N:
            raise ValueError(f"{what}: component {c} of shape {tuple(t.shape)} cannot hold {a.batch_size} x {limbs} "
                             f"limbs of {ctx.N} words")
        if int(t.stride(2)) != 1 or int(t.stride(1)) != ctx.N:
            raise ValueError(f"{what}: component {c} needs unit word stride and limb stride N")


def _ew(ctx: Context, op: int, a: torch.Tensor, b: torch.Tensor | None, out: torch.Tensor, limbs: int) -> None:
    _lib.call("holmes_elementwise", ctx.handle, op, a.data_ptr(), 0 if b is None else b.data_ptr(), out.data_ptr(),
              int(a.shape[0]), int(limbs), _item_stride(a), 0 if b is None else _item_stride(b), _item_stride(out),
              _stream())


def _run(cv, batch: int):
    """(first component, items, item stride) when the components lie one after another at one item stride (a cipher
    from ``_new_cipher``, or limb views of one), so that one launch over ``len(cv) * batch`` items serves them all;
    else None."""
    t0 = cv[0]
    st = int(t0.stride(0))
    base = t0.data_ptr()
    for c in range(1, len(cv)):
        t = cv[c]
        if int(t.stride(0)) != st or t.data_ptr() != base + c * batch * st * 8:
            return None
    return t0, len(cv) * batch, st


def _runs(batch: int, *cvs):
    """Per launch, one (tensor, items, item stride) per operand: a single launch when every operand's components
    form a run (``_run``), else one launch per component."""
    runs = [_run(cv, batch) for cv in cvs]
    if all(r is not None for r in runs):
        return [runs]
    return [[(cv[c], batch, int(cv[c].stride(0))) for cv in cvs] for c in range(len(cvs[0]))]


def _ew_cv(ctx: Context, op: int, a_cv, b_cv, out_cv, batch: int, limbs: int) -> None:
    """``_ew`` over every component (op 3, negation, takes no ``b_cv``)."""
    if b_cv is None:
        for (a, items, ai), (o, _, oi) in _runs(batch, a_cv, out_cv):
            _lib.call("holmes_elementwise", ctx.handle, op, a.data_ptr(), 0, o.data_ptr(), items, int(limbs), ai, 0, oi,
                      _stream())
        return
    for (a, items, ai), (b, _, bi), (o, _, oi) in _runs(batch, a_cv, b_cv, out_cv):
        _lib.call("holmes_elementwise", ctx.handle, op, a.data_ptr(), b.data_ptr(), o.data_ptr(), items, int(limbs), ai,
                  bi, oi, _stream())


CONST_ADD, CONST_MUL, CONST_AXPY = 0, 1, 2
_CONST_LIMBS = 64


def const_cv(ctx: Context, op: int, a_cv, residues, out_cv, batch: int, limbs: int) -> None:
    """Per-limb scalar op over every component: CONST_ADD out = a + k, CONST_MUL out = a * k, CONST_AXPY out += a * k
    (``residues`` the host list k[0 .. limbs-1]; passed by value to the kernel, no device copy)."""
    limbs = int(limbs)
    if limbs > _CONST_LIMBS:   # beyond the launch-parameter table: the device-table kernels
        if op == CONST_AXPY:
            raise ValueError(f"scalar multiply-accumulate supports at most {_CONST_LIMBS} limbs")
        k = ctx.device_u64(list(residues)[:limbs])
        name = "holmes_add_const" if op == CONST_ADD else "holmes_mul_const"
        for (a, items, ai), (o, _, oi) in _runs(batch, a_cv, out_cv):
            _lib.call(name, ctx.handle, a.data_ptr(), k.data_ptr(), o.data_ptr(), items, limbs, ai, oi, _stream())
        return
    host = (_lib.ctypes.c_uint64 * limbs)(*[int(v) for v in list(residues)[:limbs]])
    for (a, items, ai), (o, _, oi) in _runs(batch, a_cv, out_cv):
        _lib.call("holmes_const_op", ctx.handle, int(op), a.data_ptr(), host, o.data_ptr(), items, limbs, ai, oi,
                  _stream())


def _ctx(ctx) -> Context:
    return ctx.context if hasattr(ctx, "context") and isinstance(ctx.context, Context) else ctx


# ----------------------------------------------------------------------------------------------------- ops


def _add_sub(a: Cipher, b: Cipher, ctx, op: int, what: str) -> Cipher:
    """a + b (op 0) or a - b (op 1), component by component.  Either may be an unrelinearised three-component
    product (the lazy accumulators of ``homo_mul_no_relin``); a component only one operand has is copied (negated
    for the subtrahend)."""
    ctx = _ctx(ctx)
    _valid(ctx, a, what)
    _valid(ctx, b, what)
    # operands at different levels meet at the lower one (the deeper operand's extra limbs are dropped; at a
    # fixed nominal scale per level that is exact), as EasyFHE's adds do
    cur = min(int(a.state.cur_limbs), int(b.state.cur_limbs))
    low = a if int(a.state.cur_limbs) == cur else b
    _check_same(_drop_limbs(a, cur), _drop_limbs(b, cur), what)
    na, nb = len(a.cv), len(b.cv)
    out = _new_cipher(ctx, a.batch_size, cur, low.state, a.slots, max(na, nb))
    if na == nb:
        _ew_cv(ctx, op, a.cv, b.cv, out.cv, a.batch_size, cur)
        return out
    for c in range(max(na, nb)):
        if c < na and c < nb:
            _ew(ctx, op, a.cv[c], b.cv[c], out.cv[c], cur)
        elif c < na:
            out.cv[c].copy_(a.cv[c][:, :cur])
        elif op == 1:
            _ew(ctx, 3, b.cv[c], None, out.cv[c], cur)
        else:
            out.cv[c].copy_(b.cv[c][:, :cur])
    return out


def homo_add(a: Cipher, b: Cipher, ctx) -> Cipher:
    return _add_sub(a, b, ctx, 0, "homo_add")


def homo_sub(a: Cipher, b: Cipher, ctx) -> Cipher:
    return _add_sub(a, b, ctx, 1, "homo_sub")


def homo_mul_i(a: Cipher, ctx, negative: bool = False) -> Cipher:
    """a * i (a * X^(N/2)); ``negative``: a * (-i)."""
    ctx = _ctx(ctx)
    _valid(ctx, a, "homo_mul_i")
    cur = int(a.state.cur_limbs)
    out = _new_cipher(ctx, a.batch_size, cur, a.state, a.slots, len(a.cv))
    for (x, items, xi), (o, _, oi) in _runs(a.batch_size, a.cv, out.cv):
        _lib.call("holmes_mul_i", ctx.handle, x.data_ptr(), o.data_ptr(), items, cur, xi, oi, _stream())
    if negative:
        _ew_cv(ctx, 3, out.cv, None, out.cv, a.batch_size, cur)
    return out


def rescale(a: Cipher, ctx) -> Cipher:
    ctx = _ctx(ctx)
    _valid(ctx, a, "rescale")
    cur = int(a.state.cur_limbs)
    if cur < 2:
        raise ValueError(f"rescale: cur_limbs must be > 1, got {cur}")
    ql = ctx.q(cur - 1)
    sf = None if a.state.scaling_factor is None else float(a.state.scaling_factor) / ql
    state = CipherState(cur - 1, max(1, int(a.state.scale_degree) - 1), sf)
    out = _new_cipher(ctx, a.batch_size, cur - 1, state, a.slots)
    scratch = ctx.workspace("rescale", 2 * a.batch_size * ctx.N)
    tok = OPTIMER.start("rescale")
    for (x, items, xi), (o, _, oi) in _runs(a.batch_size, a.cv[:2], out.cv):
        _lib.call("holmes_rescale", ctx.handle, x.data_ptr(), xi, o.data_ptr(), oi, cur, items, scratch.data_ptr(),
                  _stream())
    OPTIMER.stop(tok, 2 * a.batch_size * (2 * cur - 1) * ctx.N * 8)
    return out


def align_to(a: Cipher, target: CipherState, ctx) -> Cipher:
    """Bring ``a`` to ``target``: rescale while its degree is above the target's, then drop limbs."""
    ctx = _ctx(ctx)
    _valid(ctx, a, "align_to")
    cur = a
    while int(cur.state.scale_degree) > int(target.scale_degree):
        cur = rescale(cur, ctx)
    want = int(target.cur_limbs)
    have = int(cur.state.cur_limbs)
    if want > have:
        raise ValueError(f"align_to: cannot raise {have} limbs to {want}")
    if want == have:   # a distinct object the caller owns (releasing it must not release ``a``)
        return cur if cur is not a else a.cipher_like([c.clone() for c in a.cv])
    state = cur.state.replace(cur_limbs=want)
    return cur.cipher_like([c[:, :want].contiguous() for c in cur.cv], state=state)


def _modup(ctx: Context, c1: torch.Tensor, cur: int, items: int, reuse: bool = False) -> tuple[torch.Tensor, int]:
    """The ModUp digits of ``c1`` (its first ``cur`` limbs, ``items`` items).  Digits of a recent input are reused:
    the reference rotates one ciphertext by many offsets one call at a time (attention's per-head rotations), and
    every such rotation needs the same digits.  An input is the same when its memory, item stride, level, item count
    and torch version counter (bumped by every in-place torch write, shared by all views) are; the cache holds the
    input tensor, so its memory cannot be handed to another tensor while the entry lives, and the engine's own calls
    that write into caller-provided buffers drop the entries they overlap (``_modup_forget``).  ``reuse`` marks a
    call whose digits are worth keeping (a rotation of a caller's ciphertext, which may be rotated again); the
    third component of a product, relinearised once, is looked up but not kept."""
    dig_item = ctx.beta(cur) * (cur + ctx.K) * ctx.N
    key = (c1.data_ptr(), int(c1._version), int(c1.stride(0)), int(cur), int(items))
    hit = ctx._modup_cache.get(key)
    if hit is not None and hit[0].untyped_storage().data_ptr() == c1.untyped_storage().data_ptr():
        ctx._modup_cache.move_to_end(key)
        return hit[1], dig_item
    digits = torch.empty(items * dig_item, dtype=torch.uint64, device=ctx.device)
    scratch = ctx.workspace("modup", items * cur * ctx.N)
    tok = OPTIMER.start("modup")
    _lib.call("holmes_modup", ctx.handle, c1.data_ptr(), _item_stride(c1), cur, items, digits.data_ptr(), dig_item,
              scratch.data_ptr(), _stream())
    OPTIMER.stop(tok, items * (cur + dig_item // ctx.N) * ctx.N * 8)
    nbytes = int(digits.numel()) * 8
    if reuse and nbytes <= MODUP_CACHE_BYTES // 4:
        cache = ctx._modup_cache
        sp = c1.untyped_storage().data_ptr()
        cache[key] = (c1, digits, nbytes, sp)
        ctx._modup_by_storage.setdefault(sp, set()).add(key)
        ctx._modup_cache_bytes += nbytes
        while ctx._modup_cache_bytes > MODUP_CACHE_BYTES:
            _modup_drop(ctx, next(iter(cache)))
    return digits, dig_item


def _modup_drop(ctx: Context, key) -> None:
    entry = ctx._modup_cache.pop(key)
    ctx._modup_cache_bytes -= entry[2]
    keys = ctx._modup_by_storage.get(entry[3])
    if keys is not None:
        keys.discard(key)
        if not keys:
            del ctx._modup_by_storage[entry[3]]


#: device bytes of ModUp digits kept for reuse per context
MODUP_CACHE_BYTES = 2 << 30


def _modup_forget(ctx: Context, *tensors) -> None:
    """Drop the cached digits of every input that shares storage with one of ``tensors`` (about to be written by a raw
    kernel launch, which torch's version counter does not see); memory of different storages never overlaps."""
    if not ctx._modup_cache:
        return
    for t in tensors:
        if t is None:
            continue
        for key in list(ctx._modup_by_storage.get(t.untyped_storage().data_ptr(), ())):
            _modup_drop(ctx, key)


def _keyswitch(ctx: Context, digits: torch.Tensor, dig_item: int, cur: int, galois: int, key, add0, add1, add_item,
               out0: torch.Tensor, out1: torch.Tensor, items: int, post0=None, post1=None, post_item: int = 0,
               workspace: str = "ks") -> None:
    key_t, cap = key
    scratch = ctx.workspace(workspace, items * 2 * (ctx.K + cur) * ctx.N)
    beta = ctx.beta(cur)
    words = items * (beta * (cur + ctx.K) + 2 * cur) + 2 * beta * (cur + ctx.K)
    words += items * cur * ((add0 is not None) + (add1 is not None) + (post0 is not None) + (post1 is not None))
    tok = OPTIMER.start("keyswitch")
    _lib.call("holmes_keyswitch", ctx.handle, digits.data_ptr(), dig_item, cur, key_t.data_ptr(), cap, int(galois),
              0 if add0 is None else add0.data_ptr(), 0 if add1 is None else add1.data_ptr(), int(add_item),
              0 if post0 is None else post0.data_ptr(), 0 if post1 is None else post1.data_ptr(), int(post_item),
              out0.data_ptr(), out1.data_ptr(), _item_stride(out0), items, scratch.data_ptr(), _stream())
    OPTIMER.stop(tok, words * ctx.N * 8)


def rotate_batch(ctx: Context, c0: torch.Tensor, c1: torch.Tensor, cur: int, rotation: int, out0: torch.Tensor,
                 out1: torch.Tensor, post0=None, post1=None, reuse: bool = True) -> None:
    """out = rot((c0, c1), rotation) [+ post] for a batch [items][>= cur][N] sharing one key.  ``reuse``: keep the
    input's ModUp digits for further rotations of it (off for one-off intermediates such as a Horner accumulator)."""
    items = int(c0.shape[0])
    g = ctx.galois(rotation)
    _modup_forget(ctx, out0, out1)
    if g == 1:
        if post0 is None:
            out0.copy_(c0[:, :cur])
            out1.copy_(c1[:, :cur])
        else:
            _ew(ctx, 0, c0, post0, out0, cur)
            _ew(ctx, 0, c1, post1, out1, cur)
        return
    digits, dig_item = _modup(ctx, c1, cur, items, reuse)
    _keyswitch(ctx, digits, dig_item, cur, g, ctx.switch_key(g, cur), c0, None, _item_stride(c0), out0, out1, items,
               post0, post1, 0 if post0 is None else _item_stride(post0))


def homo_rotate(a: Cipher, rotation: int, ctx) -> Cipher:
    ctx = _ctx(ctx)
    _valid(ctx, a, "homo_rotate")
    cur = int(a.state.cur_limbs)
    out = _new_cipher(ctx, a.batch_size, cur, a.state, a.slots)
    rotate_batch(ctx, a.cv[0], a.cv[1], cur, int(rotation), out.cv[0], out.cv[1])
    return out


def fast_rotate(a: Cipher, rotations, ctx, output_ext: bool = False) -> Cipher:
    """One rotation (an int: ``homo_rotate``) or, for a sequence of offsets, the batch ``[len(offsets)]`` of
    rotations from one hoisted ModUp (the reference's use: ``operators/linear/shifted_lane.py:75-76``, unpacked
    with ``unpack_cipher_batch``).  Residue-identical to rotating one at a time.

    ``output_ext`` (``operators/attention/prefill/input.py:1200-1205``): the rotations stay in the extended basis
    Q u P, before their ModDown -- ``(P perm(c0) + <perm(d), key_b>, <perm(d), key_a>)`` over ``cur + K`` limbs,
    ``is_ext`` set -- so that a multiply-accumulate over them (``grouped_pairwise_mac``) pays one ModDown
    (``moddown_from_ext``) instead of one per rotation.  ``moddown_from_ext`` of one is ``homo_rotate``, word for word."""
    if isinstance(rotations, (int, np.integer)):
        rotations = (int(rotations),)
        single = True
    else:
        single = False
    if not output_ext:
        if single:
            return homo_rotate(a, rotations[0], ctx)
        return prepare_hoisted_baby_rotations(a, tuple(int(r) for r in rotations), ctx)[0]
    ctx = _ctx(ctx)
    _valid(ctx, a, "fast_rotate")
    if a.batch_size != 1 or a.is_ext:
        raise ValueError("fast_rotate(output_ext=True) expects one non-extended ciphertext")
    cur = int(a.state.cur_limbs)
    offsets = [int(r) for r in rotations]
    block = _new_cipher(ctx, len(offsets), cur + ctx.K, a.state, a.slots)
    block.is_ext = True
    switches = []
    for b, off in enumerate(offsets):
        g = ctx.galois(off)
        if g == 1:   # (P c0, P c1): P is 0 modulo the special primes
            pm = ctx.p_mod_q_dev(cur)
            for c in range(2):
                block.cv[c][b, cur:].zero_()
                _lib.call("holmes_mul_const", ctx.handle, a.cv[c][:1, :cur].data_ptr(), pm.data_ptr(),
                          block.cv[c][b:b + 1].data_ptr(), 1, cur, _item_stride(a.cv[c]), _item_stride(block.cv[c]),
                          _stream())
        else:
            switches.append((b, g, ctx.switch_key(g, cur)))
    if not switches:
        return block
    digits, dig_item = _modup(ctx, a.cv[1], cur, 1, True)
    lanes = _ks_lanes(ctx, len(switches))        # independent key switches: the caller's and side streams
    for i, (b, g, (key_t, cap)) in enumerate(switches):
        with torch.cuda.stream(lanes[i % len(lanes)]):
            _lib.call("holmes_keyswitch_ext", ctx.handle, digits.data_ptr(), dig_item, cur, key_t.data_ptr(), cap,
                      int(g), a.cv[0].data_ptr(), _item_stride(a.cv[0]), block.cv[0][b:b + 1].data_ptr(),
                      block.cv[1][b:b + 1].data_ptr(), _item_stride(block.cv[0]), 1, _stream())
    _ks_join(lanes)
    return block


def moddown_from_ext(a: Cipher, ctx) -> Cipher:
    """ModDown of an extended-basis ciphertext (``is_ext``, ``cur + K`` limbs) back to its ``cur`` Q limbs."""
    ctx = _ctx(ctx)
    _valid(ctx, a, "moddown_from_ext")
    if not a.is_ext:
        raise ValueError("moddown_from_ext expects an extended-basis ciphertext")
    cur = int(a.state.cur_limbs)
    out = _new_cipher(ctx, a.batch_size, cur, a.state, a.slots)
    scratch = ctx.workspace("ks", a.batch_size * 2 * (ctx.K + cur) * ctx.N)
    _lib.call("holmes_moddown", ctx.handle, a.cv[0].data_ptr(), a.cv[1].data_ptr(), _item_stride(a.cv[0]), cur,
              out.cv[0].data_ptr(), out.cv[1].data_ptr(), _item_stride(out.cv[0]), a.batch_size, scratch.data_ptr(),
              _stream())
    return out


def grouped_pairwise_mac(batch: Cipher, plaintexts: Plaintext, groups: int, ctx) -> Cipher:
    """``out[g] = sum_b plaintexts[g B + b] * batch[b]`` for a batch of B ciphertexts and ``groups * B`` plaintext
    rows, a ``groups``-item batch (the reference's attention transforms call it with one group,
    ``operators/attention/prefill/input.py:1019-1021``).  Extended-basis inputs (``is_ext``, e.g. from
    ``fast_rotate(output_ext=True)``) need extended plaintexts (``Session.plaintext(..., is_ext=True)``) and give an
    extended result."""
    ctx = _ctx(ctx)
    _valid(ctx, batch, "grouped_pairwise_mac")
    _valid(ctx, plaintexts, "grouped_pairwise_mac")
    groups = int(groups)
    nb = int(batch.batch_size)
    cur = int(batch.state.cur_limbs)
    pv = plaintexts.cv[0]
    if int(pv.shape[0]) != groups * nb:
        raise ValueError(f"grouped_pairwise_mac: {pv.shape[0]} plaintext rows for {groups} groups of {nb}")
    if bool(batch.is_ext) != bool(plaintexts.is_ext):
        raise ValueError("grouped_pairwise_mac: ciphertexts and plaintexts must both be extended or both not")
    limbs = cur + (ctx.K if batch.is_ext else 0)
    if int(pv.shape[1]) < limbs or int(plaintexts.state.cur_limbs) < cur:
        raise ValueError("grouped_pairwise_mac: plaintexts have fewer limbs than the ciphertexts")
    sf = None
    if batch.state.scaling_factor is not None and plaintexts.state.scaling_factor is not None:
        sf = float(batch.state.scaling_factor) * float(plaintexts.state.scaling_factor)
    state = CipherState(cur, int(batch.state.scale_degree) + int(plaintexts.state.scale_degree), sf)
    res = torch.empty((2, groups, 1, limbs, ctx.N), dtype=torch.uint64, device=ctx.device)
    c0s = _lib.ptr_array([batch.cv[0].data_ptr()])
    c1s = _lib.ptr_array([batch.cv[1].data_ptr()])
    if batch.is_ext:
        _lib.call("holmes_bsgs_mac_ext", ctx.handle, res.data_ptr(), c0s, c1s, _item_stride(batch.cv[0]), nb, 1,
                  pv.data_ptr(), _item_stride(pv), groups, cur, _stream())
    else:
        _lib.call("holmes_bsgs_mac", ctx.handle, res.data_ptr(), c0s, c1s, _item_stride(batch.cv[0]), nb, 1,
                  pv.data_ptr(), _item_stride(pv), groups, cur, _stream())
    return Cipher([res[0, :, 0], res[1, :, 0]], state, batch.slots, bool(batch.is_ext), groups, ctx)


def pack_cipher_batch(ciphers) -> Cipher:
    """One batch cipher from single (or batch) ciphers of one level, scale and slot count, items in order."""
    ciphers = tuple(ciphers)
    if not ciphers:
        raise ValueError("pack_cipher_batch needs at least one cipher")
    first = ciphers[0]
    cur = int(first.state.cur_limbs)
    for c in ciphers[1:]:
        if int(c.state.cur_limbs) != cur or int(c.state.scale_degree) != int(first.state.scale_degree) \
                or c.slots != first.slots or c.is_ext != first.is_ext or len(c.cv) != len(first.cv):
            raise ValueError("pack_cipher_batch: ciphers differ in level, scale degree, slots or form")
    limbs = cur + (int(first.context.K) if first.is_ext else 0)
    total = sum(int(c.batch_size) for c in ciphers)
    first_t = first.cv[0]
    # the components one after another in one storage: later element-wise launches cover them in one go
    storage = torch.empty((len(first.cv), total, limbs, int(first_t.shape[2])), dtype=first_t.dtype,
                          device=first_t.device)
    for k in range(len(first.cv)):
        torch.cat([c.cv[k][:int(c.batch_size), :limbs] for c in ciphers], dim=0, out=storage[k])
    return first.cipher_like([storage[k] for k in range(len(first.cv))], batch_size=total)


def unpack_cipher_batch(batch: Cipher) -> tuple:
    """The items of a batch cipher as single ciphers (views of the batch storage)."""
    return tuple(batch.cipher_like([c[i:i + 1] for c in batch.cv], batch_size=1) for i in range(batch.batch_size))


def prepare_hoisted_baby_rotations(a: Cipher, baby_offsets, ctx, strategy: str = "normal",
                                   baby_anchor_step: int = -1):
    """Baby basis rot(a, offset) for every offset from one hoisted ModUp; one block ``[nb]`` batch.  ``ext_normal``
    and ``ext_double_hoist`` keep the block over the extended basis Q u P (``fast_rotate(output_ext=True)``)."""
    del baby_anchor_step
    strategy = str(strategy).lower()
    if strategy in ("ext_normal", "ext_double_hoist"):
        return (fast_rotate(a, tuple(int(o) for o in baby_offsets), ctx, output_ext=True),)
    if strategy != "normal":
        raise ValueError(f"unknown hoist strategy {strategy!r}")
    ctx = _ctx(ctx)
    _valid(ctx, a, "prepare_hoisted_baby_rotations")
    if a.batch_size != 1:
        raise ValueError("prepare_hoisted_baby_rotations expects one ciphertext")
    offsets = [int(o) for o in baby_offsets]
    cur = int(a.state.cur_limbs)
    block = _new_cipher(ctx, len(offsets), cur, a.state, a.slots)
    switches = []
    for b, off in enumerate(offsets):
        g = ctx.galois(off)
        if g == 1:
            block.cv[0][b].copy_(a.cv[0][0, :cur])
            block.cv[1][b].copy_(a.cv[1][0, :cur])
        else:
            switches.append((b, g, ctx.switch_key(g, cur)))   # keys fetched (or generated) on the caller's stream
    if not switches:
        return (block,)
    digits, dig_item = _modup(ctx, a.cv[1], cur, 1, True)
    # The offsets' key switches are independent (one ciphertext's key switch fills less than the GPU): they run on
    # the caller's stream and KS_STREAMS - 1 side streams, each with its own scratch, after the ModUp; the caller's
    # stream waits for all of them before returning, so every later use of the block is ordered after them.
    lanes = _ks_lanes(ctx, len(switches))
    for i, (b, g, key) in enumerate(switches):
        k = i % len(lanes)
        with torch.cuda.stream(lanes[k]):
            _keyswitch(ctx, digits, dig_item, cur, g, key, a.cv[0], None, 0, block.cv[0][b:b + 1],
                       block.cv[1][b:b + 1], 1, workspace=f"ks{k}")
    _ks_join(lanes)
    return (block,)


#: streams the independent key switches of one hoisted rotation set are spread over (the caller's and side streams)
KS_STREAMS = 4


def _ks_lanes(ctx: Context, jobs: int) -> list:
    """The caller's stream, then side streams (created once per context) that first wait for everything the caller's
    stream has queued."""
    main = torch.cuda.current_stream(ctx.device)
    n = max(1, min(int(KS_STREAMS), int(jobs)))
    if n == 1 or OPTIMER.enabled:   # the per-family timers measure each key switch alone
        return [main]
    side = ctx.__dict__.get("_side_streams")
    if side is None:
        side = ctx._side_streams = [torch.cuda.Stream(device=ctx.device) for _ in range(int(KS_STREAMS) - 1)]
    lanes = [main] + side[:n - 1]
    for s in lanes[1:]:
        s.wait_stream(main)
    return lanes


def _ks_join(lanes: list) -> None:
    for s in lanes[1:]:
        lanes[0].wait_stream(s)


def bsgs_partial_sums(ctx: Context, baby_blocks, plaintexts: Plaintext, giants: int) -> torch.Tensor:
    """res [2][giants][inputs][cur][N] = sum_b pt[g B + b] * baby_i[b] for every input's baby block (extended
    blocks and plaintexts: [cur + K] limbs, over Q u P)."""
    blocks = list(baby_blocks)
    cur = int(blocks[0].state.cur_limbs)
    nb = int(blocks[0].batch_size)
    ext = bool(blocks[0].is_ext)
    if ext != bool(plaintexts.is_ext):
        raise ValueError("bsgs_partial_sums: babies and plaintexts must both be extended or both not")
    limbs = cur + (ctx.K if ext else 0)
    pv = plaintexts.cv[0]
    if int(pv.shape[0]) != giants * nb:
        raise ValueError(f"plaintext chunk has {pv.shape[0]} rows, expected {giants} x {nb}")
    if int(plaintexts.state.cur_limbs) < cur or int(pv.shape[1]) < limbs:
        raise ValueError("plaintext chunk has fewer limbs than the baby basis")
    res = torch.empty((2, giants, len(blocks), limbs, ctx.N), dtype=torch.uint64, device=ctx.device)
    bstride = _item_stride(blocks[0].cv[0])
    c0s = _lib.ptr_array([b.cv[0].data_ptr() for b in blocks])
    c1s = _lib.ptr_array([b.cv[1].data_ptr() for b in blocks])
    tok = OPTIMER.start("bsgs_mac")
    _lib.call("holmes_bsgs_mac_ext" if ext else "holmes_bsgs_mac", ctx.handle, res.data_ptr(), c0s, c1s, bstride, nb,
              len(blocks), pv.data_ptr(), _item_stride(pv), giants, cur, _stream())
    OPTIMER.stop(tok, (giants * nb + len(blocks) * nb * 2 + 2 * giants * len(blocks)) * cur * ctx.N * 8)
    return res


def giant_horner(ctx: Context, res: torch.Tensor, giant_offset: int) -> tuple[torch.Tensor, torch.Tensor]:
    """acc = res[G-1]; acc = rot(acc, giant_offset) + res[g] for g = G-2 .. 0 (all inputs at once)."""
    G = int(res.shape[1])
    cur = int(res.shape[3])
    acc0, acc1 = res[0, G - 1], res[1, G - 1]
    for g in range(G - 2, -1, -1):
        n0 = torch.empty_like(acc0)
        n1 = torch.empty_like(acc1)
        rotate_batch(ctx, acc0, acc1, cur, giant_offset, n0, n1, post0=res[0, g], post1=res[1, g], reuse=False)
        acc0, acc1 = n0, n1
    return acc0, acc1


def giant_double_hoist(ctx: Context, res: torch.Tensor, giant_offset: int) -> tuple[torch.Tensor, torch.Tensor]:
    """sum_g rot(res[g], g giant_offset) for res [2][G][items][cur][N], double hoisted (the ``ext_double_hoist``
    strategy, whose key set has every local giant offset, ``operators/linear/config.py:354-359``): each giant's
    key switch stays over Q u P (``holmes_keyswitch_ext``; giant 0 lifted as (P c0, P c1)), the G results are summed
    over Q u P by one multiply-accumulate launch against a plaintext of ones, and ONE ModDown brings the sum back,
    where the Horner chain pays a ModDown per giant."""
    G, items, cur = int(res.shape[1]), int(res.shape[2]), int(res.shape[3])
    K, N = ctx.K, ctx.N
    ext = torch.empty((2, G, items, cur + K, N), dtype=torch.uint64, device=ctx.device)
    pm = ctx.p_mod_q_dev(cur)
    for c in range(2):
        ext[c, 0, :, cur:].zero_()
        _lib.call("holmes_mul_const", ctx.handle, res[c, 0].data_ptr(), pm.data_ptr(), ext[c, 0].data_ptr(), items,
                  cur, cur * N, (cur + K) * N, _stream())
    for g in range(1, G):
        gal = ctx.galois(g * int(giant_offset))
        c0, c1 = res[0, g], res[1, g]
        digits, dig_item = _modup(ctx, c1, cur, items)
        key_t, cap = ctx.switch_key(gal, cur)
        tok = OPTIMER.start("keyswitch")
        _lib.call("holmes_keyswitch_ext", ctx.handle, digits.data_ptr(), dig_item, cur, key_t.data_ptr(), cap, int(gal),
                  c0.data_ptr(), _item_stride(c0), ext[0, g].data_ptr(), ext[1, g].data_ptr(), (cur + K) * N, items,
                  _stream())
        OPTIMER.stop(tok, items * (ctx.beta(cur) * (cur + K) + 3 * cur + 2 * K) * N * 8)
    cache = ctx.__dict__.setdefault("_ones_rows", {})   # the all-ones plaintext, kept per (G, limbs)
    ones = cache.get((G, cur + K))
    if ones is None:
        ones = cache[(G, cur + K)] = torch.ones((G, cur + K, N), dtype=torch.uint64, device=ctx.device)
    summed = torch.empty((2, 1, items, cur + K, N), dtype=torch.uint64, device=ctx.device)
    c0s = _lib.ptr_array([ext[0, 0, i].data_ptr() for i in range(items)])
    c1s = _lib.ptr_array([ext[1, 0, i].data_ptr() for i in range(items)])
    _lib.call("holmes_bsgs_mac_ext", ctx.handle, summed.data_ptr(), c0s, c1s, items * (cur + K) * N, G, items,
              ones.data_ptr(), (cur + K) * N, 1, cur, _stream())
    out = torch.empty((2, items, cur, N), dtype=torch.uint64, device=ctx.device)
    scratch = ctx.workspace("ks", items * 2 * (K + cur) * N)
    _lib.call("holmes_moddown", ctx.handle, summed[0, 0].data_ptr(), summed[1, 0].data_ptr(), (cur + K) * N, cur,
              out[0].data_ptr(), out[1].data_ptr(), cur * N, items, scratch.data_ptr(), _stream())
    return out[0], out[1]


def hoisted_mac_sum(cipher: Cipher, baby_offsets, plaintexts: Plaintext, giant_offset: int, giant_count: int, ctx,
                    strategy: str = "normal", baby_anchor_step: int = -1, baby_rotations=None) -> Cipher:
    """sum_g rot(sum_b pt[g B + b] baby[b], g giant_offset) via Horner (``ext_double_hoist``: every giant rotated
    directly over Q u P and one ModDown of the sum); scale degree adds the plaintext's."""
    ctx = _ctx(ctx)
    _valid(ctx, cipher, "hoisted_mac_sum")
    _valid(ctx, plaintexts, "hoisted_mac_sum")
    if baby_rotations is None:
        baby_rotations = prepare_hoisted_baby_rotations(cipher, baby_offsets, ctx, strategy, baby_anchor_step)
    block = baby_rotations[0]
    res = bsgs_partial_sums(ctx, [block], plaintexts, int(giant_count))
    if block.is_ext:   # one ModDown per giant partial, then the plain Horner chain
        down = moddown_from_ext(Cipher([res[0, :, 0], res[1, :, 0]], block.state, block.slots, True,
                                       int(giant_count), ctx), ctx)
        res = torch.stack([down.cv[0], down.cv[1]]).unsqueeze(2)
    if str(strategy).lower() == "ext_double_hoist":
        acc0, acc1 = giant_double_hoist(ctx, res, int(giant_offset))
    else:
        acc0, acc1 = giant_horner(ctx, res, int(giant_offset))
    sf = None
    if block.state.scaling_factor is not None and plaintexts.state.scaling_factor is not None:
        sf = float(block.state.scaling_factor) * float(plaintexts.state.scaling_factor)
    state = CipherState(int(block.state.cur_limbs),
                        int(block.state.scale_degree) + int(plaintexts.state.scale_degree), sf)
    return Cipher([acc0, acc1], state, cipher.slots, False, 1, ctx)


def homo_mul_pt(a: Cipher, pt: Plaintext, ctx) -> Cipher:
    ctx = _ctx(ctx)
    _valid(ctx, a, "homo_mul_pt")
    _valid(ctx, pt, "homo_mul_pt")
    cur = int(a.state.cur_limbs)
    if int(pt.state.cur_limbs) < cur:
        raise ValueError("homo_mul_pt: plaintext has fewer limbs than the ciphertext")
    sf = None
    if a.state.scaling_factor is not None and pt.state.scaling_factor is not None:
        sf = float(a.state.scaling_factor) * float(pt.state.scaling_factor)
    state = CipherState(cur, int(a.state.scale_degree) + int(pt.state.scale_degree), sf)
    out = _new_cipher(ctx, a.batch_size, cur, state, a.slots)
    p = pt.cv[0][:1].expand(a.batch_size, -1, -1) if pt.cv[0].shape[0] == 1 else pt.cv[0]
    for c in range(2):
        _lib.call("holmes_elementwise", ctx.handle, 2, a.cv[c].data_ptr(), p.data_ptr(), out.cv[c].data_ptr(),
                  a.batch_size, cur, _item_stride(a.cv[c]), int(p.stride(0)), _item_stride(out.cv[c]), _stream())
    return out


def homo_mul_no_relin(a: Cipher, b: Cipher, ctx) -> Cipher:
    ctx = _ctx(ctx)
    _valid(ctx, a, "homo_mul")
    _valid(ctx, b, "homo_mul")
    if len(a.cv) != 2 or len(b.cv) != 2:
        raise ValueError("homo_mul: relinearise a three-component operand first")
    if a.batch_size != b.batch_size:
        raise ValueError(f"homo_mul: batch mismatch {a.batch_size} != {b.batch_size}")
    if a.is_ext or b.is_ext:
        raise ValueError("homo_mul: extended ciphertexts are not supported")
    # operands at different levels meet at the lower one (the deeper operand's extra limbs are dropped; the nominal
    # scale is the same at every level)
    cur = min(int(a.state.cur_limbs), int(b.state.cur_limbs))
    n = a.batch_size
    storage = torch.empty((3, n, cur, ctx.N), dtype=torch.uint64, device=ctx.device)
    d0, d1, d2 = storage[0], storage[1], storage[2]
    if _item_stride(a.cv[0]) != _item_stride(a.cv[1]) or _item_stride(b.cv[0]) != _item_stride(b.cv[1]):
        t = torch.empty_like(d0)
        _ew(ctx, 2, a.cv[0], b.cv[0], d0, cur)
        _ew(ctx, 2, a.cv[0], b.cv[1], d1, cur)
        _ew(ctx, 2, a.cv[1], b.cv[0], t, cur)
        _ew(ctx, 0, d1, t, d1, cur)
        _ew(ctx, 2, a.cv[1], b.cv[1], d2, cur)
    else:
        _lib.call("holmes_tensor_product", ctx.handle, a.cv[0].data_ptr(), a.cv[1].data_ptr(), _item_stride(a.cv[0]),
                  b.cv[0].data_ptr(), b.cv[1].data_ptr(), _item_stride(b.cv[0]), d0.data_ptr(), d1.data_ptr(),
                  d2.data_ptr(), cur * ctx.N, n, cur, _stream())
    sf = None
    if a.state.scaling_factor is not None and b.state.scaling_factor is not None:
        sf = float(a.state.scaling_factor) * float(b.state.scaling_factor)
    state = CipherState(cur, int(a.state.scale_degree) + int(b.state.scale_degree), sf)
    return Cipher([d0, d1, d2], state, a.slots, False, n, ctx)


def homo_relinearize(a: Cipher, ctx) -> Cipher:
    ctx = _ctx(ctx)
    _valid(ctx, a, "homo_relinearize")
    if len(a.cv) != 3:
        raise ValueError("homo_relinearize expects a three-component ciphertext")
    cur = int(a.state.cur_limbs)
    n = a.batch_size
    out = _new_cipher(ctx, n, cur, a.state, a.slots)
    digits, dig_item = _modup(ctx, a.cv[2], cur, n)
    _keyswitch(ctx, digits, dig_item, cur, 1, ctx.switch_key(0, cur), a.cv[0], a.cv[1], _item_stride(a.cv[0]),
               out.cv[0], out.cv[1], n)
    return out


def homo_mul_relin(a: Cipher, b: Cipher, ctx) -> Cipher:
    return homo_relinearize(homo_mul_no_relin(a, b, ctx), ctx)


def _drop_limbs(a: Cipher, limbs: int) -> Cipher:
    if int(a.state.cur_limbs) == int(limbs):
        return a
    return a.cipher_like([c[:, :limbs] for c in a.cv], state=a.state.replace(cur_limbs=int(limbs)))


def homo_mul_relin_rescale_postop(a: Cipher, b: Cipher, ctx, apply_double: bool = False, sub: Cipher | None = None,
                                  scalar: EncodedScalar | None = None) -> Cipher:
    """``rescale(a * b)``, then doubled (``apply_double``), minus ``sub``, plus ``scalar``, the post-operations
    fused into the rescale's store (EasyFHE's fused kernel as llama3fhe calls it,
    ``operators/nonlinear/polynomial.py:139-193``: ``T_2j = 2 T_j^2 - 1``, ``T_2j+1 = 2 T_j T_j+1 - T_1``).

    The deeper operand is dropped to the other's limbs first; ``sub`` (a deeper ciphertext is read at the
    output's limbs, its modulus drop) and ``scalar`` (encoded for the output state, ``ctx.rescale_divisor_at``)
    land at the output, which has one limb fewer than the shallower operand."""
    ctx = _ctx(ctx)
    _valid(ctx, a, "homo_mul_relin_rescale_postop")
    _valid(ctx, b, "homo_mul_relin_rescale_postop")
    if sub is not None:
        _valid(ctx, sub, "homo_mul_relin_rescale_postop")
    cur = min(int(a.state.cur_limbs), int(b.state.cur_limbs))
    prod = homo_mul_relin(_drop_limbs(a, cur), _drop_limbs(b, cur), ctx)
    if cur < 2:
        raise ValueError("homo_mul_relin_rescale_postop needs at least two limbs")
    ql = ctx.q(cur - 1)
    sf = None if prod.state.scaling_factor is None else float(prod.state.scaling_factor) / ql
    state = CipherState(cur - 1, max(1, int(prod.state.scale_degree) - 1), sf)
    n = prod.batch_size
    broadcast = False
    if sub is not None:
        if sub.is_ext or len(sub.cv) != 2:
            raise ValueError("homo_mul_relin_rescale_postop: sub must be a two-component, non-extended ciphertext")
        if int(sub.state.cur_limbs) < cur - 1:
            raise ValueError(f"homo_mul_relin_rescale_postop: sub has {sub.state.cur_limbs} limbs, the output "
                             f"{cur - 1}")
        if int(sub.state.scale_degree) != int(state.scale_degree):
            raise ValueError("homo_mul_relin_rescale_postop: sub's scale degree differs from the output's")
        if sub.batch_size not in (1, n):
            raise ValueError(f"homo_mul_relin_rescale_postop: sub batch {sub.batch_size} for {n} products")
        broadcast = sub.batch_size == 1 and n > 1
    k = None
    if scalar is not None:
        if int(scalar.state.cur_limbs) < cur - 1:
            raise ValueError("homo_mul_relin_rescale_postop: the scalar is encoded for fewer limbs than the output")
        k = scalar.residues(ctx, cur - 1)
    out = _new_cipher(ctx, n, cur - 1, state, prod.slots)
    scratch = ctx.workspace("rescale", n * ctx.N)
    tok = OPTIMER.start("rescale")
    for c in range(2):
        _lib.call("holmes_rescale_postop", ctx.handle, prod.cv[c].data_ptr(), _item_stride(prod.cv[c]),
                  out.cv[c].data_ptr(), _item_stride(out.cv[c]), cur, n, scratch.data_ptr(), int(bool(apply_double)),
                  0 if sub is None else sub.cv[c].data_ptr(),
                  0 if (sub is None or broadcast) else _item_stride(sub.cv[c]),
                  0 if (k is None or c) else k.data_ptr(), _stream())
    OPTIMER.stop(tok, 2 * n * (2 * cur - 1) * ctx.N * 8)
    return out


# ----------------------------------------------------------------------------------------------------- scalars
# A real scalar v at scale S is the constant polynomial round(v S): the same residue in every NTT word, so scalar
# products and sums are per-limb constant kernels (holmes_mul_const / holmes_add_const).  Names and argument
# meaning follow the EasyFHE calls llama3fhe makes (operators/nonlinear/bootstrap.py:604-623,
# operators/norm/refresh.py:21-31).


class EncodedScalar:
    """One encoded scalar ``EncodedScalar(value, integer, state)`` (``integer = round(value * scaling_factor)``), or
    the reference's weight table ``EncodedScalar(residues, cur_limbs, scale_degree, scaling_factor)`` with
    ``residues`` a ``[groups][n][cur]`` uint64 tensor (``operators/nonlinear/polynomial.py:286-291``) for
    ``grouped_scalar_weighted_acc``."""

    def __init__(self, *args) -> None:
        if args and torch.is_tensor(args[0]):
            residues, cur_limbs, scale_degree, scaling_factor = args
            self.table = residues
            self.value = None
            self.integer = None
            self.state = CipherState(int(cur_limbs), int(scale_degree),
                                     None if scaling_factor is None else float(scaling_factor))
        else:
            value, integer, state = args
            self.table = None
            self.value = float(value)
            self.integer = int(integer)
            self.state = state

    def residues(self, ctx, limbs: int) -> torch.Tensor:
        if self.table is not None:
            raise ValueError("a weight table has no single residue vector")
        return ctx.device_u64(self.residue_list(ctx, limbs))

    def residue_list(self, ctx, limbs: int) -> list:
        if self.table is not None:
            raise ValueError("a weight table has no single residue vector")
        return ctx.residues(self.integer, limbs)


def grouped_scalar_weighted_acc(batch: Cipher, table: EncodedScalar, ctx) -> Cipher:
    """``out[g] = sum_k table[g][k] * batch[k]`` in one launch per component, residue-identical to the loop of
    scalar multiplies and adds (each product reduced mod q_l, the sum exact mod q_l); ``groups`` items out."""
    ctx = _ctx(ctx)
    _valid(ctx, batch, "grouped_scalar_weighted_acc")
    if table.table is None:
        raise ValueError("grouped_scalar_weighted_acc needs a weight table EncodedScalar")
    res = table.table.to(device=ctx.device, dtype=torch.uint64).contiguous()
    cur = int(batch.state.cur_limbs)
    n = int(batch.batch_size)
    if res.dim() != 3 or int(res.shape[1]) != n or int(res.shape[2]) < cur:
        raise ValueError(f"weight table of shape {tuple(res.shape)} for {n} ciphertexts at {cur} limbs")
    if int(res.shape[2]) != cur:
        res = res[:, :, :cur].contiguous()
    groups = int(res.shape[0])
    sf = None
    if batch.state.scaling_factor is not None and table.state.scaling_factor is not None:
        sf = float(batch.state.scaling_factor) * float(table.state.scaling_factor)
    state = CipherState(cur, int(batch.state.scale_degree) + int(table.state.scale_degree), sf)
    out = _new_cipher(ctx, groups, cur, state, batch.slots)
    for c in range(len(batch.cv)):
        _lib.call("holmes_weighted_acc", ctx.handle, batch.cv[c].data_ptr(), _item_stride(batch.cv[c]), n,
                  res.data_ptr(), out.cv[c].data_ptr(), _item_stride(out.cv[c]), groups, cur, _stream())
    return out


def encode_scalar(value, cur_limbs: int, scale_degree: int = 1, scaling_factor: float | None = None,
                  context=None, mode: str = "real") -> EncodedScalar:
    """``mode="integer"`` encodes the integer itself (scale 1, degree 0): multiplying by it keeps the scale."""
    ctx = _ctx(context)
    if isinstance(value, complex) or np.iscomplexobj(value):
        raise ValueError("encode_scalar encodes real values; multiply by i with homo_mul_i")
    if mode == "integer":
        if int(value) != value:
            raise ValueError("integer-mode scalars must be integers")
        return EncodedScalar(float(value), int(value), CipherState(int(cur_limbs), 0, 1.0))
    if mode != "real":
        raise ValueError(f"unknown scalar mode {mode!r}")
    sf = float(scaling_factor) if scaling_factor is not None else ctx.scale_at(int(cur_limbs))
    return EncodedScalar(float(value), int(round(float(value) * sf)), CipherState(int(cur_limbs), int(scale_degree), sf))


def homo_mul_scalar(a: Cipher, scalar: EncodedScalar, ctx) -> Cipher:
    """a * scalar without rescale: the scale degrees and factors multiply."""
    ctx = _ctx(ctx)
    _valid(ctx, a, "homo_mul_scalar")
    cur = int(a.state.cur_limbs)
    sf = None
    if a.state.scaling_factor is not None and scalar.state.scaling_factor is not None:
        sf = float(a.state.scaling_factor) * float(scalar.state.scaling_factor)
    out = _new_cipher(ctx, a.batch_size, cur,
                      CipherState(cur, int(a.state.scale_degree) + int(scalar.state.scale_degree), sf), a.slots)
    const_cv(ctx, CONST_MUL, a.cv, scalar.residue_list(ctx, cur), out.cv, a.batch_size, cur)
    return out


def homo_mul_scalar_rescale(a: Cipher, scalar: EncodedScalar, ctx) -> Cipher:
    return rescale(homo_mul_scalar(a, scalar, ctx), ctx)


def homo_add_scalar(a: Cipher, scalar, ctx) -> Cipher:
    """a + scalar; a float is encoded at the ciphertext's own scale, an EncodedScalar must carry that scale."""
    ctx = _ctx(ctx)
    _valid(ctx, a, "homo_add_scalar")
    cur = int(a.state.cur_limbs)
    sf = float(a.state.scaling_factor if a.state.scaling_factor is not None else ctx.scale_at(cur))
    if not isinstance(scalar, EncodedScalar):
        scalar = encode_scalar(float(scalar), cur, int(a.state.scale_degree), sf, ctx)
    elif scalar.state.scaling_factor is not None and abs(float(scalar.state.scaling_factor) - sf) > 1e-9 * sf:
        raise ValueError("homo_add_scalar: the scalar's scale differs from the ciphertext's")
    out = a.cipher_like([torch.empty_like(a.cv[0][:, :cur])] + [c[:, :cur].clone() for c in a.cv[1:]],
                        state=a.state)
    const_cv(ctx, CONST_ADD, a.cv[:1], scalar.residue_list(ctx, cur), out.cv[:1], a.batch_size, cur)
    return out


def homo_add_pt(a: Cipher, pt: Plaintext, ctx) -> Cipher:
    """a + pt (pt at the ciphertext's scale and degree, at least as many limbs)."""
    ctx = _ctx(ctx)
    _valid(ctx, a, "homo_add_pt")
    _valid(ctx, pt, "homo_add_pt")
    cur = int(a.state.cur_limbs)
    if int(pt.state.cur_limbs) < cur:
        raise ValueError("homo_add_pt: plaintext has fewer limbs than the ciphertext")
    if int(pt.state.scale_degree) != int(a.state.scale_degree):
        raise ValueError("homo_add_pt: scale degree mismatch")
    out = a.cipher_like([torch.empty_like(a.cv[0][:, :cur])] + [c[:, :cur].clone() for c in a.cv[1:]],
                        state=a.state)
    p = pt.cv[0][:1].expand(a.batch_size, -1, -1) if pt.cv[0].shape[0] == 1 else pt.cv[0]
    _lib.call("holmes_elementwise", ctx.handle, 0, a.cv[0].data_ptr(), p.data_ptr(), out.cv[0].data_ptr(),
              a.batch_size, cur, _item_stride(a.cv[0]), int(p.stride(0)), _item_stride(out.cv[0]), _stream())
    return out


# ----------------------------------------------------------------------------------------------------- constants


class PackedRaw:
    """Slot values already packed: a tensor ``[rows][slots]`` (or ``[slots]``), real or complex."""

    def __init__(self, tensor) -> None:
        self.tensor = tensor

    def packed(self, slots: int, context) -> torch.Tensor:
        del context
        return self.tensor


class UnpackedRaw:
    """A raw source plus the packer that turns it into ``[rows][slots]`` slot values."""

    def __init__(self, source, packer) -> None:
        self.source = source
        self.packer = packer

    def packed(self, slots: int, context) -> torch.Tensor:
        return self.packer(self.source, int(slots), context)


class ConstantBundle:
    """Named plaintext constants with an optional cache of the FFT'd values ("middle") and/or the final
    NTT plaintexts ("plain"), per ``cache_mode`` in {"none", "middle", "plain", "both"}."""

    def __init__(self, vectors: dict | None = None, cache_mode: str = "none", scalars: dict | None = None) -> None:
        if cache_mode not in ("none", "middle", "plain", "both"):
            raise ValueError(f"unknown cache_mode {cache_mode!r}")
        self.vectors = dict(vectors or {})
        self.scalars = {str(k): float(v) for k, v in (scalars or {}).items()}
        self.cache_mode = cache_mode
        self._middle: dict = {}
        self._plain: dict = {}
        self._stats = {"middle_hits": 0, "middle_misses": 0, "plain_hits": 0, "plain_misses": 0}

    def _encoded_middle(self, name: str, *, slots: int, context) -> torch.Tensor:
        ctx = _ctx(context)
        key = (name, int(slots))
        mid = self._middle.get(key)
        if mid is not None:
            self._stats["middle_hits"] += 1
            return mid
        self._stats["middle_misses"] += 1
        raw = self.vectors[name].packed(int(slots), ctx)
        if not torch.is_tensor(raw):
            raw = torch.from_numpy(np.asarray(raw))
        raw = raw.reshape(-1, int(slots))
        mid = fft_special_inv_rows(ctx, raw, int(slots))
        if self.cache_mode in ("middle", "both"):
            self._middle[key] = mid
        return mid

    def plaintext(self, name: str, *, state: CipherState, slots: int, context, is_ext: bool = False,
                  cache: bool = False) -> Plaintext:
        """``is_ext``: encoded over the extended basis Q u P (``cur + K`` limbs, Q first)."""
        ctx = _ctx(context)
        key = (name, int(slots), int(state.cur_limbs), float(state.scaling_factor or ctx.scale), bool(is_ext))
        hit = self._plain.get(key)
        if hit is not None:
            self._stats["plain_hits"] += 1
            return hit
        self._stats["plain_misses"] += 1
        mid = self._encoded_middle(name, slots=slots, context=ctx)
        scale = float(state.scaling_factor) if state.scaling_factor is not None else ctx.scale_at(state.cur_limbs)
        pv = encode_rows(ctx, mid, int(state.cur_limbs), scale, int(slots), already_transformed=True, ext=bool(is_ext))
        pt = Plaintext([pv], CipherState(int(state.cur_limbs), int(state.scale_degree), scale), int(slots),
                       bool(is_ext), int(pv.shape[0]), ctx)
        if self.cache_mode in ("plain", "both") or (cache and self.cache_mode != "none"):
            self._plain[key] = pt
        return pt

    def encoded_scalars(self, names, *, cur_limbs: int, scale_degree: int = 1, context=None,
                        scaling_factor: float | None = None, cache: bool = False):
        """The named scalars as residues ``[len(names)][cur]`` of ``round(value * scaling_factor)`` (the reference's
        weight-table source, ``operators/nonlinear/polynomial.py:278-285``)."""
        del cache
        ctx = _ctx(context)
        cur = int(cur_limbs)
        sf = float(scaling_factor) if scaling_factor is not None else ctx.scale_at(cur)
        ints = [int(round(self.scalars[str(nm)] * sf)) for nm in names]
        residues = ctx.device_u64([ctx.residues(v, cur) for v in ints])
        return types.SimpleNamespace(residues=residues, cur_limbs=cur, scale_degree=int(scale_degree),
                                     scaling_factor=sf)

    def cache_info(self) -> dict:
        mb = sum(int(t.numel()) * t.element_size() for t in self._middle.values())
        pb = sum(int(p.cv[0].numel()) * 8 for p in self._plain.values())
        return {"middle_entries": len(self._middle), "plain_entries": len(self._plain), "middle_bytes": mb,
                "plain_bytes": pb, "total_bytes": mb + pb, **self._stats}

    def clear_cache(self) -> None:
        self._middle.clear()
        self._plain.clear()
