"""Run the reference's unchanged ``llama3fhe`` operators on this engine: register it under the import name ``easyfhe``.

``llama3fhe`` reaches its engine only through the EasyFHE package (``from easyfhe import fhe``, ``import
easyfhe.bs.openfhe as bs``, ``easyfhe.cuda.*`` streams and events, ``easyfhe.from_numpy`` / ``get_device_module``;
``llama3fhe/backend.py:18-20, 249-396, 556-596``, ``operators/linear/operator.py:9, 24-31``,
``operators/linear/weight.py:105-114, 373-376, 570-582``).  :func:`install` puts module objects under those names in
``sys.modules`` so that those imports resolve to:

* ``easyfhe.fhe``          -> :mod:`holmes_b200.fhe` (every name the operators call; ``ciphertext``, ``ops.layout`` and
  ``constants`` sub-modules for the three deep imports, ``operators/attention/sparse_fused.py:154``,
  ``operators/nonlinear/polynomial.py:294``, ``operators/attention/prefill/softmax.py:559``);
* ``easyfhe.bs.openfhe``   -> :mod:`holmes_b200.bootstrap` (``BootstrapSpec``, ``generate``, ``bootstrap``,
  ``requirements``; ``operators/nonlinear/bootstrap.py:18``);
* ``easyfhe.cuda``         -> ``torch.cuda`` (streams, events, synchronisation -- the engine launches on torch's current
  stream, so the operators' side-stream encode schedule orders the engine's kernels);
* ``easyfhe`` itself       -> a tensor namespace: ``from_numpy``, ``get_device_module``, ``multiprocessing`` and, for any
  other name, torch's (EasyFHE's tensors are torch-like; here they are torch tensors).

It also replaces the reference's two Triton diagonal packers (``operators/linear/gpu_packer.py:48-476``, which the
north star rules out) with this engine's CUDA packers (``holmes_pack_diagonals`` / ``holmes_pack_structured``) under
the same function names, so ``LinearWeight`` with ``raw_weight_policy="device"`` packs on the engine.

The module objects forward attribute reads to the engine modules, so a test's ``monkeypatch.setattr(fhe, ...)``
replaces the name for the operators (as it would on EasyFHE's module) without touching :mod:`holmes_b200.fhe`
itself.  :func:`uninstall` removes the names again.  Nothing here does arithmetic; with no CUDA device the engine
raises on first use (there is no CPU path).
"""
from __future__ import annotations

import sys
import types

import torch

from . import _lib
from . import bootstrap as _bootstrap
from . import fhe as _fhe

#: the encoder's range limit in bits (values must stay below 2^61, ``bench/cmp/holmes_fast_encode.py:93-112``)
MAX_ENCODED_BITS = 61

_NAMES = ("easyfhe", "easyfhe.fhe", "easyfhe.fhe.ciphertext", "easyfhe.fhe.ops", "easyfhe.fhe.ops.layout",
          "easyfhe.fhe.constants", "easyfhe.bs", "easyfhe.bs.openfhe", "easyfhe.cuda", "easyfhe.multiprocessing")
_PACKER = "llama3fhe.operators.linear.gpu_packer"
_saved: dict = {}


def _forwarding(name: str, target, **extra) -> types.ModuleType:
    """A module named ``name`` whose own attributes are ``extra`` and whose other attributes are ``target``'s."""
    mod = types.ModuleType(name)
    mod.__dict__.update(extra)

    def __getattr__(attr: str):
        try:
            return getattr(target, attr)
        except AttributeError:
            raise AttributeError(f"module {name!r} has no attribute {attr!r}") from None

    mod.__getattr__ = __getattr__
    return mod


class _HostDevice:
    """``get_device_module("cpu")``: nothing to synchronise or trim."""

    @staticmethod
    def synchronize(*_args, **_kwargs) -> None:
        return None

    @staticmethod
    def empty_cache() -> None:
        return None

    @staticmethod
    def is_available() -> bool:
        return True


def get_device_module(device: str = "cuda"):
    return torch.cuda if str(device).startswith("cuda") else _HostDevice


def cipher_batch_item(cipher, index: int):
    """Item ``index`` of a batch cipher as a one-item cipher (EasyFHE ``fhe.ops.layout.cipher_batch_item``)."""
    index = int(index)
    if not 0 <= index < int(cipher.batch_size):
        raise IndexError(f"batch item {index} outside [0, {cipher.batch_size})")
    return cipher.cipher_like([c[index:index + 1] for c in cipher.cv], batch_size=1)


# ------------------------------------------------------------------------------------------- diagonal packers


def _check_geometry(slots, dimension, token_lanes, baby_steps, giant_base, giant_count, lane_shift) -> None:
    if slots <= 0 or dimension <= 0 or token_lanes <= 0:
        raise ValueError("slots/dimension/token_lanes must be positive.")
    if dimension * token_lanes != slots:
        raise ValueError(f"token-lane packing requires dimension*token_lanes == slots, got "
                         f"{dimension}*{token_lanes} != {slots}.")
    if baby_steps <= 0 or giant_base < 0 or giant_count <= 0:
        raise ValueError("baby_steps/giant_count must be positive and giant_base non-negative.")
    if lane_shift < 0 or (lane_shift and lane_shift * token_lanes != dimension):
        raise ValueError(f"lane_shift must be 0 or dimension/token_lanes, got {lane_shift} "
                         f"(dimension={dimension}, token_lanes={token_lanes}).")


def pack_token_lane_bsgs_weight_chunk_triton_gpu(weight, *, slots: int, dimension: int, token_lanes: int,
                                                  baby_steps: int, giant_base: int, giant_count: int,
                                                  lane_shift: int = 0, device: str = "cuda", block_size: int = 256):
    """``row(g, b)[s] = W[(f(s) - g B) mod D, (f(s) + b + lane_shift lane(s)) mod D]`` as complex128 rows
    ``[giant_count * B][slots]``, on ``holmes_pack_diagonals`` (same name and arguments as the reference's Triton
    packer, ``operators/linear/gpu_packer.py:49-154``; ``block_size`` is a Triton launch detail and is ignored)."""
    del block_size
    slots, dimension, token_lanes = int(slots), int(dimension), int(token_lanes)
    baby_steps, giant_base, giant_count, lane_shift = int(baby_steps), int(giant_base), int(giant_count), int(lane_shift)
    _check_geometry(slots, dimension, token_lanes, baby_steps, giant_base, giant_count, lane_shift)
    if not torch.is_tensor(weight) or not weight.is_cuda:
        raise ValueError("token-lane GPU packer requires a CUDA-resident weight tensor.")
    if tuple(int(v) for v in weight.shape) != (dimension, dimension):
        raise ValueError(f"weight must have shape {(dimension, dimension)}, got {tuple(weight.shape)}.")
    if weight.is_complex():
        kind, weight = 1, weight.to(torch.complex128).contiguous()
    elif weight.dtype == torch.float32:
        kind, weight = 2, weight.contiguous()
    else:
        kind, weight = 0, weight.to(torch.float64).contiguous()
    rows = giant_count * baby_steps
    packed = torch.empty((rows, slots), dtype=torch.complex128, device=weight.device)
    _lib.call("holmes_pack_diagonals", weight.data_ptr(), kind, dimension, token_lanes, baby_steps, giant_base,
              giant_count, lane_shift, slots, packed.data_ptr(), 2 * slots, torch.cuda.current_stream().cuda_stream)
    return packed


_STRUCT_MAPS = ("real_source", "real_row", "real_scale", "imag_source", "imag_row", "imag_scale", "column",
                "column_scale")


def pack_structured_token_lane_bsgs_weight_chunk_triton_gpu(sources, metadata, *, slots: int, dimension: int,
                                                             token_lanes: int, baby_steps: int, giant_base: int,
                                                             giant_count: int, lane_shift: int = 0,
                                                             device: str = "cuda", block_size: int = 256):
    """The structured variant (``operators/linear/gpu_packer.py:201-358``): one to three real logical sources and
    per-row / per-column maps, never building the physical square matrix; on ``holmes_pack_structured``."""
    del block_size
    slots, dimension, token_lanes = int(slots), int(dimension), int(token_lanes)
    baby_steps, giant_base, giant_count, lane_shift = int(baby_steps), int(giant_base), int(giant_count), int(lane_shift)
    _check_geometry(slots, dimension, token_lanes, baby_steps, giant_base, giant_count, lane_shift)
    sources = tuple(sources)
    if not 1 <= len(sources) <= 3:
        raise ValueError("structured GPU packer requires one to three sources.")
    for i, src in enumerate(sources):
        if not torch.is_tensor(src) or not src.is_cuda:
            raise ValueError(f"structured source {i} must be a CUDA tensor.")
        if src.ndim != 2:
            raise ValueError(f"structured source {i} must be rank two, got {src.shape}.")
    dtype = sources[0].dtype
    if any(s.dtype != dtype for s in sources):
        raise TypeError("structured GPU sources must use one common dtype.")
    if dtype not in (torch.float32, torch.float64):
        raise TypeError(f"structured GPU sources must use float32 or float64, got {dtype}.")
    missing = [n for n in _STRUCT_MAPS if n not in metadata]
    if missing:
        raise ValueError(f"structured GPU metadata is missing {missing}.")
    maps = {n: metadata[n] for n in _STRUCT_MAPS}
    maps["real_column"] = metadata.get("real_column", metadata["column"])
    maps["imag_column"] = metadata.get("imag_column", metadata["column"])
    for n, v in maps.items():
        if not torch.is_tensor(v) or not v.is_cuda:
            raise ValueError(f"structured metadata {n!r} must be a CUDA tensor.")
        if tuple(int(x) for x in v.shape) != (dimension,):
            raise ValueError(f"structured metadata {n!r} must have shape {(dimension,)}, got {tuple(v.shape)}.")
        want = torch.float64 if n.endswith("scale") else torch.int64
        maps[n] = v.to(want).contiguous()
    rows = giant_count * baby_steps
    packed = torch.empty((rows, slots), dtype=torch.complex128, device=sources[0].device)
    ptrs = _lib.ptr_array([s.data_ptr() for s in sources])
    rs = (_lib.ctypes.c_longlong * 3)(*[int(s.stride(0)) for s in sources])
    cs = (_lib.ctypes.c_longlong * 3)(*[int(s.stride(1)) for s in sources])
    _lib.call("holmes_pack_structured", ptrs, rs, cs, len(sources), int(dtype == torch.float32),
              maps["real_source"].data_ptr(), maps["real_row"].data_ptr(), maps["real_scale"].data_ptr(),
              maps["imag_source"].data_ptr(), maps["imag_row"].data_ptr(), maps["imag_scale"].data_ptr(),
              maps["real_column"].data_ptr(), maps["imag_column"].data_ptr(), maps["column_scale"].data_ptr(),
              dimension, token_lanes, baby_steps, giant_base, giant_count, lane_shift, slots, packed.data_ptr(),
              2 * slots, torch.cuda.current_stream().cuda_stream)
    return packed


def _packer_module() -> types.ModuleType:
    mod = types.ModuleType(_PACKER)
    mod.__doc__ = "CUDA diagonal packers of libholmes_cuda under the reference's packer names (holmes_b200)."
    mod.SLOTS = 2 ** 15
    mod.torch = torch      # the reference module's own name for its tensor namespace
    mod.synchronize = torch.cuda.synchronize
    mod.pack_token_lane_bsgs_weight_chunk_triton_gpu = pack_token_lane_bsgs_weight_chunk_triton_gpu
    mod.pack_structured_token_lane_bsgs_weight_chunk_triton_gpu = \
        pack_structured_token_lane_bsgs_weight_chunk_triton_gpu
    return mod


# ------------------------------------------------------------------------------------------- host arrays


class HostTensor(torch.Tensor):
    """What ``easyfhe.from_numpy`` returns: a CPU tensor over the array whose ``.to(cuda)`` copies through pinned
    memory without waiting for the device (a plain ``Tensor.to`` from host memory synchronises the stream, which
    drains the GPU's queue at every constant upload).  The device tensor is ordered after everything already queued on
    the current stream, as the synchronous copy was; the pinned staging buffer is held until the copy has run."""

    def to(self, *args, **kwargs):
        plain = self.as_subclass(torch.Tensor)
        target = kwargs.get("device", args[0] if args else None)
        if isinstance(target, (str, torch.device)) and torch.device(target).type == "cuda" and \
                not kwargs.get("non_blocking", False) and not any(isinstance(a, torch.dtype) for a in args) and \
                "dtype" not in kwargs and "copy" not in kwargs and "memory_format" not in kwargs:
            return plain.pin_memory().to(torch.device(target), non_blocking=True)
        return plain.to(*args, **kwargs)


def from_numpy(array) -> torch.Tensor:
    """``easyfhe.from_numpy``: the array as a CPU tensor (a ``HostTensor``; see there)."""
    return torch.from_numpy(array).as_subclass(HostTensor)


# ------------------------------------------------------------------------------------------- registration


def _build() -> dict:
    ciphertext = _forwarding("easyfhe.fhe.ciphertext", _fhe)
    layout = types.ModuleType("easyfhe.fhe.ops.layout")
    layout.cipher_batch_item = cipher_batch_item
    ops = types.ModuleType("easyfhe.fhe.ops")
    ops.layout = layout
    constants = types.ModuleType("easyfhe.fhe.constants")
    constants.MAX_ENCODED_BITS = MAX_ENCODED_BITS
    fhe = _forwarding("easyfhe.fhe", _fhe, ciphertext=ciphertext, ops=ops, constants=constants)
    fhe.__path__ = []    # a package, so that the deep imports resolve through sys.modules
    ops.__path__ = []
    openfhe = _forwarding("easyfhe.bs.openfhe", _bootstrap)
    bs = types.ModuleType("easyfhe.bs")
    bs.openfhe = openfhe
    bs.__path__ = []
    top = _forwarding("easyfhe", torch, fhe=fhe, bs=bs, cuda=torch.cuda, multiprocessing=torch.multiprocessing,
                      from_numpy=from_numpy, get_device_module=get_device_module)
    top.__path__ = []
    return {"easyfhe": top, "easyfhe.fhe": fhe, "easyfhe.fhe.ciphertext": ciphertext, "easyfhe.fhe.ops": ops,
            "easyfhe.fhe.ops.layout": layout, "easyfhe.fhe.constants": constants, "easyfhe.bs": bs,
            "easyfhe.bs.openfhe": openfhe, "easyfhe.cuda": torch.cuda, "easyfhe.multiprocessing": torch.multiprocessing}


def batched_bootstrap(ciphers, crypto_context, program) -> list:
    """The reference's batched-refresh hook (``BootstrapOperator.batch_backend``, ``callable(ciphers, crypto_context,
    program) -> list``; ``llama3fhe/operators/nonlinear/bootstrap.py:183-188, 484-560``): ciphertexts of one state go
    through one bootstrap as a batch, so every key switch of C2S / EvalMod / S2C is shared (each key read once per
    batch, not once per ciphertext).  Per ciphertext the arithmetic is the single refresh's, word for word."""
    ciphers = list(ciphers)
    batch = _fhe.pack_cipher_batch(ciphers)
    out = _bootstrap.bootstrap(batch, crypto_context, program)
    return list(_fhe.unpack_cipher_batch(out))


def _install_batch_backend() -> None:
    """Set the reference's ``BootstrapOperator.batch_backend`` when its package is importable (the reference's own
    GPU benches install theirs the same way, ``bench/cmp/holmes_batch_bs.py``)."""
    try:
        import importlib

        mod = importlib.import_module("llama3fhe.operators.nonlinear.bootstrap")
    except ImportError:
        return
    if getattr(mod.BootstrapOperator, "batch_backend", None) is None:
        mod.BootstrapOperator.batch_backend = staticmethod(batched_bootstrap)


def install(replace_packers: bool = True, batch_bootstrap: bool = True) -> types.ModuleType:
    """Register the engine as ``easyfhe`` (and, with ``replace_packers``, the CUDA packers in place of the
    reference's Triton module; with ``batch_bootstrap``, :func:`batched_bootstrap` as the reference's batched-refresh
    hook once its package is importable).  Idempotent; returns the ``easyfhe`` module object."""
    current = sys.modules.get("easyfhe")
    if current is not None and getattr(current, "__holmes_b200__", False):
        return current
    mods = _build()
    mods["easyfhe"].__holmes_b200__ = True
    for name, mod in mods.items():
        if name not in _saved:
            _saved[name] = sys.modules.get(name)
        sys.modules[name] = mod
    if replace_packers:
        if _PACKER not in _saved:
            _saved[_PACKER] = sys.modules.get(_PACKER)
        sys.modules[_PACKER] = _packer_module()
        parent = sys.modules.get("llama3fhe.operators.linear")
        if parent is not None:
            parent.gpu_packer = sys.modules[_PACKER]
    if batch_bootstrap:
        _install_batch_backend()
    return mods["easyfhe"]


def uninstall() -> None:
    """Undo :func:`install` (restores whatever those names held before)."""
    for name, prev in list(_saved.items()):
        if prev is None:
            sys.modules.pop(name, None)
        else:
            sys.modules[name] = prev
    _saved.clear()
