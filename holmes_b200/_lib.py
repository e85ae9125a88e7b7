"""ctypes binding of libholmes_cuda (include/holmes_cuda.h).

There is no fallback: if the library is missing or a call returns a non-zero status, the caller gets
an exception.  ``load()`` builds the library in-tree when the source is newer (only possible where
nvcc exists; a GPU host uses the library that travelled with the tree).
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("HOLMES_LIB", os.path.join(HERE, "lib", "libholmes_cuda.so"))

_lib = None

u64, i32, i64, p, d = ctypes.c_uint64, ctypes.c_int, ctypes.c_longlong, ctypes.c_void_p, ctypes.c_double
PP = ctypes.POINTER(ctypes.c_void_p)


class HolmesParams(ctypes.Structure):
    _fields_ = [("log_n", i32), ("limbs", i32), ("dnum", i32), ("dcrt_bits", i32), ("first_mod_bits", i32),
                ("special_bits", i32), ("special_limbs", i32), ("hamming", i32), ("seed", u64)]


SIGNATURES = {
    "holmes_ctx_create": [ctypes.POINTER(HolmesParams), ctypes.POINTER(p)],
    "holmes_ctx_destroy": [p],
    "holmes_ctx_moduli": [p, p],
    "holmes_ctx_dims": [p, p],
    "holmes_ctx_secret": [p, ctypes.POINTER(p)],
    "holmes_galois": [p, i64, ctypes.POINTER(u64)],
    "holmes_key_words": [p, i32, ctypes.POINTER(i64)],
    "holmes_keygen": [p, u64, i32, p, p],
    "holmes_encrypt": [p, p, i32, u64, p, p, p],
    "holmes_decrypt": [p, p, p, i32, p, p],
    "holmes_ntt": [p, p, i32, i32, i64, i32, i32, p],
    "holmes_encode": [p, p, i64, i32, i32, d, i32, p, i64, p, p],
    "holmes_fft_special_inv": [p, p, i64, i32, i32, p],
    "holmes_encode_fft": [p, p, i64, i32, i32, d, i32, p, i64, p, p],
    "holmes_encode_fft_ext": [p, p, i64, i32, i32, d, i32, p, i64, p, p],
    "holmes_encode_stage2": [p, p, i64, i32, d, i32, p, p, p, p, p, p, p, i32, i32, i32],
    "holmes_pack_diagonals":[p, i32, i32, i32, i32, i32, i32, i32, i32, p, i64, p],
    "holmes_pack_structured": [p, p, p, i32, i32, p, p, p, p, p, p, p, p, p, i32, i32, i32, i32, i32, i32, i32, p,
                               i64, p],
    "holmes_elementwise": [p, i32, p, p, p, i32, i32, i64, i64, i64, p],
    "holmes_tensor_product": [p, p, p, i64, p, p, i64, p, p, p, i64, i32, i32, p],
    "holmes_mul_i": [p, p, p, i32, i32, i64, i64, p],
    "holmes_automorph": [p, p, p, u64, i32, i32, i64, i64, p],
    "holmes_mul_const": [p, p, p, p, i32, i32, i64, i64, p],
    "holmes_weighted_acc": [p, p, i64, i32, p, p, i64, i32, i32, p],
    "holmes_rescale": [p, p, i64, p, i64, i32, i32, p, p],
    "holmes_rotate_scratch_words": [p, i32, i32, p],
    "holmes_scratch_words": [p, i32, i32, i32, p],
    "holmes_rotate": [p, p, p, i64, i32, p, i32, u64, p, p, i64, i32, p, p],
    "holmes_hoisted_rotations": [p, p, p, i64, i32, i32, i32, p, p, p, p, p, i64, i64, p, p],
    "holmes_giant_sum": [p, p, p, i64, i64, i32, i32, i32, p, i32, u64, p, p, i64, p, p],
    "holmes_mul_relin": [p, p, p, p, p, i64, i32, i32, p, i32, p, p, i64, p, p],
    "holmes_encode_diag_rows": [p, p, i32, i32, i32, i32, i32, i32, i32, i32, d, i32, p, i64, p, p, p],
    "holmes_rescale_postop": [p, p, i64, p, i64, i32, i32, p, i32, p, i64, p, p],
    "holmes_modraise": [p, p, i64, p, i64, i32, i32, p, p],
    "holmes_add_const": [p, p, p, p, i32, i32, i64, i64, p],
    "holmes_const_op": [p, i32, p, p, p, i32, i32, i64, i64, p],
    "holmes_rescale_noalloc":[p, p, i64, p, i64, i32, i32, p],
    "holmes_modup": [p, p, i64, i32, i32, p, i64, p, p],
    "holmes_peer_alloc": [ctypes.c_ulonglong, p],
    "holmes_peer_free": [p],
    "holmes_ipc_export": [p, p],
    "holmes_ipc_import": [p, p],
    "holmes_ipc_close": [p],
    "holmes_peer_signal": [p, i32, u64, p],
    "holmes_peer_wait": [p, i32, u64, i64, p, p],
    "holmes_modreduce_scatter": [p, p, i32, p, i32, i32, i64, p, p],
    "holmes_keyswitch": [p, p, i64, i32, p, i32, u64, p, p, i64, p, p, i64, p, p, i64, i32, p, p],
    "holmes_bsgs_mac": [p, p, p, p, i64, i32, i32, p, i64, i32, i32, p],
    "holmes_mac_gather": [p, p, p, i64, p, p, p, i32, i32, p, i64, i32, i32, p, p, p, p],
    "holmes_keyswitch_ext": [p, p, i64, i32, p, i32, u64, p, i64, p, p, i64, i32, p],
    "holmes_moddown": [p, p, p, i64, i32, p, p, i64, i32, p, p],
    "holmes_bsgs_mac_ext": [p, p, p, p, i64, i32, i32, p, i64, i32, i32, p],
    "holmes_modsum": [p, p, i32, p, i32, i32, i64, p],
    "holmes_launch_count": [ctypes.POINTER(ctypes.c_ulonglong)],
    "holmes_device_error": [i32, ctypes.POINTER(ctypes.c_int)],
    "holmes_mac_multi":[p, p, p, i64, i32, i32, p, i64, i32, i32, i32, p, p, p, p],
}


class HolmesError(RuntimeError):
    pass


def load():
    """The loaded library; raises when it is absent (there is no CPU fallback)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH) or os.environ.get("HOLMES_REBUILD") == "1":
        from . import build

        build.build()
    if not os.path.exists(LIB_PATH):
        raise HolmesError(f"libholmes_cuda is not built ({LIB_PATH}); run python -m holmes_b200.build")
    lib = ctypes.CDLL(LIB_PATH)
    for name, args in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = i32
    _lib = lib
    return lib


def check(rc: int, what: str) -> None:
    if rc != 0:
        kind = "argument error" if rc < 0 else "CUDA error"
        raise HolmesError(f"{what} failed: {kind} {rc}")


_FNS: dict = {}


def call(name: str, *args) -> None:
    fn = _FNS.get(name)
    if fn is None:
        fn = _FNS[name] = getattr(load(), name)
    rc = fn(*args)
    if rc != 0:
        check(rc, name)


def ptr_array(ptrs) -> ctypes.Array:
    arr = (ctypes.c_void_p * max(1, len(ptrs)))()
    for i, v in enumerate(ptrs):
        arr[i] = int(v)
    return arr
