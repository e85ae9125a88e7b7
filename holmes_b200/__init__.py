"""holmes_b200: a B200-native RNS-CKKS engine for the Holmes linear / key-switch hot path.

``holmes_b200.fhe`` is the EasyFHE-shaped CKKS API, ``holmes_b200.linear`` the diagonal (BSGS) linear
operators with the reference's interface, ``holmes_b200.collectives`` the multi-GPU exchange.  All
arithmetic runs in ``lib/libholmes_cuda.so`` (``holmes_b200/csrc``, C ABI in ``include/holmes_cuda.h``).
"""
__all__ = ["fhe", "linear"]
