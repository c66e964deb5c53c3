"""fhe_mamba_b200 — B200-native RNS-CKKS evaluation backend for fhemamba.

Host side of the C ABI in include/fhe_b200.h.  The compute path is
libfhe_b200.so (hand-written sm_100a CUDA); this package only marshals
arguments and raises on error statuses.
"""
from ._lib import FheError, InvalidArgument, StateError, load  # noqa: F401
from .ckks import CCParams, Ciphertext, CryptoContext, GenCryptoContext, Plaintext  # noqa: F401
from .ntt import NttContext  # noqa: F401

__all__ = ["FheError", "InvalidArgument", "StateError", "NttContext", "load", "CCParams", "CryptoContext",
           "GenCryptoContext", "Ciphertext", "Plaintext"]
