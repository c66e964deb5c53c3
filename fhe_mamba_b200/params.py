"""Host-side CKKS parameter generation through the C ABI (no device work)."""
from __future__ import annotations

import ctypes

import numpy as np

from ._lib import P32, P64, call


def ckks_moduli(log_n: int, mult_depth: int, scaling_mod_size: int, first_mod_size: int,
                num_large_digits: int):
    """(Q primes, P primes) exactly as fhe_ctx_create will use them."""
    q = np.zeros(mult_depth + 1, dtype=np.uint64)
    p = np.zeros(64, dtype=np.uint64)
    nq, np_ = ctypes.c_uint32(), ctypes.c_uint32()
    call("fhe_gen_ckks_moduli", log_n, mult_depth, scaling_mod_size, first_mod_size,
         num_large_digits, q.ctypes.data_as(P64), ctypes.byref(nq), p.ctypes.data_as(P64),
         ctypes.byref(np_))
    return [int(x) for x in q[: nq.value]], [int(x) for x in p[: np_.value]]


def ntt_primes(log_n: int, bits: int, count: int):
    out = np.zeros(count, dtype=np.uint64)
    call("fhe_gen_ntt_primes", log_n, bits, count, out.ctypes.data_as(P64))
    return [int(x) for x in out]
