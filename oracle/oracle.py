"""ctypes front end of the CPU oracle — TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import
this module.  It builds (if needed) and loads ``oracle/libckks_oracle.so``, the
plain-C restatement of the reference's RNS-CKKS arithmetic, and exposes numpy
friendly wrappers.  Nothing in the product package imports it.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import threading

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libckks_oracle.so")
_lock = threading.Lock()
_lib = None

u64 = ctypes.c_uint64
u32 = ctypes.c_uint32
i32 = ctypes.c_int
P64 = ctypes.POINTER(ctypes.c_uint64)
PD = ctypes.POINTER(ctypes.c_double)


def build() -> str:
    """Compile the oracle with its Makefile (no-op when up to date)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def _sig(lib, name, res, args):
    fn = getattr(lib, name)
    fn.restype = res
    fn.argtypes = args
    return fn


def lib():
    global _lib
    with _lock:
        if _lib is None:
            build()
            L = ctypes.CDLL(_LIB_PATH)
            _sig(L, "oc_mulmod", u64, [u64, u64, u64])
            _sig(L, "oc_powmod", u64, [u64, u64, u64])
            _sig(L, "oc_invmod", u64, [u64, u64])
            _sig(L, "oc_is_prime", i32, [u64])
            _sig(L, "oc_first_prime", u64, [u32, u64])
            _sig(L, "oc_previous_prime", u64, [u64, u64])
            _sig(L, "oc_next_prime", u64, [u64, u64])
            _sig(L, "oc_ckks_moduli", i32, [u32, u32, u32, u32, u32, P64, P64, u32])
            _sig(L, "oc_ntt_primes", None, [u32, u32, u32, P64])
            _sig(L, "oc_root_of_unity", u64, [u64, u64])
            _sig(L, "oc_ntt_forward", None, [P64, u32, u64, u64])
            _sig(L, "oc_ntt_inverse", None, [P64, u32, u64, u64])
            _sig(L, "oc_ntt_batch", None, [P64, u32, u32, u32, P64, P64, i32, i32])
            _sig(L, "oc_rand_u64", u64, [u64, u64, u64])
            _lib = L
        return _lib


def _p64(a: np.ndarray):
    assert a.dtype == np.uint64 and a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(P64)


def ckks_moduli(log_n: int, num_q: int, scale_bits: int, first_bits: int, dnum: int):
    q = np.zeros(num_q, dtype=np.uint64)
    p = np.zeros(64, dtype=np.uint64)
    k = lib().oc_ckks_moduli(log_n, num_q, scale_bits, first_bits, dnum, _p64(q), _p64(p), 64)
    if k < 0:
        raise ValueError(f"oc_ckks_moduli failed ({k})")
    return [int(x) for x in q], [int(x) for x in p[:k]]


def ntt_primes(log_n: int, bits: int, k: int):
    out = np.zeros(k, dtype=np.uint64)
    lib().oc_ntt_primes(log_n, bits, k, _p64(out))
    return [int(x) for x in out]


def root_of_unity(m: int, q: int) -> int:
    return int(lib().oc_root_of_unity(m, q))


def ntt_batch(data: np.ndarray, primes, psis, inverse: bool, threads: int = 1) -> np.ndarray:
    """In-place batched NTT on u64[n_polys][n_limbs][N]."""
    assert data.ndim == 3
    n_polys, n_limbs, n = data.shape
    log_n = n.bit_length() - 1
    q = np.asarray(primes, dtype=np.uint64)
    r = np.asarray(psis, dtype=np.uint64)
    assert len(q) == n_limbs and len(r) == n_limbs
    lib().oc_ntt_batch(_p64(data), n_polys, n_limbs, log_n, _p64(q), _p64(r), int(inverse), threads)
    return data


def rand_u64(seed: int, stream: int, index: int) -> int:
    return int(lib().oc_rand_u64(seed, stream, index))
