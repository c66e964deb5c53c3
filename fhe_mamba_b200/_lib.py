"""ctypes binding of libfhe_b200.so (the C ABI in include/fhe_b200.h).

The shared library is the product: every call here goes to CUDA kernels.  If
the library is missing it is built with nvcc; if it cannot be loaded the import
fails loudly — there is no CPU fallback.
"""
from __future__ import annotations

import ctypes
import os
import re
import threading

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "libfhe_b200.so")
HEADER = os.path.join(os.path.dirname(_PKG), "include", "fhe_b200.h")

FHE_OK = 0
FHE_ERR_INVALID = -1
FHE_ERR_CUDA = -2
FHE_ERR_ALLOC = -3
FHE_ERR_STATE = -4
FHE_ERR_INTERNAL = -5
FHE_MEM_HOST = 0
FHE_MEM_DEVICE = 1

u32 = ctypes.c_uint32
i32 = ctypes.c_int32
u64 = ctypes.c_uint64
f64 = ctypes.c_double
vp = ctypes.c_void_p
P64 = ctypes.POINTER(ctypes.c_uint64)
P32 = ctypes.POINTER(ctypes.c_uint32)
PD = ctypes.POINTER(ctypes.c_double)
PI32 = ctypes.POINTER(ctypes.c_int32)


class FheError(RuntimeError):
    """Raised when an fhe_* call returns a negative status."""

    def __init__(self, code: int, fn: str, msg: str):
        super().__init__(f"{fn} failed ({code}): {msg}")
        self.code = code


class InvalidArgument(FheError, ValueError):
    pass


class StateError(FheError):
    pass


class Params(ctypes.Structure):
    _fields_ = [
        ("log_n", u32),
        ("mult_depth", u32),
        ("scaling_mod_size", u32),
        ("first_mod_size", u32),
        ("num_large_digits", u32),
        ("batch_size", u32),
        ("device", i32),
        ("reserved", u32),
    ]


# name -> (argtypes); all return int status.
SIGNATURES = {
    "fhe_last_error": [ctypes.c_char_p, ctypes.c_size_t],
    "fhe_ctx_create": [ctypes.POINTER(Params), ctypes.POINTER(vp)],
    "fhe_ctx_create_ntt": [u32, P64, u32, i32, ctypes.POINTER(vp)],
    "fhe_ctx_destroy": [vp],
    "fhe_ctx_moduli": [vp, P64, P32, P64, P32],
    "fhe_gen_ckks_moduli": [u32, u32, u32, u32, u32, P64, P32, P64, P32],
    "fhe_gen_ntt_primes": [u32, u32, u32, P64],
    "fhe_ctx_roots": [vp, P64, u32],
    "fhe_ctx_stream": [vp, ctypes.POINTER(vp)],
    "fhe_ctx_synchronize": [vp],
    "fhe_ntt": [vp, P64, u32, u32, u32, ctypes.c_int],
    "fhe_intt": [vp, P64, u32, u32, u32, ctypes.c_int],
    # CKKS
    "fhe_ctx_info": [vp, ctypes.c_void_p],
    "fhe_level_scale": [vp, u32, ctypes.POINTER(f64)],
    "fhe_keygen": [vp, u64],
    "fhe_galois_element": [vp, i32, P64],
    "fhe_rotation_keygen": [vp, PI32, u32],
    "fhe_conjugation_keygen": [vp],
    "fhe_key_download": [vp, ctypes.c_int, u64, P64, ctypes.c_size_t],
    "fhe_encode": [vp, PD, PD, u32, u32, f64, ctypes.POINTER(vp)],
    "fhe_decode": [vp, vp, PD, PD, u32],
    "fhe_encrypt": [vp, vp, ctypes.POINTER(vp)],
    "fhe_decrypt": [vp, vp, ctypes.POINTER(vp)],
    "fhe_ct_free": [vp],
    "fhe_pt_free": [vp],
    "fhe_ct_info": [vp, P32, P32, P32, ctypes.POINTER(f64)],
    "fhe_pt_info": [vp, P32, ctypes.POINTER(f64)],
    "fhe_ct_download": [vp, vp, P64],
    "fhe_ct_upload": [vp, P64, u32, u32, u32, f64, ctypes.POINTER(vp)],
    "fhe_pt_download": [vp, vp, P64],
    "fhe_pt_upload": [vp, P64, u32, f64, ctypes.POINTER(vp)],
    "fhe_ct_clone": [vp, vp, ctypes.POINTER(vp)],
    "fhe_add": [vp, vp, vp, ctypes.POINTER(vp)],
    "fhe_sub": [vp, vp, vp, ctypes.POINTER(vp)],
    "fhe_negate": [vp, vp, ctypes.POINTER(vp)],
    "fhe_add_plain": [vp, vp, vp, ctypes.POINTER(vp)],
    "fhe_sub_plain": [vp, vp, vp, ctypes.POINTER(vp)],
    "fhe_mul_plain": [vp, vp, vp, ctypes.POINTER(vp)],
    "fhe_add_scalar": [vp, vp, f64, ctypes.POINTER(vp)],
    "fhe_mul_scalar": [vp, vp, f64, ctypes.POINTER(vp)],
    "fhe_mul_int": [vp, vp, ctypes.c_int64, ctypes.POINTER(vp)],
    "fhe_tensor": [vp, vp, vp, ctypes.POINTER(vp)],
    "fhe_relinearize": [vp, vp, ctypes.POINTER(vp)],
    "fhe_mul": [vp, vp, vp, ctypes.POINTER(vp)],
    "fhe_rescale": [vp, vp],
    "fhe_level_reduce": [vp, vp, u32],
    "fhe_rotate": [vp, vp, i32, ctypes.POINTER(vp)],
    "fhe_conjugate": [vp, vp, ctypes.POINTER(vp)],
    "fhe_rotate_hoisted": [vp, vp, PI32, u32, ctypes.POINTER(vp)],
    "fhe_rescale_noalloc": [vp, vp, u32, u32, vp],
    "fhe_encode_batch": [vp, PD, PD, u32, u32, u32, f64, ctypes.POINTER(vp)],
    "fhe_encode_replicated_diagonals": [vp, vp, u32, u32, u32, u32, u32, u32, u32, f64, vp],
    "fhe_linear_transform": [vp, vp, ctypes.POINTER(vp), u32, u32, i32, i32, ctypes.POINTER(vp)],
    "fhe_ctx_counters": [vp, vp, i32],
    "fhe_ctx_level_counts": [vp, i32, vp, u32],
    "fhe_ctx_set_conversion": [vp, i32],
    "fhe_ctx_set_keyswitch_fusion": [vp, i32],
    "fhe_ctx_set_giant_hoisting": [vp, i32],
    "fhe_device_trim": [i32],
    "fhe_tc_timeouts": [vp],
    "fhe_kernel_launches": [ctypes.POINTER(ctypes.c_uint64)],
    "fhe_ntt_butterfly_ceiling": [vp, ctypes.POINTER(ctypes.c_double)],
    "fhe_refresh": [vp, vp, f64, i32, ctypes.POINTER(vp)],
    "fhe_refresh_support": [vp, vp, f64, i32, u32, ctypes.POINTER(vp)],
    "fhe_security_audit": [u32, u32, u32, u32, u32, ctypes.c_char_p, ctypes.c_size_t, ctypes.POINTER(i32)],
    "fhe_ct_save": [vp, vp, ctypes.c_char_p],
    "fhe_ct_load": [vp, ctypes.c_char_p, ctypes.POINTER(vp)],
    "fhe_keys_save": [vp, ctypes.c_char_p, i32],
    "fhe_keys_load": [vp, ctypes.c_char_p],
    "fhe_shard_init": [vp, u32, u32],
    "fhe_shard_plan_get": [vp, u32, vp],
    "fhe_shard_load_key": [vp, i32, u64],
    "fhe_shard_modup_prepare": [vp, u32, vp, vp],
    "fhe_shard_inner": [vp, u32, i32, u64, vp, vp, vp, vp],
    "fhe_shard_inner_digit": [vp, u32, u32, vp, vp],
    "fhe_shard_inner_tail": [vp, u32, i32, u64, vp, vp],
    "fhe_shard_moddown": [vp, u32, vp, vp, vp, vp, vp],
    "fhe_shard_automorphism": [vp, u32, u64, vp, vp],
    "fhe_bootstrap_setup": [vp, u32, u32, u32, i32, i32, u32],
    "fhe_bootstrap_subslot_setup": [vp, u32, u32, u32, i32],
    "fhe_bootstrap_keygen": [vp],
    "fhe_bootstrap": [vp, vp, ctypes.POINTER(vp)],
    "fhe_bootstrap_stage": [vp, i32, vp, ctypes.POINTER(vp)],
    "fhe_bootstrap_info": [vp, ctypes.POINTER(i32), ctypes.POINTER(u32), ctypes.POINTER(u32)],
    "fhe_bootstrap_levels": [vp, ctypes.POINTER(u32)],
    "fhe_program_validate": [ctypes.c_char_p, ctypes.POINTER(i32), ctypes.POINTER(i32), ctypes.POINTER(i32)],
    "fhe_program_run": [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_char_p, f64, f64, vp],
    "fhe_mod_raise": [vp, vp, ctypes.POINTER(vp)],
    "fhe_mul_i": [vp, vp, ctypes.POINTER(vp)],
    "fhe_ct_set_scale": [vp, vp, f64],
    "fhe_chebyshev": [vp, vp, PD, u32, f64, f64, ctypes.POINTER(vp)],
}

_lock = threading.Lock()
_lib = None


def header_symbols() -> list[str]:
    """Names of every function declared in include/fhe_b200.h."""
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*int\s+(fhe_\w+)\s*\(", text, flags=re.M)))


def load(build_if_missing: bool = True):
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            if not build_if_missing:
                raise OSError(f"{LIB_PATH} is missing; run fhe_mamba_b200.build.build()")
            from . import build as _build
            _build.build()
        lib = ctypes.CDLL(LIB_PATH)
        for name, args in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = ctypes.c_int
            fn.argtypes = args
        _lib = lib
        return lib


def last_error() -> str:
    buf = ctypes.create_string_buffer(4096)
    load().fhe_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def check(code: int, fn: str) -> None:
    if code == FHE_OK:
        return
    msg = last_error()
    if code == FHE_ERR_INVALID:
        raise InvalidArgument(code, fn, msg)
    if code == FHE_ERR_STATE:
        raise StateError(code, fn, msg)
    raise FheError(code, fn, msg)


def call(name: str, *args) -> None:
    check(getattr(load(), name)(*args), name)


def kernel_launches() -> int:
    """Kernels launched by libfhe_b200 in this process so far."""
    c = ctypes.c_uint64()
    call("fhe_kernel_launches", ctypes.byref(c))
    return c.value
