"""Packed-program execution through the C ABI (fhe_program_validate / fhe_program_run).

``run_program`` is the in-process form of the ``packed_b200`` executable, the
drop-in for the reference's ``packed_fideslib PROGRAM RESULT POLY_TOL EXACT_TOL``
(native/fideslib_stage0/src/packed_fideslib.cpp:882-1403).
"""
from __future__ import annotations

import ctypes
import os

from . import _lib
from ._lib import call

CLI = os.path.join(os.path.dirname(os.path.abspath(__file__)), "packed_b200")


class ProgramOptions(ctypes.Structure):
    _fields_ = [("log_n", ctypes.c_uint32), ("depth", ctypes.c_uint32), ("scale_bits", ctypes.c_uint32),
                ("first_bits", ctypes.c_uint32), ("dnum", ctypes.c_uint32), ("bootstrap_passes", ctypes.c_int32),
                ("s2c_first", ctypes.c_int32), ("trace", ctypes.c_int32), ("device", ctypes.c_int32),
                ("sparse_h", ctypes.c_uint32), ("seed", ctypes.c_uint64), ("security128", ctypes.c_int32),
                ("security_digits", ctypes.c_uint32)]


def security_audit(log_n: int, depth: int = 44, scale_bits: int = 59, first_bits: int = 60, dnum: int = 4) -> dict:
    """Classical-128 audit of a parameter set (no GPU): the parameters.json
    that --security 128-classic writes, with its `passed` verdict."""
    import json
    buf = ctypes.create_string_buffer(2048)
    ok = ctypes.c_int32()
    call("fhe_security_audit", log_n, depth, scale_bits, first_bits, dnum, buf, len(buf), ctypes.byref(ok))
    return json.loads(buf.value.decode())


def validate_program(path: str) -> dict:
    """Parses a fhemamba-packed-v1/v2 program (no GPU); raises InvalidArgument when malformed."""
    s, n, o = ctypes.c_int32(), ctypes.c_int32(), ctypes.c_int32()
    call("fhe_program_validate", os.fsencode(path), ctypes.byref(s), ctypes.byref(n), ctypes.byref(o))
    return {"slots": s.value, "nodes": n.value, "outputs": o.value}


def run_program(program: str, result: str, poly_tol: float, exact_tol: float, client_head: str | None = None,
                **options) -> bool:
    """Evaluates the program on the GPU and writes the result JSON; True when every gate passes."""
    opt = ProgramOptions(**options)
    rc = _lib.load().fhe_program_run(os.fsencode(program), os.fsencode(client_head) if client_head else None,
                                     os.fsencode(result), float(poly_tol), float(exact_tol), ctypes.byref(opt))
    if rc < 0:
        _lib.check(rc, "fhe_program_run")
    return rc == 0
