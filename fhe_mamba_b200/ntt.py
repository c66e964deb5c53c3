"""Raw RNS limb transforms through the C ABI (fhe_ntt / fhe_intt).

``NttContext`` mirrors what the reference's NTT probe drives through FIDESlib
(experiments/ntt_warp_tail/probe.cu:57-77): forward/inverse negacyclic
transforms of u64[n_polys][n_limbs][N] residue buffers, OpenFHE ordering.
Buffers may be numpy arrays (host; copied to the GPU and back inside the call)
or torch CUDA tensors of dtype uint64/int64 (device; transformed in place).
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import _lib
from ._lib import P64, call


def _is_torch_cuda(x) -> bool:
    return type(x).__module__.startswith("torch") and getattr(x, "is_cuda", False)


class NttContext:
    def __init__(self, log_n: int, primes, device: int = 0):
        arr = np.ascontiguousarray(np.asarray(primes, dtype=np.uint64))
        h = ctypes.c_void_p()
        call("fhe_ctx_create_ntt", log_n, arr.ctypes.data_as(P64), len(arr), device, ctypes.byref(h))
        self._h = h
        self.log_n = log_n
        self.n = 1 << log_n
        self.primes = [int(v) for v in arr]
        self.device = device

    @property
    def handle(self):
        return self._h

    def roots(self):
        out = np.zeros(len(self.primes), dtype=np.uint64)
        call("fhe_ctx_roots", self._h, out.ctypes.data_as(P64), len(out))
        return [int(v) for v in out]

    def stream_ptr(self) -> int:
        s = ctypes.c_void_p()
        call("fhe_ctx_stream", self._h, ctypes.byref(s))
        return int(s.value or 0)

    def synchronize(self):
        call("fhe_ctx_synchronize", self._h)

    def butterfly_ceiling(self) -> float:
        """Butterflies/s of the forward butterfly run on registers only (the
        integer-pipe roofline of the transform on this GPU)."""
        out = ctypes.c_double()
        call("fhe_ntt_butterfly_ceiling", self._h, ctypes.byref(out))
        return out.value

    def _run(self, name, data, limb0):
        if _is_torch_cuda(data):
            if data.dim() != 3 or data.shape[-1] != self.n or not data.is_contiguous():
                raise ValueError("device buffer must be a contiguous [polys, limbs, N] tensor")
            if data.element_size() != 8:
                raise ValueError("device buffer must hold 64-bit words")
            ptr = ctypes.cast(ctypes.c_void_p(data.data_ptr()), P64)
            call(name, self._h, ptr, data.shape[0], limb0, data.shape[1], _lib.FHE_MEM_DEVICE)
            return data
        if not isinstance(data, np.ndarray) or data.dtype != np.uint64 or data.ndim != 3:
            raise ValueError("host buffer must be a uint64 numpy array [polys, limbs, N]")
        if data.shape[-1] != self.n or not data.flags["C_CONTIGUOUS"]:
            raise ValueError("host buffer must be C-contiguous with last dimension N")
        call(name, self._h, data.ctypes.data_as(P64), data.shape[0], limb0, data.shape[1],
             _lib.FHE_MEM_HOST)
        return data

    def forward(self, data, limb0: int = 0):
        """In-place forward NTT; limb l of every poly uses prime limb0 + l."""
        return self._run("fhe_ntt", data, limb0)

    def inverse(self, data, limb0: int = 0):
        """In-place inverse NTT."""
        return self._run("fhe_intt", data, limb0)

    def close(self):
        if getattr(self, "_h", None) and self._h.value:
            call("fhe_ctx_destroy", self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
