"""OpenFHE-style CKKS API over the C ABI.

Mirrors the CryptoContext calls the reference's native executor makes
(native/fideslib_stage0/src/packed_fideslib.cpp:117-281, 1060-1090):
GenCryptoContext, KeyGen, EvalMultKeyGen, EvalRotateKeyGen,
MakeCKKSPackedPlaintext, Encrypt, Decrypt, EvalAdd/EvalSub/EvalMult,
RescaleInPlace, EvalRotate, EvalFastRotationPrecompute/EvalFastRotation.
Every operation runs on the GPU through libfhe_b200.so; errors surface as
FheError (InvalidArgument / StateError) the way OpenFHE throws.
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass

import numpy as np

from . import _lib
from ._lib import P32, P64, PD, PI32, call

vp = ctypes.c_void_p


@dataclass
class CCParams:
    """CCParams<CryptoContextCKKSRNS> fields the reference sets."""

    ring_dim: int = 1 << 16
    multiplicative_depth: int = 44
    scaling_mod_size: int = 59
    first_mod_size: int = 60
    num_large_digits: int = 3
    batch_size: int = 0  # 0 -> ring_dim / 2
    device: int = 0

    def SetRingDim(self, n):
        self.ring_dim = n

    def SetMultiplicativeDepth(self, d):
        self.multiplicative_depth = d

    def SetScalingModSize(self, b):
        self.scaling_mod_size = b

    def SetFirstModSize(self, b):
        self.first_mod_size = b

    def SetNumLargeDigits(self, d):
        self.num_large_digits = d

    def SetBatchSize(self, s):
        self.batch_size = s


class Plaintext:
    def __init__(self, cc: "CryptoContext", h):
        self.cc, self._h = cc, h

    @property
    def handle(self):
        return self._h

    def info(self):
        nl, sc = ctypes.c_uint32(), ctypes.c_double()
        call("fhe_pt_info", self._h, ctypes.byref(nl), ctypes.byref(sc))
        return nl.value, sc.value

    def GetLevel(self):
        return self.cc.n_q - self.info()[0]

    def GetScalingFactor(self):
        return self.info()[1]

    def GetCKKSPackedValue(self, count=None):
        n = self.cc.slots if count is None else count
        re = np.zeros(n)
        im = np.zeros(n)
        call("fhe_decode", self.cc.h, self._h, re.ctypes.data_as(PD), im.ctypes.data_as(PD), n)
        return re + 1j * im

    def GetRealPackedValue(self, count=None):
        return self.GetCKKSPackedValue(count).real

    def residues(self):
        nl, _ = self.info()
        out = np.zeros((nl, self.cc.n), dtype=np.uint64)
        call("fhe_pt_download", self.cc.h, self._h, out.ctypes.data_as(P64))
        return out

    def __del__(self):
        try:
            if self._h and self._h.value:
                call("fhe_pt_free", self._h)
        except Exception:
            pass


class Ciphertext:
    def __init__(self, cc: "CryptoContext", h):
        self.cc, self._h = cc, h

    @property
    def handle(self):
        return self._h

    def info(self):
        nc, nl, nd, sc = ctypes.c_uint32(), ctypes.c_uint32(), ctypes.c_uint32(), ctypes.c_double()
        call("fhe_ct_info", self._h, ctypes.byref(nc), ctypes.byref(nl), ctypes.byref(nd), ctypes.byref(sc))
        return nc.value, nl.value, nd.value, sc.value

    def GetLevel(self):
        return self.cc.n_q - self.info()[1]

    def GetNoiseScaleDeg(self):
        return self.info()[2]

    def GetScalingFactor(self):
        return self.info()[3]

    def n_limbs(self):
        return self.info()[1]

    def Clone(self):
        return self.cc._ct("fhe_ct_clone", self._h)

    def residues(self):
        nc, nl, _, _ = self.info()
        out = np.zeros((nc, nl, self.cc.n), dtype=np.uint64)
        call("fhe_ct_download", self.cc.h, self._h, out.ctypes.data_as(P64))
        return out

    def __del__(self):
        try:
            if self._h and self._h.value:
                call("fhe_ct_free", self._h)
        except Exception:
            pass


class CryptoContext:
    """GenCryptoContext(params) + LoadContext on one GPU."""

    def __init__(self, params: CCParams):
        log_n = int(params.ring_dim).bit_length() - 1
        if 1 << log_n != params.ring_dim:
            raise _lib.InvalidArgument(-1, "GenCryptoContext", "ring dimension must be a power of two")
        p = _lib.Params(log_n, params.multiplicative_depth, params.scaling_mod_size, params.first_mod_size,
                        params.num_large_digits, params.batch_size or params.ring_dim // 2, params.device, 0)
        h = vp()
        call("fhe_ctx_create", ctypes.byref(p), ctypes.byref(h))
        self.h = h
        self.device = params.device
        self.subslot_sizes = ()  # sub-slot refresh setups (slot counts)
        info = (ctypes.c_uint32 * 8)()
        call("fhe_ctx_info", h, ctypes.cast(info, vp))
        self.log_n, self.n_q, self.n_p, self.dnum, self.alpha, self.slots = list(info)[:6]
        self.n = 1 << self.log_n
        q = np.zeros(self.n_q, dtype=np.uint64)
        pp = np.zeros(max(self.n_p, 1), dtype=np.uint64)
        call("fhe_ctx_moduli", h, q.ctypes.data_as(P64), None, pp.ctypes.data_as(P64), None)
        self.q = [int(x) for x in q]
        self.p = [int(x) for x in pp[: self.n_p]]

    # -- context queries
    def GetRingDimension(self):
        return self.n

    def GetBatchSize(self):
        return self.slots

    def level_scale(self, n_limbs=None):
        out = ctypes.c_double()
        call("fhe_level_scale", self.h, self.n_q if n_limbs is None else n_limbs, ctypes.byref(out))
        return out.value

    def stream_ptr(self):
        s = vp()
        call("fhe_ctx_stream", self.h, ctypes.byref(s))
        return int(s.value or 0)

    def synchronize(self):
        call("fhe_ctx_synchronize", self.h)

    # -- keys
    def KeyGen(self, seed: int = 0):
        call("fhe_keygen", self.h, seed)

    def EvalMultKeyGen(self, *_):
        """The relinearisation key is generated by KeyGen."""

    def EvalRotateKeyGen(self, steps):
        arr = np.ascontiguousarray(np.asarray(list(steps), dtype=np.int32))
        call("fhe_rotation_keygen", self.h, arr.ctypes.data_as(PI32), len(arr))

    def EvalConjugateKeyGen(self):
        call("fhe_conjugation_keygen", self.h)

    def galois_element(self, step: int) -> int:
        g = ctypes.c_uint64()
        call("fhe_galois_element", self.h, step, ctypes.byref(g))
        return g.value

    def key(self, kind: int, galois: int = 0):
        D = (self.n_q + self.alpha - 1) // self.alpha
        words = {0: (self.n_q + self.n_p) * self.n, 4: (self.n_q + self.n_p) * self.n, 1: 2 * self.n_q * self.n}.get(
            kind, D * 2 * (self.n_q + self.n_p) * self.n)
        out = np.zeros(words, dtype=np.uint64)
        call("fhe_key_download", self.h, kind, galois, out.ctypes.data_as(P64), words)
        return out

    # -- encoding / encryption
    def MakeCKKSPackedPlaintext(self, values, noise_scale_deg=1, level=0, params=None, slots=None,
                                scale=0.0):
        v = np.ascontiguousarray(np.asarray(values, dtype=np.complex128))
        re = np.ascontiguousarray(v.real)
        im = np.ascontiguousarray(v.imag)
        h = vp()
        call("fhe_encode", self.h, re.ctypes.data_as(PD), im.ctypes.data_as(PD), len(v), self.n_q - level,
             float(scale), ctypes.byref(h))
        return Plaintext(self, h)

    def MakeCKKSPackedPlaintexts(self, vectors, level=0, scale=0.0):
        """Batched MakeCKKSPackedPlaintext (one device pass for many vectors)."""
        arr = np.asarray(vectors, dtype=np.complex128)
        if arr.ndim != 2:
            raise _lib.InvalidArgument(-1, "MakeCKKSPackedPlaintexts", "expected a 2-D array of vectors")
        re = np.ascontiguousarray(arr.real)
        im = np.ascontiguousarray(arr.imag)
        outs = (vp * arr.shape[0])()
        call("fhe_encode_batch", self.h, re.ctypes.data_as(PD), im.ctypes.data_as(PD), arr.shape[0],
             arr.shape[1], self.n_q - level, float(scale), outs)
        return [Plaintext(self, vp(o)) for o in outs]

    def MakeReplicatedDiagonals(self, w_dev_ptr: int, m: int, cols: int, R: int, T: int, win: int, baby: int,
                                level=0, scale=0.0):
        """The T diagonal plaintexts of a replicated BSGS layout generated on the
        device from W (m x cols, fp64, row-major, device pointer w_dev_ptr)."""
        outs = (vp * T)()
        call("fhe_encode_replicated_diagonals", self.h, vp(w_dev_ptr), m, cols, R, T, win, baby, self.n_q - level,
             float(scale), outs)
        return [Plaintext(self, vp(o)) for o in outs]

    def EvalLinearTransform(self, ct, diagonals, baby: int, giant: int, stride: int = 1, giant_offset: int = 0):
        """out = sum_g rot(sum_j diagonals[g*baby+j] (.) rot(ct, j*stride), (g*baby - giant_offset)*stride);
        None = zero diagonal."""
        if len(diagonals) != baby * giant:
            raise _lib.InvalidArgument(-1, "EvalLinearTransform", "need baby*giant diagonals")
        arr = (vp * len(diagonals))(*[d.handle if d is not None else None for d in diagonals])
        return self._ct("fhe_linear_transform", ct.handle, arr, baby, giant, int(stride), int(giant_offset))

    def EvalBootstrapSetup(self, level_budget=(4, 4), dim1=(0, 0), slots: int = 0, correction_factor: int = 0,
                           slots_to_coeffs_first: bool = False, sparse_hamming_weight: int = 0):
        """OpenFHE EvalBootstrapSetup(levelBudget, dim1, slots, correctionFactor[, slotsToCoeffsFirst]);
        dim1 is accepted for signature compatibility (the BSGS split is chosen per group).
        sparse_hamming_weight > 0 selects sparse-secret encapsulation."""
        call("fhe_bootstrap_setup", self.h, int(level_budget[0]), int(level_budget[1]), int(slots),
             int(correction_factor), int(bool(slots_to_coeffs_first)), int(sparse_hamming_weight))

    def EvalBootstrapSubslotSetup(self, slots: int, level_budget=(4, 4), correction_factor: int = 0):
        """A sub-slot refresh for inputs zero outside slots [0, slots) (a power
        of two <= half the context's slots): one EvalMod instead of two, the
        same levels as the full bootstrap, output zero outside [0, slots).
        EvalBootstrapKeyGen generates its keys; refresh(..., support=) picks it."""
        call("fhe_bootstrap_subslot_setup", self.h, int(slots), int(level_budget[0]), int(level_budget[1]),
             int(correction_factor))
        self.subslot_sizes = tuple(sorted(set(self.subslot_sizes) | {int(slots)}))

    def bootstrap_components(self, ct, passes: int = 2, merge: bool = False):
        """The reference's two-pass refresh (PackedEvaluator::bootstrap_components,
        packed_fideslib.cpp:235-270): first = bootstrap(x); the residual
        (x - first) * 4096 is bootstrapped again as `second`.  With merge, the
        pair becomes 4096 * first + second by an exact integer multiple
        (merge_refresh_correction) and divisor = 4096.
        Returns (first, second or None, divisor); x ~ (first + second / 4096) / divisor-corrected."""
        x = ct.Clone()
        while x.GetNoiseScaleDeg() > 1:
            self.RescaleInPlace(x)
        first = self.EvalBootstrap(x)
        if passes == 1:
            return first, None, 1.0
        a, b = x.Clone(), first.Clone()
        while b.GetNoiseScaleDeg() > 1:
            self.RescaleInPlace(b)
        target = max(a.GetLevel(), b.GetLevel())
        for name in ("a", "b"):
            v = a if name == "a" else b
            while v.GetLevel() < target:
                v = self.EvalMult(v, 1.0)
                while v.GetNoiseScaleDeg() > 1:
                    self.RescaleInPlace(v)
            if name == "a":
                a = v
            else:
                b = v
        residual = self.EvalMult(self.EvalSub(a, b), 4096.0)
        while residual.GetNoiseScaleDeg() > 1:
            self.RescaleInPlace(residual)
        second = self.EvalBootstrap(residual)
        if merge and first.GetLevel() == second.GetLevel() and \
                first.GetNoiseScaleDeg() == second.GetNoiseScaleDeg():
            return self.EvalAdd(self.MultByInteger(first, 4096), second), None, 4096.0
        return first, second, 1.0

    def refresh(self, ct, bound: float = 1.0, passes: int = 2, merge: bool = False, support: int = 0):
        """PackedEvaluator::refresh (packed_fideslib.cpp:271-281): bootstrap x / bound
        (one or two passes) and scale back by bound.  Without merge this is one
        library call (fhe_refresh); the merge variant composes the host steps.
        support > 0 declares ct zero outside slots [0, support): a sub-slot
        refresh set up for at least that many slots then runs it."""
        if not merge:
            return self.EvalRefresh(ct, bound, passes, support)
        return self.host_refresh(ct, bound, passes, merge)

    def host_refresh(self, ct, bound: float = 1.0, passes: int = 2, merge: bool = False):
        """refresh() composed from host-side calls (bootstrap_components)."""
        scaled = self.EvalMult(ct, 1.0 / bound)
        first, second, divisor = self.bootstrap_components(scaled, passes, merge)
        if second is None:
            return self.EvalMult(first, bound / divisor)
        return self.EvalMult(self.EvalAdd(first, self.EvalMult(second, 1.0 / 4096.0)), bound)

    # -- files for a process-separated client and server
    def SerializeCiphertext(self, ct, path):
        """OpenFHE Serial::SerializeToFile(path, ct) (the reference's handoff)."""
        call("fhe_ct_save", self.h, ct.handle, os.fsencode(str(path)))

    def DeserializeCiphertext(self, path):
        return self._ct("fhe_ct_load", os.fsencode(str(path)))

    def SerializeKeys(self, path, include_secret: bool = False):
        """Public, relinearisation and rotation keys (+ the secret key if asked)."""
        call("fhe_keys_save", self.h, os.fsencode(str(path)), int(bool(include_secret)))

    def DeserializeKeys(self, path):
        """Installs a key bundle; without the secret the context evaluates but
        cannot decrypt or generate keys (a server)."""
        call("fhe_keys_load", self.h, os.fsencode(str(path)))

    def EvalRefresh(self, ct, bound: float = 1.0, passes: int = 2, support: int = 0):
        """One library call for the reference's refresh (fhe_refresh): the same
        arithmetic as refresh() without the host round trips (fhe_refresh_support
        with a support)."""
        if support:
            return self._ct("fhe_refresh_support", ct.handle, float(bound), int(passes), int(support))
        return self._ct("fhe_refresh", ct.handle, float(bound), int(passes))

    def EvalBootstrapKeyGen(self, secret_key=None, slots: int = 0):
        call("fhe_bootstrap_keygen", self.h)

    def EvalBootstrap(self, ct):
        return self._ct("fhe_bootstrap", ct.handle)

    def EvalBootstrapStage(self, stage: int, ct):
        """0 = scale down and ModRaise, 1 = CoeffToSlot, 2 = EvalMod, 3 = SlotToCoeff."""
        return self._ct("fhe_bootstrap_stage", int(stage), ct.handle)

    _COUNTERS = ("tensor", "relin", "rotations", "modup", "moddown", "key_inner", "rescales", "ntt_limbs",
                 "bootstraps")

    def counters(self, reset: bool = False) -> dict:
        """Operation counters since creation or the last reset."""
        a = (ctypes.c_uint64 * len(self._COUNTERS))()
        call("fhe_ctx_counters", self.h, ctypes.cast(a, vp), int(reset))
        return dict(zip(self._COUNTERS, (int(v) for v in a)))

    def SetConversionKernel(self, kernel: str):
        """'cuda' (64-bit multiply-accumulates), 'tensor' (tcgen05 int8 MMA for
        bases of 12+ limbs, where it is faster) or 'tensor-all' (every base;
        tests) for the key switches' basis conversions; identical results."""
        call("fhe_ctx_set_conversion", self.h, {"cuda": 0, "tensor": 1, "tensor-all": 2}[kernel])

    def SetKeySwitchFusion(self, fused: bool):
        """Form the Q limbs' key inner product inside ModDown's last NTT pass
        (True) or in a separate kernel (False); the results are identical."""
        call("fhe_ctx_set_keyswitch_fusion", self.h, int(bool(fused)))

    def SetGiantStepHoisting(self, on: bool):
        """Giant steps of a linear transform share one ModDown (True, the
        default) or each take a full key switch (False); the results agree
        within the key switching noise."""
        call("fhe_ctx_set_giant_hoisting", self.h, int(bool(on)))

    def level_counts(self):
        """The ModUps, key inner products, rescales and tensor products since the
        last counter reset, by the number of live Q limbs they ran at:
        {kind: {nq: count}} for the non-zero entries."""
        out = {}
        for kind, name in enumerate(("modup", "key_inner", "rescale", "tensor")):
            a = (ctypes.c_uint64 * 64)()
            call("fhe_ctx_level_counts", self.h, kind, ctypes.cast(a, vp), 64)
            out[name] = {i: int(v) for i, v in enumerate(a) if v}
        return out

    def bootstrap_info(self):
        c, d, k = ctypes.c_int32(), ctypes.c_uint32(), ctypes.c_uint32()
        call("fhe_bootstrap_info", self.h, ctypes.byref(c), ctypes.byref(d), ctypes.byref(k))
        return {"correction": c.value, "chebyshev_degree": d.value, "rotation_keys": k.value}

    def bootstrap_levels(self):
        """Limb counts of the last bootstrap after ModRaise, CoeffToSlot, EvalMod, SlotToCoeff."""
        a = (ctypes.c_uint32 * 4)()
        call("fhe_bootstrap_levels", self.h, a)
        return list(a)

    def ModRaise(self, ct):
        return self._ct("fhe_mod_raise", ct.handle)

    def MultByI(self, ct):
        return self._ct("fhe_mul_i", ct.handle)

    def SetScalingFactor(self, ct, scale: float):
        call("fhe_ct_set_scale", self.h, ct.handle, float(scale))

    def EvalChebyshevSeries(self, ct, coefficients, a: float, b: float):
        """sum_i c_i T_i(u), u = (2x - a - b) / (b - a), Paterson-Stockmeyer on the device."""
        c = np.ascontiguousarray(np.asarray(coefficients, dtype=np.float64))
        return self._ct("fhe_chebyshev", ct.handle, c.ctypes.data_as(PD), len(c), float(a), float(b))

    def EvalChebyshevFunction(self, func, ct, a: float, b: float, degree: int):
        """Interpolates func at Chebyshev nodes on [a, b] and evaluates the series."""
        return self.EvalChebyshevSeries(ct, chebyshev_coefficients(func, a, b, degree), a, b)

    def Encrypt(self, pt: Plaintext, _unused=None):
        if isinstance(_unused, Plaintext):  # Encrypt(publicKey, pt) call order
            pt = _unused
        return self._ct("fhe_encrypt", pt.handle)

    def Decrypt(self, ct: Ciphertext, _unused=None):
        if isinstance(ct, Ciphertext):
            c = ct
        else:
            c = _unused
        h = vp()
        call("fhe_decrypt", self.h, c.handle, ctypes.byref(h))
        return Plaintext(self, h)

    def upload(self, residues: np.ndarray, noise_deg=1, scale=1.0):
        r = np.ascontiguousarray(residues, dtype=np.uint64)
        h = vp()
        call("fhe_ct_upload", self.h, r.ctypes.data_as(P64), r.shape[0], r.shape[1], noise_deg, scale,
             ctypes.byref(h))
        return Ciphertext(self, h)

    def upload_plain(self, residues: np.ndarray, scale=1.0):
        r = np.ascontiguousarray(residues, dtype=np.uint64)
        h = vp()
        call("fhe_pt_upload", self.h, r.ctypes.data_as(P64), r.shape[0], scale, ctypes.byref(h))
        return Plaintext(self, h)

    # -- arithmetic
    def _ct(self, fn, *args):
        h = vp()
        call(fn, self.h, *args, ctypes.byref(h))
        return Ciphertext(self, h)

    def EvalAdd(self, a, b):
        if isinstance(b, Ciphertext):
            return self._ct("fhe_add", a.handle, b.handle)
        if isinstance(b, Plaintext):
            return self._ct("fhe_add_plain", a.handle, b.handle)
        return self._ct("fhe_add_scalar", a.handle, float(b))

    def EvalSub(self, a, b):
        if isinstance(b, Ciphertext):
            return self._ct("fhe_sub", a.handle, b.handle)
        if isinstance(b, Plaintext):
            return self._ct("fhe_sub_plain", a.handle, b.handle)
        return self._ct("fhe_add_scalar", a.handle, -float(b))

    def EvalNegate(self, a):
        return self._ct("fhe_negate", a.handle)

    def EvalMult(self, a, b):
        if isinstance(b, Ciphertext):
            return self._ct("fhe_mul", a.handle, b.handle)
        if isinstance(b, Plaintext):
            return self._ct("fhe_mul_plain", a.handle, b.handle)
        return self._ct("fhe_mul_scalar", a.handle, float(b))

    def EvalSquare(self, a):
        return self._ct("fhe_mul", a.handle, a.handle)

    def EvalMultNoRelin(self, a, b):
        return self._ct("fhe_tensor", a.handle, b.handle)

    def Relinearize(self, a):
        return self._ct("fhe_relinearize", a.handle)

    def MultByInteger(self, a, v: int):
        return self._ct("fhe_mul_int", a.handle, int(v))

    def RescaleInPlace(self, a):
        call("fhe_rescale", self.h, a.handle)

    def Rescale(self, a):
        c = a.Clone()
        self.RescaleInPlace(c)
        return c

    def LevelReduceInPlace(self, a, levels: int):
        call("fhe_level_reduce", self.h, a.handle, levels)

    def EvalRotate(self, a, step: int):
        return self._ct("fhe_rotate", a.handle, int(step))

    def EvalConjugate(self, a):
        return self._ct("fhe_conjugate", a.handle)

    def EvalFastRotationPrecompute(self, a):
        """Hoisting handle: the ModUp is shared inside EvalFastRotation's batch call."""
        return a

    def EvalFastRotation(self, a, steps, m=None, precomp=None):
        steps = list(steps) if hasattr(steps, "__iter__") else [steps]
        arr = np.ascontiguousarray(np.asarray(steps, dtype=np.int32))
        outs = (vp * len(arr))()
        call("fhe_rotate_hoisted", self.h, a.handle, arr.ctypes.data_as(PI32), len(arr), outs)
        res = [Ciphertext(self, vp(o)) for o in outs]
        return res

    def close(self):
        if getattr(self, "h", None) and self.h.value:
            call("fhe_ctx_destroy", self.h)
            self.h = vp()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def GenCryptoContext(params: CCParams) -> CryptoContext:
    return CryptoContext(params)


def chebyshev_coefficients(func, a: float, b: float, degree: int) -> np.ndarray:
    """Chebyshev interpolation coefficients c_0..c_degree of func on [a, b]
    (Chebyshev nodes of the first kind; the series is sum c_i T_i(u))."""
    n = degree + 1
    j = np.arange(n)
    nodes = np.cos(np.pi * (j + 0.5) / n)
    fx = np.asarray(func((b - a) / 2 * nodes + (a + b) / 2), dtype=np.float64)
    c = np.array([2.0 / n * np.sum(fx * np.cos(np.pi * k * (j + 0.5) / n)) for k in range(n)])
    c[0] /= 2
    return c


def bsgs_diagonals(W: np.ndarray, baby: int, giant: int, slots: int):
    """Diagonal layout for y = W x (W: m x n) with the input replicated twice
    (slot s holds x[s mod n] for s < 2n).  Diagonal d = g*baby + j holds
    W[i, (i + d) mod n] at slot i + g*baby (pre-rotated by the giant step), so
    sum_g rot(sum_j diag (.) rot(x_rep, j), g*baby) puts y[i] in slot i.
    Returns baby*giant arrays (None for diagonals d >= n)."""
    m, n = W.shape
    if baby * giant < n:
        raise ValueError("baby*giant must cover every diagonal")
    if (giant - 1) * baby + m > slots or 2 * n > slots:
        raise ValueError("layout does not fit the slots")
    rows = np.arange(m)
    out = []
    for g in range(giant):
        for j in range(baby):
            d = g * baby + j
            if d >= n:
                out.append(None)
                continue
            v = np.zeros(slots)
            v[g * baby + rows] = W[rows, (rows + d) % n]
            out.append(v)
    return out
