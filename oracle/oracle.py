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


# ---------------------------------------------------------------------------
# RNS-CKKS oracle (ckks_oracle_ckks.c)

PI64 = ctypes.POINTER(ctypes.c_int64)
STREAM_SECRET = 1 << 56
STREAM_PK_A = 2 << 56
STREAM_PK_E = 3 << 56


def stream_enc(kind: int, nonce: int) -> int:
    return (kind << 56) | (nonce & ((1 << 56) - 1))


def stream_key(kind: int, key_id: int, digit: int) -> int:
    return (kind << 56) | ((key_id & ((1 << 40) - 1)) << 8) | digit


def _ckks_sigs(L):
    vpp = ctypes.c_void_p
    _sig(L, "oc_ctx_new", vpp, [u32, u32, u32, P64, u32, u32])
    _sig(L, "oc_ctx_free", None, [vpp])
    _sig(L, "oc_ctx_psi", u64, [vpp, u32])
    _sig(L, "oc_num_digits", u32, [vpp, u32])
    _sig(L, "oc_poly_ntt", None, [vpp, P64, u32, u32, i32])
    _sig(L, "oc_sample_ternary_coef", ctypes.c_int64, [u64, u64, u64])
    _sig(L, "oc_sample_error_coef", ctypes.c_int64, [u64, u64, u64])
    _sig(L, "oc_sample_uniform_coef", u64, [u64, u64, u32, u32, u64, u64])
    _sig(L, "oc_sample_small", None, [vpp, u64, u64, i32, PI64])
    _sig(L, "oc_lift_small", None, [vpp, PI64, P64, u32, u32, i32])
    _sig(L, "oc_sample_uniform_poly", None, [vpp, u64, u64, P64, u32, u32])
    _sig(L, "oc_keygen_secret", None, [vpp, u64, PI64, P64])
    _sig(L, "oc_keygen_public", None, [vpp, u64, P64, P64])
    _sig(L, "oc_keygen_switch", None, [vpp, u64, u64, P64, P64, P64])
    _sig(L, "oc_automorphism_ntt", None, [vpp, P64, u32, u64, P64])
    _sig(L, "oc_automorphism_coef", None, [vpp, PI64, u64, PI64])
    _sig(L, "oc_rotation_galois", u64, [vpp, ctypes.c_int64])
    _sig(L, "oc_encode", i32, [vpp, PD, PD, u32, ctypes.c_double, u32, P64])
    _sig(L, "oc_decode", None, [vpp, P64, u32, ctypes.c_double, PD, PD])
    _sig(L, "oc_encrypt_pk", None, [vpp, u64, u64, P64, P64, u32, P64])
    _sig(L, "oc_decrypt", None, [vpp, P64, P64, u32, u32, P64])
    for nm in ("oc_add", "oc_sub", "oc_mul_pointwise"):
        _sig(L, nm, None, [vpp, P64, P64, u32, P64])
    _sig(L, "oc_tensor", None, [vpp, P64, P64, u32, P64])
    _sig(L, "oc_modup", None, [vpp, P64, u32, P64])
    _sig(L, "oc_key_inner", None, [vpp, P64, u32, P64, P64])
    _sig(L, "oc_moddown", None, [vpp, P64, u32, P64])
    _sig(L, "oc_keyswitch", None, [vpp, P64, u32, P64, P64])
    _sig(L, "oc_relinearize", None, [vpp, P64, u32, P64, P64])
    _sig(L, "oc_rotate", None, [vpp, P64, u32, u64, P64, P64])
    _sig(L, "oc_rescale", None, [vpp, P64, u32, u32, P64])


_ckks_ready = False


def _pd(a: np.ndarray):
    assert a.dtype == np.float64 and a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(PD)


def _pi64(a: np.ndarray):
    assert a.dtype == np.int64 and a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(PI64)


class Ckks:
    """Oracle CKKS context: primes = Q (L) then P (K)."""

    def __init__(self, log_n: int, q, p, dnum: int, slots: int):
        global _ckks_ready
        L_ = lib()
        if not _ckks_ready:
            _ckks_sigs(L_)
            _ckks_ready = True
        self.L_ = L_
        self.log_n, self.n = log_n, 1 << log_n
        self.q, self.p = list(q), list(p)
        self.L, self.K = len(q), len(p)
        self.dnum = dnum
        self.alpha = (self.L + dnum - 1) // dnum
        self.slots = slots
        primes = np.array(self.q + self.p, dtype=np.uint64)
        self.h = L_.oc_ctx_new(log_n, self.L, self.K, _p64(primes), dnum, slots)
        if not self.h:
            raise ValueError("oc_ctx_new failed")

    def __del__(self):
        try:
            if self.h:
                self.L_.oc_ctx_free(self.h)
                self.h = None
        except Exception:
            pass

    # helpers
    def zeros(self, *shape):
        return np.zeros(shape + (self.n,), dtype=np.uint64)

    def psi(self, i):
        return int(self.L_.oc_ctx_psi(self.h, i))

    def num_digits(self, nq):
        return int(self.L_.oc_num_digits(self.h, nq))

    def ntt(self, a, nq, np_=0, inverse=False):
        self.L_.oc_poly_ntt(self.h, _p64(a), nq, np_, int(inverse))
        return a

    # keys
    def keygen_secret(self, seed):
        s = np.zeros(self.n, dtype=np.int64)
        sn = self.zeros(self.L + self.K)
        self.L_.oc_keygen_secret(self.h, seed, _pi64(s), _p64(sn))
        return s, sn

    def keygen_public(self, seed, s_ntt):
        pk = self.zeros(2, self.L)
        self.L_.oc_keygen_public(self.h, seed, _p64(s_ntt), _p64(pk))
        return pk

    def keygen_switch(self, seed, key_id, s_ntt, sp_ntt):
        D = self.num_digits(self.L)
        evk = self.zeros(D, 2, self.L + self.K)
        self.L_.oc_keygen_switch(self.h, seed, key_id, _p64(s_ntt), _p64(sp_ntt), _p64(evk))
        return evk

    def sparse_secret(self, seed, h):
        """Sparse ternary secret of Hamming weight h for bootstrapping's key
        encapsulation (FIDESlib's SPARSE_ENCAPSULATED distribution, selected by
        the reference's decode driver at
        native/fideslib_stage0/src/stage1_mamba2_decode_fideslib.cpp:284-291).
        FIDESlib itself is not vendored; the sampler here is this build's own
        definition: a splitmix64 stream keyed by seed ^ golden ^ (h << 32) picks
        h distinct positions by Floyd's algorithm and a sign for each.
        Returns (coefficients, NTT form over all L+K primes)."""
        m64 = (1 << 64) - 1
        st = [(seed ^ 0x9E3779B97F4A7C15 ^ (h << 32)) & m64]

        def nxt():
            st[0] = (st[0] + 0x9E3779B97F4A7C15) & m64
            z = st[0]
            z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & m64
            z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & m64
            return z ^ (z >> 31)

        coef = np.zeros(self.n, dtype=np.int64)
        for j in range(self.n - h, self.n):
            t = nxt() % (j + 1)
            pos = t if coef[t] == 0 else j
            coef[pos] = 1 if nxt() & 1 else -1
        sn = self.zeros(self.L + self.K)
        self.L_.oc_lift_small(self.h, _pi64(coef), _p64(sn), self.L, self.K, 1)
        return coef, sn

    def sparse_keys(self, seed, s_ntt, sp_ntt):
        """Switching keys s -> s' and s' -> s of the encapsulation, under the
        key ids 2N+1 and 2N+3 (past every Galois element)."""
        return (self.keygen_switch(seed, 2 * self.n + 1, sp_ntt, s_ntt),
                self.keygen_switch(seed, 2 * self.n + 3, s_ntt, sp_ntt))

    def relin_key(self, seed, s_ntt):
        # s^2 over all L+K limbs (limb l of a full-width array sits on prime l)
        sq = self._bin("oc_mul_pointwise", s_ntt, s_ntt, self.L + self.K)
        return self.keygen_switch(seed, 0, s_ntt, sq)

    def rot_key(self, seed, s_coef, s_ntt, g):
        """Key for oc_rotate by Galois element g: switches s -> sigma_g^{-1}(s)."""
        ginv = pow(g, -1, 2 * self.n)
        sg = np.zeros(self.n, dtype=np.int64)
        self.L_.oc_automorphism_coef(self.h, _pi64(s_coef), ginv, _pi64(sg))
        sgn = self.zeros(self.L + self.K)
        self.L_.oc_lift_small(self.h, _pi64(sg), _p64(sgn), self.L, self.K, 1)
        return self.keygen_switch(seed, g, sgn, s_ntt)

    def galois(self, r):
        return int(self.L_.oc_rotation_galois(self.h, r))

    # encoding
    def encode(self, values, scale, nq):
        v = np.ascontiguousarray(np.asarray(values, dtype=np.complex128))
        re = np.ascontiguousarray(v.real)
        im = np.ascontiguousarray(v.imag)
        out = self.zeros(nq)
        rc = self.L_.oc_encode(self.h, _pd(re), _pd(im), len(v), scale, nq, _p64(out))
        if rc != 0:
            raise ValueError("encode overflow")
        return out

    def decode(self, pt, nq, scale):
        re = np.zeros(self.slots)
        im = np.zeros(self.slots)
        self.L_.oc_decode(self.h, _p64(np.ascontiguousarray(pt)), nq, scale, _pd(re), _pd(im))
        return re + 1j * im

    def encrypt(self, seed, nonce, pk, pt, nq):
        ct = self.zeros(2, nq)
        self.L_.oc_encrypt_pk(self.h, seed, nonce, _p64(pk), _p64(np.ascontiguousarray(pt)), nq, _p64(ct))
        return ct

    def decrypt(self, s_ntt, ct):
        ncomp, nq = ct.shape[0], ct.shape[1]
        pt = self.zeros(nq)
        self.L_.oc_decrypt(self.h, _p64(s_ntt), _p64(np.ascontiguousarray(ct)), ncomp, nq, _p64(pt))
        return pt

    def _bin(self, name, a, b, nl):
        out = np.empty_like(a)
        getattr(self.L_, name)(self.h, _p64(np.ascontiguousarray(a)), _p64(np.ascontiguousarray(b)), nl, _p64(out))
        return out

    def add(self, a, b):
        return self._cadd("oc_add", a, b)

    def _cadd(self, name, a, b):
        out = np.empty_like(a)
        for i in range(a.shape[0]):
            out[i] = self._bin(name, a[i], b[i], a.shape[1])
        return out

    def sub(self, a, b):
        return self._cadd("oc_sub", a, b)

    def mul_plain(self, ct, pt):
        out = np.empty_like(ct)
        for i in range(ct.shape[0]):
            out[i] = self._bin("oc_mul_pointwise", ct[i], pt, ct.shape[1])
        return out

    def tensor(self, a, b):
        nq = a.shape[1]
        d = self.zeros(3, nq)
        self.L_.oc_tensor(self.h, _p64(a), _p64(b), nq, _p64(d))
        return d

    def modup(self, d, nq):
        D = self.num_digits(nq)
        ext = self.zeros(D, nq + self.K)
        self.L_.oc_modup(self.h, _p64(np.ascontiguousarray(d)), nq, _p64(ext))
        return ext

    def key_inner(self, ext, nq, evk):
        acc = self.zeros(2, nq + self.K)
        self.L_.oc_key_inner(self.h, _p64(ext), nq, _p64(evk), _p64(acc))
        return acc

    def moddown(self, x, nq):
        out = self.zeros(nq)
        self.L_.oc_moddown(self.h, _p64(np.ascontiguousarray(x)), nq, _p64(out))
        return out

    def keyswitch(self, d, evk):
        nq = d.shape[0]
        out = self.zeros(2, nq)
        self.L_.oc_keyswitch(self.h, _p64(np.ascontiguousarray(d)), nq, _p64(evk), _p64(out))
        return out

    def relinearize(self, d3, rlk):
        nq = d3.shape[1]
        out = self.zeros(2, nq)
        self.L_.oc_relinearize(self.h, _p64(d3), nq, _p64(rlk), _p64(out))
        return out

    def rotate(self, ct, g, rk):
        nq = ct.shape[1]
        out = self.zeros(2, nq)
        self.L_.oc_rotate(self.h, _p64(np.ascontiguousarray(ct)), nq, g, _p64(rk), _p64(out))
        return out

    def automorphism(self, a, g):
        nl = a.size // self.n
        out = np.empty_like(a)
        self.L_.oc_automorphism_ntt(self.h, _p64(np.ascontiguousarray(a)), nl, g, _p64(out))
        return out

    def rescale(self, ct):
        ncomp, nq = ct.shape[0], ct.shape[1]
        out = self.zeros(ncomp, nq - 1)
        self.L_.oc_rescale(self.h, _p64(np.ascontiguousarray(ct)), ncomp, nq, _p64(out))
        return out

    # bootstrapping pieces
    def mod_raise(self, ct):
        """ModRaise of OpenFHE's FHECKKSRNS::EvalBootstrap (the raise step): limb 0
        of each component in coefficient form, centred (NativePoly::SwitchModulus),
        lifted to every Q prime, back to NTT form."""
        ncomp = ct.shape[0]
        q0 = np.int64(self.q[0])
        out = self.zeros(ncomp, self.L)
        for c in range(ncomp):
            a = np.ascontiguousarray(ct[c, 0:1]).copy()
            self.ntt(a, 1, 0, inverse=True)
            v = a[0].astype(np.int64)
            v = np.where(v > q0 // 2, v - q0, v)
            for l in range(self.L):
                out[c, l] = (v % np.int64(self.q[l])).astype(np.uint64)
            comp = np.ascontiguousarray(out[c])
            self.ntt(comp, self.L, 0, inverse=False)
            out[c] = comp
        return out

    def mul_i(self, ct):
        """ct * X^{N/2} in NTT form: evaluation point psi^{2 brv(k) + 1} gives the
        factor psi^{N/2} for k < N/2 and -psi^{N/2} above."""
        ncomp, nq = ct.shape[0], ct.shape[1]
        out = np.empty_like(ct)
        h = self.n // 2
        for l in range(nq):
            q = self.q[l]
            iq = pow(self.psi(l), h, q)
            for c in range(ncomp):
                x = [int(v) for v in ct[c, l]]
                out[c, l] = np.array([(v * iq) % q if k < h else (-(v * iq)) % q for k, v in enumerate(x)],
                                     dtype=np.uint64)
        return out
