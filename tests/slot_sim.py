"""A slot-level model of the CryptoContext API for CPU tests of host-side
schedules (test infrastructure only; nothing under fhe_mamba_b200 imports it).

Ciphertexts carry their slot values in fp64 and the level bookkeeping of the
device library: `left` = levels still available (limbs - 1, minus one while a
product awaits its rescale).  Products (ciphertext, plaintext or non-integer
scalar) spend one level, additions and rotations none, a Chebyshev series the
levels of the device's Paterson-Stockmeyer evaluation (plus one for a
non-trivial interval), a linear transform one.  Every check the device would
make, or whose failure would make the device's result meaningless, raises
SimError: a level underflow, a rotation without a generated key, a plaintext
with fewer limbs than its ciphertext operand, a refresh input outside
[-bound, bound] or with fewer than two levels.  Refreshes return the levels of
the library's refresh at the context's depth and add uniform noise of
`refresh_noise` x bound (the bootstrap error), so the decrypted error of a
schedule is an estimate of the device's."""
from __future__ import annotations

import math

import numpy as np


class SimError(RuntimeError):
    pass


def ps_depth(n: int) -> int:
    """Levels Ckks::chebyshev (fhe_mamba_b200/csrc/ckks.cu) spends on an
    n-coefficient series whose input is already in [-1, 1]."""
    levels = 0
    while (1 << levels) < n:
        levels += 1
    baby = 1 << ((max(1, levels) + 1) // 2)
    memo = {1: 0}

    def d(i):
        if i not in memo:
            memo[i] = (d(i // 2) if i % 2 == 0 else max(d((i + 1) // 2), d(i // 2))) + 1
        return memo[i]

    def ev(deg):
        if deg < baby:
            return max(d(j) for j in range(1, min(baby - 1, n - 1) + 1)) + 1
        k = baby
        while 2 * k - 1 < deg:
            k *= 2
        return max(ev(k - 1), max(d(k), ev(deg - k)) + 1)

    return ev(n - 1)


class SimPlaintext:
    def __init__(self, values, limbs):
        self.values, self.limbs = values, limbs


class SimCiphertext:
    def __init__(self, values, left, deg=1):
        if left < 0:
            raise SimError("level underflow")
        self.values, self.left, self.deg = values, left, deg

    def n_limbs(self):
        return self.left + 1 + (1 if self.deg >= 2 else 0)

    def Clone(self):
        return SimCiphertext(self.values.copy(), self.left, self.deg)

    def GetNoiseScaleDeg(self):
        return self.deg

    def GetScalingFactor(self):
        return 2.0 ** 59


class _Decrypted:
    def __init__(self, values):
        self.values = values

    def GetRealPackedValue(self, count=None):
        v = self.values.real
        return v if count is None else v[:count]


def _clenshaw(coeffs, t):
    b1 = np.zeros_like(t)
    b2 = np.zeros_like(t)
    for c in coeffs[:0:-1]:
        b1, b2 = 2.0 * t * b1 - b2 + c, b1
    return t * b1 - b2 + coeffs[0]


class SlotContext:
    """depth: multiplicative depth (limbs = depth + 1); refresh_left: levels
    after a two-pass refresh (one more after a single pass)."""

    def __init__(self, slots: int, depth: int = 44, refresh_left: int = 21, refresh_noise: float = 1e-4,
                 seed: int = 0):
        self.slots, self.n, self.n_q = slots, 2 * slots, depth + 1
        self.n_p, self.dnum = 12, 4  # key-size bookkeeping only
        self.refresh_left, self.refresh_noise = refresh_left, refresh_noise
        self.keys = set()
        self.rng = np.random.default_rng(seed)
        self.refresh_count = 0
        self.max_refresh_ratio = 0.0
        self.has_secret = True
        self.subslot_sizes = ()
        self.subslot_extra = {}
        self.subslot_refreshes = 0

    # -- keys and files (a pickled stand-in for the library's key bundles and
    # ciphertext files: a bundle without the secret makes an evaluation-only
    # context that refuses to decrypt or to generate keys)
    def KeyGen(self, seed=0):
        self.has_secret = True

    def EvalRotateKeyGen(self, steps):
        steps = {int(s) % self.slots for s in steps} - {0}
        if steps - self.keys and not self.has_secret:
            raise SimError("this context holds no secret key")
        self.keys |= steps

    def EvalBootstrapSetup(self, *_, **__):
        pass

    def EvalBootstrapSubslotSetup(self, slots, level_budget=(4, 4), *_, **__):
        """The levels a sub-slot refresh returns follow its level budget: each
        transform level below the full refresh's {4, 4} is one more left."""
        if slots & (slots - 1) or not 2 <= slots <= self.slots // 2:
            raise SimError("sub-slot refresh slots must be a power of two <= half the slots")
        self.subslot_sizes = tuple(sorted(set(self.subslot_sizes) | {int(slots)}))
        self.subslot_extra[int(slots)] = 8 - int(level_budget[0]) - int(level_budget[1])

    def EvalBootstrapKeyGen(self, *_):
        pass

    def SerializeKeys(self, path, include_secret=False):
        import pickle
        with open(path, "wb") as f:
            pickle.dump({"keys": sorted(self.keys), "secret": bool(include_secret and self.has_secret)}, f)

    def DeserializeKeys(self, path):
        import pickle
        with open(path, "rb") as f:
            d = pickle.load(f)
        self.keys, self.has_secret = set(d["keys"]), d["secret"]

    def SerializeCiphertext(self, ct, path):
        np.savez(path, values=ct.values, meta=np.array([ct.left, ct.deg]))

    def DeserializeCiphertext(self, path):
        with np.load(path if str(path).endswith(".npz") else str(path) + ".npz") as d:
            return SimCiphertext(d["values"], int(d["meta"][0]), int(d["meta"][1]))

    def _rot(self, values, k):
        k = int(k) % self.slots
        if k and k not in self.keys:
            raise SimError(f"missing rotation key for step {k}")
        return np.roll(values, -k)

    # -- encoding
    def MakeCKKSPackedPlaintext(self, values, level=0, scale=0.0, **_):
        v = np.zeros(self.slots, dtype=np.complex128)
        a = np.asarray(values, dtype=np.complex128)
        v[:a.size] = a
        return SimPlaintext(v, self.n_q - level)

    def MakeCKKSPackedPlaintexts(self, vectors, level=0, scale=0.0):
        return [self.MakeCKKSPackedPlaintext(v, level=level) for v in np.asarray(vectors)]

    def Encrypt(self, pt, _unused=None):
        return SimCiphertext(pt.values.copy(), self.n_q - 1)

    def Decrypt(self, ct, _unused=None):
        if not self.has_secret:
            raise SimError("this context holds no secret key")
        return _Decrypted(ct.values)

    # -- arithmetic
    @staticmethod
    def _eff(ct):
        return ct.left

    def _check_pt(self, ct, pt):
        if pt.limbs < ct.left + 1:
            raise SimError(f"plaintext has {pt.limbs} limbs, its operand {ct.left + 1}")

    def EvalAdd(self, a, b):
        if isinstance(b, SimCiphertext):
            return SimCiphertext(a.values + b.values, min(a.left, b.left), max(a.deg, b.deg))
        if isinstance(b, SimPlaintext):
            self._check_pt(a, b)
            return SimCiphertext(a.values + b.values, a.left, a.deg)
        return SimCiphertext(a.values + float(b), a.left, a.deg)

    def EvalSub(self, a, b):
        if isinstance(b, (SimCiphertext, SimPlaintext)):
            neg = SimPlaintext(-b.values, b.limbs) if isinstance(b, SimPlaintext) else \
                SimCiphertext(-b.values, b.left, b.deg)
            return self.EvalAdd(a, neg)
        return self.EvalAdd(a, -float(b))

    def EvalNegate(self, a):
        return SimCiphertext(-a.values, a.left, a.deg)

    def EvalMult(self, a, b):
        if isinstance(b, SimCiphertext):
            return SimCiphertext(a.values * b.values, min(a.left, b.left) - 1, 2)
        if isinstance(b, SimPlaintext):
            self._check_pt(a, b)
            return SimCiphertext(a.values * b.values, a.left - 1, 2)
        return SimCiphertext(a.values * float(b), a.left - 1, 2)

    def RescaleInPlace(self, a):
        a.deg = 1

    def EvalRotate(self, a, step):
        return SimCiphertext(self._rot(a.values, step), a.left, a.deg)

    def EvalFastRotation(self, a, steps, *_):
        return [self.EvalRotate(a, s) for s in steps]

    def EvalLinearTransform(self, ct, diagonals, baby, giant, stride=1, giant_offset=0):
        out = np.zeros(self.slots, dtype=np.complex128)
        for g in range(giant):
            inner = np.zeros(self.slots, dtype=np.complex128)
            for j in range(baby):
                d = diagonals[g * baby + j]
                if d is None:
                    continue
                self._check_pt(ct, d)
                inner += d.values * self._rot(ct.values, j * stride)
            out += self._rot(inner, (g * baby - giant_offset) * stride)
        return SimCiphertext(out, ct.left - 1, 2)

    def EvalChebyshevSeries(self, ct, coefficients, a, b):
        c = np.asarray(coefficients, dtype=np.float64)
        t = (2.0 * ct.values.real - a - b) / (b - a)
        affine = 0 if (a == -1.0 and b == 1.0) else 1
        return SimCiphertext(_clenshaw(c, t).astype(np.complex128), ct.left - affine - ps_depth(len(c)), 1)

    def EvalChebyshevFunction(self, func, ct, a, b, degree):
        k = np.arange(degree + 1)
        t = np.cos(np.pi * (k + 0.5) / (degree + 1))
        coeffs = np.polynomial.chebyshev.chebfit(t, func(0.5 * (t + 1) * (b - a) + a), degree)
        return self.EvalChebyshevSeries(ct, coeffs, a, b)

    def refresh(self, ct, bound: float = 1.0, passes: int = 2, merge: bool = False, support: int = 0):
        """support > 0 with a sub-slot setup of n >= support slots: the device
        replicates the input with period n and bootstraps it, so slot i < n
        comes back as the sum of the input's slots i + j n and every slot from
        n on as 0; the input must be zero (up to noise) outside [0, support)."""
        ratio = float(np.max(np.abs(ct.values))) / bound
        self.max_refresh_ratio = max(self.max_refresh_ratio, ratio)
        if ratio > 1.0:
            raise SimError(f"refresh input {ratio:.3f} x its bound")
        if ct.left < 2:
            raise SimError("too few levels left to refresh")
        self.refresh_count += 1
        left = self.refresh_left + (1 if passes == 1 else 0)
        sizes = [n for n in self.subslot_sizes if n >= support] if support else []
        if not sizes:
            noise = self.rng.uniform(-1, 1, self.slots) * self.refresh_noise * bound
            return SimCiphertext(ct.values + noise, left, 1)
        n = sizes[0]
        outside = float(np.max(np.abs(ct.values[support:]))) / bound if support < self.slots else 0.0
        if outside > 1e-3:
            raise SimError(f"sub-slot refresh input is {outside:.3g} x its bound outside [0, {support})")
        self.subslot_refreshes += 1
        out = np.zeros(self.slots, dtype=ct.values.dtype)
        out[:n] = ct.values.reshape(-1, n).sum(axis=0)
        out[:n] += self.rng.uniform(-1, 1, n) * self.refresh_noise * bound
        return SimCiphertext(out, left + self.subslot_extra[n], 1)

    EvalRefresh = refresh
