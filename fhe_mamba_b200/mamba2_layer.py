"""One Mamba-2 decode layer on CKKS ciphertexts (BASELINE config 4 shape) and
its plaintext polynomial reference.

The layer follows the reference's Mamba-2 decode (``mixer2_forward``,
src/fhemamba/reference.py:182-294, and the native
stage1_mamba2_decode_fideslib.cpp run_layer :3634-4286): block RMSNorm ->
in_proj (BSGS matvec) -> causal conv over a FIFO of the last conv_kernel
xBC streams -> SiLU -> dt = softplus(dt + dt_bias), decay = exp(A dt) ->
state update S <- decay S + (dt x) (x) B and readout y = S C + D x ->
y * SiLU(z) -> gated RMSNorm -> out_proj -> residual.  Nonlinearities are
Chebyshev polynomials on calibrated domains, inverse square roots a
Chebyshev seed plus Newton steps; values are refreshed (two-pass
bootstrapping) when a stage would run out of levels.

Weights are synthetic (config 4: ~N(0, 0.02^2), seeded); the plaintext path
``plain_step`` evaluates the same polynomials in fp64, so the decrypted layer
output is compared with it directly.
"""
from __future__ import annotations

import os
from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass, field

import numpy as np

from .mamba import PackedMamba2, PlaintextMemo, StateLayout


def _silu(x):
    return x / (1.0 + np.exp(-x))


def _softplus(x):
    return np.log1p(np.exp(-np.abs(x))) + np.maximum(x, 0)


def cheb_fit(fn, lo, hi, degree):
    """Chebyshev interpolant of fn on [lo, hi]: coefficients c with p = c0 + sum c_i T_i."""
    k = np.arange(degree + 1)
    t = np.cos(np.pi * (k + 0.5) / (degree + 1))
    return np.polynomial.chebyshev.chebfit(t, fn(0.5 * (t + 1) * (hi - lo) + lo), degree)


@dataclass
class Poly:
    coeffs: np.ndarray
    lo: float
    hi: float

    def position(self, x):
        """Where x falls on the interval: -1 at lo, 1 at hi."""
        return (2 * np.asarray(x, dtype=np.float64) - self.lo - self.hi) / (self.hi - self.lo)

    def __call__(self, x):
        return np.polynomial.chebyshev.chebval(self.position(x), self.coeffs)


@dataclass
class Mamba2Weights:
    d_model: int
    d_state: int
    heads: int
    conv_kernel: int = 4
    eps: float = 1e-5
    std: float = 0.02
    seed: int = 4
    arrays: dict = field(default_factory=dict)

    @property
    def d_inner(self):
        return 2 * self.d_model

    @property
    def head_dim(self):
        return self.d_inner // self.heads

    @property
    def conv_dim(self):
        return self.d_inner + 2 * self.d_state

    @property
    def proj_dim(self):
        return 2 * self.d_inner + 2 * self.d_state + self.heads

    def __post_init__(self):
        r = np.random.default_rng(self.seed)
        E, D, S, H = self.d_inner, self.d_model, self.d_state, self.heads
        dt = r.uniform(0.001, 0.1, H)
        self.arrays = {
            "norm_w": 1.0 + r.normal(0, 0.02, D),
            "w_in": r.normal(0, self.std, (self.proj_dim, D)),
            "conv_w": r.normal(0, 0.2, (self.conv_dim, self.conv_kernel)),
            "conv_b": r.normal(0, 0.02, self.conv_dim),
            "dt_bias": np.log(np.expm1(dt)),
            "a": -np.exp(np.log(r.uniform(1, 16, H))),
            "d": np.ones(H),
            "gn_w": 1.0 + r.normal(0, 0.02, E),
            "w_out": r.normal(0, self.std, (D, E)),
        }

    def __getitem__(self, k):
        return self.arrays[k]


def _single_threaded_blas():
    """One BLAS thread per calling thread while the calibration runs its own
    thread pool (nested pools oversubscribe the cores)."""
    try:
        from threadpoolctl import threadpool_limits
        return threadpool_limits(1)
    except ImportError:  # pragma: no cover - threadpoolctl ships with the image
        import contextlib
        return contextlib.nullcontext()


def _rms(x, w, eps):
    return x / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + eps) * w


def _split_proj(W: Mamba2Weights, proj):
    E = W.d_inner
    return proj[..., :E], proj[..., E:E + W.conv_dim], proj[..., E + W.conv_dim:]


def _split_xa(W: Mamba2Weights, xa):
    E, S = W.d_inner, W.d_state
    return xa[..., :E].reshape(xa.shape[:-1] + (W.heads, W.head_dim)), xa[..., E:E + S], xa[..., E + S:]


def _ssm(st, decay, dts, x, B, C, d):
    """S <- decay S + (dt x) (x) B (S = update when there is no state yet) and
    y = S C + D x, over any leading batch axes."""
    upd = np.einsum("...hp,...n->...hpn", dts[..., :, None] * x, B)
    if st is not None:
        upd += decay[..., :, None, None] * st
    return upd, np.einsum("...hpn,...n->...hp", upd, C) + d[:, None] * x


def exact_step(W: Mamba2Weights, h, conv, st, upd=lambda k, v: None):
    """The layer with the exact nonlinearities (calibration); upd(site, values)
    observes the inputs of every polynomial and inverse square root.  h may
    carry leading batch axes (one row per calibration sequence)."""
    K = W.conv_kernel
    upd("v1", np.mean(h * h, axis=-1) + W.eps)
    u = _rms(h, W["norm_w"], W.eps)
    z, xbc, dt = _split_proj(W, u @ W["w_in"].T)
    window = list(conv) + [xbc]
    xc = sum(W["conv_w"][:, k] * window[k] for k in range(K)) + W["conv_b"]
    upd("xc", xc)
    xa = _silu(xc)
    upd("dt", dt + W["dt_bias"])
    dts = _softplus(dt + W["dt_bias"])
    upd("adt", W["a"] * dts)
    upd("z", z)
    x, B, C = _split_xa(W, xa)
    st, y = _ssm(st, np.exp(W["a"] * dts), dts, x, B, C, W["d"])
    g = y.reshape(y.shape[:-2] + (W.d_inner,)) * _silu(z)
    upd("v2", np.mean(g * g, axis=-1) + W.eps)
    out = _rms(g, W["gn_w"], W.eps) @ W["w_out"].T
    return h + out, window[1:], st


def new_ranges():
    return {k: [np.inf, -np.inf] for k in ("xc", "dt", "adt", "z", "v1", "v2")}


def range_updater(ranges):
    def upd(k, v):
        ranges[k][0] = min(ranges[k][0], float(np.min(v)))
        ranges[k][1] = max(ranges[k][1], float(np.max(v)))
    return upd


@dataclass
class HeadPoly:
    """One Chebyshev series per head on a shared domain [lo, hi]: coeffs[i, h]
    is head h's coefficient of T_i.  On ciphertexts the heads sit at slots
    [0, heads): one basis T_1..T_D of the slot-masked affine map is weighted by
    plaintext coefficient vectors (zero outside the heads, so the result is
    too), the way the reference's joint gates evaluate per-head polynomials."""

    coeffs: np.ndarray
    lo: float
    hi: float

    @classmethod
    def fit(cls, fn, params, lo, hi, degree):
        """Head h interpolates t -> fn(params[h], t) at Chebyshev nodes."""
        return cls(np.stack([cheb_fit(lambda t, q=q: fn(q, t), lo, hi, degree) for q in params], axis=1), lo, hi)

    def position(self, x):
        return (2.0 * np.asarray(x, dtype=np.float64) - self.lo - self.hi) / (self.hi - self.lo)

    def __call__(self, x):
        t = self.position(x)
        b1 = np.zeros_like(t)
        b2 = np.zeros_like(t)
        for c in self.coeffs[:0:-1]:
            b1, b2 = 2.0 * t * b1 - b2 + c, b1
        return t * b1 - b2 + self.coeffs[0]

    @property
    def degree(self) -> int:
        return self.coeffs.shape[0] - 1

    @property
    def levels(self) -> int:
        # the affine map, the basis up to T_D, the coefficient products
        return 2 + max(0, int(np.ceil(np.log2(max(1, self.degree)))))

    def encrypted(self, pm, z, heads):
        c, n = pm.cc, pm.L.slots
        a = np.zeros(n)
        b = np.zeros(n)
        a[:heads] = 2.0 / (self.hi - self.lo)
        b[:heads] = -(self.lo + self.hi) / (self.hi - self.lo)
        t = pm._mul_mask(z, a)
        if t.GetNoiseScaleDeg() >= 2:
            c.RescaleInPlace(t)
        t = c.EvalAdd(t, pm.plain(b, level=c.n_q - t.n_limbs(), scale=t.GetScalingFactor()))
        basis = {1: t}

        def T(i):  # T_2k = 2 T_k^2 - 1, T_2k+1 = 2 T_k+1 T_k - T_1
            if i not in basis:
                if i % 2 == 0:
                    sq = c.EvalMult(T(i // 2), T(i // 2))
                    basis[i] = c.EvalAdd(c.EvalAdd(sq, sq), -1.0)
                else:
                    pr = c.EvalMult(T(i // 2 + 1), T(i // 2))
                    basis[i] = c.EvalSub(c.EvalAdd(pr, pr), T(1))
            return basis[i]

        acc = None
        for i in range(1, self.coeffs.shape[0]):
            vec = np.zeros(n)
            vec[:heads] = self.coeffs[i]
            term = pm._mul_mask(T(i), vec)
            acc = term if acc is None else c.EvalAdd(acc, term)
        if acc.GetNoiseScaleDeg() >= 2:
            c.RescaleInPlace(acc)
        const = np.zeros(n)
        const[:heads] = self.coeffs[0]
        return c.EvalAdd(acc, pm.plain(const, level=c.n_q - acc.n_limbs(), scale=acc.GetScalingFactor()))


class Mamba2Polys:
    """Polynomial domains calibrated on exact-function trajectories (random
    residual inputs over a few tokens, recurrent state U[-1, 1]), widened by half
    their span.  `ranges` (site -> [lo, hi]) replaces the layer-local
    calibration when the layer sits inside a model."""

    def __init__(self, W: Mamba2Weights, degree: int = 31, seed_degree: int = 15, samples: int = 16,
                 tokens: int = 3, seed: int = 9, ranges=None, fused_decay: bool = False):
        if ranges is None:
            r = np.random.default_rng(seed)
            ranges = new_ranges()
            upd = range_updater(ranges)
            for _ in range(samples):
                conv = [np.zeros(W.conv_dim) for _ in range(W.conv_kernel - 1)]
                st = r.uniform(-1, 1, (W.heads, W.head_dim, W.d_state))
                for _ in range(tokens):
                    _, conv, st = exact_step(W, r.normal(0, 1, W.d_model), conv, st, upd)

        def widen(k, frac=0.5, floor=1.0):
            lo, hi = ranges[k]
            m = max(frac * (hi - lo), floor)
            return lo - m, hi + m

        self.silu_x = self._fit(_silu, *widen("xc"), degree)
        self.softplus = self._fit(_softplus, *widen("dt"), degree)
        lo, hi = widen("adt")
        self.exp = self._fit(np.exp, lo, min(hi, 0.0), degree)
        self.silu_z = self._fit(_silu, *widen("z"), degree)
        self.v1 = (0.25 * ranges["v1"][0], 4.0 * ranges["v1"][1])
        self.v2 = (0.25 * ranges["v2"][0], 4.0 * ranges["v2"][1])
        self.rsqrt1 = self._fit(lambda t: 1 / np.sqrt(t), *self.v1, seed_degree)
        self.rsqrt2 = self._fit(lambda t: 1 / np.sqrt(t), *self.v2, seed_degree)
        self.seed_degree = seed_degree
        # fused_decay: decay = exp(a_h softplus(x)) as one per-head series of the
        # raw dt input x on the softplus domain, instead of exp of a * softplus
        # (which needs a * dt on the exp domain, and a refresh before it)
        self.decay = HeadPoly.fit(lambda a, t: np.exp(a * _softplus(t)), W["a"], self.softplus.lo,
                                  self.softplus.hi, degree) if fused_decay else None

    @staticmethod
    def _fit(fn, lo, hi, degree):
        return Poly(cheb_fit(fn, lo, hi, degree), lo, hi)


def plain_rms(x, w, eps, seed, newton=2, rec=None, key=None, dom=None):
    """x * rsqrt(mean(x^2) + eps) * w.  `seed` is a Chebyshev seed refined by
    `newton` Newton steps, or an inverse square root with its own refinement
    (an object with ``inv_sqrt``, as a chain payload exports them); rec(key_*)
    then observes the variance and every iterate, at the variance and at the
    value that fills the slots outside the vector.  dom(key, t) observes where
    the variance falls on a Chebyshev seed's interval (t in [-1, 1] inside)."""
    v = np.mean(x * x, axis=-1) + eps
    if hasattr(seed, "inv_sqrt"):
        if rec is not None:
            probe = np.array([v, seed.fill])
            rec(key + "_v", probe)
            seed.inv_sqrt(probe, trace=lambda name, val: rec(key + "_" + name, val))
        return x * np.expand_dims(seed.inv_sqrt(v), -1) * w
    if dom is not None:
        dom(key, seed.position(v))
    y = seed(v)
    for _ in range(newton):
        y = 1.5 * y - 0.5 * v * y ** 3
    return x * np.expand_dims(y, -1) * w


def plain_step(W: Mamba2Weights, P: Mamba2Polys, h, conv_state, ssm_state):
    """The layer on plaintext with the same polynomials.  conv_state: list of the
    last conv_kernel-1 xBC vectors (oldest first); ssm_state: [H, P, S] or None."""
    return poly_step_record(W, P, h, conv_state, ssm_state, lambda k, v: None)


def rect_diagonals(Wm: np.ndarray, baby: int, giant: int, slots: int):
    """BSGS diagonals of y = W x (W: m x n) for an input replicated with period n
    over at least m + n slots: diagonal d = g*baby + j holds W[i, (i + d) mod n]
    at slot i + g*baby (pre-rotated by the giant step)."""
    m, n = Wm.shape
    if baby * giant < n or (giant - 1) * baby + m > slots:
        raise ValueError("BSGS layout does not fit")
    rows = np.arange(m)
    out = []
    for g in range(giant):
        for j in range(baby):
            d = g * baby + j
            if d >= n:
                out.append(None)
                continue
            v = np.zeros(slots)
            v[g * baby + rows] = Wm[rows, (rows + d) % n]
            out.append(v)
    return out


def rotation_sum_schedule(count: int):
    """(offset, accumulated) steps whose sums give sum_{r < count} rot(x, r * stride)
    with about log2(count) rotations (doubling, plus one step per set bit)."""
    steps, bit, filled = [], 1, 1
    while bit <= count // 2:
        bit *= 2
    bit //= 2
    while bit > 0:
        steps.append((filled, True))
        filled *= 2
        if count & bit:
            steps.append((filled, False))
            filled += 1
        bit //= 2
    return steps


class ReplicatedLayout:
    """Replicated BSGS layout of y = W x (W: m x n) in `slots` slots.

    R windows of w = n/R + ceil(m/n) n slots each; window r accumulates the
    diagonals d = r n/R + t (t < n/R) of rows i < m at slots r w + i.  The input
    is replicated with period n over the whole span, which makes slot
    r w + i + t hold x[(i + r n/R + t) mod n] (r w = r n/R mod n), so all windows
    share one set of n/R diagonal plaintexts and one BSGS over t.  A rotate-and-
    add over the windows then sums the R partial results into slots [0, m)."""

    def __init__(self, m: int, n: int, slots: int):
        k = -(-m // n)
        R = 1
        while n % (2 * R) == 0:
            R2 = 2 * R
            w2 = n // R2 + k * n
            if (R2 - 1) * w2 + m + n // R2 > slots:
                break
            R = R2
        self.m, self.n, self.R = m, n, R
        self.T = n // R
        self.w = self.T + k * n
        self.span = (R - 1) * self.w + m + self.T
        if self.span > slots:
            raise ValueError("matrix does not fit the slots")
        self.copies = -(-self.span // n)
        b = 1
        while b * b < self.T:
            b *= 2
        self.b = b
        self.G = -(-self.T // b)

    def diagonals(self, Wm: np.ndarray, slots: int):
        m, n, R, T, w, b = self.m, self.n, self.R, self.T, self.w, self.b
        rows = np.arange(m)
        out = []
        for g in range(self.G):
            for j in range(b):
                t = g * b + j
                if t >= T:
                    out.append(None)
                    continue
                v = np.zeros(slots)
                for r in range(R):
                    v[r * w + rows] = Wm[rows, (rows + r * T + t) % n]
                out.append(np.roll(v, g * b))  # pre-rotated by the giant step
        return out

    def rotation_steps(self):
        s = {j for j in range(1, self.b)} | {g * self.b for g in range(1, self.G)}
        s |= {-o * self.n for o, _ in rotation_sum_schedule(self.copies)}
        s |= {o * self.w for o, _ in rotation_sum_schedule(self.R)}
        return s


class PlaintextCache:
    """Encoded diagonal plaintexts kept across tokens up to a byte budget (LRU)."""

    def __init__(self, budget_bytes: float):
        self.budget = budget_bytes
        self.items = {}
        self.bytes = 0
        self.hits = self.misses = 0

    def get(self, key, nbytes, build):
        if key in self.items:
            self.hits += 1
            v = self.items.pop(key)
            self.items[key] = v
            return v[0]
        self.misses += 1
        value = build()
        while self.items and self.bytes + nbytes > self.budget:
            k0 = next(iter(self.items))
            self.bytes -= self.items.pop(k0)[1]
        if nbytes <= self.budget:
            self.items[key] = (value, nbytes)
            self.bytes += nbytes
        return value


class EncryptedMamba2Layer:
    """The layer on ciphertexts of one CryptoContext (full packing)."""

    # Levels each refresh point must leave for what follows it (plus the
    # margin): the layer input before a Chebyshev-seeded norm (rms), the normed
    # input before in_proj (u), the projection feeding the conv, dt and gate
    # branches (proj), the conv FIFO entries (xbc), the packed SSM inputs
    # (pack), the carried states (state), the readout before the gate (y) and
    # the normed gated value before out_proj (gn).
    NEEDS = {"rms": 14, "u": 2, "proj": 19, "xbc": 2, "pack": 8, "state": 4, "y": 2, "gn": 2}

    def __init__(self, cc, W: Mamba2Weights, P: Mamba2Polys, passes: int = 2, margin: int = 4,
                 cache: PlaintextCache | None = None, needs: dict | None = None, device_diagonals: bool = True,
                 memo=None):
        self.cc, self.W, self.P = cc, W, P
        # Diagonal plaintexts generated on the device from the weights (the
        # context's MakeReplicatedDiagonals) instead of built on the host and
        # uploaded; identical words.  Contexts without it use the host path.
        self.device_diagonals = device_diagonals and hasattr(cc, "MakeReplicatedDiagonals")
        self._wdev = {}
        self.passes, self.margin = passes, margin
        self.needs = dict(self.NEEDS, **(needs or {}))
        self.cache = cache if cache is not None else PlaintextCache(0)
        self.rep = {"w_in": ReplicatedLayout(W.proj_dim, W.d_model, cc.slots),
                    "w_out": ReplicatedLayout(W.d_model, W.d_inner, cc.slots)}
        E, S, H = W.d_inner, W.d_state, W.heads
        self.layout = StateLayout(H, W.head_dim, S, cc.slots)
        # SSM inputs share one ciphertext: xa at [0, conv_dim), dt and decay per head
        # at their own offsets, so a single refresh serves the whole update.
        self.dt_base = -(-W.conv_dim // 64) * 64
        self.decay_base = self.dt_base + -(-H // 64) * 64
        if self.decay_base + H > cc.slots:
            raise ValueError("packed SSM inputs do not fit the slots")
        self.pm = PackedMamba2(cc, self.layout, b_base=E, c_base=E + S, head_base=self.dt_base,
                               decay_base=self.decay_base)
        self.pm.memo = memo  # constant plaintexts (masks, taps, biases) shared across layers and tokens
        self.refreshes = self.two_pass_refreshes = 0
        self.site_refreshes = {}  # refreshes by site name
        self._lin = {}
        n = cc.slots
    # ---- setup --------------------------------------------------------------
    def rotation_steps(self):
        W, n = self.W, self.cc.slots
        s = set(self.pm.rotation_steps())
        for lay in self.rep.values():
            s |= lay.rotation_steps()
        for width in (W.d_model, W.d_inner):
            win = 1 << (width - 1).bit_length()
            s |= {1 << i for i in range(win.bit_length() - 1)} | {-win}
        s |= {W.d_inner, W.d_inner + W.conv_dim, -self.dt_base, -self.decay_base}
        return sorted(v % n for v in s if v % n)

    def transform_steps(self):
        """The baby and giant steps of this layer's fused linear transforms
        (the replicated matvecs and the state-block placement): the library
        switches keys per step there, so they need keys of their own."""
        n = self.cc.slots
        s = set()
        for lay in self.rep.values():
            s |= set(range(1, lay.b)) | {g * lay.b for g in range(1, lay.G)}
        stride = -(self.layout.group_block - 1)
        b, G = self.pm._state_baby, self.pm._state_giant
        s |= {j * stride for j in range(1, b)} | {g * b * stride for g in range(1, G)}
        return sorted(v % n for v in s if v % n)

    def _weights_on_device(self, name):
        """The layer's weight matrix as a row-major fp64 tensor on the context's
        device (uploaded once per layer and matrix)."""
        if name not in self._wdev:
            import torch
            if not np.all(np.isfinite(self.W[name])):  # the device encoder checks only at the next decode
                raise ValueError(f"weight matrix {name} holds non-finite values")
            self._wdev[name] = torch.from_numpy(np.ascontiguousarray(self.W[name], dtype=np.float64)).to(
                torch.device("cuda", self.cc.device))
            torch.cuda.synchronize(self.cc.device)
        return self._wdev[name]

    def _diags(self, name):
        if name not in self._lin:
            self._lin[name] = self.rep[name].diagonals(self.W[name], self.cc.slots)
        return self._lin[name]

    # ---- helpers --------------------------------------------------------------
    def _left(self, ct):
        return ct.n_limbs() - 1 - (1 if ct.GetNoiseScaleDeg() >= 2 else 0)

    def _fit(self, ct, need, bound, site=None, support=0):
        """Refreshes ct when fewer than need + margin levels remain; the margin keeps
        every stage's output refreshable (a two-pass refresh spends two levels
        before its second bootstrap, which needs two limbs).  `passes` is the
        refresh's pass count, or a function of the refresh site's name (a
        refresh policy such as the reference's selective Meta-BTS).  support > 0
        says ct is zero outside slots [0, support): a context with sub-slot
        refreshes (``subslot_sizes``) then refreshes it over fewer slots."""
        if self._left(ct) >= need + self.margin:
            return ct
        passes = self.passes(site) if callable(self.passes) else self.passes
        self.refreshes += 1
        self.two_pass_refreshes += passes == 2
        self.site_refreshes[site] = self.site_refreshes.get(site, 0) + 1
        if support and getattr(self.cc, "subslot_sizes", ()):
            return self.cc.refresh(ct, bound, passes=passes, support=support)
        return self.cc.refresh(ct, bound, passes=passes)

    def _rotation_sum(self, x, count, stride):
        c = self.cc
        acc = x
        for off, accumulated in rotation_sum_schedule(count):
            acc = c.EvalAdd(acc, c.EvalRotate(acc if accumulated else x, off * stride))
        return acc

    def _linear(self, x, name):
        """Replicated BSGS matvec: replicate, one BSGS over n/R diagonals shared by
        R windows, rotate-and-add the windows, mask to the m outputs."""
        c = self.cc
        lay = self.rep[name]
        x = self._rotation_sum(x, lay.copies, -lay.n)
        nq = x.n_limbs() - (1 if x.GetNoiseScaleDeg() >= 2 else 0)

        def build():
            if self.device_diagonals:
                w = self._weights_on_device(name)
                pts = c.MakeReplicatedDiagonals(w.data_ptr(), lay.m, lay.n, lay.R, lay.T, lay.w, lay.b,
                                                level=c.n_q - nq)
                return [pts[t] if t < lay.T else None for t in range(lay.G * lay.b)]
            diags = self._diags(name)
            dense = [d for d in diags if d is not None]
            pts = iter(c.MakeCKKSPackedPlaintexts(np.array(dense), level=c.n_q - nq))
            return [next(pts) if d is not None else None for d in diags]

        nbytes = lay.T * nq * c.n * 8
        plist = self.cache.get((id(self), name, nq), nbytes, build)
        y = c.EvalLinearTransform(x, plist, lay.b, lay.G)
        y = self._rotation_sum(y, lay.R, lay.w)
        return self.pm._mul_mask(y, self.pm._block_mask(0, lay.m))

    def _poly(self, x, p, lo_slot, hi_slot):
        """A Chebyshev Poly on the slots [lo_slot, hi_slot), or a payload
        nonlinearity (an object with ``encrypted``) evaluated its own way."""
        if hasattr(p, "encrypted"):
            return p.encrypted(self.pm, x, lo_slot, hi_slot)
        return self.pm.poly(x, p.coeffs, p.lo, p.hi, lo_slot, hi_slot)

    @staticmethod
    def _need(p):
        """Levels a nonlinearity consumes from its input (8: a degree-31 Poly)."""
        return getattr(p, "levels", 8)

    def _rms(self, x, width, weight, seed, bounds, key, prefix, eps):
        """RMSNorm of x at [0, width).  A Chebyshev Poly seed runs the fixed
        seed + 2 Newton steps of ``rms_norm``; a payload inverse square root
        (``encrypted_inv_sqrt``) runs its own iteration on the variance, which
        refreshes its iterates through bounds[prefix_*] as their levels run out."""
        if hasattr(seed, "encrypted_inv_sqrt"):
            x = self._fit(x, 2 + seed.levels, bounds[key], key, width)
            v = self.pm.mean_square(x, width, eps, seed.fill)
            y = seed.encrypted_inv_sqrt(
                self.cc, v, lambda ct, need, name: self._fit(ct, need, bounds[prefix + "_" + name], prefix + "_" + name))
            x = self._fit(x, 2, bounds[key], key, width)
            y = self._fit(y, 2, bounds[prefix + "_y"], prefix + "_y")
            return self.pm.scale_rows(x, y, width, weight)
        x = self._fit(x, self.needs["rms"], bounds[key], key, width)
        return self.pm.rms_norm(x, width, weight, eps, (seed.lo, seed.hi), degree=len(seed.coeffs) - 1)

    # ---- one token ------------------------------------------------------------
    def step(self, h, conv_state, ssm_state, bounds):
        """h: ciphertext of the residual stream at [0, d_model); conv_state: list
        of conv_kernel-1 xBC ciphertexts (None for zeros); ssm_state: list of
        group ciphertexts or None.  Returns (h_out, conv_state, ssm_state).

        Refresh points: the layer input (before the block norm), the in_proj
        output (once for the conv, dt and gate branches), the packed SSM inputs
        (xa, dt, decay in one ciphertext) and the gated value before its norm;
        states are refreshed only when their own levels run out."""
        c, W, P = self.cc, self.W, self.P
        E, S, H, Dm = W.d_inner, W.d_state, W.heads, W.d_model
        cd = W.conv_dim
        u = self._rms(h, Dm, W["norm_w"], P.rsqrt1, bounds, "h", "n1", W.eps)
        u = self._fit(u, self.needs["u"], bounds["u"], "u", Dm)
        proj = self._linear(u, "w_in")
        proj = self._fit(proj, self.needs["proj"], bounds["proj"], "proj", W.proj_dim)
        # xBC stream at [0, conv_dim) and the causal conv
        xbc = self.pm._mul_mask(c.EvalRotate(proj, E), self.pm._block_mask(0, cd))
        window = [self._fit(w, self.needs["xbc"], bounds["xbc"], "xbc", cd) if w is not None else None
                  for w in conv_state] + [xbc]
        taps = []
        for k in range(W.conv_kernel):
            t = np.zeros(c.slots)
            t[:cd] = W["conv_w"][:, k]
            taps.append(t)
        bias = np.zeros(c.slots)
        bias[:cd] = W["conv_b"]
        xc = self.pm.conv(window, taps, bias)
        xc = self._fit(xc, self._need(P.silu_x), bounds["xc"], "xc", cd)
        xa = self._poly(xc, P.silu_x, 0, cd)
        # dt and decay at [0, heads)
        dtv = self.pm._mul_mask(c.EvalRotate(proj, E + cd), self.pm._block_mask(0, H))
        if dtv.GetNoiseScaleDeg() >= 2:
            c.RescaleInPlace(dtv)
        bias_dt = np.zeros(c.slots)
        bias_dt[:H] = W["dt_bias"]
        dtv = c.EvalAdd(dtv, self.pm.plain(bias_dt, level=c.n_q - dtv.n_limbs(), scale=dtv.GetScalingFactor()))
        gates = getattr(P, "gates", None)
        if gates is not None:  # joint gates: write and decay from one shared factor
            dtv = self._fit(dtv, gates.levels, bounds["dt"], "dt", H)
            dts, decay = gates.encrypted(self.pm, dtv, H)
            pack = c.EvalAdd(xa, c.EvalRotate(dts, -self.dt_base))
            if ssm_state is not None:
                pack = c.EvalAdd(pack, c.EvalRotate(decay, -self.decay_base))
        elif getattr(P, "decay", None) is not None:  # fused decay: dts and decay both from dt
            dtv = self._fit(dtv, max(self._need(P.softplus), P.decay.levels), bounds["dt"], "dt", H)
            dts = self._poly(dtv, P.softplus, 0, H)
            pack = c.EvalAdd(xa, c.EvalRotate(dts, -self.dt_base))
            if ssm_state is not None:
                pack = c.EvalAdd(pack, c.EvalRotate(P.decay.encrypted(self.pm, dtv, H), -self.decay_base))
        else:
            dtv = self._fit(dtv, self._need(P.softplus), bounds["dt"], "dt", H)
            dts = self._poly(dtv, P.softplus, 0, H)
            pack = c.EvalAdd(xa, c.EvalRotate(dts, -self.dt_base))
        if gates is None and getattr(P, "decay", None) is None and ssm_state is not None:
            # heads a payload prunes (head mask 0) get input 0, inside the
            # decay polynomial's domain; the polynomial's output mask zeroes them
            mask = getattr(P.exp, "head_mask", None)
            avec = np.zeros(c.slots)
            avec[:H] = W["a"] if mask is None else W["a"] * mask
            adt = self._fit(self.pm._mul_mask(dts, avec), self._need(P.exp), bounds["adt"], "adt", H)
            decay = self._poly(adt, P.exp, 0, H)
            pack = c.EvalAdd(pack, c.EvalRotate(decay, -self.decay_base))
        pack = self._fit(pack, self.needs["pack"], bounds["pack"], "pack", self.decay_base + H)
        # state update and readout from the packed inputs
        if ssm_state is not None:
            ssm_state = [self._fit(st, self.needs["state"], bounds["state"], "state") for st in ssm_state]
        states, y = self.pm.step(ssm_state, pack, pack, pack if ssm_state is not None else None)
        dvec = np.zeros(c.slots)
        dvec[:E] = np.repeat(W["d"], W.head_dim)
        y = c.EvalAdd(y, self.pm._mul_mask(pack, dvec))
        # gate
        z = self.pm._mul_mask(proj, self.pm._block_mask(0, E))
        z = self._fit(z, self._need(P.silu_z), bounds["z"], "z", E)
        sz = self._poly(z, P.silu_z, 0, E)
        y = self._fit(y, self.needs["y"], bounds["y"], "y", E)
        g = c.EvalMult(y, sz)
        gn = self._rms(g, E, W["gn_w"], P.rsqrt2, bounds, "g", "n2", getattr(W, "gated_eps", W.eps))
        gn = self._fit(gn, self.needs["gn"], bounds["gn"], "gn", E)
        out = self._linear(gn, "w_out")
        h_out = c.EvalAdd(h, out)
        return h_out, window[1:], states


def poly_step_record(W: Mamba2Weights, P: Mamba2Polys, h, conv, st, rec, dom=None):
    """The layer on plaintext with the polynomials, reporting the magnitude of
    every refreshed intermediate (rec(site, values)) and, when dom is given,
    where every Chebyshev input falls on its interval (dom(name, t), |t| <= 1
    inside).  h may carry leading batch axes."""
    def at(name, p, x):
        if dom is not None and isinstance(p, (Poly, HeadPoly)):
            dom(name, p.position(x))
        return x

    rec("h", h)
    u = plain_rms(h, W["norm_w"], W.eps, P.rsqrt1, rec=rec, key="n1", dom=dom)
    rec("u", u)
    proj = u @ W["w_in"].T
    rec("proj", proj)
    z, xbc, dt = _split_proj(W, proj)
    rec("xbc", xbc)
    rec("z", z)
    window = list(conv) + [xbc]
    xc = sum(W["conv_w"][:, k] * window[k] for k in range(W.conv_kernel)) + W["conv_b"]
    rec("xc", xc)
    xa = P.silu_x(at("silu_x", P.silu_x, xc))
    rec("xa", xa)
    rec("dt", dt + W["dt_bias"])
    gates = getattr(P, "gates", None)
    if gates is not None:  # joint gates: (write, decay) from one factorisation
        dts, decay = gates(dt + W["dt_bias"])
    else:
        dts = P.softplus(at("softplus", P.softplus, dt + W["dt_bias"]))
        decay = None
        if getattr(P, "decay", None) is not None:
            decay = P.decay(at("decay", P.decay, dt + W["dt_bias"]))
        else:
            rec("adt", W["a"] * dts)
    rec("dts", dts)
    rec("pack", xa)
    rec("pack", dts)
    rec("pack", [1.0])
    x, B, C = _split_xa(W, xa)
    if st is not None and decay is None:
        decay = P.exp(at("exp", P.exp, W["a"] * dts))
    st, y = _ssm(st, decay, dts, x, B, C, W["d"])
    rec("state", st)
    rec("y", y)
    g = y.reshape(y.shape[:-2] + (W.d_inner,)) * P.silu_z(at("silu_z", P.silu_z, z))
    rec("g", g)
    gn = plain_rms(g, W["gn_w"], getattr(W, "gated_eps", W.eps), P.rsqrt2, rec=rec, key="n2", dom=dom)
    rec("gn", gn)
    out = gn @ W["w_out"].T
    return h + out, window[1:], st


def calibrate_bounds(W: Mamba2Weights, P: Mamba2Polys, samples: int = 4, seed: int = 11, tokens: int = 3):
    """Refresh bounds (max |value| x 2, at least 1) of every refreshed intermediate,
    from plaintext runs of the polynomial path over a few tokens."""
    r = np.random.default_rng(seed)
    E, S, H, Pd = W.d_inner, W.d_state, W.heads, W.head_dim
    m = {}

    def rec(k, v):
        m[k] = max(m.get(k, 0.0), float(np.max(np.abs(v))))

    for _ in range(samples):
        conv = [np.zeros(W.conv_dim) for _ in range(W.conv_kernel - 1)]
        st = r.uniform(-1, 1, (H, Pd, S))
        for _ in range(tokens):
            h = r.normal(0, 1, W.d_model)
            h2, conv, st = poly_step_record(W, P, h, conv, st, rec)
    return {k: max(1.0, 2.0 * v) for k, v in m.items()}


class Mamba2Model:
    """A layers-deep Mamba-2 language model (tied embedding, final RMSNorm) with
    synthetic weights, for the encrypted greedy token loop:
    the client encrypts the embedding of the current token, the server runs
    every layer on ciphertexts, the client decrypts the final hidden vector and
    picks the argmax token (the reference's GenerationClient::select,
    native/fideslib_stage0/src/packed_fideslib.cpp:842-880)."""

    def __init__(self, layers: int, d_model: int, d_state: int, heads: int, vocab: int, std: float = 0.02,
                 seed: int = 6, calib_sequences: int = 8, calib_tokens: int = 32, calib_prompt: int = 8,
                 bound_factor: float = 3.0, fused_decay: bool = False, calib_threads: int | None = None):
        self.layers = [Mamba2Weights(d_model=d_model, d_state=d_state, heads=heads, std=std, seed=seed * 1000 + i)
                       for i in range(layers)]
        r = np.random.default_rng(seed)
        self.embedding = r.normal(0, 1.0, (vocab, d_model))
        self.norm_f = 1.0 + r.normal(0, 0.02, d_model)
        eps = self.layers[0].eps
        self.d_model = d_model
        # Calibration through the whole stack, never on the inputs a run is
        # checked on: calib_sequences token sequences of calib_tokens tokens
        # from this model's own seed, each a random prompt of calib_prompt
        # tokens; half continue greedily (the generation protocol, whose
        # repeated tokens drive the slowly decaying state heads furthest), half
        # with random tokens.  The horizon must cover the run: the recurrent
        # state keeps growing for about 1 / (1 - decay) tokens.
        B, T = calib_sequences, calib_tokens
        toks = r.integers(0, vocab, (B, T))
        greedy = np.arange(B) % 2 == 0
        # Sequences run in chunks on a thread pool (numpy releases the GIL in
        # its array loops); the reductions below do not depend on the split.
        workers = max(1, min(B, calib_threads or os.cpu_count() or 1, 8))
        step = -(-B // workers)
        chunks = [slice(i, min(B, i + step)) for i in range(0, B, step)]

        def exact_chunk(sl):  # exact-function trajectories give the polynomial domains ...
            tk, gr = toks[sl], greedy[sl]
            ranges = [new_ranges() for _ in self.layers]
            finals = []
            b = tk.shape[0]
            state = [([np.zeros((b, W.conv_dim)) for _ in range(W.conv_kernel - 1)],
                      np.zeros((b, W.heads, W.head_dim, W.d_state))) for W in self.layers]
            for t in range(T):
                h = self.embedding[tk[:, t]]
                for li, W in enumerate(self.layers):
                    h, c_, s_ = exact_step(W, h, state[li][0], state[li][1], range_updater(ranges[li]))
                    state[li] = (c_, s_)
                finals.append(np.mean(h * h, axis=-1) + eps)
                if calib_prompt <= t + 1 < T:
                    nxt = np.argmax(_rms(h, self.norm_f, eps) @ self.embedding.T, axis=-1)
                    tk[gr, t + 1] = nxt[gr]
            return ranges, np.concatenate(finals)

        with _single_threaded_blas(), ThreadPoolExecutor(workers) as ex:
            parts = list(ex.map(exact_chunk, chunks))
        ranges = [new_ranges() for _ in self.layers]
        for part, _ in parts:
            for li, rg in enumerate(part):
                for k, (lo, hi) in rg.items():
                    ranges[li][k][0] = min(ranges[li][k][0], lo)
                    ranges[li][k][1] = max(ranges[li][k][1], hi)
        finals = np.concatenate([f for _, f in parts])
        self.polys = [Mamba2Polys(W, ranges=rg, fused_decay=fused_decay) for W, rg in zip(self.layers, ranges)]
        lo, hi = 0.25 * float(finals.min()), 4.0 * float(finals.max())
        self.rsqrt_f = Poly(cheb_fit(lambda t: 1 / np.sqrt(t), lo, hi, 15), lo, hi)

        # ... and the polynomial path's magnitudes over the same tokens the
        # refresh bounds (bound_factor x the largest magnitude, at least 1:
        # single random tokens reach almost twice the largest value of a few
        # hundred calibration tokens)
        def poly_chunk(sl):
            tk = toks[sl]
            mags = [{} for _ in self.layers]
            final = 0.0
            state = [([np.zeros((tk.shape[0], W.conv_dim)) for _ in range(W.conv_kernel - 1)], None)
                     for W in self.layers]
            for t in range(T):
                h = self.embedding[tk[:, t]]
                for li, (W, P) in enumerate(zip(self.layers, self.polys)):
                    def rec(k, v, m=mags[li]):
                        m[k] = max(m.get(k, 0.0), float(np.max(np.abs(v))))
                    h, c_, s_ = poly_step_record(W, P, h, state[li][0], state[li][1], rec)
                    state[li] = (c_, s_)
                final = max(final, float(np.max(np.abs(h))))
            return mags, final

        with _single_threaded_blas(), ThreadPoolExecutor(workers) as ex:
            parts = list(ex.map(poly_chunk, chunks))
        mags = [{} for _ in self.layers]
        for part, _ in parts:
            for li, m in enumerate(part):
                for k, v in m.items():
                    mags[li][k] = max(mags[li].get(k, 0.0), v)
        final = max(f for _, f in parts)
        self.bounds = [{k: max(1.0, bound_factor * v) for k, v in m.items()} for m in mags]
        self.final_bound = max(1.0, bound_factor * final)
        self.calibration = {"sequences": B, "tokens": T, "prompt": calib_prompt, "greedy_sequences": int(greedy.sum()),
                            "bound_factor": bound_factor, "seed": seed}

    def audit(self, inputs):
        """The plaintext polynomial path over one sequence of input tokens, as
        the encrypted loop runs it: for every refresh site the largest
        |value| / bound (above 1 the refresh leaves its interval), and for every
        Chebyshev series the largest |position| of its input on its interval
        (above 1 the series extrapolates), each with the evaluation and layer
        where it falls.  The final hidden vector's refresh counts as layer
        len(layers)."""
        ratio, dom = {}, {}

        def keep(table, k, r, e, li):
            if r > table.get(k, {"max": -1.0})["max"]:
                table[k] = {"max": r, "eval": e, "layer": li}

        state = self.initial_state()
        for e, tok in enumerate(inputs):
            h = self.embedding[tok].copy()
            for li, (W, P) in enumerate(zip(self.layers, self.polys)):
                b = self.bounds[li]

                def rec(k, v, li=li, b=b):
                    if k in b:
                        keep(ratio, k, float(np.max(np.abs(v))) / b[k], e, li)

                def dm(k, t, li=li):
                    keep(dom, k, float(np.max(np.abs(t))), e, li)

                h, c_, s_ = poly_step_record(W, P, h, state[li][0], state[li][1], rec, dm)
                state[li] = (c_, s_)
            keep(ratio, "final", float(np.max(np.abs(h))) / self.final_bound, e, len(self.layers))
            keep(dom, "rsqrt_f", float(np.max(np.abs(self.rsqrt_f.position(np.mean(h * h) + self.layers[0].eps)))),
                 e, len(self.layers))
        return {"bound_ratio": ratio, "domain": dom,
                "max_bound_ratio": max(v["max"] for v in ratio.values()),
                "max_domain_position": max(v["max"] for v in dom.values())}

    def initial_state(self):
        return [([np.zeros(W.conv_dim) for _ in range(W.conv_kernel - 1)], None) for W in self.layers]

    def plain_token(self, token: int, state):
        """One token on plaintext (polynomial path); returns (hidden, logits, state)."""
        h = self.embedding[token].copy()
        new = []
        for W, P, (conv, st) in zip(self.layers, self.polys, state):
            h, conv, st = plain_step(W, P, h, conv, st)
            new.append((conv, st))
        hf = plain_rms(h, self.norm_f, self.layers[0].eps, self.rsqrt_f)
        return hf, self.embedding @ hf, new


class EncryptedMamba2Model:
    """The model's layers on one CryptoContext; client-side encryption and
    selection around them."""

    def __init__(self, cc, model: Mamba2Model, passes: int = 2, cache_gb: float = 0.0, margin: int = 4,
                 needs: dict | None = None, device_diagonals: bool = True, memo_gb: float = 4.0):
        self.cc, self.m = cc, model
        self.cache = PlaintextCache(cache_gb * 2 ** 30)
        # the layers' constant slot vectors, encoded once per level and scale
        self.memo = PlaintextMemo(cc, memo_gb * 2 ** 30) if memo_gb > 0 else None
        self.layers = [EncryptedMamba2Layer(cc, W, P, passes=passes, margin=margin, cache=self.cache, needs=needs,
                                            device_diagonals=device_diagonals, memo=self.memo)
                       for W, P in zip(model.layers, model.polys)]
        self.state = [([None] * (W.conv_kernel - 1), None) for W in model.layers]
        self.tokens, self.margins = [], []

    def rotation_steps(self):
        s = set()
        for layer in self.layers:
            s |= set(layer.rotation_steps())
        return sorted(s)

    def step(self, token: int):
        """Server pass for one token: returns the encrypted final hidden vector."""
        c, m = self.cc, self.m
        h = c.Encrypt(c.MakeCKKSPackedPlaintext(np.pad(m.embedding[token], (0, c.slots - m.d_model))))
        new = []
        for layer, (conv, st), bounds in zip(self.layers, self.state, m.bounds):
            h, conv, st = layer.step(h, conv, st, bounds)
            new.append((conv, st))
        self.state = new
        last = self.layers[-1]
        h = last._fit(h, 14, m.final_bound, support=m.d_model)
        return last.pm.rms_norm(h, m.d_model, m.norm_f, m.layers[0].eps, (m.rsqrt_f.lo, m.rsqrt_f.hi),
                                degree=len(m.rsqrt_f.coeffs) - 1)

    def select(self, hidden_ct):
        """Client: decrypt the final hidden vector and pick the greedy token."""
        hf = self.cc.Decrypt(hidden_ct).GetRealPackedValue()[:self.m.d_model]
        logits = self.m.embedding @ hf
        order = np.argsort(logits)[::-1]
        self.tokens.append(int(order[0]))
        self.margins.append(float(logits[order[0]] - logits[order[1]]))
        return int(order[0]), hf

    def refreshes(self):
        return sum(layer.refreshes for layer in self.layers)
