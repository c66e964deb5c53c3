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

from dataclasses import dataclass, field

import numpy as np

from .mamba import PackedMamba2, StateLayout


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

    def __call__(self, x):
        return np.polynomial.chebyshev.chebval((2 * x - self.lo - self.hi) / (self.hi - self.lo), self.coeffs)


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


def _rms(x, w, eps):
    return x / np.sqrt(np.mean(x * x) + eps) * w


class Mamba2Polys:
    """Polynomial domains calibrated on exact-function trajectories (random
    residual inputs over a few tokens, recurrent state U[-1, 1]), widened by half
    their span."""

    def __init__(self, W: Mamba2Weights, degree: int = 31, seed_degree: int = 15, samples: int = 16,
                 tokens: int = 3, seed: int = 9):
        r = np.random.default_rng(seed)
        E, S, H, K, Pd = W.d_inner, W.d_state, W.heads, W.conv_kernel, W.head_dim
        ranges = {k: [np.inf, -np.inf] for k in ("xc", "dt", "adt", "z", "v1", "v2")}

        def upd(k, v):
            ranges[k][0] = min(ranges[k][0], float(np.min(v)))
            ranges[k][1] = max(ranges[k][1], float(np.max(v)))

        for _ in range(samples):
            conv = [np.zeros(W.conv_dim) for _ in range(K - 1)]
            st = r.uniform(-1, 1, (H, Pd, S))
            for _ in range(tokens):
                h = r.normal(0, 1, W.d_model)
                upd("v1", [np.mean(h * h) + W.eps])
                u = _rms(h, W["norm_w"], W.eps)
                proj = W["w_in"] @ u
                z, xbc, dt = proj[:E], proj[E:E + W.conv_dim], proj[E + W.conv_dim:]
                window = conv + [xbc]
                xc = sum(W["conv_w"][:, k] * window[k] for k in range(K)) + W["conv_b"]
                upd("xc", xc)
                xa = _silu(xc)
                upd("dt", dt + W["dt_bias"])
                dts = _softplus(dt + W["dt_bias"])
                upd("adt", W["a"] * dts)
                upd("z", z)
                x, B, C = xa[:E].reshape(H, Pd), xa[E:E + S], xa[E + S:]
                st = np.exp(W["a"] * dts)[:, None, None] * st + (dts[:, None] * x)[:, :, None] * B[None, None, :]
                y = (st * C[None, None, :]).sum(-1) + W["d"][:, None] * x
                g = y.reshape(E) * _silu(z)
                upd("v2", [np.mean(g * g) + W.eps])
                conv = window[1:]

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

    @staticmethod
    def _fit(fn, lo, hi, degree):
        return Poly(cheb_fit(fn, lo, hi, degree), lo, hi)


def plain_rms(x, w, eps, seed: Poly, newton=2):
    v = np.mean(x * x) + eps
    y = seed(v)
    for _ in range(newton):
        y = 1.5 * y - 0.5 * v * y ** 3
    return x * y * w


def plain_step(W: Mamba2Weights, P: Mamba2Polys, h, conv_state, ssm_state):
    """The layer on plaintext with the same polynomials.  conv_state: list of the
    last conv_kernel-1 xBC vectors (oldest first); ssm_state: [H, P, S] or None."""
    E, S, H, Pd = W.d_inner, W.d_state, W.heads, W.head_dim
    u = plain_rms(h, W["norm_w"], W.eps, P.rsqrt1)
    proj = W["w_in"] @ u
    z, xbc, dt = proj[:E], proj[E:E + W.conv_dim], proj[E + W.conv_dim:]
    window = list(conv_state) + [xbc]
    xc = sum(W["conv_w"][:, k] * window[k] for k in range(W.conv_kernel)) + W["conv_b"]
    xa = P.silu_x(xc)
    x, B, C = xa[:E].reshape(H, Pd), xa[E:E + S], xa[E + S:]
    dts = P.softplus(dt + W["dt_bias"])
    decay = P.exp(W["a"] * dts)
    upd = (dts[:, None] * x)[:, :, None] * B[None, None, :]
    st = upd if ssm_state is None else decay[:, None, None] * ssm_state + upd
    y = (st * C[None, None, :]).sum(-1) + W["d"][:, None] * x
    g = y.reshape(E) * P.silu_z(z)
    gn = plain_rms(g, W["gn_w"], W.eps, P.rsqrt2)
    out = W["w_out"] @ gn
    return h + out, window[1:], st


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


class EncryptedMamba2Layer:
    """The layer on ciphertexts of one CryptoContext (full packing)."""

    def __init__(self, cc, W: Mamba2Weights, P: Mamba2Polys, passes: int = 2, margin: int = 3):
        self.cc, self.W, self.P = cc, W, P
        self.passes, self.margin = passes, margin
        E, S, H = W.d_inner, W.d_state, W.heads
        self.layout = StateLayout(H, W.head_dim, S, cc.slots)
        self.pm = PackedMamba2(cc, self.layout, b_base=E, c_base=E + S, head_base=0)
        self.refreshes = 0
        self._lin = {}
        n = cc.slots
        # BSGS shapes: baby 32 or sqrt(n_in); replicated inputs
        self.lin_shapes = {}
        for name, (m, k) in {"w_in": (W.proj_dim, W.d_model), "w_out": (W.d_model, E)}.items():
            b = 1
            while b * b < k and b < 32:
                b *= 2
            G = -(-k // b)
            reps = 1
            while reps * k < m + k:
                reps *= 2
            if reps * k > n:
                raise ValueError("input replication does not fit the slots")
            self.lin_shapes[name] = (b, G, reps)

    # ---- setup --------------------------------------------------------------
    def rotation_steps(self):
        W, n = self.W, self.cc.slots
        s = set(self.pm.rotation_steps())
        for name, (b, G, reps) in self.lin_shapes.items():
            k = W.d_model if name == "w_in" else W.d_inner
            s |= {j for j in range(1, b)} | {g * b for g in range(1, G)}
            s |= {-(k << i) for i in range(reps.bit_length() - 1)}
        for width in (W.d_model, W.d_inner):
            win = 1 << (width - 1).bit_length()
            s |= {1 << i for i in range(win.bit_length() - 1)} | {-win}
        s |= {W.d_inner, W.d_inner + W.conv_dim}
        return sorted(v % n for v in s if v % n)

    def _diags(self, name):
        if name not in self._lin:
            b, G, _ = self.lin_shapes[name]
            self._lin[name] = rect_diagonals(self.W[name], b, G, self.cc.slots)
        return self._lin[name]

    # ---- helpers --------------------------------------------------------------
    def _left(self, ct):
        return ct.n_limbs() - 1 - (1 if ct.GetNoiseScaleDeg() >= 2 else 0)

    def _fit(self, ct, need, bound):
        """Refreshes ct when fewer than need (+ margin) levels remain."""
        if self._left(ct) >= need + self.margin:
            return ct
        self.refreshes += 1
        return self.cc.refresh(ct, bound, passes=self.passes)

    def _linear(self, x, name):
        c = self.cc
        b, G, reps = self.lin_shapes[name]
        k = self.W[name].shape[1]
        for i in range(reps.bit_length() - 1):
            x = c.EvalAdd(x, c.EvalRotate(x, -(k << i)))
        nq = x.n_limbs() - (1 if x.GetNoiseScaleDeg() >= 2 else 0)
        diags = self._diags(name)
        dense = [d for d in diags if d is not None]
        pts = iter(c.MakeCKKSPackedPlaintexts(np.array(dense), level=c.n_q - nq))
        plist = [next(pts) if d is not None else None for d in diags]
        return c.EvalLinearTransform(x, plist, b, G)

    def _poly(self, x, p: Poly, lo_slot, hi_slot):
        return self.pm.poly(x, p.coeffs, p.lo, p.hi, lo_slot, hi_slot)

    def _rms(self, x, width, weight, seed: Poly, bound):
        c = self.cc
        x = self._fit(x, 14, bound)
        return self.pm.rms_norm(x, width, weight, self.W.eps, (seed.lo, seed.hi), degree=len(seed.coeffs) - 1)

    # ---- one token ------------------------------------------------------------
    def step(self, h, conv_state, ssm_state, bounds):
        """h: ciphertext of the residual stream at [0, d_model); conv_state: list
        of conv_kernel-1 xBC ciphertexts (None for zeros); ssm_state: list of
        group ciphertexts or None.  Returns (h_out, conv_state, ssm_state)."""
        c, W, P = self.cc, self.W, self.P
        E, S, H, Dm = W.d_inner, W.d_state, W.heads, W.d_model
        cd = W.conv_dim
        u = self._rms(h, Dm, W["norm_w"], P.rsqrt1, bounds["h"])
        u = self._fit(u, 1, bounds["u"])
        proj = self._linear(u, "w_in")
        # xBC stream at [0, conv_dim)
        xbc = self.pm._mul_mask(c.EvalRotate(proj, E), self.pm._block_mask(0, cd))
        window = [self._fit(w, 2, bounds["xbc"]) if w is not None else None for w in conv_state] + [xbc]
        taps = []
        for k in range(W.conv_kernel):
            t = np.zeros(c.slots)
            t[:cd] = W["conv_w"][:, k]
            taps.append(t)
        bias = np.zeros(c.slots)
        bias[:cd] = W["conv_b"]
        xc = self.pm.conv(window, taps, bias)
        xc = self._fit(xc, 8, bounds["xc"])
        xa = self._poly(xc, P.silu_x, 0, cd)
        # dt and decay at [0, heads)
        dtv = self.pm._mul_mask(c.EvalRotate(proj, E + cd), self.pm._block_mask(0, H))
        if dtv.GetNoiseScaleDeg() >= 2:
            c.RescaleInPlace(dtv)
        bias_dt = np.zeros(c.slots)
        bias_dt[:H] = W["dt_bias"]
        dtv = c.EvalAdd(dtv, c.MakeCKKSPackedPlaintext(bias_dt, level=c.n_q - dtv.n_limbs(),
                                                        scale=dtv.GetScalingFactor()))
        dtv = self._fit(dtv, 8, bounds["dt"])
        dts = self._poly(dtv, P.softplus, 0, H)
        avec = np.zeros(c.slots)
        avec[:H] = W["a"]
        adt = self.pm._mul_mask(dts, avec)
        adt = self._fit(adt, 8, bounds["adt"])
        decay = self._poly(adt, P.exp, 0, H) if ssm_state is not None else None
        # state update and readout
        xa = self._fit(xa, 8, bounds["xa"])
        dts = self._fit(dts, 8, bounds["dts"])
        if ssm_state is not None:
            decay = self._fit(decay, 6, 1.0)
            ssm_state = [self._fit(s, 4, bounds["state"]) for s in ssm_state]
        states, y = self.pm.step(ssm_state, xa, dts, decay)
        dvec = np.zeros(c.slots)
        dvec[:E] = np.repeat(W["d"], W.head_dim)
        y = c.EvalAdd(y, self.pm._mul_mask(xa, dvec))
        # gate
        z = self.pm._mul_mask(proj, self.pm._block_mask(0, E))
        z = self._fit(z, 8, bounds["z"])
        sz = self._poly(z, P.silu_z, 0, E)
        y = self._fit(y, 2, bounds["y"])
        g = c.EvalMult(y, sz)
        gn = self._rms(g, E, W["gn_w"], P.rsqrt2, bounds["g"])
        gn = self._fit(gn, 1, bounds["gn"])
        out = self._linear(gn, "w_out")
        h_out = c.EvalAdd(h, out)
        return h_out, window[1:], states


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
            rec("h", h)
            u = plain_rms(h, W["norm_w"], W.eps, P.rsqrt1)
            rec("u", u)
            proj = W["w_in"] @ u
            z, xbc, dt = proj[:E], proj[E:E + W.conv_dim], proj[E + W.conv_dim:]
            rec("xbc", xbc)
            rec("z", z)
            window = conv + [xbc]
            xc = sum(W["conv_w"][:, k] * window[k] for k in range(W.conv_kernel)) + W["conv_b"]
            rec("xc", xc)
            xa = P.silu_x(xc)
            rec("xa", xa)
            rec("dt", dt + W["dt_bias"])
            dts = P.softplus(dt + W["dt_bias"])
            rec("dts", dts)
            rec("adt", W["a"] * dts)
            x, B, C = xa[:E].reshape(H, Pd), xa[E:E + S], xa[E + S:]
            st = P.exp(W["a"] * dts)[:, None, None] * st + (dts[:, None] * x)[:, :, None] * B[None, None, :]
            rec("state", st)
            y = (st * C[None, None, :]).sum(-1) + W["d"][:, None] * x
            rec("y", y)
            g = y.reshape(E) * P.silu_z(z)
            rec("g", g)
            rec("gn", plain_rms(g, W["gn_w"], W.eps, P.rsqrt2))
            conv = window[1:]
    return {k: max(1.0, 2.0 * v) for k, v in m.items()}
