"""The reference's Mamba-2 chain payload and its encrypted decode loop.

A chain payload is what the reference's exporter writes for its native Mamba-2
decode (``export_chain_payload``, src/fhemamba/m1_payload.py:901-1085) and what
that decode reads (``read_chain_payload`` / ``read_m1_payload``,
native/fideslib_stage0/src/stage1_mamba2_payload.cpp:233-528):

* ``chain.json`` -- format ``fhemamba-m2-chain-v1``, ``n_layers``,
  ``n_test_tokens``, ``final_norm_eps``, ``layer_dirs``, ``tensors`` (name ->
  shape of ``<name>.bin``, float32 little endian: ``final_norm_w``,
  ``chain_input_embeddings``, ``chain_expected_final``,
  ``chain_expected_poly_final``), an optional ``final_norm_poly`` and an
  optional ``autoregressive`` block (protocol ``client-in-loop-greedy-v1``:
  prompt and greedy ids, ``client_embedding_w``, optional untied
  ``client_lm_head_w`` / ``client_lm_head_b``, the polynomial circuit's
  embeddings and final hidden vectors per server evaluation);
* ``layer_XX/meta.json`` -- format ``fhemamba-m1-v1``, ``dims``, ``eps``,
  ``polys`` (one nonlinearity per site), ``carried_bounds`` and ``tensors``
  (``in_proj_w``, ``conv_w``, ``conv_b``, ``dt_bias``, ``a_log``, ``d_skip``,
  ``block_norm_w``, ``gated_norm_w``, ``out_proj_w`` and the layer's test
  vectors).

The nonlinearity kinds (``_poly_from_export_spec``,
src/fhemamba/m1_payload.py:372-408, with the evaluators of src/fhemamba/ops.py
and src/fhemamba/normalization.py) are evaluated here both in fp64 -- the
polynomial circuit that ``chain_expected_poly_final`` records -- and on
ciphertexts through the device library:

* ``cheb``: sum c_i T_i((2x - lo - hi) / (hi - lo)) (Clenshaw);
* ``cheb-squared``: p(x)^2, p fitted to sqrt(softplus);
* ``cheb-resquared``: p(x / 2^k)^(2^k), p fitted to exp on [lo, 0], optionally
  times a per-head 0/1 mask (pruned heads);
* ``const-newton`` / ``poly-newton`` / ``sq-poly-newton``: inverse square
  roots as Newton iterations y <- y (1.5 - 0.5 v y^2) from a constant, from
  0.9 p(v), or from damping * q(v)^2;
* ``scaled-goldschmidt-invsqrt-v1``: a coupled (y, u = v y^2) iteration
  y <- y (a_i - b_i u), u <- u (a_i - b_i u)^2 from a public seed, then one
  Newton step recomputed from v.

The joint formats (``fhemamba-m2-chain-joint-v1`` / ``fhemamba-m1-joint-v1``)
add shared-dissipation-factor gates (``JointGate``) that replace the softplus
and decay sites.
"""
from __future__ import annotations

import json
import math
import time
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np

from .mamba2_layer import EncryptedMamba2Layer, PlaintextCache, plain_rms, poly_step_record

CHAIN_FORMAT = "fhemamba-m2-chain-v1"
JOINT_CHAIN_FORMAT = "fhemamba-m2-chain-joint-v1"
LAYER_FORMAT = "fhemamba-m1-v1"
JOINT_LAYER_FORMAT = "fhemamba-m1-joint-v1"
SITES = ("conv_silu", "gate_silu", "dt_softplus", "decay_exp", "rms_invsqrt", "gated_rms_invsqrt")
NORM_SITES = ("rms_invsqrt", "gated_rms_invsqrt")


class PayloadError(ValueError):
    """A chain payload that the decode cannot use (the reference raises
    std::runtime_error with the same message)."""


# ---------------------------------------------------------------------------
# nonlinearities


def _clenshaw(coeffs, t):
    b1 = np.zeros_like(t)
    b2 = np.zeros_like(t)
    for c in coeffs[:0:-1]:
        b1, b2 = 2.0 * t * b1 - b2 + c, b1
    return t * b1 - b2 + coeffs[0]


def chebyshev_levels(n_coeffs: int) -> int:
    """Levels the device Paterson-Stockmeyer evaluation of an n-coefficient
    series spends on an input already in [-1, 1] (an upper bound: the power
    basis up to 2^ceil(log2 n), the leaf weights, one product per split)."""
    return max(1, math.ceil(math.log2(max(2, n_coeffs)))) + 1


@dataclass(frozen=True)
class ChebSeries:
    """``cheb``: a Chebyshev series on [lo, hi] (ChebPoly, src/fhemamba/ops.py:180-196)."""

    coeffs: tuple
    lo: float
    hi: float

    def __call__(self, x):
        x = np.asarray(x, dtype=np.float64)
        return _clenshaw(self.coeffs, (2.0 * x - (self.lo + self.hi)) / (self.hi - self.lo))

    @property
    def degree(self) -> int:
        return len(self.coeffs) - 1

    @property
    def levels(self) -> int:
        # slot-masked affine map, the series, the output mask
        return chebyshev_levels(len(self.coeffs)) + 2

    def encrypted(self, pm, x, lo_slot, hi_slot, out_mask=None):
        return pm.poly(x, np.asarray(self.coeffs), self.lo, self.hi, lo_slot, hi_slot, out_mask)


@dataclass(frozen=True)
class SquaredSeries:
    """``cheb-squared``: p(x)^2 (SquaredPoly, src/fhemamba/ops.py:262-280)."""

    base: ChebSeries

    def __call__(self, x):
        y = self.base(x)
        return y * y

    @property
    def levels(self) -> int:
        return self.base.levels + 1

    def encrypted(self, pm, x, lo_slot, hi_slot):
        y = self.base.encrypted(pm, x, lo_slot, hi_slot)
        return pm.cc.EvalMult(y, y)


@dataclass(frozen=True)
class ResquaredExp:
    """``cheb-resquared``: exp on [lo 2^k, 0] as p(x / 2^k)^(2^k), times a 0/1
    head mask when heads are pruned (SquaredExpPoly and HeadMaskedDecay,
    src/fhemamba/ops.py:228-258,300-340).  Pruned heads' inputs are clamped to
    the domain in fp64 (their output is zeroed anyway); on ciphertexts their
    input is zeroed before the series and the mask is the series' output mask,
    which the squarings keep."""

    base: ChebSeries
    squarings: int
    head_mask: np.ndarray | None = None

    @property
    def lo(self) -> float:
        return self.base.lo * 2.0 ** self.squarings

    def __call__(self, x):
        x = np.asarray(x, dtype=np.float64)
        if self.head_mask is not None:
            x = np.where(self.head_mask > 0.0, x, np.maximum(x, self.lo))
        y = self.base(x / 2.0 ** self.squarings)
        for _ in range(self.squarings):
            y = y * y
        return y if self.head_mask is None else y * self.head_mask

    @property
    def levels(self) -> int:
        return self.base.levels + self.squarings

    def encrypted(self, pm, x, lo_slot, hi_slot):
        mask = None
        if self.head_mask is not None:
            if self.head_mask.size != hi_slot - lo_slot:
                raise PayloadError("decay_exp head_mask must contain one value per head")
            mask = np.zeros(pm.L.slots)
            mask[lo_slot:hi_slot] = self.head_mask
        k = 2.0 ** self.squarings
        y = pm.poly(x, np.asarray(self.base.coeffs), self.base.lo * k, self.base.hi * k, lo_slot, hi_slot, mask)
        for _ in range(self.squarings):
            y = pm.cc.EvalMult(y, y)
        return y


def _newton_step(c, y, vh):
    """y (1.5 - 0.5 v y^2) = 1.5 y + (vh y) y^2 with vh = -v/2: two levels."""
    y2 = c.EvalMult(y, y)
    vy = c.EvalMult(vh, y)
    return c.EvalAdd(c.EvalMult(y, 1.5), c.EvalMult(vy, y2))


class _InvSqrt:
    """Common shape of the inverse square roots: ``inv_sqrt`` in fp64 (with a
    trace of every iterate for refresh bounds), ``encrypted_inv_sqrt`` on a
    ciphertext of v, ``fill`` (a value inside the domain for unused slots)
    and ``levels`` (levels from v to the first refreshable iterate)."""

    iterations: int

    def _newton(self, v, y, trace):
        for _ in range(self.iterations):
            y = y * (1.5 - 0.5 * v * y * y)
            if trace:
                trace("y", y)
        return y

    def _encrypted_newton(self, c, v, y, fit):
        """Newton steps on ciphertexts.  Each step starts with four levels on
        y and -v/2: a refresh before a step costs no precision (the step
        squares the relative error), one after the last step would, so the
        last step leaves the two levels the final x y w products need."""
        vh = c.EvalMult(v, -0.5)
        for _ in range(self.iterations):
            y = fit(y, 4, "y")
            vh = fit(vh, 4, "v")
            y = _newton_step(c, y, vh)
        return y


@dataclass(frozen=True)
class ConstNewton(_InvSqrt):
    """``const-newton``: Newton from the constant guess (NewtonInvSqrt,
    src/fhemamba/ops.py:355-383, with hi = 1 / (4 guess^2))."""

    guess: float
    iterations: int

    @property
    def fill(self) -> float:
        return 0.25 / (self.guess * self.guess)

    levels = 1

    def inv_sqrt(self, v, trace=None):
        y = np.full_like(np.asarray(v, dtype=np.float64), self.guess)
        return self._newton(np.asarray(v, dtype=np.float64), y, trace)

    def encrypted_inv_sqrt(self, c, v, fit):
        if self.iterations == 0:
            raise PayloadError("const-newton needs at least one iteration on ciphertexts")
        g = self.guess
        y = c.EvalAdd(c.EvalMult(v, -0.5 * g ** 3), 1.5 * g)  # the first step from y = g
        inner = ConstNewton(g, self.iterations - 1)
        return inner._encrypted_newton(c, v, y, fit)


@dataclass(frozen=True)
class PolyNewton(_InvSqrt):
    """``poly-newton``: Newton from 0.9 p(v), p fitted to rsqrt (PolyInitNewton,
    src/fhemamba/ops.py:386-410; the 0.9 is the evaluator's constant, which the
    exporter also writes as ``damping``).  The 0.9 is folded into the series."""

    base: ChebSeries
    iterations: int

    @property
    def fill(self) -> float:
        return 0.5 * (self.base.lo + self.base.hi)

    @property
    def levels(self) -> int:
        return chebyshev_levels(len(self.base.coeffs)) + 1

    def inv_sqrt(self, v, trace=None):
        v = np.asarray(v, dtype=np.float64)
        y = 0.9 * self.base(v)
        if trace:
            trace("y", y)
        return self._newton(v, y, trace)

    def encrypted_inv_sqrt(self, c, v, fit):
        y = c.EvalChebyshevSeries(v, 0.9 * np.asarray(self.base.coeffs), self.base.lo, self.base.hi)
        return self._encrypted_newton(c, v, y, fit)


@dataclass(frozen=True)
class SquaredPolyNewton(_InvSqrt):
    """``sq-poly-newton``: Newton from damping * q(v)^2, q fitted to v^(-1/4)
    (SquaredPolyInitNewton, src/fhemamba/ops.py:413-441).  sqrt(damping) is
    folded into the series, whose square is the seed."""

    base: ChebSeries
    iterations: int
    damping: float

    @property
    def fill(self) -> float:
        return 0.5 * (self.base.lo + self.base.hi)

    @property
    def levels(self) -> int:
        return chebyshev_levels(len(self.base.coeffs)) + 2

    def inv_sqrt(self, v, trace=None):
        v = np.asarray(v, dtype=np.float64)
        q = self.base(v)
        y = self.damping * q * q
        if trace:
            trace("y", y)
        return self._newton(v, y, trace)

    def encrypted_inv_sqrt(self, c, v, fit):
        q = c.EvalChebyshevSeries(v, math.sqrt(self.damping) * np.asarray(self.base.coeffs), self.base.lo,
                                  self.base.hi)
        return self._encrypted_newton(c, v, c.EvalMult(q, q), fit)


@dataclass(frozen=True)
class ScheduledInvSqrt(_InvSqrt):
    """``scaled-goldschmidt-invsqrt-v1`` (ScheduledInvSqrt,
    src/fhemamba/normalization.py:40-91): u = v s^2, y = s; per coefficient
    pair f = a - b u, y <- y f and (but for the last pair) u <- u f^2; then
    y (1.5 - 0.5 v y^2) from the original v."""

    lo: float
    hi: float
    seed: float
    coefficients: tuple
    iterations = 1  # the final recomputed Newton step

    @property
    def fill(self) -> float:
        # the geometric mean: inside the interval and, for the wide public
        # intervals these schedules cover (lo ~ 1e-6), near the variances
        # themselves, so that it does not set the refresh bound of v
        return math.sqrt(self.lo * self.hi)

    # v keeps enough levels for u = v s^2 and the final Newton step's -v/2,
    # so that neither is refreshed (v spans the whole public interval, whose
    # bound would swamp the variances themselves)
    levels = 8

    def inv_sqrt(self, v, trace=None):
        v = np.asarray(v, dtype=np.float64)
        u = v * self.seed * self.seed
        y = self.seed
        last = len(self.coefficients) - 1
        for i, (a, b) in enumerate(self.coefficients):
            if trace:
                trace(f"u{i}", u)
            f = a - b * u
            y = y * f
            if trace:
                trace(f"y{i}", y)
            if i < last:
                u = u * (f * f)
        return self._newton(v, y, trace)

    def encrypted_inv_sqrt(self, c, v, fit):
        """u and y move over orders of magnitude during the schedule (u from
        v s^2 towards 1), so each step's refreshes have their own bounds
        (``u<i>``, ``y<i>``): a refresh's error is relative to its bound."""
        s = self.seed
        u = c.EvalMult(v, s * s)
        y = None
        last = len(self.coefficients) - 1
        for i, (a, b) in enumerate(self.coefficients):
            u = fit(u, 3, f"u{i}")
            f = c.EvalAdd(c.EvalMult(u, -b), a)
            y = c.EvalMult(f, s) if y is None else c.EvalMult(fit(y, 2, f"y{i - 1}"), f)
            if i < last:
                u = c.EvalMult(u, c.EvalMult(f, f))
        return self._encrypted_newton(c, v, y, fit)


@dataclass(frozen=True)
class JointGate:
    """Shared-dissipation-factor gates of the joint format (DissipativeGate,
    src/fhemamba/selective_gates.py:82-135, built by gate_from_spec,
    src/fhemamba/payload_surrogate.py:79-92): per head h a Chebyshev domain
    [lo_h, hi_h] and coefficient columns p[:, h], q[:, h]; for z = dt + dt_bias,
    write (the step size) = p(z)^2 q(z)^2 and decay = 1 - p(z)^2.  They replace
    the softplus and decay sites.  On ciphertexts the per-head coefficients
    are plaintext slot vectors over one shared Chebyshev basis T_1..T_D of the
    per-head affine map, zero outside the heads."""

    lo: np.ndarray
    hi: np.ndarray
    p: np.ndarray  # (degree + 1, heads)
    q: np.ndarray
    rates: np.ndarray

    def _series(self, coeffs, t):
        b1 = np.zeros_like(t)
        b2 = np.zeros_like(t)
        for c in coeffs[:0:-1]:
            b1, b2 = 2.0 * t * b1 - b2 + c, b1
        return t * b1 - b2 + coeffs[0]

    def __call__(self, z):
        z = np.asarray(z, dtype=np.float64)
        t = (2.0 * z - (self.lo + self.hi)) / (self.hi - self.lo)
        p, q = self._series(self.p, t), self._series(self.q, t)
        d = p * p
        return d * q * q, 1.0 - d

    @property
    def degree(self) -> int:
        return max(self.p.shape[0], self.q.shape[0]) - 1

    @property
    def levels(self) -> int:
        # affine map, the basis, the coefficient products, p^2 and p^2 q^2
        return 1 + max(0, math.ceil(math.log2(max(1, self.degree)))) + 1 + 2

    def encrypted(self, pm, z, heads):
        """(write, decay) ciphertexts at [0, heads) from z at [0, heads)."""
        c, n = pm.cc, pm.L.slots
        a = np.zeros(n)
        b = np.zeros(n)
        a[:heads] = 2.0 / (self.hi - self.lo)
        b[:heads] = -(self.lo + self.hi) / (self.hi - self.lo)
        t = pm._mul_mask(z, a)
        if t.GetNoiseScaleDeg() >= 2:
            c.RescaleInPlace(t)
        t = c.EvalAdd(t, c.MakeCKKSPackedPlaintext(b, level=c.n_q - t.n_limbs(), scale=t.GetScalingFactor()))
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

        def series(coeffs):
            acc = None
            for i in range(1, coeffs.shape[0]):
                vec = np.zeros(n)
                vec[:heads] = coeffs[i]
                term = pm._mul_mask(T(i), vec)
                acc = term if acc is None else c.EvalAdd(acc, term)
            if acc is None:  # a constant: 0 * t carries it as a ciphertext
                acc = pm._mul_mask(t, np.zeros(n))
            if acc.GetNoiseScaleDeg() >= 2:
                c.RescaleInPlace(acc)
            const = np.zeros(n)
            const[:heads] = coeffs[0]
            return c.EvalAdd(acc, c.MakeCKKSPackedPlaintext(const, level=c.n_q - acc.n_limbs(),
                                                             scale=acc.GetScalingFactor()))

        p, q = series(self.p), series(self.q)
        d = c.EvalMult(p, p)
        if d.GetNoiseScaleDeg() >= 2:
            c.RescaleInPlace(d)
        write = c.EvalMult(d, c.EvalMult(q, q))
        ones = np.zeros(n)
        ones[:heads] = 1.0
        decay = c.EvalAdd(c.EvalNegate(d), c.MakeCKKSPackedPlaintext(ones, level=c.n_q - d.n_limbs(),
                                                                     scale=d.GetScalingFactor()))
        return write, decay


def parse_joint_gate(spec: dict, heads: int, a_log: np.ndarray) -> JointGate:
    """parse_joint_gate (native/fideslib_stage0/src/stage1_mamba2_payload.cpp:206-231)
    plus the rate check of PolyOps.mamba2_gates (src/fhemamba/ops.py:548-556)."""
    if spec.get("kind") != "shared-dissipation-factor-v1" or \
            spec.get("coefficient_layout") != "degree-major-head-minor":
        raise PayloadError("unsupported joint gate recipe")
    try:
        arr = {k: np.asarray(spec[k], dtype=np.float64) for k in ("lo", "hi", "p", "q", "rates")}
    except (KeyError, TypeError, ValueError) as e:
        raise PayloadError("invalid joint gate numeric array") from e
    if any(not np.all(np.isfinite(v)) or v.ndim != 1 for v in arr.values()):
        raise PayloadError("invalid joint gate numeric array")
    if arr["lo"].size != heads or arr["hi"].size != heads or arr["rates"].size != heads or \
            np.any(arr["lo"] >= arr["hi"]) or arr["p"].size % heads or arr["q"].size % heads or \
            not arr["p"].size or not arr["q"].size or np.any(arr["rates"] <= 0):
        raise PayloadError("joint gate needs one domain, one positive rate and whole coefficient rows per head")
    if not np.allclose(arr["rates"], np.exp(a_log), rtol=1e-6, atol=0):
        raise PayloadError("joint gate checkpoint rates differ from the layer's A")
    return JointGate(arr["lo"], arr["hi"], arr["p"].reshape(-1, heads), arr["q"].reshape(-1, heads), arr["rates"])


def _count(spec: dict, key: str, default=None) -> int:
    """A non-negative integer field of a spec (squarings, iterations)."""
    value = spec.get(key, default)
    if value is None:
        raise PayloadError(f"meta.json key not found: {key}")
    if int(value) != value or int(value) < 0 or int(value) > 64:
        raise PayloadError(f"{key} must be an integer in [0, 64]")
    return int(value)


def parse_poly_spec(spec: dict, site: str, heads: int | None = None):
    """One exported nonlinearity (parse_poly_spec,
    native/fideslib_stage0/src/stage1_mamba2_payload.cpp:153-204, and
    _poly_from_export_spec, src/fhemamba/m1_payload.py:372-408)."""
    kind = spec.get("kind")
    if kind == "scaled-goldschmidt-invsqrt-v1":
        if spec.get("final_recomputed_newton") is not True or spec.get("oracle_workspace_dtype") != "float64":
            raise PayloadError("unsupported scheduled normalization contract")
        lo, hi, seed, tol = (float(spec.get(k, float("nan"))) for k in ("lo", "hi", "seed", "tolerance"))
        if not all(math.isfinite(x) for x in (lo, hi, seed, tol)) or not (0 < lo < hi) or seed <= 0 \
                or not (0 < tol < 1):
            raise PayloadError("invalid scheduled normalization parameters")
        pairs = spec.get("coefficients")
        if not isinstance(pairs, list) or not pairs or len(pairs) > 64:
            raise PayloadError("invalid scheduled normalization coefficient list")
        for p in pairs:
            if not isinstance(p, list) or len(p) != 2 or not all(math.isfinite(float(x)) and float(x) > 0 for x in p):
                raise PayloadError("invalid scheduled normalization coefficient pair")
        if site not in NORM_SITES:
            raise PayloadError("scheduled normalization recipe used at a non-normalization site")
        return ScheduledInvSqrt(lo, hi, seed, tuple((float(a), float(b)) for a, b in pairs))
    base = None
    if "coeffs" in spec:
        coeffs = tuple(float(c) for c in spec["coeffs"])
        lo, hi = float(spec["lo"]), float(spec["hi"])
        if not coeffs or not all(math.isfinite(c) for c in coeffs) or not hi > lo:
            raise PayloadError(f"invalid polynomial for {site}")
        base = ChebSeries(coeffs, lo, hi)

    def need_base():
        if base is None:
            raise PayloadError(f"{site}: kind {kind} needs coeffs, lo and hi")
        return base

    if kind == "cheb":
        return need_base()
    if kind == "cheb-squared":
        return SquaredSeries(need_base())
    if kind == "cheb-resquared":
        mask = None
        if "head_mask" in spec:
            mask = np.asarray(spec["head_mask"], dtype=np.float64)
            if heads is not None and mask.size != heads:
                raise PayloadError("decay_exp head_mask must contain one value per head")
            if np.any((mask != 0.0) & (mask != 1.0)):
                raise PayloadError("decay_exp head_mask values must be zero or one")
        return ResquaredExp(need_base(), _count(spec, "squarings", 0), mask)
    if kind == "const-newton":
        guess = float(spec["guess"])
        if guess <= 0.0:
            raise PayloadError("const-newton guess must be positive")
        return ConstNewton(guess, _count(spec, "iterations"))
    if kind == "poly-newton":
        return PolyNewton(need_base(), _count(spec, "iterations"))
    if kind == "sq-poly-newton":
        damping = float(spec["damping"])
        if not 0.0 < damping <= 1.0:
            raise PayloadError("sq-poly-newton damping must be in (0, 1]")
        return SquaredPolyNewton(need_base(), _count(spec, "iterations"), damping)
    raise PayloadError(f"unsupported exported polynomial kind: {kind}")


# ---------------------------------------------------------------------------
# payload


@dataclass
class PayloadWeights:
    """One layer's weights under the names the encrypted layer reads
    (norm_w, w_in, conv_w, conv_b, dt_bias, a = -exp(a_log), d, gn_w, w_out)."""

    d_model: int
    d_state: int
    heads: int
    head_dim: int
    d_inner: int
    conv_kernel: int
    conv_dim: int
    eps: float
    gated_eps: float
    arrays: dict = field(default_factory=dict)

    @property
    def proj_dim(self) -> int:
        return self.d_inner + self.conv_dim + self.heads

    def __getitem__(self, k):
        return self.arrays[k]


@dataclass
class PayloadPolys:
    """The six sites under the encrypted layer's names."""

    silu_x: object   # conv_silu
    silu_z: object   # gate_silu
    softplus: object  # dt_softplus
    exp: object      # decay_exp
    rsqrt1: object   # rms_invsqrt (block norm)
    rsqrt2: object   # gated_rms_invsqrt
    gates: object = None  # JointGate (joint format): replaces softplus and exp


@dataclass
class LayerPayload:
    index: int
    weights: PayloadWeights
    polys: PayloadPolys
    carried: dict
    tensors: dict


@dataclass
class ChainPayload:
    path: Path
    n_layers: int
    n_test_tokens: int
    layers: list
    final_norm_w: np.ndarray
    final_norm_eps: float
    final_norm: object
    input_embeddings: np.ndarray
    expected_final: np.ndarray
    expected_poly_final: np.ndarray | None
    test_token_ids: list | None = None
    autoregressive: dict | None = None
    client_embedding_w: np.ndarray | None = None
    client_lm_head_w: np.ndarray | None = None
    client_lm_head_b: np.ndarray | None = None
    ar_embeddings: np.ndarray | None = None
    ar_expected_poly_final: np.ndarray | None = None
    ar_expected_exact_final: np.ndarray | None = None
    chain_mode: bool = True  # False: one m1 layer payload (--input), no final norm

    @property
    def d_model(self) -> int:
        return self.layers[0].weights.d_model

    @property
    def full_chain(self) -> bool:
        return self.chain_mode and len(self.layers) == self.n_layers


def _read_json(path: Path) -> dict:
    try:
        return json.loads(path.read_text())
    except OSError as e:
        raise PayloadError(f"failed to open {path}") from e


def _tensor(dirpath: Path, name: str, shape) -> np.ndarray:
    """<name>.bin as float32 little endian with the manifest's shape (read_bin_tensor)."""
    path = dirpath / f"{name}.bin"
    try:
        raw = np.fromfile(path, dtype="<f4")
    except OSError as e:
        raise PayloadError(f"failed to open {path}") from e
    shape = [int(s) for s in shape]
    count = int(np.prod(shape)) if shape else 1
    if raw.size != count:
        raise PayloadError(f"tensor size mismatch for {name}: expected {count} values, {path} holds {raw.size}")
    return raw.reshape(shape).astype(np.float64)


_LAYER_TENSORS = ("in_proj_w", "conv_w", "conv_b", "dt_bias", "a_log", "d_skip", "block_norm_w", "gated_norm_w",
                  "out_proj_w", "test_layer_input", "test_layer_output")
_LAYER_OPTIONAL = ("test_layer_output_poly", "test_state_output", "test_state_output_poly",
                   "autoregressive_poly_layer_output", "autoregressive_poly_state_output",
                   "autoregressive_poly_decay_output", "autoregressive_poly_state_update",
                   "autoregressive_poly_state_decayed")


def read_layer_payload(dirpath, index: int = 0) -> LayerPayload:
    """One ``layer_XX/`` directory (read_m1_payload, stage1_mamba2_payload.cpp:233-402)."""
    d = Path(dirpath)
    meta = _read_json(d / "meta.json")
    fmt = meta.get("format")
    joint = fmt == JOINT_LAYER_FORMAT
    if not joint and fmt != LAYER_FORMAT:
        raise PayloadError("unexpected payload format (want fhemamba-m1-v1)")
    if not joint and "joint_gates" in meta:
        raise PayloadError("joint gate payload requires the versioned joint format")
    if joint and "joint_gates" not in meta:
        raise PayloadError("meta.json key not found: joint_gates")
    try:
        dims = {k: int(meta["dims"][k]) for k in ("d_model", "d_inner", "num_heads", "head_dim", "state_size",
                                                   "n_groups", "conv_kernel", "conv_dim")}
        eps_block, eps_gated = float(meta["eps"]["block_norm"]), float(meta["eps"]["gated_norm"])
        specs = meta["polys"]
        manifest = meta["tensors"]
        if meta.get("dtype", "float32-le") != "float32-le":
            raise PayloadError("tensor dtype must be float32-le")
    except KeyError as e:
        raise PayloadError(f"meta.json key not found: {e.args[0]}") from e
    H = dims["num_heads"]
    sites = {}
    for name in SITES:
        if name not in specs:
            raise PayloadError(f"meta.json key not found: {name}")
        sites[name] = parse_poly_spec(specs[name], name, H)
    tensors = {}
    for name in _LAYER_TENSORS:
        if name not in manifest:
            raise PayloadError(f"meta.json key not found: {name}")
        tensors[name] = _tensor(d, name, manifest[name])
    for name in _LAYER_OPTIONAL:
        if name in manifest:
            tensors[name] = _tensor(d, name, manifest[name])
    for name in ("test_state_output", "test_state_output_poly", "autoregressive_poly_state_output",
                 "autoregressive_poly_state_update", "autoregressive_poly_state_decayed"):
        if name in tensors:
            s = tensors[name].shape
            ar = name.startswith("autoregressive_poly_")
            if len(s) != 4 or s[0] < 1 or (not ar and s[0] > int(meta.get("n_test_tokens", s[0]))) \
                    or s[1:] != (H, dims["head_dim"], dims["state_size"]):
                raise PayloadError(f"{name} shape must be (tokens, heads, head_dim, state_size)")
    proj_dim = tensors["in_proj_w"].shape[0]
    if proj_dim != dims["d_inner"] + dims["conv_dim"] + H:
        raise PayloadError("in_proj packing with d_mlp != 0 is not supported")
    if dims["d_inner"] != H * dims["head_dim"]:
        raise PayloadError("d_inner must equal num_heads * head_dim")
    if dims["n_groups"] != 1:
        raise PayloadError("only n_groups == 1 payloads are supported")
    if dims["conv_dim"] != dims["d_inner"] + 2 * dims["state_size"]:
        raise PayloadError("conv_dim must equal d_inner + 2 * state_size")
    expect = {"in_proj_w": (proj_dim, dims["d_model"]), "conv_w": (dims["conv_dim"], dims["conv_kernel"]),
              "conv_b": (dims["conv_dim"],), "dt_bias": (H,), "a_log": (H,), "d_skip": (H,),
              "block_norm_w": (dims["d_model"],), "gated_norm_w": (dims["d_inner"],),
              "out_proj_w": (dims["d_model"], dims["d_inner"])}
    for name, shape in expect.items():
        if tensors[name].shape != shape:
            raise PayloadError(f"{name} shape {tensors[name].shape} does not match the dims {shape}")
    limit = meta.get("time_step_limit", [0.0, float("inf")])
    if float(limit[0]) > 0.0 or math.isfinite(float(limit[1])):
        raise PayloadError("finite Mamba-2 time_step_limit is not supported")
    W = PayloadWeights(d_model=dims["d_model"], d_state=dims["state_size"], heads=H, head_dim=dims["head_dim"],
                       d_inner=dims["d_inner"], conv_kernel=dims["conv_kernel"], conv_dim=dims["conv_dim"],
                       eps=eps_block, gated_eps=eps_gated)
    W.arrays = {"norm_w": tensors["block_norm_w"], "w_in": tensors["in_proj_w"], "conv_w": tensors["conv_w"],
                "conv_b": tensors["conv_b"], "dt_bias": tensors["dt_bias"], "a": -np.exp(tensors["a_log"]),
                "d": tensors["d_skip"], "gn_w": tensors["gated_norm_w"], "w_out": tensors["out_proj_w"]}
    gates = None
    if joint:
        gates = parse_joint_gate(meta["joint_gates"], H, tensors["a_log"])
        mask = sites["decay_exp"].head_mask if isinstance(sites["decay_exp"], ResquaredExp) else None
        if mask is not None and np.any(mask != 1.0):
            raise PayloadError("joint gates retain all heads")
    P = PayloadPolys(silu_x=sites["conv_silu"], silu_z=sites["gate_silu"], softplus=sites["dt_softplus"],
                     exp=sites["decay_exp"], rsqrt1=sites["rms_invsqrt"], rsqrt2=sites["gated_rms_invsqrt"],
                     gates=gates)
    for name in ("silu_x", "silu_z", "softplus", "exp"):
        if isinstance(getattr(P, name), _InvSqrt):
            raise PayloadError(f"an inverse square root is not a valid {name} nonlinearity")
    for name in ("rsqrt1", "rsqrt2"):
        if not isinstance(getattr(P, name), _InvSqrt):
            raise PayloadError("normalization sites need a Newton or scheduled inverse square root")
    carried = meta.get("carried_bounds") or {}
    if carried.get("source") != "calibration_text":
        carried = {}  # bounds without independent-calibration provenance are not used
    return LayerPayload(index=index, weights=W, polys=P, carried=carried, tensors=tensors)


def read_chain_payload(dirpath, max_layers: int = 0, autoregressive: bool = True) -> ChainPayload:
    """``chain.json`` plus its first ``max_layers`` layers (0: all), as
    read_chain_payload (stage1_mamba2_payload.cpp:428-528) and the decode's
    layer loading (stage1_mamba2_decode_fideslib.cpp:765-800) do."""
    d = Path(dirpath)
    meta = _read_json(d / "chain.json")
    if meta.get("format") not in (CHAIN_FORMAT, JOINT_CHAIN_FORMAT):
        raise PayloadError("unexpected chain payload format (want fhemamba-m2-chain-v1)")
    n_layers = int(meta["n_layers"])
    dirs = meta.get("layer_dirs") or []
    if n_layers <= 0 or len(dirs) != n_layers:
        raise PayloadError("chain.json layer_dirs does not match n_layers")
    final_spec = None
    if "final_norm_poly" in meta:
        final_spec = parse_poly_spec(meta["final_norm_poly"], "rms_invsqrt")
        if not isinstance(final_spec, ScheduledInvSqrt):
            raise PayloadError("dedicated final norm requires a scheduled normalization recipe")
    manifest = meta["tensors"]
    if meta.get("dtype", "float32-le") != "float32-le":
        raise PayloadError("tensor dtype must be float32-le")
    for name in ("final_norm_w", "chain_input_embeddings", "chain_expected_final"):
        if name not in manifest:
            raise PayloadError(f"chain.json key not found: {name}")
    count = n_layers if max_layers <= 0 else min(max_layers, n_layers)
    layers = [read_layer_payload(d / dirs[i], i) for i in range(count)]
    first = layers[0].weights
    for i, L in enumerate(layers[1:], 1):
        w = L.weights
        if (w.d_model, w.d_inner, w.heads, w.head_dim, w.d_state, w.conv_kernel, w.conv_dim) != \
                (first.d_model, first.d_inner, first.heads, first.head_dim, first.d_state, first.conv_kernel,
                 first.conv_dim):
            raise PayloadError(f"chain layer payload dims mismatch at index {i}")
    if final_spec is None and count == n_layers and isinstance(layers[-1].polys.rsqrt1, ScheduledInvSqrt):
        raise PayloadError("scheduled normalization requires a dedicated final_norm_poly")
    D = first.d_model
    emb = _tensor(d, "chain_input_embeddings", manifest["chain_input_embeddings"])
    exp_final = _tensor(d, "chain_expected_final", manifest["chain_expected_final"])
    poly_final = (_tensor(d, "chain_expected_poly_final", manifest["chain_expected_poly_final"])
                  if "chain_expected_poly_final" in manifest else None)
    n_test = int(meta["n_test_tokens"])
    for name, arr in (("chain_input_embeddings", emb), ("chain_expected_final", exp_final),
                      ("chain_expected_poly_final", poly_final)):
        if arr is not None and arr.shape != (n_test, D):
            raise PayloadError(f"{name} shape must be (n_test_tokens, d_model)")
    chain = ChainPayload(path=d, n_layers=n_layers, n_test_tokens=n_test, layers=layers,
                         final_norm_w=_tensor(d, "final_norm_w", manifest["final_norm_w"]),
                         final_norm_eps=float(meta["final_norm_eps"]),
                         final_norm=final_spec if final_spec is not None else layers[-1].polys.rsqrt1,
                         input_embeddings=emb, expected_final=exp_final, expected_poly_final=poly_final,
                         test_token_ids=meta.get("test_token_ids"))
    ar = meta.get("autoregressive")
    if isinstance(ar, dict):
        if ar.get("protocol") != "client-in-loop-greedy-v1":
            raise PayloadError("unsupported autoregressive payload protocol")
        chain.autoregressive = ar
        if autoregressive:
            chain.client_embedding_w = _tensor(d, "client_embedding_w", manifest["client_embedding_w"])
            if chain.client_embedding_w.ndim != 2:
                raise PayloadError("client_embedding_w must be rank 2")
            if "client_lm_head_w" in manifest:
                chain.client_lm_head_w = _tensor(d, "client_lm_head_w", manifest["client_lm_head_w"])
            if "client_lm_head_b" in manifest:
                chain.client_lm_head_b = _tensor(d, "client_lm_head_b", manifest["client_lm_head_b"])
            chain.ar_embeddings = _tensor(d, "autoregressive_poly_embeddings",
                                          manifest["autoregressive_poly_embeddings"])
            chain.ar_expected_poly_final = _tensor(d, "autoregressive_poly_expected_final",
                                                   manifest["autoregressive_poly_expected_final"])
            chain.ar_expected_exact_final = _tensor(d, "autoregressive_exact_expected_final",
                                                    manifest["autoregressive_exact_expected_final"])
    return chain


def read_layer_as_chain(dirpath) -> ChainPayload:
    """One m1 layer payload as the decode's single-layer mode reads it
    (``--input``, stage1_mamba2_decode_fideslib.cpp:781-783): the layer's test
    inputs in, its test outputs as the reference, no final norm."""
    L = read_layer_payload(dirpath, 0)
    t = L.tensors
    return ChainPayload(path=Path(dirpath), n_layers=1, n_test_tokens=t["test_layer_input"].shape[0], layers=[L],
                        final_norm_w=np.zeros(0), final_norm_eps=0.0, final_norm=L.polys.rsqrt1,
                        input_embeddings=t["test_layer_input"], expected_final=t["test_layer_output"],
                        expected_poly_final=t.get("test_layer_output_poly"), chain_mode=False)


# ---------------------------------------------------------------------------
# plaintext polynomial circuit (what chain_expected_poly_final records)


def initial_state(payload: ChainPayload):
    """Zero conv FIFO and no recurrent state (init_states, src/fhemamba/reference.py:42-44)."""
    return [([np.zeros(L.weights.conv_dim) for _ in range(L.weights.conv_kernel - 1)], None)
            for L in payload.layers]


def plain_token(payload: ChainPayload, h, state, rec=None):
    """One token through the loaded layers in fp64 with the payload's
    nonlinearities (model_forward with PolyOps, src/fhemamba/reference.py:300-339
    and mixer2_forward :182-294), then the final RMSNorm when the chain is
    complete.  rec(layer, key, values) observes every refreshed intermediate
    (layer = len(layers) for the final norm).  Returns (output, new state)."""
    new = []
    for L, (conv, st) in zip(payload.layers, state):
        r = (lambda k, v, i=L.index: rec(i, k, v)) if rec else (lambda k, v: None)
        h, conv, st = poly_step_record(L.weights, L.polys, h, conv, st, r)
        new.append((conv, st))
    if payload.full_chain:
        i = len(payload.layers)
        r = (lambda k, v: rec(i, k, v)) if rec else None
        if rec:
            rec(i, "h", h)
        h = plain_rms(h, payload.final_norm_w, payload.final_norm_eps, payload.final_norm, rec=r, key="nf")
    return h, new


def plain_decode(payload: ChainPayload, embeddings, rec=None):
    """The polynomial circuit over a sequence of input embeddings (state carried from zero)."""
    state = initial_state(payload)
    out = []
    for e in np.asarray(embeddings, dtype=np.float64):
        h, state = plain_token(payload, e, state, rec)
        out.append(h)
    return np.array(out)


def _carried_keys(carried: dict):
    """(refresh-bound key, value) pairs from a layer's calibration-text bounds.
    The exporter's ``y`` checkpoint is the gated value y * silu(z)
    (mixer2_forward, src/fhemamba/reference.py:290), ``g`` here."""
    cp = carried.get("checkpoint_abs_max", {}) or {}
    pairs = [("h", cp.get("residual")), ("proj", cp.get("proj")), ("pack", cp.get("conv_silu")),
             ("pack", cp.get("dt")), ("g", cp.get("y")), ("xbc", carried.get("fifo_abs_max")),
             ("state", carried.get("state_abs_max"))]
    return [(k, float(v)) for k, v in pairs if v is not None]


# Fallback magnitudes for refresh sites the payload gives no number for (the
# reference decode's checkpoint_bound table,
# native/fideslib_stage0/src/stage1_mamba2_decode_fideslib.cpp:174-214).
FALLBACK_BOUNDS = {"h": 8.0, "proj": 6.0, "xbc": 6.0, "y": 24.0, "state": 24.0}


def calibration_sequences(payload: ChainPayload, count: int = 8, length: int = 4, seed: int = 0):
    """Seeded random token sequences embedded with the payload's client
    embedding table (present with the client-loop assets), or none."""
    if payload.client_embedding_w is None:
        return []
    r = np.random.default_rng(seed)
    vocab = payload.client_embedding_w.shape[0]
    return [payload.client_embedding_w[r.integers(0, vocab, length)] for _ in range(count)]


def _inv_sqrt_domain(spec):
    if isinstance(spec, ScheduledInvSqrt):
        lo, hi = spec.lo, spec.hi
    elif isinstance(spec, ConstNewton):
        lo, hi = 0.01 * spec.fill, spec.fill
    else:
        lo, hi = spec.base.lo, spec.base.hi
    return (lo if lo > 0 else 1e-4 * hi), hi


def domain_bounds(L: LayerPayload | None, norms) -> dict:
    """Magnitudes that follow from the exported domains alone: activation
    inputs within their fitted intervals, activation outputs over them, every
    inverse-square-root iterate over its variance interval (and the fill),
    normalised vectors at most sqrt(width) x max |weight|."""
    out = {}

    def put(k, v):
        out[k] = max(out.get(k, 0.0), float(np.max(np.abs(v))))

    if L is not None:
        P, W = L.polys, L.weights
        put("xc", [P.silu_x.lo, P.silu_x.hi])
        put("z", [P.silu_z.lo, P.silu_z.hi])
        xa = P.silu_x(np.linspace(P.silu_x.lo, P.silu_x.hi, 513))
        put("xa", xa)
        put("pack", xa)
        out["silu_z_max"] = float(np.max(np.abs(P.silu_z(np.linspace(P.silu_z.lo, P.silu_z.hi, 513)))))
        if P.gates is not None:
            g = P.gates
            put("dt", [g.lo, g.hi])
            write, decay = g(g.lo[None, :] + np.linspace(0.0, 1.0, 257)[:, None] * (g.hi - g.lo)[None, :])
            put("dts", write)
            put("pack", write)
            put("pack", decay)
        else:
            b = P.softplus.base
            put("dt", [b.lo, b.hi])
            dts = P.softplus(np.linspace(b.lo, b.hi, 513))
            put("dts", dts)
            put("pack", dts)
            put("adt", [P.exp.lo])
            put("pack", 1.0)
        put("u", math.sqrt(W.d_model) * np.max(np.abs(W["norm_w"])))
        put("gn", math.sqrt(W.d_inner) * np.max(np.abs(W["gn_w"])))
    for prefix, spec in norms:
        lo, hi = _inv_sqrt_domain(spec)
        v = np.concatenate([np.geomspace(lo, hi, 257), [spec.fill]])
        put(prefix + "_v", v)
        spec.inv_sqrt(v, trace=lambda name, val, pre=prefix: put(pre + "_" + name, val))
    return out


def chain_bounds(payload: ChainPayload, sequences=None, margin: float = 2.0):
    """Refresh bounds per layer (and for the final norm, index len(layers)),
    as the reference decode derives them: never from the inputs it is tested
    on.  Per refreshed intermediate, `margin` x the largest of

    * its magnitude in the fp64 circuit over calibration `sequences` (default:
      seeded random token sequences from the client embedding table, when the
      payload has one) and in the layer's calibration-text carried bounds;
    * for activation inputs and outputs, their extent over the exported
      polynomial domains;

    and, for a site none of these reaches, its domain-derived magnitude
    (inverse-square-root iterates, normalised vectors, the gated value from
    the carried gated-variance range) or the reference's fallback constant.  There is no floor: a refresh's error is relative to
    its bound, and small values (the gated variance, the first steps of a
    scheduled inverse square root) keep their precision only under a bound of
    their own size."""
    if sequences is None:
        sequences = calibration_sequences(payload)
    n = len(payload.layers)
    mags = [dict() for _ in range(n + 1)]

    def rec(i, k, v):
        m = mags[i]
        m[k] = max(m.get(k, 0.0), float(np.max(np.abs(v))))

    for seq in sequences:
        plain_decode(payload, seq, rec)
    for L, m in zip(payload.layers, mags):
        for k, v in _carried_keys(L.carried):
            m[k] = max(m.get(k, 0.0), v)
        dom = domain_bounds(L, [("n1", L.polys.rsqrt1), ("n2", L.polys.rsqrt2)])
        for k in ("xc", "z", "dt", "adt", "xa", "dts", "pack"):
            if k in dom:
                m[k] = max(m.get(k, 0.0), dom[k])
        for k, v in dom.items():
            if k != "silu_z_max":
                m.setdefault(k, v)
        for k, v in FALLBACK_BOUNDS.items():
            m.setdefault(k, v)
        gv = L.carried.get("gated_variance_range")
        if "g" not in m and gv:  # mean(g^2) <= var_hi gives |g_i| <= sqrt(width var_hi)
            m["g"] = math.sqrt(L.weights.d_inner * float(gv[1]))
        m.setdefault("g", m["y"] * dom["silu_z_max"])
    if payload.full_chain:
        final = mags[n]
        last = payload.layers[-1].carried.get("checkpoint_abs_max", {}) or {}
        if last.get("output") is not None:
            final["h"] = max(final.get("h", 0.0), float(last["output"]))
        for k, v in domain_bounds(None, [("nf", payload.final_norm)]).items():
            final.setdefault(k, v)
        final.setdefault("h", FALLBACK_BOUNDS["h"])
    return [{k: max(1e-9, margin * v) for k, v in m.items()} for m in mags]


# ---------------------------------------------------------------------------
# encrypted decode


CARRIED_SITES = ("xbc", "state")


def meta_bts_policy(layer: int, enabled: bool, residual_layers=(), scheduled: bool = False):
    """Refresh pass count per site of one layer under the reference decode's
    Meta-BTS selection (should_use_meta_bts,
    native/fideslib_stage0/src/stage1_mamba2_config.cpp:69-86): a refresh
    is two-pass (Meta-BTS, residual amplified by 2^12) for every transient
    value of a layer with a scheduled normalization, and with Meta-BTS enabled
    for the carried values (conv FIFO ``xbc`` and recurrent ``state``), the
    gated norm's polynomial input (``gated_poly_input`` there; here the gated
    value ``g`` refreshed before its variance is taken, and the variance
    ``n2_v``) and the layer's residual input (``h``) at the selected layers;
    every other refresh is one bootstrap."""
    residual_layers = frozenset(residual_layers)

    def passes(site):
        site = site or ""
        if scheduled and site not in CARRIED_SITES:
            return 2
        if not enabled:
            return 1
        if site in CARRIED_SITES or site in ("g", "n2_v"):
            return 2
        return 2 if site == "h" and layer in residual_layers else 1

    return passes


class EncryptedChain:
    """The payload's layers on one CryptoContext: the client encrypts a token's
    embedding, every loaded layer runs on ciphertexts (EncryptedMamba2Layer with
    the payload's weights and nonlinearities, state and conv FIFO carried), and
    a complete chain ends with the final RMSNorm (the reference's run_layer loop
    and final_norm, stage1_mamba2_decode_fideslib.cpp:3634-4520)."""

    def __init__(self, cc, payload: ChainPayload, passes: int = 2, cache_gb: float = 8.0, bounds=None,
                 meta_bts: bool | None = None, meta_bts_residual_layers=(), rotation_keys: str = "full",
                 rotation_key_gib: float = 45.0):
        """passes: every refresh's pass count (2: each refresh is Meta-BTS), or,
        with meta_bts set (True / False), the reference's selective policy.
        rotation_keys: full | compact | balanced key plan (rotation_keys.py),
        balanced under rotation_key_gib GiB of rotation keys."""
        self.cc, self.p = cc, payload
        self.cache = PlaintextCache(cache_gb * 2 ** 30)

        def policy(L):
            if meta_bts is None:
                return passes
            scheduled = isinstance(L.polys.rsqrt1, ScheduledInvSqrt) or isinstance(L.polys.rsqrt2, ScheduledInvSqrt)
            return meta_bts_policy(L.index, meta_bts, meta_bts_residual_layers, scheduled)

        self.layers = [EncryptedMamba2Layer(cc, L.weights, L.polys, passes=policy(L), cache=self.cache)
                       for L in payload.layers]
        self.bounds = bounds if bounds is not None else chain_bounds(payload)
        self.plan = None
        if rotation_keys != "full":
            from .rotation_keys import ComposedRotations, key_bytes, plan_keys
            steps, required = set(), set()
            for layer in self.layers:
                steps |= set(layer.rotation_steps())
                required |= set(layer.transform_steps())
            per_key = key_bytes(cc.n, cc.n_q + cc.n_p, cc.dnum)
            self.plan = plan_keys({s: 1.0 for s in steps}, cc.slots, rotation_keys, rotation_key_gib * 2 ** 30,
                                  per_key, required)
            self.cc = ComposedRotations(cc, self.plan)
            for layer in self.layers:
                layer.cc = layer.pm.cc = self.cc
        self.reset()

    def reset(self):
        self.state = [([None] * (L.weights.conv_kernel - 1), None) for L in self.p.layers]

    def rotation_steps(self):
        """The rotation keys to generate (the plan's, under a key plan)."""
        if self.plan is not None:
            return sorted(k % self.cc.slots for k in self.plan.keys)
        s = set()
        for layer in self.layers:
            s |= set(layer.rotation_steps())
        return sorted(s)

    def refreshes(self) -> int:
        return sum(layer.refreshes for layer in self.layers)

    def two_pass_refreshes(self) -> int:
        return sum(layer.two_pass_refreshes for layer in self.layers)

    def encrypt(self, embedding):
        """Client: the token's embedding at slots [0, d_model)."""
        c, D = self.cc, self.p.d_model
        return c.Encrypt(c.MakeCKKSPackedPlaintext(np.pad(np.asarray(embedding, dtype=np.float64), (0, c.slots - D))))

    def step(self, embedding):
        """One token from its embedding (client encryption + server pass)."""
        return self.step_ct(self.encrypt(embedding))

    def step_ct(self, h, on_layer=None):
        """Server pass for one encrypted token: the encrypted final hidden
        vector (the last loaded layer's output when max_layers cuts the chain).
        on_layer(i, ct) sees every layer's output (debug attribution)."""
        c, D = self.cc, self.p.d_model
        new = []
        for i, (layer, (conv, st), bounds) in enumerate(zip(self.layers, self.state, self.bounds)):
            h, conv, st = layer.step(h, conv, st, bounds)
            new.append((conv, st))
            if on_layer is not None:
                on_layer(i, h)
        self.state = new
        if not self.p.full_chain:
            return h
        last = self.layers[-1]
        return last._rms(h, D, self.p.final_norm_w, self.p.final_norm, self.bounds[-1], "h", "nf",
                         self.p.final_norm_eps)

    def decrypt(self, ct):
        return self.cc.Decrypt(ct).GetRealPackedValue()[:self.p.d_model]


def select_token(payload: ChainPayload, hidden) -> int:
    """Client greedy selection over the (tied or untied) LM head
    (stage1_mamba2_decode_fideslib.cpp:4551-4575)."""
    head = payload.client_lm_head_w if payload.client_lm_head_w is not None else payload.client_embedding_w
    logits = head @ hidden
    if payload.client_lm_head_b is not None:
        logits = logits + payload.client_lm_head_b
    if not np.all(np.isfinite(logits)):
        raise PayloadError("non-finite autoregressive client logit")
    return int(np.argmax(logits))


def run_chain(cc, payload: ChainPayload, tokens: int, tolerance: float = 5e-2,
              autoregressive_client_loop: bool = False, passes: int = 2, cache_gb: float = 8.0,
              meta_bts: bool | None = None, meta_bts_residual_layers=(), debug_layer_errors: bool = False,
              rotation_keys: str = "full", rotation_key_gib: float = 45.0):
    """The decode's chain mode: encrypt each test (or client-selected) token's
    embedding, evaluate, decrypt, and compare with the polynomial-circuit
    reference (``chain_expected_poly_final``, or the last layer's
    ``test_layer_output_poly`` when max_layers cuts the chain) and with the
    exact model.  `cc` holds the secret, relinearisation and bootstrapping
    keys; the layers' rotation keys are generated here.  debug_layer_errors
    also decrypts every layer's output and compares it with that layer's
    polynomial reference (the decode's --debug-layer-errors).  Returns the
    result document of the reference's decode (stage1_mamba2_decode_fideslib.cpp:
    4823-5060, the fields this backend has)."""
    p = payload
    if tokens < 1:
        raise PayloadError("--tokens must be positive")
    if autoregressive_client_loop:
        if p.autoregressive is None:
            raise PayloadError("autoregressive-client-loop requested but payload has no assets")
        if not p.full_chain:
            raise PayloadError("autoregressive-client-loop requires the full layer chain")
        if p.ar_embeddings is None:
            raise PayloadError("autoregressive assets were not loaded")
        if tokens > int(p.autoregressive["server_evaluations"]):
            raise PayloadError("--tokens exceeds the payload's autoregressive server evaluations")
        poly_ref, exact_ref = p.ar_expected_poly_final, p.ar_expected_exact_final
        prompt = int(p.autoregressive["prompt_tokens"])
        expected_ids = list(p.autoregressive["poly_generated_ids"])[:max(0, tokens - prompt + 1)]
    else:
        if tokens > p.n_test_tokens:
            raise PayloadError("--tokens exceeds n_test_tokens in the chain payload")
        last = p.layers[-1].tensors
        if p.full_chain:
            poly_ref, exact_ref = p.expected_poly_final, p.expected_final
        else:
            poly_ref, exact_ref = last.get("test_layer_output_poly"), last["test_layer_output"]
        expected_ids = []
    has_poly = poly_ref is not None
    reference = poly_ref if has_poly else exact_ref
    t0 = time.perf_counter()
    chain = EncryptedChain(cc, p, passes=passes, cache_gb=cache_gb, meta_bts=meta_bts,
                           meta_bts_residual_layers=meta_bts_residual_layers, rotation_keys=rotation_keys,
                           rotation_key_gib=rotation_key_gib)
    cc.EvalRotateKeyGen(chain.rotation_steps())
    setup = time.perf_counter() - t0
    per_token, per_token_exact, ok, selected, outputs, per_layer = [], [], [], [], [], []
    next_embedding = None
    t1 = time.perf_counter()
    for t in range(tokens):
        if autoregressive_client_loop:
            emb = p.ar_embeddings[t] if t < prompt or next_embedding is None else next_embedding
        else:
            emb = p.input_embeddings[t]
        layer_errors = []

        def on_layer(i, ct, t=t):
            key = "autoregressive_poly_layer_output" if autoregressive_client_loop else "test_layer_output_poly"
            ref = p.layers[i].tensors.get(key)
            if ref is not None and t < ref.shape[0]:
                layer_errors.append(float(np.max(np.abs(chain.decrypt(ct) - ref[t]))))

        got = chain.decrypt(chain.step_ct(chain.encrypt(emb), on_layer if debug_layer_errors else None))
        if debug_layer_errors:
            per_layer.append(layer_errors)
        outputs.append(got)
        finite = bool(np.all(np.isfinite(got)))
        ok.append(int(finite))
        per_token.append(float(np.max(np.abs(got - reference[t]))) if finite else float("inf"))
        per_token_exact.append(float(np.max(np.abs(got - exact_ref[t]))) if finite else float("inf"))
        if autoregressive_client_loop and t >= prompt - 1:
            sel = select_token(p, got)
            selected.append(sel)
            next_embedding = p.client_embedding_w[sel]
    seconds = time.perf_counter() - t1
    max_error = max(per_token)
    tokens_match = (not autoregressive_client_loop) or selected == expected_ids
    passed = max_error <= tolerance and tokens_match
    w = p.layers[0].weights
    return {
        "schema": "fhemamba-stage1-mamba2-result-v1",
        "backend": "fhe_b200",
        "status": "passed" if passed else "failed",
        "passed": passed,
        "parameters": {"d_model": w.d_model, "d_inner": w.d_inner, "num_heads": w.heads, "head_dim": w.head_dim,
                       "state_size": w.d_state, "n_groups": 1, "conv_kernel": w.conv_kernel,
                       "conv_dim": w.conv_dim, "proj_dim": w.proj_dim, "layers": len(p.layers),
                       "chain_layers": p.n_layers, "tokens": tokens, "ring_dim": cc.n, "slots": cc.slots,
                       "autoregressive_client_loop": autoregressive_client_loop, "tolerance": tolerance,
                       "refresh_passes": passes if meta_bts is None else None, "meta_bts": meta_bts,
                       "meta_bts_alpha": 12, "meta_bts_residual_layers": sorted(meta_bts_residual_layers)},
        "measurements": {
            "correctness_reference": "polynomial-circuit" if has_poly else "exact-legacy",
            "max_abs_error": max_error,
            "per_token_max_abs_error": per_token,
            "max_abs_error_vs_exact": max(per_token_exact),
            "per_token_max_abs_error_vs_exact": per_token_exact,
            "per_token_decrypt_ok": ok,
            "autoregressive_selected_ids": selected,
            "autoregressive_expected_ids": expected_ids,
            "autoregressive_tokens_match": tokens_match,
            "token0_decrypted_sample": [float(v) for v in outputs[0][:8]],
            "token0_expected_sample": [float(v) for v in reference[0][:8]],
            "token0_exact_sample": [float(v) for v in exact_ref[0][:8]],
            "refreshes": chain.refreshes(),
            "meta_bts_applied": chain.two_pass_refreshes(),
            "per_token_layer_max_abs_error": per_layer if debug_layer_errors else None,
            "rotation_keys": len(chain.rotation_steps()),
            "rotation_key_plan": chain.plan.stats if chain.plan is not None else {"mode": "full"},
            "composite_rotation_applications": getattr(chain.cc, "composite_applications", 0),
            "setup_seconds": setup,
            "decode_seconds": seconds,
            "seconds_per_token": seconds / tokens,
        },
    }
