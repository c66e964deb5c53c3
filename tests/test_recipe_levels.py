"""Depth parity with the reference: the levels each nonlinearity recipe of
the Mamba-2 decode consumes here, against the levels the reference recorded
for the same recipe (degree, interval, squarings, Newton iterations) in its
OpenFHE runs (tests/golden/ckks_recipe_levels.json, extracted from its
tests/fixtures/ckks-recipes.json).  The evaluation is the chain payload's
(chain_payload.py) on the slot-level model of the CryptoContext API, whose
level accounting is the device library's (the same model reproduces the
device's 236 bootstraps per token of the token loop).  The layer's slot
masks (the affine map and the output mask of `PackedMamba2.poly`) are layout
costs outside these recipes.  No GPU."""
import json
import os

import numpy as np
import pytest

from conftest import GOLDEN
from fhe_mamba_b200.chain_payload import (ChebSeries, PolyNewton, ResquaredExp, SquaredPolyNewton,
                                          SquaredSeries)
from fhe_mamba_b200.mamba2_layer import _silu, _softplus, cheb_fit
from slot_sim import SlotContext

with open(os.path.join(GOLDEN, "ckks_recipe_levels.json")) as f:
    RECIPES = {r["name"]: r for r in json.load(f)["recipes"]}


def _series(fn, lo, hi, degree):
    return ChebSeries(tuple(cheb_fit(fn, lo, hi, degree)), lo, hi)


def _spec(r):
    lo, hi = r["interval"]
    d = r["degree"]
    name = r["name"]
    if name.startswith("ps_cheb_silu"):
        return _series(_silu, lo, hi, d)
    if name.startswith("sqrt_softplus"):
        return SquaredSeries(_series(lambda t: np.sqrt(_softplus(t)), lo, hi, d))
    if name.startswith("squared_exp"):
        k = 2 ** r["squarings"]
        return ResquaredExp(_series(np.exp, lo / k, hi / k, d), r["squarings"])
    if name.startswith("poly_newton"):
        return PolyNewton(_series(lambda t: 1 / np.sqrt(t), lo, hi, d), r["iterations"])
    if name.startswith("sq_poly_newton"):
        return SquaredPolyNewton(_series(lambda t: np.abs(t) ** -0.25, lo, hi, d), r["iterations"], r["damping"])
    raise AssertionError(name)


def _encrypted(cc, spec, ct):
    """The recipe itself, without the layer's slot masks."""
    if isinstance(spec, ChebSeries):
        return cc.EvalChebyshevSeries(ct, spec.coeffs, spec.lo, spec.hi)
    if isinstance(spec, SquaredSeries):
        y = _encrypted(cc, spec.base, ct)
        return cc.EvalMult(y, y)
    if isinstance(spec, ResquaredExp):
        k = 2.0 ** spec.squarings
        y = cc.EvalChebyshevSeries(ct, spec.base.coeffs, spec.base.lo * k, spec.base.hi * k)
        for _ in range(spec.squarings):
            y = cc.EvalMult(y, y)
        return y
    return spec.encrypted_inv_sqrt(cc, ct, lambda c, need, name: c)  # no refresh: the whole depth


def _ps_excess(degree: int) -> int:
    """Levels the device's Paterson-Stockmeyer split spends above
    ceil(log2(degree + 1)): one for the degrees just below a power of two
    (24-31, 56-63, 112-127, ...), where the top giant product sits one level
    above the weighted leaves; zero elsewhere."""
    from slot_sim import ps_depth
    return ps_depth(degree + 1) - int(np.ceil(np.log2(degree + 1)))


@pytest.mark.parametrize("name", sorted(RECIPES))
def test_recipe_depth_at_most_the_reference(name):
    """At most the reference's levels, except the one-level excess of the
    series split at degrees just below a power of two (the decay exp's 24)."""
    r = RECIPES[name]
    spec = _spec(r)
    lo, hi = r["interval"]
    x = np.linspace(lo, hi, 257) if lo < 0 else np.geomspace(lo, hi, 257)
    cc = SlotContext(512, refresh_noise=0.0)
    ct = cc.Encrypt(cc.MakeCKKSPackedPlaintext(np.pad(x, (0, 512 - x.size), constant_values=x[0])))
    out = _encrypted(cc, spec, ct)
    consumed = ct.left - out.left
    want = spec.inv_sqrt(x) if hasattr(spec, "inv_sqrt") else spec(x)
    assert np.max(np.abs(out.values.real[:x.size] - want)) <= 1e-9 * max(1.0, np.max(np.abs(want)))
    assert consumed <= r["levels_consumed"] + _ps_excess(r["degree"]), (name, consumed, r["levels_consumed"])


def test_recorded_depths():
    """The measured comparison, recipe by recipe (here, reference)."""
    got = {}
    for name, r in RECIPES.items():
        spec = _spec(r)
        cc = SlotContext(512, refresh_noise=0.0)
        ct = cc.Encrypt(cc.MakeCKKSPackedPlaintext(np.full(512, np.mean(r["interval"]))))
        got[name] = (ct.left - _encrypted(cc, spec, ct).left, r["levels_consumed"])
    assert got == {"ps_cheb_silu_deg96": (8, 8), "sqrt_softplus_sq_deg64": (9, 9),
                   "squared_exp_deg24_sq3": (10, 9), "poly_newton_invsqrt_deg47_it4": (15, 15),
                   "sq_poly_newton_invsqrt_deg31_it4": (16, 17)}
    assert _ps_excess(24) == 1 and _ps_excess(96) == 0 and _ps_excess(64) == 0 and _ps_excess(47) == 0


def test_every_recorded_recipe_is_covered():
    assert set(RECIPES) == {"ps_cheb_silu_deg96", "sqrt_softplus_sq_deg64", "squared_exp_deg24_sq3",
                            "poly_newton_invsqrt_deg47_it4", "sq_poly_newton_invsqrt_deg31_it4"}
