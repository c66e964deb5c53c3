"""Paterson-Stockmeyer Chebyshev evaluation.

CPU: the recursion the device runs (baby basis by doubling products, division
by T_k for powers of two k, the reference's split formulas from
packed_fideslib.cpp:533-599) replayed on plain slot vectors equals numpy's
chebval.  GPU: the encrypted evaluation decrypts to the same polynomial within
1e-3 max-abs (SiLU, softplus, exp on declared domains, degree <= 63)."""
import numpy as np
import pytest

from fhe_mamba_b200.ckks import chebyshev_coefficients


def ps_replay(x, c, lo, hi):
    u = (2 * x - lo - hi) / (hi - lo)
    levels = 0
    while (1 << levels) < len(c):
        levels += 1
    baby = 1 << ((max(1, levels) + 1) // 2)
    cache = {1: u}

    def basis(i):
        if i not in cache:
            cache[i] = 2 * basis(i // 2) ** 2 - 1 if i % 2 == 0 else 2 * basis((i + 1) // 2) * basis(i // 2) - u
        return cache[i]

    def evaluate(cc):
        degree = len(cc) - 1
        if degree < baby:
            return sum(cc[i] * basis(i) for i in range(1, degree + 1)) + cc[0]
        k = baby
        while 2 * k - 1 < degree:
            k *= 2
        upper, lower = list(cc[k:]), list(cc[:k])
        for i in range(1, len(upper)):
            upper[i] *= 2
        for i in range(k + 1, degree + 1):
            lower[2 * k - i] -= cc[i]
        return evaluate(lower) + basis(k) * evaluate(upper)

    return evaluate(list(c))


FUNCS = {
    "silu": (lambda x: x / (1 + np.exp(-x)), -8.0, 8.0, 63),
    "softplus": (lambda x: np.log1p(np.exp(x)), -6.0, 6.0, 31),
    "exp": (np.exp, -4.0, 0.0, 15),
}


@pytest.mark.parametrize("name", sorted(FUNCS))
def test_ps_recursion_equals_chebval(name):
    f, lo, hi, deg = FUNCS[name]
    c = chebyshev_coefficients(f, lo, hi, deg)
    x = np.linspace(lo, hi, 257)
    want = np.polynomial.chebyshev.chebval((2 * x - lo - hi) / (hi - lo), c)
    assert np.allclose(ps_replay(x, c, lo, hi), want, atol=1e-9)


@pytest.mark.gpu
def test_encrypted_chebyshev_matches_polynomial():
    from fhe_mamba_b200 import CCParams, CryptoContext
    cc = CryptoContext(CCParams(ring_dim=1 << 14, multiplicative_depth=14, scaling_mod_size=50,
                                first_mod_size=60, num_large_digits=3))
    cc.KeyGen(5)
    rng = np.random.default_rng(0)
    for name in sorted(FUNCS):
        f, lo, hi, deg = FUNCS[name]
        x = rng.uniform(lo, hi, cc.slots)
        c = chebyshev_coefficients(f, lo, hi, deg)
        ct = cc.Encrypt(cc.MakeCKKSPackedPlaintext(x))
        out = cc.EvalChebyshevSeries(ct, c, lo, hi)
        got = cc.Decrypt(out).GetRealPackedValue()
        want = np.polynomial.chebyshev.chebval((2 * x - lo - hi) / (hi - lo), c)
        assert np.max(np.abs(got - want)) < 1e-3, name
        assert out.GetLevel() <= 10, (name, out.GetLevel())
