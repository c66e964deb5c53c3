"""The sparse ternary secret of the bootstrapping encapsulation, as the
oracle restates it (the device draws the same one, checked word for word in
tests/test_gpu_bootstrap.py): weight h, values in {-1, 0, 1}, deterministic
in the seed, different for different seeds and weights."""
import numpy as np


def _ctx(oracle):
    q, p = oracle.ckks_moduli(12, 8, 50, 55, 2)
    return oracle.Ckks(12, q, p, 2, 2048)


def test_weight_values_and_determinism(oracle):
    oc = _ctx(oracle)
    for h in (1, 32, 64, 192):
        c1, n1 = oc.sparse_secret(4321, h)
        c2, n2 = oc.sparse_secret(4321, h)
        assert np.count_nonzero(c1) == h and set(np.unique(c1)) <= {-1, 0, 1}
        assert np.array_equal(c1, c2) and np.array_equal(n1, n2)
    a, _ = oc.sparse_secret(1, 32)
    b, _ = oc.sparse_secret(2, 32)
    c, _ = oc.sparse_secret(1, 33)
    assert not np.array_equal(a, b) and not np.array_equal(a, c)


def test_ntt_form_is_the_lifted_polynomial(oracle):
    oc = _ctx(oracle)
    coef, sn = oc.sparse_secret(7, 16)
    back = oc.ntt(sn[: oc.L].copy(), oc.L, 0, inverse=True)
    for l in range(oc.L):
        q = oc.q[l]
        want = np.array([int(v) % q for v in coef], dtype=np.uint64)
        assert np.array_equal(back[l], want)
