"""Oracle NTT against the O(N^2) definition (KAT fixture) and algebraic properties."""
import numpy as np

from conftest import probe_values


def test_forward_matches_definition_kat(oracle, ntt_kat):
    for a, out, q, psi in zip(ntt_kat["inputs"], ntt_kat["outputs"], ntt_kat["primes"], ntt_kat["psi"]):
        x = a.copy().reshape(1, 1, -1)
        oracle.ntt_batch(x, [int(q)], [int(psi)], inverse=False)
        assert np.array_equal(x[0, 0], out)


def test_inverse_matches_definition_kat(oracle, ntt_kat):
    for a, out, q, psi in zip(ntt_kat["inputs"], ntt_kat["outputs"], ntt_kat["primes"], ntt_kat["psi"]):
        x = out.copy().reshape(1, 1, -1)
        oracle.ntt_batch(x, [int(q)], [int(psi)], inverse=True)
        assert np.array_equal(x[0, 0], a)


def test_negacyclic_convolution(oracle):
    n = 1024
    q = oracle.ntt_primes(10, 59, 1)[0]
    psi = oracle.root_of_unity(2 * n, q)
    rng = np.random.default_rng(5)
    a = [int(v) for v in rng.integers(0, 2**40, n)]
    b = [int(v) for v in rng.integers(0, 2**40, n)]
    c = [0] * n
    for i, ai in enumerate(a):
        if ai == 0:
            continue
        for j, bj in enumerate(b):
            k = i + j
            if k < n:
                c[k] += ai * bj
            else:
                c[k - n] -= ai * bj
    c = np.array([v % q for v in c], dtype=np.uint64)
    A = np.array(a, dtype=np.uint64).reshape(1, 1, n) % np.uint64(q)
    B = np.array(b, dtype=np.uint64).reshape(1, 1, n) % np.uint64(q)
    oracle.ntt_batch(A, [q], [psi], False)
    oracle.ntt_batch(B, [q], [psi], False)
    prod = np.array([int(x) * int(y) % q for x, y in zip(A.ravel(), B.ravel())], dtype=np.uint64)
    P = prod.reshape(1, 1, n)
    oracle.ntt_batch(P, [q], [psi], True)
    assert np.array_equal(P.ravel(), c)


def test_batch_threads_agree(oracle):
    log_n, L = 12, 5
    qs = oracle.ntt_primes(log_n, 59, L)
    psis = [oracle.root_of_unity(2 << log_n, q) for q in qs]
    x = np.stack([np.stack([probe_values(1 << log_n, q, 3, 7 * p + i) for i, q in enumerate(qs)])
                  for p in range(3)])
    y1 = oracle.ntt_batch(x.copy(), qs, psis, False, threads=1)
    y4 = oracle.ntt_batch(x.copy(), qs, psis, False, threads=4)
    assert np.array_equal(y1, y4)
    z = oracle.ntt_batch(y4, qs, psis, True, threads=4)
    assert np.array_equal(z, x)
