"""The oracle's CKKS modulus generator against the chain the reference recorded."""
import pytest


def test_chain_matches_recorded_openfhe_chain(oracle, golden_chain):
    g = golden_chain
    q, p = oracle.ckks_moduli(g["log_n"], g["mult_depth"] + 1, g["scaling_mod_size"],
                              g["first_mod_size"], g["num_large_digits"])
    assert q == g["q"]
    assert p == g["p"]


def test_chain_invariants(oracle):
    for log_n, depth, scale, first, dnum in [(14, 8, 50, 60, 2), (16, 19, 59, 60, 3),
                                            (16, 44, 59, 60, 3), (17, 44, 59, 60, 4)]:
        q, p = oracle.ckks_moduli(log_n, depth + 1, scale, first, dnum)
        m = 2 << log_n
        allp = q + p
        assert len(set(allp)) == len(allp)
        for x in allp:
            assert x % m == 1 and oracle.lib().oc_is_prime(x)
        assert q[0].bit_length() == first
        assert all(x.bit_length() in (scale, scale + 1) for x in q[1:])
        assert all(x.bit_length() == 60 for x in p)


def test_equal_first_and_scale_rejected(oracle):
    with pytest.raises(ValueError):
        oracle.ckks_moduli(14, 9, 50, 50, 2)


def test_ntt_bench_primes(oracle):
    ps = oracle.ntt_primes(16, 59, 36)
    assert len(set(ps)) == 36
    for x in ps:
        assert x < 2**59 and x % (2 << 16) == 1 and oracle.lib().oc_is_prime(x)
    assert ps == sorted(ps, reverse=True)


def test_min_root_is_minimal_primitive(oracle, ntt_kat):
    # Against the pure-Python definition recorded in the KAT fixture.
    for q, psi in zip(ntt_kat["primes"], ntt_kat["psi"]):
        assert oracle.root_of_unity(2048, int(q)) == int(psi)
