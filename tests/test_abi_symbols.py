"""The C-ABI library builds, loads, and exports every symbol include/fhe_b200.h declares.
No compute call is made (no GPU in this container)."""
import ctypes

from fhe_mamba_b200 import _lib


def test_header_declares_expected_core():
    names = _lib.header_symbols()
    for n in ("fhe_ctx_create", "fhe_ctx_destroy", "fhe_ntt", "fhe_intt", "fhe_last_error"):
        assert n in names


def test_library_exports_every_header_symbol():
    lib = _lib.load()
    missing = [n for n in _lib.header_symbols() if not hasattr(lib, n)]
    assert not missing, missing


def test_bindings_cover_header():
    assert set(_lib.header_symbols()) == set(_lib.SIGNATURES)


def test_null_arguments_report_errors_without_gpu():
    lib = _lib.load()
    assert lib.fhe_ctx_create(None, None) == _lib.FHE_ERR_INVALID
    assert "null" in _lib.last_error()
    assert lib.fhe_ntt(None, None, 1, 0, 1, 0) == _lib.FHE_ERR_INVALID
    assert lib.fhe_ctx_destroy(None) == _lib.FHE_OK
    buf = ctypes.create_string_buffer(8)
    assert lib.fhe_last_error(buf, 8) == 0


def test_product_moduli_match_recorded_chain(golden_chain, oracle):
    from fhe_mamba_b200.params import ckks_moduli, ntt_primes
    g = golden_chain
    q, p = ckks_moduli(g["log_n"], g["mult_depth"], g["scaling_mod_size"], g["first_mod_size"],
                       g["num_large_digits"])
    assert q == g["q"] and p == g["p"]
    for args in [(14, 8, 50, 60, 2), (16, 19, 59, 60, 3), (16, 44, 59, 60, 3)]:
        assert ckks_moduli(*args) == oracle.ckks_moduli(args[0], args[1] + 1, *args[2:])
    assert ntt_primes(16, 59, 36) == oracle.ntt_primes(16, 59, 36)
