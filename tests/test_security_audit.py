"""Classical-128 parameter audit (the reference's CkksSecurityAudit,
native/fideslib_stage0/src/fideslib_security.hpp:18-80), on CPU: exact bit
lengths of Q, P and Q*P for the chains the library generates, against the
2024 guidelines' bound for the ring."""
import json
import math
import os

from fhe_mamba_b200.program import security_audit

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def test_reference_128_classic_chain_passes():
    with open(os.path.join(GOLDEN, "prime_chain_n17_d44_s59_f60_dnum4.json")) as f:
        chain = json.load(f)
    q = [int(x) for x in chain["q"]]
    p = [int(x) for x in chain["p"]]
    a = security_audit(17, 44, 59, 60, 4)
    assert a["ring_dimension"] == 131072 and a["guideline_max_qp_bits"] == 3523
    assert (a["q_bits"], a["p_bits"], a["qp_bits"]) == (
        math.prod(q).bit_length(), math.prod(p).bit_length(), math.prod(q + p).bit_length())
    assert a["q_towers"] == 45 and a["p_towers"] == 12 and a["hybrid_digits"] == 4
    assert a["error_sigma"] >= 3.19 and a["passed"]


def test_ring_2_16_depth_44_fails_the_bound():
    a = security_audit(16, 44, 59, 60, 3)
    assert a["guideline_max_qp_bits"] == 1747 and a["qp_bits"] > 1747 and not a["passed"]


def test_small_chain_within_its_ring_bound():
    a = security_audit(15, 8, 50, 55, 2)
    assert a["guideline_max_qp_bits"] == 868 and a["qp_bits"] <= 868 and a["passed"]
    b = security_audit(14, 6, 50, 55, 2)  # BASELINE config 1's chain exceeds 430 bits
    assert b["qp_bits"] > 430 and not b["passed"]
