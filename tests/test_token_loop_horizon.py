"""The bench's 24-layer token loop (seed-7 prompt of 8
tokens, then greedy generation) on the plaintext polynomial path, over the
driver's full horizon: every refresh input stays inside its bound and every
Chebyshev input inside its interval, so the encrypted loop's bootstraps and
series see only values they were built for.  A calibration over 4-token
sequences (the earlier setting) fails the same audit.  No GPU."""
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def test_config5_horizon_inside_bounds_and_domains():
    import bench
    horizon = bench.PROMPT_TOKENS + 20  # prompt prefill + the driver's 20 timed tokens
    m = bench.synthetic_model(6, horizon)
    inputs = bench.plaintext_protocol(m, horizon)
    assert inputs[:bench.PROMPT_TOKENS] == bench.config5_prompt()
    a = m.audit(inputs)
    assert a["max_bound_ratio"] <= 0.75, a["bound_ratio"]
    assert a["max_domain_position"] <= 1.0 + 1e-6, a["domain"]
    assert set(a["bound_ratio"]) >= {"h", "u", "proj", "xbc", "xc", "dt", "adt", "pack", "state", "z", "y", "g",
                                     "gn", "final"}


def test_short_calibration_fails_the_audit():
    """A mistake planted on the CPU: the round-one calibration (4-token
    sequences, bounds at 2x) lets the same horizon leave its refresh bounds."""
    import bench
    from fhe_mamba_b200.mamba2_layer import Mamba2Model
    m = Mamba2Model(layers=24, d_model=768, d_state=128, heads=24, vocab=bench.VOCAB, seed=6, calib_sequences=4,
                    calib_tokens=4, calib_prompt=4, bound_factor=2.0)
    a = m.audit(bench.plaintext_protocol(m, bench.PROMPT_TOKENS + 20))
    assert a["max_bound_ratio"] > 1.0
    assert np.isfinite(a["max_bound_ratio"])
