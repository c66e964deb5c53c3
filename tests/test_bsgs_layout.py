"""Slot-exact simulation of the BSGS diagonal layout (CPU): the same roll /
multiply / add schedule the device linear transform runs equals W @ x, as the
reference's replicated-BSGS simulator does for its own layout
(src/fhemamba/bsgs_layout.py, tests/test_bsgs_layout.py)."""
import numpy as np
import pytest

from fhe_mamba_b200.ckks import bsgs_diagonals


def simulate(diags, x_rep, baby, giant):
    out = np.zeros_like(x_rep)
    babies = [np.roll(x_rep, -j) for j in range(baby)]
    for g in range(giant):
        inner = np.zeros_like(x_rep)
        for j in range(baby):
            d = diags[g * baby + j]
            if d is not None:
                inner += d * babies[j]
        out += np.roll(inner, -g * baby)
    return out


@pytest.mark.parametrize("m,n,baby,giant,slots", [(768, 1536, 32, 48, 1 << 15), (24, 48, 8, 6, 2048),
                                                   (5, 7, 3, 3, 64), (16, 16, 4, 4, 64)])
def test_layout_equals_matmul(m, n, baby, giant, slots):
    rng = np.random.default_rng(m + n)
    W = rng.normal(0, 0.02, size=(m, n))
    x = rng.uniform(-1, 1, n)
    x_rep = np.zeros(slots)
    x_rep[:n] = x
    x_rep[n:2 * n] = x
    y = simulate(bsgs_diagonals(W, baby, giant, slots), x_rep, baby, giant)
    assert np.allclose(y[:m], W @ x, atol=1e-12)
    assert np.allclose(y[m:], 0, atol=1e-12)


def test_layout_rejects_bad_shapes():
    W = np.zeros((8, 8))
    with pytest.raises(ValueError):
        bsgs_diagonals(W, 2, 3, 64)  # 6 < 8 diagonals
    with pytest.raises(ValueError):
        bsgs_diagonals(np.zeros((40, 40)), 8, 5, 64)  # does not fit
