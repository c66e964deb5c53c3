"""The sparse-packing trace used by bootstrapping, checked in exact integer
arithmetic on CPU: for slots n < N/2 the sum of the automorphisms
X -> X^(5^(j n)), j < g = N/(2n), maps any polynomial t mod X^N + 1 to g times
its part in the subring Z[X^(N/2n)] (the coefficients at multiples of N/2n),
which is what the device computes with log2 g rotations by multiples of n."""
import numpy as np
import pytest


def automorphism(t, k):
    """t(X) -> t(X^k) mod X^N + 1 (k odd)."""
    n = len(t)
    out = np.zeros(n, dtype=object)
    for e, c in enumerate(t):
        f = (e * k) % (2 * n)
        if f < n:
            out[f] += c
        else:
            out[f - n] -= c
    return out


@pytest.mark.parametrize("N,slots", [(64, 8), (64, 4), (128, 16), (128, 32)])
def test_trace_keeps_g_times_the_subring_part(N, slots):
    rng = np.random.default_rng(N + slots)
    t = np.array([int(v) for v in rng.integers(-10**12, 10**12, N)], dtype=object)
    g, gap = N // (2 * slots), N // (2 * slots)
    # doubling as on the device: x += rot(x, j n) for j = 1, 2, 4, ... < g
    x = t.copy()
    j = 1
    while j < g:
        x = x + automorphism(x, pow(5, j * slots, 2 * N))
        j *= 2
    want = np.array([g * c if e % gap == 0 else 0 for e, c in enumerate(t)], dtype=object)
    assert list(x) == list(want)


def test_rotation_by_a_multiple_of_the_slots_fixes_the_subring():
    N, slots = 128, 16
    gap = N // (2 * slots)
    rng = np.random.default_rng(1)
    t = np.zeros(N, dtype=object)
    for e in range(0, N, gap):
        t[e] = int(rng.integers(-1000, 1000))
    for j in range(1, N // (2 * slots)):
        assert list(automorphism(t, pow(5, j * slots, 2 * N))) == list(t)
