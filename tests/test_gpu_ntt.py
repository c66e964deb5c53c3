"""CUDA NTT/INTT (through the C ABI) bit-exact against the CPU oracle.

Cases follow the reference NTT probe (experiments/ntt_warp_tail/probe.cu:164-206):
every ring size, 1/4/many limbs, input patterns zero / q-1 / alternating / mixed,
every output word compared.  Plus the O(N^2) definition KAT and the full
BASELINE config-2 shape (N=2^16, 36 limbs x 4 polys).
"""
import numpy as np
import pytest

from conftest import probe_values

pytestmark = pytest.mark.gpu


def _ctx(log_n, primes):
    from fhe_mamba_b200 import NttContext
    return NttContext(log_n, primes)


def _batch(log_n, qs, n_polys, pattern, salt=0):
    n = 1 << log_n
    return np.stack([np.stack([probe_values(n, q, pattern, salt + 131 * p + i) for i, q in enumerate(qs)])
                     for p in range(n_polys)])


def test_kat_definition_n1024(ntt_kat):
    for a, out, q in zip(ntt_kat["inputs"], ntt_kat["outputs"], ntt_kat["primes"]):
        ctx = _ctx(10, [int(q)])
        x = a.copy().reshape(1, 1, -1)
        ctx.forward(x)
        assert np.array_equal(x[0, 0], out)
        ctx.inverse(x)
        assert np.array_equal(x[0, 0], a)


@pytest.mark.parametrize("log_n", list(range(10, 18)))
def test_ring_sizes_all_patterns(oracle, log_n):
    qs = oracle.ntt_primes(log_n, 59, 4)
    ctx = _ctx(log_n, qs)
    psis = ctx.roots()
    assert psis == [oracle.root_of_unity(2 << log_n, q) for q in qs]
    for pattern in range(4):
        for limbs in (1, 4):
            x = _batch(log_n, qs[:limbs], 2, pattern, salt=log_n)
            want = oracle.ntt_batch(x.copy(), qs[:limbs], psis[:limbs], False, threads=8)
            got = ctx.forward(x.copy())
            assert np.array_equal(got, want), (log_n, pattern, limbs)
            back = ctx.inverse(got)
            assert np.array_equal(back, x), (log_n, pattern, limbs)


def test_ckks_chain_60bit_primes(oracle, golden_chain):
    # 60-bit q_0 and P primes stress the lazy [0, 4q) bounds; use the recorded chain.
    allp = golden_chain["q"] + golden_chain["p"]
    ctx = _ctx(16, allp)
    psis = ctx.roots()
    limbs = [0, 1, 44, 45, 56]
    for pattern in range(4):
        for l in limbs:
            x = _batch(16, [allp[l]], 1, pattern, salt=l)
            want = oracle.ntt_batch(x.copy(), [allp[l]], [psis[l]], False)
            got = ctx.forward(x.copy(), limb0=l)
            assert np.array_equal(got, want), (pattern, l)
            assert np.array_equal(ctx.inverse(got, limb0=l), x)


def test_config2_full_shape_host_and_device(oracle):
    import torch
    qs = oracle.ntt_primes(16, 59, 36)
    ctx = _ctx(16, qs)
    psis = ctx.roots()
    x = _batch(16, qs, 4, 3, salt=99)
    want = oracle.ntt_batch(x.copy(), qs, psis, False, threads=8)
    got = ctx.forward(x.copy())
    assert np.array_equal(got, want)
    d = torch.from_numpy(x.view(np.int64).copy()).cuda()
    ctx.forward(d)
    ctx.synchronize()
    assert np.array_equal(d.cpu().numpy().view(np.uint64), want)
    ctx.inverse(d)
    ctx.synchronize()
    assert np.array_equal(d.cpu().numpy().view(np.uint64), x)


def test_limb_offsets_and_errors(oracle):
    from fhe_mamba_b200 import InvalidArgument
    qs = oracle.ntt_primes(12, 59, 6)
    ctx = _ctx(12, qs)
    psis = ctx.roots()
    x = _batch(12, qs[2:5], 3, 3, salt=4)
    want = oracle.ntt_batch(x.copy(), qs[2:5], psis[2:5], False)
    assert np.array_equal(ctx.forward(x.copy(), limb0=2), want)
    with pytest.raises(InvalidArgument):
        ctx.forward(x.copy(), limb0=4)
    with pytest.raises(InvalidArgument):
        _ctx(12, [qs[0] + 2])
