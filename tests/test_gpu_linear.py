"""Device BSGS matvec (fhe_linear_transform) against the oracle and fp64.

Small ring: the device result equals, word for word, the oracle composition
of the same schedule (rotations of the input, plaintext products and sums per
giant step, giant rotations).  BASELINE config 3 (768 x 1536, N=2^16, 2^15
slots, 20 limbs, dnum 3, baby 32 / giant 48): decrypted error <= 1e-4 max-abs
against the fp64 matmul.
"""
import numpy as np
import pytest

from fhe_mamba_b200.ckks import bsgs_diagonals

pytestmark = pytest.mark.gpu

SEED = 99


def _ext_add(a, b, q, p):
    """a + b over extended limbs ([..., nq + K, N]: Q primes, then P primes)."""
    primes = np.array(list(q[:a.shape[-2] - len(p)]) + list(p), dtype=np.uint64)[:, None]
    return (a + b) % primes


@pytest.mark.parametrize("hoist", [False, True])
def test_linear_transform_matches_oracle_small(oracle, hoist):
    """hoist False: a full key switch per giant step; True (the default): the
    rotating giants' key inner products permuted and summed in the extended
    basis, one ModDown for all of them plus the permuted c0 parts."""
    from fhe_mamba_b200 import CCParams, CryptoContext
    log_n, depth, sb, fb, dnum = 12, 6, 45, 55, 2
    cc = CryptoContext(CCParams(ring_dim=1 << log_n, multiplicative_depth=depth, scaling_mod_size=sb,
                                first_mod_size=fb, num_large_digits=dnum))
    oc = oracle.Ckks(log_n, cc.q, cc.p, dnum, cc.slots)
    cc.KeyGen(SEED)
    s, sn = oc.keygen_secret(SEED)
    m, n, baby, giant = 24, 48, 8, 6
    rng = np.random.default_rng(1)
    W = rng.normal(0, 0.02, size=(m, n))
    x = rng.uniform(-1, 1, n)
    x_rep = np.zeros(cc.slots)
    x_rep[:n] = x
    x_rep[n:2 * n] = x
    steps = list(range(1, baby)) + [g * baby for g in range(1, giant)]
    cc.EvalRotateKeyGen(steps)
    ct = cc.Encrypt(cc.MakeCKKSPackedPlaintext(x_rep))
    diags = bsgs_diagonals(W, baby, giant, cc.slots)
    dense = [d for d in diags if d is not None]
    pts = iter(cc.MakeCKKSPackedPlaintexts(np.array(dense)))
    dpts = [next(pts) if d is not None else None for d in diags]
    for d, p in zip(diags, dpts):
        if d is not None:
            assert np.array_equal(p.residues(), oc.encode(d, cc.level_scale(), cc.n_q))
    cc.SetGiantStepHoisting(hoist)
    out = cc.EvalLinearTransform(ct, dpts, baby, giant)
    cc.SetGiantStepHoisting(True)
    # oracle composition of the same schedule
    a = ct.residues()
    nq = a.shape[1]
    keys = {st: oc.rot_key(SEED, s, sn, oc.galois(st)) for st in steps}
    babies = [a] + [oc.rotate(a, oc.galois(j), keys[j]) for j in range(1, baby)]
    total, ext_sum, c0_sum = None, None, None
    for g in range(giant):
        inner = None
        for j in range(baby):
            p = dpts[g * baby + j]
            if p is None:
                continue
            t = oc.mul_plain(babies[j], p.residues())
            inner = t if inner is None else oc.add(inner, t)
        if g and hoist:
            gal = oc.galois(g * baby)
            acc = oc.automorphism(oc.key_inner(oc.modup(inner[1], nq), nq, keys[g * baby]), gal)
            c0 = oc.automorphism(inner[0], gal)
            ext_sum = acc if ext_sum is None else _ext_add(ext_sum, acc, cc.q, cc.p)
            c0_sum = c0 if c0_sum is None else oc.add(c0_sum[None], c0[None])[0]
            continue
        if g:
            inner = oc.rotate(inner, oc.galois(g * baby), keys[g * baby])
        total = inner if total is None else oc.add(total, inner)
    if hoist:
        u = np.stack([oc.moddown(ext_sum[0], nq), oc.moddown(ext_sum[1], nq)])
        u[0] = oc.add(u[0][None], c0_sum[None])[0]
        total = oc.add(total, u)
    assert np.array_equal(out.residues(), total)
    y = cc.Decrypt(out).GetRealPackedValue()
    assert np.max(np.abs(y[:m] - W @ x)) < 1e-4


def test_config3_matvec_accuracy():
    from fhe_mamba_b200 import CCParams, CryptoContext
    cc = CryptoContext(CCParams(ring_dim=1 << 16, multiplicative_depth=19, scaling_mod_size=59,
                                first_mod_size=60, num_large_digits=3))
    assert cc.n_q == 20 and cc.slots == 1 << 15
    cc.KeyGen(SEED)
    m, n, baby, giant = 768, 1536, 32, 48
    rng = np.random.default_rng(2)
    W = rng.normal(0, 0.02, size=(m, n))
    x = rng.uniform(-1, 1, n)
    cc.EvalRotateKeyGen(list(range(1, baby)) + [g * baby for g in range(1, giant)] + [-n])
    v = np.zeros(cc.slots)
    v[:n] = x
    ct = cc.Encrypt(cc.MakeCKKSPackedPlaintext(v))
    ct_rep = cc.EvalAdd(ct, cc.EvalRotate(ct, -n))  # replicate the input once
    diags = bsgs_diagonals(W, baby, giant, cc.slots)
    pts = cc.MakeCKKSPackedPlaintexts(np.array([d for d in diags if d is not None]))
    out = cc.EvalLinearTransform(ct_rep, pts, baby, giant)
    cc.RescaleInPlace(out)
    y = cc.Decrypt(out).GetRealPackedValue()
    err = np.max(np.abs(y[:m] - W @ x))
    assert err <= 1e-4, err
    assert np.max(np.abs(y[m:m + 64])) <= 1e-4
