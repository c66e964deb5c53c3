"""Bootstrapping on the device.

ModRaise and the exact multiplication by i are compared word for word with the
oracle's restatement; the strided BSGS linear transform (the CoeffToSlot /
SlotToCoeff shape: diagonals at multiples of a stride, giant steps offset so
that negative diagonals are reached) is checked against the fp64 product; the
full bootstrap (ModRaise -> CoeffToSlot -> EvalMod -> SlotToCoeff) is checked
by decryption against its input.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

SEED = 4321


@pytest.fixture(scope="module")
def small(oracle):
    from fhe_mamba_b200 import CCParams, CryptoContext
    log_n, depth, sb, fb, dnum = 12, 6, 45, 55, 2
    cc = CryptoContext(CCParams(ring_dim=1 << log_n, multiplicative_depth=depth, scaling_mod_size=sb,
                                first_mod_size=fb, num_large_digits=dnum))
    oc = oracle.Ckks(log_n, cc.q, cc.p, dnum, cc.slots)
    cc.KeyGen(SEED)
    s, sn = oc.keygen_secret(SEED)
    return cc, oc, s, sn


def _rand_ct(oc, nq, seed, ncomp=2):
    rng = np.random.default_rng(seed)
    x = np.empty((ncomp, nq, oc.n), dtype=np.uint64)
    for l in range(nq):
        x[:, l, :] = rng.integers(0, oc.q[l], size=(ncomp, oc.n), dtype=np.uint64)
    return x


def test_mul_i_matches_oracle_and_decrypts(small):
    cc, oc, s, sn = small
    a = _rand_ct(oc, 3, 5)
    assert np.array_equal(cc.MultByI(cc.upload(a)).residues(), oc.mul_i(a))
    r = np.random.default_rng(6)
    z = r.uniform(-1, 1, cc.slots) + 1j * r.uniform(-1, 1, cc.slots)
    ct = cc.Encrypt(cc.MakeCKKSPackedPlaintext(z))
    got = cc.Decrypt(cc.MultByI(ct)).GetCKKSPackedValue()
    assert np.max(np.abs(got - 1j * z)) < 1e-6


def test_mod_raise_matches_oracle(small):
    cc, oc, s, sn = small
    for nq in (1, 3):
        a = _rand_ct(oc, nq, 7 + nq)
        got = cc.ModRaise(cc.upload(a))
        assert got.GetLevel() == 0 and got.residues().shape == (2, oc.L, oc.n)
        assert np.array_equal(got.residues(), oc.mod_raise(a)), nq


def test_mod_raise_keeps_message_mod_q0(small):
    """Decrypting the raised ciphertext gives m + q0*I with small integer I."""
    cc, oc, s, sn = small
    r = np.random.default_rng(8)
    z = r.uniform(-1, 1, cc.slots)
    ct = cc.Encrypt(cc.MakeCKKSPackedPlaintext(z))
    cc.LevelReduceInPlace(ct, cc.n_q - 1)
    raised = cc.ModRaise(ct)
    dec = oc.decrypt(sn, raised.residues())  # [L][N] NTT form
    dec = oc.ntt(np.ascontiguousarray(dec).copy(), oc.L, 0, inverse=True)
    q0, q1 = oc.q[0], oc.q[1]
    # exact coefficients from the first two limbs (CRT): t = m + q0*I
    inv = pow(q0, -1, q1)
    t = [int(a) + q0 * (((int(b) - int(a)) * inv) % q1) for a, b in zip(dec[0], dec[1])]
    t = [v - q0 * q1 if v > q0 * q1 // 2 else v for v in t]
    I = np.array([round(v / q0) for v in t], dtype=np.float64)
    assert np.max(np.abs(I)) <= oc.n  # |I| is bounded by the secret's weight
    m = np.array([v - q0 * round(v / q0) for v in t], dtype=np.float64)
    assert np.max(np.abs(m)) < q0 / 4


def _strided_diags(W, b, G, stride, off, slots):
    """Pre-rotated diagonal plaintext values for the strided BSGS schedule."""
    out = []
    k = np.arange(slots)
    for g in range(G):
        r = (g * b - off) * stride
        for j in range(b):
            t = g * b + j - off
            d = W[k, (k + t * stride) % slots]
            out.append(np.roll(d, r) if np.any(d) else None)
    return out


def test_strided_linear_transform(small):
    cc, oc, s, sn = small
    n = cc.slots
    b, G, off, stride = 4, 4, 7, 8
    rng = np.random.default_rng(9)
    W = np.zeros((n, n), dtype=complex)
    k = np.arange(n)
    for t in range(-off, G * b - off):
        if t == 5:
            continue  # one all-zero diagonal
        W[k, (k + t * stride) % n] = rng.uniform(-1, 1, n) + 1j * rng.uniform(-1, 1, n)
    diags = _strided_diags(W, b, G, stride, off, n)
    assert sum(d is None for d in diags) == 1
    steps = sorted({j * stride for j in range(1, b)} | {(g * b - off) * stride for g in range(G)} - {0})
    cc.EvalRotateKeyGen(steps)
    x = rng.uniform(-1, 1, n) + 1j * rng.uniform(-1, 1, n)
    ct = cc.Encrypt(cc.MakeCKKSPackedPlaintext(x))
    pts = [cc.MakeCKKSPackedPlaintext(d) if d is not None else None for d in diags]
    out = cc.EvalLinearTransform(ct, pts, b, G, stride=stride, giant_offset=off)
    got = cc.Decrypt(out).GetCKKSPackedValue()
    assert np.max(np.abs(got - W @ x)) < 1e-4


@pytest.fixture(scope="module")
def boot_ctx():
    from fhe_mamba_b200 import CCParams, CryptoContext
    cc = CryptoContext(CCParams(ring_dim=1 << 12, multiplicative_depth=25, scaling_mod_size=59,
                                first_mod_size=60, num_large_digits=3))
    cc.KeyGen(SEED)
    cc.EvalBootstrapSetup((4, 4))
    cc.EvalBootstrapKeyGen()
    return cc


@pytest.mark.parametrize("cplx", [False, True])
def test_bootstrap_refreshes_levels(boot_ctx, cplx):
    """A ciphertext with 2 limbs left comes back with fresh limbs and the same slots."""
    cc = boot_ctx
    r = np.random.default_rng(11 + cplx)
    x = r.uniform(-1, 1, cc.slots)
    if cplx:
        x = x + 1j * r.uniform(-1, 1, cc.slots)
    ct = cc.Encrypt(cc.MakeCKKSPackedPlaintext(x))
    cc.LevelReduceInPlace(ct, cc.n_q - 2)
    out = cc.EvalBootstrap(ct)
    lv = cc.bootstrap_levels()
    # 4 CoeffToSlot levels, 7 Chebyshev + 6 double-angle levels, 4 SlotToCoeff levels
    assert lv == [cc.n_q, cc.n_q - 4, cc.n_q - 17, cc.n_q - 21] and out.n_limbs() == cc.n_q - 21
    y = cc.Decrypt(out).GetCKKSPackedValue()
    if not cplx:
        y = y.real
    assert np.max(np.abs(y - x)) < 1e-4


def test_bootstrap_stages_chain(boot_ctx):
    """Stages 0..3 chained equal the one-call bootstrap's accuracy; a constant
    vector (the worst case for the sine approximation) also comes back."""
    cc = boot_ctx
    x = np.full(cc.slots, 0.9)
    ct = cc.Encrypt(cc.MakeCKKSPackedPlaintext(x))
    cc.LevelReduceInPlace(ct, cc.n_q - 2)
    c = ct
    for st in range(4):
        c = cc.EvalBootstrapStage(st, c)
    assert np.max(np.abs(cc.Decrypt(c).GetRealPackedValue() - x)) < 1e-4


def test_bootstrap_rejects_one_limb(boot_ctx):
    from fhe_mamba_b200 import StateError
    cc = boot_ctx
    ct = cc.Encrypt(cc.MakeCKKSPackedPlaintext(np.zeros(4)))
    cc.LevelReduceInPlace(ct, cc.n_q - 1)
    with pytest.raises(StateError):
        cc.EvalBootstrap(ct)


def test_bootstrap_then_multiply(boot_ctx):
    """The refreshed ciphertext supports further multiplications."""
    cc = boot_ctx
    x = np.random.default_rng(13).uniform(-1, 1, cc.slots)
    ct = cc.Encrypt(cc.MakeCKKSPackedPlaintext(x))
    cc.LevelReduceInPlace(ct, cc.n_q - 3)
    out = cc.EvalBootstrap(ct)
    sq = cc.EvalMult(out, out)
    y = cc.Decrypt(sq).GetRealPackedValue()
    assert np.max(np.abs(y - x * x)) < 2e-4


def test_two_pass_refresh_gains_precision(boot_ctx):
    """bootstrap_components with two passes (residual * 4096 bootstrapped again)
    beats one pass by orders of magnitude; merge gives the same value."""
    cc = boot_ctx
    x = np.random.default_rng(17).uniform(-1, 1, cc.slots)
    ct = cc.Encrypt(cc.MakeCKKSPackedPlaintext(x))
    cc.LevelReduceInPlace(ct, cc.n_q - 4)  # the scaling and the residual each take a level
    one = cc.Decrypt(cc.refresh(ct, 1.0, passes=1)).GetRealPackedValue()
    two = cc.Decrypt(cc.refresh(ct, 1.0, passes=2)).GetRealPackedValue()
    e1, e2 = np.max(np.abs(one - x)), np.max(np.abs(two - x))
    assert e2 < 1e-6 and e2 < e1 / 30
    first, second, div = cc.bootstrap_components(ct, passes=2, merge=True)
    assert second is None and div == 4096.0
    merged = cc.Decrypt(first).GetRealPackedValue() / 4096.0
    assert np.max(np.abs(merged - x)) < 1e-6


def test_refresh_with_bound(boot_ctx):
    cc = boot_ctx
    x = np.random.default_rng(19).uniform(-6, 6, cc.slots)
    ct = cc.Encrypt(cc.MakeCKKSPackedPlaintext(x))
    cc.LevelReduceInPlace(ct, cc.n_q - 4)
    y = cc.Decrypt(cc.refresh(ct, 8.0, passes=2)).GetRealPackedValue()
    assert np.max(np.abs(y - x)) < 1e-5


def test_s2c_first_bootstrap():
    """SlotToCoeff before ModRaise: same values, budget_stc (4) more limbs left."""
    from fhe_mamba_b200 import CCParams, CryptoContext
    cc = CryptoContext(CCParams(ring_dim=1 << 12, multiplicative_depth=25, scaling_mod_size=59,
                                first_mod_size=60, num_large_digits=3))
    cc.KeyGen(SEED)
    cc.EvalBootstrapSetup((4, 4), slots_to_coeffs_first=True)
    cc.EvalBootstrapKeyGen()
    r = np.random.default_rng(23)
    x = r.uniform(-1, 1, cc.slots) + 1j * r.uniform(-1, 1, cc.slots)
    ct = cc.Encrypt(cc.MakeCKKSPackedPlaintext(x))
    cc.LevelReduceInPlace(ct, cc.n_q - 6)
    out = cc.EvalBootstrap(ct)
    assert out.n_limbs() == cc.n_q - 17
    y = cc.Decrypt(out).GetCKKSPackedValue()
    assert np.max(np.abs(y - x)) < 1e-4
    short = cc.Encrypt(cc.MakeCKKSPackedPlaintext(x.real))
    cc.LevelReduceInPlace(short, cc.n_q - 5)
    from fhe_mamba_b200 import StateError
    with pytest.raises(StateError):
        cc.EvalBootstrap(short)


def test_sparse_encapsulated_bootstrap(oracle):
    """Sparse-secret encapsulation: the sparse secret and both switching keys
    equal the oracle's word for word; the bootstrap keeps more limbs than the
    uniform-ternary one (smaller EvalMod interval, lower degree, 3 double
    angles) and decrypts to its input."""
    from fhe_mamba_b200 import CCParams, CryptoContext
    h = 32
    cc = CryptoContext(CCParams(ring_dim=1 << 12, multiplicative_depth=25, scaling_mod_size=59,
                                first_mod_size=60, num_large_digits=3))
    cc.KeyGen(SEED)
    cc.EvalBootstrapSetup((4, 4), sparse_hamming_weight=h)
    cc.EvalBootstrapKeyGen()
    oc = oracle.Ckks(12, cc.q, cc.p, 3, cc.slots)
    coef, spn = oc.sparse_secret(SEED, h)
    assert np.count_nonzero(coef) == h and set(np.unique(coef)) <= {-1, 0, 1}
    assert np.array_equal(cc.key(4).reshape(spn.shape), spn)
    s, sn = oc.keygen_secret(SEED)
    to_sparse, to_dense = oc.sparse_keys(SEED, sn, spn)
    assert np.array_equal(cc.key(5).reshape(to_sparse.shape), to_sparse)
    assert np.array_equal(cc.key(6).reshape(to_dense.shape), to_dense)
    info = cc.bootstrap_info()
    assert info["chebyshev_degree"] < 60
    r = np.random.default_rng(29)
    for cplx in (False, True):
        x = r.uniform(-1, 1, cc.slots) + (1j * r.uniform(-1, 1, cc.slots) if cplx else 0)
        ct = cc.Encrypt(cc.MakeCKKSPackedPlaintext(x))
        cc.LevelReduceInPlace(ct, cc.n_q - 2)
        out = cc.EvalBootstrap(ct)
        lv = cc.bootstrap_levels()
        assert lv[0] == cc.n_q and lv[1] == cc.n_q - 4 and lv[2] - lv[3] == 4
        assert out.n_limbs() > cc.n_q - 21 + 2  # at least 3 levels above uniform ternary
        y = cc.Decrypt(out).GetCKKSPackedValue()
        assert np.max(np.abs((y if cplx else y.real) - x)) < 1e-4


@pytest.mark.parametrize("slots", [512, 1024])
def test_sparse_packing_bootstrap(slots):
    """Sparsely packed slots (n < N/2, the reference's 128-bit mode runs 2^15
    slots at N = 2^17): ModRaise, the trace over the rotations by multiples of
    n, then CoeffToSlot / EvalMod / SlotToCoeff on n slots; the slots come back
    with fresh limbs."""
    from fhe_mamba_b200 import CCParams, CryptoContext
    cc = CryptoContext(CCParams(ring_dim=1 << 12, multiplicative_depth=25, scaling_mod_size=59,
                                first_mod_size=60, num_large_digits=3, batch_size=slots))
    assert cc.slots == slots
    cc.KeyGen(SEED)
    cc.EvalBootstrapSetup((4, 4))
    cc.EvalBootstrapKeyGen()
    r = np.random.default_rng(31 + slots)
    for cplx in (False, True):
        x = r.uniform(-1, 1, slots) + (1j * r.uniform(-1, 1, slots) if cplx else 0)
        ct = cc.Encrypt(cc.MakeCKKSPackedPlaintext(x))
        cc.LevelReduceInPlace(ct, cc.n_q - 2)
        out = cc.EvalBootstrap(ct)
        assert out.n_limbs() == cc.n_q - 21
        y = cc.Decrypt(out).GetCKKSPackedValue()[:slots]
        assert np.max(np.abs((y if cplx else y.real) - x)) < 1e-4
        sq = cc.Decrypt(cc.EvalMult(out, out)).GetCKKSPackedValue()[:slots]
        assert np.max(np.abs(sq - x * x)) < 4e-4


def test_library_refresh_matches_host_refresh(boot_ctx):
    """fhe_refresh (one call) against the host-side refresh: same values within
    the two-pass precision; two passes beat one; values up to the bound."""
    cc = boot_ctx
    x = np.random.default_rng(37).uniform(-5, 5, cc.slots)
    ct = cc.Encrypt(cc.MakeCKKSPackedPlaintext(x))
    cc.LevelReduceInPlace(ct, cc.n_q - 4)
    one = cc.Decrypt(cc.EvalRefresh(ct, 8.0, passes=1)).GetRealPackedValue()
    two = cc.Decrypt(cc.EvalRefresh(ct, 8.0, passes=2)).GetRealPackedValue()
    host = cc.Decrypt(cc.host_refresh(ct, 8.0, passes=2)).GetRealPackedValue()
    assert np.max(np.abs(two - x)) < 1e-5 and np.max(np.abs(two - x)) < np.max(np.abs(one - x)) / 10
    assert np.max(np.abs(two - host)) < 1e-5


def test_subslot_refresh():
    """Sub-slot refreshes (n = 256, 512 of 2048 slots): an input zero outside
    [0, support) is replicated with period n, bootstrapped with one EvalMod
    (split and merge folded into the edge CoeffToSlot / SlotToCoeff groups)
    and masked back: the same limbs as the full refresh, the values on
    [0, support) within the full refresh's precision, zeros from n on; real
    and complex values; a support above every sub-slot size takes the full
    refresh."""
    from fhe_mamba_b200 import CCParams, CryptoContext
    cc = CryptoContext(CCParams(ring_dim=1 << 12, multiplicative_depth=25, scaling_mod_size=59,
                                first_mod_size=60, num_large_digits=3))
    cc.KeyGen(SEED)
    cc.EvalBootstrapSetup((4, 4))
    cc.EvalBootstrapSubslotSetup(512, (4, 4))
    cc.EvalBootstrapSubslotSetup(256, (4, 4))
    cc.EvalBootstrapKeyGen()
    assert cc.subslot_sizes == (256, 512)
    r = np.random.default_rng(41)
    for support, n, cplx in ((200, 256, False), (512, 512, False), (300, 512, True), (1000, 0, False)):
        x = np.zeros(cc.slots, dtype=complex)
        x[:support] = r.uniform(-5, 5, support) + (1j * r.uniform(-5, 5, support) if cplx else 0)
        ct = cc.Encrypt(cc.MakeCKKSPackedPlaintext(x if cplx else x.real))
        cc.LevelReduceInPlace(ct, cc.n_q - 4)
        full = cc.EvalRefresh(ct, 8.0, passes=2)
        for passes, tol in ((1, 1e-3), (2, 1e-5)):
            out = cc.EvalRefresh(ct, 8.0, passes=passes, support=support)
            ref = cc.EvalRefresh(ct, 8.0, passes=passes)
            assert out.n_limbs() == ref.n_limbs(), (support, passes)
            y = cc.Decrypt(out).GetCKKSPackedValue()
            if not cplx:
                y = y.real
            assert np.max(np.abs(y[:support] - x[:support])) < tol, (support, passes)
            if n:
                assert np.max(np.abs(y[n:])) < tol, (support, passes)
        yf = cc.Decrypt(full).GetCKKSPackedValue()
        assert np.max(np.abs((yf if cplx else yf.real) - x)) < 1e-5
    cc.close()


def test_subslot_refresh_in_sparse_context():
    """A sparsely packed context (1024 of N/2 = 2048 slots, the classical-128
    layout at a small ring) takes sub-slot refreshes too: 256 slots, values
    back on [0, support) within the two-pass precision, zeros from 256 on,
    the limbs of the context's own refresh."""
    from fhe_mamba_b200 import CCParams, CryptoContext, InvalidArgument
    cc = CryptoContext(CCParams(ring_dim=1 << 12, multiplicative_depth=25, scaling_mod_size=59,
                                first_mod_size=60, num_large_digits=3, batch_size=1024))
    assert cc.slots == 1024
    cc.KeyGen(SEED)
    cc.EvalBootstrapSetup((4, 4))
    cc.EvalBootstrapSubslotSetup(256, (4, 4))
    with pytest.raises(InvalidArgument):
        cc.EvalBootstrapSubslotSetup(1024, (4, 4))  # above half the slots
    cc.EvalBootstrapKeyGen()
    x = np.zeros(cc.slots)
    x[:200] = np.random.default_rng(43).uniform(-5, 5, 200)
    ct = cc.Encrypt(cc.MakeCKKSPackedPlaintext(x))
    cc.LevelReduceInPlace(ct, cc.n_q - 4)
    out = cc.EvalRefresh(ct, 8.0, passes=2, support=200)
    assert out.n_limbs() == cc.EvalRefresh(ct, 8.0, passes=2).n_limbs()
    y = cc.Decrypt(out).GetRealPackedValue()
    assert np.max(np.abs(y[:200] - x[:200])) < 1e-5 and np.max(np.abs(y[256:])) < 1e-5
    cc.close()


def test_bootstrap_at_token_loop_parameters():
    """The token loop's own parameter set (N = 2^16, 2^15 slots, depth 44,
    59/60-bit primes, dnum 3, level budget {4, 4}, uniform ternary secret): a
    2-limb input comes back with 24 limbs within 5e-4 (one bootstrap), and a
    two-pass refresh of values up to a bound of 4 within 1e-5."""
    from fhe_mamba_b200 import CCParams, CryptoContext
    cc = CryptoContext(CCParams(ring_dim=1 << 16, multiplicative_depth=44, scaling_mod_size=59,
                                first_mod_size=60, num_large_digits=3))
    cc.KeyGen(SEED)
    cc.EvalBootstrapSetup((4, 4))
    cc.EvalBootstrapSubslotSetup(4096, (3, 3))
    cc.EvalBootstrapKeyGen()
    x = np.random.default_rng(16).uniform(-1, 1, cc.slots)
    ct = cc.Encrypt(cc.MakeCKKSPackedPlaintext(x))
    cc.LevelReduceInPlace(ct, cc.n_q - 2)
    out = cc.EvalBootstrap(ct)
    assert out.n_limbs() == 24
    assert np.max(np.abs(cc.Decrypt(out).GetRealPackedValue() - x)) < 5e-4
    ct4 = cc.Encrypt(cc.MakeCKKSPackedPlaintext(4 * x))
    cc.LevelReduceInPlace(ct4, cc.n_q - 6)  # 6 limbs: the scaling by 1 / bound and two passes
    two_ct = cc.EvalRefresh(ct4, 4.0, passes=2)
    two = cc.Decrypt(two_ct).GetRealPackedValue()
    assert np.max(np.abs(two - 4 * x)) < 1e-5
    # the sub-slot refresh (level budget {3, 3}: two more limbs) of the same
    # values cut to the in_proj width
    v = np.zeros(cc.slots)
    v[:3352] = 4 * x[:3352]
    cv = cc.Encrypt(cc.MakeCKKSPackedPlaintext(v))
    cc.LevelReduceInPlace(cv, cc.n_q - 6)
    out = cc.EvalRefresh(cv, 4.0, passes=2, support=3352)
    assert out.n_limbs() == two_ct.n_limbs() + 2
    sub = cc.Decrypt(out).GetRealPackedValue()
    assert np.max(np.abs(sub[:3352] - v[:3352])) < 1e-5 and np.max(np.abs(sub[4096:])) < 1e-5
    cc.close()
