"""CUDA CKKS path (through the C ABI) against the CPU oracle, word for word.

Keys are sampled on the device from the same ChaCha20 streams the oracle uses,
so identical seeds give identical keys; every primitive is then compared on
identical inputs.  Shapes: BASELINE config 1 (N=2^14, 1x60 + 8x50-bit Q,
dnum 2) and the config-3 key-switch shape (N=2^16, 20 limbs, dnum 3).
Decrypted values are checked against plaintext math as a second level.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

SEED = 1234


def _setup(oracle, log_n, depth, scale_bits, first_bits, dnum):
    from fhe_mamba_b200 import CCParams, CryptoContext
    cc = CryptoContext(CCParams(ring_dim=1 << log_n, multiplicative_depth=depth, scaling_mod_size=scale_bits,
                                first_mod_size=first_bits, num_large_digits=dnum))
    oq, op = oracle.ckks_moduli(log_n, depth + 1, scale_bits, first_bits, dnum)
    assert cc.q == oq and cc.p == op
    oc = oracle.Ckks(log_n, cc.q, cc.p, dnum, cc.slots)
    cc.KeyGen(SEED)
    s, sn = oc.keygen_secret(SEED)
    return cc, oc, s, sn


@pytest.fixture(scope="module")
def cfg1(oracle):
    return _setup(oracle, 14, 8, 50, 60, 2)


def _msg(n, seed, cplx=False):
    r = np.random.default_rng(seed)
    v = r.uniform(-1, 1, n)
    return v + 1j * r.uniform(-1, 1, n) if cplx else v


def test_keys_match_oracle(cfg1):
    cc, oc, s, sn = cfg1
    assert np.array_equal(cc.key(0).reshape(sn.shape), sn)
    pk = oc.keygen_public(SEED, sn)
    assert np.array_equal(cc.key(1).reshape(pk.shape), pk)
    rlk = oc.relin_key(SEED, sn)
    assert np.array_equal(cc.key(2).reshape(rlk.shape), rlk)
    for step in (1, -1, 7):
        g = cc.galois_element(step)
        assert g == oc.galois(step)
        cc.EvalRotateKeyGen([step])
        rk = oc.rot_key(SEED, s, sn, g)
        assert np.array_equal(cc.key(3, g).reshape(rk.shape), rk)


def test_encode_matches_oracle_and_decodes(cfg1):
    cc, oc, s, sn = cfg1
    for nq in (oc.L, 4):
        z = _msg(cc.slots, 3 + nq, cplx=True)
        scale = cc.level_scale(nq)
        pt = cc.MakeCKKSPackedPlaintext(z, level=oc.L - nq)
        want = oc.encode(z, scale, nq)
        assert np.array_equal(pt.residues(), want)
        out = pt.GetCKKSPackedValue()
        assert np.max(np.abs(out - z)) < 1e-9


def test_encrypt_decrypt_matches_oracle(cfg1):
    cc, oc, s, sn = cfg1
    from fhe_mamba_b200 import CCParams, CryptoContext
    # fresh context so the device encryption nonce starts at 1
    c2 = CryptoContext(CCParams(ring_dim=cc.n, multiplicative_depth=oc.L - 1, scaling_mod_size=50,
                                first_mod_size=60, num_large_digits=2))
    c2.KeyGen(SEED)
    pk = oc.keygen_public(SEED, sn)
    z = _msg(c2.slots, 5)
    pt = c2.MakeCKKSPackedPlaintext(z)
    ct = c2.Encrypt(pt)
    want = oc.encrypt(SEED, 1, pk, pt.residues(), oc.L)
    assert np.array_equal(ct.residues(), want)
    dec = c2.Decrypt(ct)
    assert np.array_equal(dec.residues(), oc.decrypt(sn, want))
    assert np.max(np.abs(dec.GetRealPackedValue() - z)) < 1e-6


def _rand_ct(oc, nq, seed, ncomp=2):
    rng = np.random.default_rng(seed)
    x = np.empty((ncomp, nq, oc.n), dtype=np.uint64)
    for l in range(nq):
        x[:, l, :] = rng.integers(0, oc.q[l], size=(ncomp, oc.n), dtype=np.uint64)
    return x


def test_tensor_relinearize_rescale_match_oracle(cfg1):
    cc, oc, s, sn = cfg1
    rlk = oc.relin_key(SEED, sn)
    for nq in (oc.L, 7, 5, 3):
        a, b = _rand_ct(oc, nq, 10 + nq), _rand_ct(oc, nq, 20 + nq)
        ga, gb = cc.upload(a), cc.upload(b)
        d = cc.EvalMultNoRelin(ga, gb)
        want_d = oc.tensor(a, b)
        assert np.array_equal(d.residues(), want_d), nq
        r = cc.Relinearize(d)
        want_r = oc.relinearize(want_d, rlk)
        assert np.array_equal(r.residues(), want_r), nq
        cc.RescaleInPlace(r)
        assert np.array_equal(r.residues(), oc.rescale(want_r)), nq


def test_rotation_and_hoisting_match_oracle(cfg1):
    cc, oc, s, sn = cfg1
    steps = [1, 2, -1, 7]
    cc.EvalRotateKeyGen(steps)
    for nq in (oc.L, 4):
        a = _rand_ct(oc, nq, 30 + nq)
        ga = cc.upload(a)
        hoisted = cc.EvalFastRotation(ga, steps)
        for st, h in zip(steps, hoisted):
            g = cc.galois_element(st)
            want = oc.rotate(a, g, oc.rot_key(SEED, s, sn, g))
            assert np.array_equal(cc.EvalRotate(ga, st).residues(), want), (nq, st)
            assert np.array_equal(h.residues(), want), (nq, st)


def test_config1_rotation_sweep_matches_oracle(cfg1):
    """BASELINE config 1's HRotate by {1, 2, 4, ..., 4096}: every rotation key
    and every rotated ciphertext word for word against the oracle at the top
    level, and the decrypted slots equal the rotated message."""
    cc, oc, s, sn = cfg1
    steps = [1 << k for k in range(13)]
    cc.EvalRotateKeyGen(steps)
    a = _rand_ct(oc, oc.L, 4096)
    ga = cc.upload(a)
    x = _msg(cc.slots, 4097)
    cx = cc.Encrypt(cc.MakeCKKSPackedPlaintext(x))
    for st in steps:
        g = cc.galois_element(st)
        assert g == oc.galois(st)
        rk = oc.rot_key(SEED, s, sn, g)
        assert np.array_equal(cc.key(3, g).reshape(rk.shape), rk), st
        assert np.array_equal(cc.EvalRotate(ga, st).residues(), oc.rotate(a, g, rk)), st
        got = cc.Decrypt(cc.EvalRotate(cx, st)).GetRealPackedValue()
        assert np.max(np.abs(got - np.roll(x, -st))) < 1e-4, st


def test_conjugate_matches_oracle(cfg1):
    cc, oc, s, sn = cfg1
    cc.EvalConjugateKeyGen()
    g = 2 * oc.n - 1
    a = _rand_ct(oc, oc.L, 77)
    want = oc.rotate(a, g, oc.rot_key(SEED, s, sn, g))
    assert np.array_equal(cc.EvalConjugate(cc.upload(a)).residues(), want)


def test_encrypted_arithmetic_decrypts(cfg1):
    cc, oc, s, sn = cfg1
    x, y = _msg(cc.slots, 41), _msg(cc.slots, 42)
    cx = cc.Encrypt(cc.MakeCKKSPackedPlaintext(x))
    cy = cc.Encrypt(cc.MakeCKKSPackedPlaintext(y))
    def dec(c):
        return cc.Decrypt(c).GetRealPackedValue()
    assert np.max(np.abs(dec(cc.EvalAdd(cx, cy)) - (x + y))) < 1e-5
    assert np.max(np.abs(dec(cc.EvalSub(cx, cy)) - (x - y))) < 1e-5
    m = cc.EvalMult(cx, cy)
    assert m.GetNoiseScaleDeg() == 2
    assert np.max(np.abs(dec(m) - x * y)) < 1e-4
    m2 = cc.EvalMult(m, cx)  # auto-rescale of the degree-2 input
    assert np.max(np.abs(dec(m2) - x * y * x)) < 1e-4
    assert np.max(np.abs(dec(cc.EvalAdd(m2, cy)) - (x * y * x + y))) < 1e-4  # level alignment
    assert np.max(np.abs(dec(cc.EvalMult(cx, 0.75)) - 0.75 * x)) < 1e-5
    assert np.max(np.abs(dec(cc.EvalAdd(cx, -0.5)) - (x - 0.5))) < 1e-5
    pw = cc.MakeCKKSPackedPlaintext(y)
    assert np.max(np.abs(dec(cc.EvalMult(cx, pw)) - x * y)) < 1e-4
    cc.EvalRotateKeyGen([3])
    assert np.max(np.abs(dec(cc.EvalRotate(cx, 3)) - np.roll(x, -3))) < 1e-4


def test_errors_are_reported(cfg1):
    from fhe_mamba_b200 import FheError, InvalidArgument, StateError
    cc, oc, s, sn = cfg1
    x = cc.Encrypt(cc.MakeCKKSPackedPlaintext(_msg(cc.slots, 1)))
    with pytest.raises(StateError):
        cc.EvalRotate(x, 12345)  # no key generated for this step
    with pytest.raises(InvalidArgument):
        cc.MakeCKKSPackedPlaintext(np.zeros(cc.slots + 1))
    y = x.Clone()
    cc.LevelReduceInPlace(y, oc.L - 1)
    with pytest.raises(StateError):
        cc.RescaleInPlace(y)
    with pytest.raises(FheError):
        cc.MakeCKKSPackedPlaintext(np.full(4, 1e30))
    # encodes return without waiting for the device unless a value could be
    # rejected: non-finite values still raise at the call, batched ones too,
    # and the next encode after an error is clean
    for bad in (np.inf, -np.inf, np.nan):
        v = np.zeros(8)
        v[3] = bad
        with pytest.raises(FheError):
            cc.MakeCKKSPackedPlaintext(v)
        with pytest.raises(FheError):
            cc.MakeCKKSPackedPlaintexts(np.stack([np.zeros(8), v]))
    z = _msg(cc.slots, 2)
    assert np.max(np.abs(cc.MakeCKKSPackedPlaintext(z).GetRealPackedValue() - z)) < 1e-9


def test_config3_keyswitch_shape(oracle):
    """N=2^16, 20 active limbs, dnum 3 (alpha 7): relinearisation and a hoisted
    rotation batch equal the oracle on random ciphertexts."""
    cc, oc, s, sn = _setup(oracle, 16, 19, 59, 60, 3)
    assert cc.n_q == 20 and cc.alpha == 7
    rlk = oc.relin_key(SEED, sn)
    a = _rand_ct(oc, 20, 5, ncomp=3)
    got = cc.Relinearize(cc.upload(a, noise_deg=2)).residues()
    assert np.array_equal(got, oc.relinearize(a, rlk))
    steps = [1, 5]
    cc.EvalRotateKeyGen(steps)
    b = _rand_ct(oc, 20, 6)
    outs = cc.EvalFastRotation(cc.upload(b), steps)
    for st, o in zip(steps, outs):
        g = cc.galois_element(st)
        assert np.array_equal(o.residues(), oc.rotate(b, g, oc.rot_key(SEED, s, sn, g)))


def test_encode_values_beyond_2_62(cfg1):
    """Scaled coefficients above 2^63 are encoded exactly (integer-valued doubles
    split into 64-bit halves before the RNS lift)."""
    cc, oc, s, sn = cfg1
    r = np.random.default_rng(5)
    big = r.uniform(-1, 1, cc.slots) * 3e6  # x 2^50 scale -> coefficients near 2^70
    pt = cc.MakeCKKSPackedPlaintext(big)
    assert np.max(np.abs(pt.GetRealPackedValue() - big)) < 1e-6 * 3e6
    x = _msg(cc.slots, 6)
    ct = cc.EvalAdd(cc.Encrypt(cc.MakeCKKSPackedPlaintext(x)), pt)
    assert np.max(np.abs(cc.Decrypt(ct).GetRealPackedValue() - (x + big))) < 1e-5 * 3e6


def test_wide_digit_keyswitch(oracle):
    """Depth 44, dnum 3 (15-limb digits, 15 special primes: the token loop's
    key-switching shape) at N=2^13: relinearisation and a rotation equal the
    oracle word for word at the top level and two lower levels."""
    cc, oc, s, sn = _setup(oracle, 13, 44, 59, 60, 3)
    assert cc.alpha == 15 and cc.n_p == 15
    rlk = oc.relin_key(SEED, sn)
    cc.EvalRotateKeyGen([3])
    g = cc.galois_element(3)
    rk = oc.rot_key(SEED, s, sn, g)
    for nq in (45, 31, 16):
        a = _rand_ct(oc, nq, 300 + nq, ncomp=3)
        got = cc.Relinearize(cc.upload(a, noise_deg=2)).residues()
        assert np.array_equal(got, oc.relinearize(a, rlk)), nq
        b = _rand_ct(oc, nq, 400 + nq)
        assert np.array_equal(cc.EvalRotate(cc.upload(b), 3).residues(), oc.rotate(b, g, rk)), nq


@pytest.mark.parametrize("shape", ["config1", "config3", "depth44"])
def test_tensor_core_conversion_matches_oracle(oracle, shape):
    """The key switch with its ModUp and ModDown basis conversions on the
    tensor cores (tcgen05 int8 MMA over byte-split residues) and with the Q
    limbs' key inner product fused into ModDown's last NTT pass:
    relinearisation, a rotation and hoisted rotations word for word against
    the oracle and against the CUDA-core, unfused key switch, at config 1
    (5 + 5 limbs), the config-3 shape (digits of 7 and 6 limbs) and the token
    loop's 45 + 15 limbs."""
    from fhe_mamba_b200 import _lib
    args = {"config1": (14, 8, 50, 60, 2), "config3": (16, 19, 59, 60, 3), "depth44": (16, 44, 59, 60, 3)}[shape]
    cc, oc, s, sn = _setup(oracle, *args)
    rng = np.random.default_rng(77)
    nq = cc.n_q if shape != "depth44" else 31
    d = np.empty((3, nq, cc.n), dtype=np.uint64)
    for l in range(nq):
        d[:, l, :] = rng.integers(0, cc.q[l], size=(3, cc.n), dtype=np.uint64)
    steps = [1, -3]
    cc.EvalRotateKeyGen(steps)
    out = {}
    for kernel in ("cuda", "tensor-all"):
        for fused in (False, True):
            cc.SetConversionKernel(kernel)
            cc.SetKeySwitchFusion(fused)
            ct2 = cc.upload(d[:2])
            out[kernel, fused] = ([cc.Relinearize(cc.upload(d, noise_deg=2)).residues(),
                                   cc.EvalRotate(ct2, 1).residues()] +
                                  [h.residues() for h in cc.EvalFastRotation(ct2, steps)])
    cc.SetConversionKernel("cuda")
    cc.SetKeySwitchFusion(False)
    for key in out:
        for a, b in zip(out["cuda", False], out[key]):
            assert np.array_equal(a, b), key
    out["tensor-all"] = out["tensor-all", True]
    assert np.array_equal(out["tensor-all"][0], oc.relinearize(d, oc.relin_key(SEED, sn)))
    g = cc.galois_element(1)
    assert np.array_equal(out["tensor-all"][1], oc.rotate(d[:2], g, oc.rot_key(SEED, s, sn, g)))
    n = ctypes_u64()
    _lib.call("fhe_tc_timeouts", ctypes.byref(n))
    assert n.value == 0
    cc.close()


def ctypes_u64():
    import ctypes
    return ctypes.c_uint64()
