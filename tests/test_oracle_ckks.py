"""CKKS semantics of the CPU oracle, checked by decryption against plaintext math.

These pin the oracle's algorithms (encode/decode, public-key encryption, HYBRID
key switching, relinearisation, FLEXIBLEAUTO rescale, rotations, hoisting
identity) before the GPU path is compared to it word for word.
"""
import numpy as np
import pytest


@pytest.fixture(scope="module")
def ck(oracle):
    # BASELINE config 1 shape, reduced ring: 1 x 60-bit + 8 x 50-bit, dnum 2.
    q, p = oracle.ckks_moduli(11, 9, 50, 60, 2)
    c = oracle.Ckks(11, q, p, 2, 1 << 10)
    s, sn = c.keygen_secret(11)
    pk = c.keygen_public(12, sn)
    rlk = c.relin_key(13, sn)
    return c, s, sn, pk, rlk


def _msg(n, seed):
    return np.random.default_rng(seed).uniform(-1, 1, n)


def test_encode_decode_roundtrip(ck):
    c, *_ = ck
    z = _msg(c.slots, 1)
    pt = c.encode(z, 2.0**40, c.L)
    out = c.decode(pt, c.L, 2.0**40)
    assert np.max(np.abs(out.real - z)) < 1e-9
    assert np.max(np.abs(out.imag)) < 1e-9


def test_encrypt_decrypt(ck):
    c, s, sn, pk, rlk = ck
    z = _msg(c.slots, 2)
    scale = float(c.q[-1])
    ct = c.encrypt(7, 1, pk, c.encode(z, scale, c.L), c.L)
    out = c.decode(c.decrypt(sn, ct), c.L, scale)
    assert np.max(np.abs(out.real - z)) < 1e-9


def test_add_mult_relin_rescale(ck):
    c, s, sn, pk, rlk = ck
    a, b = _msg(c.slots, 3), _msg(c.slots, 4)
    scale = float(c.q[-1])
    L = c.L
    ca = c.encrypt(7, 2, pk, c.encode(a, scale, L), L)
    cb = c.encrypt(7, 3, pk, c.encode(b, scale, L), L)
    s_add = c.decode(c.decrypt(sn, c.add(ca, cb)), L, scale)
    assert np.max(np.abs(s_add.real - (a + b))) < 1e-8
    d3 = c.tensor(ca, cb)
    m3 = c.decode(c.decrypt(sn, d3), L, scale * scale)
    assert np.max(np.abs(m3.real - a * b)) < 1e-8
    ct = c.relinearize(d3, rlk)
    m2 = c.decode(c.decrypt(sn, ct), L, scale * scale)
    assert np.max(np.abs(m2.real - a * b)) < 1e-7
    r = c.rescale(ct)
    new_scale = scale * scale / c.q[L - 1]
    mr = c.decode(c.decrypt(sn, r), L - 1, new_scale)
    assert np.max(np.abs(mr.real - a * b)) < 1e-7


def test_keyswitch_lower_level(ck):
    c, s, sn, pk, rlk = ck
    a = _msg(c.slots, 5)
    scale = 2.0**45
    nq = 5  # partial last digit (alpha = 5 -> digits of 5 limbs; level 5 = one digit)
    for nq in (5, 7):
        ca = c.encrypt(9, 10 + nq, pk, c.encode(a, scale, nq), nq)
        d3 = c.tensor(ca, ca)
        ct = c.relinearize(d3, rlk)
        m2 = c.decode(c.decrypt(sn, ct), nq, scale * scale)
        assert np.max(np.abs(m2.real - a * a)) < 1e-6, nq


def test_rotation_and_conjugation(ck):
    c, s, sn, pk, rlk = ck
    z = _msg(c.slots, 6)
    scale = 2.0**40
    ct = c.encrypt(3, 4, pk, c.encode(z, scale, c.L), c.L)
    for r in (1, 5, -3, c.slots // 2):
        g = c.galois(r)
        rk = c.rot_key(21, s, sn, g)
        out = c.decode(c.decrypt(sn, c.rotate(ct, g, rk)), c.L, scale)
        assert np.max(np.abs(out.real - np.roll(z, -r))) < 1e-6, r
    g = 2 * c.n - 1
    ck_ = c.rot_key(21, s, sn, g)
    zc = _msg(c.slots, 7) + 1j * _msg(c.slots, 8)
    ct = c.encrypt(3, 5, pk, c.encode(zc, scale, c.L), c.L)
    out = c.decode(c.decrypt(sn, c.rotate(ct, g, ck_)), c.L, scale)
    assert np.max(np.abs(out - np.conj(zc))) < 1e-6


def test_hoisted_rotation_is_bit_identical(ck):
    """Rotation = key switch of c1, then the automorphism (OpenFHE order).  So a
    hoisted rotation — one ModUp of c1 shared by all steps, then per step the
    key inner product, ModDown and the automorphism — gives the same words as
    the plain rotation (what EvalFastRotationPrecompute/EvalFastRotation rely on)."""
    c, s, sn, pk, rlk = ck
    z = _msg(c.slots, 9)
    nq = c.L
    ct = c.encrypt(3, 6, pk, c.encode(z, 2.0**40, nq), nq)
    ext = c.modup(ct[1], nq)
    for r in (1, 3, -2):
        g = c.galois(r)
        rk = c.rot_key(21, s, sn, g)
        plain = c.rotate(ct, g, rk)
        acc = c.key_inner(ext, nq, rk)
        u0 = c.add(ct[0][None], c.moddown(acc[0], nq)[None])[0]
        u1 = c.moddown(acc[1], nq)
        hoisted = np.stack([c.automorphism(u0, g), c.automorphism(u1, g)])
        assert np.array_equal(hoisted, plain), r


def test_rescale_matches_exact_division(ck, oracle):
    """Rescale = round-towards-centred-lift division of the CRT value by q_last."""
    c, *_ = ck
    nq = 3
    rng = np.random.default_rng(3)
    vals = rng.integers(-2**40, 2**40, size=c.n)
    x = c.zeros(1, nq)
    for l in range(nq):
        x[0, l] = np.array([int(v) % c.q[l] for v in vals], dtype=np.uint64)
    c.ntt(x[0], nq)
    y = c.rescale(x)
    c.ntt(y[0], nq - 1, inverse=True)
    ql = c.q[nq - 1]
    for k in range(0, c.n, 97):
        v = int(vals[k])
        r = v % ql
        if r > ql // 2:
            r -= ql
        want = (v - r) // ql
        for l in range(nq - 1):
            assert int(y[0, l, k]) == want % c.q[l]
