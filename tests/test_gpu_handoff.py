"""Process-separated client and server through files (the reference's
handoff): keys and ciphertexts saved by a client context, loaded by a server
context created with the same parameters, evaluated there (including a
bootstrap) and read back by the client.  Results equal the client's own
evaluation word for word; the server can neither decrypt nor make keys."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

SEED = 2718
PARAMS = dict(ring_dim=1 << 12, multiplicative_depth=25, scaling_mod_size=59, first_mod_size=60,
              num_large_digits=3)


def test_client_server_handoff(tmp_path):
    from fhe_mamba_b200 import CCParams, CryptoContext, InvalidArgument, StateError
    client = CryptoContext(CCParams(**PARAMS))
    client.KeyGen(SEED)
    client.EvalRotateKeyGen([1, -2])
    client.EvalBootstrapSetup((4, 4))
    client.EvalBootstrapKeyGen()
    client.SerializeKeys(tmp_path / "eval.keys")
    client.SerializeKeys(tmp_path / "client.keys", include_secret=True)
    x = np.random.default_rng(3).uniform(-1, 1, client.slots)
    ct = client.Encrypt(client.MakeCKKSPackedPlaintext(x))
    client.SerializeCiphertext(ct, tmp_path / "in.ct")

    server = CryptoContext(CCParams(**PARAMS))
    server.DeserializeKeys(tmp_path / "eval.keys")
    server.EvalBootstrapSetup((4, 4))
    server.EvalBootstrapKeyGen()  # every key is in the bundle: nothing generated
    a = server.DeserializeCiphertext(tmp_path / "in.ct")
    assert np.array_equal(a.residues(), ct.residues())
    y = server.EvalRotate(server.EvalMult(a, a), 1)
    low = y.Clone()
    server.LevelReduceInPlace(low, low.n_limbs() - 3)
    z = server.EvalBootstrap(low)
    server.SerializeCiphertext(y, tmp_path / "y.ct")
    server.SerializeCiphertext(z, tmp_path / "z.ct")
    with pytest.raises(StateError):
        server.Decrypt(a)
    with pytest.raises(StateError):
        server.EvalRotateKeyGen([5])

    want = client.EvalRotate(client.EvalMult(ct, ct), 1)
    got = client.DeserializeCiphertext(tmp_path / "y.ct")
    assert np.array_equal(got.residues(), want.residues())
    assert np.max(np.abs(client.Decrypt(got).GetRealPackedValue() - np.roll(x * x, -1))) < 1e-4
    zb = client.Decrypt(client.DeserializeCiphertext(tmp_path / "z.ct")).GetRealPackedValue()
    assert np.max(np.abs(zb - np.roll(x * x, -1))) < 2e-4

    # a restored client (bundle with the secret) decrypts the same values
    again = CryptoContext(CCParams(**PARAMS))
    again.DeserializeKeys(tmp_path / "client.keys")
    assert np.array_equal(again.Decrypt(got).residues(), client.Decrypt(got).residues())

    # files only load into a context with the same parameters, and intact
    other = CryptoContext(CCParams(**dict(PARAMS, multiplicative_depth=20)))
    with pytest.raises(InvalidArgument):
        other.DeserializeCiphertext(tmp_path / "in.ct")
    raw = bytearray((tmp_path / "in.ct").read_bytes())
    raw[200] ^= 1
    (tmp_path / "bad.ct").write_bytes(bytes(raw))
    with pytest.raises(InvalidArgument):
        server.DeserializeCiphertext(tmp_path / "bad.ct")
