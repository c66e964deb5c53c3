"""One encrypted Mamba-2 decode layer (BASELINE config 4 structure at a reduced
width) against the plaintext polynomial path, over two tokens so that the conv
FIFO and the recurrent state are carried; bootstrapping refreshes values
inside the layer."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_two_tokens_match_plaintext_polynomial_path():
    from fhe_mamba_b200 import CCParams, CryptoContext
    from fhe_mamba_b200.mamba2_layer import (EncryptedMamba2Layer, Mamba2Polys, Mamba2Weights, calibrate_bounds,
                                             plain_step)
    W = Mamba2Weights(d_model=64, d_state=32, heads=16, std=0.1)
    P = Mamba2Polys(W)
    bounds = calibrate_bounds(W, P)
    cc = CryptoContext(CCParams(ring_dim=1 << 12, multiplicative_depth=44, scaling_mod_size=59,
                                first_mod_size=60, num_large_digits=3))
    cc.KeyGen(31)
    cc.EvalBootstrapSetup((4, 4))
    cc.EvalBootstrapKeyGen()
    layer = EncryptedMamba2Layer(cc, W, P)
    cc.EvalRotateKeyGen(layer.rotation_steps())
    rng = np.random.default_rng(12)
    conv_p = [np.zeros(W.conv_dim) for _ in range(W.conv_kernel - 1)]
    conv_c = [None] * (W.conv_kernel - 1)
    st_p, st_c = None, None
    for token in range(2):
        h = rng.normal(0, 1, W.d_model)
        want, conv_p, st_p = plain_step(W, P, h, conv_p, st_p)
        hc = cc.Encrypt(cc.MakeCKKSPackedPlaintext(np.pad(h, (0, cc.slots - h.size))))
        out, conv_c, st_c = layer.step(hc, conv_c, st_c, bounds)
        got = cc.Decrypt(out).GetRealPackedValue()[:W.d_model]
        err = np.max(np.abs(got - want))
        assert err < 2e-3, (token, err)
    assert layer.refreshes >= 1
