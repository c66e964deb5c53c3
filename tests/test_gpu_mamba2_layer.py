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


def test_greedy_token_loop_matches_plaintext():
    """Two-layer model: prompt of 2 tokens then 2 generated tokens; the
    encrypted loop picks the same tokens as the plaintext polynomial path and
    its final hidden vectors agree."""
    from fhe_mamba_b200 import CCParams, CryptoContext
    from fhe_mamba_b200.mamba2_layer import EncryptedMamba2Model, Mamba2Model
    m = Mamba2Model(layers=2, d_model=64, d_state=32, heads=16, vocab=128, std=0.1)
    cc = CryptoContext(CCParams(ring_dim=1 << 12, multiplicative_depth=44, scaling_mod_size=59,
                                first_mod_size=60, num_large_digits=3))
    cc.KeyGen(41)
    cc.EvalBootstrapSetup((4, 4))
    cc.EvalBootstrapKeyGen()
    em = EncryptedMamba2Model(cc, m)
    cc.EvalRotateKeyGen(em.rotation_steps())
    state = m.initial_state()
    prompt, generated = [3, 17], 2
    token, plain_tokens, enc_tokens = None, [], []
    for i in range(len(prompt) + generated - 1):
        tok = prompt[i] if i < len(prompt) else token
        hf, logits, state = m.plain_token(tok, state)
        token = int(np.argmax(logits))
        enc_tok, ehf = em.select(em.step(tok))
        assert np.max(np.abs(ehf - hf)) < 1e-3, i
        if i >= len(prompt) - 1:
            plain_tokens.append(token)
            enc_tokens.append(enc_tok)
    assert enc_tokens == plain_tokens


def test_config5_protocol_horizon_matches_plaintext():
    """The config-5 protocol at a reduced width: an 8-token prompt, then 16
    greedily generated tokens fed back (23 evaluations) plus one more, so the
    recurrent state is carried over the whole horizon.  Every selection equals
    the plaintext polynomial path's and every decrypted final hidden vector
    stays within 1e-4 of it."""
    from fhe_mamba_b200 import CCParams, CryptoContext
    from fhe_mamba_b200.mamba2_layer import EncryptedMamba2Model, Mamba2Model
    m = Mamba2Model(layers=2, d_model=64, d_state=32, heads=16, vocab=128, std=0.1, calib_tokens=32)
    cc = CryptoContext(CCParams(ring_dim=1 << 12, multiplicative_depth=44, scaling_mod_size=59,
                                first_mod_size=60, num_large_digits=3))
    cc.KeyGen(43)
    cc.EvalBootstrapSetup((4, 4))
    cc.EvalBootstrapKeyGen()
    em = EncryptedMamba2Model(cc, m)
    cc.EvalRotateKeyGen(em.rotation_steps())
    prompt = [int(t) for t in np.random.default_rng(7).integers(0, 128, 8)]
    state, token, inputs, errs = m.initial_state(), None, [], []
    for i in range(24):
        tok = prompt[i] if i < len(prompt) else token
        inputs.append(tok)
        hf, logits, state = m.plain_token(tok, state)
        token = int(np.argmax(logits))
        enc_tok, ehf = em.select(em.step(tok))
        errs.append(float(np.max(np.abs(ehf - hf))))
        assert enc_tok == token, (i, em.margins[-1])
    assert max(errs) < 1e-4, errs
    assert m.audit(inputs)["max_bound_ratio"] <= 1.0


def test_device_diagonals_equal_host_diagonals():
    """The replicated BSGS diagonals generated on the device from the weights
    (fhe_encode_replicated_diagonals) equal the host-built, uploaded and encoded
    ones word for word, for both matvecs of a config-4-shape layer (in_proj
    3352 x 768, out_proj 768 x 1536) at two levels."""
    from fhe_mamba_b200 import CCParams, CryptoContext
    from fhe_mamba_b200.mamba2_layer import EncryptedMamba2Layer, Mamba2Polys, Mamba2Weights
    W = Mamba2Weights(d_model=768, d_state=128, heads=24)
    P = Mamba2Polys(W, samples=1, tokens=1)
    cc = CryptoContext(CCParams(ring_dim=1 << 16, multiplicative_depth=7, scaling_mod_size=59,
                                first_mod_size=60, num_large_digits=3))
    layer = EncryptedMamba2Layer(cc, W, P)
    for name in ("w_in", "w_out"):
        lay = layer.rep[name]
        for nq in (cc.n_q, 3):
            dev = cc.MakeReplicatedDiagonals(layer._weights_on_device(name).data_ptr(), lay.m, lay.n, lay.R, lay.T,
                                             lay.w, lay.b, level=cc.n_q - nq)
            diags = layer._diags(name)
            host = cc.MakeCKKSPackedPlaintexts(np.array([d for d in diags if d is not None]), level=cc.n_q - nq)
            assert len(dev) == len(host) == lay.T
            for t in (0, 1, lay.b, lay.T - 1):
                assert np.array_equal(dev[t].residues(), host[t].residues()), (name, nq, t)
    cc.close()
