"""Packed Mamba-2 pieces on encrypted data against the reference's plaintext formulas.

The recurrence ``S <- decay * S + (dt * x) (x) B``, readout ``y = S C`` over
the state axis (``mixer2_forward``, src/fhemamba/reference.py:182-294), the
depthwise causal conv window and ``rms_normalize`` (src/fhemamba/tensor_ops.py:53-56)
are evaluated under CKKS at N = 2^12 on a two-group state layout and compared,
after decryption, with numpy evaluations of the same formulas.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

HEADS, HD, S = 16, 8, 32
D_INNER = HEADS * HD


@pytest.fixture(scope="module")
def env():
    from fhe_mamba_b200 import CCParams, CryptoContext
    from fhe_mamba_b200.mamba import PackedMamba2, StateLayout
    cc = CryptoContext(CCParams(ring_dim=1 << 12, multiplicative_depth=20, scaling_mod_size=59,
                                first_mod_size=60, num_large_digits=3))
    cc.KeyGen(21)
    lay = StateLayout(HEADS, HD, S, cc.slots)
    pm = PackedMamba2(cc, lay, b_base=D_INNER, c_base=D_INNER + S, head_base=0)
    cc.EvalRotateKeyGen(pm.rotation_steps(norm_width=D_INNER))
    return cc, lay, pm


def _stream(cc, parts):
    v = np.zeros(cc.slots)
    for off, vals in parts:
        v[off:off + len(vals)] = vals
    return cc.Encrypt(cc.MakeCKKSPackedPlaintext(v))


def test_state_update_and_readout(env):
    cc, lay, pm = env
    rng = np.random.default_rng(1)
    state = None
    S_ref = np.zeros((HEADS, HD, S))
    for token in range(2):
        x = rng.uniform(-1, 1, (HEADS, HD))
        B, C = rng.uniform(-1, 1, S), rng.uniform(-1, 1, S)
        dt = rng.uniform(0.01, 0.5, HEADS)
        decay = np.exp(-dt * rng.uniform(0.5, 2, HEADS))
        xbc = _stream(cc, [(0, x.ravel()), (D_INNER, B), (D_INNER + S, C)])
        dt_ct = _stream(cc, [(0, dt)])
        dec_ct = _stream(cc, [(0, decay)]) if state is not None else None
        state, y = pm.step(state, xbc, dt_ct, dec_ct)
        S_ref = decay[:, None, None] * S_ref + (dt[:, None] * x)[:, :, None] * B[None, None, :]
        y_ref = (S_ref * C[None, None, :]).sum(-1)
        got = cc.Decrypt(y).GetRealPackedValue()
        assert np.max(np.abs(got[:D_INNER] - y_ref.ravel())) < 1e-5, token
        assert np.max(np.abs(got[D_INNER:])) < 1e-5  # the stream stays clean beyond its values
        packed = np.array([cc.Decrypt(s).GetRealPackedValue() for s in state])
        assert np.max(np.abs(lay.unpack(packed) - S_ref)) < 1e-5, token


def test_causal_conv_window(env):
    cc, lay, pm = env
    rng = np.random.default_rng(2)
    width, k = 96, 4
    xs = [rng.uniform(-1, 1, width) for _ in range(k)]
    w = rng.normal(0, 0.5, (k, width))
    bias = rng.normal(0, 0.1, width)
    window = [_stream(cc, [(0, x)]) for x in xs]
    out = pm.conv(window, [np.pad(wi, (0, cc.slots - width)) for wi in w], np.pad(bias, (0, cc.slots - width)))
    want = sum(w[i] * xs[i] for i in range(k)) + bias
    got = cc.Decrypt(out).GetRealPackedValue()[:width]
    assert np.max(np.abs(got - want)) < 1e-6


def test_rms_norm(env):
    cc, lay, pm = env
    rng = np.random.default_rng(3)
    x = rng.uniform(-1, 1, D_INNER)
    weight = rng.uniform(0.5, 1.5, D_INNER)
    eps = 1e-5
    ct = _stream(cc, [(0, x)])
    out = pm.rms_norm(ct, D_INNER, weight, eps, domain=(0.125, 0.625), degree=31, newton=2)
    want = x / np.sqrt(np.mean(x * x) + eps) * weight
    got = cc.Decrypt(out).GetRealPackedValue()
    assert np.max(np.abs(got[:D_INNER] - want)) < 1e-4
