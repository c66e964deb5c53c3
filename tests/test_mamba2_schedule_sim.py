"""The synthetic Mamba-2 layer and token loop (mamba2_layer.py: BASELINE
configs 4 and 5, the bench's token loop) on the slot-level model of the
CryptoContext API (tests/slot_sim.py): masks, rotations, replicated BSGS
layouts, level budgeting and refresh bounds of the host schedule, at the
config-4 shape (d_model 768, 24 heads x 64, d_state 128, 2^15 slots).
Without bootstrap noise the schedule reproduces the fp64 polynomial path to
rounding; every rotation must find a generated key and every refresh input
must sit inside its bound.  No GPU."""
import numpy as np

from slot_sim import SlotContext


def test_config4_layer_schedule():
    from fhe_mamba_b200.mamba2_layer import (EncryptedMamba2Layer, Mamba2Polys, Mamba2Weights, calibrate_bounds,
                                             plain_step)
    W = Mamba2Weights(d_model=768, d_state=128, heads=24)
    P = Mamba2Polys(W, samples=2)
    bounds = calibrate_bounds(W, P, samples=2)
    cc = SlotContext(1 << 15, refresh_noise=0.0)
    layer = EncryptedMamba2Layer(cc, W, P)
    cc.EvalRotateKeyGen(layer.rotation_steps())
    rng = np.random.default_rng(12)
    conv_p = [np.zeros(W.conv_dim) for _ in range(W.conv_kernel - 1)]
    conv_c = [None] * (W.conv_kernel - 1)
    st_p = st_c = None
    for _ in range(2):
        h = rng.normal(0, 1, W.d_model)
        want, conv_p, st_p = plain_step(W, P, h, conv_p, st_p)
        out, conv_c, st_c = layer.step(cc.Encrypt(cc.MakeCKKSPackedPlaintext(h)), conv_c, st_c, bounds)
        assert np.max(np.abs(cc.Decrypt(out).GetRealPackedValue()[:W.d_model] - want)) < 1e-10
    assert layer.refreshes >= 1 and cc.max_refresh_ratio <= 1.0


def test_token_loop_schedule():
    """The 2-layer greedy loop of the GPU test at its shape: same tokens, same hidden vectors."""
    from fhe_mamba_b200.mamba2_layer import EncryptedMamba2Model, Mamba2Model
    m = Mamba2Model(layers=2, d_model=64, d_state=32, heads=16, vocab=128, std=0.1)
    cc = SlotContext(2048, refresh_noise=0.0)
    em = EncryptedMamba2Model(cc, m)
    cc.EvalRotateKeyGen(em.rotation_steps())
    state = m.initial_state()
    for tok in (3, 17, 5):
        hf, logits, state = m.plain_token(tok, state)
        picked, ehf = em.select(em.step(tok))
        assert picked == int(np.argmax(logits)) and np.max(np.abs(ehf - hf)) < 1e-10
    assert em.refreshes() >= 1 and cc.max_refresh_ratio <= 1.0


def test_fused_decay():
    """decay = exp(a_h softplus(x)) as one per-head series of the raw dt input
    (HeadPoly, off by default): accurate over the whole softplus domain, exact
    against its own plaintext circuit on the slot model, and one refresh per
    layer and token fewer than exp of a * softplus (no refresh of a * dt)."""
    from fhe_mamba_b200.mamba2_layer import (EncryptedMamba2Model, HeadPoly, Mamba2Model, Mamba2Polys,
                                             Mamba2Weights, _softplus)
    W = Mamba2Weights(d_model=768, d_state=128, heads=24, seed=6000)
    P = Mamba2Polys(W, samples=2, fused_decay=True)
    assert isinstance(P.decay, HeadPoly) and P.decay.coeffs.shape == (32, 24) and P.decay.levels == 7
    x = np.linspace(P.softplus.lo, P.softplus.hi, 2001)
    want = np.exp(W["a"][None, :] * _softplus(x)[:, None])
    assert np.max(np.abs(P.decay(x[:, None]) - want)) < 1e-4
    counts = {}
    for fused in (False, True):
        m = Mamba2Model(layers=2, d_model=64, d_state=32, heads=16, vocab=128, std=0.1, fused_decay=fused)
        cc = SlotContext(2048, refresh_noise=0.0)
        em = EncryptedMamba2Model(cc, m)
        cc.EvalRotateKeyGen(em.rotation_steps())
        state = m.initial_state()
        for tok in (3, 17, 5):
            hf, logits, state = m.plain_token(tok, state)
            picked, ehf = em.select(em.step(tok))
            assert picked == int(np.argmax(logits)) and np.max(np.abs(ehf - hf)) < 1e-10
        assert cc.max_refresh_ratio <= 1.0
        counts[fused] = em.refreshes()
    assert counts[True] < counts[False]


def test_subslot_refresh_schedule():
    """Refreshes over fewer slots (EvalBootstrapSubslotSetup): every site that
    declares a support is zero outside it (the slot model raises otherwise and
    returns the sum of the input's n-periodic copies, as the device's
    replicate-then-bootstrap does), so the loop still reproduces the fp64
    polynomial path to rounding; the carried states keep the full refresh."""
    from fhe_mamba_b200.mamba2_layer import (EncryptedMamba2Layer, EncryptedMamba2Model, Mamba2Model, Mamba2Polys,
                                             Mamba2Weights, calibrate_bounds, plain_step)
    W = Mamba2Weights(d_model=768, d_state=128, heads=24)
    P = Mamba2Polys(W, samples=2)
    bounds = calibrate_bounds(W, P, samples=2)
    cc = SlotContext(1 << 15, refresh_noise=0.0)
    cc.EvalBootstrapSubslotSetup(4096, (3, 3))
    cc.EvalBootstrapSubslotSetup(2048, (3, 3))
    layer = EncryptedMamba2Layer(cc, W, P)
    cc.EvalRotateKeyGen(layer.rotation_steps())
    rng = np.random.default_rng(12)
    conv_p = [np.zeros(W.conv_dim) for _ in range(W.conv_kernel - 1)]
    conv_c = [None] * (W.conv_kernel - 1)
    st_p = st_c = None
    for _ in range(2):
        h = rng.normal(0, 1, W.d_model)
        want, conv_p, st_p = plain_step(W, P, h, conv_p, st_p)
        out, conv_c, st_c = layer.step(cc.Encrypt(cc.MakeCKKSPackedPlaintext(h)), conv_c, st_c, bounds)
        assert np.max(np.abs(cc.Decrypt(out).GetRealPackedValue()[:W.d_model] - want)) < 1e-10
    assert cc.subslot_refreshes >= 1 and cc.max_refresh_ratio <= 1.0

    for fused in (False, True):
        m = Mamba2Model(layers=2, d_model=64, d_state=32, heads=16, vocab=128, std=0.1, fused_decay=fused)
        cc = SlotContext(2048, refresh_noise=0.0)
        cc.EvalBootstrapSubslotSetup(512)
        em = EncryptedMamba2Model(cc, m)
        cc.EvalRotateKeyGen(em.rotation_steps())
        state = m.initial_state()
        for tok in (3, 17, 5, 9):
            hf, logits, state = m.plain_token(tok, state)
            picked, ehf = em.select(em.step(tok))
            assert picked == int(np.argmax(logits)) and np.max(np.abs(ehf - hf)) < 1e-10
        assert 1 <= cc.subslot_refreshes <= em.refreshes()


def test_plaintext_memo():
    """The model's constant slot vectors (masks, taps, biases) come from the
    shared memo after the first token: same results to rounding, most lookups
    hits, and a budget too small for any entry only encodes."""
    from fhe_mamba_b200.mamba import PlaintextMemo
    from fhe_mamba_b200.mamba2_layer import EncryptedMamba2Model, Mamba2Model
    m = Mamba2Model(layers=2, d_model=64, d_state=32, heads=16, vocab=128, std=0.1, fused_decay=True)
    outs = {}
    for memo_gb in (0.0, 4.0):
        cc = SlotContext(2048, refresh_noise=0.0)
        em = EncryptedMamba2Model(cc, m, memo_gb=memo_gb)
        cc.EvalRotateKeyGen(em.rotation_steps())
        outs[memo_gb] = [em.select(em.step(tok))[1] for tok in (3, 17, 5)]
        if memo_gb:
            assert em.memo.hits > 2 * em.memo.misses and 0 < em.memo.bytes <= memo_gb * 2 ** 30
        else:
            assert em.memo is None
    for a, b in zip(outs[0.0], outs[4.0]):
        assert np.max(np.abs(a - b)) < 1e-12
    cc = SlotContext(2048, refresh_noise=0.0)
    tiny = PlaintextMemo(cc, 1.0)
    v = np.zeros(cc.slots)
    v[:5] = 1.0
    assert tiny.get(v, 3) is not tiny.get(v, 3) and tiny.misses == 2 and not tiny.entries
    memo = PlaintextMemo(cc, 2 * (cc.n_q - 3) * cc.n * 8)
    a = memo.get(v, 3)
    assert memo.get(v.copy(), 3) is a and memo.get(v, 4) is not a and memo.get(v, 3, scale=2.0) is not a
    assert len(memo.entries) == 2 and memo.bytes <= 2 * (cc.n_q - 3) * cc.n * 8


def test_subslot_supports_over_the_horizon():
    """28 greedy tokens of the small loop with sub-slot refreshes over 256 and
    512 of 2048 slots: every declared support holds on every token, through
    the carried states' own (full-slot) refreshes, and the loop stays equal to
    the fp64 polynomial path."""
    from fhe_mamba_b200.mamba2_layer import EncryptedMamba2Model, Mamba2Model
    m = Mamba2Model(layers=2, d_model=64, d_state=32, heads=16, vocab=128, std=0.1, fused_decay=True)
    cc = SlotContext(2048, refresh_noise=0.0)
    cc.EvalBootstrapSubslotSetup(512)
    cc.EvalBootstrapSubslotSetup(256)
    em = EncryptedMamba2Model(cc, m)
    cc.EvalRotateKeyGen(em.rotation_steps())
    state, tok = m.initial_state(), 3
    for _ in range(28):
        hf, logits, state = m.plain_token(tok, state)
        picked, ehf = em.select(em.step(tok))
        assert picked == int(np.argmax(logits)) and np.max(np.abs(ehf - hf)) < 1e-9
        tok = picked
    full = em.refreshes() - cc.subslot_refreshes
    assert cc.subslot_refreshes > 0 and full > 0  # the states refresh over all slots
    assert sum(layer.site_refreshes.get("state", 0) for layer in em.layers) == full
