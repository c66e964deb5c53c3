"""The Mamba-2 chain payload reader and its fp64 polynomial circuit against the
reference's own exporter output (tests/golden/mamba2_chain, written by
tests/golden/make_mamba2_chain.py with ``export_chain_payload``): weights and
nonlinearities are read as the reference's native decode reads them, and the
circuit reproduces the exporter's plaintext polynomial references
(``chain_expected_poly_final``, per-layer ``test_layer_output_poly`` and
``test_state_output_poly``, the client loop's greedy ids).  The exporter
computes in float32, this circuit in float64: the agreement bound below is
float32 rounding.  No GPU."""
import json
import math
import os
import shutil

import numpy as np
import pytest

from conftest import GOLDEN
from fhe_mamba_b200.chain_payload import (ChebSeries, ConstNewton, JointGate, PayloadError, PolyNewton,
                                          ResquaredExp, ScheduledInvSqrt, SquaredPolyNewton, SquaredSeries,
                                          chain_bounds, chebyshev_levels, initial_state, parse_joint_gate,
                                          parse_poly_spec, plain_decode, plain_token, read_chain_payload,
                                          select_token)

CHAIN = os.path.join(GOLDEN, "mamba2_chain")
JOINT = os.path.join(GOLDEN, "mamba2_chain_joint")
FP32 = 2e-5  # float32 evaluation of the exporter vs float64 here


@pytest.fixture(scope="module")
def payload():
    return read_chain_payload(CHAIN)


def test_reader(payload):
    p = payload
    assert p.n_layers == 2 and p.full_chain and p.n_test_tokens == 3 and p.d_model == 64
    w = p.layers[0].weights
    assert (w.d_inner, w.heads, w.head_dim, w.d_state, w.conv_kernel, w.conv_dim, w.proj_dim) == \
        (128, 16, 8, 32, 4, 192, 336)
    assert w["w_in"].shape == (336, 64) and w["w_out"].shape == (64, 128)
    assert np.all(w["a"] < 0)
    P0, P1 = p.layers[0].polys, p.layers[1].polys
    assert isinstance(P0.silu_x, ChebSeries) and P0.silu_x.degree == 96
    assert isinstance(P0.silu_z, ChebSeries) and P0.silu_z.degree == 64
    assert isinstance(P0.softplus, SquaredSeries) and P0.softplus.base.degree == 64
    assert isinstance(P0.rsqrt1, PolyNewton) and P0.rsqrt1.iterations == 4 and P0.rsqrt1.base.degree == 47
    assert isinstance(P0.rsqrt2, SquaredPolyNewton) and P0.rsqrt2.damping == 0.85
    # decay: head 0 pruned in both layers, one squaring in layer 1
    for P in (P0, P1):
        assert isinstance(P.exp, ResquaredExp) and P.exp.head_mask[0] == 0 and P.exp.head_mask[1:].all()
    assert P1.exp.squarings == 1
    assert p.final_norm is P1.rsqrt1  # no dedicated final_norm_poly: the last layer's block fit
    assert p.autoregressive["protocol"] == "client-in-loop-greedy-v1"
    assert p.client_embedding_w.shape == (128, 64)


def test_nonlinearities_match_reference_evaluators():
    """Every exported kind against the reference's own evaluator (float64 grid)."""
    with open(os.path.join(GOLDEN, "mamba2_nonlinearities.json")) as f:
        cases = json.load(f)
    kinds = set()
    for case in cases:
        site = case["name"].split(".")[-1] if "." in case["name"] else "rms_invsqrt"
        x, want = np.array(case["x"]), np.array(case["y"])
        if site == "gates":
            rates = np.asarray(case["spec"]["rates"])
            got = np.array(parse_joint_gate(case["spec"], rates.size, np.log(rates))(x))
        else:
            spec = parse_poly_spec(case["spec"], site)
            got = spec.inv_sqrt(x) if hasattr(spec, "inv_sqrt") else spec(x)
        assert np.allclose(got, want, rtol=1e-12, atol=1e-12 * np.max(np.abs(want))), case["name"]
        kinds.add(case["spec"]["kind"])
    assert kinds == {"cheb", "cheb-squared", "cheb-resquared", "poly-newton", "sq-poly-newton", "const-newton",
                     "scaled-goldschmidt-invsqrt-v1", "shared-dissipation-factor-v1"}


def test_chain_poly_final(payload):
    out = plain_decode(payload, payload.input_embeddings)
    scale = np.max(np.abs(payload.expected_poly_final))
    assert np.max(np.abs(out - payload.expected_poly_final)) < FP32 * scale
    # the surrogate is close to, not equal to, the exact model
    assert np.max(np.abs(out - payload.expected_final)) > 10 * np.max(np.abs(out - payload.expected_poly_final))


def test_layer_outputs_and_states(payload):
    from fhe_mamba_b200.mamba2_layer import plain_step
    st = initial_state(payload)
    for t in range(payload.n_test_tokens):
        h = payload.input_embeddings[t]
        for i, L in enumerate(payload.layers):
            assert np.max(np.abs(h - L.tensors["test_layer_input"][t])) < FP32 * 10
            conv, s = st[i]
            h, conv, s = plain_step(L.weights, L.polys, h, conv, s)
            st[i] = (conv, s)
            assert np.max(np.abs(h - L.tensors["test_layer_output_poly"][t])) < FP32 * 10, (t, i)
            assert np.max(np.abs(s - L.tensors["test_state_output_poly"][t])) < FP32, (t, i)
            h = L.tensors["test_layer_output_poly"][t]


def test_client_loop_greedy_ids(payload):
    p = payload
    ar = p.autoregressive
    out = plain_decode(p, p.ar_embeddings)
    assert np.max(np.abs(out - p.ar_expected_poly_final)) < FP32 * np.max(np.abs(out))
    prompt = ar["prompt_tokens"]
    picked = [select_token(p, h) for h in out[prompt - 1:]]
    assert picked == ar["poly_generated_ids"]
    # the generated token's embedding is the next server input
    assert np.allclose(p.client_embedding_w[picked[0]], p.ar_embeddings[prompt], atol=1e-7)


def test_max_layers_cuts_the_chain():
    p = read_chain_payload(CHAIN, max_layers=1, autoregressive=False)
    assert not p.full_chain and len(p.layers) == 1 and p.client_embedding_w is None
    h, _ = plain_token(p, p.input_embeddings[0], initial_state(p))
    assert np.max(np.abs(h - p.layers[0].tensors["test_layer_output_poly"][0])) < FP32 * 10


def test_refresh_bounds(payload):
    """Bounds never come from the test inputs: calibration sequences from the
    embedding table, carried calibration-text bounds, exported domains."""
    from fhe_mamba_b200.chain_payload import FALLBACK_BOUNDS, calibration_sequences
    seqs = calibration_sequences(payload)
    assert len(seqs) == 8 and not any(np.allclose(s[0], e) for s in seqs for e in payload.input_embeddings[:1])
    assert chain_bounds(payload) == chain_bounds(payload, seqs)
    b = chain_bounds(payload)
    assert len(b) == 3
    for m in b[:2]:
        for k in ("h", "u", "proj", "xbc", "xc", "dt", "adt", "pack", "state", "y", "z", "g", "gn",
                  "n1_v", "n1_y", "n2_v", "n2_y"):
            assert m[k] > 0, k
    # no floor: the gated variance (~0.004-0.04) keeps a bound of its own size
    assert b[0]["n2_v"] < 0.5
    # exported domains widen the activation inputs' bounds
    assert b[0]["xc"] >= 2 * max(abs(payload.layers[0].polys.silu_x.lo), payload.layers[0].polys.silu_x.hi)
    # without calibration data: domains, carried bounds and the fallback table
    d = chain_bounds(payload, sequences=[])
    assert d[0]["u"] == pytest.approx(2 * 8 * np.max(np.abs(payload.layers[0].weights["norm_w"])))
    assert d[0]["proj"] == pytest.approx(2 * payload.layers[0].carried["checkpoint_abs_max"]["proj"])
    joint = read_chain_payload(JOINT)
    dj = chain_bounds(joint)
    # the exporter's "y" checkpoint is the gated value: its calibration-text maximum bounds g
    assert joint.client_embedding_w is None and dj[0]["g"] == pytest.approx(
        2 * joint.layers[0].carried["checkpoint_abs_max"]["y"])
    # without it, the carried gated-variance range does: |g_i| <= sqrt(width var_hi)
    carried = dict(joint.layers[0].carried, checkpoint_abs_max={})
    joint.layers[0].carried = carried
    assert chain_bounds(joint)[0]["g"] == pytest.approx(2 * np.sqrt(128 * carried["gated_variance_range"][1]))
    assert FALLBACK_BOUNDS["state"] == 24.0
    assert {"h", "nf_v", "nf_y"} <= set(b[2])
    # the calibration-text bounds the exporter carries only widen the circuit's own
    carried = payload.layers[0].carried["checkpoint_abs_max"]
    assert b[0]["proj"] >= 2 * carried["proj"]


def _ps_depth(n):
    """Levels spent by Ckks::chebyshev (fhe_mamba_b200/csrc/ckks.cu) on an
    n-coefficient series: T_2i = 2 T_i^2 - 1 and T_2i+1 = 2 T_i T_i+1 - T_1 one
    level above their factors, leaves a weighted sum of the baby basis (one
    level above its deepest member), each split T_k * upper one level above both."""
    levels = 0
    while (1 << levels) < n:
        levels += 1
    baby = 1 << ((max(1, levels) + 1) // 2)
    memo = {1: 0}

    def d(i):
        if i not in memo:
            memo[i] = (d(i // 2) if i % 2 == 0 else max(d((i + 1) // 2), d(i // 2))) + 1
        return memo[i]

    def ev(deg):
        if deg < baby:
            return max(d(j) for j in range(1, min(baby - 1, n - 1) + 1)) + 1
        k = baby
        while 2 * k - 1 < deg:
            k *= 2
        return max(ev(k - 1), max(d(k), ev(deg - k)) + 1)

    return ev(n - 1)


def test_level_estimate_bounds_the_device_series():
    assert all(_ps_depth(n) <= chebyshev_levels(n) for n in range(2, 1100))
    assert chebyshev_levels(97) == 8 and chebyshev_levels(32) == 6


def _copy(tmp_path):
    dst = tmp_path / "chain"
    shutil.copytree(CHAIN, dst)
    return dst


def _edit(path, fn):
    meta = json.loads(path.read_text())
    fn(meta)
    path.write_text(json.dumps(meta))


@pytest.mark.parametrize("case,message", [
    ("chain_format", "unexpected chain payload format"),
    ("joint_without_format", "requires the versioned joint format"),
    ("layer_format", "unexpected payload format"),
    ("groups", "only n_groups == 1"),
    ("kind", "unsupported exported polynomial kind"),
    ("mask_value", "head_mask values must be zero or one"),
    ("mask_length", "one value per head"),
    ("scheduled_site", "non-normalization site"),
    ("layer_dirs", "layer_dirs does not match n_layers"),
    ("tensor", "tensor size mismatch for conv_b"),
    ("protocol", "unsupported autoregressive payload protocol"),
    ("time_step", "time_step_limit"),
    ("dtype", "float32-le"),
    ("squarings", "squarings must be an integer"),
    ("iterations", "iterations must be an integer"),
    ("damping", "damping must be in"),
])
def test_payload_errors(tmp_path, case, message):
    d = _copy(tmp_path)
    chain, layer = d / "chain.json", d / "layer_01" / "meta.json"
    sched = {"kind": "scaled-goldschmidt-invsqrt-v1", "lo": 0.05, "hi": 1.0, "seed": 1.0,
             "coefficients": [[1.5, 0.5]], "tolerance": 1e-7, "final_recomputed_newton": True,
             "oracle_workspace_dtype": "float64"}
    edits = {
        "chain_format": (chain, lambda m: m.update(format="fhemamba-m2-chain-v0")),
        "joint_without_format": (layer, lambda m: m.update(joint_gates={})),
        "layer_format": (layer, lambda m: m.update(format="fhemamba-m1-v0")),
        "groups": (layer, lambda m: m["dims"].update(n_groups=2)),
        "kind": (layer, lambda m: m["polys"]["conv_silu"].update(kind="taylor")),
        "mask_value": (layer, lambda m: m["polys"]["decay_exp"].update(head_mask=[0.5] * 16)),
        "mask_length": (layer, lambda m: m["polys"]["decay_exp"].update(head_mask=[1.0] * 15)),
        "scheduled_site": (layer, lambda m: m["polys"].update(conv_silu=sched)),
        "layer_dirs": (chain, lambda m: m.update(layer_dirs=["layer_00"])),
        "tensor": (layer, lambda m: m["tensors"].update(conv_b=[193])),
        "protocol": (chain, lambda m: m["autoregressive"].update(protocol="server-side")),
        "time_step": (layer, lambda m: m.update(time_step_limit=[0.0, 100.0])),
        "dtype": (chain, lambda m: m.update(dtype="float16-le")),
        "squarings": (layer, lambda m: m["polys"]["decay_exp"].update(squarings=-1)),
        "iterations": (layer, lambda m: m["polys"]["rms_invsqrt"].update(iterations=2.5)),
        "damping": (layer, lambda m: m["polys"]["gated_rms_invsqrt"].update(damping=1.5)),
    }
    path, fn = edits[case]
    _edit(path, fn)
    with pytest.raises(PayloadError, match=message):
        read_chain_payload(d)


def test_scheduled_final_norm(tmp_path):
    """A dedicated final_norm_poly must be a scheduled recipe, and is then the final norm."""
    d = _copy(tmp_path)
    sched = {"kind": "scaled-goldschmidt-invsqrt-v1", "lo": 0.05, "hi": 4.0, "seed": 0.5,
             "coefficients": [[1.5, 0.5]] * 10, "tolerance": 1e-7, "final_recomputed_newton": True,
             "oracle_workspace_dtype": "float64"}
    _edit(d / "chain.json", lambda m: m.update(final_norm_poly=sched))
    p = read_chain_payload(d)
    assert isinstance(p.final_norm, ScheduledInvSqrt) and p.final_norm.fill == pytest.approx(math.sqrt(0.2))
    v = np.geomspace(0.5, 4.0, 7)
    assert np.allclose(p.final_norm.inv_sqrt(v), 1 / np.sqrt(v), rtol=1e-6)
    _edit(d / "chain.json", lambda m: m.update(final_norm_poly={"kind": "poly-newton", "coeffs": [1.0],
                                                                 "lo": 0.1, "hi": 1.0, "iterations": 2}))
    with pytest.raises(PayloadError, match="dedicated final norm requires a scheduled"):
        read_chain_payload(d)


def test_inverse_square_root_kinds_converge():
    v = np.geomspace(0.1, 1.0, 11)
    k = ConstNewton(guess=1.0, iterations=8)
    assert np.allclose(k.inv_sqrt(v), 1 / np.sqrt(v), rtol=1e-9)
    trace = {}
    k.inv_sqrt(v, trace=lambda name, val: trace.setdefault(name, []).append(val))
    assert len(trace["y"]) == 8
    with pytest.raises(PayloadError, match="guess must be positive"):
        parse_poly_spec({"kind": "const-newton", "guess": 0.0, "iterations": 2}, "rms_invsqrt")
    assert math.isfinite(ConstNewton(1.0, 1).fill)


def test_cli_reports_errors_without_a_gpu(tmp_path):
    """Argument and payload errors are reported in the result file with exit code 2
    (the reference's artifact on failure) before any device work."""
    from fhe_mamba_b200 import mamba2_decode
    out = tmp_path / "r.json"
    rc = mamba2_decode.main(["--input-chain", CHAIN, "--output-json", str(out), "--secret-key-dist",
                             "sparse-ternary"])
    r = json.loads(out.read_text())
    assert rc == 2 and r["status"] == "error" and "sparse-ternary" in r["error"]
    rc = mamba2_decode.main(["--input-chain", str(tmp_path / "missing"), "--output-json", str(out),
                             "--security", "not-set"])
    assert rc == 2 and "failed to open" in json.loads(out.read_text())["error"]
    rc = mamba2_decode.main(["--input-chain", CHAIN, "--output-json", str(out), "--meta-bts-alpha", "16"])
    assert rc == 2 and "2^12" in json.loads(out.read_text())["error"]
    # 128-classic over a ring too small for the chain is refused by the audit
    rc = mamba2_decode.main(["--input-chain", CHAIN, "--output-json", str(out), "--ring-dim", "4096"])
    assert rc == 2 and "classical-128" in json.loads(out.read_text())["error"]


def test_joint_payload():
    """The joint format (fhemamba-m2-chain-joint-v1): scheduled inverse square
    roots at every norm site and a dedicated final norm, public-envelope SiLU
    fits (degrees 768 / 384) and shared-dissipation-factor gates in place of
    the softplus and decay sites; the fp64 circuit against the exporter's
    polynomial references."""
    p = read_chain_payload(JOINT)
    assert isinstance(p.final_norm, ScheduledInvSqrt)
    for L in p.layers:
        P = L.polys
        assert isinstance(P.gates, JointGate) and P.gates.degree == 2 and P.gates.p.shape == (3, 16)
        assert isinstance(P.rsqrt1, ScheduledInvSqrt) and isinstance(P.rsqrt2, ScheduledInvSqrt)
        assert P.silu_x.degree == 768 and P.silu_z.degree == 384
    out = plain_decode(p, p.input_embeddings)
    assert np.max(np.abs(out - p.expected_poly_final)) < FP32 * np.max(np.abs(p.expected_poly_final))
    from fhe_mamba_b200.mamba2_layer import plain_step
    st = initial_state(p)
    for t in range(p.n_test_tokens):
        h = p.input_embeddings[t]
        for i, L in enumerate(p.layers):
            conv, s = st[i]
            h, conv, s = plain_step(L.weights, L.polys, h, conv, s)
            st[i] = (conv, s)
            assert np.max(np.abs(h - L.tensors["test_layer_output_poly"][t])) < FP32 * 10, (t, i)
            assert np.max(np.abs(s - L.tensors["test_state_output_poly"][t])) < FP32, (t, i)


@pytest.mark.parametrize("case,message", [
    ("recipe", "unsupported joint gate recipe"),
    ("rates", "rates differ"),
    ("rows", "whole coefficient rows per head"),
    ("pruned", "joint gates retain all heads"),
    ("missing", "key not found: joint_gates"),
])
def test_joint_payload_errors(tmp_path, case, message):
    d = tmp_path / "joint"
    shutil.copytree(JOINT, d)
    layer = d / "layer_00" / "meta.json"
    edits = {
        "recipe": lambda m: m["joint_gates"].update(coefficient_layout="head-major-degree-minor"),
        "rates": lambda m: m["joint_gates"].update(rates=[2.0 * r for r in m["joint_gates"]["rates"]]),
        "rows": lambda m: m["joint_gates"].update(p=m["joint_gates"]["p"][:-1]),
        "pruned": lambda m: m["polys"]["decay_exp"].update(head_mask=[0.0] + [1.0] * 15),
        "missing": lambda m: m.pop("joint_gates"),
    }
    _edit(layer, edits[case])
    with pytest.raises(PayloadError, match=message):
        read_chain_payload(d)
