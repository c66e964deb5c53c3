"""Generates a small Mamba-2 chain payload with the reference's own exporter.

Run in a checkout that has the reference next to it:
    python tests/golden/make_mamba2_chain.py /path/to/reference
It builds a random-init 2-layer HuggingFace Mamba-2 language model (d_model 64,
d_inner 128 = 16 heads x 8, d_state 32, one group, conv 4, vocabulary 128,
seed 6), and runs the reference's ``fhemamba.m1_payload.export_chain_payload``
on it exactly as its decode experiments do: calibration of the polynomial
domains on the exporter's default calibration text, the frozen degrees
(conv SiLU 96, gate SiLU 64, sqrt-softplus 64, decay exp 24, RMS Newton seed 47,
gated Newton seed 31), three test tokens, and the plaintext
polynomial-circuit references (``test_layer_output_poly``,
``chain_expected_poly_final``), plus the client-in-the-loop assets of a
2-token prompt and 2 greedy tokens (tied embedding, the polynomial circuit's
per-evaluation final hidden vectors and its greedy ids).  The trained checkpoint and its tokenizer are
not available here, so the weights are synthetic and the tokenizer maps each
byte of the text to ``byte mod 128``; the payload layout is the exporter's.
Writes ``mamba2_chain/`` next to this script, and
``mamba2_nonlinearities.json``: every exported nonlinearity kind evaluated
by the reference's own evaluators on a grid, and ``mamba2_chain_joint/``: the
same model in the joint format (scheduled normalizations, dedicated final
norm, shared-dissipation-factor gates; see ``write_joint``).
"""
import json
import shutil
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
OUT = HERE / "mamba2_chain"


class ByteTokenizer:
    """Stands in for the checkpoint's tokenizer: one id per UTF-8 byte."""

    def __init__(self, vocab: int):
        self.vocab = vocab

    def __call__(self, text, return_tensors="pt"):
        ids = torch.tensor([[b % self.vocab for b in text.encode()]])
        return type("Encoded", (), {"input_ids": ids})()


def main(reference: str) -> None:
    sys.path.insert(0, str(Path(reference) / "src"))
    from fhemamba.m1_payload import export_chain_payload
    from transformers import Mamba2Config, Mamba2ForCausalLM

    torch.manual_seed(6)
    cfg = Mamba2Config(vocab_size=128, hidden_size=64, num_hidden_layers=2, state_size=32, num_heads=16,
                       head_dim=8, expand=2, n_groups=1, conv_kernel=4, tie_word_embeddings=True)
    model = Mamba2ForCausalLM(cfg).eval()
    # Decay rates A = -exp(A_log) spread over 1..24 with one far faster head:
    # the exporter then fits exp on a range that needs repeated squarings and
    # prunes the fast head (its head mask entry is 0), so the fixture covers
    # both paths of the decay polynomial.
    with torch.no_grad():
        for layer in model.backbone.layers:
            rates = torch.linspace(1.0, 24.0, cfg.num_heads)
            rates[0] = 400.0
            layer.mixer.A_log.copy_(torch.log(rates))
    if OUT.exists():
        shutil.rmtree(OUT)
    export_chain_payload(model, ByteTokenizer(cfg.vocab_size), OUT, n_test_tokens=3, cal_tokens=128,
                         bound_cal_tokens=128, autoregressive_prompt_tokens=2,
                         autoregressive_generate_tokens=2)
    write_joint(model, cfg)
    write_nonlinearities()


def write_joint(model, cfg) -> None:
    """The same model exported in the joint format (``fhemamba-m2-chain-joint-v1``):
    scheduled inverse square roots at every norm site, a dedicated final norm
    (``plan_invsqrt`` on public variance intervals, as the reference's
    scheduled-payload tests plan them) and shared-dissipation-factor gates on
    the public gate domains with degree-2 dissipation and degree-1
    equilibrium roots per head (certified: |p| <= 0.8)."""
    from fhemamba.m1_payload import export_chain_payload
    from fhemamba.normalization import plan_invsqrt
    from fhemamba.payload_surrogate import public_gate_domains

    work = HERE / "_joint_inputs"
    if work.exists():
        shutil.rmtree(work)
    work.mkdir()
    his = {(0, "rms_invsqrt"): 50, (0, "gated_rms_invsqrt"): 100, (1, "rms_invsqrt"): 50,
           (1, "gated_rms_invsqrt"): 100, (2, "rms_invsqrt"): 200}
    bundle = {"format": "fhemamba-normalization-schedules-v1",
              "operators": [{"layer": layer, "site": site, "recipe": plan_invsqrt(1e-6, hi).recipe()}
                            for (layer, site), hi in his.items()]}
    (work / "schedules.json").write_text(json.dumps(bundle))
    arrays = {}
    heads = cfg.num_heads
    for layer, block in enumerate(model.backbone.layers):
        lo, hi = public_gate_domains(block)
        shade = np.linspace(0.0, 1.0, heads)
        arrays.update({f"layer_{layer}_lo": lo, f"layer_{layer}_hi": hi,
                       f"layer_{layer}_p": np.stack([0.5 - 0.2 * shade, 0.2 + 0.05 * shade, np.full(heads, 0.1)]),
                       f"layer_{layer}_q": np.stack([0.75 + 0.1 * shade, np.full(heads, -0.15)]),
                       f"layer_{layer}_rates": block.mixer.A_log.detach().exp().double().numpy()})
    arrays["manifest"] = np.array(json.dumps({"format": "dissipative-mamba2-gates-v1", "layers": [0, 1],
                                              "input_payload_sha256": "0" * 64}))
    np.savez(work / "gates.npz", **arrays)
    out = HERE / "mamba2_chain_joint"
    if out.exists():
        shutil.rmtree(out)
    try:
        export_chain_payload(model, ByteTokenizer(cfg.vocab_size), out, n_test_tokens=3, cal_tokens=128,
                             bound_cal_tokens=128, normalization_bundle=work / "schedules.json",
                             stabilized_gate_bundle=work / "gates.npz")
    finally:
        shutil.rmtree(work)


def write_nonlinearities() -> None:
    """Every exported nonlinearity kind evaluated by the reference's own
    evaluators (``_poly_from_export_spec``, ``gate_from_spec``) in float64 on a
    grid: the layer specs of both payloads (the joint payload's scheduled
    inverse square roots and its gates), plus a ``const-newton`` and a
    ``scaled-goldschmidt-invsqrt-v1`` spec (coupled Newton coefficient pairs)
    that the exporters do not emit."""
    from fhemamba.m1_payload import _poly_from_export_spec
    from fhemamba.payload_surrogate import gate_from_spec

    metas = [json.loads((OUT / f"layer_{i:02d}" / "meta.json").read_text()) for i in (0, 1)]
    cases = []

    def add(name, spec, x):
        y = _poly_from_export_spec(spec)(torch.tensor(x, dtype=torch.float64))
        cases.append({"name": name, "spec": spec, "x": np.asarray(x).tolist(), "y": y.numpy().tolist()})

    for li, meta in enumerate(metas):
        for site, spec in meta["polys"].items():
            if site == "decay_exp":
                heads = len(spec["head_mask"])
                lo = spec["lo"] * 2 ** spec["squarings"]
                x = np.linspace(lo * 1.5, 0.0, 7)[:, None] * np.linspace(0.2, 1.0, heads)[None, :]
            elif site in ("rms_invsqrt", "gated_rms_invsqrt"):
                x = np.geomspace(max(spec["lo"], 1e-6), spec["hi"], 9)
            else:
                x = np.linspace(spec["lo"], spec["hi"], 9)
            add(f"layer{li}.{site}", spec, x)
    joint = HERE / "mamba2_chain_joint"
    for li in (0, 1):
        meta = json.loads((joint / f"layer_{li:02d}" / "meta.json").read_text())
        for site in ("rms_invsqrt", "gated_rms_invsqrt"):
            spec = meta["polys"][site]
            add(f"joint{li}.{site}", spec, np.geomspace(spec["lo"] * 10, spec["hi"] / 10, 9))
        gate, _ = gate_from_spec(meta["joint_gates"])
        lo, hi = np.asarray(meta["joint_gates"]["lo"]), np.asarray(meta["joint_gates"]["hi"])
        z = lo[None, :] + np.linspace(0.0, 1.0, 7)[:, None] * (hi - lo)[None, :]
        write, decay = gate(torch.tensor(z, dtype=torch.float64))
        cases.append({"name": f"joint{li}.gates", "spec": meta["joint_gates"], "x": z.tolist(),
                      "y": [write.numpy().tolist(), decay.numpy().tolist()]})
    add("const-newton", {"kind": "const-newton", "guess": 2.0, "iterations": 7}, np.geomspace(0.02, 0.2, 9))
    add("scheduled", {"kind": "scaled-goldschmidt-invsqrt-v1", "lo": 0.05, "hi": 1.0, "seed": 1.0,
                      "coefficients": [[1.5, 0.5]] * 6, "tolerance": 1e-7, "final_recomputed_newton": True,
                      "oracle_workspace_dtype": "float64"}, np.geomspace(0.05, 1.0, 9))
    (HERE / "mamba2_nonlinearities.json").write_text(json.dumps(cases, indent=1))


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: make_mamba2_chain.py /path/to/reference")
    main(sys.argv[1])
