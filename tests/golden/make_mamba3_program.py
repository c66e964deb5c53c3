"""Generates a small Mamba-3 SISO packed program with the reference's own compiler.

Run in a checkout that has the reference next to it:
    python tests/golden/make_mamba3_program.py /path/to/reference
It builds a random-init 2-layer Mamba-3 SISO language model (the reference's
``fhemamba.mamba3_lm.Mamba3LM``, d_model 64, d_state 16, MLP width 128,
vocabulary 256, weights ~N(0, 0.1^2) from a seed), calibrates its polynomial
nonlinearities with the reference's ``Calibration`` exactly as
``workloads/mamba3_export.py`` does, and compiles a 3-token prompt plus 3
greedy tokens (client feedback of the decrypted hidden) into
fhemamba-packed-v2.  The trained 187M checkpoint is not available here, so the
weights are synthetic; the program structure is the exporter's.  Writes
packed_mamba3_siso_v2.txt, mamba3_client_head.f32 and mamba3_tokens.json next
to this script.
"""
import json
import struct
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def main(reference: str) -> None:
    sys.path.insert(0, str(Path(reference) / "src"))
    from fhemamba.mamba3 import FactoredMamba3State
    from fhemamba.mamba3_lm import Mamba3LM
    from fhemamba.packed_program import Calibration, PackedProgram

    torch.manual_seed(3)
    cfg = {"d_model": 64, "d_intermediate": 128, "n_layer": 2, "vocab_size": 256, "rms_norm": True,
           "tie_embeddings": True, "pad_vocab_size_multiple": 16,
           "ssm_cfg": {"layer": "Mamba3", "d_state": 16, "expand": 2, "headdim": 32, "rope_fraction": 0.5}}
    model = Mamba3LM(cfg).eval()
    with torch.no_grad():
        for p in model.parameters():
            if p.dim() >= 2:
                p.normal_(0, 0.1)
    rng = np.random.default_rng(7)
    recorder = Calibration()
    for _ in range(6):
        model.generate([int(x) for x in rng.integers(0, 256, 3)], 4, recorder, factored=False, rotary="angle")
    poly, _ = recorder.fit(tolerance=1e-6, max_degree=1023, margin=0.2, quadrature=True,
                           kind_tolerances={"negative_a": 1e-4}, positive_lower_fraction=0.5)
    prompt, new_tokens = [5, 17, 33], 3
    exact_ids, exact_trace = model.generate(prompt, new_tokens, factored=False)
    poly_ids, poly_trace = model.generate(prompt, new_tokens, poly, factored=True, rotary="angle")
    assert exact_ids == poly_ids, (exact_ids, poly_ids)
    program = PackedProgram(poly.polynomials, slots=2048, bound=1e8, extended=True)
    states = [FactoredMamba3State(program.constant(s.angle))
              for s in model.initial_states(factored=True, rotary="angle")]
    all_ids = prompt + poly_ids
    hidden = None
    for step in range(len(exact_trace)):
        embedding = model.backbone.embedding.weight[all_ids[step]][None]
        x = program.input(embedding) if step < len(prompt) else program.client_input(hidden, embedding)
        hidden, states = model.step(x, states, program)
        np.testing.assert_allclose(hidden.value, poly_trace[step].numpy(), atol=1e-9, rtol=1e-9)
        program.output(hidden, exact_trace[step])
    program.write(HERE / "packed_mamba3_siso_v2.txt")
    # the reference's client-head format (workloads/client_head.py:51-61):
    # little-endian u32 vocab, u32 width, then f32[vocab * width]
    head = np.asarray(model.lm_head.weight.detach().numpy(), dtype="<f4")
    with open(HERE / "mamba3_client_head.f32", "wb") as f:
        f.write(struct.pack("<II", *head.shape))
        head.tofile(f)
    (HERE / "mamba3_tokens.json").write_text(json.dumps(
        {"prompt_ids": prompt, "exact_token_ids": exact_ids, "polynomial_token_ids": poly_ids,
         "summary": program.summary()}, indent=1) + "\n")
    print(exact_ids, poly_ids, program.summary())


if __name__ == "__main__":
    main(sys.argv[1])
