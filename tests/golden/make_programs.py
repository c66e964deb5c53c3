"""Generates the packed-program fixtures with the reference's own compiler.

Run in a checkout that has the reference next to it:
    python tests/golden/make_programs.py /path/to/reference
It builds small fhemamba-packed-v2 programs with the reference's
``fhemamba.packed_program.PackedProgram`` (polynomial and exact output
references computed by the reference itself) and writes them next to this
script.  The GPU tests read only the written files.
"""
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def main(reference: str) -> None:
    sys.path.insert(0, str(Path(reference) / "src"))
    from fhemamba.ops import fit_chebyshev
    from fhemamba.packed_program import PackedProgram

    rng = np.random.default_rng(2024)
    silu = fit_chebyshev(lambda t: t * torch.sigmoid(t), -8.0, 8.0, 31)
    polys = {(0, "silu"): silu}

    # every operation of the v2 grammar except feedback
    p = PackedProgram(polys, slots=256, bound=64.0, extended=True)
    x0 = rng.uniform(-1, 1, 8)
    w1 = rng.normal(0, 0.4, (16, 8))
    x = p.input(x0)
    y = p.linear(x, w1)                       # linear
    y2 = p.linear(x, w1)                      # linear_ref (shared weights)
    z = y + y2                                # add
    m = z * z                                 # mul
    c = m * 0.25 + 0.125                      # mulp, addp
    s = p.nonlinear(c, "silu", (0, "silu"))   # cheb
    exact_s = torch.nn.functional.silu(torch.from_numpy(c.value)).numpy()
    r = s.reshape(4, 4)
    t = p.sum_last(r)                         # sum (width 4)
    b = t.reshape(4, 1) * r                   # repeat (broadcast) + mul
    g = b.reshape(16)[::3]                    # gather
    k = p.constant(rng.uniform(-1, 1, 6))     # public
    cat = p.concatenate([g, k])               # scatter + add
    p.output(s, exact_s)
    ex_r = exact_s.reshape(4, 4)
    ex_t = ex_r.sum(-1, keepdims=True)
    ex_b = (ex_t * ex_r).reshape(16)
    p.output(cat, np.concatenate([ex_b[::3], k.value]))
    p.write(HERE / "packed_all_ops_v2.txt")

    # a wide matvec (more than 32 diagonals: the BSGS path) and a wide gather
    q = PackedProgram({}, slots=2048, bound=64.0, extended=True)
    xv = rng.uniform(-1, 1, 96)
    wv = rng.normal(0, 0.1, (80, 96))
    xq = q.input(xv)
    yq = q.linear(xq, wv)
    gq = yq[5:77:2]                           # monotone gather with many offsets
    q.output(yq, wv @ xv)
    q.output(gq, (wv @ xv)[5:77:2])
    q.write(HERE / "packed_linear_v2.txt")

    # a chain deeper than one modulus chain: the executor must refresh
    r = PackedProgram({}, slots=256, bound=64.0, extended=True)
    v = r.input(rng.uniform(-1, 1, 8))
    for i in range(60):
        v = v * rng.choice([-1.0, 1.0], 8)
    r.output(v, v.value)
    r.write(HERE / "packed_refresh_v2.txt")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "../reference")
