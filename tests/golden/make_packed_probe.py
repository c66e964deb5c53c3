"""Exports a small packed-program payload with the reference's own exporter.

Run in a checkout that has the reference next to it:
    python tests/golden/make_packed_probe.py /path/to/reference
It calls the reference's ``fhemamba.workloads.mamba3_probe.export_probe``
(one synthetic Mamba-3 SISO mixer, d_model 32, 2 recurrent steps, seed 19:
program.txt in fhemamba-packed-v1, fixture.npz and manifest.json with the
files' digests) into packed_probe/ next to this script.  The payload is what
the reference's runner (``fhemamba.benchmarks.packed._run``) hands to its
native executable; record_packed_run.py runs packed_b200 on it the same way.
"""
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent


def main(reference: str) -> None:
    sys.path.insert(0, str(Path(reference) / "src"))
    from fhemamba.workloads.mamba3_probe import export_probe
    out = HERE / "packed_probe"
    report = export_probe(out, tokens=2)
    print(report["program"], len(report["output_names"]), "outputs")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: make_packed_probe.py REFERENCE_CHECKOUT")
    main(sys.argv[1])
