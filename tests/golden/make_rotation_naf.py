"""Writes rotation_naf.json: the reference's own NAF digits
(``fhemamba.rotation_keys.naf``) for the values its tests use and a sweep.

    python tests/golden/make_rotation_naf.py /path/to/reference
"""
import json
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent


def main(reference: str) -> None:
    sys.path.insert(0, str(Path(reference) / "src"))
    from fhemamba.rotation_keys import naf

    values = sorted({*range(-70, 71), 28, 511, -4088, 767, 3351, -1792, 32767, -32768, 65535, 12345, -9999})
    (HERE / "rotation_naf.json").write_text(json.dumps({str(v): naf(v) for v in values}))


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: make_rotation_naf.py /path/to/reference")
    main(sys.argv[1])
