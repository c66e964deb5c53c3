"""Extracts ckks_recipe_levels.json: the levels each nonlinearity recipe
consumed in the reference's OpenFHE runs, as its own test fixture records them
(tests/fixtures/ckks-recipes.json, "primitives" suite: recipe name, degree,
interval, squarings / Newton iterations and damping, levels consumed, and the
recorded CKKS-vs-float64 error).

    python tests/golden/make_recipe_levels.py /path/to/reference
"""
import json
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
KEYS = ("name", "degree", "interval", "squarings", "iterations", "damping", "levels_consumed",
        "max_abs_err_ckks_vs_plain64")


def main(reference: str) -> None:
    fixture = json.loads((Path(reference) / "tests/fixtures/ckks-recipes.json").read_text())
    record = fixture["primitives"]["record"]
    recipes = [{k: p[k] for k in KEYS if k in p} for p in record["primitives"] if "degree" in p]
    out = {"source": "tests/fixtures/ckks-recipes.json (primitives)", "config": record["config"],
           "recipes": recipes}
    (HERE / "ckks_recipe_levels.json").write_text(json.dumps(out, indent=1))


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: make_recipe_levels.py /path/to/reference")
    main(sys.argv[1])
