"""Packed-program reader (host logic of the executor, no GPU).

The fixtures under tests/golden/ were written by the reference's own compiler
(tests/golden/make_programs.py); the reader must accept them and reject the
malformed variants that the reference's read_packed_program rejects
(native/fideslib_stage0/include/packed_program.hpp:60-163).
"""
import os

import pytest

from fhe_mamba_b200 import InvalidArgument
from fhe_mamba_b200.program import validate_program

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


@pytest.mark.parametrize("name,slots,nodes,outputs", [
    ("packed_all_ops_v2.txt", 256, 16, 2),
    ("packed_linear_v2.txt", 2048, 3, 2),
    ("packed_refresh_v2.txt", 256, 61, 1),
    ("packed_mamba3_siso_v2.txt", 2048, 1335, 5),
])
def test_fixtures_parse(name, slots, nodes, outputs):
    assert validate_program(os.path.join(GOLDEN, name)) == {"slots": slots, "nodes": nodes, "outputs": outputs}


def _write(tmp_path, text):
    p = tmp_path / "p.txt"
    p.write_text(text)
    return str(p)


@pytest.mark.parametrize("text", [
    "fhemamba-packed-v3 16 8 1 1\ninput 2 0 2 1 2\n0 2 1 2 1 2\n",           # magic
    "fhemamba-packed-v1 12 8 1 1\ninput 2 0 2 1 2\n0 2 1 2 1 2\n",           # slots not a power of two
    "fhemamba-packed-v1 16 8 1 1\ninput 2 1 0 2 1 2\n0 2 1 2 1 2\n",         # source with a parent
    "fhemamba-packed-v1 16 8 2 1\ninput 2 0 2 1 2\ngather 2 1 0 2 0 5\n1 2 1 2 1 2\n",  # index out of range
    "fhemamba-packed-v1 16 8 2 1\ninput 2 0 2 1 2\nfeedback 2 1 0 0\n1 2 1 2 1 2\n",    # feedback needs v2
    "fhemamba-packed-v1 16 8 1 1\ninput 2 0 2 1 2\n0 2 1 2 1 2\nextra\n",    # trailing data
    "fhemamba-packed-v2 16 8 1 1\ninput 2 9 0 2 1 2\n0 2 1 2 1 2\n",         # node bound above program bound
])
def test_malformed_programs_are_rejected(tmp_path, text):
    with pytest.raises(InvalidArgument):
        validate_program(_write(tmp_path, text))


def test_minimal_program(tmp_path):
    text = "fhemamba-packed-v1 16 8 2 1\ninput 2 0 2 1 2\nmulp 2 1 0 2 3 4\n1 2 3 8 3 8\n"
    assert validate_program(_write(tmp_path, text)) == {"slots": 16, "nodes": 2, "outputs": 1}
