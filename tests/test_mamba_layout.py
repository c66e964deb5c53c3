"""Slot layout of the packed Mamba-2 recurrent state (host logic, no GPU)."""
import numpy as np

HEADS, HD, S = 16, 8, 32


def test_state_layout_roundtrip():
    from fhe_mamba_b200.mamba import StateLayout
    lay = StateLayout(HEADS, HD, S, 2048)
    assert (lay.group_heads, lay.group_block, lay.groups) == (8, 64, 2)
    st = np.random.default_rng(0).normal(size=(HEADS, HD, S))
    packed = lay.pack(st)
    g, s = lay.slot(9, 3, 5)
    assert packed[g, s] == st[9, 3, 5]
    assert np.array_equal(lay.unpack(packed), st)


def test_rotation_steps_cover_the_schedule():
    from fhe_mamba_b200.mamba import PackedMamba2, StateLayout

    class _Ctx:
        slots = 2048

    pm = PackedMamba2(_Ctx(), StateLayout(HEADS, HD, S, 2048), b_base=128, c_base=160)
    steps = pm.rotation_steps(norm_width=128)
    gb = 64
    assert all(0 < s < 2048 for s in steps)
    assert (-gb) % 2048 in steps and gb in steps and 128 in steps and 160 in steps
    assert (-(gb - 1)) % 2048 in steps  # strided BSGS baby of place_state_blocks
