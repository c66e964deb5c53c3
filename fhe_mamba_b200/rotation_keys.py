"""Rotation-key plans: which rotations get a key of their own and how the
others compose from signed powers of two.

The reference decode's ``--rotation-keys full|compact|balanced`` with
``--rotation-key-gib`` (native/fideslib_stage0/src/stage1_mamba2_decode_fideslib.cpp:1080-1140,
design in src/fhemamba/rotation_keys.py): *full* keys every rotation index;
*compact* keys only the signed powers of two that the non-adjacent-form (NAF)
digits of the indices use, and composes every other rotation from them;
*balanced* adds, under a key-memory budget, the non-base indices with the
largest saving frequency x (NAF weight - 1) (ties: the smaller index).
Rotations compose exactly and spend no level, so the plan changes only the
key memory and the number of key switches.

Deviation: the library's fused linear transform (``EvalLinearTransform``)
switches keys per baby and giant step, so those steps (``required``) keep
direct keys in every mode.
"""
from __future__ import annotations

from dataclasses import dataclass, field

MODES = ("full", "compact", "balanced")


def naf(value: int) -> list[int]:
    """Signed powers of two summing to `value`, ascending in magnitude, no two
    adjacent (naf_steps, native/fideslib_stage0/include/rotation_steps.hpp:13-27)."""
    steps, remaining, power = [], int(value), 1
    while remaining:
        if remaining & 1:
            digit = 2 - (remaining & 3)
            steps.append(digit * power)
            remaining -= digit
        remaining //= 2
        power *= 2
    return steps


def canonical_rotation(offset: int, slots: int) -> int:
    """The rotation in (-slots/2, slots/2] (canonical_rotation, rotation_steps.hpp:30-37)."""
    if slots < 2 or slots & (slots - 1):
        raise ValueError("rotation slots must be a power of two")
    offset %= slots
    return offset - slots if offset > slots // 2 else offset


def key_bytes(ring: int, towers: int, dnum: int) -> int:
    """Device bytes of one key-switching key: dnum digits x 2 polynomials x
    (Q + P towers) x ring words of 8 bytes."""
    return 2 * dnum * towers * ring * 8


@dataclass
class KeyPlan:
    mode: str
    slots: int
    direct: frozenset
    frequencies: dict = field(default_factory=dict)

    @property
    def keys(self) -> list[int]:
        return sorted(self.direct)

    def steps(self, offset: int) -> list[int]:
        """The key applications of one rotation: itself when keyed, else its NAF digits."""
        r = canonical_rotation(offset, self.slots)
        if r == 0:
            return []
        return [r] if r in self.direct else [canonical_rotation(d, self.slots) for d in naf(r)]

    @property
    def stats(self) -> dict:
        total = sum(self.frequencies.values()) or 1.0
        applied = sum(f * len(self.steps(i)) for i, f in self.frequencies.items())
        return {"mode": self.mode, "keys_total": len(self.direct),
                "composite_indices": sum(1 for i in self.frequencies if len(self.steps(i)) > 1),
                "rotation_overhead_factor": applied / total}


def plan_keys(frequencies: dict, slots: int, mode: str = "full", budget_bytes: float | None = None,
              bytes_per_key: float | None = None, required=()) -> KeyPlan:
    """A key plan for rotation indices used `frequencies[index]` times (per token)."""
    if mode not in MODES:
        raise ValueError(f"--rotation-keys must be one of {', '.join(MODES)}")
    freqs = {}
    for index, f in frequencies.items():
        r = canonical_rotation(index, slots)
        if r:
            freqs[r] = freqs.get(r, 0.0) + float(f)
    req = {canonical_rotation(i, slots) for i in required} - {0}
    if mode == "full":
        return KeyPlan(mode, slots, frozenset(set(freqs) | req), freqs)
    base = {canonical_rotation(s, slots) for i in freqs for s in naf(i)}  # -slots/2 is +slots/2
    direct = base | req
    if mode == "balanced":
        if budget_bytes is None or not bytes_per_key:
            raise ValueError("a balanced plan needs a key budget and the size of a key")
        affordable = int(budget_bytes // bytes_per_key) - len(direct)
        candidates = sorted(((f * (len(naf(i)) - 1), i) for i, f in freqs.items() if i not in direct),
                            key=lambda c: (-c[0], abs(c[1])))
        for saving, index in candidates:
            if affordable <= 0 or saving <= 0:
                break
            direct.add(index)
            affordable -= 1
    return KeyPlan(mode, slots, frozenset(direct), freqs)


class ComposedRotations:
    """A CryptoContext whose rotations follow a key plan: keyed rotations run
    as they are, the others as a chain of key applications (hoisted together
    where they are keyed).  Everything else is the wrapped context's."""

    def __init__(self, cc, plan: KeyPlan):
        self._cc, self.plan = cc, plan
        self.composite_applications = 0

    def __getattr__(self, name):
        return getattr(self._cc, name)

    def EvalRotate(self, ct, offset):
        steps = self.plan.steps(offset)
        if not steps:  # the identity needs no key
            return ct.Clone()
        if len(steps) == 1:
            return self._cc.EvalRotate(ct, steps[0])
        self.composite_applications += len(steps)
        out = ct
        for s in steps:
            out = self._cc.EvalRotate(out, s)
        return out

    def EvalFastRotation(self, ct, offsets, *rest):
        offsets = list(offsets)
        keyed = [i for i, o in enumerate(offsets) if len(self.plan.steps(o)) == 1]
        out = [None] * len(offsets)
        if keyed:
            for i, r in zip(keyed, self._cc.EvalFastRotation(ct, [offsets[i] for i in keyed], *rest)):
                out[i] = r
        for i, o in enumerate(offsets):
            if out[i] is None:
                out[i] = self.EvalRotate(ct, o)
        return out
