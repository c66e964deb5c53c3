"""The slot algebra of the sub-slot refresh (fhe_mamba_b200/csrc/bootstrap.cu,
Bootstrapper::build_groups with its Split / Merge / Mask edits), restated in
numpy on plain complex slot vectors: test infrastructure, independent of the
library.  It checks the design the device code implements:

- the butterfly stages of CoeffToSlot (inverse) and SlotToCoeff (forward),
  grouped as the bootstrapper groups them, invert each other;
- the last CoeffToSlot group with its companion on conj(u) (diagonal
  factors 1 / 1 on the lower half of every 2n-block, -i / i on the upper)
  yields 2 Re and 2 Im of the unedited transform side by side;
- the first SlotToCoeff group with its companion on rot(e, n) (factors chosen
  by whether row r + d is in the lower or upper half) rebuilds the transform
  of re + i im exactly, and the masked last group leaves zeros from slot n;
- all of it through the strided BSGS schedule (baby steps j * stride, giant
  steps (g b - offset) * stride, diagonals pre-rotated by the giant amount
  over their period n, 2n or S).

No GPU; the device path is checked by decryption in tests/test_gpu_bootstrap.py."""
import numpy as np
import pytest


def _stage(n, h, inverse):
    """One butterfly stage over n slots, half-distance h: {diagonal: row vector}."""
    m = 8 * h
    xi = [np.exp(2j * np.pi * pow(5, j, m) / m) for j in range(h)]
    out = {}

    def put(d, r, v):
        out.setdefault(d % n, np.zeros(n, complex))[r] += v

    for i in range(0, n, 2 * h):
        for j in range(h):
            r, r2 = i + j, i + j + h
            if not inverse:
                put(0, r, 1.0), put(h, r, xi[j]), put(-h, r2, 1.0), put(0, r2, -xi[j])
            else:
                c = np.conj(xi[j]) * 0.5
                put(0, r, 0.5), put(h, r, 0.5), put(-h, r2, c), put(0, r2, -c)
    return out


def _compose(a, b, n):
    """Diagonals of A B."""
    out = {}
    for d1, v1 in a.items():
        for d2, v2 in b.items():
            k = (d1 + d2) % n
            out.setdefault(k, np.zeros(n, complex))
            out[k] += v1 * np.roll(v2, -d1)
    return out


def _ceil_log2(x):
    return max(0, int(x - 1).bit_length())


def _groups(n, S, halves, budget, inverse, first, last):
    """The bootstrapper's groups: stages split evenly, diagonals edited and
    laid out over S slots for the BSGS schedule."""
    groups, pos, stages = [], 0, len(halves)
    lower = lambda k: (k % (2 * n)) < n  # noqa: E731
    for gi in range(budget):
        k = stages // budget + (1 if gi < stages % budget else 0)
        M, hmin, hmax = None, n, 0
        for s in range(k):
            h = halves[pos + s]
            st = _stage(n, h, inverse)
            M = st if M is None else _compose(st, M, n)
            hmin, hmax = min(hmin, h), max(hmax, h)
        pos += k
        top = hmax == n // 2
        count = (1 << k) if top else (1 << (k + 1)) - 1
        T = (1 << k) - 1
        b = 1 << ((_ceil_log2(count) + 1) // 2)
        off = 0 if top else -(-T // b) * b
        G = -(-count // b) if top else (off + T + b) // b
        edit = first if gi == 0 else "none"
        if gi + 1 == budget and last != "none":
            edit = last
        aux = {"split": 1, "merge": 2}.get(edit, 0)
        d1, d2 = [None] * (b * G), [None] * (b * G)
        P = {"none": n, "mask": S}.get(edit, 2 * n)
        i = np.arange(P)
        for g in range(G):
            for j in range(b):
                t = g * b + j - off
                if (t < 0 or t >= count) if top else (t < -T or t > T):
                    continue
                amount = t * hmin
                v = M.get(amount % n)
                if v is None or not np.any(v):
                    continue
                x = v[i % n]
                if edit == "none":
                    D, D2 = x, None
                elif edit == "mask":
                    D, D2 = np.where(i < n, x, 0), None
                elif edit == "split":
                    D = np.where(lower(i), x, -1j * x)
                    D2 = np.where(lower(i), np.conj(x), 1j * np.conj(x))
                else:  # merge
                    lo = lower(i + amount)
                    D, D2 = x * np.where(lo, 1, 1j), x * np.where(lo, 1j, 1)
                rr = ((g * b - off) * hmin) % P
                place = lambda src: src[(np.arange(S) % P - rr) % P]  # noqa: E731
                d1[g * b + j] = place(D)
                if aux:
                    d2[g * b + j] = place(D2)
        groups.append(dict(b=b, G=G, stride=hmin, off=off, d1=d1, d2=d2, aux=aux))
    return groups


def _rot(x, k):
    return np.roll(x, -k)


def _bsgs(x, diags, b, G, stride, off):
    babies = [_rot(x, j * stride) for j in range(b)]
    out = np.zeros_like(x)
    for g in range(G):
        inner = np.zeros_like(x)
        for j in range(b):
            if diags[g * b + j] is not None:
                inner += diags[g * b + j] * babies[j]
        out += _rot(inner, (g * b - off) * stride)
    return out


def _transform(groups, x, n):
    for g in groups:
        y = _bsgs(x, g["d1"], g["b"], g["G"], g["stride"], g["off"])
        if g["aux"]:
            x2 = np.conj(x) if g["aux"] == 1 else _rot(x, n)
            y = y + _bsgs(x2, g["d2"], g["b"], g["G"], g["stride"], g["off"])
        x = y
    return x


@pytest.mark.parametrize("n,S,bc,bs", [(16, 64, 2, 2), (32, 128, 4, 4), (64, 256, 3, 2), (16, 32, 1, 2),
                                       (64, 128, 4, 3), (128, 1024, 4, 4)])
def test_split_merge_mask(n, S, bc, bs):
    halves = [n >> (i + 1) for i in range(n.bit_length() - 1)]  # n/2 ... 1
    v = np.random.default_rng(n + S).uniform(-1, 1, n) + 0j
    # unedited transforms on n slots: CoeffToSlot then SlotToCoeff is 2x the identity on 2 Re + 2i Im
    w = _transform(_groups(n, n, halves, bc, True, "none", "none"), v.copy(), n)
    ref = _transform(_groups(n, n, halves[::-1], bs, False, "none", "none"), 2 * w.real + 2j * w.imag, n)
    assert np.max(np.abs(ref - 2 * v)) < 1e-12
    # the edited pipeline on S slots, input replicated with period n
    z = _transform(_groups(n, S, halves, bc, True, "none", "split"), np.tile(v, S // n), n)
    want = np.tile(np.concatenate([2 * w.real, 2 * w.imag]), S // (2 * n))
    assert np.max(np.abs(z - want)) < 1e-12
    out = _transform(_groups(n, S, halves[::-1], bs, False, "merge", "mask"), z, n)
    assert np.max(np.abs(out[:n] - ref)) < 1e-12 and np.max(np.abs(out[n:])) == 0.0


def test_one_coeff_to_slot_group_keeps_the_split():
    """With a budget of one CoeffToSlot group the split edit (always the last
    group's) still applies, as the bootstrapper orders its edits."""
    n, S = 16, 64
    halves = [8, 4, 2, 1]
    (g,) = _groups(n, S, halves, 1, True, "none", "split")
    assert g["aux"] == 1 and any(d is not None for d in g["d2"])
