"""Packed Mamba-2 decode pieces on CKKS ciphertexts: the recurrent-state
update and readout, the causal-conv window and the gated RMSNorm.

These follow the reference's native Mamba-2 decode
(``native/fideslib_stage0/src/stage1_mamba2_decode_fideslib.cpp``):

* state layout -- the (head, channel, state) tensor of one layer is split into
  groups of ``group_heads`` whole heads; within a group, state coordinate
  (h, p, k) sits at slot ``k * group_block + h_local * head_dim + p`` with
  ``group_block = group_heads * head_dim`` (packing of ``update_state_group`` /
  ``readout_state_group``, :3971-4057);
* ``expand_x`` / ``place_heads`` / ``place_state_blocks`` / ``doubling_fill``
  (:3271-3410, :1802) -- masks, rotations and the strided BSGS that move the
  packed streams into that layout;
* the update ``S <- decay * S + (dt * x) (x) B`` and the readout
  ``y = sum_k S * C`` by a rotate-and-add over the state axis, a block mask and
  a placement rotation;
* the RMSNorm inverse square root as a Chebyshev seed refined by Newton steps
  ``y <- 1.5 y - 0.5 V y^3`` (``newton_refine``, :2388-2400) on
  ``V = mean(x^2) + eps``.

The plaintext formulas they implement are ``mixer2_forward`` and
``rms_normalize`` / ``ssm_update_readout`` (``src/fhemamba/reference.py:182-294``,
``src/fhemamba/tensor_ops.py:53-118``).  Every operation runs on the device
through the C ABI; this module only schedules them.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from . import _lib


def _log2(v: int) -> int:
    if v <= 0 or v & (v - 1):
        raise _lib.InvalidArgument(-1, "mamba", f"{v} is not a power of two")
    return v.bit_length() - 1


@dataclass(frozen=True)
class StateLayout:
    """Slot layout of one layer's recurrent state (heads x head_dim x state_size)."""

    heads: int
    head_dim: int
    state_size: int
    slots: int

    def __post_init__(self):
        for v in (self.head_dim, self.state_size, self.slots):
            _log2(v)
        if self.heads < 1 or self.head_dim * self.state_size > self.slots:
            raise _lib.InvalidArgument(-1, "StateLayout", "one head's state does not fit the slots")

    @property
    def group_heads(self) -> int:
        """Largest power of two that fits the slots and divides the head count."""
        g = 1
        cap = min(self.heads, self.slots // (self.head_dim * self.state_size))
        while 2 * g <= cap and self.heads % (2 * g) == 0:
            g *= 2
        return g

    @property
    def group_block(self) -> int:
        return self.group_heads * self.head_dim

    @property
    def groups(self) -> int:
        return self.heads // self.group_heads

    def slot(self, h: int, p: int, k: int):
        g, hl = divmod(h, self.group_heads)
        return g, k * self.group_block + hl * self.head_dim + p

    def pack(self, state: np.ndarray) -> np.ndarray:
        """[heads, head_dim, state_size] -> [groups, slots] slot vectors."""
        s = np.asarray(state).reshape(self.groups, self.group_heads, self.head_dim, self.state_size)
        out = np.zeros((self.groups, self.slots), dtype=s.dtype)
        blk = s.transpose(0, 3, 1, 2).reshape(self.groups, self.state_size * self.group_block)
        out[:, :blk.shape[1]] = blk
        return out

    def unpack(self, vecs: np.ndarray) -> np.ndarray:
        v = np.asarray(vecs)[:, :self.state_size * self.group_block]
        v = v.reshape(self.groups, self.state_size, self.group_heads, self.head_dim).transpose(0, 2, 3, 1)
        return v.reshape(self.heads, self.head_dim, self.state_size)


class PlaintextMemo:
    """Device plaintexts of constant slot vectors (masks, conv taps, biases,
    per-head coefficients) kept across calls, keyed by the vector's non-zero
    positions and values, the limb count and the scale: an encode of the same
    vector at the same level and scale gives the same words, so a hit returns
    the earlier plaintext.  Least recently used entries go beyond
    `budget_bytes` of plaintext words."""

    def __init__(self, cc, budget_bytes: float):
        from collections import OrderedDict
        self.cc, self.budget = cc, float(budget_bytes)
        self.entries, self.bytes, self.hits, self.misses = OrderedDict(), 0, 0, 0

    def get(self, values, level: int = 0, scale: float = 0.0):
        c = self.cc
        v = np.asarray(values, dtype=float)
        nz = np.flatnonzero(v)
        key = (v.shape[0], nz.tobytes(), v[nz].tobytes(), int(level), float(scale))
        pt = self.entries.get(key)
        if pt is not None:
            self.entries.move_to_end(key)
            self.hits += 1
            return pt
        self.misses += 1
        pt = c.MakeCKKSPackedPlaintext(v, level=level, scale=scale)
        nbytes = (c.n_q - level) * c.n * 8
        if nbytes <= self.budget:
            self.entries[key] = pt
            self.bytes += nbytes
            while self.bytes > self.budget:
                (_, _, _, lv, _), _ = self.entries.popitem(last=False)
                self.bytes -= (c.n_q - lv) * c.n * 8
        return pt


class PackedMamba2:
    """Encrypted Mamba-2 state update / readout / conv / RMSNorm over one CryptoContext.

    Streams: ``xbc`` holds x (d_inner = heads * head_dim values) at [0, d_inner),
    B at [b_base, b_base + state_size) and C at [c_base, c_base + state_size);
    per-head vectors (dt, decay) sit at [head_base, head_base + heads).  Every
    stream is zero outside its values.
    """

    def __init__(self, cc, layout: StateLayout, b_base: int, c_base: int, head_base: int = 0,
                 decay_base: int | None = None):
        if cc.slots != layout.slots:
            raise _lib.InvalidArgument(-1, "PackedMamba2", "layout slots differ from the context")
        self.cc, self.L = cc, layout
        self.b_base, self.c_base, self.head_base = b_base, c_base, head_base
        # decay may sit in the same ciphertext as dt, at its own offset
        self.decay_base = head_base if decay_base is None else decay_base
        L = layout
        self._state_baby = L.group_heads if L.state_size >= L.group_heads else L.state_size
        self._state_giant = L.state_size // self._state_baby
        self._mask_cache = {}
        self._state_diags = None
        # a PlaintextMemo shared by the caller (None: encode every constant)
        self.memo = None

    # ---- keys -------------------------------------------------------------
    def rotation_steps(self, norm_width: int = 0) -> list[int]:
        L = self.L
        gb, n = L.group_block, L.slots
        s = set()
        s |= {-(gb << i) for i in range(_log2(L.state_size))}         # fill over the state axis
        s |= {gb << i for i in range(_log2(L.state_size))}            # readout rotate-sum
        s |= {-(1 << i) for i in range(_log2(L.head_dim))}            # fill over a head
        s |= {-(1 << i) for i in range(_log2(gb))}                    # fill over a state block
        s |= {g * gb for g in range(1, L.groups)} | {-g * gb for g in range(1, L.groups)}
        s |= {base + L.group_heads * g for g in range(L.groups) for base in (self.head_base, self.decay_base)}
        s |= {-(L.head_dim - 1) * hl for hl in range(1, L.group_heads)}
        s |= {self.b_base, self.c_base}
        stride = -(gb - 1)
        b, G = self._state_baby, self._state_giant
        s |= {j * stride for j in range(1, b)} | {g * b * stride for g in range(1, G)}
        if norm_width:
            win = 1 << max(0, (norm_width - 1).bit_length())
            s |= {1 << i for i in range(_log2(win))} | {-win}
        return sorted(v % n for v in s if v % n)

    # ---- plaintext helpers ------------------------------------------------
    def _block_mask(self, lo: int, hi: int):
        key = (lo, hi)
        if key not in self._mask_cache:
            m = np.zeros(self.L.slots)
            m[lo:hi] = 1.0
            self._mask_cache[key] = m
        return self._mask_cache[key]

    def plain(self, values, level: int = 0, scale: float = 0.0):
        """A constant slot vector as a plaintext (through the memo when set)."""
        if self.memo is not None:
            return self.memo.get(values, level, scale)
        return self.cc.MakeCKKSPackedPlaintext(np.asarray(values, dtype=float), level=level, scale=scale)

    def _plain_for(self, ct, values):
        """Plaintext at the level `ct` multiplies on (after its pending rescale)."""
        c = self.cc
        nq = ct.n_limbs() - (1 if ct.GetNoiseScaleDeg() >= 2 else 0)
        return self.plain(values, level=c.n_q - nq)

    def _mul_mask(self, ct, mask):
        return self.cc.EvalMult(ct, self._plain_for(ct, mask))

    def _fill(self, ct, stride: int, count: int):
        """doubling_fill: copies [0, stride) to count consecutive blocks (needs zeros beyond)."""
        c = self.cc
        for i in range(_log2(count)):
            ct = c.EvalAdd(ct, c.EvalRotate(ct, -(stride << i)))
        return ct

    # ---- expansions into the state layout ---------------------------------
    def expand_x(self, xbc, group: int):
        """x of the group's heads, replicated over the state axis."""
        gb = self.L.group_block
        m = self._mul_mask(xbc, self._block_mask(group * gb, (group + 1) * gb))
        if group:
            m = self.cc.EvalRotate(m, group * gb)
        return self._fill(m, gb, self.L.state_size)

    def expand_heads(self, v, group: int, base: int | None = None):
        """Per-head values (dt, decay) of the group, repeated over channels and states."""
        c, L = self.cc, self.L
        gh, hd = L.group_heads, L.head_dim
        base = self.head_base if base is None else base
        shifted = c.EvalRotate(v, base + gh * group) if base + gh * group else v
        steps = [-(hd - 1) * hl for hl in range(1, gh)]
        rots = [shifted] + (c.EvalFastRotation(shifted, steps) if steps else [])
        acc = None
        for hl, r in enumerate(rots):
            term = self._mul_mask(r, self._block_mask(hl * hd, hl * hd + 1))
            acc = term if acc is None else c.EvalAdd(acc, term)
        acc = self._fill(acc, 1, hd)
        return self._fill(acc, L.group_block, L.state_size)

    def _state_block_diagonals(self, nq: int):
        """Unit diagonals of place_state_blocks: element k of the source lands at slot k * group_block."""
        if self._state_diags is None or self._state_diags[0] != nq:
            L = self.L
            gb, n = L.group_block, L.slots
            stride = -(gb - 1)
            b, G = self._state_baby, self._state_giant
            vals = []
            for g in range(G):
                for j in range(b):
                    t = g * b + j
                    d = np.zeros(n)
                    d[t * gb] = 1.0
                    vals.append(np.roll(d, (g * b * stride) % n))
            pts = self.cc.MakeCKKSPackedPlaintexts(np.array(vals), level=self.cc.n_q - nq)
            self._state_diags = (nq, pts)
        return self._state_diags[1]

    def expand_states(self, xbc, base: int):
        """B or C (state_size values at `base` of the stream), each value filling one state block."""
        c, L = self.cc, self.L
        src = c.EvalRotate(xbc, base)
        src = self._mul_mask(src, self._block_mask(0, L.state_size))
        pts = self._state_block_diagonals(src.n_limbs() - (1 if src.GetNoiseScaleDeg() >= 2 else 0))
        placed = c.EvalLinearTransform(src, pts, self._state_baby, self._state_giant, stride=-(L.group_block - 1))
        return self._fill(placed, 1, L.group_block)

    # ---- recurrence ---------------------------------------------------------
    def update(self, state, decay, x_exp, dt_exp, b_exp):
        """S <- decay * S + (dt * x) * B on one group (state None: first token)."""
        c = self.cc
        upd = c.EvalMult(c.EvalMult(x_exp, dt_exp), b_exp)
        if state is None:
            return upd
        return c.EvalAdd(c.EvalMult(decay, state), upd)

    def readout(self, state, c_exp, group: int):
        """y[h, p] = sum_k S[h, p, k] C[k] for the group's heads, placed at the group's x block."""
        c, L = self.cc, self.L
        gb = L.group_block
        prod = c.EvalMult(state, c_exp)
        for i in range(_log2(L.state_size)):
            prod = c.EvalAdd(prod, c.EvalRotate(prod, gb << i))
        out = self._mul_mask(prod, self._block_mask(0, gb))
        return c.EvalRotate(out, -gb * group) if group else out

    def step(self, states, xbc, dt, decay):
        """One token of the SSM: updates every group's state, returns (states, y stream)."""
        c = self.cc
        b_exp = self.expand_states(xbc, self.b_base)
        c_exp = self.expand_states(xbc, self.c_base)
        new_states, y = [], None
        for g in range(self.L.groups):
            x_g = self.expand_x(xbc, g)
            dt_g = self.expand_heads(dt, g)
            dec_g = self.expand_heads(decay, g, self.decay_base) if states is not None else None
            s = self.update(states[g] if states is not None else None, dec_g, x_g, dt_g, b_exp)
            new_states.append(s)
            r = self.readout(s, c_exp, g)
            y = r if y is None else c.EvalAdd(y, r)
        return new_states, y

    # ---- causal conv ----------------------------------------------------------
    def conv(self, window, weights, bias=None):
        """Depthwise causal conv over a FIFO of stream ciphertexts (oldest first):
        out = sum_i weights[i] (.) window[i] + bias, weights[i] a slot vector per tap."""
        c = self.cc
        if len(window) != len(weights):
            raise _lib.InvalidArgument(-1, "conv", "one weight vector per window entry")
        acc = None
        for ct, w in zip(window, weights):
            if ct is None:
                continue
            t = c.EvalMult(ct, self._plain_for(ct, w))
            acc = t if acc is None else c.EvalAdd(acc, t)
        if bias is not None:
            if acc.GetNoiseScaleDeg() >= 2:
                c.RescaleInPlace(acc)
            acc = c.EvalAdd(acc, self.plain(np.asarray(bias, dtype=float), level=c.n_q - acc.n_limbs(),
                                            scale=acc.GetScalingFactor()))
        return acc

    # ---- polynomial gates -------------------------------------------------
    def poly(self, x, coeffs, lo: float, hi: float, lo_slot: int, hi_slot: int, out_mask=None):
        """Chebyshev series sum c_i T_i(u) on the slots [lo_slot, hi_slot) only:
        u = (2x - lo - hi) / (hi - lo) there and 0 elsewhere (so inactive slots
        stay inside [-1, 1]); the result is masked back to the active slots
        (or multiplied by `out_mask`, a slot vector zero outside them)."""
        c = self.cc
        a = np.zeros(self.L.slots)
        b = np.zeros(self.L.slots)
        a[lo_slot:hi_slot] = 2.0 / (hi - lo)
        b[lo_slot:hi_slot] = -(lo + hi) / (hi - lo)
        u = self._mul_mask(x, a)
        if u.GetNoiseScaleDeg() >= 2:
            c.RescaleInPlace(u)
        u = c.EvalAdd(u, self.plain(b, level=c.n_q - u.n_limbs(), scale=u.GetScalingFactor()))
        out = c.EvalChebyshevSeries(u, coeffs, -1.0, 1.0)
        return self._mul_mask(out, self._block_mask(lo_slot, hi_slot) if out_mask is None else out_mask)

    # ---- RMSNorm ----------------------------------------------------------
    def mean_square(self, x, width: int, eps: float, fill: float):
        """V = mean(x^2) + eps on [0, width) and `fill` on every other slot, for x
        at [0, width) (zeros elsewhere): a copy, a rotate-and-add window sum over
        the next power of two and a 1/width mask.  Two levels below x."""
        c = self.cc
        win = 1 << max(0, (width - 1).bit_length())
        sq = c.EvalMult(x, x)
        sq = c.EvalAdd(sq, c.EvalRotate(sq, -win))
        for i in range(_log2(win)):
            sq = c.EvalAdd(sq, c.EvalRotate(sq, 1 << i))
        inv = np.zeros(self.L.slots)
        inv[:width] = 1.0 / width
        v = self._mul_mask(sq, inv)  # mean(x^2) on [0, width), 0 elsewhere
        if v.GetNoiseScaleDeg() >= 2:
            c.RescaleInPlace(v)
        shift = np.full(self.L.slots, fill)
        shift[:width] = eps
        return c.EvalAdd(v, self.plain(shift, level=c.n_q - v.n_limbs(), scale=v.GetScalingFactor()))

    def scale_rows(self, x, y, width: int, weight):
        """x * y * weight on [0, width): the normalised, weighted vector."""
        w = np.zeros(self.L.slots)
        w[:width] = np.asarray(weight, dtype=float)
        xy = self.cc.EvalMult(x, y)
        return self.cc.EvalMult(xy, self._plain_for(xy, w))

    def rms_norm(self, x, width: int, weight, eps: float, domain, degree: int = 31, newton: int = 2):
        """x * rsqrt(mean(x^2) + eps) * weight for x at [0, width) (zeros elsewhere).

        V = mean(x^2) + eps (`mean_square`, slots outside [0, width) set to the
        middle of `domain`, the bounds of V, so that they stay inside it) is the
        input of a Chebyshev seed of rsqrt, which Newton steps
        y <- 1.5 y - 0.5 V y^3 refine (the reference's newton_refine works on
        sum + width * eps and rescales by sqrt(width); the mean form keeps every
        constant small)."""
        c = self.cc
        lo, hi = domain
        v = self.mean_square(x, width, eps, 0.5 * (lo + hi))
        y = c.EvalChebyshevFunction(lambda t: 1.0 / np.sqrt(t), v, lo, hi, degree)
        v_neg_half = c.EvalMult(v, -0.5)
        for _ in range(newton):
            y2 = c.EvalMult(y, y)
            vy = c.EvalMult(v_neg_half, y)
            y = c.EvalAdd(c.EvalMult(y, 1.5), c.EvalMult(vy, y2))
        return self.scale_rows(x, y, width, weight)
