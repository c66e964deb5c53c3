"""Limb-sharded HYBRID key switching across GPUs, one process per GPU.

The north star partitions the CKKS state "over one 8xB200 box by RNS limb,
with NCCL over NVLink only for the basis-conversion exchange in key
switching".  Limbs are dealt out round-robin: rank r of W owns the Q limbs
l % W == r and the P limbs p % W == r.  Limb-local work (NTT, products,
rescale epilogue, automorphism) needs no communication; a key switch (the
reference's FIDESlib KeySwitch behind EvalMult / EvalRotate,
native/fideslib_stage0/src/packed_fideslib.cpp:149,215-217) takes two
all-gathers between three device stages of libfhe_b200:

    modup_prepare  INTT of the own rows of d            -> all-gather [W][q_chunk][N]
    inner          ModUp to the own extended rows, key inner product, INTT of
                   the own P rows of the accumulator     -> all-gather [W][2][p_chunk][N]
    moddown        P -> own Q conversion, (acc - conv) P^{-1} (+ addends)

The collectives are torch.distributed (NCCL on GPUs, gloo in the CPU tests of
the host logic) issued on the context's CUDA stream, so the device stages and
the exchanges stay ordered without host synchronisation.  Every output word
equals the single-GPU key switch's.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np

from . import _lib
from ._lib import call, vp


@dataclass(frozen=True)
class ShardPlan:
    """Round-robin limb ownership (host logic; fhe_shard_plan_get computes
    the same numbers in the library)."""
    n_q: int      # Q limbs of the context (L)
    n_p: int      # P limbs (K)
    alpha: int    # limbs per HYBRID digit
    rank: int
    world: int

    def q_limbs(self, nq: int) -> list[int]:
        return list(range(self.rank, nq, self.world))

    def p_limbs(self) -> list[int]:
        return list(range(self.rank, self.n_p, self.world))

    def q_chunk(self, nq: int) -> int:
        return -(-nq // self.world)

    @property
    def p_chunk(self) -> int:
        return -(-self.n_p // self.world)

    def rows(self, nq: int) -> int:
        return len(self.q_limbs(nq)) + len(self.p_limbs())

    def digits(self, nq: int) -> int:
        return -(-nq // self.alpha)

    def gathered_q_row(self, l: int, nq: int) -> int:
        """Row of Q limb l in the first all-gather's output [W][q_chunk][N]."""
        return (l % self.world) * self.q_chunk(nq) + l // self.world

    def gathered_p_row(self, p: int, comp: int) -> int:
        """Row of P limb p, component comp, in the second all-gather's output [W][2][p_chunk][N]."""
        return ((p % self.world) * 2 + comp) * self.p_chunk + p // self.world

    # per-digit exchange (fhe_shard_inner_digit)
    @property
    def digit_chunk(self) -> int:
        """Rows per rank in a digit's all-gather: ceil(alpha / world)."""
        return -(-self.alpha // self.world)

    def digit_rows(self, nq: int, j: int) -> tuple[int, int]:
        """[lo, hi): this rank's own rows (send-buffer rows) of HYBRID digit j."""
        lo, hi = j * self.alpha, min((j + 1) * self.alpha, nq)
        rows = [i for i, l in enumerate(self.q_limbs(nq)) if lo <= l < hi]
        return (rows[0], rows[-1] + 1) if rows else (0, 0)

    def split_row(self, l: int) -> int:
        """Row of Q limb l in its digit's all-gather output [W][digit_chunk][N]
        (the library's source-row map of fhe_shard_inner_digit)."""
        lo = (l // self.alpha) * self.alpha
        first = lo + (l % self.world - lo % self.world) % self.world
        return (l % self.world) * self.digit_chunk + (l - first) // self.world

    # host-side packing (numpy or torch arrays of rows)
    def own_rows(self, full, nq: int):
        """The own Q rows of a [..., nq, N] array."""
        return full[..., self.rank:nq:self.world, :]

    def pack_send(self, own, nq: int, xp=np):
        """Own rows [q_own, N] -> zero-padded send buffer [q_chunk, N]."""
        out = xp.zeros((self.q_chunk(nq),) + tuple(own.shape[1:]), dtype=own.dtype)
        out[: own.shape[0]] = own
        return out

    def unpack_gathered(self, gathered, nq: int):
        """First all-gather's output [W * q_chunk, N] -> all limbs [nq, N] in limb order."""
        idx = [self.gathered_q_row(l, nq) for l in range(nq)]
        return gathered[idx]


def all_gather_rows(send, group=None):
    """[rows, ...] on every rank -> [world * rows, ...] in rank order."""
    import torch
    import torch.distributed as dist
    world = dist.get_world_size(group)
    out = torch.empty((world * send.shape[0],) + tuple(send.shape[1:]), dtype=send.dtype, device=send.device)
    dist.all_gather_into_tensor(out, send.contiguous(), group=group)
    return out


class ShardedKeySwitch:
    """Key switching of limb-sharded ciphertexts on this rank's GPU.

    ``cc`` is the rank's CryptoContext (same parameters and key seed on every
    rank, created on the rank's device).  Ciphertexts are torch int64 tensors
    holding the own Q rows ([components][q_own][N], bit patterns of the u64
    residues)."""

    def __init__(self, cc, group=None, rank=None, world=None, device=None):
        import torch
        import torch.distributed as dist
        self.cc, self.group = cc, group
        self.rank = dist.get_rank(group) if rank is None else rank
        self.world = dist.get_world_size(group) if world is None else world
        if device is not None:
            torch.cuda.set_device(device)
        call("fhe_shard_init", cc.h, self.rank, self.world)
        self.plan = ShardPlan(cc.n_q, cc.n_p, cc.alpha, self.rank, self.world)
        self.device = torch.device("cuda", torch.cuda.current_device())
        self.stream = torch.cuda.ExternalStream(cc.stream_ptr(), device=self.device)

    def plan_info(self, nq: int) -> dict:
        buf = (ctypes.c_uint32 * 8)()
        call("fhe_shard_plan_get", self.cc.h, nq, ctypes.cast(buf, vp))
        keys = ("n_limbs", "q_own", "q_chunk", "p_own", "p_chunk", "rows", "digits")
        return dict(zip(keys, list(buf)[:7]))

    def load_key(self, kind: int, galois: int = 0):
        call("fhe_shard_load_key", self.cc.h, kind, galois)

    @staticmethod
    def _p(t):
        return None if t is None else vp(t.data_ptr())

    # the three device stages (enqueued on the context stream)
    def stage_prepare(self, d_own, nq: int):
        import torch
        send = torch.empty((self.plan.q_chunk(nq), self.cc.n), dtype=torch.int64, device=self.device)
        call("fhe_shard_modup_prepare", self.cc.h, nq, self._p(d_own), self._p(send))
        return send

    def stage_inner(self, nq: int, kind: int, galois: int, gathered, d_own):
        import torch
        pl, n = self.plan, self.cc.n
        acc = torch.empty((2, pl.rows(nq), n), dtype=torch.int64, device=self.device)
        p_send = torch.empty((2, pl.p_chunk, n), dtype=torch.int64, device=self.device)
        call("fhe_shard_inner", self.cc.h, nq, kind, galois, self._p(gathered), self._p(d_own), self._p(acc),
             self._p(p_send))
        return acc, p_send

    def digit_rows(self, nq: int, j: int) -> tuple[int, int]:
        return self.plan.digit_rows(nq, j)

    def stage_inner_split(self, nq: int, kind: int, galois: int, send, d_own):
        """The inner stage with the first exchange split by digit: digit j + 1's
        all-gather (asynchronous, NCCL's own stream) overlaps digit j's
        conversion on the context stream."""
        import torch
        import torch.distributed as dist
        pl, n, W = self.plan, self.cc.n, self.world
        D = pl.digits(nq)
        dchunk = pl.digit_chunk
        gathered = torch.empty((D, W * dchunk, n), dtype=torch.int64, device=self.device)
        works = []
        for j in range(D):
            lo, hi = self.digit_rows(nq, j)
            part = torch.zeros((dchunk, n), dtype=torch.int64, device=self.device)
            if hi > lo:
                part[: hi - lo] = send[lo:hi]
            works.append(dist.all_gather_into_tensor(gathered[j], part, group=self.group, async_op=True))
        for j in range(D):
            works[j].wait()  # the context stream waits for digit j's rows only
            call("fhe_shard_inner_digit", self.cc.h, nq, j, self._p(gathered[j]), self._p(d_own))
        acc = torch.empty((2, pl.rows(nq), n), dtype=torch.int64, device=self.device)
        p_send = torch.empty((2, pl.p_chunk, n), dtype=torch.int64, device=self.device)
        call("fhe_shard_inner_tail", self.cc.h, nq, kind, galois, self._p(acc), self._p(p_send))
        return acc, p_send

    def stage_moddown(self, nq: int, acc, p_gathered, add0=None, add1=None):
        import torch
        out = torch.empty((2, len(self.plan.q_limbs(nq)), self.cc.n), dtype=torch.int64, device=self.device)
        call("fhe_shard_moddown", self.cc.h, nq, self._p(acc), self._p(p_gathered), self._p(add0), self._p(add1),
             self._p(out))
        return out

    STAGES = ("modup_prepare", "gather_modup_rows", "modup_inner", "gather_p_rows", "moddown")

    def keyswitch(self, d_own, nq: int, kind: int, galois: int = 0, add0=None, add1=None, events=None,
                  split: bool = False):
        """[2][q_own][N]: KS(d) (+ add0 on component 0, + add1 on component 1).
        events: optional list of 6 CUDA timing events, recorded on the context
        stream around the five steps (STAGES), for a per-step breakdown.
        split: the first exchange runs per digit, overlapped with the
        conversions (its events then bracket the gathers and conversions
        together)."""
        import torch
        q_own = len(self.plan.q_limbs(nq))
        assert tuple(d_own.shape) == (q_own, self.cc.n) and d_own.dtype == torch.int64
        caller = torch.cuda.current_stream(self.device)
        self.stream.wait_stream(caller)

        def mark(i):
            if events is not None:
                events[i].record(self.stream)

        with torch.cuda.stream(self.stream):
            mark(0)
            send = self.stage_prepare(d_own, nq)
            mark(1)
            if split:
                acc, p_send = self.stage_inner_split(nq, kind, galois, send, d_own)
                mark(2)
            else:
                gathered = all_gather_rows(send, self.group)
                mark(2)
                acc, p_send = self.stage_inner(nq, kind, galois, gathered, d_own)
            mark(3)
            p_gathered = all_gather_rows(p_send, self.group)
            mark(4)
            out = self.stage_moddown(nq, acc, p_gathered, add0, add1)
            mark(5)
        caller.wait_stream(self.stream)
        return out

    def relinearize(self, ct_own, nq: int, events=None, split: bool = False):
        """(d0, d1, d2) own rows -> (d0 + KS0(d2), d1 + KS1(d2)) with the relinearisation key."""
        self.load_key(2)
        return self.keyswitch(ct_own[2], nq, 2, 0, ct_own[0], ct_own[1], events, split)

    def rotate(self, ct_own, nq: int, step: int):
        """EvalRotate of own rows: KS(c1) + (c0, 0), then the automorphism."""
        import torch
        g = self.cc.galois_element(step)
        self.load_key(3, g)
        u = self.keyswitch(ct_own[1], nq, 3, g, ct_own[0], None)
        return self.automorphism(u, nq, g)

    def automorphism(self, u, nq: int, galois: int):
        import torch
        caller = torch.cuda.current_stream(self.device)
        self.stream.wait_stream(caller)
        with torch.cuda.stream(self.stream):
            out = torch.empty_like(u)
            call("fhe_shard_automorphism", self.cc.h, nq, galois, self._p(u), self._p(out))
        caller.wait_stream(self.stream)
        return out


def to_device_rows(arr: np.ndarray, device):
    """u64 numpy rows -> int64 torch tensor on `device` (same bits)."""
    import torch
    return torch.from_numpy(np.ascontiguousarray(arr).view(np.int64)).to(device)


def to_host_rows(t) -> np.ndarray:
    """int64 torch tensor -> u64 numpy array (same bits)."""
    return t.detach().cpu().numpy().view(np.uint64)


__all__ = ["ShardPlan", "ShardedKeySwitch", "all_gather_rows", "to_device_rows", "to_host_rows", "_lib"]
