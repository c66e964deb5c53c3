"""Host logic of limb-sharded key switching, on CPU: round-robin ownership,
the padded all-gather layouts, and the exchange itself over world-size 2 and
3 gloo process groups (the NCCL path on GPUs runs the same functions)."""
import os
import socket

import numpy as np
import pytest

from fhe_mamba_b200.shard import ShardPlan


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
@pytest.mark.parametrize("nq", [1, 2, 7, 20, 45])
def test_every_limb_has_one_owner(world, nq):
    L, K, alpha = 45, 15, 15
    owners = {}
    for r in range(world):
        pl = ShardPlan(L, K, alpha, r, world)
        for l in pl.q_limbs(nq):
            assert l not in owners
            owners[l] = r
        assert len(pl.q_limbs(nq)) <= pl.q_chunk(nq)
        assert len(pl.p_limbs()) <= pl.p_chunk
        # the own rows of a lower level are a prefix of the own rows of L
        assert pl.q_limbs(nq) == pl.q_limbs(L)[: len(pl.q_limbs(nq))]
    assert sorted(owners) == list(range(nq))
    counts = [len(ShardPlan(L, K, alpha, r, world).q_limbs(nq)) for r in range(world)]
    assert max(counts) - min(counts) <= 1
    ps = sorted(p for r in range(world) for p in ShardPlan(L, K, alpha, r, world).p_limbs())
    assert ps == list(range(K))


def test_gathered_rows_are_a_permutation():
    for world in (2, 3, 8):
        pl = ShardPlan(45, 15, 15, 0, world)
        for nq in (5, 45):
            rows = [pl.gathered_q_row(l, nq) for l in range(nq)]
            assert len(set(rows)) == nq and max(rows) < world * pl.q_chunk(nq)
        prow = [pl.gathered_p_row(p, c) for p in range(15) for c in (0, 1)]
        assert len(set(prow)) == 30 and max(prow) < world * 2 * pl.p_chunk


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _exchange_worker(rank, world, port, nq, K, n, results):
    import torch
    import torch.distributed as dist
    from fhe_mamba_b200.shard import ShardPlan, all_gather_rows
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(5)  # same full arrays on every rank
        full = rng.integers(0, 2**62, size=(nq, n), dtype=np.int64)
        pfull = rng.integers(0, 2**62, size=(2, K, n), dtype=np.int64)
        pl = ShardPlan(45, K, 15, rank, world)
        # first exchange: own Q rows -> every limb in limb order
        send = pl.pack_send(torch.from_numpy(pl.own_rows(full, nq)), nq, xp=torch)
        gathered = all_gather_rows(send)
        ok_q = np.array_equal(pl.unpack_gathered(gathered, nq).numpy(), full)
        # second exchange: own P rows of both components, [2][p_chunk][N] per rank
        p_send = torch.zeros((2, pl.p_chunk, n), dtype=torch.int64)
        for i, p in enumerate(pl.p_limbs()):
            p_send[:, i] = torch.from_numpy(pfull[:, p])
        pg = all_gather_rows(p_send).reshape(-1, n).numpy()
        ok_p = all(np.array_equal(pg[pl.gathered_p_row(p, c)], pfull[c, p]) for p in range(K) for c in (0, 1))
        results[rank] = bool(ok_q and ok_p)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,nq", [(2, 20), (2, 45), (3, 7), (3, 20)])
def test_gloo_exchange_reassembles_limbs(world, nq):
    import torch.multiprocessing as mp
    port = _free_port()
    ctx = mp.get_context("spawn")
    results = ctx.Manager().dict()
    procs = [ctx.Process(target=_exchange_worker, args=(r, world, port, nq, 15, 64, results)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    assert all(results[r] for r in range(world))


@pytest.mark.parametrize("world", [2, 3, 4, 8])
@pytest.mark.parametrize("nq,alpha", [(45, 15), (20, 7), (31, 15), (9, 4), (2, 15)])
def test_digit_split_exchange_places_every_limb(world, nq, alpha):
    """Per-digit exchange: every rank's own rows of digit j, padded to
    ceil(alpha / W) rows and gathered in rank order, put Q limb l of the digit
    at the row the library's conversion reads (ShardPlan.split_row)."""
    from fhe_mamba_b200.shard import ShardPlan
    plans = [ShardPlan(n_q=45, n_p=15, alpha=alpha, rank=r, world=world) for r in range(world)]
    dc = plans[0].digit_chunk
    for j in range(plans[0].digits(nq)):
        gathered = []
        for pl in plans:
            lo, hi = pl.digit_rows(nq, j)
            rows = [pl.q_limbs(nq)[i] for i in range(lo, hi)]
            assert len(rows) <= dc
            gathered += rows + [None] * (dc - len(rows))
        for l in range(j * alpha, min((j + 1) * alpha, nq)):
            assert gathered[plans[0].split_row(l)] == l, (j, l)
