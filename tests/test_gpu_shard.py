"""Limb-sharded key switching on the device.

W ranks are emulated on one GPU (one context per rank, the two all-gathers
done by concatenation with host synchronisation between the stages), so the
multi-rank arithmetic is checked without needing W GPUs: every own row of a
sharded relinearisation and rotation must equal the single-GPU result word
for word (which itself equals the oracle's, test_gpu_ckks.py).  With two or
more GPUs the same key switch also runs as two NCCL ranks.
"""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

SEED = 77
PARAMS = dict(ring_dim=1 << 13, multiplicative_depth=11, scaling_mod_size=50, first_mod_size=60,
              num_large_digits=3)


def _ctx():
    from fhe_mamba_b200 import CCParams, CryptoContext
    cc = CryptoContext(CCParams(**PARAMS))
    cc.KeyGen(SEED)
    return cc


def _rand_ct(cc, nq, ncomp, seed):
    rng = np.random.default_rng(seed)
    x = np.empty((ncomp, nq, cc.n), dtype=np.uint64)
    for l in range(nq):
        x[:, l, :] = rng.integers(0, cc.q[l], size=(ncomp, cc.n), dtype=np.uint64)
    return x


def _emulated_keyswitch(ranks, d_full, nq, kind, galois, add0_full=None, add1_full=None):
    """Run the three stages on every emulated rank; returns [rank] -> [2][q_own][N] (u64)."""
    import torch
    from fhe_mamba_b200.shard import to_device_rows, to_host_rows
    dev = torch.device("cuda", 0)

    def own(sk, full):
        return None if full is None else to_device_rows(sk.plan.own_rows(full, nq), dev)

    d_own = [own(sk, d_full) for sk in ranks]
    torch.cuda.synchronize()
    sends = [sk.stage_prepare(d, nq) for sk, d in zip(ranks, d_own)]
    for sk in ranks:
        sk.cc.synchronize()
    gathered = torch.cat(sends)
    torch.cuda.synchronize()
    inner = [sk.stage_inner(nq, kind, galois, gathered, d) for sk, d in zip(ranks, d_own)]
    for sk in ranks:
        sk.cc.synchronize()
    p_gathered = torch.cat([ps for _, ps in inner])
    torch.cuda.synchronize()
    outs = []
    for sk, (acc, _) in zip(ranks, inner):
        outs.append(sk.stage_moddown(nq, acc, p_gathered, own(sk, add0_full), own(sk, add1_full)))
    for sk in ranks:
        sk.cc.synchronize()
    torch.cuda.synchronize()
    return outs, to_host_rows


@pytest.fixture(scope="module")
def setup():
    import torch
    torch.cuda.set_device(0)
    ref = _ctx()
    return ref


@pytest.mark.parametrize("world", [2, 3])
def test_plan_matches_library(setup, world):
    from fhe_mamba_b200.shard import ShardedKeySwitch
    for r in range(world):
        cc = _ctx()
        sk = ShardedKeySwitch(cc, rank=r, world=world)
        for nq in (1, 2, 5, cc.n_q):
            info = sk.plan_info(nq)
            pl = sk.plan
            assert info == {"n_limbs": nq, "q_own": len(pl.q_limbs(nq)), "q_chunk": pl.q_chunk(nq),
                            "p_own": len(pl.p_limbs()), "p_chunk": pl.p_chunk, "rows": pl.rows(nq),
                            "digits": pl.digits(nq)}


@pytest.mark.parametrize("world,nq", [(1, 12), (2, 12), (3, 12), (2, 7), (3, 2), (4, 9)])
def test_sharded_relinearize_and_rotate_equal_single_gpu(setup, world, nq):
    from fhe_mamba_b200.shard import ShardedKeySwitch
    ref = setup
    ranks = [ShardedKeySwitch(_ctx(), rank=r, world=world) for r in range(world)]
    d = _rand_ct(ref, nq, 3, 100 + world * 16 + nq)
    want = ref.Relinearize(ref.upload(d, noise_deg=2)).residues()
    for sk in ranks:
        sk.load_key(2)
    outs, host = _emulated_keyswitch(ranks, d[2], nq, 2, 0, d[0], d[1])
    for sk, o in zip(ranks, outs):
        assert np.array_equal(host(o), sk.plan.own_rows(want, nq)), (world, nq, sk.rank)

    step = 3
    ref.EvalRotateKeyGen([step])
    g = ref.galois_element(step)
    c = _rand_ct(ref, nq, 2, 200 + world * 16 + nq)
    want = ref.EvalRotate(ref.upload(c), step).residues()
    for sk in ranks:
        sk.load_key(3, g)
    outs, host = _emulated_keyswitch(ranks, c[1], nq, 3, g, c[0], None)
    for sk, u in zip(ranks, outs):
        rot = sk.automorphism(u, nq, g)
        sk.cc.synchronize()
        assert np.array_equal(host(rot), sk.plan.own_rows(want, nq)), (world, nq, sk.rank)


@pytest.mark.parametrize("world,nq", [(2, 12), (3, 12), (4, 9), (3, 2)])
def test_split_exchange_equals_single_gpu(setup, world, nq):
    """The first exchange split by HYBRID digit (fhe_shard_inner_digit /
    fhe_shard_inner_tail, what ShardedKeySwitch(split=True) overlaps with the
    conversions): each digit's padded rows of every rank concatenated, the
    result equal to the single-GPU relinearisation word for word."""
    import torch
    from fhe_mamba_b200._lib import call
    from fhe_mamba_b200.shard import ShardedKeySwitch, to_device_rows, to_host_rows
    ref = setup
    dev = torch.device("cuda", 0)
    ranks = [ShardedKeySwitch(_ctx(), rank=r, world=world) for r in range(world)]
    d = _rand_ct(ref, nq, 3, 300 + world * 16 + nq)
    want = ref.Relinearize(ref.upload(d, noise_deg=2)).residues()
    for sk in ranks:
        sk.load_key(2)
    own = [to_device_rows(sk.plan.own_rows(d[2], nq), dev) for sk in ranks]
    torch.cuda.synchronize()
    sends = [sk.stage_prepare(x, nq) for sk, x in zip(ranks, own)]
    for sk in ranks:
        sk.cc.synchronize()
    pl = ranks[0].plan
    dchunk = -(-pl.alpha // world)
    for j in range(pl.digits(nq)):
        parts = []
        for sk, snd in zip(ranks, sends):
            lo, hi = sk.digit_rows(nq, j)
            part = torch.zeros((dchunk, ref.n), dtype=torch.int64, device=dev)
            if hi > lo:
                part[: hi - lo] = snd[lo:hi]
            parts.append(part)
        gathered = torch.cat(parts)
        torch.cuda.synchronize()
        for sk, x in zip(ranks, own):
            call("fhe_shard_inner_digit", sk.cc.h, nq, j, sk._p(gathered), sk._p(x))
            sk.cc.synchronize()
    inner = []
    for sk in ranks:
        acc = torch.empty((2, sk.plan.rows(nq), ref.n), dtype=torch.int64, device=dev)
        p_send = torch.empty((2, sk.plan.p_chunk, ref.n), dtype=torch.int64, device=dev)
        call("fhe_shard_inner_tail", sk.cc.h, nq, 2, 0, sk._p(acc), sk._p(p_send))
        sk.cc.synchronize()
        inner.append((acc, p_send))
    p_gathered = torch.cat([ps for _, ps in inner])
    torch.cuda.synchronize()
    for sk, (acc, _) in zip(ranks, inner):
        a0 = to_device_rows(sk.plan.own_rows(d[0], nq), dev)
        a1 = to_device_rows(sk.plan.own_rows(d[1], nq), dev)
        out = sk.stage_moddown(nq, acc, p_gathered, a0, a1)
        sk.cc.synchronize()
        assert np.array_equal(to_host_rows(out), sk.plan.own_rows(want, nq)), (world, nq, sk.rank)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _nccl_worker(rank, world, port, results):
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    from fhe_mamba_b200 import CCParams, CryptoContext
    from fhe_mamba_b200.shard import ShardedKeySwitch, to_device_rows, to_host_rows
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=120), device_id=torch.device("cuda", rank))
    try:
        cc = CryptoContext(CCParams(**PARAMS, device=rank))
        cc.KeyGen(SEED)
        sk = ShardedKeySwitch(cc)
        nq = cc.n_q
        d = _rand_ct(cc, nq, 3, 4242)
        want = cc.Relinearize(cc.upload(d, noise_deg=2)).residues()
        dev = torch.device("cuda", rank)
        own = to_device_rows(sk.plan.own_rows(d, nq), dev)
        out = sk.relinearize(own, nq)
        torch.cuda.synchronize()
        ok = np.array_equal(to_host_rows(out), sk.plan.own_rows(want, nq))
        out = sk.relinearize(own, nq, split=True)  # per-digit exchange overlapped with the conversions
        torch.cuda.synchronize()
        ok = ok and np.array_equal(to_host_rows(out), sk.plan.own_rows(want, nq))
        cc.EvalRotateKeyGen([5])
        c = _rand_ct(cc, nq, 2, 4343)
        want = cc.EvalRotate(cc.upload(c), 5).residues()
        rot = sk.rotate(to_device_rows(sk.plan.own_rows(c, nq), dev), nq, 5)
        torch.cuda.synchronize()
        ok = ok and np.array_equal(to_host_rows(rot), sk.plan.own_rows(want, nq))
        results[rank] = bool(ok)
    finally:
        dist.destroy_process_group()


def test_nccl_two_ranks():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    results = ctx.Manager().dict()
    port = _free_port()
    procs = [ctx.Process(target=_nccl_worker, args=(r, 2, port, results)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
        assert p.exitcode == 0
    assert results[0] and results[1]
