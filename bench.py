"""Benchmark driver (one JSON line on rank 0).

Headline (BASELINE metric "enc s/generated token (Mamba-2-130M shape)"): the
encrypted greedy token loop of a 24-layer Mamba-2-130M-shape model (d_model
768, d_inner 1536, d_state 128, 24 heads, conv 4, vocab 50280, tied
embedding; synthetic seeded weights ~N(0, 0.02^2)) at N = 2^16, 2^15 slots,
multiplicative depth 44, 59-bit scaling / 60-bit first prime, dnum 3,
two-pass bootstrapping.  One step = one generated token: the server runs all
24 layers on the encrypted embedding (value, CUDA events on the context
stream), the client encrypts the embedding and decrypts + selects the next
token around it (e2e).  Inputs: keys (~36 GB), cached diagonals and
ciphertexts far exceed the 126 MB L2.

Roofline: BASELINE config 2, the batched forward NTT (4 polys x 36 limbs x
2^16, 59-bit primes) -- the dominant kernel of every primitive -- timed with
CUDA events; key switching (config 3 shape) and bootstrapping are reported
beside it.

Timing: W untimed warm-up tokens, then exactly K tokens bracketed by a
barrier and torch.cuda.synchronize() on both sides; the device time is the
max over ranks.  Multi-GPU (torchrun): every rank runs its own replica of the
token loop (the layers are sequential; no data-path collective); value =
max time / tokens of all ranks.

``--impl reference``: FIDESlib/OpenFHE are not in the reference checkout and
cannot be built here; the reference arm times the CPU oracle (the
restatement of OpenFHE's algorithms) on one key switch at the token loop's
typical level with all host threads and scales it by the key switches of one
token (a labelled estimate; a full CPU token would take hours).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "enc s/generated token (Mamba-2-130M shape); NTT+keyswitch % HBM roofline"
UNIT = "s/generated token"
NTT_UNIT = "batched fwd+inv NTT steps/s (4 polys x 36 limbs x 2^16)"
LOG_N, LIMBS, POLYS, BITS = 16, 36, 4, 59
# Per-level operation counts of one generated token, recorded by the GPU arm
# (per_token.level_counts of its JSON line) and read by the CPU reference arm.
LEVEL_COUNTS = os.path.join(ROOT, "profiles", "token_level_counts.json")
ALG_BYTES_PER_TRANSFORM = 16 * POLYS * LIMBS * (1 << LOG_N)  # read + write every word once
N_ROTATE = 4
# Kernel of the key switches' basis conversions in the token loop and the
# side measurements ("tensor": tcgen05 int8 MMA, "cuda": 64-bit CUDA-core
# multiply-accumulates; identical words).  Set from --conversion.
CONVERSION = "tensor"
# Byte budget of the encoded-diagonal cache of the layers' matvecs (--diagonal-cache-gb).
# The diagonals are generated and encoded on the device from the weights at every
# matvec: measured 20.2 s per steady evaluation against 20.1 s with a 40 GB cache,
# and 23.4 instead of 30.7 s for the first (host-built diagonals filling the cache).
DIAGONAL_CACHE_GB = 0.0
# Key inner product of the Q limbs inside ModDown's last NTT pass (--keyswitch-fusion).
FUSED_KEY_INNER = False
# Budget of the memo of the layers' constant plaintexts (masks, taps, biases
# by level and scale; --constant-memo-gb, 0: encode at every use).
MEMO_GB = 16.0
# Slot counts of the sub-slot refreshes (--subslot-refresh): a refresh of a
# value known to be zero outside [0, n) bootstraps n slots with one EvalMod.
# Two-pass refresh at N = 2^16: 158 ms over all slots, 115 ms over 4096, 105 ms
# over 2048; the steady evaluation 15.8 s with (4096, 2048) against 20.1 s.
SUBSLOT_SIZES = (4096, 2048)
# Their level budget {CoeffToSlot, SlotToCoeff} (--subslot-budget).  {3, 3}
# returns two more limbs, which drops the packed-input refresh; but the
# carried states, updated from that input, then run out of levels every 4
# tokens instead of every 12 (slot model, 36 tokens: 76.8 sub-slot + 35.4
# full refreshes per token against 96.5 + 14.7), so {4, 4} stays.
SUBSLOT_BUDGET = (4, 4)


_JSON_OUT = None


def json_stdout():
    """Keeps file descriptor 1 for the JSON line alone: anything else written
    to it (NCCL's version banner, library logs, Python prints) goes to
    stderr from here on."""
    global _JSON_OUT
    if _JSON_OUT is None:
        sys.stdout.flush()
        _JSON_OUT = os.fdopen(os.dup(1), "w")
        os.dup2(2, 1)
        sys.stdout = sys.stderr
    return _JSON_OUT


def emit(obj):
    out = json_stdout()
    out.write(json.dumps(obj) + "\n")
    out.flush()


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        d = json.load(open(path))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def ncu_traffic():
    """Per-launch DRAM bytes of the forward transform from the committed ncu summary."""
    path = os.path.join(ROOT, "profiles", "ntt_fwd_config2.md")
    if not os.path.exists(path):
        return None
    for line in open(path):
        if line.startswith("traffic_bytes_per_forward_transform:"):
            try:
                return int(line.split(":", 1)[1].strip())
            except ValueError:
                return None
    return None


def bench_primes():
    # The 36 largest primes below 2^59 that are 1 mod 2N (host-side, product code).
    from fhe_mamba_b200.params import ntt_primes
    return ntt_primes(LOG_N, BITS, LIMBS)


def make_batch(qs, seed):
    rng = np.random.default_rng(seed)
    n = 1 << LOG_N
    out = np.empty((POLYS, LIMBS, n), dtype=np.uint64)
    for l, q in enumerate(qs):
        out[:, l, :] = rng.integers(0, q, size=(POLYS, n), dtype=np.uint64)
    return out


class ClockSampler:
    """nvidia-smi clocks/throttle sampling during the timed region."""

    FIELDS = ("index,uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, uuid):
        self.uuid = uuid
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.3)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            f = [x.strip() for x in line.split(",")]
            if len(f) < 10:
                continue
            if self.uuid and self.uuid not in f[1]:
                continue
            try:
                sm.append(float(f[2]))
                mx = float(f[3])
            except ValueError:
                continue
            for name, v in zip(names, f[6:10]):
                if v.lower() == "active":
                    reasons.add(name)
        os.unlink(self.path)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def cpu_level_times(levels, threads):
    """Seconds of one ModUp, one key inner product with its ModDown pair, one
    rescale (2 components) and one tensor product at each number of live Q
    limbs in `levels`, on the CPU oracle (OpenFHE's algorithms restated in C,
    OpenMP over the host threads) at the token loop's parameters (N = 2^16,
    depth 44, 59/60-bit primes, dnum 3)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    os.environ["OMP_NUM_THREADS"] = str(threads)
    q, p = O.ckks_moduli(16, 45, 59, 60, 3)
    oc = O.Ckks(16, q, p, 3, 1 << 15)
    s, sn = oc.keygen_secret(1)
    rlk = oc.relin_key(1, sn)
    rng = np.random.default_rng(0)
    out = {}
    for nq in sorted(levels):
        if nq < 1 or nq > len(q):
            continue
        d = np.empty((2, nq, 1 << 16), dtype=np.uint64)
        for l in range(nq):
            d[:, l, :] = rng.integers(0, q[l], size=(2, 1 << 16), dtype=np.uint64)
        t0 = time.perf_counter()
        ext = oc.modup(d[1], nq)
        t1 = time.perf_counter()
        acc = oc.key_inner(ext, nq, rlk)
        oc.moddown(acc[0], nq)
        oc.moddown(acc[1], nq)
        t2 = time.perf_counter()
        if nq >= 2:
            oc.rescale(d)
        t3 = time.perf_counter()
        oc.tensor(d, d)
        t4 = time.perf_counter()
        out[nq] = {"modup": t1 - t0, "key_inner": t2 - t1, "rescale": t3 - t2, "tensor": t4 - t3}
    return out


def cpu_estimate(level_counts, threads):
    """CPU seconds of one token from the GPU's per-level operation counts and
    the oracle's time for each operation at each level: key switching (ModUp,
    key inner product, ModDown), rescales and tensor products, NTTs included.
    Automorphisms, additions, plaintext products and encodes are not counted,
    so this is a lower bound of the CPU token."""
    levels = set()
    for kind in level_counts.values():
        levels |= {int(k) for k in kind}
    t0 = time.perf_counter()
    times = cpu_level_times(levels, threads)
    measured = time.perf_counter() - t0
    total = 0.0
    for kind, per in level_counts.items():
        for nq, count in per.items():
            total += float(count) * times.get(int(nq), {}).get(kind, 0.0)
    ops = sum(float(c) for per in level_counts.values() for c in per.values())
    return total, measured, ops, len(times)


def cpu_baseline(level_counts, threads):
    value, measured, ops, levels = cpu_estimate(level_counts, threads)
    return {"value": value, "unit": UNIT, "cores": threads, "kind": "port", "estimate": True,
            "measured_seconds": measured, "extrapolation_factor": value / measured if measured else None,
            "sample": (f"the CPU oracle timed once per operation kind at each of {levels} levels "
                       f"({measured:.1f} s), weighted by this run's {ops:.0f} counted operations per token "
                       "(ModUp, key inner product + ModDown, rescale, tensor); a lower bound: automorphisms, "
                       "additions, plaintext products and encodes are not counted")}


def measure_ckks(local, reps=20, matvec=True):
    """Key switching and the BSGS matvec at BASELINE config-3 shape
    (N=2^16, 2^15 slots, 20 limbs, dnum 3), timed with CUDA events on the
    context stream.  Returns the two report objects."""
    import torch
    from fhe_mamba_b200 import CCParams, CryptoContext
    from fhe_mamba_b200.ckks import bsgs_diagonals
    cc = CryptoContext(CCParams(ring_dim=1 << 16, multiplicative_depth=19, scaling_mod_size=59,
                                first_mod_size=60, num_large_digits=3, device=local))
    cc.KeyGen(7)
    stream = torch.cuda.ExternalStream(cc.stream_ptr(), device=torch.device("cuda", local))
    n, L, K = cc.n, cc.n_q, cc.n_p
    D = (L + cc.alpha - 1) // cc.alpha
    rng = np.random.default_rng(3)
    d3 = np.empty((3, L, n), dtype=np.uint64)
    for l, q in enumerate(cc.q):
        d3[:, l, :] = rng.integers(0, q, size=(3, n), dtype=np.uint64)
    ct3 = cc.upload(d3, noise_deg=2)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    per_kernel = {}
    for kernel, fused in (("cuda", False), ("tensor-all", False), ("cuda", True)):
        cc.SetConversionKernel(kernel)
        cc.SetKeySwitchFusion(fused)
        for _ in range(3):
            cc.Relinearize(ct3)
        cc.synchronize()
        e0.record(stream)
        for _ in range(reps):
            cc.Relinearize(ct3)  # output freed on the stream right away, as in the evaluator
        e1.record(stream)
        e1.synchronize()
        per_kernel[kernel + ("_fused" if fused else "")] = e0.elapsed_time(e1) / reps
    cc.SetConversionKernel(CONVERSION)
    cc.SetKeySwitchFusion(FUSED_KEY_INNER)
    # 7 sources per digit at this shape: the "tensor" choice keeps the CUDA cores here
    ks_ms = per_kernel["cuda_fused" if FUSED_KEY_INNER else "cuda"]
    ks_bytes = (L + 2 * L + 2 * L) * n * 8 + D * 2 * (L + K) * n * 8
    peak, kind = peaks()
    ks = {"workload": "relinearisation (HYBRID key switch), N=2^16, 20 Q limbs, 7 P limbs, dnum 3",
          "ms": ks_ms, "conversion_kernel": "cuda", "fused_key_inner": FUSED_KEY_INNER,
          "ms_by_variant": per_kernel,
          "alg_bytes": ks_bytes, "achieved_gbs": ks_bytes / (ks_ms / 1e3) / 1e9,
          "frac": ks_bytes / (ks_ms / 1e3) / 1e9 / peak, "peak_gbs": peak, "peak_source": kind}

    if not matvec:
        del ct3
        cc.close()
        return ks, None
    m, k, baby, giant = 768, 1536, 32, 48
    W = rng.normal(0, 0.02, size=(m, k))
    x = rng.uniform(-1, 1, k)
    cc.EvalRotateKeyGen(list(range(1, baby)) + [g * baby for g in range(1, giant)])
    v = np.zeros(cc.slots)
    v[:k] = x
    v[k:2 * k] = x
    ct = cc.Encrypt(cc.MakeCKKSPackedPlaintext(v))
    pts = cc.MakeCKKSPackedPlaintexts(np.array([d for d in bsgs_diagonals(W, baby, giant, cc.slots)]))
    out = cc.EvalLinearTransform(ct, pts, baby, giant)
    cc.synchronize()
    e0.record(stream)
    for _ in range(3):
        out = cc.EvalLinearTransform(ct, pts, baby, giant)
    e1.record(stream)
    e1.synchronize()
    mv_ms = e0.elapsed_time(e1) / 3
    cc.RescaleInPlace(out)
    y = cc.Decrypt(out).GetRealPackedValue()
    err = float(np.max(np.abs(y[:m] - W @ x)))
    diag_bytes = k * L * n * 8
    mv = {"workload": "BASELINE configs[2]: 768x1536 BSGS matvec, N=2^16, 2^15 slots, 20 limbs, dnum 3, "
                      "baby 32 / giant 48, diagonals pre-encoded in HBM",
          "ms": mv_ms, "max_abs_err_vs_fp64": err, "rotations": (baby - 1) + (giant - 1),
          "diagonal_bytes": diag_bytes, "diagonal_stream_gbs": diag_bytes / (mv_ms / 1e3) / 1e9}
    del pts, ct, out, ct3
    cc.close()
    return ks, mv


def measure_keyswitch_levels(cc, levels=(45, 31, 16), reps=20):
    """Relinearisation on the token loop's context (N = 2^16, depth 44, dnum 3:
    15 P limbs, digits of 15) at several levels, with the basis conversions on
    the CUDA cores and on the tensor cores; CUDA events on the context stream."""
    import torch
    stream = torch.cuda.ExternalStream(cc.stream_ptr())
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    rng = np.random.default_rng(45)
    out = []
    for nq in levels:
        d = np.empty((3, nq, cc.n), dtype=np.uint64)
        for l in range(nq):
            d[:, l, :] = rng.integers(0, cc.q[l], size=(3, cc.n), dtype=np.uint64)
        ct = cc.upload(d, noise_deg=2)
        row = {"limbs": nq}
        for kernel, fused in (("cuda", False), ("tensor", False), ("tensor", True)):
            cc.SetConversionKernel(kernel)
            cc.SetKeySwitchFusion(fused)
            for _ in range(3):
                cc.Relinearize(ct)
            cc.synchronize()
            e0.record(stream)
            for _ in range(reps):
                cc.Relinearize(ct)
            e1.record(stream)
            e1.synchronize()
            row[kernel + ("_fused" if fused else "") + "_ms"] = e0.elapsed_time(e1) / reps
        out.append(row)
        del ct
    cc.SetConversionKernel(CONVERSION)
    cc.SetKeySwitchFusion(FUSED_KEY_INNER)
    return out


def measure_bootstrap(cc, reps=3):
    """Full-packing bootstraps on the token loop's context (N=2^16, 2^15 slots,
    depth 44, 59/60-bit, dnum 3, level budget {4,4}; packed_fideslib.cpp:1061-1089),
    CUDA events on the context stream; the input has 2 limbs left."""
    import torch
    stream = torch.cuda.ExternalStream(cc.stream_ptr())
    x = np.random.default_rng(5).uniform(-1, 1, cc.slots)
    ct = cc.Encrypt(cc.MakeCKKSPackedPlaintext(x))
    cc.LevelReduceInPlace(ct, cc.n_q - 2)
    out = cc.EvalBootstrap(ct)
    cc.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(reps):
        out = cc.EvalBootstrap(ct)
    e1.record(stream)
    e1.synchronize()
    info = cc.bootstrap_info()
    res = {"workload": "full-packing bootstrap, N=2^16, 2^15 slots, depth 44 (45 Q limbs), 59/60-bit, dnum 3, "
                       "level budget {4,4}, uniform ternary secret",
           "ms": e0.elapsed_time(e1) / reps, "limbs_in": 2, "limbs_out": out.n_limbs(),
           "levels": cc.bootstrap_levels(),
           "max_abs_err": float(np.max(np.abs(cc.Decrypt(out).GetRealPackedValue() - x))),
           "correction": info["correction"], "chebyshev_degree": info["chebyshev_degree"],
           "rotation_keys": info["rotation_keys"]}
    # the token loop's two-pass refresh (6 limbs in, bound 4) over all slots
    # and over each sub-slot size, for a value at [0, min(3352, n)) (3352: the
    # in_proj width)
    refresh = {}
    for n in (0,) + tuple(getattr(cc, "subslot_sizes", ())):
        support = min(3352, n) if n else 3352
        v = np.zeros(cc.slots)
        v[:support] = 4 * x[:support]
        cv = cc.Encrypt(cc.MakeCKKSPackedPlaintext(v))
        cc.LevelReduceInPlace(cv, cc.n_q - 6)
        y = cc.EvalRefresh(cv, 4.0, passes=2, support=support if n else 0)
        cc.synchronize()
        e0.record(stream)
        for _ in range(reps):
            y = cc.EvalRefresh(cv, 4.0, passes=2, support=n)
        e1.record(stream)
        e1.synchronize()
        got = cc.Decrypt(y).GetRealPackedValue()
        refresh["all slots" if not n else f"{n} slots"] = {
            "ms": e0.elapsed_time(e1) / reps, "limbs_out": y.n_limbs(),
            "max_abs_err": float(np.max(np.abs(got[:support] - v[:support]))),
            "max_abs_outside": float(np.max(np.abs(got[max(n, support):])))}
    res["two_pass_refresh"] = {"input": "6 limbs, bound 4, values at [0, min(3352, slots))", "by_slots": refresh}
    return res


def measure_sharded_keyswitch(local, world, reps=20):
    """Limb-sharded relinearisation over the ranks (round-robin limbs, two NCCL
    all-gathers per key switch) at the token loop's top level (45 limbs) and at
    the config-3 level (20 limbs), N=2^16, dnum 3: device time per key switch
    (CUDA events on the context stream, max over ranks), the single-GPU time of
    the same key switch on this box, and a word-for-word check of the own rows
    against the single-GPU result."""
    import torch
    import torch.distributed as dist
    from fhe_mamba_b200 import CCParams, CryptoContext
    from fhe_mamba_b200.shard import ShardedKeySwitch, to_device_rows, to_host_rows
    dev = torch.device("cuda", local)
    cc = CryptoContext(CCParams(ring_dim=1 << 16, multiplicative_depth=44, scaling_mod_size=59,
                                first_mod_size=60, num_large_digits=3, device=local))
    cc.KeyGen(7)
    sk = ShardedKeySwitch(cc)
    sk.load_key(2)
    cases = []
    for nq in (cc.n_q, 20):
        rng = np.random.default_rng(nq)
        d = np.empty((3, nq, cc.n), dtype=np.uint64)
        for l in range(nq):
            d[:, l, :] = rng.integers(0, cc.q[l], size=(3, cc.n), dtype=np.uint64)
        full = cc.upload(d, noise_deg=2)
        want = cc.Relinearize(full).residues()
        own = to_device_rows(sk.plan.own_rows(d, nq), dev)
        exact = np.array_equal(to_host_rows(sk.relinearize(own, nq)), sk.plan.own_rows(want, nq))
        for _ in range(3):
            sk.relinearize(own, nq)
        dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(sk.stream)
        for _ in range(reps):
            sk.relinearize(own, nq)
        e1.record(sk.stream)
        e1.synchronize()
        ms = e0.elapsed_time(e1) / reps
        for _ in range(3):
            sk.relinearize(own, nq, split=True)
        dist.barrier()
        torch.cuda.synchronize()
        e0.record(sk.stream)
        for _ in range(reps):
            sk.relinearize(own, nq, split=True)
        e1.record(sk.stream)
        e1.synchronize()
        ms_split = e0.elapsed_time(e1) / reps
        exact_split = np.array_equal(to_host_rows(sk.relinearize(own, nq, split=True)), sk.plan.own_rows(want, nq))
        # per-step breakdown (device time on the context stream; a gather's
        # step includes waiting for the slowest rank to reach it)
        steps = {k: 0.0 for k in sk.STAGES}
        for _ in range(reps):
            evs = [torch.cuda.Event(enable_timing=True) for _ in range(6)]
            sk.relinearize(own, nq, events=evs)
            evs[5].synchronize()
            for i, k in enumerate(sk.STAGES):
                steps[k] += evs[i].elapsed_time(evs[i + 1]) / reps
        for _ in range(3):
            cc.Relinearize(full)
        cc.synchronize()
        e0.record(sk.stream)
        for _ in range(reps):
            cc.Relinearize(full)
        e1.record(sk.stream)
        e1.synchronize()
        single = e0.elapsed_time(e1) / reps
        t = torch.tensor([ms, single, 0.0 if exact and exact_split else 1.0, ms_split] +
                         [steps[k] for k in sk.STAGES], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        pl = sk.plan
        gather = (world - 1) * (pl.q_chunk(nq) + 2 * pl.p_chunk) * cc.n * 8
        breakdown = {k: float(t[4 + i]) for i, k in enumerate(sk.STAGES)}
        cases.append({"limbs": nq, "ms": float(t[0]), "single_gpu_ms": float(t[1]),
                      "speedup": float(t[1] / t[0]), "bit_exact_all_ranks": bool(t[2] == 0.0),
                      "ms_digit_split_exchange": float(t[3]), "speedup_digit_split": float(t[1] / t[3]),
                      "received_bytes_per_rank": gather, "step_ms_max_over_ranks": breakdown,
                      "largest_step": max(breakdown, key=breakdown.get)})
        del full
    cc.close()
    return {"world": world, "layout": "round-robin RNS limbs, NCCL all-gathers of the ModUp and ModDown limbs",
            "cases": cases}


# BASELINE config 5's protocol (the reference's generation request,
# src/fhemamba/generation.py:102): 8 prompt token IDs from seed 7, then 16
# greedily generated tokens, 8 + 16 - 1 = 23 server evaluations.
PROMPT_SEED, PROMPT_TOKENS, GENERATED_TOKENS, VOCAB = 7, 8, 16, 50280
# Parity bar of the loop against the plaintext polynomial path: every greedy
# token equal, and the decrypted final hidden vector within this max-abs error.
HIDDEN_TOL = 1e-4


def config5_prompt():
    return [int(t) for t in np.random.default_rng(PROMPT_SEED).integers(0, VOCAB, PROMPT_TOKENS)]


def synthetic_model(seed, horizon, layers=24, fused_decay=False, threads=None):
    """The BASELINE config-5 model (Mamba-2-130M shape, tied embedding, seeded
    random weights), calibrated on 16 token sequences of its own seed that
    cover at least the run's `horizon` evaluations (the recurrent state keeps
    growing for many tokens)."""
    from fhe_mamba_b200.mamba2_layer import Mamba2Model
    return Mamba2Model(layers=layers, d_model=768, d_state=128, heads=24, vocab=VOCAB, seed=seed,
                       calib_sequences=16, calib_tokens=max(32, horizon + 4), fused_decay=fused_decay,
                       calib_threads=threads)


def plaintext_protocol(model, evaluations):
    """The inputs of the config-5 protocol on the plaintext polynomial path:
    the prompt, then each greedy selection fed back."""
    state, inputs, tok = model.initial_state(), [], None
    prompt = config5_prompt()
    for e in range(evaluations):
        tok_in = prompt[e] if e < len(prompt) else tok
        inputs.append(tok_in)
        _, logits, state = model.plain_token(tok_in, state)
        tok = int(np.argmax(logits))
    return inputs


class TokenLoop:
    """The 24-layer encrypted greedy loop: client encrypt -> server layers -> client select.

    evaluate(token) runs one server evaluation on the encrypted embedding of
    `token` and returns the client's greedy selection; the inputs, the
    decrypted hidden vectors and each evaluation's device time are kept for
    the checks after the timed region."""

    def __init__(self, local, layers=24, passes=2, seed=6, sparse_h=0, classical128=False, fused_decay=False,
                 horizon=32, cache_gb=None, model=None):
        from fhe_mamba_b200 import CCParams, CryptoContext
        from fhe_mamba_b200.mamba2_layer import EncryptedMamba2Model
        import torch
        t0 = time.perf_counter()
        # ranks of one node share the host cores for the calibration
        threads = max(1, host_threads() // int(os.environ.get("LOCAL_WORLD_SIZE", "1")))
        self.model = model if model is not None else synthetic_model(seed, horizon, layers, fused_decay, threads)
        self.calibration_seconds = time.perf_counter() - t0
        # 128-classic as the reference's executable sets it up: ring 2^17, four
        # digits, 2^15 slots sparsely packed (packed_fideslib.cpp:1060-1076)
        ring, dnum = (1 << 17, 4) if classical128 else (1 << 16, 3)
        self.cc = CryptoContext(CCParams(ring_dim=ring, multiplicative_depth=44, scaling_mod_size=59,
                                         first_mod_size=60, num_large_digits=dnum, batch_size=1 << 15,
                                         device=local))
        self.audit = None
        if classical128:
            import math
            qp = math.prod(self.cc.q + self.cc.p).bit_length()
            if qp > 3523:
                raise RuntimeError(f"Q*P has {qp} bits, above the classical-128 bound 3523 for ring 2^17")
            self.audit = {"ring_dimension": ring, "qp_bits": qp, "guideline_max_qp_bits": 3523,
                          "q_towers": self.cc.n_q, "p_towers": self.cc.n_p, "hybrid_digits": dnum,
                          "uniform_ternary": not sparse_h}
        self.cc.SetConversionKernel(CONVERSION)
        self.cc.SetKeySwitchFusion(FUSED_KEY_INNER)
        self.cc.KeyGen(41 + seed)
        self.cc.EvalBootstrapSetup((4, 4), sparse_hamming_weight=sparse_h)
        # sub-slot refreshes run with the uniform secret; not at ring 2^17, where
        # their keys (478 MB each) next to the loop's ran the B200 out of memory
        self.subslot = () if (sparse_h or classical128) else tuple(SUBSLOT_SIZES)
        for n in self.subslot:
            self.cc.EvalBootstrapSubslotSetup(n, SUBSLOT_BUDGET)
        self.cc.EvalBootstrapKeyGen()
        # ring 2^17 doubles every key and ciphertext: a smaller diagonal cache
        if cache_gb is None:
            cache_gb = DIAGONAL_CACHE_GB
        # ring 2^17 doubles every plaintext: the memo takes the 8 GB the former
        # diagonal cache held there
        self.em = EncryptedMamba2Model(self.cc, self.model, passes=passes, cache_gb=cache_gb,
                                       memo_gb=min(MEMO_GB, 8.0) if classical128 else MEMO_GB)
        self.cc.EvalRotateKeyGen(self.em.rotation_steps())
        self.cc.synchronize()
        self.setup_seconds = time.perf_counter() - t0
        self.stream = torch.cuda.ExternalStream(self.cc.stream_ptr(), device=torch.device("cuda", local))
        self.inputs, self.hidden, self.eval_ms, self.eval_stats = [], [], [], []
        self.layers, self.passes = layers, passes

    def encrypt(self, token):
        m, c = self.model, self.cc
        return c.Encrypt(c.MakeCKKSPackedPlaintext(np.pad(m.embedding[token], (0, c.slots - m.d_model))))

    def server(self, ct):
        em = self.em
        h = ct
        new = []
        for layer, (conv, st), bounds in zip(em.layers, em.state, em.m.bounds):
            h, conv, st = layer.step(h, conv, st, bounds)
            new.append((conv, st))
        em.state = new
        m, last = em.m, em.layers[-1]
        h = last._fit(h, 14, m.final_bound)
        return last.pm.rms_norm(h, m.d_model, m.norm_f, m.layers[0].eps, (m.rsqrt_f.lo, m.rsqrt_f.hi),
                                degree=len(m.rsqrt_f.coeffs) - 1)

    def select(self, hidden):
        tok, hf = self.em.select(hidden)
        self.hidden.append(hf)
        return tok

    def evaluate(self, token):
        """One server evaluation between the client's encrypt and select;
        the server's device time (CUDA events on the context stream) is kept."""
        import torch
        self.inputs.append(int(token))
        cache, memo = self.em.cache, self.em.memo
        before = (cache.hits, cache.misses, self.em.refreshes(), memo.hits if memo else 0, memo.misses if memo else 0)
        ct = self.encrypt(token)                    # client
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(self.stream)
        hidden = self.server(ct)                    # server: every layer on ciphertexts
        e1.record(self.stream)
        e1.synchronize()
        self.eval_ms.append(e0.elapsed_time(e1))
        self.eval_stats.append({"cache_hits": cache.hits - before[0], "cache_misses": cache.misses - before[1],
                                "refreshes": self.em.refreshes() - before[2],
                                "constant_encodes": (memo.misses - before[4]) if memo else None,
                                "constant_memo_hits": (memo.hits - before[3]) if memo else None})
        return self.select(hidden)                  # client

    def plaintext_check(self):
        """Replays the evaluations' inputs on the plaintext polynomial path
        (same weights and polynomials, fp64): whether every greedy selection
        agrees, the largest deviation of the decrypted final hidden vector,
        the per-evaluation logit margins (a near tie would explain a token
        difference), and the audit of every refresh input against its bound
        and every Chebyshev input against its interval over these inputs."""
        m = self.model
        state, same, err, errs = m.initial_state(), True, 0.0, []
        for tok, enc_tok, hf in zip(self.inputs, self.em.tokens, self.hidden):
            want, logits, state = m.plain_token(tok, state)
            same &= int(np.argmax(logits)) == enc_tok
            e = float(np.max(np.abs(want - hf)))
            errs.append(e)
            err = max(err, e)
        audit = m.audit(self.inputs)
        top = sorted(audit["bound_ratio"].items(), key=lambda kv: -kv[1]["max"])[:4]
        out_of_domain = {k: v for k, v in audit["domain"].items() if v["max"] > 1.0 + 1e-6}
        return {"tokens_equal_plaintext": bool(same), "max_hidden_error": err, "tolerance": HIDDEN_TOL,
                "passed": bool(same and err <= HIDDEN_TOL), "evaluations": len(self.hidden),
                "hidden_error_per_evaluation": errs, "logit_margins": self.em.margins,
                "max_refresh_bound_ratio": audit["max_bound_ratio"],
                "largest_bound_ratios": {k: v for k, v in top},
                "max_domain_position": audit["max_domain_position"],
                "outside_domain": out_of_domain, "calibration": m.calibration}


def run_classical128(local, model, evaluations, passes):
    """The same model's loop under classical-128 parameters as the reference's
    executable sets them up (ring 2^17, four digits, 45 Q + 12 P primes with
    the Q*P audit, 2^15 sparsely packed slots, uniform ternary secret) over
    the first `evaluations` prompt tokens of the config-5 protocol, with its
    own plaintext-path check; device time per evaluation (CUDA events)."""
    loop = TokenLoop(local, passes=passes, classical128=True, model=model)
    prompt = config5_prompt()
    for t in prompt[:evaluations]:
        loop.evaluate(t)
    check = loop.plaintext_check()
    out = {"workload": "config-5 loop, first prompt tokens, classical-128 (ring 2^17, dnum 4)",
           "evaluations": len(loop.eval_ms), "s_per_evaluation": sum(loop.eval_ms[1:]) / 1e3 / max(1, len(loop.eval_ms) - 1),
           "eval_ms": loop.eval_ms, "refreshes_per_evaluation": loop.em.refreshes() / len(loop.eval_ms),
           "security_audit": loop.audit, "setup_seconds": loop.setup_seconds,
           "check": {k: check[k] for k in ("tokens_equal_plaintext", "max_hidden_error", "tolerance", "passed",
                                           "hidden_error_per_evaluation", "max_refresh_bound_ratio",
                                           "max_domain_position")}}
    loop.cc.close()
    return out


def host_threads():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def run_reference(args, rank):
    """The reference arm: FIDESlib/OpenFHE are not in the reference checkout,
    so the CPU oracle (the restatement of OpenFHE's algorithms) on the host
    cores stands in.  Each step times every operation kind at every level the
    GPU arm's recorded per-token counts use, and extrapolates one token from
    those counts (a labelled lower-bound estimate; a CPU token takes hours)."""
    if rank != 0:
        return
    threads = host_threads()
    doc = json.load(open(LEVEL_COUNTS))
    counts = doc["level_counts"]
    for _ in range(args.warmup):
        cpu_estimate(counts, threads)
    values, measured = [], 0.0
    for _ in range(args.steps):
        v, m, ops, levels = cpu_estimate(counts, threads)
        values.append(v)
        measured += m
    value = sum(values) / len(values)
    sample = (f"per step, the CPU oracle timed once per operation kind (ModUp, key inner product + ModDown, "
              f"rescale, tensor) at each of {levels} levels ({measured / args.steps:.1f} s), weighted by "
              f"{ops:.0f} operations per token counted by the GPU arm ({doc['source']}); extrapolation factor "
              f"{value / (measured / args.steps):.0f}; a lower bound (automorphisms, additions, plaintext products "
              "and encodes are not counted)")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": value * 1e3,
        "higher_is_better": False, "scaling": "weak", "vs_baseline": None, "dtype": "u64",
        "data": "synthetic", "config": config_dict(args), "estimate": True,
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port", "estimate": True,
                         "measured_seconds_per_step": measured / args.steps,
                         "extrapolation_factor": value / (measured / args.steps), "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    emit(line)


def config_dict(args):
    return {"workload": "BASELINE configs[4]: encrypted greedy token loop, Mamba-2-130M shape "
                        f"({args.layers} layers, d_model 768, d_state 128, 24 heads, vocab 50280)",
            "ring_dim": 1 << 17 if args.security == "128-classic" else 1 << 16, "slots": 1 << 15, "depth": 44,
            "scale_bits": 59, "dnum": 4 if args.security == "128-classic" else 3, "security": args.security,
            "bootstrap_passes": args.passes, "conversion_kernel": args.conversion,
            "keyswitch_fusion": args.keyswitch_fusion, "decay": "fused per-head series" if args.decay == "fused" and args.security == "not-set" else "exp(a softplus)",
            "secret_key_dist": f"sparse-encapsulated h={args.sparse_h}" if args.sparse_h else "uniform-ternary",
            "l2": "inputs larger than L2 (keys ~36 GB, diagonals generated on the device)",
            "diagonal_cache_gb": args.diagonal_cache_gb,
            "subslot_refresh": [] if args.sparse_h or args.security == "128-classic" else list(SUBSLOT_SIZES),
            "subslot_budget": list(SUBSLOT_BUDGET), "constant_memo_gb": args.constant_memo_gb,
            "parallelism": "one token-loop replica per GPU"}


def ntt_config():
    return {"workload": "BASELINE configs[1]: batched forward+inverse negacyclic NTT",
            "log_n": LOG_N, "limbs": LIMBS, "polys": POLYS, "prime_bits": BITS,
            "l2": f"{N_ROTATE} rotating input batches ({N_ROTATE * ALG_BYTES_PER_TRANSFORM // 2 / 1e6:.0f} MB) > L2"}


def measure_ntt(local, steps, warmup):
    """Config-2 NTT: device-timed forward/inverse pairs and the forward roofline."""
    import torch
    from fhe_mamba_b200 import NttContext
    qs = bench_primes()
    ctx = NttContext(LOG_N, qs, device=local)
    stream = torch.cuda.ExternalStream(ctx.stream_ptr(), device=torch.device("cuda", local))
    bufs = [torch.from_numpy(make_batch(qs, 1000 + i).view(np.int64)).cuda(local) for i in range(N_ROTATE)]
    torch.cuda.synchronize()
    for i in range(warmup):
        ctx.forward(bufs[i % N_ROTATE])
        ctx.inverse(bufs[i % N_ROTATE])
    torch.cuda.synchronize()
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(steps)]
    for i in range(steps):
        b = bufs[i % N_ROTATE]
        evs[i][0].record(stream)
        ctx.forward(b)
        evs[i][1].record(stream)
        ctx.inverse(b)
        evs[i][2].record(stream)
    torch.cuda.synchronize()
    fwd = sum(e[0].elapsed_time(e[1]) for e in evs) / steps
    inv = sum(e[1].elapsed_time(e[2]) for e in evs) / steps
    ceiling = ctx.butterfly_ceiling()
    ctx.close()
    butterflies = POLYS * LIMBS * (1 << (LOG_N - 1)) * LOG_N
    achieved = ALG_BYTES_PER_TRANSFORM / (fwd / 1e3) / 1e9
    peak, kind = peaks()
    return {"bound": "hbm", "kernel": "forward NTT (ntt_fwd_cols + ntt_fwd_rows), BASELINE config 2",
            "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak, "peak_source": kind,
            "traffic": ncu_traffic(), "alg_bytes_per_launch": ALG_BYTES_PER_TRANSFORM, "fwd_ms": fwd,
            "inv_ms": inv, "ntt_steps_per_s": 1e3 / (fwd + inv), "ntt_unit": NTT_UNIT, "config": ntt_config(),
            "integer_pipe": {
                "note": "the transform is bound by the 64-bit multiply pipe, not HBM: ceiling = the same lazy "
                        "Shoup butterfly on registers only, measured live on this GPU",
                "butterflies_per_launch": butterflies, "achieved": butterflies / (fwd / 1e3),
                "ceiling": ceiling, "unit": "butterflies/s", "frac": butterflies / (fwd / 1e3) / ceiling}}


def main():
    global CONVERSION, FUSED_KEY_INNER, DIAGONAL_CACHE_GB, SUBSLOT_SIZES, SUBSLOT_BUDGET, MEMO_GB
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2, help="timed tokens")
    ap.add_argument("--warmup", type=int, default=3, help="untimed tokens")
    ap.add_argument("--layers", type=int, default=24)
    ap.add_argument("--passes", type=int, default=2, choices=[1, 2], help="bootstrap passes per refresh")
    ap.add_argument("--sparse-h", type=int, default=0,
                    help="bootstrap by sparse-secret encapsulation with this Hamming weight (0: uniform ternary)")
    ap.add_argument("--security", default="not-set", choices=["not-set", "128-classic"],
                    help="128-classic: ring 2^17, dnum 4, 2^15 sparsely packed slots, Q*P audited")
    ap.add_argument("--decay", default="fused", choices=["fused", "separate"],
                    help="fused: decay = one per-head series of the raw dt (no refresh of a*dt); "
                         "separate: exp of a times the softplus series")
    ap.add_argument("--classical128-evaluations", type=int, default=0,
                    help="after the headline (not-set) run, this many timed evaluations of the same loop under "
                         "classical-128 parameters (0: none; about 4 minutes for 3)")
    ap.add_argument("--classical128-only", action="store_true",
                    help="print only the classical-128 side run (--classical128-evaluations, default 3) of a "
                         "freshly calibrated model")
    ap.add_argument("--conversion", default="tensor", choices=["tensor", "cuda"],
                    help="basis conversions of the key switches on the tensor cores or the CUDA cores")
    ap.add_argument("--diagonal-cache-gb", type=float, default=0.0,
                    help="encoded-diagonal cache budget in GB (0, the default: generate and encode on the device "
                         "at every matvec)")
    ap.add_argument("--keyswitch-fusion", default="off", choices=["on", "off"],
                    help="form the Q limbs' key inner product inside ModDown's last NTT pass")
    ap.add_argument("--subslot-refresh", default=",".join(map(str, SUBSLOT_SIZES)),
                    help="comma-separated slot counts of sub-slot refreshes for values known to be zero outside "
                         "[0, n) (one EvalMod over n slots instead of two over all); 0: every refresh over all slots")
    ap.add_argument("--subslot-budget", default=",".join(map(str, SUBSLOT_BUDGET)),
                    help="level budget CoeffToSlot,SlotToCoeff of the sub-slot refreshes")
    ap.add_argument("--constant-memo-gb", type=float, default=MEMO_GB,
                    help="budget of the memo of the layers' constant plaintexts in GB (0: encode at every use)")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-ckks", action="store_true", help="skip the key-switch, matvec and bootstrap side measurements")
    ap.add_argument("--ckks-only", action="store_true",
                    help="print only the key-switch and config-3 matvec measurements on one GPU, the "
                         "limb-sharded key switch under torchrun")
    ap.add_argument("--ntt-only", action="store_true",
                    help="print only the config-2 NTT roofline measurement (profiling runs)")
    ap.add_argument("--kernel-shares", action="store_true",
                    help="after the warm-up, record one token's kernels (CUPTI) and print their time shares")
    args = ap.parse_args()
    CONVERSION = args.conversion
    SUBSLOT_SIZES = tuple(int(v) for v in args.subslot_refresh.split(",") if int(v))
    SUBSLOT_BUDGET = tuple(int(v) for v in args.subslot_budget.split(","))
    MEMO_GB = args.constant_memo_gb
    if len(SUBSLOT_BUDGET) != 2:
        ap.error("--subslot-budget takes two numbers")
    DIAGONAL_CACHE_GB = args.diagonal_cache_gb
    FUSED_KEY_INNER = args.keyswitch_fusion == "on"
    if args.warmup < 3:
        ap.error("warmup must be >= 3")
    json_stdout()

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        run_reference(args, rank)
        return

    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local)
    if args.ntt_only:
        emit({"roofline": measure_ntt(local, steps=20, warmup=5)})
        return
    if args.classical128_only and world == 1:
        model = synthetic_model(6, PROMPT_TOKENS + 20, args.layers, args.decay == "fused")  # --decay separate advised
        emit({"classical128": run_classical128(local, model, (args.classical128_evaluations or 3) + 1, args.passes),
              "decay": args.decay})
        return
    if args.ckks_only and world == 1:
        ks, mv = measure_ckks(local, matvec=True)
        from fhe_mamba_b200 import CCParams, CryptoContext
        cc = CryptoContext(CCParams(ring_dim=1 << 16, multiplicative_depth=44, scaling_mod_size=59,
                                    first_mod_size=60, num_large_digits=3, device=local))
        cc.KeyGen(7)
        emit({"keyswitch": ks, "bsgs_matvec": mv, "keyswitch_by_level": measure_keyswitch_levels(cc)})
        cc.close()
        return
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=900), device_id=torch.device("cuda", local))
    if args.ckks_only:
        sharded = measure_sharded_keyswitch(local, world)
        if rank == 0:
            emit({"sharded_keyswitch": sharded})
        dist.destroy_process_group()
        return

    from fhe_mamba_b200 import _lib

    roofline = measure_ntt(local, steps=20, warmup=5)
    side = {}
    if world == 1 and not args.no_ckks:
        side["keyswitch"], side["bsgs_matvec"] = measure_ckks(local)

    if world > 1 and not args.no_ckks:
        side["sharded_keyswitch"] = measure_sharded_keyswitch(local, world)

    # prefill: the prompt's evaluations (untimed; the first W of them are the
    # warm-up, more warm-up steps generate tokens), then K timed generation
    # steps, each one evaluation that generates one token
    extra_warmup = max(0, args.warmup - PROMPT_TOKENS)
    horizon = PROMPT_TOKENS + extra_warmup + args.steps
    # classical-128 keeps the separate decay (see the classical128 side run)
    loop = TokenLoop(local, layers=args.layers, passes=args.passes, seed=6 + rank, sparse_h=args.sparse_h,
                     classical128=args.security == "128-classic",
                     fused_decay=args.decay == "fused" and args.security == "not-set", horizon=horizon)
    prompt = config5_prompt()
    tok = None
    for t in prompt:
        tok = loop.evaluate(t)
    for _ in range(extra_warmup):
        tok = loop.evaluate(tok)
    torch.cuda.synchronize()

    if args.kernel_shares:
        from torch.profiler import ProfilerActivity, profile
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            tok = loop.evaluate(tok)
            torch.cuda.synchronize()
        agg = {}
        for e in prof.events():
            if e.device_type.name != "CUDA":
                continue
            name = e.name.replace("void ", "").replace("(anonymous namespace)::", "").split("(")[0]
            a = agg.setdefault(name, [0, 0.0])
            a[0] += 1
            a[1] += getattr(e, "device_time_total", 0) or getattr(e, "cuda_time_total", 0)
        total = sum(v[1] for v in agg.values())
        rows = [{"kernel": k, "launches": c, "ms": t / 1e3, "share": t / total}
                for k, (c, t) in sorted(agg.items(), key=lambda kv: -kv[1][1])]
        if rank == 0:
            emit({"kernel_shares_one_token": rows, "total_ms": total / 1e3})
        loop.cc.close()
        return

    uuid = None
    try:
        uuid = str(torch.cuda.get_device_properties(local).uuid)
    except Exception:
        pass
    sampler = ClockSampler(uuid)
    sampler.start()
    time.sleep(0.5)
    loop.cc.counters(reset=True)
    launches0 = _lib.kernel_launches()
    first_timed = len(loop.eval_ms)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t_wall = time.perf_counter()
    for i in range(args.steps):
        tok = loop.evaluate(tok)    # client encrypt, server layers (device-timed), client select
    torch.cuda.synchronize()
    e2e_dt = time.perf_counter() - t_wall
    if world > 1:
        dist.barrier()
    clocks = sampler.stop()
    launches = _lib.kernel_launches() - launches0
    levels_by_kind = loop.cc.level_counts()
    counters = loop.cc.counters(reset=True)
    server_ms = sum(loop.eval_ms[first_timed:])
    check = loop.plaintext_check()
    t = torch.tensor([server_ms, e2e_dt, 0.0 if check["passed"] else 1.0], dtype=torch.float64,
                     device=f"cuda:{local}")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    server_ms, e2e_dt, failed = float(t[0].item()), float(t[1].item()), bool(t[2].item())
    value = server_ms / 1e3 / (args.steps * world)
    e2e_value = e2e_dt / (args.steps * world)
    slot_bytes = 16 * loop.cc.slots

    if rank == 0:
        per_token = {k: v / args.steps for k, v in counters.items()}
        level_counts = {kind: {nq: c / args.steps for nq, c in per.items()} for kind, per in levels_by_kind.items()}
        n_eval = PROMPT_TOKENS + GENERATED_TOKENS - 1
        gen = loop.em.tokens[PROMPT_TOKENS - 1:]
        config5 = {"prompt_seed": PROMPT_SEED, "prompt": prompt, "generated_tokens": GENERATED_TOKENS,
                   "server_evaluations": n_eval, "covered": len(loop.eval_ms) >= n_eval,
                   "generated": gen[:GENERATED_TOKENS]}
        if config5["covered"]:
            # the reference's accounting: all 23 evaluations over the 16 generated tokens
            config5["s_per_generated_token_incl_prompt"] = sum(loop.eval_ms[:n_eval]) / 1e3 / GENERATED_TOKENS
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": server_ms / args.steps, "higher_is_better": False,
            "scaling": "weak", "vs_baseline": None, "dtype": "u64", "data": "synthetic (seeded random weights)",
            "config": config_dict(args),
            "roofline": roofline,
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": slot_bytes,
                    "d2h_bytes_per_step": slot_bytes,
                    "path": "client encode+encrypt of the embedding (host slots to device), server layers, "
                            "client decrypt+decode (device slots to host) and greedy argmax"},
            "gpu_launches": launches,
            "clocks": clocks,
            "per_token": {"operations": per_token, "refreshes": loop.em.refreshes() / max(1, len(loop.eval_ms)),
                          "setup_seconds": loop.setup_seconds, "calibration_seconds": loop.calibration_seconds,
                          "eval_ms": loop.eval_ms, "eval_stats": loop.eval_stats, "tokens": loop.em.tokens,
                          "check": check, "diagonal_cache_gb": loop.em.cache.bytes / 2 ** 30,
                          "level_counts": level_counts},
            "config5": config5,
            "security_audit": loop.audit,
        }
        if failed:
            # the loop did not compute what it claims: no headline number
            line["check_failed"] = True
            line["value_unchecked"], line["value"] = line["value"], None
            line["e2e"]["value_unchecked"], line["e2e"]["value"] = line["e2e"]["value"], None
        line.update(side)
        if world == 1 and not args.no_ckks:
            line["bootstrap"] = measure_bootstrap(loop.cc)
            line["keyswitch_by_level"] = measure_keyswitch_levels(loop.cc)
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(level_counts, host_threads())

    model = loop.model
    loop.cc.close()
    del loop
    if rank == 0:
        if world == 1 and args.security == "not-set" and args.classical128_evaluations > 0:
            # every ciphertext and cached plaintext of the ring-2^16 loop goes
            # back to the driver first: the ring-2^17 keys need large blocks
            import gc
            gc.collect()
            torch.cuda.synchronize()
            torch.cuda.empty_cache()
            _lib.call("fhe_device_trim", local)
            try:
                # classical-128 keeps the separate decay (the fused per-head series
                # amplifies ring 2^17's sparse-packing bootstrap noise past 1e-4)
                if args.decay == "fused":
                    model = synthetic_model(6, horizon, args.layers, False)
                # the first evaluation also builds its level tables: the mean skips it
                line["classical128"] = run_classical128(local, model, args.classical128_evaluations + 1,
                                                        args.passes)
            except Exception as e:  # reported, the headline stands on its own
                line["classical128"] = {"error": f"{type(e).__name__}: {e}"}
        emit(line)
    if world > 1:
        dist.destroy_process_group()
    if failed:
        sys.exit(3)


if __name__ == "__main__":
    main()
